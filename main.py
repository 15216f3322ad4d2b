"""CLI entry point (same commands as the reference's main.py).

    python main.py train --config smoke
    python main.py generate --config smoke --prompt "hello"
    python main.py count --config full
    python main.py report --config full_g4
"""
from hanuman_b200.main import main

if __name__ == "__main__":
    main()
