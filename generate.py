"""Reference-compatible import path: ``from generate import load_for_generate``."""
from hanuman_b200.generate import generate_from_model, load_for_generate, sample_next  # noqa: F401
