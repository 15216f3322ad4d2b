"""Reference-compatible import path: ``from config import get_config``."""
from hanuman_b200.config import *  # noqa: F401,F403
from hanuman_b200.config import Config, PRESETS, get_config  # noqa: F401
