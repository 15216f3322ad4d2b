"""Reference-compatible import path: ``from train import train``."""
from hanuman_b200.flops import count_active_params, count_total_params, step_flops  # noqa: F401
from hanuman_b200.train import Trainer, memory_report, train  # noqa: F401
