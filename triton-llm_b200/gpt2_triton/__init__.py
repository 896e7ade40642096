"""GPT-2 inference on B200 (drop-in for the reference package)."""

from .config import GPT2Config
from .model import GPT2Model

__all__ = ["GPT2Config", "GPT2Model"]
