"""SmolLM2 / Llama inference on B200 (drop-in for the reference package).

Same public names as the reference (smollm2_triton/__init__.py): the config
dataclass and the model; the batched engine is in ``engine``.
"""

from .config import SmolLM2Config
from .model import SmolLM2ForCausalLM

__all__ = ["SmolLM2Config", "SmolLM2ForCausalLM"]
