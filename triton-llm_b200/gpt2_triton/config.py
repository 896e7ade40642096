"""GPT-2 configuration (drop-in for gpt2_triton/config.py:11-82): same fields,
defaults and variant table as the reference dataclass."""

from dataclasses import dataclass


@dataclass
class GPT2Config:
    vocab_size: int = 50257
    n_embd: int = 768
    n_layer: int = 12
    n_head: int = 12
    n_positions: int = 1024
    layer_norm_epsilon: float = 1e-5

    @classmethod
    def from_pretrained(cls, name: str) -> "GPT2Config":
        variants = {
            "gpt2": GPT2Config(),
            "gpt2-medium": GPT2Config(vocab_size=50257, n_embd=1024, n_layer=24,
                                      n_head=16, n_positions=1024),
            "gpt2-large": GPT2Config(vocab_size=50257, n_embd=1280, n_layer=36,
                                     n_head=20, n_positions=1024),
            "gpt2-xl": GPT2Config(vocab_size=50257, n_embd=1600, n_layer=48,
                                  n_head=25, n_positions=1024),
        }
        if name not in variants:
            raise ValueError(f"Unknown GPT-2 variant: {name!r}. "
                             f"Available: {list(variants.keys())}")
        return variants[name]
