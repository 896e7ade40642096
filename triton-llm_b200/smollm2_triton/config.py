"""SmolLM2 / Llama configuration (drop-in for smollm2_triton/config.py).

Same fields, defaults, variant table and GPT-2-style aliases as the
reference dataclass (smollm2_triton/config.py:9-126), so server code and
tests that build configs keep working. ``torch_dtype`` selects the storage
precision of the B200 path: "float32" (the reference's numerics) or
"bfloat16" (bf16 weights and KV cache, fp32 activations and accumulation).
"""

from dataclasses import dataclass


@dataclass
class SmolLM2Config:
    vocab_size: int = 49152
    hidden_size: int = 576
    num_hidden_layers: int = 30
    num_attention_heads: int = 9
    num_key_value_heads: int = 3
    intermediate_size: int = 1536
    max_position_embeddings: int = 8192
    rms_norm_eps: float = 1e-5
    rope_theta: float = 100000.0
    tie_word_embeddings: bool = True
    hidden_act: str = "silu"
    torch_dtype: str = "float32"
    repo_id: str | None = None

    @classmethod
    def from_pretrained(cls, name: str) -> "SmolLM2Config":
        """Config of a known variant (same table as the reference)."""
        s360 = dict(hidden_size=960, num_hidden_layers=32, num_attention_heads=15,
                    num_key_value_heads=5, intermediate_size=2560)
        s17 = dict(hidden_size=2048, num_hidden_layers=24, num_attention_heads=32,
                   num_key_value_heads=32, intermediate_size=8192)
        variants = {
            "SmolLM2-135M": {},
            "SmolLM2-360M": s360,
            "SmolLM2-1.7B": s17,
            "SmolLM2-135M-Instruct": {},
            "SmolLM2-360M-Instruct": s360,
            "SmolLM2-1.7B-Instruct": s17,
            # Llama-3 RoPE scaling is not part of the reference path either:
            # the supported context stays at the 8192 base window.
            "Llama-3.2-3B-Instruct": dict(
                vocab_size=128256, hidden_size=3072, num_hidden_layers=28,
                num_attention_heads=24, num_key_value_heads=8,
                intermediate_size=8192, max_position_embeddings=8192,
                rms_norm_eps=1e-5, rope_theta=500000.0, tie_word_embeddings=True,
                hidden_act="silu", torch_dtype="float32",
                repo_id="meta-llama/Llama-3.2-3B-Instruct"),
        }
        if name not in variants:
            raise ValueError(f"Unknown variant: {name!r}. Available: {list(variants.keys())}")
        return SmolLM2Config(**variants[name])

    @classmethod
    def from_dict(cls, d: dict) -> "SmolLM2Config":
        """From a HuggingFace ``config.json`` dict (unknown keys ignored)."""
        import dataclasses
        names = {f.name for f in dataclasses.fields(cls)}
        return cls(**{k: v for k, v in d.items() if k in names})

    # GPT-2 style aliases used by shared code (reference config.py:114-126)
    @property
    def n_embd(self):
        return self.hidden_size

    @property
    def n_layer(self):
        return self.num_hidden_layers

    @property
    def n_head(self):
        return self.num_attention_heads

    @property
    def n_kv_head(self):
        return self.num_key_value_heads

    @property
    def n_positions(self):
        return self.max_position_embeddings

    @property
    def n_ffn(self):
        return self.intermediate_size
