"""Model and cache configuration for the decode megakernel.

The defaults are Llama-3.2-1B: the model the reference hardcodes in its NKI
kernels (nki_kernels/attention.py:18-32, nki_kernels/mlp.py:28-34) and whose
llama3 RoPE parameters it reads from the HF config (llama.py:851-884,
llama.py:888-936).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, replace


@dataclass(frozen=True)
class LlamaDecodeConfig:
    """Architecture of a Llama decoder as the megakernel sees it.

    Field meanings follow HF ``LlamaConfig``. ``head_dim`` is fixed at 64 by
    the kernel (the reference's D, nki_kernels/attention.py:20).
    """

    num_layers: int = 16
    hidden: int = 2048
    intermediate: int = 8192
    num_q_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 64
    vocab: int = 128256
    rms_eps: float = 1e-5
    rope_theta: float = 500000.0
    rope_factor: float = 32.0
    rope_low_freq_factor: float = 1.0
    rope_high_freq_factor: float = 4.0
    rope_original_max_position: int = 8192
    tie_word_embeddings: bool = True

    @property
    def group(self) -> int:
        """Query heads per KV head (GQA group size)."""
        return self.num_q_heads // self.num_kv_heads

    @property
    def q_dim(self) -> int:
        return self.num_q_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    def replace(self, **kw) -> "LlamaDecodeConfig":
        return replace(self, **kw)

    def to_dict(self) -> dict:
        return asdict(self)

    def num_params(self) -> int:
        """Parameter count with tied embeddings (1,235,814,400 for Llama-3.2-1B)."""
        h, i = self.hidden, self.intermediate
        per_layer = h * self.q_dim + 2 * h * self.kv_dim + self.q_dim * h + 3 * h * i + 2 * h
        return self.num_layers * per_layer + self.vocab * h + h

    def weight_bytes_per_token(self) -> int:
        """Algorithmic bf16 weight bytes one bs=1 decode step must read.

        Decoder weights and norms, the tied lm_head, the final norm and one
        embedding row (2,471,632,896 B for Llama-3.2-1B).
        """
        h, i = self.hidden, self.intermediate
        per_layer = h * self.q_dim + 2 * h * self.kv_dim + self.q_dim * h + 3 * h * i + 2 * h
        return 2 * (self.num_layers * per_layer + self.vocab * h + h + h)

    def kv_bytes_per_position(self) -> int:
        """K and V bytes read per cached position per step, all layers (32,768 B)."""
        return 2 * 2 * self.num_layers * self.kv_dim

    def validate(self) -> None:
        if self.head_dim != 64:
            raise ValueError("the megakernel is built for head_dim 64")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("num_q_heads must be a multiple of num_kv_heads")
        if self.group not in (1, 2, 4, 8):
            raise ValueError("GQA group size must be 1, 2, 4 or 8")
        if self.hidden % 256 or self.intermediate % 256 or self.q_dim % 256:
            raise ValueError("hidden, intermediate and q_dim must be multiples of 256")
        if self.hidden > 4096 or self.intermediate > 8192 or self.q_dim > 8192:
            raise ValueError("hidden <= 4096, intermediate <= 8192 and q_dim <= 8192 are supported")


LLAMA_3_2_1B = LlamaDecodeConfig()

# A small model with the same structure (GQA 4, head_dim 64) for fast parity
# tests: the oracle finishes it in milliseconds.
TINY = LlamaDecodeConfig(
    num_layers=2, hidden=256, intermediate=512, num_q_heads=4, num_kv_heads=1,
    vocab=1000,
)

SMALL = LlamaDecodeConfig(
    num_layers=3, hidden=512, intermediate=1536, num_q_heads=8, num_kv_heads=2,
    vocab=5003,
)

# Two Llama-3.2-1B-shaped layers with a small vocabulary: the full-size layer
# geometry (a whole 16 KB down row per fill) at a size the oracle runs in seconds.
MID = LlamaDecodeConfig(num_layers=2, vocab=4099)
