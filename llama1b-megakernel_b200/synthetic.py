"""Seeded synthetic inputs: random-init Llama weights, token IDs and KV caches.

There is no checkpoint or dataset on the build or GPU machines, so every
benchmark and parity case draws its inputs from here. The generator is
bit-reproducible across machines and devices: element ``i`` of tensor ``t``
is ``table[hash(i, t, seed) & 0xffff]`` where ``hash`` is the SplitMix64
finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number
generators", OOPSLA 2014), evaluated with integer arithmetic only, and
``table`` holds the 65,536 equiprobable quantiles of N(0, std) rounded to
bf16. CPU (numpy) and CUDA (torch integer ops) produce identical bits, so
weights made on the GPU box match the CPU oracle's exactly.

The init recipe (normal std 0.02, norm weights 1, tied embeddings) is the
one BASELINE.json names for Llama-3.2-1B.
"""
from __future__ import annotations

import statistics
from functools import lru_cache

import numpy as np
import torch

from .config import LlamaDecodeConfig

_MASK64 = (1 << 64) - 1


def _s64(c: int) -> int:
    return c - (1 << 64) if c >= (1 << 63) else c


_C0 = _s64(0x9E3779B97F4A7C15)
_C1 = _s64(0xBF58476D1CE4E5B9)
_C2 = _s64(0x94D049BB133111EB)


@lru_cache(maxsize=8)
def normal_table(std: float) -> torch.Tensor:
    """65,536 bf16 quantiles of N(0, std) at the bin midpoints (i + 0.5) / 65536."""
    nd = statistics.NormalDist(0.0, std)
    q = np.array([nd.inv_cdf((i + 0.5) / 65536.0) for i in range(65536)], dtype=np.float32)
    return torch.from_numpy(q).to(torch.bfloat16)


def _splitmix_words(n_words: int, base: int, device) -> torch.Tensor:
    """SplitMix64 of (base + j) for j < n_words, as int64 (two's complement)."""
    z = (torch.arange(n_words, dtype=torch.int64, device=device) + base) * _C0
    z = (z ^ ((z >> 30) & ((1 << 34) - 1))) * _C1
    z = (z ^ ((z >> 27) & ((1 << 37) - 1))) * _C2
    return z ^ ((z >> 31) & ((1 << 33) - 1))


def _stream_base(seed: int, stream: int, offset: int = 0) -> int:
    return _s64(((((seed * 1_000_003) + stream) << 36) + offset) & _MASK64)


def hashed_u16(numel: int, seed: int, stream: int, device="cpu") -> torch.Tensor:
    """``numel`` pseudo-random 16-bit values as int32 in [0, 65536)."""
    words = _splitmix_words((numel + 3) // 4, _stream_base(seed, stream), device)
    u = words.view(torch.int16)[:numel]
    return u.to(torch.int32) & 0xFFFF


def hashed_normal(shape, seed: int, stream: int, std: float = 0.02, device="cpu") -> torch.Tensor:
    """bf16 tensor of N(0, std) samples, identical bits on every device."""
    numel = int(np.prod(shape)) if len(shape) else 1
    table = normal_table(float(std))
    device = torch.device(device)
    chunk = 1 << 26
    out = torch.empty(numel, dtype=torch.bfloat16, device=device)
    tab_dev = table.to(device)
    tab_np = table.view(torch.int16).numpy()
    for s in range(0, numel, chunk):
        e = min(numel, s + chunk)
        # Chunks start on multiples of 4 elements, so each chunk hashes its own
        # words: word j covers elements 4j..4j+3 of the whole tensor.
        words = _splitmix_words((e - s + 3) // 4, _stream_base(seed, stream, s // 4), device)
        if device.type == "cpu":
            idx = words.numpy().view(np.uint16)[: e - s]
            out[s:e] = torch.from_numpy(tab_np[idx]).view(torch.bfloat16)
        else:
            idx = words.view(torch.int16)[: e - s].to(torch.int32) & 0xFFFF
            out[s:e] = tab_dev[idx.long()]
    return out.view(*shape)


def hashed_ints(n: int, high: int, seed: int, stream: int) -> torch.Tensor:
    """``n`` int64 values in [0, high) from the same hash (CPU)."""
    words = _splitmix_words(n, _stream_base(seed, stream), "cpu")
    # Use the top 62 bits (non-negative) modulo high; the bias is < 2**-40.
    return ((words >> 2) & ((1 << 62) - 1)) % high


# Stream ids: one per weight tensor, in a fixed order, plus input streams.
_EMBED = 0
_PER_LAYER = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
STREAM_TOKENS = 1_000_000
STREAM_KV = 2_000_000


def weight_names(cfg: LlamaDecodeConfig) -> list[str]:
    names = ["model.embed_tokens.weight"]
    for l in range(cfg.num_layers):
        p = f"model.layers.{l}."
        names += [p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                  p + "self_attn.v_proj.weight", p + "self_attn.o_proj.weight",
                  p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight",
                  p + "mlp.down_proj.weight", p + "input_layernorm.weight",
                  p + "post_attention_layernorm.weight"]
    names.append("model.norm.weight")
    return names


def weight_shape(cfg: LlamaDecodeConfig, name: str) -> tuple[int, ...]:
    h, i = cfg.hidden, cfg.intermediate
    if name == "model.embed_tokens.weight":
        return (cfg.vocab, h)
    if name.endswith("norm.weight"):
        return (h,)
    kind = name.split(".")[-2]
    return {
        "q_proj": (cfg.q_dim, h), "k_proj": (cfg.kv_dim, h), "v_proj": (cfg.kv_dim, h),
        "o_proj": (h, cfg.q_dim), "gate_proj": (i, h), "up_proj": (i, h), "down_proj": (h, i),
    }[kind]


def _stream_of(name: str) -> int:
    if name == "model.embed_tokens.weight":
        return _EMBED
    parts = name.split(".")
    layer = int(parts[2])
    return 1 + layer * len(_PER_LAYER) + _PER_LAYER.index(parts[-2])


def make_weight(cfg: LlamaDecodeConfig, name: str, seed: int = 0, std: float = 0.02,
                device="cpu") -> torch.Tensor:
    """One HF-named bf16 weight tensor of the seeded random-init model."""
    shape = weight_shape(cfg, name)
    if name.endswith("norm.weight"):
        return torch.ones(shape, dtype=torch.bfloat16, device=device)
    return hashed_normal(shape, seed, _stream_of(name), std, device)


def make_weights(cfg: LlamaDecodeConfig, seed: int = 0, std: float = 0.02,
                 device="cpu") -> dict[str, torch.Tensor]:
    """All HF-named weights (tied: no separate lm_head tensor)."""
    return {n: make_weight(cfg, n, seed, std, device) for n in weight_names(cfg)}


def random_tokens(n: int, vocab: int, seed: int = 0, stream: int = STREAM_TOKENS) -> torch.Tensor:
    """``n`` token IDs, uniform over [0, vocab)."""
    return hashed_ints(n, vocab, seed, stream)


def random_kv_rows(cfg: LlamaDecodeConfig, length: int, seed: int, seq: int = 0,
                   device="cpu") -> tuple[torch.Tensor, torch.Tensor]:
    """N(0, 1) bf16 K and V for ``length`` cached positions of one sequence.

    Shapes are [num_layers, num_kv_heads, length, head_dim] (HF BHSD per layer).
    """
    shape = (cfg.num_layers, cfg.num_kv_heads, length, cfg.head_dim)
    k = hashed_normal(shape, seed, STREAM_KV + 2 * seq, 1.0, device)
    v = hashed_normal(shape, seed, STREAM_KV + 2 * seq + 1, 1.0, device)
    return k, v
