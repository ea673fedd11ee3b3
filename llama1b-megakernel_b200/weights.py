"""Host-side weight packer and RoPE tables (done once, at load time).

The counterpart of the reference's load-time conversion
``NeuronLlamaForCausalLMMK.convert_hf_to_neuron_state_dict``
(llama_with_megakernel.py:281-351), which pre-stacks per-layer weights and
re-tiles them for its kernel. The B200 kernel streams whole weight rows with
bulk copies, so it needs only two row permutations of the HF tensors:

* ``w_qkv``: q, k and v rows of a layer concatenated, and within every head
  the rows d and d+32 placed next to each other (a "RoPE pair"), so one warp
  reduces both halves RoPE mixes and applies the rotation in registers.
* ``w_gate_up``: gate row i and up row i adjacent, so one warp produces
  SiLU(gate_i) * up_i.

o_proj and down_proj keep HF's row-major [out, in] layout. Unlike the
reference (llama_with_megakernel.py:312-316) the RMSNorm gains are *not*
folded into the weights: the kernel applies them as HF does,
bf16(bf16(x * rsqrt(var + eps)) * gamma), so its rounding follows the HF path
it is checked against.

The cos/sin tables reproduce ``Llama3RotaryEmbedding.forward``
(llama.py:938-953): fp32 ``inv_freq`` (llama3-scaled, llama.py:917-936) times
the position, cos/sin in fp32, cast to bf16.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .config import LlamaDecodeConfig


def llama3_inv_freq(cfg: LlamaDecodeConfig) -> torch.Tensor:
    """fp32 inverse frequencies with llama3 scaling, [head_dim // 2]."""
    dim = cfg.head_dim
    base = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.float) / dim))
    low_wavelen = cfg.rope_original_max_position / cfg.rope_low_freq_factor
    high_wavelen = cfg.rope_original_max_position / cfg.rope_high_freq_factor
    out = []
    for f in base:
        wavelen = 2 * math.pi / f
        if wavelen < high_wavelen:
            out.append(f)
        elif wavelen > low_wavelen:
            out.append(f / cfg.rope_factor)
        else:
            smooth = (cfg.rope_original_max_position / wavelen - cfg.rope_low_freq_factor) / (
                cfg.rope_high_freq_factor - cfg.rope_low_freq_factor)
            out.append((1 - smooth) * f / cfg.rope_factor + smooth * f)
    return torch.tensor(out, dtype=torch.float)


def rope_tables(cfg: LlamaDecodeConfig, length: int) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos and sin tables [length, head_dim] for positions 0..length-1 (CPU)."""
    inv = llama3_inv_freq(cfg)
    pos = torch.arange(length, dtype=torch.int64)[None, :]
    inv_e = inv[None, :, None].float().expand(1, -1, 1)
    freqs = (inv_e @ pos[:, None, :].float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)[0]
    return emb.cos().to(torch.bfloat16).contiguous(), emb.sin().to(torch.bfloat16).contiguous()


@dataclass
class PackedWeights:
    """Device tensors in the layouts include/mk.h documents."""

    embed: torch.Tensor      # [V, H]
    w_qkv: torch.Tensor      # [L, NQKV*32, 2, H]
    w_o: torch.Tensor        # [L, H, NQ*64]
    w_gate_up: torch.Tensor  # [L, I, 2, H]
    w_down: torch.Tensor     # [L, H, I]
    norm_attn: torch.Tensor  # [L, H]
    norm_mlp: torch.Tensor   # [L, H]
    norm_final: torch.Tensor # [H]
    rope_cos: torch.Tensor   # [R, 64]
    rope_sin: torch.Tensor   # [R, 64]

    def tensors(self) -> dict[str, torch.Tensor]:
        return dict(self.__dict__)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors().values())


def pack_qkv_layer(cfg: LlamaDecodeConfig, wq, wk, wv) -> torch.Tensor:
    """[NQKV*64, H] q|k|v rows -> [NQKV*32, 2, H] RoPE-pair order."""
    w = torch.cat([wq, wk, wv], dim=0)
    nh = cfg.num_q_heads + 2 * cfg.num_kv_heads
    return w.view(nh, 2, cfg.head_dim // 2, cfg.hidden).permute(0, 2, 1, 3).reshape(
        nh * cfg.head_dim // 2, 2, cfg.hidden)


def unpack_qkv_layer(cfg: LlamaDecodeConfig, packed: torch.Tensor):
    """Inverse of ``pack_qkv_layer``: (wq, wk, wv)."""
    nh = cfg.num_q_heads + 2 * cfg.num_kv_heads
    w = packed.view(nh, cfg.head_dim // 2, 2, cfg.hidden).permute(0, 2, 1, 3).reshape(
        nh * cfg.head_dim, cfg.hidden)
    q = cfg.q_dim
    return w[:q], w[q:q + cfg.kv_dim], w[q + cfg.kv_dim:]


def pack_weights(cfg: LlamaDecodeConfig, sd: dict, rope_len: int, device="cuda") -> PackedWeights:
    """Pack HF-named bf16 weights (any device) into the kernel's layouts on ``device``."""
    cfg.validate()
    L = cfg.num_layers
    dev = torch.device(device)

    def get(name):
        return sd[name].to(device=dev, dtype=torch.bfloat16)

    qkv, wo, gu, wd, na, nm = [], [], [], [], [], []
    for l in range(L):
        p = f"model.layers.{l}."
        qkv.append(pack_qkv_layer(cfg, get(p + "self_attn.q_proj.weight"),
                                  get(p + "self_attn.k_proj.weight"),
                                  get(p + "self_attn.v_proj.weight")))
        wo.append(get(p + "self_attn.o_proj.weight"))
        gu.append(torch.stack([get(p + "mlp.gate_proj.weight"), get(p + "mlp.up_proj.weight")], dim=1))
        wd.append(get(p + "mlp.down_proj.weight"))
        na.append(get(p + "input_layernorm.weight"))
        nm.append(get(p + "post_attention_layernorm.weight"))
    cos, sin = rope_tables(cfg, rope_len)
    embed = get("model.embed_tokens.weight").contiguous()
    return PackedWeights(
        embed=embed,
        w_qkv=torch.stack(qkv).contiguous(),
        w_o=torch.stack(wo).contiguous(),
        w_gate_up=torch.stack(gu).contiguous(),
        w_down=torch.stack(wd).contiguous(),
        norm_attn=torch.stack(na).contiguous(),
        norm_mlp=torch.stack(nm).contiguous(),
        norm_final=get("model.norm.weight").contiguous(),
        rope_cos=cos.to(dev),
        rope_sin=sin.to(dev),
    )
