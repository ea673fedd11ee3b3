"""CPU oracle: HF Llama builder and a paged-KV restatement of one decode step.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): the checker the GPU parity
tests compare against, and the CPU baseline bench.py times. Never part of the
product path.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from llama1b_megakernel_b200.config import LlamaDecodeConfig


# ----------------------------------------------------------------------------
# RoPE (reference: llama.py:888-953, Llama3RotaryEmbedding)
# ----------------------------------------------------------------------------

def llama3_inv_freq(cfg: LlamaDecodeConfig) -> torch.Tensor:
    """fp32 llama3-scaled inverse frequencies, [head_dim // 2].

    Restates ``Llama3RotaryEmbedding.get_inv_freqs`` (llama.py:917-936): the
    base frequencies 1 / theta^(2i/d) in fp32, then per frequency: keep it when
    its wavelength is below orig/high, divide by ``factor`` when above
    orig/low, else blend with smooth = (orig/wavelen - low) / (high - low).
    """
    dim = cfg.head_dim
    idx = torch.arange(0, dim, 2, dtype=torch.float)
    inv_freq = 1.0 / (cfg.rope_theta ** (idx / dim))
    low_wavelen = cfg.rope_original_max_position / cfg.rope_low_freq_factor
    high_wavelen = cfg.rope_original_max_position / cfg.rope_high_freq_factor
    out = []
    for freq in inv_freq:
        wavelen = 2 * math.pi / freq
        if wavelen < high_wavelen:
            out.append(freq)
        elif wavelen > low_wavelen:
            out.append(freq / cfg.rope_factor)
        else:
            smooth = (cfg.rope_original_max_position / wavelen - cfg.rope_low_freq_factor) / (
                cfg.rope_high_freq_factor - cfg.rope_low_freq_factor)
            out.append((1 - smooth) * freq / cfg.rope_factor + smooth * freq)
    return torch.tensor(out, dtype=inv_freq.dtype)


def rope_cos_sin(inv_freq: torch.Tensor, positions: torch.Tensor, dtype=torch.bfloat16):
    """cos, sin [B, T, head_dim] for int positions [B, T] (llama.py:938-953)."""
    inv = inv_freq[None, :, None].float().expand(positions.shape[0], -1, 1)
    pos = positions[:, None, :].float()
    freqs = (inv.float() @ pos.float()).transpose(1, 2)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate_half(x):
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def _rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    dt = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    return w * h.to(dt)


# ----------------------------------------------------------------------------
# Paged KV cache (oracle copy)
# ----------------------------------------------------------------------------

@dataclass
class OracleKV:
    """Paged bf16 KV cache on the CPU, same layout as the GPU cache.

    ``k_pages``/``v_pages``: [num_layers, num_pages, num_kv_heads, page_size,
    head_dim]; ``block_tables``: [batch, max_blocks] int32 page ids, shared by
    all layers. Position p of sequence b lives in page
    ``block_tables[b, p // page_size]`` at slot ``p % page_size``.
    """

    k_pages: torch.Tensor
    v_pages: torch.Tensor
    block_tables: torch.Tensor

    @property
    def page_size(self) -> int:
        return self.k_pages.shape[3]

    def gather(self, layer: int, b: int, n: int):
        """K, V rows [0, n) of sequence b in layer ``layer``: [nkv, n, hd] each."""
        ps = self.page_size
        nb = (n + ps - 1) // ps
        pages = self.block_tables[b, :nb].long()
        if bool((pages < 0).any()):
            raise IndexError(f"sequence {b}: positions < {n} include unreserved pages")
        k = self.k_pages[layer, pages].permute(1, 0, 2, 3).reshape(self.k_pages.shape[2], nb * ps, -1)
        v = self.v_pages[layer, pages].permute(1, 0, 2, 3).reshape(self.v_pages.shape[2], nb * ps, -1)
        return k[:, :n], v[:, :n]

    def write(self, layer: int, b: int, pos: int, k_row: torch.Tensor, v_row: torch.Tensor):
        """Store K/V rows [nkv, hd] at position ``pos`` of sequence b."""
        ps = self.page_size
        page = int(self.block_tables[b, pos // ps])
        if page < 0:
            raise IndexError(f"sequence {b}: position {pos} is in an unreserved page")
        self.k_pages[layer, page, :, pos % ps] = k_row
        self.v_pages[layer, page, :, pos % ps] = v_row

    def fill(self, b: int, k_rows: torch.Tensor, v_rows: torch.Tensor):
        """Store rows [0, n) for all layers from [L, nkv, n, hd] tensors."""
        n = k_rows.shape[2]
        ps = self.page_size
        for p0 in range(0, n, ps):
            p1 = min(n, p0 + ps)
            page = int(self.block_tables[b, p0 // ps])
            self.k_pages[:, page, :, : p1 - p0] = k_rows[:, :, p0:p1]
            self.v_pages[:, page, :, : p1 - p0] = v_rows[:, :, p0:p1]


# ----------------------------------------------------------------------------
# One decode step, HF semantics over the paged cache
# ----------------------------------------------------------------------------

def decode_step(cfg: LlamaDecodeConfig, w: dict, kv: OracleKV, tokens, positions,
                inv_freq: torch.Tensor | None = None, layers: int | None = None,
                hidden_in: torch.Tensor | None = None) -> dict:
    """Decode one token per sequence; writes K/V at ``positions`` into ``kv``.

    Each sequence runs alone with HF's shapes ([1, 1, hidden]) and ops so the
    result matches ``LlamaForCausalLM`` with a ``DynamicCache`` bit for bit.
    Returns fp32 logits (lm_head over the bf16 final-norm output, accumulated
    in fp32), the greedy next ids (first index on ties), the bf16 residual
    before the final norm, and the K/V rows written.
    """
    if inv_freq is None:
        inv_freq = llama3_inv_freq(cfg)
    n_layers = cfg.num_layers if layers is None else layers
    tokens = torch.as_tensor(tokens).reshape(-1)
    positions = torch.as_tensor(positions).reshape(-1)
    B = positions.numel()
    hd = cfg.head_dim
    embed = w["model.embed_tokens.weight"]
    embed_f32 = None
    if layers is None:
        # The fp32 copy of the tied lm_head is made once per weight dict.
        embed_f32 = w.get("_embed_f32")
        if embed_f32 is None:
            embed_f32 = w["_embed_f32"] = embed.float()
    out_logits, out_hidden, k_new, v_new = [], [], [], []
    for b in range(B):
        pos = int(positions[b])
        if hidden_in is not None:
            h = hidden_in[b].reshape(1, 1, cfg.hidden).to(torch.bfloat16)
        else:
            h = F.embedding(tokens[b].reshape(1, 1), embed)
        cos, sin = rope_cos_sin(inv_freq, torch.tensor([[pos]]))
        cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
        ks, vs = [], []
        for l in range(n_layers):
            p = f"model.layers.{l}."
            resid = h
            x = _rmsnorm(h, w[p + "input_layernorm.weight"], cfg.rms_eps)
            q = F.linear(x, w[p + "self_attn.q_proj.weight"]).view(1, 1, -1, hd).transpose(1, 2)
            k = F.linear(x, w[p + "self_attn.k_proj.weight"]).view(1, 1, -1, hd).transpose(1, 2)
            v = F.linear(x, w[p + "self_attn.v_proj.weight"]).view(1, 1, -1, hd).transpose(1, 2)
            q = (q * cos) + (_rotate_half(q) * sin)
            k = (k * cos) + (_rotate_half(k) * sin)
            kv.write(l, b, pos, k[0, :, 0], v[0, :, 0])
            ks.append(k[0, :, 0].clone())
            vs.append(v[0, :, 0].clone())
            K, V = kv.gather(l, b, pos + 1)
            attn = F.scaled_dot_product_attention(
                q, K.unsqueeze(0), V.unsqueeze(0), attn_mask=None, dropout_p=0.0,
                scale=hd ** -0.5, is_causal=False, enable_gqa=True)
            attn = attn.transpose(1, 2).contiguous().reshape(1, 1, -1).contiguous()
            h = resid + F.linear(attn, w[p + "self_attn.o_proj.weight"])
            resid = h
            x = _rmsnorm(h, w[p + "post_attention_layernorm.weight"], cfg.rms_eps)
            g = F.linear(x, w[p + "mlp.gate_proj.weight"])
            u = F.linear(x, w[p + "mlp.up_proj.weight"])
            h = resid + F.linear(F.silu(g) * u, w[p + "mlp.down_proj.weight"])
        out_hidden.append(h.reshape(-1))
        k_new.append(torch.stack(ks) if ks else None)
        v_new.append(torch.stack(vs) if vs else None)
        if layers is None:
            x = _rmsnorm(h, w["model.norm.weight"], cfg.rms_eps).reshape(-1)
            out_logits.append(torch.mv(embed_f32, x.float()))
    res = {"hidden": torch.stack(out_hidden), "k_new": k_new, "v_new": v_new}
    if out_logits:
        logits = torch.stack(out_logits)
        res["logits"] = logits
        res["next"] = logits.argmax(dim=-1)
    return res


# ----------------------------------------------------------------------------
# HF model (the reference's own PyTorch Llama path)
# ----------------------------------------------------------------------------

def hf_config(cfg: LlamaDecodeConfig):
    from transformers import LlamaConfig

    return LlamaConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.intermediate,
        num_hidden_layers=cfg.num_layers, num_attention_heads=cfg.num_q_heads,
        num_key_value_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
        max_position_embeddings=131072, rms_norm_eps=cfg.rms_eps,
        rope_parameters={
            "rope_type": "llama3", "rope_theta": cfg.rope_theta, "factor": cfg.rope_factor,
            "low_freq_factor": cfg.rope_low_freq_factor,
            "high_freq_factor": cfg.rope_high_freq_factor,
            "original_max_position_embeddings": cfg.rope_original_max_position,
        },
        tie_word_embeddings=cfg.tie_word_embeddings, hidden_act="silu",
        attention_bias=False, mlp_bias=False, attn_implementation="sdpa",
        torch_dtype=torch.bfloat16,
    )


def hf_model(cfg: LlamaDecodeConfig, w: dict):
    """HF ``LlamaForCausalLM`` in bf16 on the CPU holding the weights ``w``.

    The model is built on the meta device and the tensors are assigned, so no
    time goes to HF's own random init. HF's rotary ``inv_freq`` buffer is then
    set to the fp32 llama3 table: a bf16 cast of the model would otherwise
    round it to bf16, which the reference avoids (llama.py:888-896).
    """
    from transformers import LlamaForCausalLM

    with torch.device("meta"):
        model = LlamaForCausalLM(hf_config(cfg))
    sd = dict(w)
    if cfg.tie_word_embeddings:
        sd["lm_head.weight"] = w["model.embed_tokens.weight"]
    model.load_state_dict(sd, strict=True, assign=True)
    if cfg.tie_word_embeddings:
        model.tie_weights()
    inv = llama3_inv_freq(cfg)
    rot = model.model.rotary_emb
    rot.inv_freq = inv.clone()
    rot.original_inv_freq = inv.clone()
    rot.attention_scaling = 1.0
    model.eval()
    return model
