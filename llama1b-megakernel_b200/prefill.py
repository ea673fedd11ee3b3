"""Prompt prefill on the GPU with PyTorch (cuBLAS GEMMs, SDPA).

The reference runs context encoding on its baseline NxDI path, not in the
megakernel (llama_with_megakernel.py:194-204; the decoder layer forward,
llama.py:1039-1139). This is the B200 counterpart: all T prompt positions of
a sequence go through each layer at once with HF Llama's rounding order (bf16
activations, fp32 RMSNorm statistics, RoPE and SwiGLU in bf16), and every
layer's post-RoPE K and V rows are written into the paged cache at their
positions, so decode steps continue from it. It works on the kernel's packed
weights in place: the RoPE-pair order of ``w_qkv`` and the gate/up
interleave of ``w_gate_up`` are undone on the GEMM outputs, not on the
weights.

The last position's logits are the bf16 lm_head output (as HF computes them)
widened to fp32; the decode kernel's logits are fp32 sums.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .kv_cache import PagedKVCache


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    h = x.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return w * h.to(x.dtype)


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """HF ``apply_rotary_pos_emb`` on [T, heads, 64] with [T, 64] tables."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def _slots(kv: PagedKVCache, seq: int, positions: torch.Tensor):
    table = torch.as_tensor(kv._host_tables[seq], dtype=torch.long)
    pos = positions.cpu()
    return (table[pos // kv.page_size].to(kv.device), (pos % kv.page_size).to(kv.device))


@torch.no_grad()
def prefill(model, input_ids, past_key_values: PagedKVCache | None = None):
    """Run ``input_ids`` — [B, T], or a list of B 1-D tensors of any lengths —
    through ``model`` (a ``MegakernelLlamaForCausalLM``), sequence b continuing
    from its cached length; returns (logits [B, V] fp32 of each sequence's
    last position, greedy ids [B] int64)."""
    cfg, pw = model.cfg, model.packed
    if getattr(model, "tp_world", 1) != 1:
        raise NotImplementedError("prefill runs on a single-GPU model")
    kv = past_key_values if past_key_values is not None else model.kv
    if isinstance(input_ids, (list, tuple)):
        rows = [torch.as_tensor(r).reshape(-1) for r in input_ids]
    else:
        ids = torch.as_tensor(input_ids)
        rows = list(ids[None, :] if ids.dim() == 1 else ids)
    B = len(rows)
    if B > model.max_batch:
        raise ValueError(f"batch {B} > max_batch {model.max_batch}")
    dev = model.device
    H, NQ, NKV, I = cfg.hidden, cfg.num_q_heads, cfg.num_kv_heads, cfg.intermediate
    nh = NQ + 2 * NKV
    starts = [kv.seq_lens[b] for b in range(B)]
    last = []
    for b in range(B):  # sequences differ in length: one at a time
        T = rows[b].numel()
        if T == 0:
            raise ValueError(f"sequence {b} has no tokens")
        if starts[b] + T > pw.rope_cos.shape[0]:
            raise ValueError(f"sequence {b}: positions up to {starts[b] + T - 1} exceed the RoPE "
                             f"table ({pw.rope_cos.shape[0]} positions)")
        kv.reserve(b, starts[b] + T)
        ids_b = rows[b].to(dev)
        pos = torch.arange(starts[b], starts[b] + T, device=dev)
        page, off = _slots(kv, b, pos.cpu())
        allpos = torch.arange(0, starts[b] + T)
        apage, aoff = _slots(kv, b, allpos)
        cos, sin = pw.rope_cos[pos], pw.rope_sin[pos]
        x = pw.embed[ids_b]  # [T, H]
        causal = allpos.to(dev)[None, :] <= pos[:, None]  # [T, P]
        for l in range(cfg.num_layers):
            h = _rms(x, pw.norm_attn[l], cfg.rms_eps)
            qkv = F.linear(h, pw.w_qkv[l].view(-1, H))  # [T, nh*64], rows (head, d, pair)
            qkv = qkv.view(T, nh, 32, 2).transpose(-1, -2).reshape(T, nh, 64)
            q = _rope(qkv[:, :NQ], cos, sin)
            k = _rope(qkv[:, NQ:NQ + NKV], cos, sin)
            v = qkv[:, NQ + NKV:]
            kv.k_pages[l, page, :, off] = k
            kv.v_pages[l, page, :, off] = v
            K = kv.k_pages[l, apage, :, aoff]  # [P, NKV, 64]
            V = kv.v_pages[l, apage, :, aoff]
            a = F.scaled_dot_product_attention(
                q.transpose(0, 1)[None], K.transpose(0, 1)[None], V.transpose(0, 1)[None],
                attn_mask=causal[None, None], enable_gqa=True)  # [1, NQ, T, 64]
            o = F.linear(a[0].transpose(0, 1).reshape(T, NQ * 64), pw.w_o[l])
            x = x + o
            h = _rms(x, pw.norm_mlp[l], cfg.rms_eps)
            gu = F.linear(h, pw.w_gate_up[l].view(2 * I, H)).view(T, I, 2)
            x = x + F.linear(F.silu(gu[..., 0]) * gu[..., 1], pw.w_down[l])
        last.append(_rms(x[-1], pw.norm_final, cfg.rms_eps))
        kv.seq_lens[b] = starts[b] + T
    logits = F.linear(torch.stack(last), pw.embed).float()
    return logits, logits.argmax(dim=-1)
