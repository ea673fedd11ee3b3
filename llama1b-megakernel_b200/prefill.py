"""Prompt prefill on this library's kernels: every prompt position is a row.

The reference runs context encoding on its baseline NxDI path, not in the
megakernel (llama_with_megakernel.py:194-204; the decoder layer forward,
llama.py:1039-1139). Here all prompt positions of all sequences go through
each layer together, as the rows of one batched step, on the same kernels as
the batched decode path (batched.py):

* ``mk_rmsnorm_rows``; the tcgen05 GEMM (``mk_gemm_bf16``, up to 128 rows per
  call) for q/k/v, o_proj (+ residual), gate/up and down (+ residual) on the
  kernel's packed weights; ``mk_rope_scatter`` writes every row's rotated K and
  its V into the paged cache at the row's position; ``mk_swiglu``;
* attention is ``mk_paged_attention`` with one "sequence" per row: the row's
  own sequence's block table and, as its length, its position + 1. Causal
  masking is that length: a row sees its sequence's cached positions up to
  and including its own, whose K/V the same layer's ``mk_rope_scatter`` wrote
  just before;
* rows go in chunks of at most 128 (a later chunk's rows see the earlier
  chunks' K/V in the cache), then the last row of each sequence is
  normalised and scored by the lm_head GEMM (fp32 logits) and
  ``mk_argmax_rows``.

Rounding is HF's in bf16 (linear outputs, residual sums, RMSNorm and SwiGLU
as the batched step); the attention output is rounded from fp32 softmax sums
with P in bf16 for P.V, as flash attention does.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .kv_cache import PagedKVCache

CHUNK = 128  # rows per batched pass (the GEMM's largest padded row count)


def _padded(rows: int) -> int:
    for bp in (16, 32, 64, 128):
        if rows <= bp:
            return bp
    raise ValueError(f"{rows} rows exceed one GEMM call")


@torch.no_grad()
def prefill(model, input_ids, past_key_values: PagedKVCache | None = None):
    """Run ``input_ids`` — [B, T], or a list of B 1-D tensors of any lengths —
    through ``model`` (a ``MegakernelLlamaForCausalLM``), sequence b continuing
    from its cached length; returns (logits [B, V] fp32 of each sequence's
    last position, greedy ids [B] int64)."""
    cfg, pw, lib = model.cfg, model.packed, model.lib
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
    H, NQ, NKV, I, L = cfg.hidden, cfg.num_q_heads, cfg.num_kv_heads, cfg.intermediate, cfg.num_layers
    nh = NQ + 2 * NKV
    starts = [kv.seq_lens[b] for b in range(B)]
    seq_of, pos_of, tok_of, last_row = [], [], [], []
    for b in range(B):
        T = rows[b].numel()
        if T == 0:
            raise ValueError(f"sequence {b} has no tokens")
        if starts[b] + T > pw.rope_cos.shape[0]:
            raise ValueError(f"sequence {b}: positions up to {starts[b] + T - 1} exceed the RoPE "
                             f"table ({pw.rope_cos.shape[0]} positions)")
        kv.reserve(b, starts[b] + T)
        seq_of += [b] * T
        pos_of += range(starts[b], starts[b] + T)
        tok_of += rows[b].tolist()
        last_row.append(len(tok_of) - 1)
    if min(tok_of) < 0 or max(tok_of) >= cfg.vocab:
        raise ValueError("token id outside the vocabulary")
    N = len(tok_of)
    max_len = max(pos_of) + 1
    tok = torch.tensor(tok_of, dtype=torch.long, device=dev)
    pos = torch.tensor(pos_of, dtype=torch.int32, device=dev)
    seq = torch.tensor(seq_of, dtype=torch.long, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    eps = ctypes.c_float(cfg.rms_eps)
    scale = ctypes.c_float(cfg.head_dim ** -0.5)
    z = lambda *shape: torch.zeros(*shape, dtype=torch.bfloat16, device=dev)  # noqa: E731
    T0 = min(N, CHUNK)
    BP0 = _padded(T0)
    h, attn, act = z(BP0, H), z(BP0, NQ * 64), z(BP0, I)
    qkv, q, gu = z(T0, nh * 64), z(T0, NQ, 64), z(T0, 2 * I)
    ws = lib.mk_paged_attention_workspace(T0, NKV, max_len)
    work = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)
    finals = torch.empty(B, H, dtype=torch.bfloat16, device=dev)

    def gemm(w, x, rows_, out, residual=None):
        n, k = w.shape
        _lib.check(lib.mk_gemm_bf16(w.data_ptr(), n, k, x.data_ptr(), rows_, x.shape[0],
                                    residual.data_ptr() if residual is not None else None,
                                    out.data_ptr(), None, None, 0, err.data_ptr(), st))

    for c0 in range(0, N, CHUNK):
        T = min(CHUNK, N - c0)
        BP = _padded(T)
        # the GEMM reads BP rows and writes the first T (padded rows only feed
        # accumulator columns that are never stored)
        hb, ab, xb = h[:BP], attn[:BP], act[:BP]
        x = pw.embed[tok[c0:c0 + T]].contiguous()  # [T, H], the residual stream
        p = pos[c0:c0 + T].contiguous()
        lengths = (p + 1).contiguous()
        bt = kv.block_tables[seq[c0:c0 + T]].contiguous()  # each row's sequence's pages
        for l in range(L):
            _lib.check(lib.mk_rmsnorm_rows(x.data_ptr(), pw.norm_attn[l].data_ptr(), eps, T, H,
                                           hb.data_ptr(), st))
            gemm(pw.w_qkv[l].view(-1, H), hb, T, qkv[:T])
            _lib.check(lib.mk_rope_scatter(
                qkv.data_ptr(), pw.rope_cos.data_ptr(), pw.rope_sin.data_ptr(), p.data_ptr(),
                bt.data_ptr(), kv.max_blocks, kv.num_pages, kv.page_size, NQ, NKV, T,
                q.data_ptr(), kv.k_pages[l].data_ptr(), kv.v_pages[l].data_ptr(), err.data_ptr(),
                st))
            _lib.check(lib.mk_paged_attention(
                q.data_ptr(), kv.k_pages[l].data_ptr(), kv.v_pages[l].data_ptr(), bt.data_ptr(),
                lengths.data_ptr(), T, NQ, NKV, kv.page_size, kv.max_blocks, kv.num_pages,
                max_len, scale, work.data_ptr(), work.numel(), ab.data_ptr(), err.data_ptr(), st))
            gemm(pw.w_o[l], ab, T, x, residual=x)
            _lib.check(lib.mk_rmsnorm_rows(x.data_ptr(), pw.norm_mlp[l].data_ptr(), eps, T, H,
                                           hb.data_ptr(), st))
            gemm(pw.w_gate_up[l].view(2 * I, H), hb, T, gu[:T])
            _lib.check(lib.mk_swiglu(gu.data_ptr(), T * I, xb.data_ptr(), st))
            gemm(pw.w_down[l], xb, T, x, residual=x)
        for b, r in enumerate(last_row):
            if c0 <= r < c0 + T:
                finals[b] = x[r - c0]
    hf = z(_padded(B), H)
    _lib.check(lib.mk_rmsnorm_rows(finals.data_ptr(), pw.norm_final.data_ptr(), eps, B, H,
                                   hf.data_ptr(), st))
    logits = torch.empty(B, cfg.vocab, dtype=torch.float32, device=dev)
    n, k = pw.embed.shape
    _lib.check(lib.mk_gemm_bf16(pw.embed.data_ptr(), n, k, hf.data_ptr(), B, hf.shape[0], None,
                                None, logits.data_ptr(), None, 0, err.data_ptr(), st))
    ids = torch.empty(B, dtype=torch.int64, device=dev)
    _lib.check(lib.mk_argmax_rows(logits.data_ptr(), B, cfg.vocab, ids.data_ptr(), st))
    code = int(err[0])  # synchronises
    if code:
        raise _lib.MkError(_lib.MK_EDEVICE, f"prefill: device error {code} (1: a page id outside "
                           "the pool; 101-103: a tensor-core GEMM wait ran out)")
    for b in range(B):
        kv.seq_lens[b] = starts[b] + rows[b].numel()
    return logits, ids
