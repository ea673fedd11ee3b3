"""Batched greedy decode (bs 8, 32, 64 at ~1024 cached positions).

At bs=1 one decode step is a chain of GEMVs, and the persistent megakernel
streams the weights once at HBM speed. At bs 8-64 the projections become
skinny GEMMs ([B, K] x [K, N]) that CUDA cores cannot keep up with, and the
KV cache (B x 2 KB x 1024 per layer) is read as much as the weights. This
path runs one step as:

* per layer: RMSNorm, the q/k/v GEMM on the packed ``w_qkv`` (the RoPE-pair
  order undone on the output), RoPE, the K/V rows scattered into the paged
  cache, attention by this library's paged split-K decode kernel
  (``mk_paged_attention``, csrc/mk_attn.cuh: the HBM-heavy part), o_proj and
  the SwiGLU MLP as GEMMs; then the final norm, lm_head and argmax;
* the GEMMs are cuBLAS (tensor cores) through ``torch.nn.functional.linear``
  on the kernel's own packed weights; the elementwise steps are torch ops;
* the whole step is captured once per batch size into a CUDA graph, so a step
  is one graph launch with the tokens and positions on the device.

Rounding follows HF's decode step in bf16 (as the prefill path does), and the
attention output is rounded to bf16 from fp32 softmax sums (as the megakernel
does).
"""
from __future__ import annotations

import ctypes

import torch
import torch.nn.functional as F

from . import _lib
from .kv_cache import PagedKVCache
from .prefill import _rms


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """HF ``apply_rotary_pos_emb`` on [B, heads, 64] with [B, 64] tables."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


class BatchedDecoder:
    """Greedy decode steps for up to ``max_batch`` sequences with the weights
    of ``model`` (a ``MegakernelLlamaForCausalLM``; single GPU)."""

    def __init__(self, model, max_batch: int, max_seq_len: int, page_size: int = 64,
                 num_pages: int | None = None):
        if getattr(model, "tp_world", 1) != 1:
            raise NotImplementedError("the batched path runs on one GPU")
        self.m = model
        self.cfg = model.cfg
        self.dev = model.device
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.kv = PagedKVCache(self.cfg, max_batch, max_seq_len, page_size, num_pages,
                               device=self.dev)
        self.lib = model.lib
        ws = self.lib.mk_paged_attention_workspace(max_batch, self.cfg.num_kv_heads, max_seq_len)
        self.work = torch.empty(max(ws, 16), dtype=torch.uint8, device=self.dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self._graphs: dict[int, tuple] = {}

    # ------------------------------------------------------------------ step
    def _attention(self, q, layer, lengths, B, out):
        c, kv = self.cfg, self.kv
        _lib.check(self.lib.mk_paged_attention(
            q.data_ptr(), kv.k_pages[layer].data_ptr(), kv.v_pages[layer].data_ptr(),
            kv.block_tables.data_ptr(), lengths.data_ptr(), B, c.num_q_heads, c.num_kv_heads,
            kv.page_size, kv.max_blocks, kv.num_pages, self.max_seq_len,
            ctypes.c_float(c.head_dim ** -0.5), self.work.data_ptr(), self.work.numel(),
            out.data_ptr(), self.err.data_ptr(), torch.cuda.current_stream().cuda_stream))

    def _step(self, tokens, positions, logits_out, ids_out):
        c, pw, kv = self.cfg, self.m.packed, self.kv
        B = tokens.numel()
        H, NQ, NKV, I = c.hidden, c.num_q_heads, c.num_kv_heads, c.intermediate
        nh = NQ + 2 * NKV
        pos = positions.long()
        x = pw.embed[tokens.long()]
        cos, sin = pw.rope_cos[pos], pw.rope_sin[pos]
        page = kv.block_tables[:B].gather(1, (pos // kv.page_size)[:, None])[:, 0].long()
        off = pos % kv.page_size
        lengths = (positions + 1).to(torch.int32)
        attn = torch.empty(B, NQ, 64, dtype=torch.bfloat16, device=self.dev)
        for l in range(c.num_layers):
            h = _rms(x, pw.norm_attn[l], c.rms_eps)
            qkv = F.linear(h, pw.w_qkv[l].view(-1, H)).view(B, nh, 32, 2).transpose(-1, -2)
            qkv = qkv.reshape(B, nh, 64)
            q = _rope(qkv[:, :NQ], cos, sin).contiguous()
            kv.k_pages[l, page, :, off] = _rope(qkv[:, NQ:NQ + NKV], cos, sin)
            kv.v_pages[l, page, :, off] = qkv[:, NQ + NKV:]
            self._attention(q, l, lengths, B, attn)
            x = x + F.linear(attn.view(B, NQ * 64), pw.w_o[l])
            h = _rms(x, pw.norm_mlp[l], c.rms_eps)
            gu = F.linear(h, pw.w_gate_up[l].view(2 * I, H)).view(B, I, 2)
            x = x + F.linear(F.silu(gu[..., 0]) * gu[..., 1], pw.w_down[l])
        lg = F.linear(_rms(x, pw.norm_final, c.rms_eps), pw.embed)
        logits_out.copy_(lg)
        ids_out.copy_(lg.argmax(dim=-1))

    def _graph(self, B: int):
        g = self._graphs.get(B)
        if g is None:
            dev = self.dev
            tok = torch.zeros(B, dtype=torch.int32, device=dev)
            pos = torch.zeros(B, dtype=torch.int32, device=dev)
            logits = torch.empty(B, self.cfg.vocab, dtype=torch.float32, device=dev)
            ids = torch.empty(B, dtype=torch.int64, device=dev)
            # warm up on a side stream, then capture. The warm-up really runs
            # (token 0 at position 0 of every slot), so the cache rows it
            # overwrites are saved and put back; capturing runs nothing.
            kv = self.kv
            for b in range(B):
                kv.reserve(b, 1)
            page0 = kv.block_tables[:B, 0].long()
            saved = (kv.k_pages[:, page0, :, 0].clone(), kv.v_pages[:, page0, :, 0].clone())
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                self._step(tok, pos, logits, ids)
            torch.cuda.current_stream().wait_stream(s)
            kv.k_pages[:, page0, :, 0] = saved[0]
            kv.v_pages[:, page0, :, 0] = saved[1]
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._step(tok, pos, logits, ids)
            g = (graph, tok, pos, logits, ids)
            self._graphs[B] = g
        return g

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, positions: torch.Tensor):
        """One greedy step for len(tokens) sequences (row b = cache slot b), K/V
        written at ``positions``; returns (logits [B, V] fp32, ids [B] int64),
        views of the step's static buffers (valid until the next step)."""
        B = int(tokens.numel())
        if B > self.max_batch:
            raise ValueError(f"batch {B} > {self.max_batch}")
        pos_host = torch.as_tensor(positions).cpu()
        for b in range(B):
            self.kv.reserve(b, int(pos_host[b]) + 1)
        graph, tok, pos, logits, ids = self._graph(B)
        tok.copy_(torch.as_tensor(tokens).to(tok.device, torch.int32).reshape(-1))
        pos.copy_(pos_host.to(pos.device, torch.int32).reshape(-1))
        graph.replay()
        for b in range(B):
            self.kv.seq_lens[b] = max(self.kv.seq_lens[b], int(pos_host[b]) + 1)
        return logits, ids

    def replay(self, B: int) -> None:
        """Replay the captured step for batch B on its current device inputs
        (benchmark loop; no host work)."""
        self._graphs[B][0].replay()

    def check(self) -> None:
        torch.cuda.synchronize(self.dev)
        if int(self.err[0]):
            self.err.zero_()
            raise _lib.MkError(_lib.MK_EDEVICE, "paged attention: block table names a page "
                               "outside the pool")
