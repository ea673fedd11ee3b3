"""Batched greedy decode (bs 8, 32, 64 at ~1024 cached positions).

At bs=1 one decode step is a chain of GEMVs, and the persistent megakernel
streams the weights once at HBM speed. At bs 8-64 the projections become
skinny GEMMs ([B, K] x [K, N]) that CUDA cores cannot keep up with, and the
KV cache (B x 2 KB x 1024 per layer) is read as much as the weights. This
path runs one step as:

* per layer: RMSNorm (``mk_rmsnorm_rows``), the q/k/v GEMM on the packed
  ``w_qkv``, RoPE with the K/V rows scattered into the paged cache
  (``mk_rope_scatter``, which reads the RoPE-pair column order directly),
  attention by this library's paged split-K decode kernel
  (``mk_paged_attention``, csrc/mk_attn.cuh: the HBM-heavy part), o_proj with
  the residual added by the GEMM, RMSNorm, the gate/up GEMM,
  ``mk_swiglu``, down with the residual; then the final norm, lm_head and
  argmax;
* the GEMMs are this library's tcgen05 skinny GEMM (``mk_gemm_bf16``,
  csrc/mk_gemm.cuh) on the kernel's own packed weights, the residual added in
  its epilogue and the logits written in fp32; the elementwise steps are the
  fused kernels of csrc/mk_batched.cuh;
* the whole step is captured once per batch size into a CUDA graph, so a step
  is one graph launch with the tokens and positions on the device.

Tensor parallelism (``model`` a ``TensorParallelLlamaForCausalLM``; BASELINE
config 5 at bs 32): each rank holds its q / kv heads, MLP rows and lm_head
rows (tp.py). The q/k/v and gate/up GEMMs, RoPE, the KV cache and attention
are local; o_proj and down write fp32 partial sums over the rank's input
columns (RowParallelLinear, llama.py:437-470) into the rank's exchange buffer,
and one kernel per exchange (``mk_allreduce_add_rmsnorm``) reads every rank's
partial over NVLink from peer memory, sums them in rank order, adds the sum to
the residual and normalises for the next GEMM: no NCCL on that path. The
buffers are mapped on every GPU through CUDA IPC handles exchanged once over
the group at construction. The lm_head scores the rank's
vocabulary rows; ``mk_argmax_keys`` packs each row's maximum and global id
into one integer key, the keys are all-gathered and ``mk_keys_to_ids`` takes
the largest (lowest id on ties).

Rounding follows HF's decode step in bf16 (the GEMM epilogue rounds W a to
bf16 before the residual add, and the sum again); the attention output is
rounded to bf16 from fp32 softmax sums (as the megakernel does).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .kv_cache import PagedKVCache


class BatchedDecoder:
    """Greedy decode steps for up to ``max_batch`` sequences with the weights
    of ``model``: a ``MegakernelLlamaForCausalLM`` (one GPU) or one rank of a
    ``TensorParallelLlamaForCausalLM`` (every rank of its group constructs
    the decoder and makes the same calls in the same order)."""

    def __init__(self, model, max_batch: int, max_seq_len: int, page_size: int = 64,
                 num_pages: int | None = None):
        self.tp_world = getattr(model, "tp_world", 1)
        self.group = getattr(model, "tp_group", None)
        if not 1 <= max_batch <= 64:
            raise ValueError(f"max_batch {max_batch} outside [1, 64] (the GEMM's padded batch)")
        if max_seq_len > model.rope_len:
            raise ValueError(f"max_seq_len {max_seq_len} exceeds the model's RoPE table "
                             f"({model.rope_len} positions)")
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
        c = self.cfg
        gws = max(self.lib.mk_gemm_workspace(n, k, max_batch) for n, k in (
            ((c.num_q_heads + 2 * c.num_kv_heads) * 64, c.hidden), (c.hidden, c.num_q_heads * 64),
            (2 * c.intermediate, c.hidden), (c.hidden, c.intermediate), (c.vocab, c.hidden)))
        self.gwork = torch.zeros(max(gws, 16), dtype=torch.uint8, device=self.dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self._graphs: dict[int, tuple] = {}
        self._xbuf = None
        if self.tp_world > 1:
            self._open_exchange()

    def _open_exchange(self) -> None:
        """This rank's exchange buffer (two fp32 [max_batch][hidden] slots and the
        flag words) and every other rank's, mapped on this GPU."""
        from . import tp

        lib, H = self.lib, self.cfg.hidden
        torch.cuda.set_device(self.dev)
        nbytes = lib.mk_xbuf_bytes(self.max_batch, H)
        handle, own = _lib.MkIpcHandle(), ctypes.c_void_p()
        _lib.check(lib.mk_xbuf_alloc(nbytes, ctypes.byref(handle), ctypes.byref(own)))
        self._xbuf = own.value
        self._xpeer_open: list[int] = []
        handles = tp.exchange_handles(bytes(handle.bytes), self.group)
        rank = dist.get_rank(self.group)
        addrs = []
        for r, hb in enumerate(handles):
            if r == rank:
                addrs.append(self._xbuf)
                continue
            h, ptr = _lib.MkIpcHandle(), ctypes.c_void_p()
            ctypes.memmove(h.bytes, hb, 64)
            _lib.check(lib.mk_xbuf_open(ctypes.byref(h), ctypes.byref(ptr)))
            self._xpeer_open.append(ptr.value)
            addrs.append(ptr.value)
        self.tp_rank = rank
        self.xpeers = torch.tensor(addrs, dtype=torch.int64, device=self.dev)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.dev)

    def _xslot(self, e: int) -> int:
        """Device address of this rank's partial-sum slot for exchange e."""
        return self._xbuf + (e % 2) * self.max_batch * self.cfg.hidden * 4

    # ------------------------------------------------------------------ step
    def _attention(self, q, layer, lengths, B, out):
        c, kv = self.cfg, self.kv
        _lib.check(self.lib.mk_paged_attention(
            q.data_ptr(), kv.k_pages[layer].data_ptr(), kv.v_pages[layer].data_ptr(),
            kv.block_tables.data_ptr(), lengths.data_ptr(), B, c.num_q_heads, c.num_kv_heads,
            kv.page_size, kv.max_blocks, kv.num_pages, self.max_seq_len,
            ctypes.c_float(c.head_dim ** -0.5), self.work.data_ptr(), self.work.numel(),
            out.data_ptr(), self.err.data_ptr(), torch.cuda.current_stream().cuda_stream))

    def _gemm(self, w, x, rows, out=None, out_f32=None, residual=None):
        """Y = X W^T (+ residual) on the tensor cores (``mk_gemm_bf16``); X has
        the padded row count, its first ``rows`` rows real. ``out_f32`` is a
        tensor or a device address."""
        n, k = w.shape
        if isinstance(out_f32, torch.Tensor):
            out_f32 = out_f32.data_ptr()
        _lib.check(self.lib.mk_gemm_bf16(
            w.data_ptr(), n, k, x.data_ptr(), rows, x.shape[0],
            residual.data_ptr() if residual is not None else None,
            out.data_ptr() if out is not None else None,
            out_f32,
            self.gwork.data_ptr(), self.gwork.numel(), self.err.data_ptr(),
            torch.cuda.current_stream().cuda_stream))

    def _buffers(self, B: int) -> dict:
        c, dev = self.cfg, self.dev
        BP = 16 if B <= 16 else 32 if B <= 32 else 64
        nh = c.num_q_heads + 2 * c.num_kv_heads
        z = lambda *shape: torch.zeros(*shape, dtype=torch.bfloat16, device=dev)  # noqa: E731
        buf = dict(x=z(B, c.hidden), h=z(BP, c.hidden), q=z(B, c.num_q_heads, 64),
                   attn=z(BP, c.num_q_heads * 64), act=z(BP, c.intermediate),
                   qkv=z(B, nh * 64), gu=z(B, 2 * c.intermediate))
        if self.tp_world > 1:
            buf["keys"] = torch.zeros(B, dtype=torch.int64, device=dev)
            buf["keys_all"] = torch.zeros(self.tp_world * B, dtype=torch.int64, device=dev)
        return buf

    def _step(self, tokens, positions, logits_out, ids_out, buf):
        if self.tp_world > 1:
            return self._step_tp(tokens, positions, logits_out, ids_out, buf)
        c, pw, kv, lib = self.cfg, self.m.packed, self.kv, self.lib
        B = tokens.numel()
        H, NQ, NKV, I = c.hidden, c.num_q_heads, c.num_kv_heads, c.intermediate
        st = torch.cuda.current_stream().cuda_stream
        x, h, q, attn, act, qkv, gu = (buf[k] for k in ("x", "h", "q", "attn", "act", "qkv", "gu"))
        x.copy_(pw.embed[tokens.long()])
        lengths = (positions + 1).to(torch.int32)
        eps = ctypes.c_float(c.rms_eps)
        for l in range(c.num_layers):
            _lib.check(lib.mk_rmsnorm_rows(x.data_ptr(), pw.norm_attn[l].data_ptr(), eps, B, H,
                                           h.data_ptr(), st))
            self._gemm(pw.w_qkv[l].view(-1, H), h, B, out=qkv)  # packed RoPE-pair column order
            _lib.check(lib.mk_rope_scatter(
                qkv.data_ptr(), pw.rope_cos.data_ptr(), pw.rope_sin.data_ptr(),
                positions.data_ptr(), kv.block_tables.data_ptr(), kv.max_blocks, kv.num_pages,
                kv.page_size, NQ, NKV, B, q.data_ptr(), kv.k_pages[l].data_ptr(),
                kv.v_pages[l].data_ptr(), self.err.data_ptr(), st))
            self._attention(q, l, lengths, B, attn)
            self._gemm(pw.w_o[l], attn, B, out=x, residual=x)  # x += o_proj(attn)
            _lib.check(lib.mk_rmsnorm_rows(x.data_ptr(), pw.norm_mlp[l].data_ptr(), eps, B, H,
                                           h.data_ptr(), st))
            self._gemm(pw.w_gate_up[l].view(2 * I, H), h, B, out=gu)  # (gate, up) interleaved
            _lib.check(lib.mk_swiglu(gu.data_ptr(), B * I, act.data_ptr(), st))
            self._gemm(pw.w_down[l], act, B, out=x, residual=x)
        _lib.check(lib.mk_rmsnorm_rows(x.data_ptr(), pw.norm_final.data_ptr(), eps, B, H,
                                       h.data_ptr(), st))
        self._gemm(pw.embed, h, B, out_f32=logits_out)
        _lib.check(lib.mk_argmax_rows(logits_out.data_ptr(), B, c.vocab, ids_out.data_ptr(), st))

    def _step_tp(self, tokens, positions, logits_out, ids_out, buf):
        """One step on this rank of a tensor-parallel group (see the module
        docstring); every rank runs the same kernels and collectives."""
        c, pw, kv, lib, m = self.cfg, self.m.packed, self.kv, self.lib, self.m
        B = tokens.numel()
        H, NQ, NKV, I, L = c.hidden, c.num_q_heads, c.num_kv_heads, c.intermediate, c.num_layers
        st = torch.cuda.current_stream().cuda_stream
        x, h, q, attn, act, qkv, gu = (buf[k] for k in ("x", "h", "q", "attn", "act", "qkv", "gu"))
        keys, keys_all = buf["keys"], buf["keys_all"]
        x.copy_(pw.embed[tokens.long()])
        lengths = (positions + 1).to(torch.int32)
        eps = ctypes.c_float(c.rms_eps)
        _lib.check(lib.mk_step_epoch(self.epoch.data_ptr(), st))

        def exchange(e: int, gamma) -> None:  # x += sum of the ranks' partials; h = norm(x)
            _lib.check(lib.mk_allreduce_add_rmsnorm(
                self.xpeers.data_ptr(), self.tp_rank, self.tp_world, self.max_batch, e,
                self.epoch.data_ptr(), x.data_ptr(), gamma.data_ptr(), eps, B, H, h.data_ptr(),
                self.err.data_ptr(), 0, st))

        _lib.check(lib.mk_rmsnorm_rows(x.data_ptr(), pw.norm_attn[0].data_ptr(), eps, B, H,
                                       h.data_ptr(), st))
        for l in range(L):
            self._gemm(pw.w_qkv[l].view(-1, H), h, B, out=qkv)
            _lib.check(lib.mk_rope_scatter(
                qkv.data_ptr(), pw.rope_cos.data_ptr(), pw.rope_sin.data_ptr(),
                positions.data_ptr(), kv.block_tables.data_ptr(), kv.max_blocks, kv.num_pages,
                kv.page_size, NQ, NKV, B, q.data_ptr(), kv.k_pages[l].data_ptr(),
                kv.v_pages[l].data_ptr(), self.err.data_ptr(), st))
            self._attention(q, l, lengths, B, attn)
            self._gemm(pw.w_o[l], attn, B, out_f32=self._xslot(2 * l))  # partial o_proj
            exchange(2 * l, pw.norm_mlp[l])
            self._gemm(pw.w_gate_up[l].view(2 * I, H), h, B, out=gu)
            _lib.check(lib.mk_swiglu(gu.data_ptr(), B * I, act.data_ptr(), st))
            self._gemm(pw.w_down[l], act, B, out_f32=self._xslot(2 * l + 1))  # partial down
            exchange(2 * l + 1, pw.norm_attn[l + 1] if l + 1 < L else pw.norm_final)
        row0, rows = m.lm_row0, m.lm_rows
        self._gemm(pw.embed[row0:row0 + rows], h, B, out_f32=logits_out)
        _lib.check(lib.mk_argmax_keys(logits_out.data_ptr(), B, rows, row0, keys.data_ptr(), st))
        dist.all_gather_into_tensor(keys_all, keys, group=self.group)
        _lib.check(lib.mk_keys_to_ids(keys_all.data_ptr(), self.tp_world, B, ids_out.data_ptr(),
                                      st))

    def _graph(self, B: int):
        g = self._graphs.get(B)
        if g is None:
            dev = self.dev
            tok = torch.zeros(B, dtype=torch.int32, device=dev)
            pos = torch.zeros(B, dtype=torch.int32, device=dev)
            # this rank's lm_head rows (the whole vocabulary on one GPU)
            logits = torch.empty(B, getattr(self.m, "lm_rows", self.cfg.vocab),
                                 dtype=torch.float32, device=dev)
            ids = torch.empty(B, dtype=torch.int64, device=dev)
            buf = self._buffers(B)
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
                self._step(tok, pos, logits, ids, buf)
            torch.cuda.current_stream().wait_stream(s)
            kv.k_pages[:, page0, :, 0] = saved[0]
            kv.v_pages[:, page0, :, 0] = saved[1]
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._step(tok, pos, logits, ids, buf)
            g = (graph, tok, pos, logits, ids, buf)
            self._graphs[B] = g
        return g

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, positions: torch.Tensor):
        """One greedy step for len(tokens) sequences (row b = cache slot b), K/V
        written at ``positions``; returns (logits [B, V] fp32, ids [B] int64),
        views of the step's static buffers (valid until the next step). On a
        tensor-parallel rank the logits are the rank's vocabulary rows
        (``tp.gather_slices`` assembles them) and the ids are global."""
        B = int(tokens.numel())
        if B > self.max_batch:
            raise ValueError(f"batch {B} > {self.max_batch}")
        pos_host = torch.as_tensor(positions).cpu()
        if bool((pos_host < 0).any()) or bool((pos_host >= self.max_seq_len).any()):
            raise ValueError(f"positions must be in [0, {self.max_seq_len})")
        for b in range(B):
            self.kv.reserve(b, int(pos_host[b]) + 1)
        graph, tok, pos, logits, ids, _ = self._graph(B)
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

    def close(self) -> None:
        """Release the captured step graphs and, on a tensor-parallel rank, the
        exchange buffers (every rank unmaps the others' buffers before any frees
        its own). A rank's graphs hold an NCCL collective (the argmax keys), and
        a process group destroyed while such a graph is alive never finishes
        tearing down: close the decoder first (on every rank of the group)."""
        torch.cuda.synchronize(self.dev)
        self._graphs.clear()
        if self._xbuf is not None:
            dist.barrier(group=self.group)  # no rank reads a peer's buffer any more
            for ptr in self._xpeer_open:
                _lib.check(self.lib.mk_xbuf_close(ptr))
            self._xpeer_open = []
            dist.barrier(group=self.group)  # every mapping of every buffer is gone
            _lib.check(self.lib.mk_xbuf_free(self._xbuf))
            self._xbuf = None

    def check(self) -> None:
        torch.cuda.synchronize(self.dev)
        code = int(self.err[0])
        if code:
            self.err.zero_()
            what = ("a block table names a page outside the pool" if code == 1 else
                    "a tensor-parallel exchange waited too long for another rank" if code == 3 else
                    f"a tcgen05 GEMM wait ran out (code {code})")
            raise _lib.MkError(_lib.MK_EDEVICE, f"batched step: {what}")
