"""PyTorch module around the decode megakernel.

``MegakernelLlamaForCausalLM`` plays the role of the reference's
``NeuronLlamaForCausalLMMK`` (llama_with_megakernel.py:355): it owns the packed
weights (converted once, like ``convert_hf_to_neuron_state_dict``,
llama_with_megakernel.py:281-351), and its ``forward`` runs decode steps with
the same inputs an HF/NxDI causal LM takes during token generation —
``input_ids``, ``position_ids`` and ``past_key_values`` — returning fp32
logits, the greedy next ids and the (in-place updated) cache.

Every step is one launch of the persistent kernel through the C ABI; there is
no CPU or PyTorch fallback: without a CUDA device or without libmk.so the
constructor raises.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .config import LlamaDecodeConfig
from .kv_cache import PagedKVCache
from .weights import PackedWeights, pack_weights


@dataclass
class DecodeOutput:
    logits: torch.Tensor | None   # [B, V] fp32 (last step), or None
    next_ids: torch.Tensor        # [B] int64 greedy ids of the last step
    past_key_values: PagedKVCache


class MegakernelLlamaForCausalLM(torch.nn.Module):
    def __init__(self, cfg: LlamaDecodeConfig, state_dict: dict, max_batch: int = 1,
                 max_seq_len: int = 2048, page_size: int = 64, device="cuda",
                 rope_len: int | None = None, lm_rows: int | None = None):
        super().__init__()
        if not torch.cuda.is_available():
            raise RuntimeError("MegakernelLlamaForCausalLM needs a CUDA device (sm_100a)")
        cfg.validate()
        self.lib = _lib.load()
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.page_size = page_size
        self.rope_len = rope_len or max_seq_len
        with torch.cuda.device(self.device):
            self.packed: PackedWeights = pack_weights(cfg, state_dict, self.rope_len, self.device)
            self.kv = PagedKVCache(cfg, max_batch, max_seq_len, page_size, device=self.device)
            self._tokens = torch.zeros(max_batch, dtype=torch.int32, device=self.device)
            self._positions = torch.zeros(max_batch, dtype=torch.int32, device=self.device)
            self._next = torch.zeros(max_batch, dtype=torch.int32, device=self.device)
            # host staging for forward()'s single-position calls (mk_decode_host
            # copies through the handle's own pinned buffer)
            self._h_in = np.zeros((2, max_batch), dtype=np.int32)
            self._h_next = np.zeros(max_batch, dtype=np.int32)
            self._h_addr = (self._h_in[0].ctypes.data, self._h_in[1].ctypes.data,
                            self._h_next.ctypes.data)
            # lm_head rows this model scores (a tensor-parallel rank scores a slice)
            self.lm_rows = lm_rows or cfg.vocab
            self._logits = torch.empty(max_batch, self.lm_rows, dtype=torch.float32,
                                       device=self.device)
        self._handle = ctypes.c_void_p()
        c = _lib.MkConfig(
            num_layers=cfg.num_layers, hidden=cfg.hidden, intermediate=cfg.intermediate,
            num_q_heads=cfg.num_q_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
            vocab=cfg.vocab, rms_eps=cfg.rms_eps, max_batch=max_batch, page_size=page_size,
            num_pages=self.kv.num_pages, max_blocks_per_seq=self.kv.max_blocks,
            rope_len=self.rope_len)
        _lib.check(self.lib.mk_init(ctypes.byref(c), self.device.index, ctypes.byref(self._handle)))
        pw = self.packed
        self._weights = _lib.MkWeights(
            embed=pw.embed.data_ptr(), w_qkv=pw.w_qkv.data_ptr(), w_o=pw.w_o.data_ptr(),
            w_gate_up=pw.w_gate_up.data_ptr(), w_down=pw.w_down.data_ptr(),
            norm_attn=pw.norm_attn.data_ptr(), norm_mlp=pw.norm_mlp.data_ptr(),
            norm_final=pw.norm_final.data_ptr(), rope_cos=pw.rope_cos.data_ptr(),
            rope_sin=pw.rope_sin.data_ptr())
        _lib.check(self.lib.mk_load_weights(self._handle, ctypes.byref(self._weights)))

    @classmethod
    def from_pretrained(cls, path, **kw) -> "MegakernelLlamaForCausalLM":
        """Build from an HF checkpoint directory (config.json + safetensors), the
        way the reference loads its model (llama.py:1287-1288); ``kw`` as for
        the constructor."""
        from .loader import load_hf_checkpoint

        cfg, sd = load_hf_checkpoint(path)
        return cls(cfg, sd, **kw)

    # ------------------------------------------------------------------ misc
    def __del__(self):
        h = self.__dict__.get("_handle")
        if h is not None and h.value:
            self.lib.mk_destroy(h)
            h.value = None

    def new_cache(self, max_seq_len: int | None = None, num_pages: int | None = None) -> PagedKVCache:
        """A fresh cache with this model's geometry (same pool size unless given)."""
        return PagedKVCache(self.cfg, self.max_batch, max_seq_len or self.max_seq_len,
                            self.page_size, num_pages or self.kv.num_pages, device=self.device)

    def query(self) -> dict:
        g, s, m = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        _lib.check(self.lib.mk_query(self._handle, ctypes.byref(g), ctypes.byref(s), ctypes.byref(m)))
        return {"grid": g.value, "ring_slots": s.value, "smem_bytes": m.value}

    def set_timeout_ns(self, ns: int) -> None:
        _lib.check(self.lib.mk_set_timeout_ns(self._handle, int(ns)))

    def debug_skip_arrival(self, cta: int) -> None:
        _lib.check(self.lib.mk_debug_skip_arrival(self._handle, int(cta)))

    def set_trace(self, enable: bool = True) -> torch.Tensor | None:
        """Record the phase trace of every later launch into a device buffer
        (int64, [grid, num_layers * 5 + 1, 12]; see ``mk_set_trace``), or stop."""
        need = ctypes.c_int64()
        if not enable:
            _lib.check(self.lib.mk_set_trace(self._handle, None, 0, ctypes.byref(need)))
            self._trace = None
            return None
        _lib.check(self.lib.mk_set_trace(self._handle, None, 0, ctypes.byref(need)))
        grid = self.query()["grid"]
        buf = torch.zeros(need.value, dtype=torch.int64, device=self.device)
        _lib.check(self.lib.mk_set_trace(self._handle, buf.data_ptr(), buf.numel(),
                                         ctypes.byref(need)))
        self._trace = buf.view(grid, self.cfg.num_layers * 5 + 1, 12)
        return self._trace

    def _kv_struct(self, kv: PagedKVCache) -> _lib.MkKVCache:
        st = kv.__dict__.get("_mk_struct")
        if st is not None and st[0] is self:
            return st[1]
        if kv.num_pages > self.kv.num_pages or kv.max_blocks != self.kv.max_blocks \
                or kv.page_size != self.page_size:
            raise ValueError("cache geometry differs from the one the model was initialised with")
        s = _lib.MkKVCache(k_pages=kv.k_pages.data_ptr(), v_pages=kv.v_pages.data_ptr(),
                           block_tables=kv.block_tables.data_ptr())
        kv._mk_struct = (self, s)  # the pool tensors never move, so the struct stays valid
        return s

    @staticmethod
    def _stream_ptr(stream) -> int:
        s = stream if stream is not None else torch.cuda.current_stream()
        return s.cuda_stream

    # ------------------------------------------------------------ low level
    def launch(self, tokens: torch.Tensor, positions: torch.Tensor, kv: PagedKVCache,
               logits: torch.Tensor | None, next_ids: torch.Tensor, feedback: bool = False,
               stream=None) -> None:
        """Enqueue one step (device int32 tensors, no host sync, no page allocation)."""
        B = positions.numel()
        kvs = self._kv_struct(kv)
        _lib.check(self.lib.mk_decode(
            self._handle, tokens.data_ptr(), positions.data_ptr(), B, ctypes.byref(kvs),
            logits.data_ptr() if logits is not None else None, next_ids.data_ptr(),
            _lib.MK_FLAG_FEEDBACK if feedback else 0, self._stream_ptr(stream)))

    def launch_hidden(self, hidden_in: torch.Tensor, positions: torch.Tensor, kv: PagedKVCache,
                      hidden_out: torch.Tensor, stream=None) -> None:
        """Enqueue the decoder layers only: hidden_in [B, H] bf16 -> hidden_out [B, H] bf16."""
        B = positions.numel()
        kvs = self._kv_struct(kv)
        _lib.check(self.lib.mk_decode_hidden(
            self._handle, hidden_in.data_ptr(), positions.data_ptr(), B, ctypes.byref(kvs),
            hidden_out.data_ptr(), self._stream_ptr(stream)))

    def sync(self, stream=None) -> None:
        """Wait for the stream and raise ``MkError`` if the device reported one."""
        _lib.check(self.lib.mk_sync(self._handle, self._stream_ptr(stream)))

    # ------------------------------------------------------------ model API
    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor | None = None,
                past_key_values: PagedKVCache | None = None, return_logits: bool = True,
                sync: bool = True) -> DecodeOutput:
        """Run ``input_ids`` [B, T] through the model one position at a time.

        ``position_ids`` [B, T] default to each sequence's current length.
        K/V rows are written at those positions of ``past_key_values`` (the
        model's own cache when None). Returns the last step's fp32 logits
        [B, V] (on the device), its greedy ids [B] int64 (on the host once
        synchronised; the device tensor with ``sync=False``) and the cache.
        """
        kv = past_key_values if past_key_values is not None else self.kv
        if (sync and position_ids is not None and type(input_ids) is torch.Tensor
                and type(position_ids) is torch.Tensor and input_ids.device.type == "cpu"
                and position_ids.device.type == "cpu"):
            n = input_ids.numel()
            if (n == position_ids.numel() and n <= self.max_batch
                    and (input_ids.dim() == 2 and input_ids.shape[1] == 1
                         or input_ids.dim() == 1 and n == 1)):
                return self._step_host(input_ids, position_ids, kv, return_logits)
        return self._forward(input_ids, position_ids, kv, return_logits, sync)

    def _step_host(self, input_ids: torch.Tensor, position_ids: torch.Tensor, kv: PagedKVCache,
                   return_logits: bool) -> DecodeOutput:
        """One position of B sequences from host tensors: the numbers go through
        numpy into the staging arrays and one C call (mk_decode_host) copies
        them in, launches, copies the greedy ids out and synchronises, so the
        step's host work is a handful of Python operations."""
        h = self._h_in
        B = input_ids.numel()
        h[0, :B] = input_ids.numpy().reshape(-1)
        h[1, :B] = position_ids.numpy().reshape(-1)
        lens = kv.seq_lens
        for b in range(B):
            p = int(h[1, b]) + 1
            kv.reserve(b, p)
            if p > lens[b]:
                lens[b] = p
        logits = self._logits[:B] if return_logits else None
        a_tok, a_pos, a_next = self._h_addr
        _lib.check(self.lib.mk_decode_host(
            self._handle, a_tok, a_pos, B, ctypes.byref(self._kv_struct(kv)),
            logits.data_ptr() if logits is not None else None, a_next,
            torch.cuda.current_stream(self.device).cuda_stream))
        return DecodeOutput(logits.clone() if logits is not None else None,
                            torch.from_numpy(self._h_next[:B].astype(np.int64)), kv)

    @torch.no_grad()
    def _forward(self, input_ids, position_ids, kv: PagedKVCache, return_logits: bool,
                 sync: bool) -> DecodeOutput:
        ids = torch.as_tensor(input_ids)
        if ids.dim() == 1:
            ids = ids[None, :]
        B, T = ids.shape
        if B > self.max_batch:
            raise ValueError(f"batch {B} > max_batch {self.max_batch}")
        if position_ids is None:
            start = torch.tensor(kv.seq_lens[:B], dtype=torch.int64)
            position_ids = start[:, None] + torch.arange(T)[None, :]
        pos = torch.as_tensor(position_ids).reshape(B, T)
        pos_host = pos if pos.device.type == "cpu" else pos.cpu()
        last = pos_host.max(dim=1).values.tolist() if T > 1 else pos_host[:, 0].tolist()
        for b in range(B):
            kv.reserve(b, last[b] + 1)
        logits = self._logits[:B] if return_logits else None
        ids_dev = ids.to(device=self.device, dtype=torch.int32, non_blocking=True)
        pos_dev = pos.to(device=self.device, dtype=torch.int32, non_blocking=True)
        for t in range(T):
            self.launch(ids_dev[:, t].contiguous(), pos_dev[:, t].contiguous(), kv,
                        logits if t == T - 1 else None, self._next[:B])
        for b in range(B):
            if last[b] + 1 > kv.seq_lens[b]:
                kv.seq_lens[b] = last[b] + 1
        if not sync:
            return DecodeOutput(logits, self._next[:B].to(torch.int64), kv)
        nxt = self._next[:B].cpu()  # waits for the stream
        self.sync()
        return DecodeOutput(logits.clone() if logits is not None else None,
                            nxt.to(torch.int64), kv)

    def sample(self, logits: torch.Tensor, top_k: int = 1, top_p: float = 1.0,
               temperature: float = 1.0, seed: int = 0, step: int = 0,
               tokens: torch.Tensor | None = None, positions: torch.Tensor | None = None,
               out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Draw one id per row of fp32 ``logits`` [B, V] on the device (``mk_sample``:
        temperature, top_k, top_p, a uniform hashed from seed/step/row). With
        ``tokens``/``positions`` the draw is fed back like MK_FLAG_FEEDBACK.
        Asynchronous; returns the int32 ids tensor."""
        B = logits.shape[0]
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=logits.device)
        if not hasattr(self, "_sample_err"):
            self._sample_err = torch.zeros(1, dtype=torch.int32, device=self.device)
        params = (_lib.MkSampling * B)(*[_lib.MkSampling(int(top_k), float(top_p), float(temperature))
                                          for _ in range(B)])
        _lib.check(self.lib.mk_sample(
            logits.data_ptr(), B, logits.shape[1], logits.stride(0), params, int(seed), int(step),
            out.data_ptr(), tokens.data_ptr() if tokens is not None else None,
            positions.data_ptr() if positions is not None else None, self._sample_err.data_ptr(),
            self._stream_ptr(stream)))
        return out

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor,
                past_key_values: PagedKVCache | None = None) -> DecodeOutput:
        """Prompt prefill with PyTorch on the GPU (all positions of a layer at
        once, see ``prefill.py``): fills the cache from each sequence's current
        length and returns the last position's logits and greedy ids."""
        from .prefill import prefill as _prefill

        kv = past_key_values if past_key_values is not None else self.kv
        logits, ids = _prefill(self, input_ids, kv)
        return DecodeOutput(logits, ids, kv)

    @torch.no_grad()
    def forward_hidden(self, hidden: torch.Tensor, position_ids: torch.Tensor,
                       past_key_values: PagedKVCache | None = None) -> torch.Tensor:
        """The decoder layers only (the reference kernel's X -> Y): [B, H] -> [B, H]."""
        kv = past_key_values if past_key_values is not None else self.kv
        h = hidden.reshape(-1, self.cfg.hidden).to(self.device, torch.bfloat16).contiguous()
        B = h.shape[0]
        pos = torch.as_tensor(position_ids).reshape(B)
        for b in range(B):
            kv.reserve(b, int(pos[b]) + 1)
        pos_dev = pos.to(device=self.device, dtype=torch.int32)
        out = torch.empty_like(h)
        self.launch_hidden(h, pos_dev, kv, out)
        for b in range(B):
            kv.seq_lens[b] = max(kv.seq_lens[b], int(pos[b]) + 1)
        self.sync()
        return out

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int,
                 past_key_values: PagedKVCache | None = None,
                 prefill: bool = False, do_sample: bool = False, top_k: int = 1,
                 top_p: float = 1.0, temperature: float = 1.0, seed: int = 0,
                 cache_last: bool = False) -> torch.Tensor:
        """Greedy decoding: feed the prompt, then ``max_new_tokens`` steps on device.

        The prompt goes through the decode kernel one position per launch, or
        with ``prefill=True`` through the PyTorch prefill (all positions of a
        layer at once; ``prefill.py``).
        The generated steps run back to back without host round trips: each
        launch writes its argmax into the next launch's token slot and bumps
        the position (MK_FLAG_FEEDBACK), or with ``do_sample`` each launch
        writes its logits and ``mk_sample`` (``sample``) draws the next token
        with ``top_k`` / ``top_p`` / ``temperature`` (draw s of the call uses
        step s of ``seed``) and feeds it back the same way. Returns
        [B, max_new_tokens] int64.

        As with HF ``generate``, the cache ends holding the prompt and every
        generated token but the last (whose K/V row no step has computed
        yet); ``cache_last=True`` runs one more step to write that row too,
        for a caller that continues from the cache (a whole 2.47 GB weight
        stream for one K/V row).
        """
        kv = past_key_values if past_key_values is not None else self.kv
        if do_sample and self.lm_rows != self.cfg.vocab:
            raise NotImplementedError("sampling needs the whole vocabulary's logits on one GPU")
        ids = torch.as_tensor(input_ids)
        if ids.dim() == 1:
            ids = ids[None, :]
        B, T = ids.shape
        if prefill:
            out = self.prefill(ids, past_key_values=kv)
        else:
            out = self.forward(ids, past_key_values=kv, return_logits=do_sample, sync=True)
        start = torch.tensor(kv.seq_lens[:B], dtype=torch.int32)
        for b in range(B):
            kv.reserve(b, int(start[b]) + max_new_tokens)
        tok = self._tokens[:B]
        pos = self._positions[:B]
        knobs = dict(top_k=top_k, top_p=top_p, temperature=temperature, seed=seed)
        if do_sample:
            self.sample(out.logits.to(self.device).contiguous(), step=0, out=tok, **knobs)
        else:
            tok.copy_(out.next_ids.to(torch.int32))
        pos.copy_(start.to(self.device))
        result = torch.empty(B, max_new_tokens, dtype=torch.int32, device=self.device)
        result[:, 0] = tok
        logits = self._logits[:B]
        for s in range(1, max_new_tokens):
            if do_sample:
                self.launch(tok, pos, kv, logits, self._next[:B])
                self.sample(logits, step=s, tokens=tok, positions=pos, out=self._next[:B], **knobs)
            else:
                self.launch(tok, pos, kv, None, self._next[:B], feedback=True)
            result[:, s] = tok
        if cache_last:
            self.launch(tok, pos, kv, None, self._next[:B], feedback=True)
        self.sync()
        if do_sample and int(self._sample_err[0]):
            self._sample_err.zero_()
            raise _lib.MkError(_lib.MK_EDEVICE, "sampling: more than 1024 logits tied at the top_k "
                               "threshold")
        for b in range(B):
            kv.seq_lens[b] = int(start[b]) + max_new_tokens - (0 if cache_last else 1)
        return result.to(torch.int64)
