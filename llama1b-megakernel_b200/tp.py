"""Tensor-parallel decode: one decode step of one model over 2, 4 or 8 GPUs.

The sharding is Megatron's, as the reference's NxDI baseline layers shard the
same model (gate/up ``ColumnParallelLinear`` and down ``RowParallelLinear``,
llama.py:437-465; q/k/v by head and o_proj row-parallel, llama.py:828): rank r
of W holds q heads [r NQ/W, (r+1) NQ/W), kv heads [r NKV/W, (r+1) NKV/W) with
their cache pages, MLP rows [r I/W, (r+1) I/W), and scores lm_head rows
[r V/W, (r+1) V/W) of the tied embedding. The reference's megakernel itself
is TP = 1 only (llama_with_megakernel.py:145-149).

Where Megatron all-reduces the o_proj and down outputs, the kernel sends its
fp32 partial sums over NVLink into every rank's exchange buffer and every
rank adds them in rank order (see ``mk_tp_setup`` in include/mk.h), so the
residual stream is identical on every rank. This module does the host side:
the shard of an HF state dict, the IPC-handle exchange over a
``torch.distributed`` group (NCCL or gloo), and gathering the logits slices.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .config import LlamaDecodeConfig
from .model import DecodeOutput, MegakernelLlamaForCausalLM

MAX_TP = 8


def shard_config(cfg: LlamaDecodeConfig, world: int) -> LlamaDecodeConfig:
    """The geometry one rank of ``world`` sees (the vocabulary stays whole)."""
    if world < 1 or world > MAX_TP:
        raise ValueError(f"tensor-parallel world {world} outside [1, {MAX_TP}]")
    if cfg.num_kv_heads % world:
        raise ValueError(f"{cfg.num_kv_heads} kv heads do not split over {world} ranks")
    if cfg.intermediate % (256 * world):
        raise ValueError(f"intermediate {cfg.intermediate} does not split into multiples of 256")
    if (cfg.q_dim // world) % 256:
        raise ValueError(f"q_dim {cfg.q_dim} does not split into multiples of 256")
    return cfg.replace(num_q_heads=cfg.num_q_heads // world,
                       num_kv_heads=cfg.num_kv_heads // world,
                       intermediate=cfg.intermediate // world)


def lm_slice(vocab: int, rank: int, world: int) -> tuple[int, int]:
    """(first row, rows) of the lm_head rows rank ``rank`` scores."""
    r0 = vocab * rank // world
    return r0, vocab * (rank + 1) // world - r0


def shard_state_dict(cfg: LlamaDecodeConfig, sd: dict, rank: int, world: int) -> dict:
    """HF-named weights of rank ``rank``: views into ``sd``, in the geometry of
    ``shard_config(cfg, world)``. Norms and the embedding stay whole."""
    local = shard_config(cfg, world)
    qd, kvd, il = local.q_dim, local.kv_dim, local.intermediate
    out = {}
    for name, t in sd.items():
        kind = name.split(".")[-2] if name.count(".") >= 2 else ""
        if kind == "q_proj":
            out[name] = t[rank * qd:(rank + 1) * qd]
        elif kind in ("k_proj", "v_proj"):
            out[name] = t[rank * kvd:(rank + 1) * kvd]
        elif kind == "o_proj":
            out[name] = t[:, rank * qd:(rank + 1) * qd]
        elif kind in ("gate_proj", "up_proj"):
            out[name] = t[rank * il:(rank + 1) * il]
        elif kind == "down_proj":
            out[name] = t[:, rank * il:(rank + 1) * il]
        else:
            out[name] = t
    return out


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's 64-byte exchange-buffer handle, in rank order."""
    out: list = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    return out


def gather_slices(local: torch.Tensor, vocab: int, group=None) -> torch.Tensor:
    """[B, rows] lm_head slices of every rank (``lm_slice`` order) -> [B, vocab]."""
    world = dist.get_world_size(group)
    sizes = [lm_slice(vocab, r, world)[1] for r in range(world)]
    width = max(sizes)  # all_gather moves equal sizes: pad, then trim
    mine = torch.zeros(local.shape[0], width, dtype=local.dtype, device=local.device)
    mine[:, :local.shape[1]] = local
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine, group=group)
    return torch.cat([p[:, :n] for p, n in zip(parts, sizes)], dim=1)


class TensorParallelLlamaForCausalLM(MegakernelLlamaForCausalLM):
    """One rank of a tensor-parallel decode group (one process per GPU).

    ``state_dict`` is the whole model's HF-named weights (any device); the
    rank keeps its shard. Every rank of ``group`` must construct it and then
    make the same calls in the same order (each launch waits for the others
    inside the kernel, with the handle's time limit). ``forward`` returns the
    whole [B, V] logits (gathered over ``group``) and the greedy ids.
    """

    def __init__(self, cfg: LlamaDecodeConfig, state_dict: dict, group=None, max_batch: int = 1,
                 max_seq_len: int = 2048, page_size: int = 64, device="cuda",
                 rope_len: int | None = None):
        self.tp_group = group
        self.tp_rank = dist.get_rank(group)
        self.tp_world = dist.get_world_size(group)
        self.full_cfg = cfg
        local = shard_config(cfg, self.tp_world)
        self.lm_row0, rows = lm_slice(cfg.vocab, self.tp_rank, self.tp_world)
        super().__init__(local, shard_state_dict(cfg, state_dict, self.tp_rank, self.tp_world),
                         max_batch=max_batch, max_seq_len=max_seq_len, page_size=page_size,
                         device=device, rope_len=rope_len, lm_rows=rows)
        handle, buf = _lib.MkIpcHandle(), ctypes.c_void_p()
        _lib.check(self.lib.mk_tp_setup(self._handle, self.tp_rank, self.tp_world, self.lm_row0,
                                        rows, ctypes.byref(handle), ctypes.byref(buf)))
        handles = exchange_handles(bytes(handle.bytes), group)
        arr = (_lib.MkIpcHandle * self.tp_world)()
        for r, h in enumerate(handles):
            ctypes.memmove(arr[r].bytes, h, 64)
        _lib.check(self.lib.mk_tp_connect(self._handle, arr, None))

    @classmethod
    def from_pretrained(cls, path, group=None, **kw) -> "TensorParallelLlamaForCausalLM":
        """This rank of ``group``, from an HF checkpoint directory."""
        from .loader import load_hf_checkpoint

        cfg, sd = load_hf_checkpoint(path)
        return cls(cfg, sd, group=group, **kw)

    @torch.no_grad()
    def forward(self, input_ids, position_ids=None, past_key_values=None, return_logits: bool = True,
                sync: bool = True) -> DecodeOutput:
        out = super().forward(input_ids, position_ids, past_key_values, return_logits, sync)
        if out.logits is not None:
            out = DecodeOutput(gather_slices(out.logits, self.full_cfg.vocab, self.tp_group),
                               out.next_ids, out.past_key_values)
        return out
