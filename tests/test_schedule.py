"""The ring's barrier-distance bound, checked on the host (no GPU).

The decode kernel's consumer warps wait only for the ring fills they read, and
an mbarrier phase is named by its parity, so a warp's wait is safe only while
it never goes more than ``64 - ring_slots - 8`` fills between two waits (64
full barriers used round-robin, producers at most 8 fills apart; the argument
is in the Ring comment of ``csrc/mk_kernel.cuh``). ``mk_init`` refuses a
geometry that breaks it, using ``mk_schedule_gap``. These tests restate the
kernel's fill schedule in Python (``walk_schedule`` and ``gemv_phase``'s item
to warp map) and require the library's walk to agree with it, and the shipped
geometries to stay inside the bound with room to spare.
"""
from __future__ import annotations

import ctypes

import pytest

from llama1b_megakernel_b200 import _lib
from llama1b_megakernel_b200.config import LLAMA_3_2_1B, MID, SMALL, TINY

CONSUMER_WARPS = 14
FULL_BARS = 64
PRODUCER_SLACK = 8
SLOT_BYTES = 16384
MAX_SPLIT = 32


def pieces_per_row(k: int) -> int:
    n = (k + 2047) // 2048
    while n <= k // 256:
        if k % n == 0 and (k // n) % 256 == 0:
            return n
        n += 1
    return k // 256


def split_units(u: int, g: int, c: int, rot: int) -> tuple[int, int]:
    base, rem = u // g, u % g
    end = rot + rem
    if end <= g:
        before = min(max(c - rot, 0), rem)
    else:
        before = min(c, end - g) + min(max(c - rot, 0), g - rot)
    extra = ((c - rot + g) % g) < rem
    u0 = c * base + before
    return u0, u0 + base + (1 if extra else 0)


def max_gap(cfg, batch: int, grid: int) -> int:
    """Largest fill distance between consecutive waits of one consumer warp
    (-1: a warp's first wait is at fill 64 or later); each attention item
    counts as one fill no warp reads."""
    h, i, qd = cfg.hidden, cfg.intermediate, cfg.num_q_heads * 64
    nqkv = cfg.num_q_heads + 2 * cfg.num_kv_heads
    nh, nqd, ni = pieces_per_row(h), pieces_per_row(qd), pieces_per_row(i)
    ns = min(MAX_SPLIT, max(1, grid // (batch * cfg.num_kv_heads)))
    t_items = batch * cfg.num_kv_heads * ns
    worst = 0
    for c in range(grid):
        rot, f = 0, 0
        last = [None] * CONSUMER_WARPS

        def gemv(units, unit_bytes, ipu):
            nonlocal rot, f, worst
            u0, u1 = split_units(units, grid, c, rot)
            rot = (rot + units % grid) % grid
            ups = max(1, SLOT_BYTES // unit_bytes)
            for u in range(u0, u1, ups):
                p_items, t0 = min(ups, u1 - u) * ipu, (u - u0) * ipu
                for w in range(CONSUMER_WARPS):
                    if t0 + (w - t0 % CONSUMER_WARPS) % CONSUMER_WARPS >= t0 + p_items:
                        continue
                    if f >= FULL_BARS:
                        worst = max(worst, 2**31 - 1 if last[w] is None else f - last[w])
                    last[w] = f
                f += 1

        items = len(range(c, t_items, grid))
        for _ in range(cfg.num_layers):
            gemv(nqkv * 32, 4 * h, 2 * nh)
            f += items
            gemv(h, 2 * qd, nqd)
            gemv(i, 4 * h, 2 * nh)
            gemv(h, 2 * i, ni)
        gemv(cfg.vocab, 2 * h, 1)
    return -1 if worst == 2**31 - 1 else worst


def _mk_cfg(cfg, max_batch=4):
    return _lib.MkConfig(
        num_layers=cfg.num_layers, hidden=cfg.hidden, intermediate=cfg.intermediate,
        num_q_heads=cfg.num_q_heads, num_kv_heads=cfg.num_kv_heads, head_dim=64, vocab=cfg.vocab,
        rms_eps=1e-5, max_batch=max_batch, page_size=64, num_pages=64, max_blocks_per_seq=16,
        rope_len=1024)


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def _lib_gap(lib, cfg, batch, grid):
    gap = ctypes.c_int32()
    rc = lib.mk_schedule_gap(ctypes.byref(_mk_cfg(cfg)), batch, grid, ctypes.byref(gap))
    assert rc == _lib.MK_OK, lib.mk_last_error().decode()
    return gap.value


@pytest.mark.parametrize("name,cfg,batch,grid", [
    ("1B", LLAMA_3_2_1B, 1, 148), ("1B", LLAMA_3_2_1B, 4, 148), ("1B", LLAMA_3_2_1B, 4, 8),
    ("MID", MID, 2, 148), ("MID", MID, 4, 1),
    ("SMALL", SMALL, 1, 8), ("SMALL", SMALL, 3, 1), ("TINY", TINY, 4, 1),
])
def test_library_walk_matches_restatement(lib, name, cfg, batch, grid):
    assert _lib_gap(lib, cfg, batch, grid) == max_gap(cfg, batch, grid)


@pytest.mark.parametrize("cfg", [LLAMA_3_2_1B, MID, SMALL, TINY])
def test_shipped_geometries_inside_the_bound(lib, cfg):
    # 12 ring slots is what mk_init picks for Llama-3.2-1B at batch 1; 16 is
    # the most it ever picks, the tightest bound.
    bound = FULL_BARS - 16 - PRODUCER_SLACK
    for batch in (1, 2, 3, 4):
        gap = _lib_gap(lib, cfg, batch, 148)
        assert 0 <= gap <= bound // 2, (batch, gap, bound)


def test_schedule_gap_argument_checks(lib):
    gap = ctypes.c_int32()
    assert lib.mk_schedule_gap(None, 1, 148, ctypes.byref(gap)) == _lib.MK_EINVAL
    cfg = _mk_cfg(TINY, max_batch=2)
    assert lib.mk_schedule_gap(ctypes.byref(cfg), 3, 148, ctypes.byref(gap)) == _lib.MK_EINVAL
    assert lib.mk_schedule_gap(ctypes.byref(cfg), 1, 0, ctypes.byref(gap)) == _lib.MK_EINVAL
    assert lib.mk_schedule_gap(ctypes.byref(cfg), 1, 148, None) == _lib.MK_EINVAL
