"""Host side of tensor-parallel decode, on CPU (no GPU).

* ``shard_config`` / ``shard_state_dict`` / ``lm_slice``: the shards of every
  rank put back together are the whole model, and each rank's shard is what
  a Megatron split gives (q/k/v rows of its heads, o_proj and down columns,
  gate/up rows, a contiguous lm_head slice).
* The exchange-buffer handles and the logits slices travel over a
  ``torch.distributed`` group: run here as two ``gloo`` ranks on 127.0.0.1.
* The arithmetic: o_proj / down summed per rank in fp32 and then across ranks
  in rank order (what the kernel's exchange does) round to the same bf16
  values as whole-row sums except at rounding ties, off by one ulp there.
"""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200 import tp
from llama1b_megakernel_b200.config import LLAMA_3_2_1B, MID, SMALL


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_config_1b(world):
    c = tp.shard_config(LLAMA_3_2_1B, world)
    assert c.num_q_heads * world == 32 and c.num_kv_heads * world == 8
    assert c.intermediate * world == 8192 and c.vocab == LLAMA_3_2_1B.vocab
    c.validate()


def test_shard_config_rejects_uneven():
    with pytest.raises(ValueError):
        tp.shard_config(SMALL, 4)  # 2 kv heads over 4 ranks
    with pytest.raises(ValueError):
        tp.shard_config(LLAMA_3_2_1B, 16)


@pytest.mark.parametrize("vocab,world", [(128256, 8), (4099, 2), (5003, 4), (7, 8)])
def test_lm_slices_cover_the_vocabulary(vocab, world):
    rows = [tp.lm_slice(vocab, r, world) for r in range(world)]
    assert rows[0][0] == 0
    for (r0, n), (r1, _) in zip(rows, rows[1:]):
        assert r0 + n == r1
    assert rows[-1][0] + rows[-1][1] == vocab


@pytest.mark.parametrize("cfg,world", [(SMALL, 2), (MID, 2), (MID, 8)])
def test_shards_reassemble_the_model(cfg, world):
    sd = syn.make_weights(cfg.replace(num_layers=1), seed=3)
    shards = [tp.shard_state_dict(cfg, sd, r, world) for r in range(world)]
    for name, full in sd.items():
        kind = name.split(".")[-2] if name.count(".") >= 2 else ""
        parts = [s[name] for s in shards]
        if kind in ("q_proj", "k_proj", "v_proj", "gate_proj", "up_proj"):
            assert torch.equal(torch.cat(parts, 0), full)
        elif kind in ("o_proj", "down_proj"):
            assert torch.equal(torch.cat(parts, 1), full)
        else:
            assert all(p is full for p in parts)
    local = tp.shard_config(cfg, world)
    q = shards[1]["model.layers.0.self_attn.q_proj.weight"]
    assert q.shape == (local.q_dim, cfg.hidden)
    assert torch.equal(q, sd["model.layers.0.self_attn.q_proj.weight"][local.q_dim:2 * local.q_dim])


# ---------------------------------------------------------------------------
# gloo world 2: handle exchange and logits gathering
# ---------------------------------------------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _work(rank, world, q)
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, repr(e), None, False))
    finally:
        dist.destroy_process_group()


def _work(rank: int, world: int, q) -> None:
    handle = bytes([rank + 1]) * 64
    got = tp.exchange_handles(handle)
    vocab = 4099
    r0, n = tp.lm_slice(vocab, rank, world)
    rows = 1000.0 * torch.arange(2, dtype=torch.float32)[:, None]
    local = torch.arange(r0, r0 + n, dtype=torch.float32)[None, :] + rows
    full = tp.gather_slices(local, vocab)
    want = torch.arange(vocab, dtype=torch.float32)[None, :] + rows
    q.put((rank, [h[0] for h in got], full.shape, bool(torch.equal(full, want))))


def test_gloo_world2_exchange_and_gather():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, order, shape, ok in res:
        assert order == [1, 2], order
        assert tuple(shape) == (2, 4099) and ok


# ---------------------------------------------------------------------------
# arithmetic: rank-order sum of per-rank fp32 partials
# ---------------------------------------------------------------------------

def _rbf(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def test_rank_order_partial_sums_match_whole_rows():
    """o_proj / down as the kernel computes them under TP: each rank's fp32
    dot product over its columns, then the ranks' partials added in rank
    order, then one bf16 rounding; against the whole-row fp32 dot product
    rounded once. The two differ only by fp32 summation order, so after the
    bf16 rounding they agree except at rounding ties (< 1% of the outputs,
    off by one bf16 ulp)."""
    g = torch.Generator().manual_seed(0)
    w = _rbf(torch.randn(2048, 8192, generator=g) * 0.02)
    x = _rbf(torch.randn(8192, generator=g))
    whole = _rbf((w.double() @ x.double()).float())
    for world in (2, 4, 8):
        cols = 8192 // world
        acc = torch.zeros(2048)
        for r in range(world):
            acc = acc + (w[:, r * cols:(r + 1) * cols].double() @ x[r * cols:(r + 1) * cols].double()).float()
        tpv = _rbf(acc)
        diff = (tpv != whole)
        assert diff.float().mean() < 0.01
        ulp = (whole.abs() * 2.0 ** -7).clamp_min(2.0 ** -133)
        assert ((tpv - whole).abs()[diff] <= ulp[diff] * 1.01).all()
