"""Tensor-parallel decode on 2+ GPUs against the single-GPU kernel.

Runs ``tests/tp_worker.py`` under torchrun (one process per GPU, NCCL for
the host-side plumbing, the kernel's own peer-memory exchange for the
partial sums) and checks what rank 0 measured. Skipped on a box with fewer
than two GPUs. Tolerances: the TP and single-GPU steps differ only by fp32
summation order inside o_proj / down (a partial per rank, then the ranks in
order), which flips a bf16 rounding now and then and grows through the
layers' residual; logits must agree to cosine >= 0.9999 and max-abs <= 5e-2
(measured on 1B-shaped layers: cosine 0.99999), greedy ids at >= 95% of
teacher-forced steps, the layer-0 K/V rows (computed before any exchange)
bit for bit, and the on-device greedy feedback exactly as step-by-step
forward calls.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world: int, config: str, tmp_path: Path) -> dict:
    out = tmp_path / f"tp{world}_{config}.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           str(ROOT / "tests" / "tp_worker.py"), "--config", config, "--out", str(out)]
    proc = subprocess.run(["timeout", "-k", "30", "300", *cmd], cwd=ROOT, env=env,
                          capture_output=True, text=True)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    res = json.loads(out.read_text())
    print(json.dumps(res))
    assert res.get("ok"), res
    return res


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("config", ["mid", "small"])
def test_tp2_matches_single_gpu(tmp_path, config):
    r = _run(2, config, tmp_path)
    assert r["kv_layer0_exact"], r
    assert r["cos_min"] >= 0.9999, r
    assert r["maxabs_max"] <= 5e-2, r
    assert r["ids_match"] >= 0.95, r
    assert r["generate_self_consistent"], r
    assert r["batch_cos_min"] >= 0.9999, r
    _check_oracle_and_batched(r)


def _check_oracle_and_batched(r):
    # against the oracle: the single-GPU parity bar (these are 2- and 3-layer
    # models). With Llama-3.2-1B-shaped layers (config "mid") that bar is the
    # single-GPU tests' fp32 envelope: distance to an fp32 evaluation of the
    # step at most 1.5x the oracle's own distance (+1e-3), since rounding order
    # alone moves those logits by ~3e-2 (measured on 2 GPUs: 0.035 max-abs
    # against the oracle, inside the envelope).
    assert r["oracle_cos_min"] >= 0.999, r
    assert r["tp_batched_oracle_cos_min"] >= 0.999, r
    if r.get("oracle_envelope_excess") is None:
        assert r["oracle_maxabs_max"] <= 3e-2, r
        assert r["tp_batched_oracle_maxabs"] <= 3e-2, r
    else:
        assert r["oracle_envelope_excess"] <= 1e-3, r
        assert r["tp_batched_envelope_excess"] <= 1e-3, r
    # batched TP step against the single-GPU batched step
    assert r["tp_batched_cos_min"] >= 0.9999, r
    assert r["tp_batched_ids_equal"] and r["tp_batched_oracle_ids_equal"], r


@pytest.mark.skipif(_gpus() < 8, reason="needs 8 GPUs")
def test_tp8_one_kv_head_per_gpu(tmp_path):
    r = _run(8, "mid", tmp_path)
    assert r["kv_layer0_exact"], r
    assert r["cos_min"] >= 0.9999 and r["maxabs_max"] <= 5e-2, r
    assert r["ids_match"] >= 0.95, r
    assert r["generate_self_consistent"], r
    _check_oracle_and_batched(r)


@pytest.mark.skipif(_gpus() < 4, reason="needs 4 GPUs")
def test_tp4_two_kv_heads_per_gpu(tmp_path):
    """Four ranks: the peer exchanges sum four partials in rank order."""
    r = _run(4, "mid", tmp_path)
    assert r["kv_layer0_exact"], r
    assert r["cos_min"] >= 0.9999 and r["maxabs_max"] <= 5e-2, r
    assert r["ids_match"] >= 0.95, r
    assert r["generate_self_consistent"], r
    _check_oracle_and_batched(r)
