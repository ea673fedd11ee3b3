"""The tcgen05 skinny GEMM (``mk_gemm_bf16``, csrc/mk_gemm.cuh) against fp64 sums.

Y = X W^T (+ R) for the batched decode and prefill shapes: every output within
one bf16 rounding (2^-7 relative, 1e-4 absolute for the fp32 sum) of the
exactly summed product of the same bf16 inputs (with a residual, HF's two
roundings: bf16(R + bf16(X W^T))), fp32 outputs within 1e-4, for padded
batches 16 / 32 / 64 / 128 with fewer real rows, with and without the split
along K, with a residual, and with fp32 output.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from llama1b_megakernel_b200 import _lib

pytestmark = pytest.mark.gpu


def _run(lib, w, x, rows, residual=None, f32=False):
    n, k = w.shape
    bp = x.shape[0]
    dev = w.device
    out = torch.empty(rows, n, dtype=torch.float32 if f32 else torch.bfloat16, device=dev)
    ws = lib.mk_gemm_workspace(n, k, rows)
    work = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.mk_gemm_bf16(
        w.data_ptr(), n, k, x.data_ptr(), rows, bp,
        residual.data_ptr() if residual is not None else None,
        None if f32 else out.data_ptr(), out.data_ptr() if f32 else None,
        work.data_ptr(), work.numel(), err.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(err[0]) == 0
    return out


@pytest.mark.parametrize("n,k,rows,bp", [(3072, 2048, 8, 16), (2048, 2048, 32, 32),
                                         (16384, 2048, 64, 64), (2048, 8192, 20, 32),
                                         (128 * 11, 192, 1, 16), (5003, 512, 3, 16),
                                         (3072, 2048, 128, 128), (2048, 8192, 100, 128),
                                         (5003, 512, 77, 128)])
def test_gemm_matches_exact_sum(n, k, rows, bp):
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(n + k + rows)
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    x = torch.zeros(bp, k, dtype=torch.bfloat16, device="cuda")
    x[:rows] = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
    res = torch.randn(rows, n, generator=g, device="cuda").bfloat16()
    exact = x[:rows].double() @ w.double().T
    y = _run(lib, w, x, rows)
    # one bf16 rounding (<= 2^-8 relative) of an fp32 sum (absolute slack 1e-4)
    assert ((y.double() - exact).abs() <= exact.abs() * 2.0 ** -7 + 1e-4).all()
    yr = _run(lib, w, x, rows, residual=res)
    er = exact + res.double()
    # two roundings: of the product (relative to it) and of the sum
    assert ((yr.double() - er).abs() <= (exact.abs() + er.abs()) * 2.0 ** -8 + 1e-4).all()
    yf = _run(lib, w, x, rows, f32=True)
    assert ((yf.double() - exact).abs() <= exact.abs() * 1e-4 + 1e-4).all()


def test_gemm_rejects_bad_shapes():
    lib = _lib.load()
    w = torch.zeros(128, 100, dtype=torch.bfloat16, device="cuda")  # k not a multiple of 64
    x = torch.zeros(16, 100, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1, 128, dtype=torch.bfloat16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.mk_gemm_bf16(w.data_ptr(), 128, 100, x.data_ptr(), 1, 16, None, out.data_ptr(), None,
                          None, 0, err.data_ptr(), None)
    assert rc == _lib.MK_EINVAL


def test_gemms_sharing_one_workspace():
    """Split-K GEMMs of different shapes in sequence on one workspace (as a
    batched step runs them): each matches its own exact sum."""
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(5)
    shapes = [(3072, 2048), (2048, 2048), (2048, 8192), (3072, 2048)]
    rows, bp = 24, 32
    ws = max(lib.mk_gemm_workspace(n, k, rows) for n, k in shapes)
    work = torch.zeros(ws, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for n, k in shapes:
        w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
        x = torch.zeros(bp, k, dtype=torch.bfloat16, device="cuda")
        x[:rows] = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
        out = torch.empty(rows, n, dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.mk_gemm_bf16(w.data_ptr(), n, k, x.data_ptr(), rows, bp, None,
                                    out.data_ptr(), None, work.data_ptr(), ws, err.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        exact = x[:rows].double() @ w.double().T
        assert int(err[0]) == 0
        assert ((out.double() - exact).abs() <= exact.abs() * 2.0 ** -7 + 1e-4).all(), (n, k)
