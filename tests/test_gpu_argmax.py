"""mk_argmax_rows (csrc/mk_batched.cuh) against torch.argmax.

The batched decode step's greedy ids: the first column holding each row's
maximum, bit-exact against torch.argmax (which also returns the first
occurrence), for the Llama-3.2-1B vocabulary (128-bit loads), an odd width
(the scalar path), rows whose maximum repeats, and rows that are not 16-byte
aligned.
"""
from __future__ import annotations

import pytest
import torch

from llama1b_megakernel_b200 import _lib

pytestmark = pytest.mark.gpu


def _argmax(x: torch.Tensor) -> torch.Tensor:
    lib = _lib.load()
    ids = torch.full((x.shape[0],), -1, dtype=torch.int64, device=x.device)
    _lib.check(lib.mk_argmax_rows(x.data_ptr(), x.shape[0], x.shape[1], ids.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return ids


@pytest.mark.parametrize("rows,cols", [(64, 128256), (3, 5003), (1, 1), (8, 4096)])
def test_matches_torch(rows, cols):
    g = torch.Generator(device="cuda").manual_seed(rows + cols)
    x = torch.randn(rows, cols, device="cuda", generator=g)
    assert torch.equal(_argmax(x), x.argmax(dim=-1))


def test_ties_take_the_first_column():
    x = torch.zeros(4, 2048, device="cuda")
    x[0, [7, 900, 2047]] = 3.0
    x[1, [2047, 5]] = 1.0
    x[3, :] = -1.0  # all equal: column 0
    ids = _argmax(x)
    assert ids.tolist() == [7, 5, 0, 0]
    assert torch.equal(ids, x.argmax(dim=-1))


def test_unaligned_rows():
    base = torch.randn(5 * 1001 + 1, device="cuda")
    x = base[1:].view(5, 1001)  # 4-byte offset: the scalar path
    assert torch.equal(_argmax(x), x.argmax(dim=-1))
