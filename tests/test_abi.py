"""The C ABI library without a GPU: it loads, exports every declared symbol,
and rejects bad configurations before touching CUDA."""
import ctypes
import re
from pathlib import Path

import pytest

from llama1b_megakernel_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "mk.h"


@pytest.fixture(scope="module")
def lib():
    from llama1b_megakernel_b200 import build

    build.build()
    return _lib.load()


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(mk_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_bound_symbols():
    assert declared_symbols() == sorted(_lib.EXPORTED)


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def _cfg(**kw):
    base = dict(num_layers=16, hidden=2048, intermediate=8192, num_q_heads=32, num_kv_heads=8,
                head_dim=64, vocab=128256, rms_eps=1e-5, max_batch=1, page_size=64,
                num_pages=32, max_blocks_per_seq=32, rope_len=4096)
    base.update(kw)
    return _lib.MkConfig(**base)


@pytest.mark.parametrize("bad", [
    dict(head_dim=128), dict(num_q_heads=24), dict(hidden=2000), dict(intermediate=16384),
    dict(max_batch=0), dict(max_batch=9), dict(page_size=12), dict(num_pages=0),
    dict(rope_len=0), dict(rms_eps=0.0), dict(num_layers=0),
])
def test_init_rejects_bad_config_without_cuda(lib, bad):
    h = ctypes.c_void_p()
    rc = lib.mk_init(ctypes.byref(_cfg(**bad)), 0, ctypes.byref(h))
    assert rc == _lib.MK_EINVAL
    assert h.value is None
    assert lib.mk_last_error().decode()


def test_null_arguments(lib):
    assert lib.mk_init(None, 0, None) == _lib.MK_EINVAL
    assert lib.mk_load_weights(None, None) == _lib.MK_EINVAL
    assert lib.mk_sync(None, None) == _lib.MK_EINVAL
    assert lib.mk_query(None, None, None, None) == _lib.MK_EINVAL
    assert lib.mk_destroy(None) == _lib.MK_OK
    kv = _lib.MkKVCache()
    rc = lib.mk_decode(None, None, None, 1, ctypes.byref(kv), None, None, 0, None)
    assert rc == _lib.MK_EINVAL and "NULL" in lib.mk_last_error().decode()


def test_check_raises_with_message(lib):
    lib.mk_sync(None, None)
    with pytest.raises(_lib.MkError, match="MK_EINVAL"):
        _lib.check(_lib.MK_EINVAL)


def test_exchange_buffer_layout(lib):
    """Two fp32 [rows][hidden] slots, then the flag words at the next 256-byte
    boundary: 2 slots x 8 ranks of 64-bit words."""
    for rows, hidden in ((1, 8), (32, 2048), (3, 264)):
        slots = 2 * rows * hidden * 4
        flags_at = (slots + 255) // 256 * 256
        assert lib.mk_xbuf_bytes(rows, hidden) == flags_at + 2 * 8 * 8
    assert lib.mk_xbuf_bytes(0, 2048) == 0 and lib.mk_xbuf_bytes(4, 12) == 0


def test_host_entry_points_reject_bad_arguments_without_cuda(lib):
    kv = _lib.MkKVCache()
    tok = (ctypes.c_int32 * 1)(0)
    assert lib.mk_decode_host(None, tok, tok, 1, ctypes.byref(kv), None, tok, None) == _lib.MK_EINVAL
    assert lib.mk_allreduce_add_rmsnorm(None, 0, 2, 1, 0, None, None, None, ctypes.c_float(1e-5),
                                        1, 8, None, None, 0, None) == _lib.MK_EINVAL
    assert lib.mk_step_epoch(None, None) == _lib.MK_EINVAL
    assert lib.mk_xbuf_alloc(0, None, None) == _lib.MK_EINVAL
    assert lib.mk_xbuf_open(None, None) == _lib.MK_EINVAL
    assert lib.mk_xbuf_close(None) == _lib.MK_OK and lib.mk_xbuf_free(None) == _lib.MK_OK
