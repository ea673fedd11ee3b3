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
