"""ctypes binding of libmk.so (the C ABI declared in include/mk.h).

The shared library is built in-tree by ``build.py`` (nvcc, sm_100a). There is
no fallback: if the library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libmk.so"

MK_OK, MK_EINVAL, MK_ECUDA, MK_ETIMEOUT, MK_ENOMEM, MK_ESTATE, MK_EDEVICE = range(7)
MK_FLAG_FEEDBACK = 1

STATUS_NAMES = {
    MK_OK: "MK_OK", MK_EINVAL: "MK_EINVAL", MK_ECUDA: "MK_ECUDA", MK_ETIMEOUT: "MK_ETIMEOUT",
    MK_ENOMEM: "MK_ENOMEM", MK_ESTATE: "MK_ESTATE", MK_EDEVICE: "MK_EDEVICE",
}

# Every symbol include/mk.h declares (checked by tests/test_abi.py).
EXPORTED = (
    "mk_init", "mk_load_weights", "mk_decode", "mk_decode_host", "mk_decode_static", "mk_decode_hidden",
    "mk_sync",
    "mk_set_timeout_ns", "mk_debug_skip_arrival", "mk_set_trace",
    "mk_query", "mk_schedule_gap", "mk_sample", "mk_paged_attention_workspace",
    "mk_paged_attention", "mk_gemm_workspace", "mk_gemm_bf16", "mk_rmsnorm_rows", "mk_rope_scatter", "mk_swiglu", "mk_argmax_rows",
    "mk_add_rmsnorm_rows", "mk_argmax_keys", "mk_keys_to_ids", "mk_tp_setup", "mk_tp_connect",
    "mk_xbuf_bytes", "mk_xbuf_alloc", "mk_xbuf_open", "mk_xbuf_close", "mk_xbuf_free", "mk_step_epoch",
    "mk_allreduce_add_rmsnorm", "mk_last_error",
    "mk_destroy",
)


class MkError(RuntimeError):
    """A non-zero MkStatus from the library."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class MkConfig(ctypes.Structure):
    _fields_ = [
        ("num_layers", ctypes.c_int32), ("hidden", ctypes.c_int32),
        ("intermediate", ctypes.c_int32), ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("vocab", ctypes.c_int32), ("rms_eps", ctypes.c_float),
        ("max_batch", ctypes.c_int32), ("page_size", ctypes.c_int32),
        ("num_pages", ctypes.c_int32), ("max_blocks_per_seq", ctypes.c_int32),
        ("rope_len", ctypes.c_int32),
    ]


class MkWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "embed", "w_qkv", "w_o", "w_gate_up", "w_down", "norm_attn", "norm_mlp",
        "norm_final", "rope_cos", "rope_sin")]


class MkSampling(ctypes.Structure):
    _fields_ = [("top_k", ctypes.c_int32), ("top_p", ctypes.c_float),
                ("temperature", ctypes.c_float)]


class MkIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class MkKVCache(ctypes.Structure):
    _fields_ = [("k_pages", ctypes.c_void_p), ("v_pages", ctypes.c_void_p),
                ("block_tables", ctypes.c_void_p)]


_lib = None


def load() -> ctypes.CDLL:
    """Load libmk.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FileNotFoundError(
            f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`"
            " or `python -m llama1b_megakernel_b200.build`")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    P, I32, VP = ctypes.POINTER, ctypes.c_int32, ctypes.c_void_p
    lib.mk_init.argtypes = [P(MkConfig), ctypes.c_int, P(VP)]
    lib.mk_load_weights.argtypes = [VP, P(MkWeights)]
    lib.mk_decode.argtypes = [VP, VP, VP, I32, P(MkKVCache), VP, VP, I32, VP]
    lib.mk_decode_host.argtypes = [VP, VP, VP, I32, P(MkKVCache), VP, VP, VP]
    lib.mk_decode_static.argtypes = [P(MkConfig), P(MkWeights), VP, VP, I32, P(MkKVCache), VP, VP,
                                     I32, VP, VP]
    lib.mk_decode_hidden.argtypes = [VP, VP, VP, I32, P(MkKVCache), VP, VP]
    lib.mk_sync.argtypes = [VP, VP]
    lib.mk_set_timeout_ns.argtypes = [VP, ctypes.c_uint64]
    lib.mk_debug_skip_arrival.argtypes = [VP, I32]
    lib.mk_set_trace.argtypes = [VP, VP, ctypes.c_int64, P(ctypes.c_int64)]
    lib.mk_schedule_gap.argtypes = [P(MkConfig), I32, I32, P(I32)]
    lib.mk_query.argtypes = [VP, P(I32), P(I32), P(I32)]
    lib.mk_sample.argtypes = [VP, I32, I32, ctypes.c_int64, P(MkSampling), ctypes.c_uint64,
                              ctypes.c_uint64, VP, VP, VP, VP, VP]
    lib.mk_paged_attention_workspace.argtypes = [I32, I32, I32]
    lib.mk_paged_attention_workspace.restype = ctypes.c_int64
    lib.mk_paged_attention.argtypes = [VP, VP, VP, VP, VP, I32, I32, I32, I32, I32, I32, I32,
                                       ctypes.c_float, VP, ctypes.c_int64, VP, VP, VP]
    lib.mk_gemm_workspace.argtypes = [I32, I32, I32]
    lib.mk_gemm_workspace.restype = ctypes.c_int64
    lib.mk_gemm_bf16.argtypes = [VP, I32, I32, VP, I32, I32, VP, VP, VP, VP, ctypes.c_int64, VP, VP]
    lib.mk_rmsnorm_rows.argtypes = [VP, VP, ctypes.c_float, I32, I32, VP, VP]
    lib.mk_rope_scatter.argtypes = [VP, VP, VP, VP, VP, I32, I32, I32, I32, I32, I32, VP, VP, VP,
                                    VP, VP]
    lib.mk_swiglu.argtypes = [VP, ctypes.c_int64, VP, VP]
    lib.mk_argmax_rows.argtypes = [VP, I32, I32, VP, VP]
    lib.mk_add_rmsnorm_rows.argtypes = [VP, VP, VP, ctypes.c_float, I32, I32, VP, VP]
    lib.mk_argmax_keys.argtypes = [VP, I32, I32, I32, VP, VP]
    lib.mk_keys_to_ids.argtypes = [VP, I32, I32, VP, VP]
    lib.mk_tp_setup.argtypes = [VP, I32, I32, I32, I32, P(MkIpcHandle), P(VP)]
    lib.mk_tp_connect.argtypes = [VP, P(MkIpcHandle), P(VP)]
    lib.mk_xbuf_bytes.argtypes = [I32, I32]
    lib.mk_xbuf_bytes.restype = ctypes.c_int64
    lib.mk_xbuf_alloc.argtypes = [ctypes.c_int64, P(MkIpcHandle), P(VP)]
    lib.mk_xbuf_open.argtypes = [P(MkIpcHandle), P(VP)]
    lib.mk_xbuf_close.argtypes = [VP]
    lib.mk_xbuf_free.argtypes = [VP]
    lib.mk_step_epoch.argtypes = [VP, VP]
    lib.mk_allreduce_add_rmsnorm.argtypes = [VP, I32, I32, I32, I32, VP, VP, VP, ctypes.c_float,
                                             I32, I32, VP, VP, ctypes.c_uint64, VP]
    lib.mk_last_error.argtypes = []
    lib.mk_last_error.restype = ctypes.c_char_p
    lib.mk_destroy.argtypes = [VP]
    for name in EXPORTED:
        if name not in ("mk_last_error", "mk_paged_attention_workspace", "mk_gemm_workspace",
                        "mk_xbuf_bytes"):
            getattr(lib, name).restype = ctypes.c_int
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != MK_OK:
        msg = load().mk_last_error().decode(errors="replace")
        raise MkError(status, msg)
