"""mk_decode_static, the allocation-free decode entry point, against mk_decode.

Some callers of this library cannot allocate device memory: their own pool
already owns it, they run inside another runtime's allocator callback, or a
cudaMalloc (which can synchronise the device) would stall a latency-critical
loop. For them the library keeps the kernel's scratch in a static device
array and mk_decode_static takes everything else from the caller. These tests
call it through the C ABI and check it against the handle-based mk_decode,
with the parity tolerances of the other GPU tests. The file is named to be
collected last.
"""
import ctypes

import pytest
import torch

from llama1b_megakernel_b200 import _lib
from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200.config import LLAMA_3_2_1B, SMALL, TINY

pytestmark = pytest.mark.gpu

COS_MIN = 0.999  # per-step logits cosine similarity
MAXABS = 3e-2    # per-step logits max |diff|


def _config(m, **over):
    kw = dict(num_layers=m.cfg.num_layers, hidden=m.cfg.hidden, intermediate=m.cfg.intermediate,
              num_q_heads=m.cfg.num_q_heads, num_kv_heads=m.cfg.num_kv_heads,
              head_dim=m.cfg.head_dim, vocab=m.cfg.vocab, rms_eps=m.cfg.rms_eps,
              max_batch=m.max_batch, page_size=m.page_size, num_pages=m.kv.num_pages,
              max_blocks_per_seq=m.kv.max_blocks, rope_len=m.rope_len)
    kw.update(over)
    return _lib.MkConfig(**kw)


def _static_step(m, kv, tok, pos, logits, nxt, err):
    cfg = _config(m)
    kvs = m._kv_struct(kv)
    rc = m.lib.mk_decode_static(ctypes.byref(cfg), ctypes.byref(m._weights), tok.data_ptr(),
                                pos.data_ptr(), tok.numel(), ctypes.byref(kvs), logits.data_ptr(),
                                nxt.data_ptr(), 0, err.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)


@pytest.fixture(scope="module")
def small_model():
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    w = syn.make_weights(SMALL, seed=31)
    return MegakernelLlamaForCausalLM(SMALL, w, max_batch=1, max_seq_len=256, page_size=32,
                                      device="cuda:0")


def _model(cfg, seed, max_seq_len, page_size):
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    w = syn.make_weights(cfg, seed=seed, device="cuda:0")
    return MegakernelLlamaForCausalLM(cfg, w, max_batch=1, max_seq_len=max_seq_len,
                                      page_size=page_size, device="cuda:0")


def _compare_steps(m, kv_ref, kv_st, tok, pos, err, what):
    """One step through mk_decode (kv_ref) and mk_decode_static (kv_st)."""
    dev = m.device
    lg_ref = torch.empty(1, m.cfg.vocab, dtype=torch.float32, device=dev)
    lg_st = torch.empty_like(lg_ref)
    id_ref = torch.empty(1, dtype=torch.int32, device=dev)
    id_st = torch.empty_like(id_ref)
    m.launch(tok, pos, kv_ref, lg_ref, id_ref)
    m.sync()
    _static_step(m, kv_st, tok, pos, lg_st, id_st, err)
    torch.cuda.synchronize()
    assert err.tolist() == [0, 0, 0, 0], what
    cos = torch.nn.functional.cosine_similarity(lg_st, lg_ref, dim=-1).item()
    diff = (lg_st - lg_ref).abs().max().item()
    assert cos >= COS_MIN and diff <= MAXABS, (what, cos, diff)
    assert int(id_st[0]) == int(id_ref[0]), what


def _filled_cache(m, n, seed):
    kv = m.new_cache()
    k, v = syn.random_kv_rows(m.cfg, n, seed=seed)
    kv.fill(0, k, v)
    kv.reserve(0, n + 2)
    return kv


def test_static_matches_handle_on_two_consecutive_steps(small_model):
    m = small_model
    n = 77
    kv_ref, kv_st = _filled_cache(m, n, seed=5), _filled_cache(m, n, seed=5)
    dev = m.device
    toks = syn.random_tokens(2, m.cfg.vocab, seed=6).to(torch.int32)
    err = torch.full((4,), -1, dtype=torch.int32, device=dev)
    for step in range(2):
        tok = toks[step:step + 1].to(dev)
        pos = torch.tensor([n + step], dtype=torch.int32, device=dev)
        lg_ref = torch.empty(1, m.cfg.vocab, dtype=torch.float32, device=dev)
        lg_st = torch.empty_like(lg_ref)
        id_ref = torch.empty(1, dtype=torch.int32, device=dev)
        id_st = torch.empty_like(id_ref)
        m.launch(tok, pos, kv_ref, lg_ref, id_ref)
        m.sync()
        _static_step(m, kv_st, tok, pos, lg_st, id_st, err)
        torch.cuda.synchronize()
        assert err.tolist() == [0, 0, 0, 0]
        cos = torch.nn.functional.cosine_similarity(lg_st, lg_ref, dim=-1).item()
        diff = (lg_st - lg_ref).abs().max().item()
        assert cos >= COS_MIN and diff <= MAXABS, (step, cos, diff)
        assert int(id_st[0]) == int(id_ref[0]), step
    # Both paths wrote the same K/V rows at both positions.
    k_ref, v_ref = kv_ref.gather(0, n + 2)
    k_st, v_st = kv_st.gather(0, n + 2)
    assert torch.equal(k_ref, k_st) and torch.equal(v_ref, v_st)


def test_static_reports_device_errors_and_recovers(small_model):
    m = small_model
    dev = m.device
    kv = _filled_cache(m, 10, seed=8)
    err = torch.zeros(4, dtype=torch.int32, device=dev)
    lg = torch.empty(1, m.cfg.vocab, dtype=torch.float32, device=dev)
    nxt = torch.empty(1, dtype=torch.int32, device=dev)
    bad = torch.tensor([m.cfg.vocab + 3], dtype=torch.int32, device=dev)
    pos = torch.tensor([10], dtype=torch.int32, device=dev)
    _static_step(m, kv, bad, pos, lg, nxt, err)
    torch.cuda.synchronize()
    assert int(err[0]) == 5  # token outside the vocabulary
    good = torch.tensor([7], dtype=torch.int32, device=dev)
    _static_step(m, kv, good, pos, lg, nxt, err)
    torch.cuda.synchronize()
    assert err.tolist() == [0, 0, 0, 0]
    assert 0 <= int(nxt[0]) < m.cfg.vocab


def test_static_rejects_geometry_beyond_the_array(small_model):
    m = small_model
    big = _lib.MkConfig(num_layers=16, hidden=2048, intermediate=8192, num_q_heads=32,
                        num_kv_heads=8, head_dim=64, vocab=128256, rms_eps=1e-5, max_batch=4,
                        page_size=64, num_pages=16, max_blocks_per_seq=16, rope_len=1024)
    kvs = m._kv_struct(m.kv)
    dummy = torch.zeros(4, dtype=torch.int32, device=m.device)
    rc = m.lib.mk_decode_static(ctypes.byref(big), ctypes.byref(m._weights), dummy.data_ptr(),
                                dummy.data_ptr(), 1, ctypes.byref(kvs), None, dummy.data_ptr(), 0,
                                None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MK_EINVAL
    assert "static array" in m.lib.mk_last_error().decode()


def test_static_at_llama_1b_geometry():
    """Llama-3.2-1B at max_batch 1, the geometry the static array is sized
    for: two consecutive steps at ctx 1024 against mk_decode."""
    m = _model(LLAMA_3_2_1B, seed=0, max_seq_len=1088, page_size=64)
    n = 1024
    kv_ref, kv_st = _filled_cache(m, n, seed=11), _filled_cache(m, n, seed=11)
    toks = syn.random_tokens(2, m.cfg.vocab, seed=12).to(torch.int32)
    err = torch.full((4,), -1, dtype=torch.int32, device=m.device)
    for step in range(2):
        tok = toks[step:step + 1].to(m.device)
        pos = torch.tensor([n + step], dtype=torch.int32, device=m.device)
        _compare_steps(m, kv_ref, kv_st, tok, pos, err, f"1B step {step}")
    k_ref, v_ref = kv_ref.gather(0, n + 2)
    k_st, v_st = kv_st.gather(0, n + 2)
    assert torch.equal(k_ref, k_st) and torch.equal(v_ref, v_st)
    del m, kv_ref, kv_st
    torch.cuda.empty_cache()


def test_static_alternating_geometries():
    """Calls that alternate between two models of different depth and width
    share the one static array; each step must still equal its own model's
    handle-based mk_decode step (stale words of the other model's layout
    must never pass for this call's activations)."""
    tiny = _model(TINY, seed=41, max_seq_len=128, page_size=16)
    small = _model(SMALL, seed=42, max_seq_len=128, page_size=32)
    caches = {}
    for name, m in (("tiny", tiny), ("small", small)):
        caches[name] = (_filled_cache(m, 40, seed=43), _filled_cache(m, 40, seed=43))
    err = torch.full((4,), -1, dtype=torch.int32, device=tiny.device)
    for step in range(6):
        for name, m in (("tiny", tiny), ("small", small)):
            kv_ref, kv_st = caches[name]
            tok = torch.tensor([(17 * step + 5) % m.cfg.vocab], dtype=torch.int32, device=m.device)
            pos = torch.tensor([40 + step], dtype=torch.int32, device=m.device)
            for c in (kv_ref, kv_st):
                c.reserve(0, 40 + step + 1)
            _compare_steps(m, kv_ref, kv_st, tok, pos, err, f"{name} step {step}")
