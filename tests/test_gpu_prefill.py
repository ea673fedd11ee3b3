"""GPU prefill (``prefill.py``) against HF ``LlamaForCausalLM`` on the CPU.

HF's forward over the whole prompt is the reference's context-encoding
semantics (its prefill stays on the PyTorch/NxDI path,
llama_with_megakernel.py:194-204). Both sides round the same way in bf16;
they differ by GEMM accumulation order (cuBLAS on the GPU, the CPU's own
kernels), so the bars are the decode bars: cached K/V rows within a few bf16
ulps at layer 0 and cosine >= 0.999 in every layer, last-position logits at
cosine >= 0.999 and max-abs <= 3e-2, and decode steps of the kernel that
continue from the prefilled cache within the same bars of HF continuing from
its own cache.
"""
from __future__ import annotations

import pytest
import torch

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200.config import SMALL
from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM
from oracle import llama_oracle as O

pytestmark = pytest.mark.gpu
KV_ROW_TOL = 0.0625


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm()))


def _hf_kv(cache, layer):
    lay = cache.layers[layer]
    return lay.keys[0], lay.values[0]  # [nkv, T, 64]


@pytest.fixture(scope="module")
def small():
    w = syn.make_weights(SMALL, seed=31)
    return w, O.hf_model(SMALL, w)


def test_prefill_matches_hf_prompt(small):
    w, hf = small
    m = MegakernelLlamaForCausalLM(SMALL, w, max_batch=1, max_seq_len=96, page_size=16)
    toks = syn.random_tokens(37, SMALL.vocab, seed=3).reshape(1, -1)
    out = m.prefill(toks)
    with torch.no_grad():
        ref = hf(toks, use_cache=True)
    rl = ref.logits[0, -1].float()
    assert _cos(out.logits[0].cpu(), rl) >= 0.999
    assert (out.logits[0].cpu() - rl).abs().max() <= 3e-2
    top2 = rl.topk(2).values
    if float(top2[0] - top2[1]) > 3e-2:
        assert int(out.next_ids[0]) == int(rl.argmax())
    k, v = m.kv.gather(0, 37)
    for l in range(SMALL.num_layers):
        hk, hv = _hf_kv(ref.past_key_values, l)
        if l == 0:
            assert (k[l].float().cpu() - hk.float()).abs().max() <= KV_ROW_TOL
            assert (v[l].float().cpu() - hv.float()).abs().max() <= KV_ROW_TOL
        assert _cos(k[l].cpu(), hk) >= 0.999 and _cos(v[l].cpu(), hv) >= 0.999
    assert m.kv.seq_lens[0] == 37

    # decode steps continue from the prefilled cache
    cache = ref.past_key_values
    nxt = int(rl.argmax())
    for _ in range(4):
        o = m.forward(torch.tensor([[nxt]]))
        with torch.no_grad():
            r = hf(torch.tensor([[nxt]]), past_key_values=cache, use_cache=True)
        cache = r.past_key_values
        rl = r.logits[0, -1].float()
        assert _cos(o.logits[0].cpu(), rl) >= 0.999
        assert (o.logits[0].cpu() - rl).abs().max() <= 3e-2
        nxt = int(rl.argmax())


def test_prefill_in_two_parts_and_batched(small):
    w, _ = small
    m = MegakernelLlamaForCausalLM(SMALL, w, max_batch=2, max_seq_len=96, page_size=16)
    toks = syn.random_tokens(30, SMALL.vocab, seed=5).reshape(1, -1)
    whole = m.prefill(toks, past_key_values=m.new_cache())
    kv = m.new_cache()
    m.prefill(toks[:, :11], past_key_values=kv)
    split = m.prefill(toks[:, 11:], past_key_values=kv)
    assert _cos(whole.logits, split.logits) >= 0.9999
    assert kv.seq_lens[0] == 30
    # two sequences in one call, the second continuing after 6 cached tokens
    kv2 = m.new_cache()
    other = syn.random_tokens(6, SMALL.vocab, seed=8).reshape(1, -1)
    m.prefill(torch.cat([toks[:, :6], other]), past_key_values=kv2)
    both = m.prefill(torch.cat([toks[:, 6:18], toks[:, 6:18]]), past_key_values=kv2)
    ref0 = m.prefill(toks[:, :18], past_key_values=m.new_cache())
    assert _cos(both.logits[0], ref0.logits[0]) >= 0.9999
    assert kv2.seq_lens[:2] == [18, 18]


def test_generate_with_prefill_agrees_with_kernel_prompt(small):
    w, _ = small
    m = MegakernelLlamaForCausalLM(SMALL, w, max_batch=1, max_seq_len=96, page_size=16)
    toks = syn.random_tokens(25, SMALL.vocab, seed=12).reshape(1, -1)
    a = m.generate(toks, 8, past_key_values=m.new_cache(), prefill=True)
    b = m.generate(toks, 8, past_key_values=m.new_cache(), prefill=False)
    # the two prompt paths round differently; the first tokens agree
    assert int(a[0, 0]) == int(b[0, 0])


def test_llama1b_prefill_128_token_prompt():
    """BASELINE config 2's prompt: 128 seeded tokens through the prefill
    kernels of full-size Llama-3.2-1B, against HF on the CPU (the reference's
    PyTorch path). Every K/V row lands at its position (nothing else in the
    cache changes), layer-0 rows within a few bf16 ulps, every layer's rows at
    cosine >= 0.999, and the last position's logits at cosine >= 0.999 with
    max-abs inside the 1B bf16 envelope (test_gpu_batched.MAXABS_1B)."""
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg

    w = syn.make_weights(cfg, seed=0, device="cuda")
    m = MegakernelLlamaForCausalLM(cfg, w, max_batch=1, max_seq_len=192, page_size=64)
    w_cpu = {k: v.cpu() for k, v in w.items()}
    del w
    toks = syn.random_tokens(128, cfg.vocab, seed=1).reshape(1, -1)
    m.kv.shuffle_free_pages(3)
    before_k = m.kv.k_pages.clone()
    out = m.prefill(toks)
    hf = O.hf_model(cfg, w_cpu)
    with torch.no_grad():
        ref = hf(toks, use_cache=True)
    rl = ref.logits[0, -1].float()
    err = float((out.logits[0].cpu() - rl).abs().max())
    print(f"1B prefill last logits: cos {_cos(out.logits[0].cpu(), rl):.6f} max|diff| {err:.4f}")
    assert _cos(out.logits[0].cpu(), rl) >= 0.999 and err <= 0.2
    # rows at exactly positions 0..127 of the sequence's pages, nothing else
    changed = (m.kv.k_pages != before_k).any(dim=(0, 2, 4))  # [num_pages, page_size]
    expect = torch.zeros_like(changed)
    for p in range(128):
        expect[int(m.kv.block_tables[0, p // 64]), p % 64] = True
    assert not (changed & ~expect).any(), "prefill wrote outside the prompt's rows"
    k, v = m.kv.gather(0, 128)
    for l in range(cfg.num_layers):
        hk, hv = _hf_kv(ref.past_key_values, l)
        if l == 0:
            assert (k[l].float().cpu() - hk.float()).abs().max() <= KV_ROW_TOL
            assert (v[l].float().cpu() - hv.float()).abs().max() <= KV_ROW_TOL
        assert _cos(k[l].cpu(), hk) >= 0.999 and _cos(v[l].cpu(), hv) >= 0.999, l
    assert m.kv.seq_lens[0] == 128
    del m
    torch.cuda.empty_cache()
