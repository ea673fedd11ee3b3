"""Batched decode (batched.py + the paged attention kernel) on the GPU.

Against the oracle (HF semantics over the same paged cache, CPU) for batches
of sequences at different lengths: logits cosine >= 0.999 and max-abs <=
3e-2 per sequence, argmax equal where the oracle's top-2 margin exceeds the
measured error, the step's K/V rows written exactly at the step positions
(layer-0 rows within a few bf16 ulps of the oracle's), nothing else touched;
against the persistent megakernel on the same caches (bs 4). A block-table
entry outside the page pool is reported by the attention kernel, not read.
"""
from __future__ import annotations

import pytest
import torch

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200.batched import BatchedDecoder
from llama1b_megakernel_b200.config import SMALL
from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM
from oracle import llama_oracle as O

pytestmark = pytest.mark.gpu
KV_ROW_TOL = 0.0625


def _cos(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float(a @ b / (a.norm() * b.norm()))


@pytest.fixture(scope="module")
def setup():
    w = syn.make_weights(SMALL, seed=17)
    m = MegakernelLlamaForCausalLM(SMALL, w, max_batch=4, max_seq_len=640, page_size=16)
    return w, m


def _fill(kv, cfg, lengths, seed):
    kv.shuffle_free_pages(seed)
    for b, n in enumerate(lengths):
        kv.reserve(b, n + 1)
        if n:
            k, v = syn.random_kv_rows(cfg, n, seed=seed, seq=b)
            kv.fill(b, k, v)


@pytest.mark.parametrize("lengths", [[0, 1, 17, 255, 256, 257, 400, 600],
                                     [31, 32, 33, 5, 511, 512, 513, 100, 7, 300]])
def test_batched_step_matches_oracle(setup, lengths):
    w, m = setup
    B = len(lengths)
    dec = BatchedDecoder(m, max_batch=B, max_seq_len=640, page_size=16)
    _fill(dec.kv, SMALL, lengths, seed=B)
    before_k, before_v = dec.kv.k_pages.clone(), dec.kv.v_pages.clone()
    kv_ref = O.OracleKV(dec.kv.k_pages.cpu().clone(), dec.kv.v_pages.cpu().clone(),
                        dec.kv.block_tables.cpu().clone())
    toks = syn.random_tokens(B, SMALL.vocab, seed=B + 1)
    logits, ids = dec.step(toks, torch.tensor(lengths))
    dec.check()
    logits, ids = logits.cpu(), ids.cpu()
    ref = O.decode_step(SMALL, w, kv_ref, toks, lengths)
    for b in range(B):
        rl = ref["logits"][b].float()
        err = float((logits[b] - rl).abs().max())
        assert _cos(logits[b], rl) >= 0.999 and err <= 3e-2, (b, err)
        top2 = rl.topk(2).values
        if float(top2[0] - top2[1]) > 2 * err:
            assert int(ids[b]) == int(rl.argmax()), b
    ps = dec.kv.page_size
    changed = (dec.kv.k_pages != before_k) | (dec.kv.v_pages != before_v)
    expect = torch.zeros_like(changed)
    for b, n in enumerate(lengths):
        page = int(dec.kv.block_tables[b, n // ps])
        expect[:, page, :, n % ps] = True
        k0 = dec.kv.k_pages[0, page, :, n % ps].float().cpu()
        assert (k0 - ref["k_new"][b][0].float()).abs().max() <= KV_ROW_TOL
    assert not (changed & ~expect).any()


def test_batched_matches_megakernel_bs4(setup):
    w, m = setup
    lengths = [40, 200, 333, 7]
    dec = BatchedDecoder(m, max_batch=4, max_seq_len=640, page_size=16)
    _fill(dec.kv, SMALL, lengths, seed=3)
    kv2 = m.new_cache(max_seq_len=640)
    _fill(kv2, SMALL, lengths, seed=3)
    toks = syn.random_tokens(4, SMALL.vocab, seed=9)
    lb, _ = dec.step(toks, torch.tensor(lengths))
    out = m.forward(toks.reshape(4, 1), torch.tensor(lengths).reshape(4, 1), past_key_values=kv2)
    for b in range(4):
        assert _cos(lb[b].cpu(), out.logits[b].cpu()) >= 0.999


def test_bad_page_reported(setup):
    _, m = setup
    dec = BatchedDecoder(m, max_batch=2, max_seq_len=640, page_size=16)
    _fill(dec.kv, SMALL, [300, 20], seed=5)
    dec.kv.block_tables[0, 3] = dec.kv.num_pages + 7  # an old block: only attention reads it
    dec.step(syn.random_tokens(2, SMALL.vocab, seed=1), torch.tensor([300, 20]))
    with pytest.raises(Exception, match="outside the pool"):
        dec.check()


def test_positions_beyond_rope_table_refused(setup):
    _, m = setup  # RoPE table of 640 positions
    with pytest.raises(ValueError, match="RoPE"):
        BatchedDecoder(m, max_batch=2, max_seq_len=m.rope_len + 1)
    dec = BatchedDecoder(m, max_batch=1, max_seq_len=m.rope_len)
    with pytest.raises(ValueError):
        dec.step(torch.tensor([1]), torch.tensor([m.rope_len]))
    kv = m.new_cache(max_seq_len=m.rope_len + 64, num_pages=64)
    kv.seq_lens[0] = m.rope_len - 2
    with pytest.raises(ValueError, match="RoPE"):
        m.prefill(torch.arange(5)[None], past_key_values=kv)


# ----------------------------------------------------------------------------
# Llama-3.2-1B (bs 8 and 64 at KV length ~1024)
# ----------------------------------------------------------------------------

# The 1B bar: cosine >= 0.999 against the oracle and max-abs within the spread
# that bf16 rounding order alone produces at this size (the reference's own
# bf16 path lies 0.09-0.14 from exact fp32 arithmetic and HF in bf16 on the
# GPU 0.11-0.14 from the reference, test_gpu_parity.py), with margin.
MAXABS_1B = 0.2


@pytest.fixture(scope="module")
def llama():
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B

    w = syn.make_weights(LLAMA_3_2_1B, seed=0, device="cuda")
    m = MegakernelLlamaForCausalLM(LLAMA_3_2_1B, w, max_batch=1, max_seq_len=1088, page_size=64)
    w_cpu = {k: v.cpu() for k, v in w.items()}
    del w
    return LLAMA_3_2_1B, w_cpu, m


@pytest.mark.parametrize("B", [8, 64])
def test_llama1b_batched_step_matches_oracle(llama, B):
    cfg, w, m = llama
    lengths = [1024 - 7 * b % 61 for b in range(B)]  # ragged around 1024
    dec = BatchedDecoder(m, max_batch=B, max_seq_len=1088, page_size=64)
    _fill(dec.kv, cfg, lengths, seed=B)
    toks = syn.random_tokens(B, cfg.vocab, seed=B + 3)
    sample = list(range(B)) if B <= 8 else [0, 1, B // 3, B // 2, B - 2, B - 1]
    # the oracle's sequence i is the decoder's sequence sample[i] (its block-table row)
    kv_ref = O.OracleKV(dec.kv.k_pages.cpu().clone(), dec.kv.v_pages.cpu().clone(),
                        dec.kv.block_tables[sample].cpu().clone())
    logits, ids = dec.step(toks, torch.tensor(lengths))
    dec.check()
    logits, ids = logits.cpu(), ids.cpu()
    ref = O.decode_step(cfg, w, kv_ref, toks[sample], [lengths[b] for b in sample])
    for i, b in enumerate(sample):
        rl = ref["logits"][i].float()
        err = float((logits[b] - rl).abs().max())
        print(f"bs {B} row {b}: cos {_cos(logits[b], rl):.6f} max|diff| {err:.4f}")
        assert _cos(logits[b], rl) >= 0.999 and err <= MAXABS_1B, (b, err)
        top2 = rl.topk(2).values
        if float(top2[0] - top2[1]) > 2 * err:
            assert int(ids[b]) == int(rl.argmax()), b
        page = int(dec.kv.block_tables[b, lengths[b] // 64])
        k0 = dec.kv.k_pages[0, page, :, lengths[b] % 64].float().cpu()
        assert (k0 - ref["k_new"][i][0].float()).abs().max() <= KV_ROW_TOL
    del dec
    torch.cuda.empty_cache()
