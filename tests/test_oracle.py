"""The CPU oracle, pinned against the reference's own code and HF Llama.

* RoPE: the oracle's inv_freq / cos / sin equal, bit for bit, what the
  reference's ``Llama3RotaryEmbedding`` (llama.py:888-953) produced when
  run on CPU (tests/golden/rope_llama3.json, made by make_golden.py).
* Decode step: the paged-KV restatement equals HF ``LlamaForCausalLM`` with a
  ``DynamicCache`` bit for bit (bf16 logits) over many steps, with the pages
  deliberately out of order.
* The greedy fixture is self-consistent and was made from the weights the
  seeded generator still produces.
"""
import json
from pathlib import Path

import pytest
import torch

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200 import weights as W
from llama1b_megakernel_b200.config import LLAMA_3_2_1B, SMALL, TINY
from oracle import llama_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def _rope_golden():
    return json.loads((GOLDEN / "rope_llama3.json").read_text())


def test_inv_freq_matches_reference_class():
    g = _rope_golden()
    want = torch.tensor([float.fromhex(h) for h in g["inv_freq_f32_hex"]], dtype=torch.float32)
    got = O.llama3_inv_freq(LLAMA_3_2_1B)
    assert torch.equal(got, want)
    # The product's own table builder restates the same function.
    assert torch.equal(W.llama3_inv_freq(LLAMA_3_2_1B), want)


def test_cos_sin_match_reference_class():
    g = _rope_golden()
    inv = O.llama3_inv_freq(LLAMA_3_2_1B)
    cos_t, sin_t = W.rope_tables(LLAMA_3_2_1B, 8193)
    for p, cb, sb in zip(g["positions"], g["cos_bf16_bits"], g["sin_bf16_bits"]):
        cos, sin = O.rope_cos_sin(inv, torch.tensor([[p]]))
        assert cos.reshape(-1).view(torch.int16).tolist() == cb, p
        assert sin.reshape(-1).view(torch.int16).tolist() == sb, p
        if p < cos_t.shape[0]:
            # The kernel's table rows are the same bits.
            assert cos_t[p].view(torch.int16).tolist() == cb, p
            assert sin_t[p].view(torch.int16).tolist() == sb, p


@pytest.mark.parametrize("cfg", [TINY, SMALL], ids=["tiny", "small"])
def test_restatement_matches_hf_bitwise(cfg):
    from transformers import DynamicCache

    w = syn.make_weights(cfg, seed=11)
    model = O.hf_model(cfg, w)
    steps, ps = 20, 8
    toks = syn.random_tokens(steps, cfg.vocab, seed=12)
    nblk = (steps + ps - 1) // ps
    perm = torch.randperm(nblk + 3, generator=torch.Generator().manual_seed(0))[:nblk]
    kv = O.OracleKV(
        torch.zeros(cfg.num_layers, nblk + 3, cfg.num_kv_heads, ps, 64, dtype=torch.bfloat16),
        torch.zeros(cfg.num_layers, nblk + 3, cfg.num_kv_heads, ps, 64, dtype=torch.bfloat16),
        perm.to(torch.int32).reshape(1, -1))
    cache = DynamicCache(config=model.config)
    with torch.no_grad():
        for t in range(steps):
            out = model(input_ids=toks[t].reshape(1, 1), position_ids=torch.tensor([[t]]),
                        past_key_values=cache, use_cache=True)
            r = O.decode_step(cfg, w, kv, toks[t:t + 1], [t])
            x = O._rmsnorm(r["hidden"].reshape(1, 1, -1), w["model.norm.weight"], cfg.rms_eps)
            bf16_logits = torch.nn.functional.linear(x, w["model.embed_tokens.weight"]).reshape(-1)
            assert torch.equal(bf16_logits, out.logits[0, -1]), t
            # fp32 logits differ from HF's bf16 ones only by the final rounding.
            assert (r["logits"][0] - out.logits[0, -1].float()).abs().max() < 0.02
    # The cache holds exactly HF's K/V rows, at the pages the block table names.
    for l in range(cfg.num_layers):
        K, V = kv.gather(l, 0, steps)
        hk, hv = cache.layers[l].keys[0], cache.layers[l].values[0]
        assert torch.equal(K, hk) and torch.equal(V, hv)


def test_paged_write_lands_in_named_page():
    cfg = TINY
    kv = O.OracleKV(torch.zeros(1, 4, 1, 8, 64, dtype=torch.bfloat16),
                    torch.zeros(1, 4, 1, 8, 64, dtype=torch.bfloat16),
                    torch.tensor([[2, 0, 3]], dtype=torch.int32))
    row = torch.full((1, 64), 3.0, dtype=torch.bfloat16)
    kv.write(0, 0, 13, row, -row)
    assert kv.k_pages[0, 0, 0, 5].eq(3).all() and kv.v_pages[0, 0, 0, 5].eq(-3).all()
    assert kv.k_pages.ne(0).sum() == 64
    del cfg


def test_batched_restatement_is_per_sequence():
    cfg = TINY
    w = syn.make_weights(cfg, seed=5)
    ps, nb = 8, 4

    def fresh(nbatch):
        return O.OracleKV(torch.zeros(cfg.num_layers, nbatch * nb, 1, ps, 64, dtype=torch.bfloat16),
                          torch.zeros(cfg.num_layers, nbatch * nb, 1, ps, 64, dtype=torch.bfloat16),
                          torch.arange(nbatch * nb, dtype=torch.int32).reshape(nbatch, nb))

    kv2 = fresh(2)
    kvs = [fresh(1), fresh(1)]
    toks = syn.random_tokens(10, cfg.vocab, seed=6).reshape(2, 5)
    for t in range(5):
        r2 = O.decode_step(cfg, w, kv2, toks[:, t], [t, t])
        for b in range(2):
            r1 = O.decode_step(cfg, w, kvs[b], toks[b, t:t + 1], [t])
            assert torch.equal(r2["logits"][b], r1["logits"][0])


def test_greedy_fixture_consistent():
    from tests.golden.make_golden import weight_fingerprint

    d = json.loads((GOLDEN / "llama1b_greedy640.json").read_text())
    assert len(d["tokens"]) == 640 and len(d["prompt"]) == 128
    assert d["prompt"] == syn.random_tokens(128, LLAMA_3_2_1B.vocab, seed=d["prompt_seed"]).tolist()
    assert [ids[0] for ids in d["top2_ids"]] == d["tokens"]
    assert d["weight_fingerprint"] == weight_fingerprint(LLAMA_3_2_1B, 0)
