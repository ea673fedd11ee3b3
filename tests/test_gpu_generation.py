"""The HF-style generate adapter (generation.py) on the GPU.

Rows of a left-padded batch must decode exactly as the same prompts do one
by one through ``MegakernelLlamaForCausalLM.generate(prefill=True)``; scores
are the per-step logits; eos ends a row with padding after it; an HF
``GenerationConfig`` supplies the knobs.
"""
from __future__ import annotations

import pytest
import torch

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200.config import SMALL
from llama1b_megakernel_b200.generation import HuggingFaceGenerationAdapter
from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    return MegakernelLlamaForCausalLM(SMALL, syn.make_weights(SMALL, seed=41), max_batch=3,
                                      max_seq_len=128, page_size=16)


def test_padded_batch_matches_single_rows(model):
    p = [syn.random_tokens(n, SMALL.vocab, seed=n) for n in (5, 11, 8)]
    T = 11
    ids = torch.full((3, T), 2, dtype=torch.int64)
    mask = torch.zeros(3, T, dtype=torch.int64)
    for b, r in enumerate(p):  # left padding
        ids[b, T - r.numel():] = r
        mask[b, T - r.numel():] = 1
    out = HuggingFaceGenerationAdapter(model).generate(
        input_ids=ids, attention_mask=mask, max_new_tokens=10, min_new_tokens=10,
        do_sample=False, return_dict_in_generate=True, output_scores=True)
    assert out.sequences.shape == (3, T + 10)
    assert torch.equal(out.sequences[:, :T], ids)
    assert len(out.scores) == 10 and out.scores[0].shape == (3, SMALL.vocab)
    for b, r in enumerate(p):
        one = model.generate(r.reshape(1, -1), 10, past_key_values=model.new_cache(), prefill=True)
        assert torch.equal(out.sequences[b, T:], one[0].cpu()), b
        # greedy: each generated token is the argmax of the step's scores
        assert all(int(out.scores[s][b].argmax()) == int(out.sequences[b, T + s]) for s in range(10))


def test_eos_pads_and_generation_config(model):
    from transformers import GenerationConfig

    prompt = syn.random_tokens(6, SMALL.vocab, seed=77).reshape(1, -1)
    ad = HuggingFaceGenerationAdapter(model)
    free = ad.generate(prompt, max_new_tokens=8)
    eos = int(free[0, 6 + 2])  # the third new token
    cut = ad.generate(prompt, generation_config=GenerationConfig(max_new_tokens=8, eos_token_id=eos,
                                                                 pad_token_id=0, do_sample=False))
    first = next(j for j in range(8) if int(free[0, 6 + j]) == eos)
    assert torch.equal(cut[0, :6 + first + 1], free[0, :6 + first + 1])
    assert (cut[0, 6 + first + 1:] == 0).all()
