"""HF checkpoint loading (config.json + safetensors) on CPU.

A checkpoint written by HF ``save_pretrained`` (the reference loads with
``LlamaForCausalLM.from_pretrained``, llama.py:1287-1288) must come back as
the same config and the same bf16 tensors; sharded checkpoints (an index
file), transformers-4 style ``rope_scaling`` configs and untied heads are
covered too.
"""
from __future__ import annotations

import json

import pytest
import torch
from safetensors.torch import save_file

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200.config import LLAMA_3_2_1B, TINY
from llama1b_megakernel_b200.loader import config_from_hf, load_hf_checkpoint
from oracle import llama_oracle as O

HF_1B_V4 = {  # the fields of Llama-3.2-1B's published config.json (transformers 4 layout)
    "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 2048,
    "intermediate_size": 8192, "num_attention_heads": 32, "num_hidden_layers": 16,
    "num_key_value_heads": 8, "head_dim": 64, "vocab_size": 128256, "rms_norm_eps": 1e-05,
    "rope_theta": 500000.0, "tie_word_embeddings": True, "torch_dtype": "bfloat16",
    "rope_scaling": {"factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
                     "original_max_position_embeddings": 8192, "rope_type": "llama3"},
}


def test_config_from_v4_json_is_llama_3_2_1b():
    assert config_from_hf(HF_1B_V4) == LLAMA_3_2_1B


def test_save_pretrained_round_trip(tmp_path):
    w = syn.make_weights(TINY, seed=4)
    O.hf_model(TINY, w).save_pretrained(tmp_path, safe_serialization=True)
    cfg, sd = load_hf_checkpoint(tmp_path)
    assert cfg == TINY
    assert sd.keys() == w.keys()
    for k in w:
        assert sd[k].dtype == torch.bfloat16 and torch.equal(sd[k], w[k]), k


def test_sharded_checkpoint_with_index(tmp_path):
    w = syn.make_weights(TINY, seed=6)
    names = sorted(w)
    half = len(names) // 2
    save_file({k: w[k].contiguous() for k in names[:half]}, str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file({k: w[k].contiguous() for k in names[half:]}, str(tmp_path / "model-00002-of-00002.safetensors"))
    wm = {k: ("model-00001-of-00002.safetensors" if i < half else "model-00002-of-00002.safetensors")
          for i, k in enumerate(names)}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": wm}))
    hf = dict(HF_1B_V4, hidden_size=TINY.hidden, intermediate_size=TINY.intermediate,
              num_attention_heads=TINY.num_q_heads, num_hidden_layers=TINY.num_layers,
              num_key_value_heads=TINY.num_kv_heads, vocab_size=TINY.vocab)
    (tmp_path / "config.json").write_text(json.dumps(hf))
    cfg, sd = load_hf_checkpoint(tmp_path)
    assert cfg == TINY
    assert all(torch.equal(sd[k], w[k]) for k in w)


def test_untied_head_refused(tmp_path):
    w = syn.make_weights(TINY, seed=7)
    t = {k: v.contiguous() for k, v in w.items()}
    t["lm_head.weight"] = torch.zeros_like(w["model.embed_tokens.weight"])
    save_file(t, str(tmp_path / "model.safetensors"))
    hf = dict(HF_1B_V4, hidden_size=TINY.hidden, intermediate_size=TINY.intermediate,
              num_attention_heads=TINY.num_q_heads, num_hidden_layers=TINY.num_layers,
              num_key_value_heads=TINY.num_kv_heads, vocab_size=TINY.vocab, tie_word_embeddings=False)
    (tmp_path / "config.json").write_text(json.dumps(hf))
    with pytest.raises(ValueError, match="tied"):
        load_hf_checkpoint(tmp_path)


def test_non_llama_refused():
    with pytest.raises(ValueError):
        config_from_hf(dict(HF_1B_V4, model_type="mistral"))


@pytest.mark.gpu
def test_from_pretrained_matches_in_memory_weights(tmp_path):
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    w = syn.make_weights(TINY, seed=4)
    O.hf_model(TINY, w).save_pretrained(tmp_path, safe_serialization=True)
    a = MegakernelLlamaForCausalLM.from_pretrained(tmp_path, max_batch=1, max_seq_len=64)
    b = MegakernelLlamaForCausalLM(TINY, w, max_batch=1, max_seq_len=64)
    toks = syn.random_tokens(9, TINY.vocab, seed=2).reshape(1, -1)
    oa, ob = a.forward(toks), b.forward(toks)
    assert torch.equal(oa.logits, ob.logits) and torch.equal(oa.next_ids, ob.next_ids)
