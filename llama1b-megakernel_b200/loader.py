"""Load a Hugging Face Llama checkpoint directory for the megakernel.

The counterpart of the reference's load path: ``load_hf_model``
(llama.py:1287-1288, HF ``LlamaForCausalLM.from_pretrained``), the state-dict
conversion ``convert_hf_to_neuron_state_dict`` (llama_with_megakernel.py:
281-351) and the tied lm_head (``update_state_dict_for_tied_weights``,
llama.py:1405-1406). Reads ``config.json`` and the ``*.safetensors`` files
(one file, or shards listed in ``model.safetensors.index.json``) without
building a torch model, and returns the kernel's ``LlamaDecodeConfig`` plus
the HF-named bf16 weights that ``pack_weights`` / ``shard_state_dict`` take.
RoPE parameters follow the reference's reading of the HF config
(llama.py:852-880): ``rope_theta`` and the llama3 ``rope_scaling`` block
(``rope_parameters`` in configs written by transformers 5).
"""
from __future__ import annotations

import json
from pathlib import Path

import torch
from safetensors.torch import load_file

from .config import LlamaDecodeConfig

_LAYER_KEYS = ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
               "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
               "mlp.down_proj.weight", "input_layernorm.weight", "post_attention_layernorm.weight")


def config_from_hf(hf: dict) -> LlamaDecodeConfig:
    """``LlamaDecodeConfig`` from an HF Llama ``config.json`` dict."""
    if hf.get("model_type", "llama") != "llama":
        raise ValueError(f"not a Llama checkpoint (model_type={hf.get('model_type')!r})")
    nq = hf["num_attention_heads"]
    head_dim = hf.get("head_dim") or hf["hidden_size"] // nq
    kw = dict(num_layers=hf["num_hidden_layers"], hidden=hf["hidden_size"],
              intermediate=hf["intermediate_size"], num_q_heads=nq,
              num_kv_heads=hf.get("num_key_value_heads", nq), head_dim=head_dim,
              vocab=hf["vocab_size"], rms_eps=float(hf.get("rms_norm_eps", 1e-5)),
              rope_theta=float(hf.get("rope_theta", 10000.0)),
              tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)))
    # transformers 5 writes "rope_parameters" (theta inside); 4.x "rope_theta" + "rope_scaling"
    rs = hf.get("rope_parameters") or hf.get("rope_scaling")
    if rs and "rope_theta" in rs:
        kw["rope_theta"] = float(rs["rope_theta"])
    if rs and rs.get("rope_type", rs.get("type")) == "default":
        rs = None
    if rs:
        kind = rs.get("rope_type", rs.get("type"))
        if kind != "llama3":
            raise ValueError(f"rope_scaling type {kind!r} is not supported (llama3 only)")
        kw.update(rope_factor=float(rs["factor"]), rope_low_freq_factor=float(rs["low_freq_factor"]),
                  rope_high_freq_factor=float(rs["high_freq_factor"]),
                  rope_original_max_position=int(rs["original_max_position_embeddings"]))
    else:
        # no scaling: inv_freq unchanged for every wavelength
        kw.update(rope_factor=1.0, rope_low_freq_factor=1.0, rope_high_freq_factor=4.0,
                  rope_original_max_position=2**30)
    return LlamaDecodeConfig(**kw)


def _tensor_files(path: Path) -> list[Path]:
    index = path / "model.safetensors.index.json"
    if index.exists():
        names = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        return [path / n for n in names]
    files = sorted(path.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no *.safetensors in {path}")
    return files


def load_hf_checkpoint(path, device="cpu") -> tuple[LlamaDecodeConfig, dict[str, torch.Tensor]]:
    """(config, HF-named bf16 weights) of the checkpoint directory ``path``.

    The lm_head must be tied to the embedding (Llama-3.2-1B ties them); an
    untied ``lm_head.weight`` that differs from the embedding is refused,
    since the kernel scores the embedding rows.
    """
    path = Path(path)
    cfg = config_from_hf(json.loads((path / "config.json").read_text()))
    cfg.validate()
    raw: dict[str, torch.Tensor] = {}
    for f in _tensor_files(path):
        raw.update(load_file(str(f), device="cpu"))
    sd: dict[str, torch.Tensor] = {}

    def take(name: str) -> torch.Tensor:
        if name not in raw:
            raise KeyError(f"checkpoint lacks {name}")
        return raw[name].to(device=device, dtype=torch.bfloat16)

    sd["model.embed_tokens.weight"] = take("model.embed_tokens.weight")
    for l in range(cfg.num_layers):
        for k in _LAYER_KEYS:
            sd[f"model.layers.{l}.{k}"] = take(f"model.layers.{l}.{k}")
    sd["model.norm.weight"] = take("model.norm.weight")
    head = raw.get("lm_head.weight")
    if head is not None and not torch.equal(head.to(torch.bfloat16), raw["model.embed_tokens.weight"].to(torch.bfloat16)):
        raise ValueError("lm_head.weight is not tied to the embedding; the kernel scores "
                         "embedding rows")
    expect = {"model.embed_tokens.weight": (cfg.vocab, cfg.hidden)}
    for name, shape in expect.items():
        if tuple(sd[name].shape) != shape:
            raise ValueError(f"{name}: shape {tuple(sd[name].shape)} != {shape}")
    return cfg, sd
