"""Generate the committed golden fixtures under tests/golden/.

Run from the repository root; the RoPE fixture needs a checkout of the
reference, named by the environment variable MK_REFERENCE_DIR (the directory
holding its llama.py):

    MK_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py rope
                                                 # rope_llama3.json
    python tests/golden/make_golden.py greedy    # llama1b_greedy640.json (~1 min)
    python tests/golden/make_golden.py envelope  # adds the fp32 agreement (~20 min)

``rope``: the reference's own ``Llama3RotaryEmbedding`` class is lifted out of
its llama.py with ``ast`` (the module itself cannot be imported here: it
imports the Neuron SDK at the top, llama.py:30) and run on CPU to record
inv_freq and the bf16 cos/sin it produces for a set of positions. The oracle's
restatement (oracle/llama_oracle.py) is tested against these numbers.

``greedy``: the oracle restatement decodes the BASELINE.json workload on CPU:
seeded random-init Llama-3.2-1B, a 128-token seeded prompt fed one token per
step, then 640 greedy steps. The fixture stores the prompt, the 640 greedy
tokens, per-step top-2 logits, and a fingerprint of the weights so a test can
tell whether it regenerated the same model.
"""
from __future__ import annotations

import ast
import json
import math
import os
import sys
import time
from pathlib import Path
from typing import Optional

import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

HERE = Path(__file__).resolve().parent
ROPE_POSITIONS = [0, 1, 2, 7, 63, 127, 128, 511, 767, 1023, 1024, 4095, 8191, 8192, 100000]


def _reference_llama() -> Path:
    d = os.environ.get("MK_REFERENCE_DIR")
    if not d:
        raise SystemExit("set MK_REFERENCE_DIR to the reference checkout (the directory holding "
                         "its llama.py)")
    return Path(d) / "llama.py"


def _reference_rope_class():
    ref = _reference_llama()
    src = ref.read_text()
    tree = ast.parse(src)
    cls = next(n for n in tree.body if isinstance(n, ast.ClassDef) and n.name == "Llama3RotaryEmbedding")
    mod = ast.Module(body=[cls], type_ignores=[])
    ns = {"torch": torch, "nn": torch.nn, "math": math, "Optional": Optional}
    exec(compile(mod, str(ref), "exec"), ns)
    return ns["Llama3RotaryEmbedding"]


def make_rope() -> None:
    cls = _reference_rope_class()
    rot = cls(dim=64, max_position_embeddings=131072, base=500000.0, factor=32.0,
              low_freq_factor=1.0, high_freq_factor=4.0, original_max_position_embeddings=8192)
    inv = rot.get_inv_freqs()
    x = torch.zeros(1, 1, 1, 64, dtype=torch.bfloat16)
    cos_rows, sin_rows = [], []
    for p in ROPE_POSITIONS:
        cos, sin = rot(x, torch.tensor([[p]]))
        cos_rows.append(cos.reshape(-1).view(torch.int16).tolist())
        sin_rows.append(sin.reshape(-1).view(torch.int16).tolist())
    out = {
        "source": "reference llama.py Llama3RotaryEmbedding (get_inv_freqs, forward), run on CPU",
        "params": {"dim": 64, "base": 500000.0, "factor": 32.0, "low_freq_factor": 1.0,
                   "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
        "inv_freq_f32_hex": [float(v).hex() for v in inv.tolist()],
        "positions": ROPE_POSITIONS,
        "cos_bf16_bits": cos_rows,
        "sin_bf16_bits": sin_rows,
    }
    (HERE / "rope_llama3.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote rope_llama3.json")


def weight_fingerprint(cfg, seed: int = 0) -> str:
    """Fingerprint of the seeded weights: the bits of the first 65,536 elements
    of every tensor, in name order. Cheap, because element i of a tensor depends
    only on (seed, tensor, i), so a test can check it without making the model."""
    from llama1b_megakernel_b200 import synthetic as syn

    acc = 0
    for name in sorted(syn.weight_names(cfg)):
        n = min(65536, int(torch.tensor(syn.weight_shape(cfg, name)).prod()))
        if name.endswith("norm.weight"):
            t = torch.ones(n, dtype=torch.bfloat16)
        else:
            t = syn.hashed_normal((n,), seed, syn._stream_of(name), 0.02)
        s = t.view(torch.int16).to(torch.int64)
        acc = (acc * 1_000_003 + int((s * torch.arange(1, n + 1)).sum())) % (1 << 61)
    return f"{acc:016x}"


def make_greedy(n_prompt: int = 128, n_steps: int = 640, seed: int = 0, prompt_seed: int = 1) -> None:
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg
    from oracle import llama_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.time()
    w = syn.make_weights(cfg, seed=seed)
    print(f"weights {time.time() - t0:.1f}s")
    fp = weight_fingerprint(cfg, seed)
    prompt = syn.random_tokens(n_prompt, cfg.vocab, seed=prompt_seed)
    ps = 64
    max_len = n_prompt + n_steps
    nblk = (max_len + ps - 1) // ps
    kv = O.OracleKV(
        torch.zeros(cfg.num_layers, nblk, cfg.num_kv_heads, ps, cfg.head_dim, dtype=torch.bfloat16),
        torch.zeros(cfg.num_layers, nblk, cfg.num_kv_heads, ps, cfg.head_dim, dtype=torch.bfloat16),
        torch.arange(nblk, dtype=torch.int32).reshape(1, -1),
    )
    inv = O.llama3_inv_freq(cfg)
    t0 = time.time()
    with torch.no_grad():
        for t in range(n_prompt - 1):
            O.decode_step(cfg, w, kv, prompt[t:t + 1], [t], inv_freq=inv, layers=cfg.num_layers)
        tok = int(prompt[-1])
        tokens, top2v, top2i = [], [], []
        for s in range(n_steps):
            r = O.decode_step(cfg, w, kv, [tok], [n_prompt - 1 + s], inv_freq=inv)
            v, i = r["logits"][0].topk(2)
            top2v.append([float(x).hex() for x in v.tolist()])
            top2i.append(i.tolist())
            tok = int(r["next"][0])
            tokens.append(tok)
    print(f"decode {time.time() - t0:.1f}s")
    out = {
        "config": "Llama-3.2-1B (LLAMA_3_2_1B), synthetic.make_weights(seed=%d)" % seed,
        "weight_fingerprint": fp,
        "prompt_seed": prompt_seed,
        "prompt": prompt.tolist(),
        "page_size": ps,
        "first_decode_position": n_prompt - 1,
        "tokens": tokens,
        "top2_logits_f32_hex": top2v,
        "top2_ids": top2i,
    }
    (HERE / "llama1b_greedy640.json").write_text(json.dumps(out) + "\n")
    print("wrote llama1b_greedy640.json")


def make_envelope() -> None:
    """fp32 evaluation of the greedy workload, teacher-forced on the fixture.

    The same decode steps in fp32 arithmetic (weights widened from the same
    bf16 values, fp32 cache, the same bf16 RoPE table), fed the fixture's own
    tokens. Its argmax agreement with the bf16 greedy tokens measures how many
    decisions in this random-init model are within bf16 rounding noise: any
    correct implementation whose rounding differs from the reference's is
    expected to agree at about this rate, not at 100%.
    """
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg
    from oracle import llama_oracle as O

    torch.set_num_threads(os.cpu_count() or 1)
    path = HERE / "llama1b_greedy640.json"
    d = json.loads(path.read_text())
    w = {k: v.float() for k, v in syn.make_weights(cfg, seed=0).items()}
    ps = d["page_size"]
    n_prompt, n_steps = len(d["prompt"]), len(d["tokens"])
    nblk = (n_prompt + n_steps + ps - 1) // ps
    kv = O.OracleKV(
        torch.zeros(cfg.num_layers, nblk, cfg.num_kv_heads, ps, cfg.head_dim),
        torch.zeros(cfg.num_layers, nblk, cfg.num_kv_heads, ps, cfg.head_dim),
        torch.arange(nblk, dtype=torch.int32).reshape(1, -1))
    inv = O.llama3_inv_freq(cfg)
    feed = [d["prompt"][-1]] + d["tokens"][:-1]
    t0 = time.time()
    ids = []
    with torch.no_grad():
        for t in range(n_prompt - 1):
            O.decode_step(cfg, w, kv, d["prompt"][t:t + 1], [t], inv_freq=inv, layers=cfg.num_layers)
        for s in range(n_steps):
            r = O.decode_step(cfg, w, kv, [feed[s]], [n_prompt - 1 + s], inv_freq=inv)
            ids.append(int(r["next"][0]))
    match = sum(int(a == b) for a, b in zip(ids, d["tokens"])) / n_steps
    print(f"fp32 teacher-forced match {match:.4f} ({time.time() - t0:.0f}s)")
    d["fp32_teacher_forced_match"] = match
    d["fp32_teacher_forced_ids"] = ids
    path.write_text(json.dumps(d) + "\n")


def refresh_fingerprint() -> None:
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg

    path = HERE / "llama1b_greedy640.json"
    d = json.loads(path.read_text())
    d["weight_fingerprint"] = weight_fingerprint(cfg, 0)
    path.write_text(json.dumps(d) + "\n")


if __name__ == "__main__":
    what = sys.argv[1:] or ["rope"]
    if "fingerprint" in what:
        refresh_fingerprint()
    if "rope" in what:
        make_rope()
    if "greedy" in what:
        make_greedy()
    if "envelope" in what:
        make_envelope()
