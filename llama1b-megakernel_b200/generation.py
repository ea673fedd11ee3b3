"""HF-style ``generate`` adapter and a latency report for the megakernel model.

The reference drives its models through NxDI's ``HuggingFaceGenerationAdapter``
(main.py:242, :285, :311): ``generate(input_ids, attention_mask,
max_new_tokens, min_new_tokens, do_sample, return_dict_in_generate,
output_scores, generation_config)``, with prompts padded to a rectangle and
the mask marking real tokens, and it reports end-to-end latencies
(``generate_report``, main.py:250-255; NxDI's benchmark module is not in the
reference sources). This module gives ``MegakernelLlamaForCausalLM`` the
same entry point:

* each row's real tokens (mask 1) are prefilled on the GPU (``prefill.py``;
  rows may differ in length), then all rows decode together, one persistent
  kernel launch per token, with the argmax (or ``mk_sample``'s draw) fed
  back on the device;
* ``output_scores`` returns each step's fp32 logits [B, V];
* ``eos_token_id`` ends a row: later tokens become ``pad_token_id``. Unlike
  HF, ``min_new_tokens`` does not forbid eos in the logits; a row simply does
  not end before it.

``generate_report`` summarises a list of end-to-end latencies the way the
reference's benchmark report does (percentiles in ms and tokens/s).
"""
from __future__ import annotations

import statistics
from dataclasses import dataclass

import torch


@dataclass
class GenerateOutput:
    sequences: torch.Tensor                      # [B, prompt columns + new tokens]
    scores: tuple[torch.Tensor, ...] | None = None  # per step [B, V] fp32


def _knob(value, config, name, default):
    if value is not None:
        return value
    got = getattr(config, name, None) if config is not None else None
    return default if got is None else got


class HuggingFaceGenerationAdapter:
    """``generate`` in the shape of HF / NxDI's adapter around a
    ``MegakernelLlamaForCausalLM`` (single GPU)."""

    def __init__(self, model):
        self.model = model

    @torch.no_grad()
    def generate(self, input_ids, attention_mask=None, max_new_tokens=None, min_new_tokens=None,
                 do_sample=None, top_k=None, top_p=None, temperature=None, eos_token_id=None,
                 pad_token_id=None, return_dict_in_generate=False, output_scores=False,
                 generation_config=None, seed: int = 0, **unused):
        gc = generation_config
        n_new = int(_knob(max_new_tokens, gc, "max_new_tokens", 20))
        min_new = int(_knob(min_new_tokens, gc, "min_new_tokens", 0))
        sample = bool(_knob(do_sample, gc, "do_sample", False))
        knobs = dict(top_k=int(_knob(top_k, gc, "top_k", 50 if sample else 1)),
                     top_p=float(_knob(top_p, gc, "top_p", 1.0)),
                     temperature=float(_knob(temperature, gc, "temperature", 1.0)), seed=seed)
        eos = _knob(eos_token_id, gc, "eos_token_id", None)
        eos = set(eos if isinstance(eos, (list, tuple)) else ([] if eos is None else [eos]))
        pad = _knob(pad_token_id, gc, "pad_token_id", None)
        pad = 0 if pad is None else int(pad)

        m = self.model
        ids = torch.as_tensor(input_ids)
        if ids.dim() == 1:
            ids = ids[None, :]
        B = ids.shape[0]
        mask = torch.ones_like(ids) if attention_mask is None else torch.as_tensor(attention_mask)
        rows = [ids[b][mask[b].bool()] for b in range(B)]
        kv = m.new_cache()
        first = m.prefill(rows, past_key_values=kv)
        lengths = [r.numel() for r in rows]
        for b in range(B):
            kv.reserve(b, lengths[b] + n_new)
        dev = m.device
        tok = torch.empty(B, dtype=torch.int32, device=dev)
        pos = torch.tensor(lengths, dtype=torch.int32, device=dev)
        nxt = torch.empty(B, dtype=torch.int32, device=dev)
        logits = torch.empty(B, m.lm_rows, dtype=torch.float32, device=dev)
        scores = [first.logits.to(dev)] if output_scores else None
        if sample:
            m.sample(first.logits.to(dev).contiguous(), step=0, out=tok, **knobs)
        else:
            tok.copy_(first.next_ids.to(torch.int32))
        new = torch.empty(B, n_new, dtype=torch.int32, device=dev)
        new[:, 0] = tok
        want_logits = sample or output_scores
        for s in range(1, n_new):
            m.launch(tok, pos, kv, logits if want_logits else None, nxt, feedback=not sample)
            if sample:
                m.sample(logits, step=s, tokens=tok, positions=pos, out=nxt, **knobs)
            if output_scores:
                scores.append(logits.clone())
            new[:, s] = tok
        m.sync()
        new = new.to(torch.int64).cpu()
        if eos:
            for b in range(B):
                row = new[b].tolist()
                for j in range(max(min_new, 1) - 1, n_new):
                    if row[j] in eos:
                        new[b, j + 1:] = pad
                        break
        seqs = torch.cat([ids.to(torch.int64).cpu(), new], dim=1)
        if return_dict_in_generate:
            return GenerateOutput(seqs, tuple(scores) if scores is not None else None)
        return seqs


def generate_report(latencies_ms, max_length: int, max_batch_size: int, n_runs: int | None = None) -> dict:
    """Latency percentiles (ms) and throughput (tokens/s: batch x max_length
    tokens per run over the mean run latency) of end-to-end runs."""
    lat = sorted(float(x) for x in latencies_ms)
    if not lat:
        raise ValueError("no latencies")

    def pct(q):
        return lat[min(len(lat) - 1, int(round(q / 100.0 * (len(lat) - 1))))]

    avg = statistics.fmean(lat)
    return {
        "latency_ms_p50": pct(50), "latency_ms_p90": pct(90), "latency_ms_p95": pct(95),
        "latency_ms_p99": pct(99), "latency_ms_p100": lat[-1], "latency_ms_avg": avg,
        "throughput": max_batch_size * max_length / (avg / 1e3),
        "n_runs": len(lat) if n_runs is None else n_runs,
    }
