"""Summaries of the kernel's phase trace (``MegakernelLlamaForCausalLM.set_trace``).

The trace holds, per CTA and per phase, globaltimer stamps (ns) of the
consumers reaching the phase's grid wait, passing it, having the activation
rows loaded and finishing the phase, plus cumulative stall totals of the
consumer warps (waiting for streamed weights) and of the producer lane
(waiting for a free ring slot). ``phase_table`` turns one launch's trace into
per-phase-type figures, averaged over the decoder layers.
"""
from __future__ import annotations

import numpy as np

PHASES = ("qkv", "attn", "o", "gu", "down")
WAIT_START, WAIT_DONE, ROWS, DONE, CONS_STALL, PROD_START, PROD_STALL, PROD_END = range(8)
ATTN_Q, ATTN_CHUNKS, ATTN_ARRIVE, ATTN_MERGED = range(8, 12)


def phase_table(trace, num_layers: int, skip_first_layer: bool = True) -> dict:
    """Per phase type: microseconds of the critical path split into
    barrier (last arrival -> first release), activation load, consumption
    (median and slowest CTA), and the stall totals accumulated in the phase.

    ``trace``: [grid, num_layers * 5 + 1, 12] int64 (one launch)."""
    t = np.asarray(trace, dtype=np.int64).astype(np.float64)
    n_ph = num_layers * 5 + 1
    assert t.shape[1] == n_ph, t.shape
    t0 = t[:, 0, WAIT_START].min()
    done_max = t[:, :, DONE].max(axis=0)
    out = {}
    names = [f"{l}.{PHASES[k]}" for l in range(num_layers) for k in range(5)] + ["lm"]
    rows = []
    for ph in range(n_ph):
        prev_done = done_max[ph - 1] if ph > 0 else t0
        cons_prev = t[:, ph - 1, CONS_STALL] if ph > 0 else 0.0
        prod_prev = t[:, ph - 1, PROD_STALL] if ph > 0 else 0.0
        rel = t[:, ph, WAIT_DONE].min() - prev_done
        load = np.median(t[:, ph, ROWS] - t[:, ph, WAIT_DONE]) if PHASES[ph % 5] != "attn" or ph == n_ph - 1 else 0.0
        start = np.where(t[:, ph, ROWS] > 0, t[:, ph, ROWS], t[:, ph, WAIT_DONE])
        cons = t[:, ph, DONE] - start
        rows.append({
            "phase": names[ph],
            "span_us": (done_max[ph] - prev_done) / 1e3,
            "barrier_us": rel / 1e3,
            "load_us": load / 1e3,
            "consume_med_us": float(np.median(cons)) / 1e3,
            "consume_max_us": float(cons.max()) / 1e3,
            "cons_stall_us": float(np.median(t[:, ph, CONS_STALL] - cons_prev)) / 1e3,
            "prod_stall_us": float(np.median(t[:, ph, PROD_STALL] - prod_prev)) / 1e3,
            "prod_lead_us": float(np.median(t[:, ph, WAIT_DONE] - t[:, ph, PROD_START])) / 1e3,
        })
    out["rows"] = rows
    out["total_us"] = (done_max[-1] - t0) / 1e3
    first = 1 if skip_first_layer and num_layers > 1 else 0
    agg = {}
    for k, name in enumerate(PHASES):
        sel = [rows[l * 5 + k] for l in range(first, num_layers)]
        agg[name] = {key: float(np.mean([r[key] for r in sel])) for key in sel[0] if key != "phase"}
    agg["lm"] = {key: rows[-1][key] for key in rows[-1] if key != "phase"}
    out["by_type"] = agg
    return out


def format_table(summary: dict) -> str:
    keys = ("span_us", "barrier_us", "load_us", "consume_med_us", "consume_max_us",
            "cons_stall_us", "prod_stall_us", "prod_lead_us")
    lines = ["phase  " + " ".join(f"{k:>15s}" for k in keys)]
    for name, r in summary["by_type"].items():
        lines.append(f"{name:6s} " + " ".join(f"{r[k]:15.2f}" for k in keys))
    lines.append(f"total {summary['total_us']:.1f} us")
    return "\n".join(lines)


def attention_breakdown(trace, num_layers: int) -> dict:
    """Attention sub-steps (us, mean over layers 1..L-1 of the median / max
    over the CTAs that had an item): q load, chunk reduction, the warp
    states' combine and publication, and split 0's merge of the splits."""
    t = np.asarray(trace, dtype=np.int64).astype(np.float64)
    keys = {"q_load": (WAIT_DONE, ATTN_Q), "chunks": (ATTN_Q, ATTN_CHUNKS),
            "arrive": (ATTN_CHUNKS, ATTN_ARRIVE), "merge": (ATTN_ARRIVE, ATTN_MERGED)}
    out = {k: [0.0, 0.0] for k in keys}
    n = 0
    for l in range(1, num_layers):
        ph = l * 5 + 1
        busy = t[:, ph, ATTN_Q] > 0
        if not busy.any():
            continue
        n += 1
        for k, (a, b) in keys.items():
            sel = busy & (t[:, ph, b] > 0)
            if not sel.any():
                continue
            d = (t[sel, ph, b] - t[sel, ph, a]) / 1e3
            out[k][0] += float(np.median(d))
            out[k][1] += float(d.max())
    return {k: (v[0] / max(n, 1), v[1] / max(n, 1)) for k, v in out.items()}
