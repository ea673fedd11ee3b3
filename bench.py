"""Benchmark: bs=1 Llama-3.2-1B greedy decode on B200 through the megakernel.

Headline workload (BASELINE.json's metric, "bs=1 decode tok/s & p50 token
latency at ctx 1024"): seeded random-init Llama-3.2-1B in bf16, a paged KV
cache pre-filled with 1024 seeded N(0,1) bf16 positions, a seeded random
token, then K back-to-back greedy decode steps from position 1024 (the cache
and RoPE table sized for 1024 + K + warm-up). One step = one launch of the
persistent kernel = all 16 layers + final norm + lm_head + argmax for one
token; the argmax feeds the next launch on the device (no host round trip).
``value`` = tokens/s over the K timed steps (CUDA events on the launching
stream), max over ranks; ``p50_ms`` / ``p90_ms`` / ``p99_ms`` per step.

``e2e`` runs the same steps, from position 1024 on a cache filled the same
way, through the public API (``MegakernelLlamaForCausalLM.forward`` with a
pinned host token and position: H2D copy, launch, D2H of the next id, host
sync per step).

``roofline``: algorithmic bytes per step (2,471,632,896 B of weights + 32,768 B
per cached position read + 32,768 B of K/V written, at the timed steps' mean
position) / average step time, against the measured HBM copy bandwidth in
MEASURED_PEAKS.json.

Extras: ``decode_640`` (a 128-token seeded prompt, then 640
greedy steps), ``ctx_sweep`` (config 3: one step at 128 / 1024 / 4096 / 8192
cached positions), ``batched`` (config 4: bs 8 / 32 / 64 at KV 1024).

``cpu_baseline`` and ``--impl reference``: the reference's PyTorch Llama path
(HF ``LlamaForCausalLM``, via oracle/) on the host CPU cores on BASELINE
config 1 exactly: one greedy step at position 1024 over the same 1024 cached
rows and the same token (the cache is cropped back to 1024 after every step),
timed over several steps; rank 0 only.

Multi-GPU (torchrun, N > 1): tensor-parallel decode
of the one sequence over the N GPUs (``TensorParallelLlamaForCausalLM``: q/kv
heads, MLP rows and lm_head rows sharded, partial sums exchanged inside the
kernel over NVLink); ``value`` = tokens/s of that sequence (strong scaling),
the step time being the max over ranks. ``--replicas`` runs N independent
single-GPU replicas instead (weak scaling, total tokens/s).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "bs=1 decode tok/s & p50 token latency at ctx 1024; % of 8 TB/s HBM roofline"
PROMPT_LEN = 128          # config 2's prompt
DECODE_STEPS = 640       # config 2's greedy steps
CTX = 1024               # the headline's context: cached positions before the first step
KV_SEED, TOKEN_SEED = 1024, 9
FALLBACK_HBM_GBS = 6650.0
WORKLOAD = ("Llama-3.2-1B bs=1 greedy decode at ctx 1024: 1024 cached N(0,1) bf16 positions "
            "(seeded), seeded random token, steps from position 1024")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--replicas", action="store_true",
                    help="N > 1: independent replicas instead of tensor parallelism")
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--no-sweep", action="store_true", help="skip the ctx sweep extra")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true", help="skip the bs 8/32/64 extra")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--small", action="store_true",
                    help="profiling case: a few steps, no e2e / sweep / cpu baseline")
    ap.add_argument("--case", choices=["small4", "gemm", "batched", "trace", "attn"], default=None,
                    help="ncu profiling cases (print timings, no JSON line): small4 - 4 "
                         "Llama-3.2-1B layers, vocab 32000, one step at ctx 512 after 4 warm-up "
                         "steps; gemm - the tcgen05 GEMM on the batched projection shapes at 8 "
                         "and 64 rows (3 warm-up + 7 timed launches each, L2 flushed, cuBLAS "
                         "beside it); batched - one bs-64 batched step at KV 1024 replayed "
                         "inside the NVTX range 'replay'; trace - the per-phase trace of "
                         "Llama-3.2-1B steps at ctx 1024 (mk_set_trace, summarised by trace.py); "
                         "attn - the batched paged attention alone, bs 64 x 4096 cached positions "
                         "of one layer (536 MB of K/V), 3 warm-up and 5 timed launches")
    return ap.parse_args()


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t)
    return float(t.item())


def traffic_summary():
    p = ROOT / "profiles" / "decode_kernel_traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get("dram_bytes_per_launch")
    return None


# ----------------------------------------------------------------------------
# CPU: the reference's PyTorch path (HF Llama) on the host cores
# ----------------------------------------------------------------------------

def cpu_model_name() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_config1(weights_cpu, seconds: float, min_steps: int = 5, max_steps: int | None = None,
                warmup: int = 1):
    """BASELINE config 1 on the host CPU: HF LlamaForCausalLM (the reference's
    PyTorch Llama path) in bf16, one greedy decode step at position 1024 over
    1024 cached N(0,1) positions (the GPU arm's cache rows and token). The
    cache is cropped back to 1024 positions after every step, so every timed
    step is that same step. Runs ``warmup`` untimed steps, then timed steps
    until ``seconds`` have passed (at least ``min_steps``, at most
    ``max_steps``). Returns (tok/s, detail)."""
    from transformers import DynamicCache

    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg
    from oracle import llama_oracle as O

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    model = O.hf_model(cfg, weights_cpu)
    k, v = syn.random_kv_rows(cfg, CTX, seed=KV_SEED)
    cache = DynamicCache(config=model.config)
    for l in range(cfg.num_layers):
        cache.update(k[l:l + 1].clone(), v[l:l + 1].clone(), l)
    tok = int(syn.random_tokens(1, cfg.vocab, seed=TOKEN_SEED)[0])
    ids, pos = torch.tensor([[tok]]), torch.tensor([[CTX]])
    times, nxt = [], None
    with torch.no_grad():
        for _ in range(warmup):
            model(input_ids=ids, position_ids=pos, past_key_values=cache, use_cache=True)
            cache.crop(CTX)
        t_end = time.perf_counter() + seconds
        while (time.perf_counter() < t_end or len(times) < min_steps) and \
                (max_steps is None or len(times) < max_steps):
            t0 = time.perf_counter()
            out = model(input_ids=ids, position_ids=pos, past_key_values=cache, use_cache=True)
            nxt = int(out.logits[0, -1].argmax())
            times.append(time.perf_counter() - t0)
            cache.crop(CTX)
    tps = len(times) / sum(times)
    return tps, {"cores": threads, "cpu_model": cpu_model_name(), "steps": len(times),
                 "p50_ms": statistics.median(times) * 1e3, "next_id": nxt}


def run_reference(args, ws, rank):
    if rank != 0:
        return
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg

    w = syn.make_weights(cfg, seed=0, device="cuda" if torch.cuda.is_available() else "cpu")
    w = {k: t.cpu() for k, t in w.items()}
    K, W = args.steps, args.warmup
    tps, det = cpu_config1(w, seconds=0.0, min_steps=K, max_steps=K, warmup=W)
    sample = (f"HF LlamaForCausalLM (the reference's PyTorch Llama path) bf16 on CPU: BASELINE "
              f"config 1, one greedy step at position {CTX} over {CTX} cached N(0,1) positions, "
              f"{det['steps']} timed steps after {W} warm-up, {det['cores']} threads, "
              f"{det['cpu_model']}")
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": det["steps"], "warmup": W,
        "ms_per_step": 1e3 / tps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random-init weights)",
        "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": CTX,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": det["cores"], "kind": "port",
                         "sample": sample},
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "p50_ms": det["p50_ms"],
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU: the megakernel
# ----------------------------------------------------------------------------

def _kv_rows_for(model, cfg, n, seed, dev):
    """N(0,1) rows of the whole model's cache, this rank's kv heads only."""
    from llama1b_megakernel_b200 import synthetic as syn

    k, v = syn.random_kv_rows(cfg, n, seed=seed, device=dev)
    nkv = model.cfg.num_kv_heads
    r = getattr(model, "tp_rank", 0)
    return k[:, r * nkv:(r + 1) * nkv].contiguous(), v[:, r * nkv:(r + 1) * nkv].contiguous()


def _timed_steps(model, kv, tok, pos, nxt, first_tok, first_pos, K, W, ws):
    """W untimed and K timed greedy steps from (first_tok, first_pos), the
    argmax fed back on the device. Returns per-step ms and the total ms
    (max over ranks)."""
    def reset():
        tok.fill_(first_tok)
        pos.fill_(first_pos)

    reset()
    for _ in range(W):
        model.launch(tok, pos, kv, None, nxt, feedback=True)
    model.sync()
    reset()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    barrier(ws)
    torch.cuda.synchronize()
    for i in range(K):
        starts[i].record()
        model.launch(tok, pos, kv, None, nxt, feedback=True)
        ends[i].record()
    torch.cuda.synchronize()
    barrier(ws)
    model.sync()
    step_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
    return step_ms, max_over_ranks(starts[0].elapsed_time(ends[-1]), ws)


def run_ours(args, ws, rank, local):
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    hbm_peak, peak_kind = peaks()
    tp_world = ws if (ws > 1 and not args.replicas) else 1
    sweep = not (args.no_sweep or args.small) and tp_world == 1
    K, W = args.steps, args.warmup
    head_len = CTX + K + W + 2
    # (the batched extras run KV length 1024 in caches of 1024 + 64 positions)
    max_seq = max(8192 + 64 if sweep else 0, head_len, PROMPT_LEN + DECODE_STEPS + 2, CTX + 64)
    w = syn.make_weights(cfg, seed=0, device=dev)
    if tp_world > 1:
        from llama1b_megakernel_b200.tp import TensorParallelLlamaForCausalLM

        model = TensorParallelLlamaForCausalLM(cfg, w, max_batch=1, max_seq_len=max_seq,
                                               page_size=64, device=dev)
    else:
        model = MegakernelLlamaForCausalLM(cfg, w, max_batch=1, max_seq_len=max_seq,
                                           page_size=64, device=dev)
    w_cpu = None
    if rank == 0 and ws == 1 and not (args.no_cpu_baseline or args.small):
        w_cpu = {k: t.cpu() for k, t in w.items()}
    del w
    torch.cuda.empty_cache()

    tok = torch.empty(1, dtype=torch.int32, device=dev)
    pos = torch.empty(1, dtype=torch.int32, device=dev)
    nxt = torch.empty(1, dtype=torch.int32, device=dev)
    first_tok = int(syn.random_tokens(1, cfg.vocab, seed=TOKEN_SEED)[0])

    # ------------------------------------------------------------ headline: ctx 1024
    kv = model.kv
    k, v = _kv_rows_for(model, cfg, CTX, KV_SEED, dev)
    kv.fill(0, k, v)
    kv.reserve(0, head_len)
    del k, v
    clocks = ClockSampler(local)
    clocks.start()
    step_ms, total_ms = _timed_steps(model, kv, tok, pos, nxt, first_tok, CTX, K, W, ws)
    clk = clocks.stop()
    seqs = ws // tp_world  # sequences decoded by the whole job
    value = K * seqs / (total_ms / 1e3)
    srt = sorted(step_ms)
    p50 = statistics.median(step_ms)
    p90 = srt[int(0.9 * (K - 1))]
    p99 = srt[int(0.99 * (K - 1))]
    kernel_ms = statistics.mean(step_ms)
    ctx_mean = CTX + (K - 1) / 2.0
    # per GPU: a tensor-parallel rank streams 1/tp_world of the weights and KV
    bytes_step = (cfg.weight_bytes_per_token() + cfg.kv_bytes_per_position() * ctx_mean +
                  cfg.kv_bytes_per_position()) / tp_world
    achieved = bytes_step / (kernel_ms / 1e3) / 1e9

    # ------------------------------------------------------------ e2e (public API), ctx 1024
    e2e_val = None
    h2d = d2h = 0
    if not args.small:
        n = K
        kv2 = model.new_cache(max_seq_len=max_seq)
        k, v = _kv_rows_for(model, cfg, CTX, KV_SEED, dev)
        kv2.fill(0, k, v)
        kv2.reserve(0, CTX + n + 4)
        del k, v
        ids = torch.empty(1, 1, dtype=torch.int32).pin_memory()
        ps = torch.empty(1, 1, dtype=torch.int32).pin_memory()
        for i in range(3):  # warm-up on the same cache positions
            ids[0, 0] = first_tok
            ps[0, 0] = CTX + i
            model.forward(ids, ps, past_key_values=kv2, return_logits=False)
        ids[0, 0] = first_tok
        barrier(ws)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(n):
            ps[0, 0] = CTX + i
            o = model.forward(ids, ps, past_key_values=kv2, return_logits=False)
            ids[0, 0] = int(o.next_ids[0])  # D2H of the result, host feeds it back
        t1 = time.perf_counter()
        e2e_val = n * seqs / max_over_ranks(t1 - t0, ws)
        h2d = 2 * 4   # token id + position (int32) per step
        d2h = 4       # next id (int32) per step
        del kv2

    # ------------------------------------------------------------ config 2: prompt + 640 steps
    dec640 = None
    if not args.small:
        kv4 = model.new_cache(max_seq_len=max_seq)
        prompt = syn.random_tokens(PROMPT_LEN, cfg.vocab, seed=1).reshape(1, -1)
        out = model.forward(prompt, past_key_values=kv4, return_logits=False)
        kv4.reserve(0, PROMPT_LEN + DECODE_STEPS + 1)
        ms640, tot640 = _timed_steps(model, kv4, tok, pos, nxt, int(out.next_ids[0]), PROMPT_LEN,
                                     DECODE_STEPS, 3, ws)
        dec640 = {"workload": f"{PROMPT_LEN}-token seeded prompt (decode kernel per position), "
                              f"then {DECODE_STEPS} greedy steps from position {PROMPT_LEN}",
                  "tok_s": DECODE_STEPS * seqs / (tot640 / 1e3),
                  "ms_p50": statistics.median(ms640),
                  "ms_p99": sorted(ms640)[int(0.99 * (DECODE_STEPS - 1))]}
        del kv4

    # ------------------------------------------------------------ ctx sweep
    sweep_res = None
    if sweep:
        sweep_res = {}
        for L in (128, 1024, 4096, 8192):
            kv3 = model.new_cache(max_seq_len=max_seq, num_pages=kv.num_pages)
            k, v = syn.random_kv_rows(cfg, L, seed=L, device=dev)
            kv3.fill(0, k, v)
            kv3.reserve(0, L + 1)
            del k, v
            t_ = torch.tensor([7], dtype=torch.int32, device=dev)
            p_ = torch.tensor([L], dtype=torch.int32, device=dev)
            for _ in range(3):
                model.launch(t_, p_, kv3, None, nxt)
            model.sync()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(21)]
            ev[0].record()
            for j in range(20):
                model.launch(t_, p_, kv3, None, nxt)
                ev[j + 1].record()
            torch.cuda.synchronize()
            model.sync()
            ms = [ev[j].elapsed_time(ev[j + 1]) for j in range(20)]
            med = statistics.median(ms)
            b = cfg.weight_bytes_per_token() + cfg.kv_bytes_per_position() * (L + 1)
            sweep_res[str(L)] = {"ms_p50": med, "tok_s": 1e3 / med,
                                 "achieved_gbs": b / (med / 1e3) / 1e9,
                                 "frac_of_peak": b / (med / 1e3) / 1e9 / hbm_peak}
            del kv3
            torch.cuda.empty_cache()

    # ------------------------------------------------------------ batched (config 4)
    batched_res = None
    if sweep and not args.no_batched:
        batched_res = run_batched(model, cfg, dev, hbm_peak)
    tp_bs32 = None
    if tp_world > 1 and not (args.no_batched or args.small):
        # an extra: a failure is reported in the line rather than losing the headline (the
        # same code runs on every rank, so a failure is expected on all of them alike)
        try:
            tp_bs32 = run_tp_batched(model, cfg, dev, ws)
        except Exception as e:  # noqa: BLE001
            tp_bs32 = {"error": f"{type(e).__name__}: {e}"[:300]}
            torch.cuda.empty_cache()

    # ------------------------------------------------------------ cpu baseline (config 1)
    cpu_b = None
    if w_cpu is not None:
        del model
        torch.cuda.empty_cache()
        tps, det = cpu_config1(w_cpu, args.cpu_seconds)
        cpu_b = {"value": tps, "unit": "tok/s", "cores": det["cores"], "kind": "port",
                 "p50_ms": det["p50_ms"],
                 "sample": (f"HF LlamaForCausalLM (the reference's PyTorch Llama path, via "
                            f"oracle/) bf16, BASELINE config 1: one greedy step at position "
                            f"{CTX} over the same {CTX} cached rows and token, {det['steps']} "
                            f"timed steps, on {det['cpu_model']}")}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": K,
            "warmup": W, "ms_per_step": total_ms / K, "higher_is_better": True,
            "scaling": "strong" if tp_world > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random-init weights, seeded N(0,1) KV cache and token)",
            "config": {"workload": WORKLOAD, "global_batch": seqs, "seq_len": CTX,
                       "parallelism": f"tp{tp_world}" if tp_world > 1 else f"replicas x{ws}",
                       "first_position": CTX, "last_position": CTX + K - 1,
                       "l2": "inputs larger than L2 (2.47 GB of weights streamed per step)"},
            "p50_ms": p50, "p90_ms": p90, "p99_ms": p99,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak,
                         "unit": "GB/s", "frac": achieved / hbm_peak,
                         "peak_kind": peak_kind,
                         "traffic": traffic_summary() if tp_world == 1 else None,
                         "bytes_per_step": bytes_step},
            "frac_of_8tbs": achieved / 8000.0,
            "clocks": clk,
            "gpu_launches": K,
            "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
        }
        if dec640 is not None:
            line["decode_640"] = dec640
        if sweep_res is not None:
            line["ctx_sweep"] = sweep_res
        if batched_res is not None:
            line["batched"] = batched_res
        if tp_bs32 is not None:
            line["tp_bs32"] = tp_bs32
        if cpu_b is not None:
            line["cpu_baseline"] = cpu_b
        print(json.dumps(line), flush=True)


def run_batched(model, cfg, dev, hbm_peak):
    """bs 8, 32, 64, one greedy step at KV length 1024 per
    sequence (independent seeded N(0,1) caches, random tokens), through the
    batched path (batched.py: paged attention kernel + tcgen05 projections, one
    CUDA graph per batch size). Step time = median of 20 graph replays."""
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.batched import BatchedDecoder

    L, BMAX = 1024, 64
    dec = BatchedDecoder(model, max_batch=BMAX, max_seq_len=L + 64, page_size=64)
    for b in range(BMAX):
        k, v = syn.random_kv_rows(cfg, L, seed=100 + b, seq=b, device=dev)
        dec.kv.fill(b, k, v)
        del k, v
    res = {}
    for B in (8, 32, 64):
        toks = syn.random_tokens(B, cfg.vocab, seed=B)
        dec.step(toks, torch.full((B,), L, dtype=torch.int32))
        for _ in range(3):
            dec.replay(B)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(21)]
        ev[0].record()
        for j in range(20):
            dec.replay(B)
            ev[j + 1].record()
        torch.cuda.synchronize()
        dec.check()
        med = statistics.median(ev[j].elapsed_time(ev[j + 1]) for j in range(20))
        byts = cfg.weight_bytes_per_token() + B * cfg.kv_bytes_per_position() * (L + 1)
        res[str(B)] = {"ms_p50": med, "tok_s": B * 1e3 / med, "bytes_per_step": byts,
                       "achieved_gbs": byts / (med / 1e3) / 1e9,
                       "frac_of_peak": byts / (med / 1e3) / 1e9 / hbm_peak,
                       "gemm": "mk_gemm_bf16 (tcgen05)", "attention": "mk_paged_attention"}
    del dec
    torch.cuda.empty_cache()
    return res


def run_tp_batched(model, cfg, dev, ws, B: int = 32, L: int = 1024):
    """BASELINE config 5 at bs 32: the batched step on every rank of the
    tensor-parallel group (BatchedDecoder on the TP model: shard GEMMs, NCCL
    all-reduce of the o_proj / down partial sums inside the graph), KV length
    1024 per sequence. Step time = median of 20 graph replays, max over ranks."""
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.batched import BatchedDecoder

    dec = BatchedDecoder(model, max_batch=B, max_seq_len=L + 64, page_size=64)
    try:
        nkv = model.cfg.num_kv_heads
        g0 = model.tp_rank * nkv
        for b in range(B):
            k, v = syn.random_kv_rows(cfg, L, seed=100 + b, seq=b, device=dev)
            dec.kv.fill(b, k[:, g0:g0 + nkv], v[:, g0:g0 + nkv])
            del k, v
        dec.step(syn.random_tokens(B, cfg.vocab, seed=B), torch.full((B,), L, dtype=torch.int32))
        for _ in range(3):
            dec.replay(B)
        torch.cuda.synchronize()
        barrier(ws)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(21)]
        ev[0].record()
        for j in range(20):
            dec.replay(B)
            ev[j + 1].record()
        torch.cuda.synchronize()
        dec.check()
        med = max_over_ranks(statistics.median(ev[j].elapsed_time(ev[j + 1]) for j in range(20)), ws)
    finally:
        dec.close()  # its graphs hold NCCL calls: released before the group is destroyed
    del dec
    torch.cuda.empty_cache()
    return {"batch": B, "kv_len": L, "ms_p50": med, "tok_s": B * 1e3 / med,
            "gemm": "mk_gemm_bf16 (tcgen05) on each rank's shard",
            "collective": "fp32 partial sums read from peer memory over NVLink and summed in rank "
                          "order inside the add+RMSNorm kernel (mk_allreduce_add_rmsnorm), x 2 per "
                          "layer; NCCL all-gather of the argmax keys once per step"}


def run_case_gemm():
    """The tcgen05 GEMM (mk_gemm_bf16) alone on the batched decode shapes."""
    import ctypes  # noqa: F401

    from llama1b_megakernel_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    flush = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for rows, bp in ((8, 16), (64, 64)):
        for n, k in ((3072, 2048), (2048, 2048), (16384, 2048), (2048, 8192), (128256, 2048)):
            w = (torch.randn(n, k, device=dev) * 0.02).bfloat16()
            x = torch.zeros(bp, k, dtype=torch.bfloat16, device=dev)
            x[:rows] = torch.randn(rows, k, device=dev).bfloat16()
            out = torch.empty(rows, n, dtype=torch.bfloat16, device=dev)
            ws = lib.mk_gemm_workspace(n, k, rows)
            work = torch.zeros(max(ws, 16), dtype=torch.uint8, device=dev)

            def run():
                _lib.check(lib.mk_gemm_bf16(w.data_ptr(), n, k, x.data_ptr(), rows, bp, None,
                                            out.data_ptr(), None, work.data_ptr(), work.numel(),
                                            err.data_ptr(), torch.cuda.current_stream().cuda_stream))

            for _ in range(3):
                run()
            ts, tc = [], []
            for _ in range(7):
                for fn, acc in ((run, ts), (lambda: torch.nn.functional.linear(x[:rows], w), tc)):
                    flush.zero_()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    fn()
                    e1.record()
                    torch.cuda.synchronize()
                    acc.append(e0.elapsed_time(e1))
            t, tcb = statistics.median(ts), statistics.median(tc)
            print(f"rows {rows:3d} n {n:6d} k {k:5d}: mk_gemm_bf16 {t * 1e3:7.1f} us "
                  f"({n * k * 2 / t / 1e6:5.0f} GB/s), cuBLAS {tcb * 1e3:7.1f} us  err {int(err)}")
            del w


def run_case_attn():
    """mk_paged_attention alone on one layer of the bs-64 batched step, at 4096
    cached positions per sequence (K/V 536 MB, larger than L2), page size 64:
    the TMA kernel. Prints the median launch time and the K/V bytes per second."""
    import ctypes

    from llama1b_megakernel_b200 import _lib

    lib = _lib.load()
    dev = torch.device("cuda", 0)
    B, NKV, NQ, L, PS = 64, 8, 32, 4096, 64
    blocks = L // PS + 1
    pages = B * blocks
    k = (torch.randn(pages, NKV, PS, 64, device=dev) * 0.5).bfloat16()
    v = torch.randn(pages, NKV, PS, 64, device=dev).bfloat16()
    table = torch.randperm(pages, device=dev, dtype=torch.int32).reshape(B, blocks).contiguous()
    lengths = torch.full((B,), L, dtype=torch.int32, device=dev)
    q = torch.randn(B, NQ, 64, device=dev).bfloat16()
    out = torch.empty(B, NQ, 64, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = lib.mk_paged_attention_workspace(B, NKV, L)
    work = torch.empty(max(ws, 16), dtype=torch.uint8, device=dev)

    def run():
        _lib.check(lib.mk_paged_attention(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), table.data_ptr(), lengths.data_ptr(), B, NQ,
            NKV, PS, blocks, pages, L, ctypes.c_float(0.125), work.data_ptr(), work.numel(),
            out.data_ptr(), err.data_ptr(), torch.cuda.current_stream().cuda_stream))

    for _ in range(3):
        run()
    ts = []
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    t = statistics.median(ts)
    kv_bytes = B * NKV * L * 64 * 2 * 2
    print(f"paged attention bs {B} x {L} positions: {t * 1e3:.1f} us, "
          f"{kv_bytes / t / 1e6:.0f} GB/s of K/V, error word {int(err)}")


def run_case_batched():
    """One bs-64 batched step at KV 1024, replayed once inside NVTX 'replay'."""
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.batched import BatchedDecoder
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    dev = torch.device("cuda", 0)
    B, L = 64, 1024
    w = syn.make_weights(cfg, seed=0, device=dev)
    m = MegakernelLlamaForCausalLM(cfg, w, max_batch=1, max_seq_len=L + 64, device=dev)
    del w
    dec = BatchedDecoder(m, max_batch=B, max_seq_len=L + 64, page_size=64)
    for b in range(B):
        k, v = syn.random_kv_rows(cfg, L, seed=100 + b, seq=b, device=dev)
        dec.kv.fill(b, k, v)
    dec.step(syn.random_tokens(B, cfg.vocab, seed=B), torch.full((B,), L, dtype=torch.int32))
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("replay")
    dec.replay(B)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    dec.check()
    print("batched case done")


def run_case_small4():
    """The ncu case: Llama-3.2-1B-shaped layers, small enough to replay (~0.7 GB)."""
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    cfg = LLAMA_3_2_1B.replace(num_layers=4, vocab=32000)
    dev = torch.device("cuda", 0)
    w = syn.make_weights(cfg, seed=0, device=dev)
    m = MegakernelLlamaForCausalLM(cfg, w, max_batch=1, max_seq_len=1024, page_size=64, device=dev)
    del w
    k, v = syn.random_kv_rows(cfg, 512, seed=5, device=dev)
    m.kv.fill(0, k, v)
    m.kv.reserve(0, 1024)
    del k, v
    tok = torch.tensor([7], dtype=torch.int32, device=dev)
    pos = torch.tensor([512], dtype=torch.int32, device=dev)
    nxt = torch.empty(1, dtype=torch.int32, device=dev)
    for _ in range(4):
        m.launch(tok, pos, m.kv, None, nxt)
    m.sync()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    m.launch(tok, pos, m.kv, None, nxt)
    ev[1].record()
    torch.cuda.synchronize()
    m.sync()
    print(f"small4 step {ev[0].elapsed_time(ev[1]):.4f} ms")


def run_case_trace():
    """Per-phase trace of the headline workload: Llama-3.2-1B, 1024 cached
    N(0,1) positions, steps from position 1024; prints the phase table and
    the attention breakdown of the median of 5 traced steps (by total)."""
    from llama1b_megakernel_b200 import synthetic as syn
    from llama1b_megakernel_b200 import trace as tr
    from llama1b_megakernel_b200.config import LLAMA_3_2_1B as cfg
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    dev = torch.device("cuda", 0)
    w = syn.make_weights(cfg, seed=0, device=dev)
    m = MegakernelLlamaForCausalLM(cfg, w, max_batch=1, max_seq_len=CTX + 64, page_size=64,
                                   device=dev)
    del w
    k, v = syn.random_kv_rows(cfg, CTX, seed=KV_SEED, device=dev)
    m.kv.fill(0, k, v)
    m.kv.reserve(0, CTX + 16)
    del k, v
    tok = torch.tensor([int(syn.random_tokens(1, cfg.vocab, seed=TOKEN_SEED)[0])],
                       dtype=torch.int32, device=dev)
    pos = torch.tensor([CTX], dtype=torch.int32, device=dev)
    nxt = torch.empty(1, dtype=torch.int32, device=dev)
    for _ in range(4):
        m.launch(tok, pos, m.kv, None, nxt)
    m.sync()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    ev[0].record()
    for j in range(5):
        m.launch(tok, pos, m.kv, None, nxt)
        ev[j + 1].record()
    torch.cuda.synchronize()
    m.sync()
    plain = [ev[j].elapsed_time(ev[j + 1]) for j in range(5)]
    buf = m.set_trace(True)
    runs = []
    for _ in range(5):
        m.launch(tok, pos, m.kv, None, nxt)
        m.sync()
        runs.append(tr.phase_table(buf.cpu().numpy(), cfg.num_layers))
        runs[-1]["_attn"] = tr.attention_breakdown(buf.cpu().numpy(), cfg.num_layers)
    m.set_trace(False)
    runs.sort(key=lambda r: r["total_us"])
    med = runs[len(runs) // 2]
    print(f"untraced step at ctx {CTX}: {statistics.median(plain) * 1e3:.1f} us (median of 5)")
    print(tr.format_table(med))
    print("attention sub-steps (median / max over CTAs, us): " +
          ", ".join(f"{k} {a:.2f}/{b:.2f}" for k, (a, b) in med["_attn"].items()))


def main():
    args = parse()
    if args.case == "trace":
        run_case_trace()
        return
    if args.case == "small4":
        run_case_small4()
        return
    if args.case == "gemm":
        run_case_gemm()
        return
    if args.case == "batched":
        run_case_batched()
        return
    if args.case == "attn":
        run_case_attn()
        return
    ws, rank, local = dist_init()
    try:
        if args.impl == "reference":
            run_reference(args, ws, rank)
        else:
            run_ours(args, ws, rank, local)
    finally:
        if ws > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
