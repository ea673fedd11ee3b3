"""GPU parity: the megakernel (through the C ABI) against the CPU oracle.

Acceptance bar: K/V rows land at bit-exact positions and nothing else in the
cache changes; per-step fp32 logits reach cosine >= 0.999 and max |diff| <=
3e-2 against the oracle (the reference's PyTorch path restated on CPU);
greedy ids match.

Full-size Llama-3.2-1B with random-init weights is the exception to the
max-abs bar, and the tests show why with a second, independent bf16
implementation: HF ``LlamaForCausalLM`` itself run in bf16 on the GPU
(cuBLAS GEMMs, SDPA attention; test infrastructure, never the product).
Its distance from the CPU reference is the spread that rounding order alone
produces, and the kernel must be no farther from the reference than it
(``SECOND_SLACK``), nor agree less often on greedy tokens. Further: in bf16 the reference's own path differs
from exact (fp32) arithmetic on the same weights and cache by about 0.14 in
max |logit| (16 layers of bf16 rounding on a residual that grows to |x| ~ 30
against N(0,1) cached values), so any implementation that rounds in another
order than PyTorch's CPU kernels lands about that far from the reference. For
the 1B cases the test therefore computes that fp32 evaluation ("truth") and
requires the kernel to be no farther from it than ``ENVELOPE`` times the
reference's own distance, with cosine >= 0.999 against both. The small
configs keep the plain 3e-2 bar.
"""
import json
from pathlib import Path

import pytest
import torch

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200.config import LLAMA_3_2_1B, MID, SMALL, TINY
from oracle import llama_oracle as O

pytestmark = pytest.mark.gpu

COS_MIN = 0.999      # per-step logits cosine similarity vs the oracle
MAXABS = 3e-2        # per-step logits max |diff| vs the oracle
KV_ROW_TOL = 0.0625  # new K/V row values: a few bf16 ulps at |x| ~ 1
ENVELOPE = 1.5       # 1B: kernel-to-fp32 distance <= ENVELOPE x reference-to-fp32
MARGIN_SURE = 0.1    # 1B greedy: top-2 margin above which fp32 arithmetic agrees 100%
DRIFT_MAX = 0.25     # 1B greedy: |kernel - reference| at the reference's top-1 logit
SECOND_SLACK = 1.25  # 1B: kernel max|logit - reference| <= this x the second implementation's
MATCH_SLACK = 0.01   # 1B greedy: kernel match rate >= second implementation's - this
GOLDEN = Path(__file__).resolve().parent / "golden"


def _model(cfg, w, B, max_seq_len, page_size, num_pages=None, shuffle=None):
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    m = MegakernelLlamaForCausalLM(cfg, w, max_batch=B, max_seq_len=max_seq_len,
                                   page_size=page_size, device="cuda:0")
    if shuffle is not None:
        m.kv.shuffle_free_pages(shuffle)
    return m


def _oracle_kv(model):
    return O.OracleKV(model.kv.k_pages.cpu().clone(), model.kv.v_pages.cpu().clone(),
                      model.kv.block_tables.cpu().clone())


def _fp32_copy(w):
    return {k: v.float() for k, v in w.items() if not k.startswith("_")}


def _check_logits(got, want, truth=None):
    """cos >= COS_MIN against the oracle; max-abs <= MAXABS against the oracle,
    or, when the fp32 evaluation ``truth`` is given, the envelope criterion."""
    got = got.float().cpu()
    cos = torch.nn.functional.cosine_similarity(got, want, dim=-1)
    err = (got - want).abs().max(dim=-1).values
    assert cos.min().item() >= COS_MIN, cos
    if truth is None:
        assert err.max().item() <= MAXABS, err
    else:
        d_ref = (want - truth).abs().max(dim=-1).values
        d_got = (got - truth).abs().max(dim=-1).values
        cos_t = torch.nn.functional.cosine_similarity(got, truth, dim=-1)
        print(f"max|ref-fp32| {d_ref.max().item():.4f}  max|kernel-fp32| {d_got.max().item():.4f}"
              f"  max|kernel-ref| {err.max().item():.4f}")
        assert cos_t.min().item() >= COS_MIN, cos_t
        assert (d_got <= ENVELOPE * d_ref + 1e-3).all(), (d_got, d_ref)
    return cos, err


def _hf_gpu_model(cfg, w):
    """HF LlamaForCausalLM in bf16 on cuda:0 (the second implementation)."""
    return O.hf_model(cfg, {k: v for k, v in w.items() if not k.startswith("_")}).to("cuda:0")


def _hf_gpu_logits(hf, w, hidden):
    """The oracle's logit head (fp32 product of the tied embedding and the bf16
    final-norm output) on HF's last hidden state [B, H]."""
    e = w.get("_embed_f32_cuda")
    if e is None:
        e = w["_embed_f32_cuda"] = w["model.embed_tokens.weight"].to("cuda:0").float()
    return hidden.float() @ e.t()


def _hf_gpu_cache(hf, cfg, k, v):
    from transformers import DynamicCache

    cache = DynamicCache(config=hf.config)
    for l in range(cfg.num_layers):
        cache.update(k[l:l + 1].to("cuda:0"), v[l:l + 1].to("cuda:0"), l)
    return cache


@torch.no_grad()
def _hf_gpu_step(hf, w, cache, tok, pos):
    out = hf.model(input_ids=torch.tensor([[int(tok)]], device="cuda:0"),
                   position_ids=torch.tensor([[int(pos)]], device="cuda:0"),
                   past_key_values=cache, use_cache=True)
    return _hf_gpu_logits(hf, w, out.last_hidden_state[:, -1]).cpu()


def _check_argmax(got_ids, logits_ref, slack):
    for b in range(logits_ref.shape[0]):
        top2 = logits_ref[b].topk(2).values
        if (top2[0] - top2[1]).item() > 2 * slack:
            assert int(got_ids[b]) == int(logits_ref[b].argmax()), b


def _run_step_case(cfg, w, B, positions, page_size, seed, w32=None, hf=None):
    """Fill random caches to positions[b], decode one step on GPU and oracle.

    With ``w32`` (fp32 weights) the step is also evaluated in fp32 and the
    logits and the deeper layers' K/V rows are held to the envelope. With
    ``hf`` (the second implementation, B = 1) the kernel's max |logit -
    reference| must be within SECOND_SLACK of HF-on-GPU's."""
    max_len = max(positions) + 1
    m = _model(cfg, w, B, max_seq_len=max_len + page_size, page_size=page_size, shuffle=seed)
    for b in range(B):
        k, v = syn.random_kv_rows(cfg, positions[b], seed=seed, seq=b)
        m.kv.reserve(b, positions[b] + 1)
        if positions[b]:
            m.kv.fill(b, k, v)
    before_k, before_v = m.kv.k_pages.clone(), m.kv.v_pages.clone()
    kv_ref = _oracle_kv(m)
    kv32 = None
    if w32 is not None:
        kv32 = O.OracleKV(kv_ref.k_pages.float(), kv_ref.v_pages.float(), kv_ref.block_tables)
    toks = syn.random_tokens(B, cfg.vocab, seed=seed + 1)
    out = m.forward(toks.reshape(B, 1), torch.tensor(positions).reshape(B, 1))
    ref = O.decode_step(cfg, w, kv_ref, toks, positions)
    truth = O.decode_step(cfg, w32, kv32, toks, positions) if w32 is not None else None
    cos, err = _check_logits(out.logits, ref["logits"],
                             truth["logits"] if truth is not None else None)
    _check_argmax(out.next_ids, ref["logits"], err.max().item())
    if hf is not None:
        assert B == 1
        k, v = syn.random_kv_rows(cfg, positions[0], seed=seed, seq=0)
        second = _hf_gpu_step(hf, w, _hf_gpu_cache(hf, cfg, k, v), toks[0], positions[0])
        d_second = (second - ref["logits"]).abs().max().item()
        cos_second = torch.nn.functional.cosine_similarity(second, ref["logits"], dim=-1).item()
        d_kernel = err.max().item()
        print(f"pos {positions[0]}: max|kernel-ref| {d_kernel:.4f} (cos {cos.min().item():.6f}), "
              f"max|hf_gpu-ref| {d_second:.4f} (cos {cos_second:.6f})")
        assert d_kernel <= SECOND_SLACK * d_second + 1e-3, (d_kernel, d_second)
    # KV scatter: exactly the rows at `positions` changed, with the oracle's values.
    ps = page_size
    changed = (m.kv.k_pages != before_k) | (m.kv.v_pages != before_v)
    expect = torch.zeros_like(changed)
    for b in range(B):
        page = int(m.kv.block_tables[b, positions[b] // ps])
        expect[:, page, :, positions[b] % ps] = True
    assert not (changed & ~expect).any(), "kernel wrote outside the new rows"
    for b in range(B):
        page = int(m.kv.block_tables[b, positions[b] // ps])
        kg = m.kv.k_pages[:, page, :, positions[b] % ps].float().cpu()
        vg = m.kv.v_pages[:, page, :, positions[b] % ps].float().cpu()
        kr, vr = ref["k_new"][b].float(), ref["v_new"][b].float()
        # Layer 0 sees identical inputs: a few ulps of its own rounding.
        assert (kg[0] - kr[0]).abs().max() <= KV_ROW_TOL
        assert (vg[0] - vr[0]).abs().max() <= KV_ROW_TOL
        if truth is None:
            assert (kg - kr).abs().max() <= KV_ROW_TOL
            assert (vg - vr).abs().max() <= KV_ROW_TOL
        else:
            kt, vt = truth["k_new"][b], truth["v_new"][b]
            for got, want, tru in ((kg, kr, kt), (vg, vr, vt)):
                d_ref = (want - tru).abs().amax(dim=(1, 2))
                d_got = (got - tru).abs().amax(dim=(1, 2))
                assert (d_got <= ENVELOPE * d_ref + KV_ROW_TOL).all(), (d_got, d_ref)
    return m, out, ref


@pytest.fixture(scope="module")
def small_w():
    return syn.make_weights(SMALL, seed=21)


@pytest.fixture(scope="module")
def tiny_w():
    return syn.make_weights(TINY, seed=22)


@pytest.mark.parametrize("pos", [0, 1, 7, 63, 64, 65, 130, 700])
def test_tiny_single_step_positions(tiny_w, pos):
    _run_step_case(TINY, tiny_w, 1, [pos], page_size=16, seed=pos + 1)


@pytest.mark.parametrize("page_size", [8, 64, 128])
def test_small_page_sizes(small_w, page_size):
    _run_step_case(SMALL, small_w, 1, [333], page_size=page_size, seed=page_size)


@pytest.mark.parametrize("positions", [[5, 300], [0, 64, 129], [1000, 17, 256, 64]],
                         ids=["b2", "b3", "b4"])
def test_small_batched_ragged(small_w, positions):
    _run_step_case(SMALL, small_w, len(positions), positions, page_size=32, seed=len(positions))


def test_small_deterministic_and_multistep(small_w):
    m = _model(SMALL, small_w, 1, max_seq_len=256, page_size=32)
    m.kv.reserve(0, 40)  # the oracle copies the block table: pages must exist first
    kv_ref = _oracle_kv(m)
    toks = syn.random_tokens(40, SMALL.vocab, seed=3)
    for t in range(40):
        out = m.forward(toks[t].reshape(1, 1), torch.tensor([[t]]))
        ref = O.decode_step(SMALL, small_w, kv_ref, toks[t:t + 1], [t])
        _check_logits(out.logits, ref["logits"])
        # teacher-forced: the oracle keeps its own cache, the kernel its own
    again = m.new_cache()
    a = m.forward(toks[:5].reshape(1, 5), past_key_values=again)
    b = m.forward(toks[:5].reshape(1, 5), torch.arange(5).reshape(1, 5), past_key_values=m.new_cache())
    assert torch.equal(a.logits, b.logits) and torch.equal(a.next_ids, b.next_ids)


def test_small_hidden_mode(small_w):
    m = _model(SMALL, small_w, 2, max_seq_len=256, page_size=32, shuffle=5)
    positions = [40, 100]
    for b in range(2):
        k, v = syn.random_kv_rows(SMALL, positions[b], seed=9, seq=b)
        m.kv.fill(b, k, v)
        m.kv.reserve(b, positions[b] + 1)
    kv_ref = _oracle_kv(m)
    x = syn.hashed_normal((2, SMALL.hidden), 4, 77, 1.0)
    y = m.forward_hidden(x.cuda(), torch.tensor(positions))
    ref = O.decode_step(SMALL, small_w, kv_ref, [0, 0], positions, layers=SMALL.num_layers,
                        hidden_in=x)
    d = (y.float().cpu() - ref["hidden"].float()).abs().max().item()
    scale = ref["hidden"].float().abs().max().item()
    assert d <= 0.02 * scale + 0.02, (d, scale)


def test_small_generate_feedback_matches_forward(small_w):
    m = _model(SMALL, small_w, 1, max_seq_len=256, page_size=32)
    prompt = syn.random_tokens(10, SMALL.vocab, seed=8).reshape(1, 10)
    gen = m.generate(prompt, 20, past_key_values=m.new_cache())
    kv = m.new_cache()
    out = m.forward(prompt, past_key_values=kv)
    toks = [int(out.next_ids[0])]
    for s in range(19):
        out = m.forward(torch.tensor([[toks[-1]]]), past_key_values=kv)
        toks.append(int(out.next_ids[0]))
    assert gen[0].tolist() == toks


# ----------------------------------------------------------------------------
# MID: two Llama-3.2-1B-shaped layers with a small vocabulary
# ----------------------------------------------------------------------------

@pytest.fixture(scope="module")
def mid_w():
    return syn.make_weights(MID, seed=23)


@pytest.fixture(scope="module")
def mid_w32(mid_w):
    return _fp32_copy(mid_w)


@pytest.mark.parametrize("pos", [0, 1, 47, 48, 130, 600])
def test_mid_single_step_positions(mid_w, mid_w32, pos):
    _run_step_case(MID, mid_w, 1, [pos], page_size=64, seed=pos + 3, w32=mid_w32)


def test_mid_batched_ragged(mid_w, mid_w32):
    _run_step_case(MID, mid_w, 2, [300, 17], page_size=32, seed=4, w32=mid_w32)


def test_mid_multistep_deterministic(mid_w):
    m = _model(MID, mid_w, 1, max_seq_len=128, page_size=64)
    toks = syn.random_tokens(6, MID.vocab, seed=13)
    a = m.forward(toks.reshape(1, 6), past_key_values=m.new_cache())
    b = m.forward(toks.reshape(1, 6), past_key_values=m.new_cache())
    assert torch.equal(a.logits, b.logits) and torch.equal(a.next_ids, b.next_ids)


# ----------------------------------------------------------------------------
# Llama-3.2-1B
# ----------------------------------------------------------------------------

@pytest.fixture(scope="module")
def llama_w():
    w = syn.make_weights(LLAMA_3_2_1B, seed=0, device="cuda")
    return {k: v.cpu() for k, v in w.items()}


@pytest.fixture(scope="module")
def llama_w32(llama_w):
    return _fp32_copy(llama_w)


@pytest.fixture(scope="module")
def llama_hf_gpu(llama_w):
    hf = _hf_gpu_model(LLAMA_3_2_1B, llama_w)
    yield hf
    del hf
    llama_w.pop("_embed_f32_cuda", None)
    torch.cuda.empty_cache()


@pytest.mark.parametrize("ctx", [128, 1024, 4096, 8192])
def test_llama1b_single_step_ctx(llama_w, llama_w32, llama_hf_gpu, ctx):
    """One step at position ctx over ctx cached N(0,1) rows (the context sweep),
    held to the fp32 envelope and to the second implementation's distance."""
    m, out, ref = _run_step_case(LLAMA_3_2_1B, llama_w, 1, [ctx], page_size=64, seed=ctx,
                                 w32=llama_w32, hf=llama_hf_gpu)
    del m


def test_llama1b_greedy_640_teacher_forced(llama_w, llama_w32, llama_hf_gpu):
    """128-token prompt, then 640 greedy steps (the bench workload).

    The kernel is fed the oracle's greedy tokens (teacher forcing, as the
    reference's logit_validation re-synchronises after a divergence). At four
    steps the kernel's own cache is copied to the oracle and the full logits
    are compared (envelope criterion, with the fp32 evaluation).

    Greedy agreement: in this random-init model the top-2 logits of many steps
    are closer than bf16 rounding noise (median margin 0.135, 13% of steps
    under 0.03), and the fixture records that exact fp32 arithmetic, fed the
    same tokens, agrees with the bf16 reference's argmax at only
    ``fp32_teacher_forced_match`` (about 93%) of the steps. So the kernel must
    (a) agree at >= 99% of the steps whose reference margin exceeds
    MARGIN_SURE (the fp32 evaluation agrees at all 388 of them; its
    disagreements all have margins under 0.08), and
    (b) agree overall at no less than the fp32 evaluation's rate minus 2%.
    A 99% bar applies where the reference's decisions are not within noise.
    (c) The second implementation (HF in bf16 on the GPU), teacher-forced the
    same way, sets the overall bar: the kernel must agree with the reference
    at no less than its rate minus MATCH_SLACK.
    """
    d = json.loads((GOLDEN / "llama1b_greedy640.json").read_text())
    from tests.golden.make_golden import weight_fingerprint

    assert d["weight_fingerprint"] == weight_fingerprint(LLAMA_3_2_1B, 0)
    cfg = LLAMA_3_2_1B
    m = _model(cfg, llama_w, 1, max_seq_len=1024, page_size=d["page_size"])
    prompt = torch.tensor(d["prompt"]).reshape(1, -1)
    m.forward(prompt[:, :-1], return_logits=False)
    feed = [d["prompt"][-1]] + d["tokens"][:-1]
    pos0 = d["first_decode_position"]
    tok_dev = torch.tensor(feed, dtype=torch.int32, device="cuda")
    pos_dev = torch.arange(pos0, pos0 + 640, dtype=torch.int32, device="cuda")
    got = torch.empty(640, dtype=torch.int32, device="cuda")
    top1 = torch.empty(640, dtype=torch.float32, device="cuda")
    want_top1 = torch.tensor([float.fromhex(v[0]) for v in d["top2_logits_f32_hex"]], device="cuda")
    want_ids = torch.tensor([i[0] for i in d["top2_ids"]], device="cuda")
    logits = torch.empty(1, cfg.vocab, dtype=torch.float32, device="cuda")
    m.kv.reserve(0, pos0 + 640)
    checks = {0, 100, 320, 639}
    for s in range(640):
        if s in checks:
            torch.cuda.synchronize()
            kv_ref = _oracle_kv(m)
        m.launch(tok_dev[s:s + 1], pos_dev[s:s + 1], m.kv, logits, got[s:s + 1])
        top1[s] = logits[0, want_ids[s]]
        if s in checks:
            m.sync()
            kv32 = O.OracleKV(kv_ref.k_pages.float(), kv_ref.v_pages.float(), kv_ref.block_tables)
            ref = O.decode_step(cfg, llama_w, kv_ref, [feed[s]], [pos0 + s])
            truth = O.decode_step(cfg, llama_w32, kv32, [feed[s]], [pos0 + s])
            _check_logits(logits, ref["logits"], truth["logits"])
    m.sync()
    # The second implementation: HF bf16 on the GPU, the prompt prefilled in
    # one forward, then the same teacher-forced tokens one step at a time.
    with torch.no_grad():
        from transformers import DynamicCache

        hf = llama_hf_gpu
        cache = DynamicCache(config=hf.config)
        hf.model(input_ids=prompt[:, :-1].to("cuda:0"), past_key_values=cache, use_cache=True)
        hf_ids, hf_top1 = [], []
        for s_ in range(640):
            lg = _hf_gpu_step(hf, llama_w, cache, feed[s_], pos0 + s_)[0]
            hf_ids.append(int(lg.argmax()))
            hf_top1.append(float(lg[int(want_ids[s_])]))
    hf_same = torch.tensor(hf_ids) == want_ids.cpu()
    hf_match = hf_same.float().mean().item()
    hf_drift = (torch.tensor(hf_top1) - want_top1.cpu()).abs().max().item()
    same = (got.long() == want_ids).cpu()
    match = same.float().mean().item()
    drift = (top1 - want_top1).abs().max().item()
    top2 = torch.tensor([[float.fromhex(v) for v in r] for r in d["top2_logits_f32_hex"]])
    margin = top2[:, 0] - top2[:, 1]
    sure = margin > MARGIN_SURE
    print(f"greedy match {match:.4f} (fp32 evaluation {d['fp32_teacher_forced_match']:.4f}, "
          f"HF bf16 on the GPU {hf_match:.4f}), steps with margin > {MARGIN_SURE}: "
          f"{int(sure.sum())}, matched {int(same[sure].sum())} (HF GPU "
          f"{int(hf_same[sure].sum())}); max |top1 logit - fixture| {drift:.4f} "
          f"(HF GPU {hf_drift:.4f})")
    assert same[sure].float().mean().item() >= 0.99
    assert match >= d["fp32_teacher_forced_match"] - 0.02
    assert match >= hf_match - MATCH_SLACK
    assert drift <= DRIFT_MAX
