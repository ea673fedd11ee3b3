"""Host-side logic without a GPU: packing, cache bookkeeping, generator, config."""
import numpy as np
import pytest
import torch

from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200 import weights as W
from llama1b_megakernel_b200.config import LLAMA_3_2_1B, SMALL, TINY, LlamaDecodeConfig
from llama1b_megakernel_b200.kv_cache import PagedKVCache


def test_param_and_byte_counts():
    assert LLAMA_3_2_1B.num_params() == 1_235_814_400
    assert LLAMA_3_2_1B.weight_bytes_per_token() == 2_471_632_896
    assert LLAMA_3_2_1B.kv_bytes_per_position() == 32_768


def test_qkv_pack_roundtrip_and_pairs():
    cfg = SMALL
    wq = torch.randn(cfg.q_dim, cfg.hidden).to(torch.bfloat16)
    wk = torch.randn(cfg.kv_dim, cfg.hidden).to(torch.bfloat16)
    wv = torch.randn(cfg.kv_dim, cfg.hidden).to(torch.bfloat16)
    packed = W.pack_qkv_layer(cfg, wq, wk, wv)
    assert packed.shape == ((cfg.num_q_heads + 2 * cfg.num_kv_heads) * 32, 2, cfg.hidden)
    # unit u = head * 32 + d holds rows d and d + 32 of that head
    for head, d in [(0, 0), (3, 17), (cfg.num_q_heads, 5), (cfg.num_q_heads + cfg.num_kv_heads + 1, 31)]:
        full = torch.cat([wq, wk, wv])
        u = head * 32 + d
        assert torch.equal(packed[u, 0], full[head * 64 + d])
        assert torch.equal(packed[u, 1], full[head * 64 + d + 32])
    q2, k2, v2 = W.unpack_qkv_layer(cfg, packed)
    assert torch.equal(q2, wq) and torch.equal(k2, wk) and torch.equal(v2, wv)


def test_pack_weights_cpu_layouts():
    cfg = TINY
    sd = syn.make_weights(cfg, seed=1)
    pw = W.pack_weights(cfg, sd, rope_len=64, device="cpu")
    assert pw.w_gate_up.shape == (cfg.num_layers, cfg.intermediate, 2, cfg.hidden)
    assert torch.equal(pw.w_gate_up[1, 7, 0], sd["model.layers.1.mlp.gate_proj.weight"][7])
    assert torch.equal(pw.w_gate_up[1, 7, 1], sd["model.layers.1.mlp.up_proj.weight"][7])
    assert torch.equal(pw.w_down[0], sd["model.layers.0.mlp.down_proj.weight"])
    assert torch.equal(pw.w_o[1], sd["model.layers.1.self_attn.o_proj.weight"])
    assert pw.rope_cos.shape == (64, 64)
    for t in pw.tensors().values():
        assert t.is_contiguous() and t.dtype == torch.bfloat16


def test_rope_table_batched_equals_per_position():
    cfg = LLAMA_3_2_1B
    cos, sin = W.rope_tables(cfg, 300)
    from oracle.llama_oracle import rope_cos_sin

    inv = W.llama3_inv_freq(cfg)
    for p in (0, 1, 17, 128, 299):
        c, s = rope_cos_sin(inv, torch.tensor([[p]]))
        assert torch.equal(cos[p], c.reshape(-1)) and torch.equal(sin[p], s.reshape(-1))


def test_generator_is_splitmix64_over_quantile_table():
    # Independent numpy restatement of the generator for a few elements.
    seed, stream, n = 7, 3, 1000
    got = syn.hashed_normal((n,), seed, stream, 0.02)
    M = np.uint64
    base = ((seed * 1_000_003 + stream) << 36) & ((1 << 64) - 1)
    words = np.arange((n + 3) // 4, dtype=np.uint64) + M(base)
    with np.errstate(over="ignore"):
        z = words * M(0x9E3779B97F4A7C15)
        z = (z ^ (z >> M(30))) * M(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> M(27))) * M(0x94D049BB133111EB)
        z = z ^ (z >> M(31))
    idx = z.view(np.uint16)[:n]
    want = syn.normal_table(0.02)[torch.from_numpy(idx.astype(np.int64))]
    assert torch.equal(got, want)
    big = syn.hashed_normal((1 << 20,), 0, 1, 0.02).float()
    assert abs(big.std().item() - 0.02) < 2e-4 and abs(big.mean().item()) < 1e-4
    # Element i depends only on (seed, stream, i): a prefix is a prefix.
    assert torch.equal(syn.hashed_normal((100,), 0, 1, 0.02), big[:100].to(torch.bfloat16))


def test_tokens_in_range_and_seeded():
    a = syn.random_tokens(1000, 128256, seed=3)
    b = syn.random_tokens(1000, 128256, seed=3)
    assert torch.equal(a, b) and int(a.min()) >= 0 and int(a.max()) < 128256
    assert len(set(a.tolist())) > 990


def test_paged_cache_bookkeeping_cpu():
    cfg = TINY
    kv = PagedKVCache(cfg, max_batch=2, max_seq_len=64, page_size=16, num_pages=6, device="cpu")
    kv.reserve(0, 20)
    kv.reserve(1, 33)
    t0, t1 = kv.pages_of(0), kv.pages_of(1)
    assert len(t0) == 2 and len(t1) == 3 and not set(t0) & set(t1)
    assert kv.block_tables[0, :2].tolist() == t0 and kv.block_tables[0, 2:].eq(-1).all()
    with pytest.raises(RuntimeError):
        kv.reserve(0, 64)  # needs 4 pages, only 1 left
    kv.release(1)
    kv.reserve(0, 64)
    k = torch.randn(cfg.num_layers, 1, 40, 64).to(torch.bfloat16)
    v = torch.randn(cfg.num_layers, 1, 40, 64).to(torch.bfloat16)
    kv.fill(0, k, v)
    k2, v2 = kv.gather(0, 40)
    assert torch.equal(k2, k) and torch.equal(v2, v)
    with pytest.raises(ValueError):
        kv.reserve(0, 65)


def test_config_validation():
    LLAMA_3_2_1B.validate()
    with pytest.raises(ValueError):
        LlamaDecodeConfig(head_dim=128).validate()
    with pytest.raises(ValueError):
        LlamaDecodeConfig(hidden=2000).validate()
