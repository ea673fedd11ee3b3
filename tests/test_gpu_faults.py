"""Failure detection on the GPU without a GPU fault.

Every device-side wait in the kernel is time-bounded and every index it
dereferences is range-checked first; failures set a device error word and the
launch returns. These tests make a wait run out (one CTA skips its barrier
arrival: the debug knob) and feed out-of-range positions, page ids and tokens,
then check that mk_sync reports the right status and that the next normal
step on the same handle is correct.
"""
import pytest
import torch

from llama1b_megakernel_b200 import _lib
from llama1b_megakernel_b200 import synthetic as syn
from llama1b_megakernel_b200.config import TINY

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    from llama1b_megakernel_b200.model import MegakernelLlamaForCausalLM

    w = syn.make_weights(TINY, seed=2)
    m = MegakernelLlamaForCausalLM(TINY, w, max_batch=1, max_seq_len=128, page_size=16,
                                   device="cuda:0")
    m.set_timeout_ns(200_000_000)  # 0.2 s per wait
    return m


def _good_step(m):
    out = m.forward(torch.tensor([[5]]), torch.tensor([[3]]), past_key_values=m.new_cache())
    assert 0 <= int(out.next_ids[0]) < TINY.vocab
    return out


def test_barrier_timeout_reports_and_recovers(model):
    ref = _good_step(model)
    model.debug_skip_arrival(7)
    with pytest.raises(_lib.MkError) as e:
        model.forward(torch.tensor([[5]]), torch.tensor([[3]]), past_key_values=model.new_cache())
    assert e.value.status == _lib.MK_ETIMEOUT
    model.debug_skip_arrival(-1)
    again = _good_step(model)
    assert torch.equal(again.logits, ref.logits)


def test_bad_page_id_is_rejected(model):
    kv = model.new_cache()
    kv.reserve(0, 40)
    kv.block_tables[0, 1] = kv.num_pages + 5  # positions 16..31 point outside the pool
    with pytest.raises(_lib.MkError) as e:
        model.forward(torch.tensor([[5]]), torch.tensor([[35]]), past_key_values=kv)
    assert e.value.status == _lib.MK_EDEVICE
    _good_step(model)


def test_position_beyond_table_is_rejected(model):
    kv = model.new_cache()
    tok = torch.tensor([5], dtype=torch.int32, device="cuda")
    pos = torch.tensor([model.rope_len + 3], dtype=torch.int32, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    model.launch(tok, pos, kv, None, nxt)
    with pytest.raises(_lib.MkError) as e:
        model.sync()
    assert e.value.status == _lib.MK_EDEVICE
    _good_step(model)


def test_token_out_of_vocab_is_rejected(model):
    kv = model.new_cache()
    kv.reserve(0, 4)
    tok = torch.tensor([TINY.vocab + 1], dtype=torch.int32, device="cuda")
    pos = torch.tensor([2], dtype=torch.int32, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int32, device="cuda")
    model.launch(tok, pos, kv, None, nxt)
    with pytest.raises(_lib.MkError) as e:
        model.sync()
    assert e.value.status == _lib.MK_EDEVICE
    _good_step(model)


def test_host_side_validation(model):
    kv = model.new_cache()
    tok = torch.zeros(2, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.MkError) as e:
        model.launch(tok, tok, kv, None, tok)  # batch 2 > max_batch 1
    assert e.value.status == _lib.MK_EINVAL
