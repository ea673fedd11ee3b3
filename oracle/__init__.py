"""CPU oracle for the Llama-3.2-1B decode hot path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or the timed CPU baseline. The product path
(``llama1b_megakernel_b200``) never imports it and has no CPU fallback.

Two checkers live here:

* ``llama_oracle.hf_model`` builds HF ``transformers.LlamaForCausalLM``
  (pinned: transformers 5.5.0 in this image), the PyTorch Llama the reference
  loads as its HF model (llama.py:1286-1288) and validates against
  (main.py:274-357).
* ``llama_oracle.decode_step`` is a compact restatement of one decode step
  over a *paged* KV cache, written with the same torch ops and shapes as HF
  so that it matches HF bit for bit (tests/test_oracle.py checks this), while
  exposing the per-stage values the GPU parity tests need (K/V rows written,
  fp32 logits, greedy argmax).

RoPE follows the reference's ``Llama3RotaryEmbedding`` (llama.py:888-953):
fp32 ``inv_freq`` with llama3 scaling, cos/sin in fp32 cast to bf16. The
inverse frequencies are pinned against vectors produced by the reference's own
class (tests/golden/rope_llama3.json, made by tests/golden/make_golden.py).
"""
