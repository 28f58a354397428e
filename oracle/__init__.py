"""CPU oracle for the vllm-jax paged-attention hot path -- TEST INFRASTRUCTURE.

This package is a NumPy restatement of the reference's algorithms, used only
as the checker by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
/ --impl reference arms. The product (vllm_b200 + libvjattn.so) never imports
it and has no CPU fallback.

Modules and the reference code each one follows (vllm-jax, simpissa):
  bf16.py        bf16 rounding helpers (ml_dtypes round-to-nearest-even)
  kv_store.py    vllm/model/qwen3.py:59-78 apply_rope, :105-111 _update_kv_cache,
                 :286-296 q/k RMSNorm (flax nnx.RMSNorm) + RoPE
  attention.py   vllm/kernels/decode_paged_attention.py:400-463
                 (paged_attention_reference) and
                 vllm/kernels/prefill_paged_attention.py:456-505
                 (prefill_paged_attention_reference), gathered through
                 block tables and generalised to a cached prefix
  host.py        vllm/src/kv_cache_manager.py, vllm/src/scheduler.py,
                 vllm/src/request.py and vllm/src/model_runner.py:185-301
                 (bucketing and batch-metadata packing), plus the chunked
                 ranges packing (prepare_ranges; equal to prepare_prefill
                 when every sequence starts at position 0)
  qwen3.py       the Qwen3 layer dataflow (vllm/model/qwen3.py:284-301,
                 :337-341, :375-389, :432-477) and greedy replays of a
                 golden schedule (C1) or of a recorded chunked / prefix-
                 cached schedule
  sampler.py     vllm/sampler.py:7-42 kept sets (top-k, top-p over
                 bf16(logits / T)) and the sampling distribution

Parity status:
  * host.py (scheduler, block manager, metadata) is PINNED: tests compare it
    with tests/golden/host_traces.json, recorded by importing the
    reference's own Python modules (tests/golden/make_golden.py).
  * kv_store.py / attention.py / qwen3.py / sampler.py: the reference's
    JAX/XLA numerics cannot run in this image (no jax, no flax), and no
    reference test pins them, so they are "parity unpinned": the restatement
    follows the reference's code and documented semantics (fp32 logits and
    softmax, bf16 rounding after every jnp op of apply_rope, flax RMSNorm
    statistics in fp32). XLA's fusion may keep excess fp32 precision between
    ops, which can move single bf16 ulps; JAX's threefry sampling stream is
    not reproduced, so draws are checked in distribution.
"""
