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
  * kv_store.py (RoPE, KV-slot scatter) and attention.py are PINNED:
    tests/test_numeric_golden.py compares them with tests/golden/numerics.npz,
    produced by running the reference's own apply_rope, _update_kv_cache,
    attention() (default Pallas path and jnp path) and its two *_reference
    functions under a numpy + ml_dtypes JAX stand-in
    (tests/golden/make_numeric_golden.py, tests/golden/jax_shim.py):
    RoPE and slot writes bit for bit, attention within max-abs 2e-2 /
    mean-abs 2e-3. The stand-in rounds after every op; XLA may fuse ops and
    keep f32 between them, which can move single bf16 ulps.
  * RMSNorm comes from flax (not in the reference tree): restated as fp32
    statistics, bf16(x * (rsqrt(mean(x^2) + eps) * scale)), the 128-dim q/k
    rows summed in the fixed fp32 order of vj_kv_store_qknorm_rope.
  * qwen3.py composes the pinned pieces with the reference's layer dataflow;
    sampler.py checks kept sets exactly and draws in distribution (JAX's
    threefry stream is not reproduced).
"""
