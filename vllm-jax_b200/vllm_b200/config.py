"""Engine configuration (vllm/config.py:3-10 of vllm-jax, plus TP and memory knobs)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class Config:
    model: str
    max_num_batched_tokens: int
    max_num_seqs: int
    num_blocks: int
    block_size: int
    # additions of this build
    tensor_parallel_size: int = 1
    gpu_memory_utilization: float = 0.9   # used when num_blocks <= 0
    max_model_len: int | None = None       # default: max_num_batched_tokens (reference)
    # compat=True reproduces the reference's host-side behaviour bit for bit:
    # finished requests keep their blocks (scheduler.py:65-70) and a decode
    # token is stored in the last allocated block (model_runner.py:282-284).
    compat: bool = True
    # Token-budget scheduling with prompts split into chunks that share a
    # forward with decode rows (not in the reference). Implies compat=False
    # behaviour: position-addressed slots and blocks freed on finish.
    enable_chunked_prefill: bool = False
    # Share the KV blocks of identical prompt prefixes between requests
    # (needs enable_chunked_prefill: a request then starts after its hit).
    enable_prefix_caching: bool = False
    # Under tensor parallelism: "nvlink" reduces decode-sized batches with the
    # fused peer-memory kernel (CUDA-graph capturable), "nccl" always uses
    # torch.distributed all-reduce (decode then runs eagerly).
    tp_allreduce: str = "nvlink"
    # With compat=False (and without chunked prefill) generate() schedules
    # step k+1 before reading step k's tokens back, so host work overlaps the
    # GPU; a request that samples EOS is computed one extra, discarded step.
    async_scheduling: bool = True
    # Forward passes of at most this many rows (decode steps, small mixed
    # steps) run their projections on this library's tcgen05 GEMMs with fused
    # epilogues: qkv + q/k norm + RoPE + KV store in one launch, gate_up +
    # SiLU-mul in one, o_proj / down_proj plain; larger ones use cuBLAS and the
    # separate kernels. 0 turns the fused path off.
    fused_gemm_max_rows: int = 0

    @property
    def max_len(self) -> int:
        return self.max_model_len or self.max_num_batched_tokens

    @property
    def max_blocks_per_seq(self) -> int:
        return (self.max_len + self.block_size - 1) // self.block_size
