"""GPU sampling (temperature / top-k / top-p / categorical), torch-facing.

`sample` launches vj_sample over a batch of logit rows. `Sampler` keeps the
interface of vllm-jax's vllm/sampler.py:7-42 (`sample(logits,
sampling_params, rng_key) -> (token_ids, rng_key)`); its rng_key is a
(seed, counter) pair of ints standing in for a JAX PRNG key: each call draws
with counter `counter` and returns (seed, counter + 1).
"""
from __future__ import annotations

import torch

from .. import _native
from ._util import require_cuda, stream_ptr


def as_i32(v: int) -> int:
    """Low 32 bits of v as a signed int32 value (same bit pattern)."""
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


def aligned_rows(logits: torch.Tensor) -> torch.Tensor:
    """logits with 16-byte aligned rows (copied into a padded buffer if not)."""
    R, V = logits.shape
    if logits.stride(1) == 1 and logits.stride(0) % 8 == 0 and logits.data_ptr() % 16 == 0:
        return logits
    buf = torch.empty((R, (V + 7) // 8 * 8), dtype=logits.dtype, device=logits.device)
    buf[:, :V].copy_(logits)
    return buf[:, :V]


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
           top_p: torch.Tensor, seeds: torch.Tensor, positions: torch.Tensor | None = None,
           num_kept: torch.Tensor | None = None, out: torch.Tensor | None = None,
           token_table: torch.Tensor | None = None,
           slots: torch.Tensor | None = None) -> torch.Tensor:
    """logits [R, V] bf16 (row stride a multiple of 8); temperature/top_p
    float32 [R]; top_k int32 [R]; seeds int32/uint32 [R, 2]; positions int32
    [R] (the Philox counter and, with token_table/slots, the column the token
    is stored at). Returns int32 [R]."""
    dev = require_cuda(logits, temperature, top_k, top_p, seeds)
    if logits.dtype != torch.bfloat16 or logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("logits must be a row-contiguous bf16 [rows, vocab] tensor")
    R, V = logits.shape
    for name, t, dt in (("temperature", temperature, torch.float32), ("top_k", top_k, torch.int32),
                        ("top_p", top_p, torch.float32)):
        if t.dtype != dt or t.shape != (R,):
            raise ValueError(f"{name} must be {dt} of shape [{R}]")
    if seeds.numel() != 2 * R or seeds.element_size() != 4:
        raise ValueError("seeds must hold two 32-bit words per row")
    if out is None:
        out = torch.empty(R, dtype=torch.int32, device=dev)
    _native.call("vj_sample", logits.data_ptr(), logits.stride(0), R, V, temperature.data_ptr(),
                 top_k.data_ptr(), top_p.data_ptr(), seeds.data_ptr(), out.data_ptr(),
                 None if num_kept is None else num_kept.data_ptr(),
                 None if token_table is None else token_table.data_ptr(),
                 0 if token_table is None else token_table.stride(0),
                 None if slots is None else slots.data_ptr(),
                 None if positions is None else positions.data_ptr(), stream_ptr(dev))
    return out


class Sampler:
    """vllm/sampler.py:7-42 with the draw on the GPU."""

    def sample(self, logits: torch.Tensor, sampling_params, rng_key=(0, 0)):
        if logits.dim() == 1:
            logits = logits[None, :]
        R = logits.shape[0]
        dev = logits.device
        seed, counter = (rng_key, 0) if isinstance(rng_key, int) else rng_key
        temp = torch.full((R,), float(sampling_params.temperature), dtype=torch.float32,
                          device=dev)
        k = torch.full((R,), int(sampling_params.top_k), dtype=torch.int32, device=dev)
        p = torch.full((R,), float(sampling_params.top_p), dtype=torch.float32, device=dev)
        seeds = torch.tensor([[as_i32(seed), as_i32(seed >> 32)]] * R, dtype=torch.int32,
                             device=dev)
        pos = torch.full((R,), counter, dtype=torch.int32, device=dev)
        toks = sample(aligned_rows(logits), temp, k, p, seeds, pos)
        return toks, (seed, counter + 1)
