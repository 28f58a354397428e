"""KV-slot scatter fused with Qwen3's per-head q/k RMSNorm and RoPE (K3).

Torch-facing wrappers of vj_kv_store_qknorm_rope. They replace, in vllm-jax:
  vllm/model/qwen3.py:105-111  _update_kv_cache(kv_cache, slot_mapping, k, v)
  vllm/model/qwen3.py:286-296  q_norm/k_norm + apply_rope (:59-78)
The KV cache is updated IN PLACE (the reference's XLA scatter into a
non-donated buffer copies the whole pool every layer).
"""
from __future__ import annotations

import torch

from .. import _native
from ._util import ptr, require_cuda, require_dtype, stream_ptr


def _cache_views(kv_cache: torch.Tensor):
    """kv_cache (2, num_blocks, block_size, Hkv, D) -> (k, v, nb, bs, strides)."""
    if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
        raise ValueError("kv_cache must have shape (2, num_blocks, block_size, Hkv, D); "
                         f"got {tuple(kv_cache.shape)}")
    require_dtype(kv_cache, torch.bfloat16, "kv_cache")
    k, v = kv_cache[0], kv_cache[1]
    if k.stride(-1) != 1:
        raise ValueError("kv_cache head_dim must be contiguous")
    nb, bs = k.shape[0], k.shape[1]
    return k, v, nb, bs, (k.stride(0), k.stride(1), k.stride(2))


_rope_tables: dict[tuple[int, float], torch.Tensor] = {}
_retired_tables: list[torch.Tensor] = []
DEFAULT_ROPE_POSITIONS = 4096


def rope_table(device: torch.device, rope_theta: float = 1e6,
               num_positions: int = DEFAULT_ROPE_POSITIONS) -> torch.Tensor:
    """The (cos, sin) bf16 pair table of positions [0, num_positions) for
    rope_theta on `device` (vj_rope_table_build), cached per device and theta
    and only grown. An outgrown table is retired, not freed, because a CUDA
    graph captured with it keeps reading its address. Positions past the end
    of the table are computed inside the kernel (same bits, slower)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, float(rope_theta))
    t = _rope_tables.get(key)
    if t is None or t.numel() < num_positions * 64:
        if t is not None:
            _retired_tables.append(t)
        n = max(num_positions, DEFAULT_ROPE_POSITIONS)
        nbytes = _native.load().vj_rope_table_bytes(n, 128)
        t = torch.empty(nbytes // 4, dtype=torch.int32, device=device)
        _native.call("vj_rope_table_build", t.data_ptr(), n, 128, float(rope_theta),
                     stream_ptr(device))
        _rope_tables[key] = t
    return t


_QSCALE = {None: 0, "div": 8, "mul": 16}


def kv_store_qknorm_rope(q: torch.Tensor | None, k: torch.Tensor, v: torch.Tensor,
                         kv_cache: torch.Tensor, slot_mapping: torch.Tensor,
                         positions: torch.Tensor | None = None,
                         q_norm_weight: torch.Tensor | None = None,
                         k_norm_weight: torch.Tensor | None = None, *,
                         eps: float = 1e-6, rope_theta: float = 1e6,
                         norm: bool = True, rope: bool = True,
                         wrap_negative_slots: bool = True,
                         q_out: torch.Tensor | None = None,
                         return_k: bool = False,
                         q_scale: str | None = None,
                         table: torch.Tensor | None = None):
    """One launch: q_out = scale(rope(norm(q))), cache[slot] = (rope(norm(k)), v).

    q [T, Hq, D] (or None), k/v [T, Hkv, D] bf16; slot_mapping/positions [T]
    int32. q_scale: None, "div" (bf16(q / bf16(sqrt(D))), the reference's
    decode scaling, vllm/model/qwen3.py:207) or "mul" (bf16(q *
    bf16(1/sqrt(D))), its prefill kernel's, prefill_paged_attention.py:60).
    table: a rope_table() for rope_theta (default: the cached one of this
    device). Returns q_out (and k_out if return_k)."""
    dev = require_cuda(k, v, kv_cache, slot_mapping)
    kc, vc, nb, bs, (sb, st, sh) = _cache_views(kv_cache)
    T, Hkv, D = k.shape
    if v.shape != k.shape:
        raise ValueError(f"k and v must have the same shape. Got {tuple(k.shape)} and {tuple(v.shape)}")
    for name, t in (("k", k), ("v", v)):
        require_dtype(t, torch.bfloat16, name)
        if t.stride(2) != 1 or t.stride(1) != D:
            raise ValueError(f"`{name}` must have contiguous head rows ([T, H, D] with packed heads)")
    require_dtype(slot_mapping, torch.int32, "slot_mapping")
    if slot_mapping.shape != (T,):
        raise ValueError("slot_mapping must have shape [num_tokens]")
    Hq = 0
    if q is not None:
        require_dtype(q, torch.bfloat16, "q")
        if q.dim() != 3 or q.shape[0] != T or q.shape[2] != D or q.stride(2) != 1 \
                or q.stride(1) != D:
            raise ValueError("q must be a [num_tokens, Hq, head_dim] tensor with packed heads")
        Hq = q.shape[1]
        if q_out is None:
            q_out = torch.empty((T, Hq, D), dtype=q.dtype, device=q.device)
    if kc.shape[2] != Hkv or kc.shape[3] != D:
        raise ValueError("kv_cache heads/head_dim do not match k")
    flags = 0
    if norm:
        flags |= _native.VJ_KV_NORM
        if k_norm_weight is None or (q is not None and q_norm_weight is None):
            raise ValueError("norm=True needs q_norm_weight and k_norm_weight")
    if rope:
        flags |= _native.VJ_KV_ROPE
        if positions is None:
            raise ValueError("rope=True needs positions")
        require_dtype(positions, torch.int32, "positions")
    if wrap_negative_slots:
        flags |= _native.VJ_KV_WRAP_NEGATIVE
    if q_scale not in _QSCALE:
        raise ValueError(f"q_scale must be None, 'div' or 'mul'; got {q_scale!r}")
    flags |= _QSCALE[q_scale]
    if rope and table is None:
        table = rope_table(dev, rope_theta)
    tab_len = table.numel() // 64 if (rope and table is not None) else 0
    k_out = torch.empty((T, Hkv, D), dtype=k.dtype, device=k.device) if return_k else None
    _native.call("vj_kv_store_qknorm_rope",
                 ptr(q), k.data_ptr(), v.data_ptr(), ptr(q_norm_weight if norm else None),
                 ptr(k_norm_weight if norm else None), ptr(positions if rope else None),
                 slot_mapping.data_ptr(), ptr(q_out), ptr(k_out), kc.data_ptr(), vc.data_ptr(),
                 T, Hq, Hkv, D, nb, bs, sb, st, sh, q.stride(0) if q is not None else 0,
                 k.stride(0), v.stride(0), ptr(table) if tab_len else None, tab_len,
                 float(eps), float(rope_theta), flags, stream_ptr(dev))
    if return_k:
        return q_out, k_out
    return q_out


def update_kv_cache(kv_cache: torch.Tensor, slot_mapping: torch.Tensor, k: torch.Tensor,
                    v: torch.Tensor) -> torch.Tensor:
    """Drop-in for vllm/model/qwen3.py:105-111 `_update_kv_cache` (in place).

    Slots are flat (block * block_size + offset); slot -1 wraps to the last
    slot like JAX's .at[] with mode="drop"; other out-of-range slots drop."""
    kv_store_qknorm_rope(None, k, v, kv_cache, slot_mapping, norm=False, rope=False)
    return kv_cache
