"""Varlen paged prefill attention on sm_100a tensor cores (K1), torch-facing.

`prefill_paged_attention` keeps the signature, argument meaning and ValueError
checks of vllm-jax's vllm/kernels/prefill_paged_attention.py:407-453 (pages in
the Pallas layout [Hkv, total_pages, page_size, D], q not pre-scaled, the
1/sqrt(D) scale applied inside, output in packed token order with padded rows
zero). The reference derives causality from input_positions with keys
numbered from the sequence's first position (prefill :100-109); its engine
always prefills from position 0, which is the case reproduced here (keys ==
new tokens). Pallas tuning knobs are accepted and ignored.

`paged_prefill` is the engine's entry on the native cache layout with an
optional cached prefix per sequence (context_lens = prefix + new tokens).
"""
from __future__ import annotations

import math

import torch

from .. import _native
from ._util import require_cuda, require_dtype, stream_ptr

DEFAULT_MASK_VALUE = -0.7 * float(torch.finfo(torch.float32).max)

_err_flags: dict[int, torch.Tensor] = {}


def _err_flag(dev: torch.device) -> torch.Tensor:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    t = _err_flags.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _err_flags[idx] = t
    return t


def pipeline_error(device: torch.device | int = 0) -> bool:
    """True if a prefill pipeline wait timed out on this device (synchronises)."""
    dev = torch.device("cuda", device) if isinstance(device, int) else device
    return bool(_err_flag(dev).item())


def _launch(q, k_base, v_base, nb, bs, strides, hkv, block_tables, cu_seqlens_q, context_lens,
            max_seqlen_q, scale, out=None):
    dev = require_cuda(q, k_base, v_base, block_tables, cu_seqlens_q)
    T, Hq, D = q.shape
    S = cu_seqlens_q.shape[0] - 1
    if out is None:
        out = torch.empty_like(q)
    _native.call("vj_paged_prefill", q.data_ptr(), k_base.data_ptr(), v_base.data_ptr(),
                 block_tables.data_ptr(), cu_seqlens_q.data_ptr(),
                 None if context_lens is None else context_lens.data_ptr(), out.data_ptr(),
                 T, S, Hq, hkv, D, nb, bs, block_tables.shape[1], block_tables.stride(0),
                 strides[0], strides[1], strides[2], int(max_seqlen_q), float(scale),
                 _err_flag(dev).data_ptr(), stream_ptr(dev))
    return out


def prefill_paged_attention(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                            block_tables: torch.Tensor, cu_seqlens: torch.Tensor,
                            slot_mapping: torch.Tensor, input_positions: torch.Tensor, *,
                            max_seqlen_bucket: int, k_scales_pages=None, v_scales_pages=None,
                            block_m: int = 16, block_h: int = 16,
                            pages_per_compute_block: int = 8, k_splits: int = 8,
                            num_warps: int = 8, num_stages: int = 2, interpret: bool = False,
                            debug: bool = False, mask_value: float = DEFAULT_MASK_VALUE,
                            attn_logits_soft_cap: float | None = None) -> torch.Tensor:
    """q [total_tokens, num_heads, head_dim]; k_pages/v_pages [num_kv_heads,
    total_num_pages, page_size, head_dim]; block_tables int32 [batch,
    pages_per_sequence]; cu_seqlens int32 [batch + 1]. Returns
    [total_tokens, num_heads, head_dim]."""
    if block_h % 16:
        raise ValueError(f"block_h must divisible by 16, but is {block_h}.")
    total_tokens, num_heads, head_dim = q.shape
    num_kv_heads, total_pages, page_size, head_dim_k = k_pages.shape
    batch, _ = block_tables.shape
    if k_pages.shape != v_pages.shape:
        raise ValueError(f"k_pages and v_pages must have the same shape. Got {tuple(k_pages.shape)} "
                         f"and {tuple(v_pages.shape)}")
    if num_heads % num_kv_heads != 0:
        raise ValueError("Number of Q heads must be divisible by number of KV heads. Got "
                         f"{num_heads} and {num_kv_heads}.")
    if head_dim_k != head_dim:
        raise ValueError(f"head_dim of Q must be the same as that of K/V. Got {head_dim} and "
                         f"{head_dim_k}.")
    if tuple(cu_seqlens.shape) != (batch + 1,):
        raise ValueError("cu_seqlens must have shape [batch + 1]")
    if block_tables.dtype != torch.int32:
        raise ValueError("block_tables must be int32")
    if k_scales_pages is not None or v_scales_pages is not None or attn_logits_soft_cap is not None:
        raise NotImplementedError("quantized pages and logit soft-cap are not implemented")
    if interpret:
        raise NotImplementedError("interpret=True (CPU) is not available: the B200 path has no "
                                  "CPU fallback")
    require_dtype(q, torch.bfloat16, "q")
    require_dtype(k_pages, torch.bfloat16, "k_pages")
    require_dtype(cu_seqlens, torch.int32, "cu_seqlens")
    if not (q.is_contiguous() and k_pages.stride(-1) == 1 and v_pages.stride() == k_pages.stride()
            and block_tables.stride(-1) == 1):
        raise ValueError("q, block_tables and the page rows must be contiguous")
    strides = (k_pages.stride(1), k_pages.stride(2), k_pages.stride(0))
    return _launch(q, k_pages, v_pages, total_pages, page_size, strides, num_kv_heads,
                   block_tables, cu_seqlens, None, max_seqlen_bucket, 1.0 / math.sqrt(head_dim))


def paged_prefill(q: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                  cu_seqlens_q: torch.Tensor, context_lens: torch.Tensor | None = None,
                  max_seqlen_q: int = 0, scale: float | None = None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Prefill attention on the engine cache (2, nb, bs, Hkv, D); keys of the
    new tokens must already be in the cache (K3 runs first)."""
    require_dtype(q, torch.bfloat16, "q")
    require_dtype(kv_cache, torch.bfloat16, "kv_cache")
    require_dtype(block_tables, torch.int32, "block_tables")
    require_dtype(cu_seqlens_q, torch.int32, "cu_seqlens_q")
    if context_lens is not None:
        require_dtype(context_lens, torch.int32, "context_lens")
        if context_lens.shape != (cu_seqlens_q.shape[0] - 1,):
            raise ValueError("context_lens must have shape [num_seqs]")
    if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
        raise ValueError("kv_cache must have shape (2, num_blocks, block_size, Hkv, D)")
    if block_tables.shape[0] != cu_seqlens_q.shape[0] - 1:
        raise ValueError("block_tables must have one row per sequence")
    if not q.is_contiguous() or block_tables.stride(-1) != 1:
        raise ValueError("q and block_tables must be contiguous")
    k, v = kv_cache[0], kv_cache[1]
    nb, bs, hkv, D = k.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    strides = (k.stride(0), k.stride(1), k.stride(2))
    return _launch(q, k, v, nb, bs, strides, hkv, block_tables, cu_seqlens_q, context_lens,
                   max_seqlen_q, scale, out)


def paged_attention_mixed(q: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                          cu_seqlens_q: torch.Tensor, context_lens: torch.Tensor,
                          num_decode: int, max_seqlen_q: int, scale: float | None = None,
                          out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                          reuse_plan: bool = False, max_chunks: int = 0) -> torch.Tensor:
    """Attention of a chunked-prefill step in ONE kernel launch (plus the
    decode plan and combine): sequences [0, num_decode) are decode rows (q row
    b = sequence b), the rest prompt chunks after a cached prefix; rows past
    cu_seqlens_q[-1] (padding) come out 0. Keys of the new tokens must already
    be in the cache. reuse_plan: keep the decode split
    plan of the previous call on this stream (same decode rows)."""
    from ._util import workspace as scratch
    require_dtype(q, torch.bfloat16, "q")
    require_dtype(kv_cache, torch.bfloat16, "kv_cache")
    for name, t in (("block_tables", block_tables), ("cu_seqlens_q", cu_seqlens_q),
                    ("context_lens", context_lens)):
        require_dtype(t, torch.int32, name)
    S = cu_seqlens_q.shape[0] - 1
    if block_tables.shape[0] != S or context_lens.shape != (S,):
        raise ValueError("block_tables and context_lens need one row per sequence")
    if not 0 <= num_decode <= S:
        raise ValueError("num_decode must lie in [0, num_seqs]")
    if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
        raise ValueError("kv_cache must have shape (2, num_blocks, block_size, Hkv, D)")
    if not q.is_contiguous() or block_tables.stride(-1) != 1:
        raise ValueError("q and block_tables must be contiguous")
    dev = require_cuda(q, kv_cache, block_tables, cu_seqlens_q, context_lens)
    T, Hq, D = q.shape
    k, v = kv_cache[0], kv_cache[1]
    nb, bs, hkv, _ = k.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    ws_bytes = _native.load().vj_paged_attention_mixed_workspace_size(num_decode, Hq, D,
                                                                      max_chunks)
    if workspace is None:
        workspace = scratch(dev, max(ws_bytes, 16), "decode")
    elif workspace.dtype != torch.uint8 or workspace.numel() < ws_bytes:
        raise ValueError(f"decode workspace must be uint8 with >= {ws_bytes} bytes")
    _native.call("vj_paged_attention_mixed", q.data_ptr(), k.data_ptr(), v.data_ptr(),
                 block_tables.data_ptr(), cu_seqlens_q.data_ptr(), context_lens.data_ptr(),
                 out.data_ptr(), T, S, int(num_decode), Hq, hkv, D, nb, bs,
                 block_tables.shape[1], block_tables.stride(0), k.stride(0), k.stride(1),
                 k.stride(2), int(max_seqlen_q), float(scale), int(max_chunks),
                 0 if reuse_plan else 1, workspace.data_ptr(), workspace.numel(),
                 _err_flag(dev).data_ptr(), stream_ptr(dev))
    return out
