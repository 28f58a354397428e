"""Split-KV paged decode attention on sm_100a (K2), torch-facing.

`decode_paged_attention` keeps the signature, argument meaning and ValueError
checks of vllm-jax's vllm/kernels/decode_paged_attention.py:300-397
(k_pages/v_pages in the Pallas page layout [Hkv, total_pages, page_size, D],
q already scaled by the caller, no scale inside). Tuning knobs of the Pallas
kernel (block_h, pages_per_compute_block, k_splits, num_warps, num_stages)
are accepted for compatibility and ignored: the CUDA kernel sizes its split
from the real context lengths and the SM count.

`paged_decode` is the engine's entry on the native cache layout
(2, num_blocks, block_size, Hkv, D) with the softmax scale applied in fp32.
"""
from __future__ import annotations

import math

import torch

from .. import _native
from ._util import require_cuda, require_dtype, stream_ptr, workspace

DEFAULT_MASK_VALUE = -0.7 * float(torch.finfo(torch.float32).max)


def _launch(q, k_base, v_base, nb, bs, strides, block_tables, lengths, scale, out=None,
            max_chunks: int = 0, ws: torch.Tensor | None = None, reuse_plan: bool = False):
    dev = require_cuda(q, k_base, v_base, block_tables, lengths)
    B, Hq, D = q.shape
    Hkv = strides[3]
    if out is None:
        out = torch.empty_like(q)
    ws_bytes = _native.load().vj_paged_decode_workspace_size(B, Hq, D, max_chunks)
    if ws is None:
        ws = workspace(dev, ws_bytes, "decode")
    elif ws.numel() < ws_bytes or ws.dtype != torch.uint8:
        raise ValueError(f"decode workspace must be uint8 with >= {ws_bytes} bytes")
    _native.call("vj_paged_decode_planned" if reuse_plan else "vj_paged_decode",
                 q.data_ptr(), k_base.data_ptr(), v_base.data_ptr(),
                 block_tables.data_ptr(), lengths.data_ptr(), out.data_ptr(),
                 B, Hq, Hkv, D, nb, bs, block_tables.shape[1], block_tables.stride(0),
                 strides[0], strides[1], strides[2], float(scale), max_chunks,
                 ws.data_ptr(), ws.numel(), stream_ptr(dev))
    return out


def decode_paged_attention(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                           block_tables: torch.Tensor, lengths: torch.Tensor | None,
                           k_scales_pages=None, v_scales_pages=None, *, block_h: int = 16,
                           pages_per_compute_block: int = 8, k_splits: int = 16,
                           num_warps: int = 8, num_stages: int = 2, interpret: bool = False,
                           debug: bool = False, mask_value: float = DEFAULT_MASK_VALUE,
                           attn_logits_soft_cap: float | None = None) -> torch.Tensor:
    """Paged grouped query attention (decode_paged_attention.py:300-341).

    q [batch, num_heads, head_dim]; k_pages/v_pages [num_kv_heads,
    total_num_pages, page_size, head_dim]; block_tables int32 [batch,
    pages_per_sequence]; lengths int32 [batch]. Returns [batch, num_heads,
    head_dim]."""
    batch_size, num_heads, head_dim = q.shape
    num_kv_heads, total_pages, page_size, head_dim_k = k_pages.shape
    batch_size_paged_indices, _ = block_tables.shape
    if k_pages.shape != v_pages.shape:
        raise ValueError(f"k_pages and v_pages must have the same shape. Got {tuple(k_pages.shape)} "
                         f"and {tuple(v_pages.shape)}")
    if num_heads % num_kv_heads != 0:
        raise ValueError("Number of Q heads must be divisible by number of KV heads. Got "
                         f"{num_heads} and {num_kv_heads}.")
    if head_dim_k != head_dim:
        raise ValueError(f"head_dim of Q must be the same as that of K/V. Got {head_dim} and "
                         f"{head_dim_k}.")
    if batch_size_paged_indices != batch_size:
        raise ValueError("`block_tables` and `q` must have the same batch size")
    if lengths is None:
        raise NotImplementedError("lengths=None is not supported by the CUDA kernel")
    if tuple(lengths.shape) != (batch_size,):
        raise ValueError("`lengths` and `q` must have the same batch size")
    if lengths.dtype != torch.int32:
        raise ValueError(f"The dtype of `lengths` must be int32. Got {lengths.dtype}")
    if block_h % 16:
        raise ValueError(f"block_h must divisible by 16, but is {block_h}.")
    if k_scales_pages is not None or v_scales_pages is not None or attn_logits_soft_cap is not None:
        raise NotImplementedError("quantized pages and logit soft-cap are not implemented")
    if interpret:
        raise NotImplementedError("interpret=True (CPU) is not available: the B200 path has no "
                                  "CPU fallback")
    require_dtype(q, torch.bfloat16, "q")
    require_dtype(k_pages, torch.bfloat16, "k_pages")
    require_dtype(block_tables, torch.int32, "block_tables")
    if not (q.is_contiguous() and k_pages.stride(-1) == 1 and v_pages.stride() == k_pages.stride()
            and block_tables.stride(-1) == 1):
        raise ValueError("q, block_tables and the page rows must be contiguous")
    # page layout [Hkv, nb, ps, D]: (block, token, head) strides
    strides = (k_pages.stride(1), k_pages.stride(2), k_pages.stride(0), num_kv_heads)
    return _launch(q, k_pages, v_pages, total_pages, page_size, strides, block_tables, lengths,
                   1.0)


def paged_decode(q: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor,
                 context_lens: torch.Tensor, scale: float | None = None,
                 out: torch.Tensor | None = None, max_chunks: int = 0,
                 workspace: torch.Tensor | None = None,
                 reuse_plan: bool = False) -> torch.Tensor:
    """Decode attention straight from the engine cache (2, nb, bs, Hkv, D).
    `workspace` (uint8, decode_workspace_bytes(...) long) pins the split-KV
    scratch to a caller-owned buffer, as CUDA-graph replays need.
    `reuse_plan`: skip the planning launch; the workspace must hold the plan of
    the previous call with the same batch and lengths (the layers of one
    decode step)."""
    require_dtype(q, torch.bfloat16, "q")
    require_dtype(kv_cache, torch.bfloat16, "kv_cache")
    require_dtype(block_tables, torch.int32, "block_tables")
    require_dtype(context_lens, torch.int32, "context_lens")
    if kv_cache.dim() != 5 or kv_cache.shape[0] != 2:
        raise ValueError("kv_cache must have shape (2, num_blocks, block_size, Hkv, D)")
    if not q.is_contiguous() or block_tables.stride(-1) != 1:
        raise ValueError("q and block_tables must be contiguous")
    if block_tables.shape[0] != q.shape[0] or context_lens.shape != (q.shape[0],):
        raise ValueError("`block_tables`, `context_lens` and `q` must have the same batch size")
    k, v = kv_cache[0], kv_cache[1]
    nb, bs, Hkv, D = k.shape
    if D != q.shape[2] or q.shape[1] % Hkv:
        raise ValueError("q heads/head_dim do not match kv_cache")
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    strides = (k.stride(0), k.stride(1), k.stride(2), Hkv)
    if reuse_plan and workspace is None:
        raise ValueError("reuse_plan needs the caller's workspace")
    return _launch(q, k, v, nb, bs, strides, block_tables, context_lens, scale, out, max_chunks,
                   workspace, reuse_plan)


def decode_workspace_bytes(batch: int, num_q_heads: int, head_dim: int = 128,
                           max_chunks: int = 0) -> int:
    return int(_native.load().vj_paged_decode_workspace_size(batch, num_q_heads, head_dim,
                                                            max_chunks))
