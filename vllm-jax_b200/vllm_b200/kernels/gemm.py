"""Decode-step projections with fused epilogues (libvjattn, tcgen05), torch-facing.

  decode_gemm(x, w)                  x @ w.T                       (vj_decode_gemm, PLAIN)
  decode_gemm(x, w_gate_up, "swiglu")  silu(x @ Wg.T) * (x @ Wu.T)  (vj_decode_gemm, SWIGLU)
  qkv_gemm_kv_store(x, w_qkv, ...)   the qkv projection followed by K3 (q/k
                                     RMSNorm, RoPE, q scaling, KV-slot store)

They replace, in vllm-jax, the decode-step dataflow of vllm/model/qwen3.py:
:286-296 (qkv projection -> q_norm/k_norm -> apply_rope) with :105-111
(_update_kv_cache), and :337-341 (gate/up projections -> SiLU * up). Built for
decode batches; prefill-sized row counts belong to cuBLAS + the separate K3 /
SiLU kernels, whose outputs these reproduce (bit for bit given equal
projections; the projections themselves are fp32 sums in another order).
"""
from __future__ import annotations

import torch

from .. import _native
from ._util import ptr, require_cuda, require_dtype, stream_ptr, workspace
from .kv_store import _QSCALE, _cache_views, rope_table

_MODES = {"plain": _native.VJ_GEMM_PLAIN, "swiglu": _native.VJ_GEMM_SWIGLU}


class TiledWeight:
    """A weight [n, k] packed by vj_pack_weight_tiles for `mode` ("plain", or
    "swiglu" for [gate; up]): contiguous 16 KB (128 rows x 64 K) blocks in
    the shared-memory swizzle order, so every pipeline stage of the GEMM is
    one bulk copy. Same results as the row-major weight, faster stream."""

    def __init__(self, w: torch.Tensor, mode: str = "plain"):
        require_cuda(w)
        require_dtype(w, torch.bfloat16, "w")
        if mode not in _MODES:
            raise ValueError(f"mode must be 'plain' or 'swiglu'; got {mode!r}")
        if w.dim() != 2 or not w.is_contiguous():
            raise ValueError("w must be a contiguous [n, k] tensor")
        self.shape = tuple(w.shape)
        self.mode = mode
        self.data = torch.empty_like(w)
        _native.call("vj_pack_weight_tiles", w.data_ptr(), self.data.data_ptr(), w.shape[0],
                     w.shape[1], _MODES[mode], stream_ptr(w.device))

    @property
    def device(self):
        return self.data.device


def _weight(w, mode: str):
    """(pointer, layout, n, k) of a row-major tensor or a TiledWeight."""
    if isinstance(w, TiledWeight):
        if w.mode != mode:
            raise ValueError(f"weight packed for {w.mode!r}, used as {mode!r}")
        return w.data.data_ptr(), _native.VJ_WEIGHTS_TILED, w.shape[0], w.shape[1]
    require_dtype(w, torch.bfloat16, "w")
    if w.dim() != 2 or not w.is_contiguous():
        raise ValueError("w must be a contiguous [n, k] tensor")
    return w.data_ptr(), _native.VJ_WEIGHTS_ROW_MAJOR, w.shape[0], w.shape[1]


def gemm_workspace_bytes(rows: int, n: int, k: int, mode: str = "plain", splits: int = 0) -> int:
    """Workspace of one call (zero-filled at allocation, reusable across calls)."""
    return int(_native.load().vj_decode_gemm_workspace_size(rows, n, k, _MODES[mode], splits))


def _workspace(dev, nbytes: int, ws: torch.Tensor | None) -> torch.Tensor:
    if ws is None:
        return workspace(dev, nbytes, "gemm", zeroed=True)
    if ws.dtype != torch.uint8 or ws.numel() < nbytes or ws.data_ptr() % 256:
        raise ValueError(f"gemm workspace must be uint8, 256-byte aligned, >= {nbytes} bytes")
    return ws


def _check_x(x: torch.Tensor, k: int) -> None:
    require_dtype(x, torch.bfloat16, "x")
    if x.dim() != 2 or x.shape[1] != k or x.stride(1) != 1:
        raise ValueError(f"x must be [rows, {k}] with contiguous rows; got {tuple(x.shape)}")


def decode_gemm(x: torch.Tensor, w: torch.Tensor, mode: str = "plain",
                out: torch.Tensor | None = None, splits: int = 0,
                ws: torch.Tensor | None = None,
                error_flag: torch.Tensor | None = None) -> torch.Tensor:
    """x [rows, k] bf16, w [n, k] bf16 (contiguous, or a TiledWeight of it).
    "plain": out [rows, n] =
    x @ w.T; "swiglu": w = [gate; up] (n = 2 I) and out [rows, I] =
    bf16(bf16(silu(bf16(x @ gate.T))) * bf16(x @ up.T)). `out` may be a row
    slice of a wider buffer (row stride a multiple of 8)."""
    if mode not in _MODES:
        raise ValueError(f"mode must be 'plain' or 'swiglu'; got {mode!r}")
    dev = require_cuda(x, w.data if isinstance(w, TiledWeight) else w)
    wp, layout, n, k = _weight(w, mode)
    _check_x(x, k)
    rows = x.shape[0]
    cols = n // 2 if mode == "swiglu" else n
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.bfloat16, device=dev)
    elif out.shape != (rows, cols) or out.stride(1) != 1 or out.dtype != torch.bfloat16:
        raise ValueError(f"out must be bf16 [{rows}, {cols}] with contiguous rows")
    if rows == 0:
        return out
    nbytes = gemm_workspace_bytes(rows, n, k, mode, splits)
    buf = _workspace(dev, nbytes, ws)
    _native.call("vj_decode_gemm", x.data_ptr(), x.stride(0), wp, layout, out.data_ptr(),
                 out.stride(0), rows, n, k, _MODES[mode], splits, buf.data_ptr(), buf.numel(),
                 ptr(error_flag), stream_ptr(dev))
    return out


def qkv_gemm_kv_store(x: torch.Tensor, w_qkv: torch.Tensor, kv_cache: torch.Tensor,
                      slot_mapping: torch.Tensor, positions: torch.Tensor,
                      q_norm_weight: torch.Tensor, k_norm_weight: torch.Tensor,
                      num_q_heads: int, *, eps: float = 1e-6, rope_theta: float = 1e6,
                      q_scale: str | None = None, table: torch.Tensor | None = None,
                      norm: bool = True, rope: bool = True, wrap_negative_slots: bool = True,
                      q_out: torch.Tensor | None = None, splits: int = 0,
                      ws: torch.Tensor | None = None,
                      error_flag: torch.Tensor | None = None) -> torch.Tensor:
    """One launch: qkv = x @ w_qkv.T (w_qkv = [Wq; Wk; Wv], or a TiledWeight
    of it packed for "plain"), then exactly
    kv_store_qknorm_rope(q, k, v, kv_cache, slot_mapping, positions, ...) on
    the bf16 projections. Returns q_out [rows, Hq, 128]."""
    dev = require_cuda(x, w_qkv.data if isinstance(w_qkv, TiledWeight) else w_qkv, kv_cache,
                       slot_mapping, positions)
    kc, vc, nb, bs, (sb, st, sh) = _cache_views(kv_cache)
    wp, layout, n, k = _weight(w_qkv, "plain")
    _check_x(x, k)
    D = kc.shape[3]
    Hkv = kc.shape[2]
    if n != (num_q_heads + 2 * Hkv) * D:
        raise ValueError(f"w_qkv has {n} rows; expected (Hq + 2 Hkv) * D = "
                         f"{(num_q_heads + 2 * Hkv) * D}")
    rows = x.shape[0]
    require_dtype(slot_mapping, torch.int32, "slot_mapping")
    if slot_mapping.shape != (rows,):
        raise ValueError("slot_mapping must have shape [num_tokens]")
    flags = 0
    if norm:
        flags |= _native.VJ_KV_NORM
    if rope:
        flags |= _native.VJ_KV_ROPE
        require_dtype(positions, torch.int32, "positions")
        if table is None:
            table = rope_table(dev, rope_theta)
    if wrap_negative_slots:
        flags |= _native.VJ_KV_WRAP_NEGATIVE
    if q_scale not in _QSCALE:
        raise ValueError(f"q_scale must be None, 'div' or 'mul'; got {q_scale!r}")
    flags |= _QSCALE[q_scale]
    if q_out is None:
        q_out = torch.empty((rows, num_q_heads, D), dtype=torch.bfloat16, device=dev)
    if rows == 0:
        return q_out
    tab_len = table.numel() // 64 if (rope and table is not None) else 0
    nbytes = gemm_workspace_bytes(rows, n, k, "plain", splits)
    buf = _workspace(dev, nbytes, ws)
    _native.call("vj_qkv_gemm_kv_store", x.data_ptr(), x.stride(0), wp, layout,
                 ptr(q_norm_weight if norm else None), ptr(k_norm_weight if norm else None),
                 positions.data_ptr(), slot_mapping.data_ptr(), q_out.data_ptr(),
                 kc.data_ptr(), vc.data_ptr(), rows, k, num_q_heads, Hkv, D, nb, bs, sb, st, sh,
                 ptr(table) if tab_len else None, tab_len, float(eps), float(rope_theta), flags,
                 splits, buf.data_ptr(), buf.numel(), ptr(error_flag), stream_ptr(dev))
    return q_out
