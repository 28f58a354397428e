"""Fused residual-add + RMSNorm and SwiGLU activation (libvjattn), torch-facing."""
from __future__ import annotations

import torch

from .. import _native
from ._util import stream_ptr


def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
                residual: torch.Tensor | None = None):
    """Without residual: y = rmsnorm(x). With residual: r = x + residual (bf16),
    y = rmsnorm(r); returns (r, y). Rows are the leading dims, hidden the last."""
    H = x.shape[-1]
    rows = x.numel() // H
    y = torch.empty_like(x)
    r = torch.empty_like(x) if residual is not None else None
    _native.call("vj_add_rmsnorm", x.data_ptr(),
                 None if residual is None else residual.data_ptr(), weight.data_ptr(),
                 None if r is None else r.data_ptr(), y.data_ptr(), rows, H, float(eps),
                 stream_ptr(x.device))
    return y if residual is None else (r, y)


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """gate_up [T, 2I] -> bf16(bf16(silu(gate)) * up) [T, I]."""
    T, I2 = gate_up.shape
    out = torch.empty((T, I2 // 2), dtype=gate_up.dtype, device=gate_up.device)
    _native.call("vj_silu_mul", gate_up.data_ptr(), out.data_ptr(), T, I2 // 2,
                 stream_ptr(gate_up.device))
    return out
