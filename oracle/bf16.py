"""bf16 helpers for the oracle (test infrastructure only).

ml_dtypes.bfloat16 rounds float32 -> bf16 to nearest-even, the same rule as
XLA's convert and CUDA's __float2bfloat16_rn.
"""
from __future__ import annotations

import ml_dtypes
import numpy as np

BF16 = ml_dtypes.bfloat16


def bf16(x) -> np.ndarray:
    """float32 -> bf16 (RNE) -> float32."""
    return np.asarray(x, dtype=np.float32).astype(BF16).astype(np.float32)


def bf16_from_f64(x) -> np.ndarray:
    """float64 -> nearest bf16 in ONE rounding (no float32 detour), as float32."""
    b = np.ascontiguousarray(np.asarray(x, dtype=np.float64)).view(np.uint64)
    lsb = (b >> np.uint64(45)) & np.uint64(1)
    b = (b + np.uint64(0x00000FFFFFFFFFFF) + lsb) & ~np.uint64((1 << 45) - 1)
    return b.view(np.float64).astype(np.float32)


def to_bf16_array(x) -> np.ndarray:
    """Return an ml_dtypes.bfloat16 array (RNE from float32)."""
    return np.asarray(x, dtype=np.float32).astype(BF16)


def f32(x) -> np.ndarray:
    return np.asarray(x).astype(np.float32)
