"""Oracle for K3: q/k RMSNorm + RoPE + KV-slot scatter (test infrastructure).

Follows vllm-jax vllm/model/qwen3.py:
  :286-296  q = q_norm(q_proj(x)); q = apply_rope(q, ...); same for k
  :59-78    apply_rope: positions.astype(bf16); inv_freq in bf16; pairs
            (x[0::2], x[1::2]); stack((x1*cos - x2*sin, x1*sin + x2*cos), -1)
  :105-111  _update_kv_cache: flat_cache.at[0|1, slot].set(k|v, mode="drop")
RMSNorm follows flax nnx.RMSNorm (flax 0.12.2, call sites qwen3.py:248-268):
fp32 statistics, y = bf16(x * (rsqrt(mean(x^2) + eps) * scale)). rmsnorm()
(hidden-size rows) takes the sum of squares exactly (fp64, then fp32);
rmsnorm_head() (the 128-dim q/k rows of K3) sums in fp32 in K3's order.

Every step below is one IEEE fp32 (or fp64 where stated) operation followed
by a bf16 round-to-nearest-even wherever jnp's result dtype is bf16, so the
CUDA kernel can be compared bit for bit.
"""
from __future__ import annotations

import numpy as np

from .bf16 import bf16, bf16_from_f64


def rope_inv_freq(rope_theta: float, head_dim: int = 128) -> np.ndarray:
    """1.0 / (rope_theta ** (arange(0, D, 2, bf16) / D)) in bf16 (qwen3.py:63-64).

    rope_theta is a weakly typed Python float, so jnp casts it to bf16 before
    the power (1e6 -> 999424)."""
    theta = float(bf16_from_f64(np.array([rope_theta], np.float64))[0])
    e = np.arange(0, head_dim, 2, dtype=np.float64) / head_dim   # exact in bf16
    p = bf16_from_f64(np.power(theta, e))
    return bf16_from_f64(1.0 / p.astype(np.float64))


def rope_cos_sin(positions: np.ndarray, rope_theta: float, head_dim: int = 128):
    """bf16 cos/sin tables [T, D/2] (qwen3.py:62-67); trig in fp64, one bf16 rounding."""
    pos = bf16(np.asarray(positions, dtype=np.int64).astype(np.float32))
    inv = rope_inv_freq(rope_theta, head_dim)
    freqs = bf16(pos[:, None] * inv[None, :])          # einsum("t,d->td") in bf16
    f64 = freqs.astype(np.float64)
    return bf16_from_f64(np.cos(f64)), bf16_from_f64(np.sin(f64))


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """flax RMSNorm over the last axis; x, w bf16-valued float32 -> bf16-valued float32."""
    x = np.asarray(x, np.float32)
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    ms = np.float32(ss.astype(np.float32)) / np.float32(x.shape[-1])
    inv = np.float32(1.0) / np.sqrt((ms + np.float32(eps)).astype(np.float32))
    mul = (inv.astype(np.float32) * np.asarray(w, np.float32)).astype(np.float32)
    return bf16((x * mul).astype(np.float32))


def rmsnorm_head(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """flax RMSNorm over a 128-dim head row with the sum of squares taken in
    fp32 in the order vj_kv_store_qknorm_rope uses: lane l of 8 owns dims
    [8l, 8l+8) and [64+8l, 64+8l+8), sums the even dims and the odd dims of
    those 16 in that order, adds the two, then lanes combine by a butterfly
    (xor 4, 2, 1). bf16 squares are exact in fp32, so only the order of the
    additions is a choice (XLA's reduction order is not observable here)."""
    x = np.asarray(x, np.float32)
    D = x.shape[-1]
    halves = (x * x).reshape(*x.shape[:-1], 2, 8, D // 16)       # [half, lane, 8 dims]
    sq = np.swapaxes(halves, -3, -2).reshape(*x.shape[:-1], 8, D // 8)   # [lane, 16 dims]
    se = sq[..., 0]
    so = sq[..., 1]
    for j in range(1, D // 16):
        se = (se + sq[..., 2 * j]).astype(np.float32)
        so = (so + sq[..., 2 * j + 1]).astype(np.float32)
    lane = (se + so).astype(np.float32)
    idx = np.arange(8)
    for o in (4, 2, 1):
        lane = (lane + lane[..., idx ^ o]).astype(np.float32)
    ss = lane[..., :1]
    ms = (ss * np.float32(1.0 / D)).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt((ms + np.float32(eps)).astype(np.float32))).astype(np.float32)
    mul = (inv * np.asarray(w, np.float32)).astype(np.float32)
    return bf16((x * mul).astype(np.float32))


def scale_q(q: np.ndarray, mode: str | None) -> np.ndarray:
    """The reference's bf16 q scalings: "div" = bf16(q / bf16(sqrt(D)))
    (decode, qwen3.py:207), "mul" = bf16(q * bf16(1/sqrt(D))) (prefill kernel,
    prefill_paged_attention.py:60); None leaves q unchanged."""
    if mode is None:
        return q
    D = q.shape[-1]
    if mode == "div":
        return bf16(q / np.float32(bf16(np.float32(np.sqrt(np.float32(D))))))
    if mode == "mul":
        return bf16(q * np.float32(bf16(np.float32(1.0 / np.sqrt(D)))))
    raise ValueError(f"unknown q scaling {mode!r}")


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """Interleaved-pair RoPE of qwen3.py:69-75, bf16 after every op. x [T, H, D]."""
    x1 = x[..., 0::2]
    x2 = x[..., 1::2]
    c = cos[:, None, :]
    s = sin[:, None, :]
    a = bf16(x1 * c)
    b = bf16(x2 * s)
    d = bf16(x1 * s)
    e = bf16(x2 * c)
    out = np.empty_like(x)
    out[..., 0::2] = bf16(a - b)
    out[..., 1::2] = bf16(d + e)
    return out


def update_kv_cache(k_cache: np.ndarray, v_cache: np.ndarray, slot_mapping: np.ndarray,
                    k: np.ndarray, v: np.ndarray, wrap_negative: bool = True) -> None:
    """In-place _update_kv_cache (qwen3.py:105-111).

    k_cache/v_cache: [num_blocks, block_size, Hkv, D]. JAX's .at[] normalises
    negative indices (slot -1 -> last slot) before mode="drop" drops the rest;
    duplicate slots keep the last write (all duplicates in the reference are
    identical padded rows)."""
    nb, bs = k_cache.shape[:2]
    n = nb * bs
    fk = k_cache.reshape(n, *k_cache.shape[2:])
    fv = v_cache.reshape(n, *v_cache.shape[2:])
    for t, s in enumerate(np.asarray(slot_mapping, dtype=np.int64)):
        if s < 0 and wrap_negative:
            s += n
        if 0 <= s < n:
            fk[s] = k[t]
            fv[s] = v[t]


def kv_store_qknorm_rope(q, k, v, q_norm_w, k_norm_w, positions, slot_mapping,
                         k_cache, v_cache, eps=1e-6, rope_theta=1e6,
                         norm=True, rope=True, wrap_negative=True, q_scale=None):
    """Oracle of vj_kv_store_qknorm_rope. Returns (q_out, k_out); updates caches.
    q_scale: None, "div" (VJ_KV_QSCALE_DIV_SQRT_D) or "mul" (VJ_KV_QSCALE_MUL_RSQRT_D)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    if norm:
        q = rmsnorm_head(q, q_norm_w, eps)
        k = rmsnorm_head(k, k_norm_w, eps)
    if rope:
        c, s = rope_cos_sin(positions, rope_theta, k.shape[-1])
        q = apply_rope(q, c, s)
        k = apply_rope(k, c, s)
    q = scale_q(q, q_scale)
    update_kv_cache(k_cache, v_cache, slot_mapping, k, np.asarray(v, np.float32),
                    wrap_negative)
    return q, k
