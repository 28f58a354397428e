"""Deterministic inputs of the numeric golden fixtures (test infrastructure).

The fixtures under tests/golden/ store only the reference's OUTPUTS; their
inputs are regenerated here from a counter hash (splitmix64 in integer
arithmetic), so they are identical on every machine and numpy version and
need no stored bytes. Values are k / 128 for integers k in [-256, 256]:
exact in bf16, spread over [-2, 2].
"""
from __future__ import annotations

import numpy as np

from oracle.bf16 import bf16

_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(counter: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = counter.astype(np.uint64) * _GOLD + _GOLD
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def det_uint(n: int, seed: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        c = np.arange(n, dtype=np.uint64) + np.uint64(seed) * np.uint64(1 << 40)
    return splitmix64(c)


def det_bf16(shape, seed: int) -> np.ndarray:
    """float32 array of bf16-exact values k/128, k in [-256, 256]."""
    n = int(np.prod(shape))
    k = (det_uint(n, seed) >> np.uint64(20)) % np.uint64(513)
    v = (k.astype(np.int64) - 256).astype(np.float32) / np.float32(128.0)
    return bf16(v.reshape(shape))


def det_permutation(n: int, seed: int) -> np.ndarray:
    """A permutation of range(n) (argsort of hashed keys)."""
    return np.argsort(det_uint(n, seed), kind="stable").astype(np.int64)


# ---------------------------------------------------------------------------
# scenario inputs (shared by the generator and the tests)
# ---------------------------------------------------------------------------
ROPE_POSITIONS = [0, 1, 2, 3, 7, 15, 16, 31, 100, 255, 256, 257, 258, 300, 511, 512, 513, 1000,
                  1023, 1025, 2047, 2049, 4095, 4097, 8191, 8193, 12345, 16383, 16385, 20000,
                  24575, 30001, 32767, 32768, 32769, 40000, 50001, 65535, 65537, 70000, 100000,
                  131071, 131073, 200000, 262143, 300000, 500000, 1048575]


def rope_inputs():
    x = det_bf16((len(ROPE_POSITIONS), 3, 128), seed=11)
    return x, np.asarray(ROPE_POSITIONS, np.int32)


# _update_kv_cache: pool (2, 4 blocks, 16, 2 heads, 128); slots include -1
# and -3 (wrap to the pool's last slots), 64 and 200 (out of range: dropped)
# and -65 (still negative after one wrap: dropped)
KV_SLOTS = [0, 5, 17, 40, -1, -3, 64, 200, 33, -65, 12]


def kv_update_inputs():
    cache = det_bf16((2, 4, 16, 2, 128), seed=21)
    k = det_bf16((len(KV_SLOTS), 2, 128), seed=22)
    v = det_bf16((len(KV_SLOTS), 2, 128), seed=23)
    return cache, np.asarray(KV_SLOTS, np.int32), k, v


# Attention scenarios at the C1 head shape (Qwen3-0.6B: 16 q heads, 8 KV
# heads, head_dim 128, block_size 16, 128-block pool, 32-entry block tables).
C1_HEADS = dict(num_q_heads=16, num_kv_heads=8, head_dim=128, block_size=16, num_blocks=128,
                width=32)


def _tables(lengths, width, bs, seed, pool_blocks):
    """Distinct blocks per sequence from a permutation of the pool minus its
    last block (which slot -1 wraps into); -1 padding."""
    perm = [int(b) for b in det_permutation(pool_blocks - 1, seed)]
    bt = np.full((len(lengths), width), -1, np.int32)
    o = 0
    for i, L in enumerate(lengths):
        nblk = (L + bs - 1) // bs
        bt[i, :nblk] = perm[o:o + nblk]
        o += nblk
    return bt


DECODE_CTX = [18, 130, 301, 0]      # 3 sequences + one bucket-padding row (ctx 0, slot -1)


def decode_inputs():
    c = C1_HEADS
    B, Hq, Hkv, D, bs, nb, W = (len(DECODE_CTX), c["num_q_heads"], c["num_kv_heads"],
                                c["head_dim"], c["block_size"], c["num_blocks"], c["width"])
    kv_cache = det_bf16((2, nb, bs, Hkv, D), seed=31)
    bt = _tables(DECODE_CTX, W, bs, seed=32, pool_blocks=nb)
    q = det_bf16((B, Hq, D), seed=33)
    k = det_bf16((B, Hkv, D), seed=34)
    v = det_bf16((B, Hkv, D), seed=35)
    ctx = np.asarray(DECODE_CTX, np.int32)
    pos = np.maximum(ctx - 1, 0).astype(np.int32)
    slots = np.asarray([int(bt[i, (L - 1) // bs]) * bs + (L - 1) % bs if L > 0 else -1
                        for i, L in enumerate(DECODE_CTX)], np.int32)
    return dict(kv_cache=kv_cache, block_tables=bt, q=q, k=k, v=v, context_lens=ctx,
                positions=pos, slot_mapping=slots)


PREFILL_LENS = [17, 30, 45]         # packed, bucket-padded to 128 tokens, 4 sequence seats
PREFILL_BUCKET_T = 128
PREFILL_SEATS = 4


def prefill_inputs():
    c = C1_HEADS
    Hq, Hkv, D, bs, nb, W = (c["num_q_heads"], c["num_kv_heads"], c["head_dim"],
                             c["block_size"], c["num_blocks"], c["width"])
    T = PREFILL_BUCKET_T
    kv_cache = det_bf16((2, nb, bs, Hkv, D), seed=41)
    bt = np.full((PREFILL_SEATS, W), -1, np.int32)
    bt[:len(PREFILL_LENS)] = _tables(PREFILL_LENS, W, bs, seed=42, pool_blocks=nb)
    q = det_bf16((T, Hq, D), seed=43)
    k = det_bf16((T, Hkv, D), seed=44)
    v = det_bf16((T, Hkv, D), seed=45)
    pos = np.zeros(T, np.int32)
    slots = np.full(T, -1, np.int32)
    cu = [0]
    t = 0
    for i, L in enumerate(PREFILL_LENS):
        for j in range(L):
            pos[t] = j
            slots[t] = int(bt[i, j // bs]) * bs + j % bs
            t += 1
        cu.append(t)
    while len(cu) < PREFILL_SEATS + 1:
        cu.append(cu[-1])               # model_runner.py:243-245: repeat the last value
    # bucket-padding rows: identical (zero) q/k/v, so that their shared slot -1
    # (wrapped to the pool's last slot, which no sequence uses) gets one value
    q[t:] = 0.0
    k[t:] = 0.0
    v[t:] = 0.0
    cu = np.asarray(cu, np.int32)
    mx = max(PREFILL_LENS)
    bucket = 1 << (mx - 1).bit_length()
    return dict(kv_cache=kv_cache, block_tables=bt, q=q, k=k, v=v, positions=pos,
                slot_mapping=slots, cu_seqlens=cu, num_tokens=t, max_seqlen_bucket=bucket)
