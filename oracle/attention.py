"""Oracle for paged decode / prefill attention (test infrastructure only).

Semantics follow the reference's own reference implementations:
  vllm/kernels/decode_paged_attention.py:400-463  paged_attention_reference:
      fp32 logits q.k, length mask, softmax, fp32 PV, cast to q.dtype
  vllm/kernels/prefill_paged_attention.py:456-505 prefill_paged_attention_reference:
      dense causal softmax per sequence, padded tokens (slot < 0) -> 0
Both are gathered here through block tables (pages of the KV pool) instead of
contiguous K/V, and prefill is generalised to a cached prefix: new token i of
a sequence with prefix p sits at position p+i and attends to keys [0, p+i].
Accumulation is fp32 with inputs rounded to bf16, outputs rounded to bf16.
"""
from __future__ import annotations

import numpy as np

from .bf16 import bf16


def gather_pages(cache: np.ndarray, block_table: np.ndarray, length: int) -> np.ndarray:
    """cache [nb, bs, Hkv, D]; entries < 0 read block 0 (safe_block_tables,
    vllm/model/qwen3.py:198-199). Returns [length, Hkv, D] float32."""
    bs = cache.shape[1]
    npages = (length + bs - 1) // bs
    blocks = np.asarray(block_table[:npages], dtype=np.int64)
    blocks = np.where(blocks >= 0, blocks, 0)
    kv = cache[blocks].reshape(npages * bs, *cache.shape[2:])
    return np.asarray(kv[:length], np.float32)


def decode_attention(q, k_cache, v_cache, block_tables, context_lens, scale):
    """q [B, Hq, D] -> out [B, Hq, D] (bf16-valued float32)."""
    q = np.asarray(q, np.float32)
    B, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    g = Hq // Hkv
    out = np.zeros((B, Hq, D), np.float32)
    for b in range(B):
        L = int(context_lens[b])
        if L <= 0:
            continue
        k = gather_pages(k_cache, block_tables[b], L)      # [L, Hkv, D]
        v = gather_pages(v_cache, block_tables[b], L)
        qh = q[b].reshape(Hkv, g, D)
        s = np.matmul(qh, k.transpose(1, 2, 0)) * np.float32(scale)     # [Hkv, g, L]
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s, dtype=np.float32)
        p /= p.sum(axis=-1, keepdims=True)
        o = np.matmul(p, v.transpose(1, 0, 2))                          # [Hkv, g, D]
        out[b] = o.reshape(Hq, D)
    return bf16(out)


def prefill_attention(q, k_cache, v_cache, block_tables, cu_seqlens_q, seq_lens_k, scale,
                      num_seqs=None):
    """Varlen causal prefill over paged K/V.

    q [T, Hq, D]; sequence s owns q rows cu_seqlens_q[s]:cu_seqlens_q[s+1]
    (n_s new tokens) and has seq_lens_k[s] = prefix_s + n_s keys in the pool.
    Rows past cu_seqlens_q[num_seqs] (bucket padding) are 0."""
    q = np.asarray(q, np.float32)
    T, Hq, D = q.shape
    Hkv = k_cache.shape[2]
    g = Hq // Hkv
    out = np.zeros((T, Hq, D), np.float32)
    S = len(cu_seqlens_q) - 1 if num_seqs is None else num_seqs
    for s_ in range(S):
        q0, q1 = int(cu_seqlens_q[s_]), int(cu_seqlens_q[s_ + 1])
        n = q1 - q0
        if n <= 0:
            continue
        Lk = int(seq_lens_k[s_])
        p0 = Lk - n
        k = gather_pages(k_cache, block_tables[s_], Lk)
        v = gather_pages(v_cache, block_tables[s_], Lk)
        qs = q[q0:q1].reshape(n, Hkv, g, D).transpose(1, 2, 0, 3)      # [Hkv, g, n, D]
        kt = np.ascontiguousarray(k.transpose(1, 2, 0))                 # [Hkv, D, Lk]
        vt = np.ascontiguousarray(v.transpose(1, 0, 2))                 # [Hkv, Lk, D]
        sc = np.matmul(qs, kt[:, None]) * np.float32(scale)             # [Hkv, g, n, Lk]
        qpos = p0 + np.arange(n)
        mask = np.arange(Lk)[None, :] <= qpos[:, None]                  # [n, Lk]
        sc = np.where(mask[None, None], sc, -np.inf)
        sc = sc - sc.max(axis=-1, keepdims=True)
        p = np.exp(sc, dtype=np.float32)
        p /= p.sum(axis=-1, keepdims=True)
        o = np.matmul(p, vt[:, None])                                   # [Hkv, g, n, D]
        out[q0:q1] = o.transpose(2, 0, 1, 3).reshape(n, Hq, D)
    return bf16(out)
