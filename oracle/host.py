"""Oracle for the model runner's batch packing (test infrastructure only).

Restates vllm/src/model_runner.py of vllm-jax:
  :185-188  _bucket_size: next power of two (1 for values <= 1)
  :204-214  pad_block_tables: rows padded with -1 to max_blocks_per_seq,
            batch padded with all -1 rows
  :217-266  prepare_prefill: every token of every request (prompt +
            completions), positions 0..len-1, slot = block[t // bs] * bs
            + t % bs; tokens padded to the bucket with (0, 0, -1); cu_seqlens
            padded to max_num_seqs + 1 by repeating the total;
            max_seqlen_bucket = bucket(max len)
  :268-301  prepare_decode: last token at position len-1, context len, slot
            in the LAST allocated block at offset (len-1) % bs; batch padded
            to a power of two with (0, 0, ctx 0, slot -1)
Inputs are plain lists: per request its token ids and block ids.
"""
from __future__ import annotations

import numpy as np


def bucket_size(value: int) -> int:
    return 1 if value <= 1 else 1 << (value - 1).bit_length()


def pad_block_tables(tables: list[list[int]], target_batch: int, width: int) -> np.ndarray:
    out = np.full((target_batch, width), -1, np.int32)
    for i, t in enumerate(tables):
        out[i, :len(t)] = t
    return out


def prepare_prefill(tokens: list[list[int]], blocks: list[list[int]], block_size: int,
                    max_num_seqs: int, max_blocks_per_seq: int) -> dict:
    ids, pos, slots, lens = [], [], [], []
    for tok, blk in zip(tokens, blocks):
        n = len(tok)
        lens.append(n)
        ids.extend(tok)
        pos.extend(range(n))
        slots.extend(blk[t // block_size] * block_size + t % block_size for t in range(n))
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    total = len(ids)
    bucket = bucket_size(total)
    pad = bucket - total
    ids += [0] * pad
    pos += [0] * pad
    slots += [-1] * pad
    cu += [cu[-1]] * (max_num_seqs + 1 - len(cu))
    return {"input_ids": np.asarray(ids, np.int32), "positions": np.asarray(pos, np.int32),
            "slot_mapping": np.asarray(slots, np.int32),
            "block_tables": pad_block_tables(blocks, max_num_seqs, max_blocks_per_seq),
            "cu_seqlens_q": np.asarray(cu, np.int32), "cu_seqlens_k": np.asarray(cu, np.int32),
            "max_seqlen_q": max(lens), "max_seqlen_k": max(lens),
            "max_seqlen_bucket": bucket_size(max(lens))}


def prepare_decode(tokens: list[list[int]], blocks: list[list[int]], block_size: int,
                   max_blocks_per_seq: int, last_block_slot: bool = True) -> dict:
    ids, pos, ctx, slots = [], [], [], []
    for tok, blk in zip(tokens, blocks):
        n = len(tok)
        ids.append(tok[-1])
        pos.append(n - 1)
        ctx.append(n)
        b = blk[-1] if last_block_slot else blk[(n - 1) // block_size]
        slots.append(b * block_size + (n - 1) % block_size)
    bucket = bucket_size(len(ids))
    pad = bucket - len(ids)
    ids += [0] * pad
    pos += [0] * pad
    ctx += [0] * pad
    slots += [-1] * pad
    return {"input_ids": np.asarray(ids, np.int32), "positions": np.asarray(pos, np.int32),
            "slot_mapping": np.asarray(slots, np.int32),
            "block_tables": pad_block_tables(blocks, bucket, max_blocks_per_seq),
            "context_lens": np.asarray(ctx, np.int32)}


def prepare_ranges(tokens: list[list[int]], blocks: list[list[int]], starts: list[int],
                   ns: list[int], block_size: int, bucket_batch: int,
                   max_blocks_per_seq: int) -> dict:
    """Chunked-prefill packing (no counterpart in the reference, which always
    prefills from position 0): sequence s contributes tokens [starts[s],
    starts[s] + ns[s]) at those positions with position-addressed slots;
    context_lens = start + n; padding like prepare_prefill (tokens to a power
    of two with (0, 0, -1), cu_seqlens repeated, context_lens 0)."""
    ids, pos, slots, cu = [], [], [], [0]
    for tok, blk, a, n in zip(tokens, blocks, starts, ns):
        for t in range(a, a + n):
            ids.append(tok[t])
            pos.append(t)
            slots.append(blk[t // block_size] * block_size + t % block_size)
        cu.append(cu[-1] + n)
    total = len(ids)
    pad = bucket_size(total) - total
    ids += [0] * pad
    pos += [0] * pad
    slots += [-1] * pad
    cu += [cu[-1]] * (bucket_batch + 1 - len(cu))
    ctx = [a + n for a, n in zip(starts, ns)]
    ctx += [0] * (bucket_batch - len(ctx))
    return {"input_ids": np.asarray(ids, np.int32), "positions": np.asarray(pos, np.int32),
            "slot_mapping": np.asarray(slots, np.int32),
            "block_tables": pad_block_tables(blocks, bucket_batch, max_blocks_per_seq),
            "cu_seqlens_q": np.asarray(cu, np.int32), "context_lens": np.asarray(ctx, np.int32)}
