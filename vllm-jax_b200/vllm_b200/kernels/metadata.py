"""Device-resident engine tables and the GPU metadata builder (K4), torch-facing.

`DeviceTables` holds, per request slot, the token ids and allocated block ids
on the GPU and applies host deltas with one small upload per step;
`build_prefill` / `build_decode` produce exactly the arrays of vllm-jax's
ModelRunner.prepare_prefill / prepare_decode (vllm/src/model_runner.py:204-301)
with vj_build_metadata; `argmax_append` is the greedy sampler
(vllm/sampler.py:13-15) that also appends the token on the device.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .. import _native
from ._util import stream_ptr


def bucket_size(value: int) -> int:
    """Next power of two (model_runner.py:185-188)."""
    return 1 if value <= 1 else 1 << (value - 1).bit_length()


@dataclass
class PrefillMeta:
    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    cu_seqlens_q: torch.Tensor
    max_seqlen_q: int
    max_seqlen_bucket: int
    seq_lens: torch.Tensor         # keys per sequence (== new tokens here)
    num_seqs: int
    num_tokens: int


@dataclass
class DecodeMeta:
    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    num_seqs: int


@dataclass
class RangesMeta:
    """Mixed batch: sequence s contributes positions [start_s, start_s + n_s)."""
    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor     # [bucket_batch, width]
    cu_seqlens_q: torch.Tensor     # [bucket_batch + 1]
    context_lens: torch.Tensor     # [bucket_batch] keys per sequence (start + n)
    num_seqs: int
    num_tokens: int
    max_new: int
    sample_rows: torch.Tensor      # packed row of each sampled sequence's last token
    sample_slots: torch.Tensor     # their token-table rows
    sample_lens: torch.Tensor      # and lengths (the sampled token is stored there)


class DeviceTables:
    """Token and block tables of every live request slot, kept on the GPU."""

    def __init__(self, max_slots: int, max_len: int, max_blocks: int, block_size: int,
                 device: torch.device):
        self.device = device
        self.max_slots, self.max_len, self.max_blocks = max_slots, max_len, max_blocks
        self.block_size = block_size
        self.tokens = torch.zeros((max_slots, max_len + 1), dtype=torch.int32, device=device)
        self.blocks = torch.zeros((max_slots, max_blocks), dtype=torch.int32, device=device)
        self.num_blocks = torch.zeros(max_slots, dtype=torch.int32, device=device)
        self.error = torch.zeros(1, dtype=torch.int32, device=device)
        self._last_extra = None
        # pinned upload buffers in a ring: a buffer is rewritten only after the
        # copy that last read it has completed (its event), so the host never
        # waits for the GPU to drain before preparing the next step
        self._ring = [torch.empty(1 << 14, dtype=torch.int32).pin_memory() for _ in range(8)]
        self._ring_events: list[torch.cuda.Event | None] = [None] * len(self._ring)
        self._ring_next = 0
        self._staging = torch.empty(1 << 16, dtype=torch.int32, device=device)

    def _upload(self, arr: np.ndarray) -> torch.Tensor:
        """Copy int32 words to the device staging buffer (stream-ordered: the
        copy lands after every kernel enqueued before it, so views returned by
        an earlier upload stay valid for the kernels enqueued in between)."""
        n = arr.size
        i = self._ring_next
        self._ring_next = (i + 1) % len(self._ring)
        ev = self._ring_events[i]
        if ev is not None:
            ev.synchronize()
        if n > self._ring[i].numel():
            self._ring[i] = torch.empty(2 * n, dtype=torch.int32).pin_memory()
        if n > self._staging.numel():
            self._staging = torch.empty(2 * n, dtype=torch.int32, device=self.device)
        buf = self._ring[i]
        buf[:n].numpy()[:] = arr
        stream = torch.cuda.current_stream(self.device)
        self._staging[:n].copy_(buf[:n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self._ring_events[i] = ev
        return self._staging[:n]

    def _scatter(self, rows: list[tuple[int, int, list[int]]], table: torch.Tensor,
                 row_len: torch.Tensor | None, max_cols: int) -> None:
        if not rows:
            return
        headers = np.zeros((len(rows), 4), np.int32)
        payload = []
        off = 0
        for i, (row, start, vals) in enumerate(rows):
            headers[i] = (row, start, len(vals), off)
            payload.extend(vals)
            off += len(vals)
        buf = self._upload(np.concatenate([headers.ravel(),
                                           np.asarray(payload, np.int32)]).astype(np.int32))
        h, p = buf[:headers.size], buf[headers.size:]
        _native.call("vj_scatter_rows", h.data_ptr(), p.data_ptr() if off else h.data_ptr(),
                     len(rows), table.data_ptr(), table.stride(0), max_cols,
                     None if row_len is None else row_len.data_ptr(), self.error.data_ptr(),
                     stream_ptr(self.device))

    def set_tokens(self, rows: list[tuple[int, int, list[int]]]) -> None:
        """rows of (slot, start column, token ids)."""
        self._scatter(rows, self.tokens, None, self.max_len + 1)

    def set_blocks(self, rows: list[tuple[int, list[int]]]) -> None:
        """rows of (slot, full block list); the slot's block count becomes len(list)."""
        self._scatter([(slot, 0, blk) for slot, blk in rows], self.blocks, self.num_blocks,
                      self.max_blocks)

    def _lists(self, slots, lens, extra: np.ndarray | None = None):
        parts = [np.asarray(slots, np.int32), np.asarray(lens, np.int32)]
        if extra is not None:
            parts.append(np.asarray(extra).view(np.int32).ravel())
        arr = self._upload(np.concatenate(parts))
        n = len(slots)
        self._last = (arr[:n], arr[n:2 * n])
        self._last_extra = arr[2 * n:] if extra is not None else None
        return self._last

    def last_extra(self) -> torch.Tensor | None:
        """Device copy of the `extra` words of the latest build_decode call."""
        return self._last_extra

    def last_lists(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Device (slots, lens) of the latest build_* call; valid until the next upload."""
        return self._last

    def build_prefill(self, slots: list[int], lens: list[int], max_num_seqs: int,
                      width: int) -> PrefillMeta:
        S = len(slots)
        total = int(sum(lens))
        bt = bucket_size(total)
        d_slots, d_lens = self._lists(slots, lens)
        dev = self.device
        ids = torch.empty(bt, dtype=torch.int32, device=dev)
        pos = torch.empty_like(ids)
        sm = torch.empty_like(ids)
        tables = torch.empty((max_num_seqs, width), dtype=torch.int32, device=dev)
        cu = torch.empty(max_num_seqs + 1, dtype=torch.int32, device=dev)
        _native.call("vj_build_metadata", _native.VJ_META_PREFILL, d_slots.data_ptr(), None,
                     d_lens.data_ptr(), S, self.tokens.data_ptr(), self.tokens.stride(0),
                     self.blocks.data_ptr(), self.num_blocks.data_ptr(), self.blocks.stride(0),
                     self.block_size, width, bt, max_num_seqs, 0, ids.data_ptr(),
                     pos.data_ptr(), sm.data_ptr(), tables.data_ptr(), cu.data_ptr(), None,
                     self.error.data_ptr(), stream_ptr(dev))
        return PrefillMeta(ids, pos, sm, tables, cu, max(lens), bucket_size(max(lens)),
                           d_lens.clone(), S, total)

    def build_ranges(self, slots: list[int], starts: list[int], ns: list[int], width: int,
                     sample: list[int], bucket_batch: int | None = None,
                     extra: np.ndarray | None = None) -> RangesMeta:
        """Metadata of a mixed batch (chunked prefill + decode) with vj_build_metadata
        in ranges mode: sequence s contributes positions [starts[s], starts[s] +
        ns[s]); tokens are padded to a power of two like prefill. `sample` lists
        the sequences whose last row is sampled. One host->device upload."""
        S = len(slots)
        total = int(sum(ns))
        bt = bucket_size(total)
        bb = bucket_batch or S
        ends = np.cumsum(np.asarray(ns, np.int64))
        sample = np.asarray(sample, np.int64)
        arr = self._upload(np.concatenate([
            np.asarray(slots, np.int32), np.asarray(starts, np.int32),
            np.asarray(ns, np.int32), (ends[sample] - 1).astype(np.int32),
            np.asarray(slots, np.int32)[sample],
            (np.asarray(starts, np.int64) + np.asarray(ns, np.int64))[sample].astype(np.int32)]
            + ([np.asarray(extra).view(np.int32).ravel()] if extra is not None else [])))
        d_slots, d_starts, d_ns = arr[:S], arr[S:2 * S], arr[2 * S:3 * S]
        K = sample.size
        rows = arr[3 * S:3 * S + K]
        s_slots, s_lens = arr[3 * S + K:3 * S + 2 * K], arr[3 * S + 2 * K:3 * S + 3 * K]
        self._last_extra = arr[3 * S + 3 * K:] if extra is not None else None
        dev = self.device
        ids = torch.empty(bt, dtype=torch.int32, device=dev)
        pos = torch.empty_like(ids)
        sm = torch.empty_like(ids)
        tables = torch.empty((bb, width), dtype=torch.int32, device=dev)
        cu = torch.empty(bb + 1, dtype=torch.int32, device=dev)
        ctx = torch.empty(bb, dtype=torch.int32, device=dev)
        _native.call("vj_build_metadata", _native.VJ_META_RANGES, d_slots.data_ptr(),
                     d_starts.data_ptr(), d_ns.data_ptr(), S, self.tokens.data_ptr(),
                     self.tokens.stride(0), self.blocks.data_ptr(), self.num_blocks.data_ptr(),
                     self.blocks.stride(0), self.block_size, width, bt, bb, 0, ids.data_ptr(),
                     pos.data_ptr(), sm.data_ptr(), tables.data_ptr(), cu.data_ptr(),
                     ctx.data_ptr(), self.error.data_ptr(), stream_ptr(dev))
        return RangesMeta(ids, pos, sm, tables, cu, ctx, S, total, max(ns), rows,
                          s_slots, s_lens)

    def build_decode(self, slots: list[int], lens: list[int], width: int,
                     last_block_slot: bool = True, out: DecodeMeta | None = None,
                     extra: np.ndarray | None = None) -> DecodeMeta:
        """Decode metadata for len(slots) rows padded to a power of two; with
        `out`, written into its (static, CUDA-graph) buffers of that bucket.
        `extra` (32-bit words, e.g. sampling parameters) rides the same
        upload; see last_extra()."""
        B = len(slots)
        bb = bucket_size(B)
        d_slots, d_lens = self._lists(slots, lens, extra)
        dev = self.device
        if out is not None:
            if out.input_ids.numel() != bb or out.block_tables.shape[1] != width:
                raise ValueError("static decode buffers do not match the batch bucket")
            ids, pos, sm, ctx, tables = (out.input_ids, out.positions, out.slot_mapping,
                                         out.context_lens, out.block_tables)
        else:
            ids = torch.empty(bb, dtype=torch.int32, device=dev)
            pos = torch.empty_like(ids)
            sm = torch.empty_like(ids)
            ctx = torch.empty_like(ids)
            tables = torch.empty((bb, width), dtype=torch.int32, device=dev)
        _native.call("vj_build_metadata", _native.VJ_META_DECODE, d_slots.data_ptr(), None,
                     d_lens.data_ptr(), B, self.tokens.data_ptr(), self.tokens.stride(0),
                     self.blocks.data_ptr(), self.num_blocks.data_ptr(), self.blocks.stride(0),
                     self.block_size, width, bb, bb,
                     _native.VJ_META_LAST_BLOCK_SLOT if last_block_slot else 0,
                     ids.data_ptr(), pos.data_ptr(), sm.data_ptr(), tables.data_ptr(), None,
                     ctx.data_ptr(), self.error.data_ptr(), stream_ptr(dev))
        if out is not None:
            out.num_seqs = B
            return out
        return DecodeMeta(ids, pos, sm, tables, ctx, B)

    def argmax_append(self, logits: torch.Tensor, slots: torch.Tensor | None,
                      lens: torch.Tensor | None, out: torch.Tensor | None = None) -> torch.Tensor:
        """Greedy token per row of logits [R, V]; also stored at tokens[slot, len]."""
        R, V = logits.shape
        if out is None:
            out = torch.empty(R, dtype=torch.int32, device=logits.device)
        _native.call("vj_argmax_append", logits.data_ptr(), logits.stride(0), R, V,
                     out.data_ptr(), None if slots is None else self.tokens.data_ptr(),
                     self.tokens.stride(0), None if slots is None else slots.data_ptr(),
                     None if lens is None else lens.data_ptr(), stream_ptr(logits.device))
        return out

    def check(self) -> None:
        code = int(self.error.item())
        if code:
            self.error.zero_()
            raise RuntimeError(f"device metadata error {code} (1: position without a block, "
                               "2: tokens beyond the bucket, 3: bad table row)")
