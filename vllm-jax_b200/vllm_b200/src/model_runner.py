"""Model runner: device-resident batch state, GPU metadata, CUDA-graph decode.

Counterpart of vllm-jax's vllm/src/model_runner.py (ModelRunner.run,
:310-333). Per engine step the host sends only what changed: the token ids
of newly admitted requests and the block lists the KV manager touched (one
small upload each), plus the scheduled (slot, length) pairs. The metadata
arrays of prepare_prefill / prepare_decode are then built on the GPU (K4),
the sampled tokens are written into the device token table by the argmax
kernel, and one device->host copy of [batch] int32 per step returns them to
the scheduler. Decode steps replay a CUDA graph captured per power-of-two
batch bucket (the reference's jit buckets, model_runner.py:125-183).
"""
from __future__ import annotations

import time

import numpy as np
import torch

from .. import _native
from ..config import Config
from ..kernels.decode_paged_attention import decode_workspace_bytes
from ..kernels.kv_store import rope_table
from ..kernels.metadata import DecodeMeta, DeviceTables, bucket_size
from ..kernels.sampler import sample
from ..model.qwen3 import Qwen3Config, Qwen3Model, Qwen3Weights
from .kv_cache_manager import KVCacheManager
from .request import Request


def kv_cache_bytes_per_block(mcfg: Qwen3Config, block_size: int, tp_size: int) -> int:
    return (mcfg.num_hidden_layers * 2 * block_size * (mcfg.num_key_value_heads // tp_size)
            * mcfg.head_dim * 2)


class PendingTokens:
    """Sampled tokens of a launched step, copied to pinned host memory."""

    def __init__(self, host: torch.Tensor, event: torch.cuda.Event, n: int):
        self.host, self.event, self.n = host, event, n

    def collect(self) -> list[int]:
        self.event.synchronize()
        return self.host[:self.n].tolist()


def sampling_words(requests: list[Request]) -> np.ndarray | None:
    """Per-row sampling parameters as 32-bit words for one upload:
    temperature f32 [n], top_k i32 [n], top_p f32 [n], seeds u32 [n, 2].
    None when every request is greedy (the argmax kernel is used then)."""
    sps = [r.sampling_params for r in requests]
    if all(sp.temperature <= 0 for sp in sps):
        return None
    n = len(requests)
    w = np.empty(5 * n, np.uint32)
    w[:n] = np.asarray([sp.temperature for sp in sps], np.float32).view(np.uint32)
    w[n:2 * n] = np.asarray([sp.top_k for sp in sps], np.int64).astype(np.uint32)
    w[2 * n:3 * n] = np.asarray([sp.top_p for sp in sps], np.float32).view(np.uint32)
    seeds = np.asarray([(sp.seed & 0xFFFFFFFF, r.sample_stream & 0xFFFFFFFF)
                        for sp, r in zip(sps, requests)], np.uint64).astype(np.uint32)
    w[3 * n:] = seeds.ravel()
    return w


class ModelRunner:

    def __init__(self, config: Config, model_cfg: Qwen3Config, kv_cache_manager: KVCacheManager,
                 device: torch.device, *, tp_rank: int = 0, tp_size: int = 1,
                 process_group=None, seed: int = 0, weights: Qwen3Weights | None = None,
                 max_slots: int = 1024, use_cuda_graphs: bool = True, tp_comm=None):
        self.config = config
        self.mcfg = model_cfg
        self.kv = kv_cache_manager
        self.device = device
        self.block_size = config.block_size
        self.width = config.max_blocks_per_seq
        self.weights = weights or Qwen3Weights(model_cfg, device, seed, tp_rank, tp_size)
        # compat=True also follows the reference's bf16 q scaling
        self.model = Qwen3Model(self.weights, process_group, tp_comm,
                                reference_q_scaling=config.compat)
        # RoPE (cos, sin) table of every position a request can reach, built
        # before any graph capture (positions repeat across layers and steps)
        self.model.rope_table = rope_table(device, model_cfg.rope_theta, config.max_len + 1)
        # one decode workspace for the largest batch bucket, allocated before
        # any graph capture and never replaced
        self.model.decode_workspace = torch.empty(
            max(decode_workspace_bytes(bucket_size(max(config.max_num_seqs, 1)),
                                       model_cfg.num_attention_heads // tp_size,
                                       model_cfg.head_dim), 16),
            dtype=torch.uint8, device=device)
        if config.fused_gemm_max_rows > 0:
            self.model.enable_fused_gemm(config.fused_gemm_max_rows)
        hkv = model_cfg.num_key_value_heads // tp_size
        shape = (2, kv_cache_manager.num_blocks, config.block_size, hkv, model_cfg.head_dim)
        # zero-initialised like the reference's pool (model_runner.py:190-199)
        self.kv_caches = [torch.zeros(shape, dtype=torch.bfloat16, device=device)
                          for _ in range(model_cfg.num_hidden_layers)]
        self.tables = DeviceTables(max_slots, config.max_len, self.width, config.block_size,
                                   device)
        self.free_slots = list(range(max_slots - 1, -1, -1))
        # Collectives of torch.distributed are not captured into CUDA graphs:
        # with tensor parallelism decode steps are captured only when the
        # NVLink communicator reduces every decode bucket.
        max_bucket = bucket_size(max(config.max_num_seqs, 1))
        self.use_cuda_graphs = use_cuda_graphs and (
            tp_size == 1 or (tp_comm is not None and tp_comm.max_rows >= max_bucket))
        self.graphs: dict[int, tuple[torch.cuda.CUDAGraph, DecodeMeta, torch.Tensor]] = {}
        self.graph_launches: dict[int, int] = {}
        n = max(config.max_num_seqs, 1)
        # when a list: (start, end) CUDA events of every decode forward, for
        # measuring decode-step device time (bench.py's roofline)
        self.decode_events: list | None = None
        self._tok_ring = [torch.empty(n, dtype=torch.int32).pin_memory() for _ in range(4)]
        self._tok_events: list[torch.cuda.Event | None] = [None] * 4
        self._tok_next = 0

    # ------------------------------------------------------------------ state sync
    def _assign_slot(self, request: Request) -> int:
        if request.slot < 0:
            if not self.free_slots:
                raise RuntimeError("no free request slot: raise max_slots")
            request.slot = self.free_slots.pop()
            # the device token row gets every token known now; later tokens are
            # appended on the device by the sampler
            self.tables.set_tokens([(request.slot, 0, list(request.token_ids))])
        return request.slot

    def release(self, request: Request) -> None:
        if request.slot >= 0:
            self.free_slots.append(request.slot)
            request.slot = -1

    def _sync_blocks(self, requests: dict[int, Request]) -> None:
        rows = []
        for rid in sorted(self.kv.dirty):
            r = requests.get(rid)
            if r is not None and r.slot >= 0:
                rows.append((r.slot, self.kv.block_ids(r)))
        self.kv.dirty.clear()
        self.tables.set_blocks(rows)

    # ------------------------------------------------------------------ decode
    def _decode_graph(self, bb: int):
        if bb in self.graphs:
            return self.graphs[bb]
        dev = self.device
        meta = DecodeMeta(torch.zeros(bb, dtype=torch.int32, device=dev),
                          torch.zeros(bb, dtype=torch.int32, device=dev),
                          torch.full((bb,), -1, dtype=torch.int32, device=dev),
                          torch.full((bb, self.width), -1, dtype=torch.int32, device=dev),
                          torch.zeros(bb, dtype=torch.int32, device=dev), bb)
        # warm up eagerly (sizes workspaces, cuBLAS handles), then capture
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            self.model.forward_decode(meta, self.kv_caches)
        torch.cuda.current_stream(dev).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        before = _native.launch_count
        with torch.cuda.graph(graph):
            logits = self.model.forward_decode(meta, self.kv_caches)
        self.graph_launches[bb] = _native.launch_count - before
        _native.launch_count = before
        self.graphs[bb] = (graph, meta, logits)
        return self.graphs[bb]

    def capture_all(self, max_batch: int) -> None:
        if not self.use_cuda_graphs:
            return
        b = 1
        while True:
            self._decode_graph(b)
            if b >= max_batch:
                break
            b *= 2

    def _draw(self, logits: torch.Tensor, d_slots: torch.Tensor, d_lens: torch.Tensor,
              words: torch.Tensor | None) -> torch.Tensor:
        """Next token of each row (stored into the device token table too):
        argmax when all rows are greedy, else the sampling kernel."""
        if words is None:
            return self.tables.argmax_append(logits, d_slots, d_lens)
        n = logits.shape[0]
        return sample(logits, words[:n].view(torch.float32), words[n:2 * n],
                      words[2 * n:3 * n].view(torch.float32), words[3 * n:5 * n],
                      positions=d_lens, token_table=self.tables.tokens, slots=d_slots)

    def _tokens_to_host(self, d_toks: torch.Tensor) -> "PendingTokens":
        """Start the device->host copy of a step's tokens into a ring buffer."""
        B = d_toks.numel()
        i = self._tok_next
        self._tok_next = (i + 1) % len(self._tok_ring)
        if self._tok_events[i] is not None:
            self._tok_events[i].synchronize()
        if B > self._tok_ring[i].numel():
            self._tok_ring[i] = torch.empty(B, dtype=torch.int32).pin_memory()
        host = self._tok_ring[i]
        host[:B].copy_(d_toks, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._tok_events[i] = ev
        return PendingTokens(host, ev, B)

    def decode(self, requests: list[Request]) -> list[int]:
        return self.decode_launch(requests).collect()

    def decode_launch(self, requests: list[Request]) -> "PendingTokens":
        """Enqueue one decode step; its tokens arrive through the returned handle."""
        slots = [r.slot for r in requests]
        lens = [len(r) for r in requests]
        B = len(requests)
        bb = bucket_size(B)
        words = sampling_words(requests)
        ev = None
        if self.decode_events is not None:
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record(torch.cuda.current_stream(self.device))
        if self.use_cuda_graphs:
            graph, meta, logits = self._decode_graph(bb)
            self.tables.build_decode(slots, lens, self.width, out=meta,
                                     last_block_slot=self.config.compat, extra=words)
            graph.replay()
            _native.launch_count += self.graph_launches[bb]
        else:
            meta = self.tables.build_decode(slots, lens, self.width,
                                            last_block_slot=self.config.compat, extra=words)
            logits = self.model.forward_decode(meta, self.kv_caches)
        if ev is not None:
            ev[1].record(torch.cuda.current_stream(self.device))
            self.decode_events.append(ev)
        d_slots, d_lens = self.tables.last_lists()
        toks = self._draw(logits[:B], d_slots, d_lens, self.tables.last_extra())
        return self._tokens_to_host(toks)

    # ------------------------------------------------------------------ prefill
    def prefill(self, requests: list[Request]) -> None:
        meta = self.tables.build_prefill([r.slot for r in requests], [len(r) for r in requests],
                                         self.config.max_num_seqs, self.width)
        self.model.forward_prefill(meta, self.kv_caches)

    # ------------------------------------------------------------------ step
    def launch(self, decode_requests: list[Request], prefill_requests: list[Request],
               live: dict[int, Request], stats: dict | None = None) -> "PendingTokens | None":
        """Enqueue one engine step without waiting for it: the decode batch
        (its tokens come back through the returned handle, not appended to the
        requests), then the prefill batch. The host can schedule the next step
        while this one runs; every later launch is ordered after it on the
        stream."""
        for r in prefill_requests:
            if r.slot < 0 and stats is not None:
                stats["h2d_bytes"] += 4 * len(r.token_ids)
            self._assign_slot(r)
        self._sync_blocks(live)
        pending = self.decode_launch(decode_requests) if decode_requests else None
        if prefill_requests:
            self.prefill(prefill_requests)
        if stats is not None:
            stats["h2d_bytes"] += 8 * (len(decode_requests) + len(prefill_requests))
            stats["d2h_bytes"] += 4 * len(decode_requests)
        return pending

    def run(self, decode_requests: list[Request], prefill_requests: list[Request],
            live: dict[int, Request], stats: dict | None = None) -> list[int]:
        """One engine step (model_runner.py:310-333): decode batch first (its
        tokens are returned and appended to the requests), then the prefill
        batch (KV only; its first token comes from the next step's decode)."""
        t0 = time.perf_counter()
        for r in prefill_requests:
            if r.slot < 0 and stats is not None:
                stats["h2d_bytes"] += 4 * len(r.token_ids)
            self._assign_slot(r)
        self._sync_blocks(live)
        out: list[int] = []
        if decode_requests:
            out = self.decode(decode_requests)   # ends with the D2H of the tokens
            for r, t in zip(decode_requests, out):
                r.token_ids.append(t)
                r.num_completion_tokens += 1
        t1 = time.perf_counter()
        if prefill_requests:
            self.prefill(prefill_requests)
        if stats is not None:
            stats["h2d_bytes"] += 8 * (len(decode_requests) + len(prefill_requests))
            stats["d2h_bytes"] += 4 * len(decode_requests)
            if decode_requests:
                stats["decode_s"] += t1 - t0
            if prefill_requests:
                torch.cuda.current_stream(self.device).synchronize()
                stats["prefill_s"] += time.perf_counter() - t1
        return out

    # ------------------------------------------------------------------ chunked step
    def run_chunked(self, batch: list[tuple[Request, int]], live: dict[int, Request],
                    stats: dict | None = None) -> dict[int, int]:
        """One step of the token-budget scheduler: (request, n) computes
        positions [num_computed_tokens, +n) of each request in ONE forward.
        A request whose last known token is among them samples a token, which
        is appended to it. Returns {request id: token}.

        All-decode steps (every row one token and sampled) replay the decode
        CUDA graph; mixed steps run eagerly with the decode kernel on the
        one-token rows and the prefill kernel, with its cached prefix, on the
        chunks."""
        t0 = time.perf_counter()
        for r, _ in batch:
            if r.slot < 0 and stats is not None:
                stats["h2d_bytes"] += 4 * len(r.token_ids)
            self._assign_slot(r)
        self._sync_blocks(live)
        sampled = [r for r, n in batch if r.num_computed_tokens + n == len(r)]
        if all(n == 1 for _, n in batch) and len(sampled) == len(batch):
            toks = self.decode([r for r, _ in batch])
            if stats is not None:
                stats["decode_s"] += time.perf_counter() - t0
                stats["h2d_bytes"] += 8 * len(batch)
                stats["d2h_bytes"] += 4 * len(batch)
        else:
            order = sorted(range(len(batch)), key=lambda i: batch[i][1] != 1)   # stable
            rows = [batch[i] for i in order]
            nd = sum(1 for _, n in rows if n == 1)
            pick = [i for i, (r, n) in enumerate(rows) if r.num_computed_tokens + n == len(r)]
            words = sampling_words([rows[i][0] for i in pick]) if pick else None
            meta = self.tables.build_ranges([r.slot for r, _ in rows],
                                            [r.num_computed_tokens for r, _ in rows],
                                            [n for _, n in rows], self.width, pick, extra=words)
            logits = self.model.forward_mixed(meta, self.kv_caches, nd, meta.sample_rows)
            K = len(pick)
            toks = []
            if K:
                d = self._draw(logits, meta.sample_slots, meta.sample_lens,
                               self.tables.last_extra())
                toks = self._tokens_to_host(d).collect()
            sampled = [rows[i][0] for i in pick]
            if stats is not None:
                torch.cuda.current_stream(self.device).synchronize()
                stats["prefill_s"] += time.perf_counter() - t0
                stats["h2d_bytes"] += 4 * (3 * len(rows) + 3 * K)
                stats["d2h_bytes"] += 4 * K
        out = {}
        for r, t in zip(sampled, toks):
            r.token_ids.append(t)
            r.num_completion_tokens += 1
            out[r.id] = t
        return out
