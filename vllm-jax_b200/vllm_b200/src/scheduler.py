"""Continuous-batching scheduler (vllm/src/scheduler.py:7-70 of vllm-jax).

Policy, identical to the reference:
  * decode first: every running request (front first) gets one token while
    fewer than max_num_seqs are scheduled and the token budget is not spent;
    a request that needs a new block when none is free preempts the request
    at the TAIL of `running` (it returns to the front of `waiting` and gives
    its blocks back), and an empty `running` with no room raises the same
    AssertionError as the reference;
  * then prefill from the front of `waiting` while the sequence budget lasts,
    the request fits strictly inside the remaining token budget
    (num_batched + len < max_num_batched_tokens) and its blocks are free;
  * postprocess finishes a request on EOS (unless ignore_eos) or when it has
    max_new_tokens completions.
With Config.compat = False finished requests also release their blocks (the
reference keeps them, so its pool shrinks over a long run)."""
from __future__ import annotations

from collections import deque

from ..config import Config
from .kv_cache_manager import KVCacheManager
from .request import Request, Status


class Scheduler:

    def __init__(self, config: Config, kv_cache_manager: KVCacheManager):
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.max_num_seqs = config.max_num_seqs
        self.compat = config.compat
        self.kv_cache_manager = kv_cache_manager
        self.waiting: deque[Request] = deque()
        self.running: deque[Request] = deque()
        self.finished_requests: list[Request] = []

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, request: Request) -> None:
        self.waiting.append(request)

    def preempt(self, request: Request) -> None:
        request.status = Status.WAITING
        self.waiting.appendleft(request)
        self.kv_cache_manager.deallocate(request)

    def schedule(self) -> tuple[list[Request], list[Request]]:
        kv = self.kv_cache_manager
        decode: list[Request] = []
        prefill: list[Request] = []
        num_tokens = num_seqs = 0
        while (self.running and num_seqs < self.max_num_seqs
               and num_tokens < self.max_num_batched_tokens):
            request = self.running.popleft()
            while not kv.can_allocate(request, False):
                assert self.running, "Request cant fit in memory"
                self.preempt(self.running.pop())
            kv.allocate_slots(request, False)
            decode.append(request)
            num_seqs += 1
            num_tokens += 1
        self.running.extendleft(reversed(decode))
        while self.waiting and num_seqs < self.max_num_seqs:
            request = self.waiting[0]
            if (num_tokens + len(request) >= self.max_num_batched_tokens
                    or not kv.can_allocate(request, True)):
                break
            self.waiting.popleft()
            self.running.append(request)
            request.status = Status.RUNNING
            kv.allocate_slots(request, True)
            prefill.append(request)
            num_seqs += 1
            num_tokens += len(request)
        return decode, prefill

    def postprocess(self, requests: list[Request], token_ids: list[int]) -> None:
        for request, token_id in zip(requests, token_ids):
            if ((not request.ignore_eos and token_id == request.eos_token_id)
                    or request.num_completion_tokens == request.max_new_tokens):
                request.status = Status.FINISHED
                self.running.remove(request)
                self.finished_requests.append(request)
                if not self.compat:
                    self.kv_cache_manager.deallocate(request)


class ChunkedScheduler:
    """Token-budget scheduler with chunked prefill mixed into decode steps.

    Beyond the reference (whose prefill must fit the budget whole and runs in
    a separate pass from decode, so a prompt >= max_num_batched_tokens is never
    admitted): every step spends at most max_num_batched_tokens tokens over at
    most max_num_seqs requests. Running requests come first, in order: one
    token for a request whose known tokens are all cached (decode), else the
    next chunk of its prompt; then waiting requests start their prompt with
    whatever budget is left, admitted only while the pool holds all their
    known tokens plus a 1% watermark (their blocks are taken at admission). A request samples a token when a step processes
    its last known token. When the pool runs dry the request at the tail of
    `running` is preempted (blocks freed, recomputed from scratch later) unless
    a shorter chunk still fits. Finished requests always release their blocks.

    With config.enable_prefix_caching, full blocks are published under a
    chained hash of their tokens once computed; a new request shares the
    cached blocks of its longest matching prefix and starts computing after
    them (freed blocks keep their content until the FIFO reuses them)."""

    def __init__(self, config: Config, kv_cache_manager: KVCacheManager):
        self.max_num_batched_tokens = config.max_num_batched_tokens
        self.max_num_seqs = config.max_num_seqs
        self.kv_cache_manager = kv_cache_manager
        self.watermark_blocks = max(1, kv_cache_manager.num_blocks // 100)
        self.prefix_caching = config.enable_prefix_caching
        self.prefix_hit_tokens = 0
        self.waiting: deque[Request] = deque()
        self.running: deque[Request] = deque()
        self.finished_requests: list[Request] = []

    def is_finished(self) -> bool:
        return not self.waiting and not self.running

    def add(self, request: Request) -> None:
        self.waiting.append(request)

    def _preempt(self, request: Request) -> None:
        request.status = Status.WAITING
        request.num_computed_tokens = 0
        self.running.remove(request)
        self.waiting.appendleft(request)
        self.kv_cache_manager.deallocate(request)

    def schedule(self) -> list[tuple[Request, int]]:
        """Returns (request, number of new tokens) in batch order."""
        kv = self.kv_cache_manager
        budget = self.max_num_batched_tokens
        out: list[tuple[Request, int]] = []
        i = 0
        while i < len(self.running) and len(out) < self.max_num_seqs and budget > 0:
            req = self.running[i]
            n = min(len(req) - req.num_computed_tokens, budget)
            while not kv.can_grow(req, req.num_computed_tokens + n):
                # a shorter chunk that fits beats a preemption
                fit = ((len(kv.get_block_table(req)) + len(kv.free_block_queue)) * kv.block_size
                       - req.num_computed_tokens)
                if fit >= 1:
                    n = fit
                    break
                victim = self.running[-1]
                self._preempt(victim)
                if victim is req:
                    n = 0
                    break
            if n <= 0:
                break
            kv.grow(req, req.num_computed_tokens + n)
            out.append((req, n))
            budget -= n
            i += 1
        while self.waiting and len(out) < self.max_num_seqs and budget > 0:
            req = self.waiting[0]
            # prefix cache: full blocks already holding this request's leading
            # tokens are shared; at least the last token is computed (it samples)
            hit = (kv.lookup_prefix(req, (len(req) - 1) // kv.block_size)
                   if self.prefix_caching else [])
            # admission reserves blocks for every known token (its later chunks
            # never allocate) and keeps a watermark free for decode growth, so
            # that a new prompt does not immediately preempt running requests
            need = -(-len(req) // kv.block_size) - len(hit)
            free_hits = sum(1 for b in hit if b.ref_count == 0)
            if need + self.watermark_blocks > len(kv.free_block_queue) - free_hits:
                break
            self.waiting.popleft()
            req.status = Status.RUNNING
            self.running.append(req)
            kv.acquire(req, hit)
            req.num_computed_tokens = len(hit) * kv.block_size
            self.prefix_hit_tokens += req.num_computed_tokens
            kv.grow(req, len(req))
            n = min(len(req) - req.num_computed_tokens, budget)
            out.append((req, n))
            budget -= n
        return out

    def postprocess(self, batch: list[tuple[Request, int]], sampled: dict[int, int]) -> None:
        """Advance computed tokens; finish requests whose sampled token ends them."""
        for req, n in batch:
            req.num_computed_tokens += n
            if self.prefix_caching:
                self.kv_cache_manager.register(req, req.num_computed_tokens)
            if req.id not in sampled:
                continue
            token = sampled[req.id]
            if ((not req.ignore_eos and token == req.eos_token_id)
                    or req.num_completion_tokens == req.max_new_tokens):
                req.status = Status.FINISHED
                self.running.remove(req)
                self.finished_requests.append(req)
                self.kv_cache_manager.deallocate(req)
