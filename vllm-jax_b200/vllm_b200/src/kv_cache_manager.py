"""Paged KV block manager (vllm/src/kv_cache_manager.py:9-70 of vllm-jax).

Free blocks form a FIFO: allocation takes from the front, release appends to
the back, starting from 0..num_blocks-1 in order, so block ids match the
reference's exactly. Prefill needs ceil(len / bs) blocks; decode allocates
one block when len % bs == 0 (one step before the new token needs it, as the
reference does). Every change to a request's block list is recorded in
`dirty` so the engine can upload only the changed rows to the GPU."""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass

from .request import Request


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


@dataclass
class Block:
    block_id: int
    ref_count: int


class KVCacheManager:

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.blocks = [Block(i, 0) for i in range(num_blocks)]
        self.free_block_queue: deque[Block] = deque(self.blocks)
        self.req_to_blocks: dict[int, list[Block]] = {}
        self.dirty: set[int] = set()      # request ids whose block list changed

    def get_block_table(self, request: Request) -> list[Block]:
        return self.req_to_blocks.setdefault(request.id, [])

    def block_ids(self, request: Request) -> list[int]:
        return [b.block_id for b in self.get_block_table(request)]

    def can_allocate(self, request: Request, is_prefill: bool) -> bool:
        table = self.get_block_table(request)
        total = len(request)
        if is_prefill:
            return ceil_div(total, self.block_size) <= len(self.free_block_queue)
        assert table, "decode of a request without blocks"
        if total % self.block_size != 0:
            return True
        return len(self.free_block_queue) > 0

    def _take(self, table: list[Block]) -> None:
        block = self.free_block_queue.popleft()
        block.ref_count += 1
        table.append(block)

    def allocate_slots(self, request: Request, is_prefill: bool) -> None:
        table = self.get_block_table(request)
        total = len(request)
        if is_prefill:
            need = ceil_div(total, self.block_size)
            while len(table) < need:
                self._take(table)
            self.dirty.add(request.id)
            return
        assert table, "decode of a request without blocks"
        if total % self.block_size == 0:
            self._take(table)
            self.dirty.add(request.id)

    # -- token-budget (chunked prefill) mode, beyond the reference ----------
    def can_grow(self, request: Request, total_tokens: int) -> bool:
        need = ceil_div(total_tokens, self.block_size) - len(self.get_block_table(request))
        return need <= len(self.free_block_queue)

    def grow(self, request: Request, total_tokens: int) -> None:
        """Own enough blocks for positions [0, total_tokens)."""
        table = self.get_block_table(request)
        need = ceil_div(total_tokens, self.block_size)
        if len(table) < need:
            while len(table) < need:
                self._take(table)
            self.dirty.add(request.id)

    def deallocate(self, request: Request) -> None:
        table = self.get_block_table(request)
        for block in table:
            block.ref_count -= 1
            if block.ref_count == 0:
                self.free_block_queue.append(block)
        table.clear()
        self.dirty.add(request.id)
