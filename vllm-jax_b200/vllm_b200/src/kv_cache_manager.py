"""Paged KV block manager (vllm/src/kv_cache_manager.py:9-70 of vllm-jax).

Free blocks form a FIFO: allocation takes from the front, release appends to
the back, starting from 0..num_blocks-1 in order, so block ids match the
reference's exactly. Prefill needs ceil(len / bs) blocks; decode allocates
one block when len % bs == 0 (one step before the new token needs it, as the
reference does). Every change to a request's block list is recorded in
`dirty` so the engine can upload only the changed rows to the GPU."""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass

from .request import Request


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


@dataclass
class Block:
    block_id: int
    ref_count: int
    hash: int | None = None   # prefix-cache key of a full block (None: not cached)
    # what the key stands for, compared on every hit so that a hash collision
    # can never hand out another prompt's KV: the block's tokens and the key
    # of the block before it in its request (0 for the first block)
    tokens: tuple | None = None
    parent: int = 0


class FreeBlockQueue:
    """FIFO of free blocks (the reference's deque, kv_cache_manager.py:20-21)
    that can also drop a block from the middle in O(1): a free block that
    still holds a cached prefix is taken back out when a request reuses it."""

    def __init__(self, blocks: list[Block]):
        self._d: OrderedDict[int, Block] = OrderedDict((b.block_id, b) for b in blocks)

    def popleft(self) -> Block:
        return self._d.popitem(last=False)[1]

    def append(self, block: Block) -> None:
        self._d[block.block_id] = block

    def remove(self, block: Block) -> None:
        del self._d[block.block_id]

    def __contains__(self, block: Block) -> bool:
        return block.block_id in self._d

    def __len__(self) -> int:
        return len(self._d)

    def __iter__(self):
        return iter(self._d.values())


class KVCacheManager:

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.blocks = [Block(i, 0) for i in range(num_blocks)]
        self.free_block_queue = FreeBlockQueue(self.blocks)
        self.req_to_blocks: dict[int, list[Block]] = {}
        self.dirty: set[int] = set()      # request ids whose block list changed
        # prefix cache (chunked mode only): hash of (parent hash, block tokens)
        # -> a block whose KV holds exactly those positions
        self.cached: dict[int, Block] = {}

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
        if block.hash is not None:       # evict its cached prefix
            if self.cached.get(block.hash) is block:
                del self.cached[block.hash]
            block.hash = None
            block.tokens = None
            block.parent = 0
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

    # -- prefix caching (chunked mode, beyond the reference) -----------------
    def block_hashes(self, token_ids: list[int], n_blocks: int,
                     known: list[int] | None = None) -> list[int]:
        """Chained hashes of the first n_blocks full blocks of token_ids;
        `known` (a prefix of the answer) is extended, not recomputed."""
        bs = self.block_size
        out = list(known or [])
        h = out[-1] if out else 0
        for i in range(len(out), n_blocks):
            h = hash((h, tuple(token_ids[i * bs:(i + 1) * bs])))
            out.append(h)
        return out

    def lookup_prefix(self, request: Request, max_blocks: int) -> list[Block]:
        """Cached blocks holding the longest prefix of the request's full blocks."""
        bs = self.block_size
        hashes = self.block_hashes(request.token_ids, min(max_blocks, len(request) // bs))
        hit = []
        parent = 0
        for i, h in enumerate(hashes):
            b = self.cached.get(h)
            if (b is None or b.parent != parent
                    or b.tokens != tuple(request.token_ids[i * bs:(i + 1) * bs])):
                break
            hit.append(b)
            parent = h
        return hit

    def acquire(self, request: Request, blocks: list[Block]) -> None:
        """Share cached blocks with `request` (they become its first blocks)."""
        table = self.get_block_table(request)
        assert not table, "prefix blocks must come first"
        for b in blocks:
            if b.ref_count == 0:
                self.free_block_queue.remove(b)
            b.ref_count += 1
            table.append(b)
        if blocks:
            self.dirty.add(request.id)

    def register(self, request: Request, num_computed: int) -> None:
        """Publish the request's blocks whose positions are all computed."""
        table = self.get_block_table(request)
        full = min(num_computed // self.block_size, len(table))
        known = getattr(request, "block_hash_chain", [])
        if len(known) >= full:
            return
        chain = self.block_hashes(request.token_ids, full, known)
        request.block_hash_chain = chain
        bs = self.block_size
        for i in range(len(known), full):
            b = table[i]
            if b.hash is None and chain[i] not in self.cached:
                b.hash = chain[i]
                b.tokens = tuple(request.token_ids[i * bs:(i + 1) * bs])
                b.parent = chain[i - 1] if i else 0
                self.cached[chain[i]] = b

    def deallocate(self, request: Request) -> None:
        table = self.get_block_table(request)
        for block in table:
            block.ref_count -= 1
            if block.ref_count == 0:
                self.free_block_queue.append(block)
        table.clear()
        request.block_hash_chain = []
        self.dirty.add(request.id)
