"""Paged KV block manager with token-keyed prefix caching.

Blocks hold 16 tokens. A full block is identified by a chained hash of
(parent block hash, its 16 token ids), exactly the key vLLM's prefix cache uses
(token ids only; reference: docs/MULTISWITCH_EXPLAINED.md:323-331). That key
is sufficient here because a block's KV is a pure function of its token
prefix: with activated LoRA every token before a control token runs base
weights, and the routing carry at any position is itself a function of the
prefix. So every adapter shares the base-computed context blocks.

Freed blocks that carry a hash stay resident in an LRU queue and are reused
on a hit; allocation takes never-hashed blocks first, then evicts the least
recently used cached block.
"""
from __future__ import annotations

from collections import OrderedDict, deque

from .request import Request

BLOCK_SIZE = 16


def chain_hashes(token_ids: list[int], n_blocks: int, start: int = 0, parent: int | None = None,
                 prev: list[int] | None = None) -> list[int]:
    """Hashes of blocks ``start .. n_blocks-1`` of ``token_ids`` (``prev`` = earlier hashes)."""
    out = list(prev or [])
    h = out[start - 1] if start > 0 else (parent if parent is not None else 0x5EED)
    for b in range(start, n_blocks):
        h = hash((h, tuple(token_ids[b * BLOCK_SIZE:(b + 1) * BLOCK_SIZE])))
        out.append(h)
    return out


class BlockManager:
    def __init__(self, num_blocks: int, enable_prefix_caching: bool = True):
        self.num_blocks = num_blocks
        self.enable_prefix_caching = enable_prefix_caching
        self.ref = [0] * num_blocks
        self.hash_of: list[int | None] = [None] * num_blocks
        self.by_hash: dict[int, int] = {}
        self.free = deque(range(num_blocks))
        self.evictable: OrderedDict[int, None] = OrderedDict()
        # prefix-cache counters, in tokens (as vLLM's prefix_cache_queries/hits)
        self.queries = 0
        self.hits = 0

    # ---------------------------------------------------------------- capacity
    @property
    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def usage(self) -> float:
        return 1.0 - self.num_free / max(1, self.num_blocks)

    def _take(self) -> int | None:
        if self.free:
            b = self.free.popleft()
        elif self.evictable:
            b, _ = self.evictable.popitem(last=False)
            h = self.hash_of[b]
            if h is not None and self.by_hash.get(h) == b:
                del self.by_hash[h]
            self.hash_of[b] = None
        else:
            return None
        self.ref[b] = 1
        return b

    # ---------------------------------------------------------------- prefix hits
    def match_prefix(self, req: Request) -> int:
        """Acquire cached blocks for the longest cached prefix; returns hit tokens.

        At least one prompt token is always left to compute so the step
        produces the logits of the last prompt token.
        """
        prompt = req.prompt_ids
        n_full = (len(prompt) - 1) // BLOCK_SIZE
        req.block_hashes = chain_hashes(prompt, len(prompt) // BLOCK_SIZE)
        self.queries += len(prompt)
        if not self.enable_prefix_caching:
            return 0
        hit = 0
        for b in range(n_full):
            blk = self.by_hash.get(req.block_hashes[b])
            if blk is None:
                break
            if self.ref[blk] == 0:
                self.evictable.pop(blk, None)
            self.ref[blk] += 1
            req.block_ids.append(blk)
            hit += 1
        req.num_registered_blocks = hit
        self.hits += hit * BLOCK_SIZE
        return hit * BLOCK_SIZE

    def first_block_cached(self, token_ids: list[int]) -> bool:
        """Whether the first full block of ``token_ids`` is in the prefix cache (one hash probe)."""
        if not self.enable_prefix_caching or len(token_ids) <= BLOCK_SIZE:
            return False
        return chain_hashes(token_ids, 1)[0] in self.by_hash

    # ---------------------------------------------------------------- allocation
    def blocks_needed(self, req: Request, num_tokens: int) -> int:
        need = (num_tokens + BLOCK_SIZE - 1) // BLOCK_SIZE
        return max(0, need - len(req.block_ids))

    def can_allocate(self, req: Request, num_tokens: int) -> bool:
        return self.blocks_needed(req, num_tokens) <= self.num_free

    def allocate(self, req: Request, num_tokens: int) -> bool:
        """Ensure blocks for the first ``num_tokens`` tokens of ``req``."""
        need = self.blocks_needed(req, num_tokens)
        if need > self.num_free:
            return False
        for _ in range(need):
            req.block_ids.append(self._take())
        return True

    def free_request(self, req: Request) -> None:
        # release in reverse so the tail of a sequence is evicted first
        for b in reversed(req.block_ids):
            self.ref[b] -= 1
            if self.ref[b] == 0:
                if self.hash_of[b] is not None and self.enable_prefix_caching:
                    self.evictable[b] = None
                else:
                    self.hash_of[b] = None
                    self.free.append(b)
        req.block_ids = []
        req.num_registered_blocks = 0

    # ---------------------------------------------------------------- publication
    def register_full_blocks(self, req: Request) -> None:
        """Publish newly completed (computed) blocks of ``req`` to the prefix cache."""
        if not self.enable_prefix_caching:
            return
        n_full = req.num_computed // BLOCK_SIZE
        if n_full <= req.num_registered_blocks:
            return
        ids = req.all_ids
        if len(req.block_hashes) < n_full:
            req.block_hashes = chain_hashes(ids, n_full, start=len(req.block_hashes), prev=req.block_hashes)
        for b in range(req.num_registered_blocks, n_full):
            blk = req.block_ids[b]
            h = req.block_hashes[b]
            if h not in self.by_hash:
                self.by_hash[h] = blk
                self.hash_of[blk] = h
            elif self.hash_of[blk] is None and self.by_hash[h] != blk:
                pass  # identical content computed twice; keep the first copy published
        req.num_registered_blocks = n_full

    def reset_prefix_cache(self) -> None:
        for b in list(self.evictable.keys()):
            self.hash_of[b] = None
            self.free.append(b)
        self.evictable.clear()
        self.by_hash = {h: b for h, b in self.by_hash.items() if self.ref[b] > 0}
