"""Paged KV block allocator with prefix caching.

The physical block ids it hands out end up in the block tables and slot
mappings the kernels read, so its decisions must equal the reference's
(microserve/engine/block_manager.py:24-151) id for id:
  * free blocks are a FIFO (allocate pops the oldest, release appends);
  * a full block is identified by a chained xxhash64 of its token ids
    (seed = the previous block's hash as 8 little-endian bytes, then the
    token ids as int64 little-endian); hashes are recorded after a step
    fills a block (hash_blocks) and stay valid until the block is reused;
  * a new prompt reuses cached blocks for its leading full blocks, except the
    last full one, and only while the chained hash and the tokens match;
  * a prefill is scheduled for min(free_blocks * block_size, budget, gap)
    tokens (plus the room left in the last block for a continuing chunk).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

import numpy as np
import xxhash

from microserve_b200.engine.sequence import Sequence


@dataclass(slots=True)
class _Block:
    block_id: int
    ref_count: int = 0
    hash: int = -1
    token_ids: list = field(default_factory=list)


def chain_hash(token_ids: list[int], prefix: int = -1) -> int:
    h = xxhash.xxh64()
    if prefix != -1:
        h.update(int(prefix).to_bytes(8, "little"))
    h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
    return h.intdigest()


class BlockManager:
    def __init__(self, nums_block: int, block_size: int):
        self.block_size = block_size
        self.blocks = [_Block(i) for i in range(nums_block)]
        self.hash_to_block: dict[int, int] = {}
        self.free_blocks: deque[int] = deque(range(nums_block))
        self.used_blocks: set[int] = set()

    @property
    def free_blocks_nums(self) -> int:
        return len(self.free_blocks)

    compute_hash = staticmethod(chain_hash)

    # -- single blocks -------------------------------------------------------
    def _take_free(self) -> int:
        bid = self.free_blocks.popleft()
        blk = self.blocks[bid]
        assert blk.ref_count == 0
        if blk.hash != -1 and self.hash_to_block.get(blk.hash) == bid:
            del self.hash_to_block[blk.hash]  # its cached contents are about to be overwritten
        blk.hash, blk.token_ids, blk.ref_count = -1, [], 1
        self.used_blocks.add(bid)
        return bid

    def _release(self, bid: int) -> None:
        assert self.blocks[bid].ref_count == 0
        self.used_blocks.remove(bid)
        self.free_blocks.append(bid)

    def _unref(self, bid: int) -> None:
        blk = self.blocks[bid]
        blk.ref_count -= 1
        if blk.ref_count == 0:
            self._release(bid)

    # -- prefix cache ----------------------------------------------------------
    def _cached_prefix(self, seq: Sequence) -> list[int]:
        """Cached blocks matching the prompt's leading full blocks (all but the last full one)."""
        bs = self.block_size
        full = seq.num_tokens_with_spec // bs
        found: list[int] = []
        h = -1
        for i in range(full - 1):
            chunk = seq.token_ids[i * bs:(i + 1) * bs]
            h = chain_hash(chunk, h)
            bid = self.hash_to_block.get(h, -1)
            if bid == -1 or self.blocks[bid].token_ids != chunk:
                break
            found.append(bid)
            self.blocks[bid].ref_count += 1
        return found

    # -- per step ----------------------------------------------------------------
    def allocate(self, seq: Sequence, token_budget: int) -> bool:
        bs = self.block_size
        if seq.gap == 1:  # decode: a new block only when the last one is full
            if seq.num_computed_tokens % bs:
                return True
            if not self.free_blocks:
                return False
            seq.block_table.append(self._take_free())
            return True

        if seq.num_computed_tokens == 0:  # first chunk of a prompt
            cached = self._cached_prefix(seq)
            for bid in cached:
                seq.block_table.append(bid)
                seq.num_computed_tokens += bs
                if bid not in self.used_blocks:  # revive a freed block that still holds the prefix
                    self.used_blocks.add(bid)
                    self.free_blocks.remove(bid)
            n = min(len(self.free_blocks) * bs, token_budget, seq.gap)
            if n == 0 and seq.gap > 0:  # nothing fits: undo the prefix hits
                for bid in cached:
                    self._unref(bid)
                del seq.block_table[:len(cached)]
                seq.num_computed_tokens -= len(cached) * bs
                return False
            seq.num_scheduled_tokens = n
            for _ in range((n - 1) // bs + 1):
                seq.block_table.append(self._take_free())
            return True

        # continuing chunk: fill the tail of the last block first
        used = seq.num_computed_tokens % bs
        room = 0 if used == 0 else bs - used
        n = min(len(self.free_blocks) * bs + room, token_budget, seq.gap)
        seq.num_scheduled_tokens = n
        for _ in range((max(0, n - room) + bs - 1) // bs):
            seq.block_table.append(self._take_free())
        return True

    def deallocate(self, seq: Sequence) -> None:
        for bid in reversed(seq.block_table):
            self._unref(bid)
        seq.block_table.clear()

    def hash_blocks(self, seq: Sequence) -> None:
        """Record the hashes of the blocks the current step fills."""
        bs = self.block_size
        first = seq.num_computed_tokens // bs
        last = (seq.num_computed_tokens + seq.num_scheduled_tokens) // bs
        if first == last:
            return
        h = self.blocks[seq.block_table[first - 1]].hash if first > 0 else -1
        for i in range(first, last):
            blk = self.blocks[seq.block_table[i]]
            chunk = seq.token_ids[i * bs:(i + 1) * bs]
            h = chain_hash(chunk, h)
            blk.hash, blk.token_ids = h, chunk
            self.hash_to_block[h] = blk.block_id
