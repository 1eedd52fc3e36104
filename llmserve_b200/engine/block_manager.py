"""Paged KV-block allocator with a chained-hash prefix cache.

Semantics follow ``llmserve/engine/block_manager.py`` of the reference (allocate ``:70-94``,
deallocate ``:98-105``, the speculative slot helpers ``:107-163``, may_append ``:166-177``):

* a block is *free* (ref 0), *sealed* (full, hashed, shareable) or the *mutable tail*;
* a full block's key is xxh64(previous block key || int64 token bytes), so a hit implies the
  whole prefix matches; the stored token list guards against hash collisions;
* speculative decoding reserves ``gamma + 2`` slots before a step (``ensure_slots``), seals blocks
  that a multi-token append filled (``finalize_full_blocks``) and gives back the reservation the
  step did not use (``release_extra_slots``).

Block ids index the device KV pools directly (``[.., num_blocks, kv_heads, block_size, head_dim]``),
and the EAGLE3 draft pool is indexed by the same ids, so a block table serves both models.
"""
from collections import deque

import numpy as np
import xxhash

from llmserve_b200.engine.sequence import Sequence


class Block:
    __slots__ = ("block_id", "ref_count", "hash", "token_ids")

    def __init__(self, block_id: int):
        self.block_id = block_id
        self.ref_count = 0
        self.hash = -1
        self.token_ids: list[int] = []

    def seal(self, h: int, token_ids: list[int]):
        self.hash = h
        self.token_ids = token_ids

    def claim(self):
        self.ref_count = 1
        self.hash = -1
        self.token_ids = []


class BlockManager:

    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0:
            raise ValueError("the KV pool needs at least one block")
        self.block_size = block_size
        self.blocks = [Block(i) for i in range(num_blocks)]
        self.hash_to_block_id: dict[int, int] = {}
        self.free_block_ids: deque[int] = deque(range(num_blocks))
        self.used_block_ids: set[int] = set()

    @staticmethod
    def compute_hash(token_ids: list[int], prefix: int = -1) -> int:
        h = xxhash.xxh64()
        if prefix != -1:
            h.update(prefix.to_bytes(8, "little"))
        h.update(np.asarray(token_ids, dtype=np.int64).tobytes())
        return h.intdigest()

    # ---- raw block ops -------------------------------------------------------------------
    def _take(self, block_id: int) -> Block:
        block = self.blocks[block_id]
        assert block.ref_count == 0, f"block {block_id} is still referenced"
        block.claim()
        self.free_block_ids.remove(block_id)
        self.used_block_ids.add(block_id)
        return block

    def _take_next_free(self) -> Block:
        return self._take(self.free_block_ids[0])

    def _give_back(self, block_id: int):
        assert self.blocks[block_id].ref_count == 0
        self.used_block_ids.remove(block_id)
        self.free_block_ids.append(block_id)

    def _unref(self, block_id: int):
        block = self.blocks[block_id]
        block.ref_count -= 1
        if block.ref_count == 0:
            self._give_back(block_id)

    # ---- whole-sequence ops --------------------------------------------------------------
    def can_allocate(self, seq: Sequence) -> bool:
        return len(self.free_block_ids) >= seq.num_blocks

    def allocate(self, seq: Sequence):
        """Build ``seq.block_table``, reusing sealed blocks along the longest cached prefix."""
        assert not seq.block_table, "sequence already owns blocks"
        chain = -1
        missed = False
        for i in range(seq.num_blocks):
            tokens = seq.block(i)
            full = len(tokens) == self.block_size
            chain = self.compute_hash(tokens, chain) if full else -1
            hit = self.hash_to_block_id.get(chain, -1)
            if hit == -1 or self.blocks[hit].token_ids != tokens:
                missed = True
            if missed:
                block = self._take_next_free()
            else:
                seq.num_cached_tokens += self.block_size
                if hit in self.used_block_ids:
                    block = self.blocks[hit]
                    block.ref_count += 1
                else:
                    block = self._take(hit)
            if chain != -1:
                block.seal(chain, tokens)
                self.hash_to_block_id[chain] = block.block_id
            seq.block_table.append(block.block_id)

    def deallocate(self, seq: Sequence):
        for block_id in reversed(seq.block_table):
            self._unref(block_id)
        seq.num_cached_tokens = 0
        seq.block_table.clear()

    # ---- single-token decode -------------------------------------------------------------
    def can_append(self, seq: Sequence) -> bool:
        needs_block = len(seq) % self.block_size == 1
        return len(self.free_block_ids) >= int(needs_block)

    def may_append(self, seq: Sequence):
        table = seq.block_table
        last = self.blocks[table[-1]]
        boundary = len(seq) % self.block_size
        if boundary == 1 and len(table) < seq.num_blocks:
            assert last.hash != -1
            table.append(self._take_next_free().block_id)
        elif boundary == 0:
            self._seal(seq, seq.num_blocks - 1)
        else:
            assert last.hash == -1

    # ---- multi-token (speculative) helpers -----------------------------------------------
    def num_required_blocks(self, seq: Sequence, num_tokens: int) -> int:
        future_blocks = -(-(len(seq) + num_tokens) // self.block_size)
        return max(future_blocks - len(seq.block_table), 0)

    def can_append_tokens(self, seq: Sequence, num_tokens: int) -> bool:
        return len(self.free_block_ids) >= self.num_required_blocks(seq, num_tokens)

    def _seal(self, seq: Sequence, index: int):
        block = self.blocks[seq.block_table[index]]
        if block.hash != -1:
            return
        tokens = seq.block(index)
        if len(tokens) != self.block_size:
            return
        prefix = self.blocks[seq.block_table[index - 1]].hash if index > 0 else -1
        h = self.compute_hash(tokens, prefix)
        block.seal(h, tokens)
        self.hash_to_block_id[h] = block.block_id

    def ensure_slots(self, seq: Sequence, num_tokens: int) -> bool:
        if not self.can_append_tokens(seq, num_tokens):
            return False
        if seq.block_table and len(seq) % self.block_size == 0:
            self._seal(seq, seq.num_blocks - 1)
        for _ in range(self.num_required_blocks(seq, num_tokens)):
            seq.block_table.append(self._take_next_free().block_id)
        return True

    def ensure_slots_batch(self, seqs: list[Sequence], num_tokens: int) -> bool:
        """All-or-nothing reservation of ``num_tokens`` future slots for every sequence."""
        needed = sum(self.num_required_blocks(seq, num_tokens) for seq in seqs)
        if needed > len(self.free_block_ids):
            return False
        for seq in seqs:
            if not self.ensure_slots(seq, num_tokens):
                raise RuntimeError("speculative batch reservation became non-atomic")
        return True

    def finalize_full_blocks(self, seq: Sequence):
        for index in range(min(seq.num_blocks, len(seq.block_table))):
            self._seal(seq, index)

    def release_extra_slots(self, seq: Sequence):
        while len(seq.block_table) > seq.num_blocks:
            self._unref(seq.block_table.pop())
