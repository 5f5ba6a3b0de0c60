"""Paged KV block allocator with reference counts and copy-on-write (host side).

Its decisions are what the device ops consume: the block ids in every block table, the slot
of every appended token and the (src, dst) copy-on-write pairs. They must equal the reference
allocator's (vflorence/engine/block_manager.py:1-73) bit for bit, so the policy is the same:

  * free blocks are handed out first-in first-out: allocation takes the oldest free id, a
    freed id joins the back of the queue (block_manager.py:15, :24, :72);
  * a sequence's blocks are released last block first (block_manager.py:69-72);
  * a token written into a block held by several sequences goes to a private copy, except for
    the last holder, which writes in place (block_manager.py:28-59).
"""

from __future__ import annotations

from collections import deque


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.reset()

    def reset(self) -> None:
        """Forget every allocation (after an aborted batch)."""
        self.ref_counts = [0] * self.num_blocks
        self.free_block_ids = deque(range(self.num_blocks))

    @property
    def num_free_blocks(self) -> int:
        return len(self.free_block_ids)

    def _take(self) -> int:
        if not self.free_block_ids:
            raise RuntimeError("KV cache is full; increase num_blocks")
        block = self.free_block_ids.popleft()
        self.ref_counts[block] = 1
        return block

    def _next_index(self, seq) -> int:
        return seq.num_cached_tokens // self.block_size

    def required_new_blocks(self, seqs) -> int:
        """Blocks that appending one token to every sequence in ``seqs`` will take: fresh
        blocks plus private copies of shared blocks (all holders but the last copy)."""
        needed = 0
        left = {}  # shared block -> holders that have not claimed a copy yet
        for seq in seqs:
            idx = self._next_index(seq)
            if idx >= len(seq.block_table):
                needed += 1
                continue
            block = seq.block_table[idx]
            holders = left.get(block, self.ref_counts[block])
            if holders > 1:
                needed += 1
                left[block] = holders - 1
        return needed

    def ensure_capacity(self, seq) -> tuple[int, int] | None:
        """Make the block that ``seq``'s next token lands in writable.

        Appends a fresh block when the table is full, or swaps a shared block for a private one
        and returns the ``(src, dst)`` pair whose contents must be copied before the write.
        """
        idx = self._next_index(seq)
        if idx >= len(seq.block_table):
            seq.block_table.append(self._take())
            return None
        src = seq.block_table[idx]
        if self.ref_counts[src] == 1:
            return None
        dst = self._take()
        self.ref_counts[src] -= 1
        seq.block_table[idx] = dst
        return src, dst

    def fork(self, parent, child) -> None:
        """``child`` shares every block of ``parent`` (one more reference each)."""
        child.block_table = list(parent.block_table)
        for block in child.block_table:
            self.ref_counts[block] += 1

    def deallocate(self, seq) -> None:
        """Drop ``seq``'s references, last block first; blocks nobody holds become free."""
        for block in reversed(seq.block_table):
            self.ref_counts[block] -= 1
            if self.ref_counts[block] == 0:
                self.free_block_ids.append(block)
        seq.block_table.clear()
