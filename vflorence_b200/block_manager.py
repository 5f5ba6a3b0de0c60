"""Paged KV block allocator with reference counts and copy-on-write (host side).

Its decisions are what the device ops consume: the block ids in every block table, the slot
of every appended token and the (src, dst) copy-on-write pairs. They must equal the reference
allocator's (vflorence/engine/block_manager.py:1-73) bit for bit, so the policy is the same:

  * free blocks are handed out first-in first-out: allocation takes the oldest free id, a
    freed id joins the back of the queue (block_manager.py:15, :24, :72);
  * a sequence's blocks are released last block first (block_manager.py:69-72);
  * a token written into a block held by several sequences goes to a private copy, except for
    the last holder, which writes in place (block_manager.py:28-59).

The bookkeeping itself is native (``vfl_rt_*`` of the host decode runtime); this class keeps
the reference's interface on sequence objects (anything with ``block_table`` and
``num_cached_tokens``), mirroring each sequence's table after every call.
"""

from __future__ import annotations

from .runtime import DecodeRuntime


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, *, num_slots: int = 1024,
                 max_blocks_per_seq: int | None = None, runtime: DecodeRuntime | None = None):
        if num_blocks <= 0 or block_size <= 0:
            raise ValueError("num_blocks and block_size must be positive")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.rt = runtime or DecodeRuntime(num_blocks, block_size, num_slots, max_blocks_per_seq or num_blocks)
        self._generation = 0

    @classmethod
    def over(cls, runtime: DecodeRuntime) -> "BlockManager":
        """A view of an engine's runtime (the engine drives it through the batched calls)."""
        return cls(runtime.num_blocks, runtime.block_size, runtime=runtime)

    def reset(self) -> None:
        """Forget every allocation (after an aborted batch)."""
        self.rt.reset()
        self._generation += 1

    @property
    def num_free_blocks(self) -> int:
        return self.rt.num_free_blocks

    @property
    def free_block_ids(self) -> list[int]:
        """Free block ids in hand-out order."""
        return self.rt.free_block_ids()

    @property
    def ref_counts(self) -> list[int]:
        return self.rt.ref_counts()

    def _slot(self, seq) -> int:
        if getattr(seq, "_bm_owner", None) != (id(self), self._generation):
            seq._bm_slot = self.rt.slot_acquire()
            seq._bm_owner = (id(self), self._generation)
        return seq._bm_slot

    def required_new_blocks(self, seqs) -> int:
        """Blocks that appending one token to every sequence in ``seqs`` will take: fresh
        blocks plus private copies of shared blocks (all holders but the last copy)."""
        seqs = list(seqs)
        return self.rt.required_new_blocks([self._slot(s) for s in seqs], [s.num_cached_tokens for s in seqs])

    def ensure_capacity(self, seq) -> tuple[int, int] | None:
        """Make the block that ``seq``'s next token lands in writable.

        Appends a fresh block when the table is full, or swaps a shared block for a private one
        and returns the ``(src, dst)`` pair whose contents must be copied before the write.
        """
        slot = self._slot(seq)
        pair = self.rt.ensure_capacity(slot, seq.num_cached_tokens)
        seq.block_table[:] = self.rt.block_table(slot)
        return pair

    def fork(self, parent, child) -> None:
        """``child`` shares every block of ``parent`` (one more reference each)."""
        slot = self._slot(child)
        self.rt.fork(self._slot(parent), slot)
        child.block_table = self.rt.block_table(slot)

    def deallocate(self, seq) -> None:
        """Drop ``seq``'s references, last block first; blocks nobody holds become free."""
        slot = self._slot(seq)
        self.rt.deallocate(slot)
        seq.block_table.clear()
        self.rt.slot_release(slot)
        seq._bm_owner = None
