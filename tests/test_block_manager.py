"""BlockManager decisions equal the reference allocator's, replayed call by call from the
reference engine's recorded log (tests/golden/engine_trace.pt), plus the reference's own unit
checks (vflorence tests/test_engine.py:79-87, :361-405)."""

from __future__ import annotations

import pytest

from vflorence_b200.block_manager import BlockManager


class Seq:
    def __init__(self, num_cached_tokens=0):
        self.block_table = []
        self.num_cached_tokens = num_cached_tokens


def _replay(run):
    bm = BlockManager(run["num_blocks"], run["block_size"])
    seqs = {}
    log = run["bm_log"]
    checked = 0
    for i, op in enumerate(log):
        kind = op[0]
        if kind == "reset":
            bm.reset()
        elif kind == "required":
            ids, want = op[1], op[2]
            # each sequence's cached count at this point is the one its next ensure records
            for sid in ids:
                seq = seqs.setdefault(sid, Seq())
                for later in log[i + 1:]:
                    if later[0] == "ensure" and later[1] == sid:
                        seq.num_cached_tokens = later[2]
                        break
            assert bm.required_new_blocks([seqs[s] for s in ids]) == want
            checked += 1
        elif kind == "ensure":
            _, sid, cached, before, want, after = op
            seq = seqs.setdefault(sid, Seq())
            seq.num_cached_tokens = cached
            assert seq.block_table == before
            assert bm.ensure_capacity(seq) == want
            assert seq.block_table == after
            checked += 1
        elif kind == "fork":
            _, parent, child, table = op
            seqs[child] = Seq()
            bm.fork(seqs[parent], seqs[child])
            assert seqs[child].block_table == table
        elif kind == "dealloc":
            _, sid, table, free_after = op
            assert seqs[sid].block_table == table
            bm.deallocate(seqs[sid])
            assert list(bm.free_block_ids) == free_after
            checked += 1
        else:
            raise AssertionError(kind)
    assert bm.num_free_blocks == bm.num_blocks and not any(bm.ref_counts)
    return checked


def test_replay_reference_allocator(engine_trace):
    total = sum(_replay(run) for run in engine_trace["runs"])
    assert total > 300


def test_cache_full_raises():
    bm = BlockManager(2, 16)
    seqs = [Seq() for _ in range(3)]
    bm.ensure_capacity(seqs[0])
    bm.ensure_capacity(seqs[1])
    assert bm.required_new_blocks(seqs[2:]) == 1
    with pytest.raises(RuntimeError, match="KV cache is full"):
        bm.ensure_capacity(seqs[2])


def test_copy_budget_preserves_nonwriting_owner():
    bm = BlockManager(8, 16)
    parent = Seq()
    bm.ensure_capacity(parent)
    parent.num_cached_tokens = 1
    children = [Seq(1), Seq(1)]
    for c in children:
        bm.fork(parent, c)
    assert bm.required_new_blocks(children) == 2
    bm.deallocate(parent)
    assert bm.required_new_blocks(children) == 1


def test_copy_on_write_pair_and_refcounts():
    bm = BlockManager(8, 16)
    parent = Seq()
    assert bm.ensure_capacity(parent) is None
    parent.num_cached_tokens = 1
    child = Seq(1)
    bm.fork(parent, child)
    src = parent.block_table[0]
    pair = bm.ensure_capacity(child)
    assert pair == (src, child.block_table[0]) and pair[1] != src
    assert (bm.ref_counts[src], bm.ref_counts[pair[1]]) == (1, 1)
    # the last holder writes in place
    assert bm.ensure_capacity(parent) is None


def test_free_order_is_fifo_last_block_first():
    bm = BlockManager(6, 16)
    s = Seq()
    for n in range(3):
        s.num_cached_tokens = 16 * n
        bm.ensure_capacity(s)
    assert s.block_table == [0, 1, 2]
    bm.deallocate(s)
    assert list(bm.free_block_ids) == [3, 4, 5, 2, 1, 0]
