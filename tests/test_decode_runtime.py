"""The native host decode runtime (include/vflorence_b200_runtime.h) against a plain-Python
restatement of the reference engine's bookkeeping, on random candidate streams (no GPU).

The restatement follows, in the vflorence project: block_manager.py:7-73 (FIFO free list,
reference counts, copy-on-write except for the last holder, release last block first),
scheduler.py:35-61 (capacity check, ensure_capacity in running order), scheduler.py:63-127
(greedy finish; beam split into finished / running, length-penalised ranking, early stop,
forks, release of every parent) and sequence.py:53-80 (fork, is_finished, score). Each step
both sides see the same candidates; the rows, tables, copy pairs and emitted tokens must agree.
"""

from __future__ import annotations

import random
from collections import deque

import numpy as np
import pytest

from vflorence_b200._native import VflError
from vflorence_b200.runtime import DecodeRules, DecodeRuntime

START, EOS = 0, 2


class _Seq:
    def __init__(self, rid, tokens, num_cached=0, cum=0.0):
        self.rid, self.tokens, self.num_cached, self.cum = rid, tokens, num_cached, cum
        self.table = []


class _Ref:
    """The reference's scheduler + block manager + sequence rules, restated."""

    def __init__(self, num_blocks, bs, nb, max_tokens, lp, early, eos):
        self.free = deque(range(num_blocks))
        self.rc = [0] * num_blocks
        self.bs, self.nb, self.max_tokens, self.lp, self.early, self.eos = bs, nb, max_tokens, lp, early, eos
        self.running, self.finished, self.out = [], {}, {}

    # block manager
    def _take(self):
        b = self.free.popleft()
        self.rc[b] = 1
        return b

    def required(self, seqs):
        need, left = 0, {}
        for s in seqs:
            i = s.num_cached // self.bs
            if i >= len(s.table):
                need += 1
                continue
            h = left.get(s.table[i], self.rc[s.table[i]])
            if h > 1:
                need += 1
                left[s.table[i]] = h - 1
        return need

    def ensure(self, s):
        i = s.num_cached // self.bs
        if i >= len(s.table):
            s.table.append(self._take())
            return None
        src = s.table[i]
        if self.rc[src] == 1:
            return None
        dst = self._take()
        self.rc[src] -= 1
        s.table[i] = dst
        return (src, dst)

    def fork_blocks(self, p, c):
        c.table = list(p.table)
        for b in c.table:
            self.rc[b] += 1

    def dealloc(self, s):
        for b in reversed(s.table):
            self.rc[b] -= 1
            if self.rc[b] == 0:
                self.free.append(b)
        s.table = []

    # sequence rules
    def done(self, s):
        return s.tokens[-1] in self.eos or len(s.tokens) - 1 >= self.max_tokens

    def score(self, s):
        return s.cum / (max(len(s.tokens) - 1, 1) ** self.lp)

    # scheduler
    def prepare(self):
        if self.required(self.running) > len(self.free):
            raise RuntimeError("KV cache is full")
        return [c for s in self.running if (c := self.ensure(s)) is not None]

    def advance_greedy(self, picks):
        seqs = list(self.running)
        for s in seqs:
            s.num_cached += 1
        done = []
        for s, t in zip(seqs, picks):
            s.tokens.append(int(t))
            if self.done(s):
                self.running.remove(s)
                self.dealloc(s)
                self.out[s.rid] = s.tokens[1:]
                done.append(s.rid)
        return done

    def advance_beam(self, cands):
        seqs = list(self.running)
        for s in seqs:
            s.num_cached += 1
        done = []
        for rid, cand in cands.items():
            fin = self.finished.setdefault(rid, [])
            run = []
            for rank, (row, tok, cum) in enumerate(cand):
                if rank >= self.nb and len(run) >= self.nb:
                    break
                p = seqs[row]
                c = _Seq(p.rid, p.tokens + [tok], p.num_cached, cum)
                if self.done(c):
                    if rank < self.nb:
                        fin.append(c)
                elif len(run) < self.nb:
                    run.append((p, c))
            fin.sort(key=self.score, reverse=True)
            del fin[self.nb:]
            best = max((self.score(c) for _, c in run), default=float("-inf"))
            if not run or (len(fin) >= self.nb and (self.early or self.score(fin[-1]) >= best)):
                self.finished.pop(rid, None)
                self.out[rid] = fin[0].tokens[1:]
                done.append(rid)
            else:
                for p, c in run:
                    self.fork_blocks(p, c)
                    self.running.append(c)
        for s in seqs:
            self.running.remove(s)
            self.dealloc(s)
        return done


def _run(seed, nb, num_requests, max_rows, max_tokens, lp, early, bs=4, vocab=9, ref_cls=_Ref):
    rng = random.Random(seed)
    num_blocks = 4 * max_rows * (-(-max_tokens // bs) + 1)
    K = 2 * nb
    ref = ref_cls(num_blocks, bs, nb, max_tokens, lp, early, {EOS})
    rt = DecodeRuntime(num_blocks, bs, (2 + K // nb) * max_rows + 4, -(-(max_tokens + 1) // bs))
    rules = DecodeRules(nb, max_tokens, lp, early, [EOS])
    waiting = deque(range(num_requests))
    active = set()
    rows_of = {}  # slot -> emulated device token row
    outputs = {}
    steps = 0
    while waiting or active:
        while waiting and (len(active) + 1) * nb <= max_rows:
            rid = waiting.popleft()
            slot = rt.admit(rid, START)
            rows_of[slot] = [START]
            ref.running.append(_Seq(rid, [START]))
            active.add(rid)
        copies = rt.prepare_step()
        assert [tuple(c) for c in copies.tolist()] == ref.prepare()
        width = -(-(max_tokens + 1) // bs)
        tables = np.zeros((max_rows, width), dtype=np.int32)
        rows = rt.pack_step(tables)
        n = rows.n
        assert n == len(ref.running)
        assert rows.request_ids.tolist() == [s.rid for s in ref.running]
        assert rows.positions.tolist() == [s.num_cached for s in ref.running]
        assert rows.lengths.tolist() == [len(s.tokens) for s in ref.running]
        assert rows.tokens.tolist() == [s.tokens[-1] for s in ref.running]
        for i, s in enumerate(ref.running):
            assert tables[i, : rows.table_lens[i]].tolist() == s.table
            assert rows_of[int(rows.slots[i])] == s.tokens
        if nb == 1:
            picks = np.array([rng.randrange(vocab) for _ in range(n)], dtype=np.int64)
            res = rt.advance_greedy(rules, picks)
            for i in range(n):
                rows_of[int(rows.slots[i])].append(int(picks[i]))
            want = ref.advance_greedy(picks.tolist())
        else:
            R = rows.num_groups
            order = list(dict.fromkeys(s.rid for s in ref.running))
            assert R == len(order)
            cand_r = np.full((R, K), -1, dtype=np.int32)
            cand_t = np.zeros((R, K), dtype=np.int32)
            cand_s = np.full((R, K), -np.inf, dtype=np.float32)
            cands = {}
            for g, rid in enumerate(order):
                members = [i for i in range(n) if rows.groups[i] == g]
                pool = [(r, t) for r in members for t in range(vocab)]
                picked = rng.sample(pool, min(K, len(pool)))
                sc = [np.float32(ref.running[r].cum - rng.choice([0.25, 0.5, 1.0, 1.5, 3.0])) for r, _ in picked]
                ordr = sorted(range(len(picked)), key=lambda j: -sc[j])  # stable
                lst = []
                for j, o in enumerate(ordr):
                    cand_r[g, j], cand_t[g, j] = picked[o]
                    cand_s[g, j] = sc[o]
                    lst.append((picked[o][0], picked[o][1], float(sc[o])))
                cands[rid] = lst
            res = rt.advance_beam(rules, cand_r, cand_t, cand_s)
            for p, c, pos, t in zip(res.born_parent, res.born_child, res.born_pos, res.born_token):
                rows_of[int(c)] = rows_of[int(p)][:pos] + [int(t)]
            want = ref.advance_beam(cands)
        assert res.done_request.tolist() == want
        for rid, slot, length in zip(res.done_request.tolist(), res.done_slot.tolist(), res.done_length.tolist()):
            outputs[rid] = rows_of[slot][1:length]
            active.discard(rid)
        steps += 1
    assert outputs == ref.out
    assert rt.num_running == 0
    assert rt.num_free_blocks == num_blocks and not any(rt.ref_counts())
    assert rt.free_block_ids() == list(ref.free)
    return steps


class _ReleaseFirstBlockFirst(_Ref):
    """Planted mistake: a finished sequence's blocks go back to the free list first block first
    (block_manager.py releases the last block first)."""

    def dealloc(self, s):
        for b in s.table:
            self.rc[b] -= 1
            if self.rc[b] == 0:
                self.free.append(b)
        s.table = []


class _PenaltyCountsStartToken(_Ref):
    """Planted mistake: the length penalty counts the decoder start token (sequence.py divides
    by the number of generated tokens)."""

    def score(self, s):
        return s.cum / (len(s.tokens) ** self.lp)


class _OneTokenLate(_Ref):
    """Planted mistake: a sequence finishes one token after max_tokens."""

    def done(self, s):
        return s.tokens[-1] in self.eos or len(s.tokens) - 1 > self.max_tokens


@pytest.mark.parametrize("mutant,nb,lp", [(_ReleaseFirstBlockFirst, 1, 1.0), (_ReleaseFirstBlockFirst, 3, 1.0),
                                          (_PenaltyCountsStartToken, 3, 2.0), (_OneTokenLate, 1, 1.0)])
def test_planted_mistakes_in_the_restatement_are_caught(mutant, nb, lp):
    """The comparison is sharp enough to see a one-rule slip in the restatement (the mistake is
    planted on the CPU side, in the Python restatement, never in the library)."""
    with pytest.raises(AssertionError):
        for seed in range(3):
            _run(200 + seed, nb=nb, num_requests=7, max_rows=3 * nb, max_tokens=10, lp=lp, early=False,
                 ref_cls=mutant)


@pytest.mark.parametrize("seed", range(4))
def test_greedy_matches_reference_bookkeeping(seed):
    assert _run(seed, nb=1, num_requests=12, max_rows=5, max_tokens=11, lp=1.0, early=False) > 11


@pytest.mark.parametrize("nb,lp,early", [(2, 1.0, False), (3, 2.0, False), (4, 0.5, True), (3, 1.0, True)])
@pytest.mark.parametrize("seed", range(3))
def test_beam_matches_reference_bookkeeping(seed, nb, lp, early):
    assert _run(100 + seed, nb=nb, num_requests=7, max_rows=3 * nb, max_tokens=10, lp=lp, early=early) > 5


def test_prepare_step_is_all_or_nothing():
    rt = DecodeRuntime(2, 4, 8, 4)
    for rid in range(3):
        rt.admit(rid, START)
    with pytest.raises(VflError, match="KV cache is full"):
        rt.prepare_step()
    # nothing was taken: a smaller batch still fits
    assert rt.num_free_blocks == 2


def test_runtime_argument_checks():
    rt = DecodeRuntime(8, 4, 8, 2)
    with pytest.raises(VflError, match="bad slot"):
        rt.deallocate(99)
    s = rt.slot_acquire()
    for n in (0, 4):
        rt.ensure_capacity(s, n)
    with pytest.raises(VflError, match="max_blocks_per_seq"):
        rt.ensure_capacity(s, 8)
    with pytest.raises(VflError, match="skips a block"):
        rt.ensure_capacity(rt.slot_acquire(), 8)
    rules = DecodeRules(2, 4, 1.0, False, [EOS])
    rt2 = DecodeRuntime(8, 4, 16, 4)
    rt2.admit(0, START)
    rt2.prepare_step()
    rt2.pack_step()
    bad = np.array([[1, -1, -1, -1]], dtype=np.int32)  # row 1 does not exist
    with pytest.raises(VflError, match="not a row"):
        rt2.advance_beam(rules, bad, np.zeros_like(bad), np.zeros(bad.shape, np.float32))
    with pytest.raises(VflError, match="no candidate"):
        rt2.advance_beam(rules, -np.ones_like(bad), np.zeros_like(bad), np.zeros(bad.shape, np.float32))


def test_pack_step_into_caller_buffers_matches_own_buffers():
    """The engine packs a step's rows straight into its pinned upload buffer: tables, positions
    and token ids as views of one int32 array. Those rows must equal the rows packed into the
    runtime's own buffers, step after step of a beam search."""
    nb, K, bs, max_tokens = 3, 6, 4, 10
    rt = DecodeRuntime(256, bs, 64, -(-(max_tokens + 1) // bs))
    rules = DecodeRules(nb, max_tokens, 1.0, False, [EOS])
    rng = random.Random(5)
    for rid in range(4):
        rt.admit(rid, START)
    B, M = 16, rt.max_blocks_per_seq
    flat = np.full(B * M + 2 * B, -7, dtype=np.int32)
    fields = ("table_lens", "positions", "tokens", "slots", "lengths", "request_ids", "groups", "ranks",
              "cum_logprobs")
    for _ in range(8):
        rt.prepare_step()
        own_tables = np.zeros((B, M), dtype=np.int32)
        own = rt.pack_step(own_tables)
        want = {f: np.copy(getattr(own, f)) for f in fields}
        want_groups, n = own.num_groups, own.n
        if n == 0:
            break
        tables, pos, tok = flat[: B * M].reshape(B, M), flat[B * M: B * M + B], flat[B * M + B:]
        got = rt.pack_step(tables, pos, tok)
        assert got.n == n and got.num_groups == want_groups
        for f in fields:
            assert np.array_equal(getattr(got, f), want[f]), f
        assert np.array_equal(tables[:n], own_tables[:n])
        assert np.array_equal(pos[:n], want["positions"]) and np.array_equal(tok[:n], want["tokens"])
        G = got.num_groups
        rows = np.full((G, K), -1, dtype=np.int32)
        toks = np.zeros((G, K), dtype=np.int32)
        scores = np.full((G, K), -np.inf, dtype=np.float32)
        for g in range(G):
            members = [i for i in range(n) if got.groups[i] == g]
            picks = sorted(((rng.choice(members), rng.randrange(3, 9), -rng.random() - 0.1) for _ in range(K)),
                           key=lambda c: -c[2])
            for j, (r, t, sc) in enumerate(picks):
                rows[g, j], toks[g, j], scores[g, j] = r, t, float(got.cum_logprobs[r]) + sc
            order = np.argsort(-scores[g], kind="stable")
            rows[g], toks[g], scores[g] = rows[g][order], toks[g][order], scores[g][order]
        rt.advance_beam(rules, rows, toks, scores)
