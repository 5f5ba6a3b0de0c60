"""Host-side bookkeeping around the kernels, checked against the reference engine's recorded
trace: encoder page allocation (vflorence/engine/model_runner.py:169-177, :232-265), step
packing (:290-306) and the beam grouping of the cross-attention staging (attention.py:9-39).
Also the measurement harness's CPU-side contracts: bench.py's reference arm, and the CPU engine
baseline's workload against bench.py's decode workload."""

from __future__ import annotations

import json
import os
import subprocess
import sys
import time

import pytest
import torch

from vflorence_b200.attention import group_rows
from vflorence_b200.kv_cache import CrossPageAllocator, pack_decode_step


def test_cross_pages_replay(engine_trace):
    for run in engine_trace["runs"]:
        alloc = CrossPageAllocator(run["num_cross_blocks"])
        clears = list(run["clears"])
        for enc in run["encodes"]:
            # apply the releases that happened before this encode
            while alloc.free != enc["cross_free_before"]:
                rid, free_after = clears.pop(0)
                alloc.release(rid)
                assert alloc.free == free_after
            for rids, n in enc["groups"]:
                pages = alloc.assign(rids, n, run["block_size"])
                for rid, row in zip(rids, pages):
                    assert torch.equal(row, enc["cross_pages"][rid][0])
            assert alloc.free == enc["cross_free_after"]
        for rid, free_after in clears:
            alloc.release(rid)
            assert alloc.free == free_after
        assert sorted(alloc.free) == list(range(run["num_cross_blocks"])) and not alloc.pages


def test_pack_decode_step_layout():
    host = pack_decode_step([[4, 9], [7], [1, 2, 3]], [20, 3, 40])
    assert host.tolist() == [4, 9, 0, 7, 0, 0, 1, 2, 3, 20, 3, 40]


def test_group_rows_by_shared_pages(engine_trace):
    a, b, c = torch.tensor([1, 2]), torch.tensor([3]), torch.tensor([4, 5])
    firsts, offsets = group_rows([a, a, a, b, c, c], [20, 20, 20, 7, 30, 30])
    assert firsts == [0, 3, 4] and offsets == [0, 3, 4, 6]
    # equal-valued but distinct tensors stay separate rows (identity marks one request)
    firsts, offsets = group_rows([a, a.clone()], [20, 20])
    assert offsets == [0, 1, 2]
    # in the reference's beam steps, the staged per-row table repeats each request's pages
    for run in engine_trace["runs"]:
        for step in run["steps"]:
            table, lens = step["cross_block_table"], step["cross_seq_lens"]
            rows = {}
            for i, rid in enumerate(step["request_ids"]):
                rows.setdefault(rid, []).append(i)
            for rid, idx in rows.items():
                assert all(torch.equal(table[i], table[idx[0]]) for i in idx)
                assert len({int(lens[i]) for i in idx}) == 1
            # beams of a request are consecutive rows, which is what group_rows relies on
            for idx in rows.values():
                assert idx == list(range(idx[0], idx[0] + len(idx)))


def test_cpu_engine_baseline_times_the_bench_workload():
    """The reference CPU engine timing (oracle/reference_engine_cpu.py) runs configs 1-4 on the
    same model shapes, requests (ids and images), sampling and pool sizes as bench.py --decode cfgN."""
    import bench
    import reference_engine_cpu as ref

    for name in ("cfg1", "cfg2", "cfg3", "cfg4"):
        ours, theirs = bench.decode_config(name), ref.CONFIGS[name]
        kind = theirs.get("kind", "bart")
        if kind == "bart":
            assert ours["text"] == ref.BART_LARGE
        else:
            assert (ours["text"], ours["vision"]) == ref.SHAPES[kind]
            ours["image_tokens"] = ref.IMAGE_TOKENS  # bench reads it off the built tower
        for key in ("dtype", "num_requests", "params", "max_num_seqs", "max_decoder_len", "max_encoder_len"):
            assert ours[key] == theirs[key], (name, key)
        if name == "cfg4":  # 512 images: compare the first few
            ours["num_requests"] = 6
            theirs = dict(theirs, num_requests=6)
        mine = bench.decode_requests(ours, "cpu")
        want = ref.requests_of(theirs)
        assert [r.input_ids for r in mine] == [ids for ids, _ in want]
        for r, (_, px) in zip(mine, want):
            assert (r.pixel_values is None and px is None) or torch.equal(r.pixel_values, px)


def _bench_reference(env_extra):
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, os.path.join(repo, "bench.py"), "--impl", "reference", "--steps", "3",
                          "--warmup", "3", "--batch", "64", "--cpu-sample", "4"],
                         capture_output=True, text=True, timeout=300, env=env, cwd=repo)
    assert res.returncode == 0, res.stderr[-2000:]
    return [json.loads(line) for line in res.stdout.splitlines() if line.startswith("{")]


def test_bench_reference_arm_prints_one_line():
    """bench.py --impl reference (the reference's CPU path, no GPU needed) prints one JSON line
    with the metric of the GPU arm, a cpu_baseline describing the run and a zero-copy e2e."""
    (line,) = _bench_reference({})
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["metric"] == "paged-attn HBM GB/s vs 8 TB/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["config"]["batch_per_gpu"] == 64


def test_bench_reference_arm_other_ranks_exit_quietly():
    """Under torchrun only rank 0 runs the reference arm; the other ranks print nothing."""
    assert _bench_reference({"WORLD_SIZE": "2", "RANK": "1", "LOCAL_RANK": "1"}) == []


def test_bench_clock_summary_reads_throttle_reasons(tmp_path, monkeypatch):
    """bench.py's clock record: the median SM clock under load, the max clock, the peak power and
    every throttle reason seen active in the nvidia-smi trace (a fake trace here, no GPU)."""
    import bench

    monkeypatch.setenv("VFL_CLOCKS_DIR", str(tmp_path))
    cs = bench.ClockSampler(0)
    with open(cs.path, "w") as f:
        f.write("1965, 1965, 410.5, 0x0, Not Active, Not Active, Not Active, Not Active\n")
        f.write("1770, 1965, 998.1, 0x4, Not Active, Not Active, Not Active, Active\n")
        f.write("1755, 1965, 1001.0, 0x4, Not Active, Not Active, Not Active, Active\n")
        f.write("garbled line\n")
    cs.proc = object()  # as if nvidia-smi had run
    s = cs.summary()
    assert s["sm_mhz"] == 1770 and s["sm_max_mhz"] == 1965 and s["samples"] == 3
    assert s["power_w_max"] == 1001.0 and s["reasons"] == ["sw_power_cap"]
    with open(cs.path, "a") as f:
        f.write("1500, 1965, 700.0, 0x40, Not Active, Active, Not Active, Not Active\n")
    assert cs.summary()["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]


def test_bench_algorithmic_bytes_and_workload():
    """The roofline numerator: the minimum HBM bytes of one bench step, by the formulas of the
    measurement notes (K/V read once per token, q and out once per row, the table slice, lengths
    and query offsets; the append reads and writes each new K/V row plus its slot; cross-attention
    reads each encoder token once). And the workload's block tables are a permutation of the pool
    whose slots land on each sequence's newest position."""
    import bench

    w = dict(batch=3, ctx=torch.tensor([1, 16, 17], dtype=torch.int32))
    row = 16 * 64 * 2  # one token's K (or V) over 16 heads of 64, bf16
    nb = bench.algorithmic_bytes(w)
    assert nb["self"] == 2 * 34 * row + 2 * 3 * row + 4 * (1 + 1 + 2) + 4 * 3 + 4 * 4
    assert nb["append"] == 4 * 3 * row + 8 * 3
    assert nb["cross"] == 2 * 3 * 1024 * row + 2 * 3 * row + 4 * 3 * 64 + 4 * 3 + 4 * 4
    assert nb["total"] == nb["self"] + nb["append"] + nb["cross"]

    w = bench.make_workload(9, 2, None)
    ctx, table, slots = w["ctx"], w["table"], w["slots"]
    nblk = (ctx + 15) // 16
    used = torch.cat([table[b, : nblk[b]] for b in range(9)])
    assert sorted(used.tolist()) == list(range(w["n_self"]))
    assert sorted(w["cross_table"].flatten().tolist()) == list(range(w["n_cross"]))
    pos = (ctx - 1).long()
    assert torch.equal(slots // 16, table[torch.arange(9), pos // 16].long()) and torch.equal(slots % 16, pos % 16)


class _FakeEngine:
    """Engine stand-in for the arrival loop: each request finishes 3 steps after its admission."""

    def __init__(self):
        self.queue, self.outputs, self.added_at, self.step_count = [], {}, {}, 0
        self.next = 0

    def add_request(self, req, params):
        rid = self.next
        self.next += 1
        self.queue.append([rid, 3])
        self.added_at[rid] = time.perf_counter()
        return rid

    def is_finished(self):
        return not self.queue

    def abort(self):
        self.queue.clear()
        self.aborted = True

    def step(self):
        self.step_count += 1
        done = []
        for item in self.queue:
            item[1] -= 1
            if item[1] == 0:
                done.append(item[0])
                self.outputs[item[0]] = [item[0]] * 2
        self.queue = [q for q in self.queue if q[1] > 0]
        return done


def test_poisson_arrivals_and_serving_loop():
    """bench.py's arrival process is seeded and increasing with the stated mean gap; the serving
    loop adds no request before its arrival time, returns outputs in request order and a
    non-negative latency per request."""
    import bench

    a = bench.poisson_arrivals(2000, 500.0)
    assert a == bench.poisson_arrivals(2000, 500.0)
    assert all(x < y for x, y in zip(a, a[1:]))
    assert abs(a[-1] / 2000 - 1 / 500) < 0.1 / 500
    arrivals = [0.0, 0.0, 0.02, 0.05]
    eng = _FakeEngine()
    t0 = time.perf_counter()
    outs, lat = bench.serve_arrivals(eng, ["r0", "r1", "r2", "r3"], None, arrivals)
    assert outs == [[0, 0], [1, 1], [2, 2], [3, 3]]
    assert all(x >= 0 for x in lat) and len(lat) == 4
    for rid, t in eng.added_at.items():
        assert t - t0 >= arrivals[rid] - 1e-3


def test_serving_loop_aborts_the_engine_on_a_failed_step():
    """A step that raises leaves no request half-served: the loop aborts the engine and re-raises."""
    import bench

    eng = _FakeEngine()

    def failing_step():
        raise RuntimeError("planted step failure")

    eng.step = failing_step
    with pytest.raises(RuntimeError, match="planted"):
        bench.serve_arrivals(eng, ["r0", "r1"], None, [0.0, 0.0])
    assert getattr(eng, "aborted", False) and eng.is_finished()
