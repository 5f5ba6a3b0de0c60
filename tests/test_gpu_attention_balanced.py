"""The balanced schedule of the tensor-core attention kernel (bf16, head_dim 64) against the CPU
oracle: one persistent wave of CTAs, equal runs of 16-token tiles, items cut across CTAs and
merged by a programmatic dependent launch.

Cases cover few and many requests, beam rows sharing pages, causal rows, zero-length and
skewed lengths, head groups of 1, 2 and 4 heads, 16- and 32-token blocks, tiny and large runs
(min_tiles 1 and 64: items cut into many pieces, or whole), the fused KV append, a workspace
holding stale records, and a CUDA graph replayed with lengths other than the planned ones.
Tolerance: bfloat16 2e-2 absolute (assert_attention_close).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import assert_attention_close
from test_gpu_attention import _appended_case, oracle_attn, random_case

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def ops():
    from vflorence_b200 import paged_ops

    return paged_ops


def balanced_meta(lens, qsl, heads, block_size, causal=False, min_tiles=0):
    o = ops()
    meta = o.get_scheduler_metadata(lens.numel(), heads, heads, 64, lens, torch.bfloat16, qsl, causal, "sm100",
                                    block_size)
    o.set_schedule(meta, o.SCHEDULE_BALANCED, min_tiles)
    p = o.plan_of(meta)
    assert p.schedule == o.SCHEDULE_BALANCED and p.balanced_ctas > 0
    return meta


@pytest.mark.parametrize("requests,rows,heads,block_size,min_len,max_len,min_tiles,causal,seed", [
    (32, 4, 16, 16, 768, 1024, 0, False, 1),    # cross-attention, beams of 32 requests
    (64, 3, 16, 16, 587, 587, 0, False, 2),     # equal encoder lengths
    (85, 3, 16, 16, 560, 592, 0, False, 3),
    (8, 1, 16, 16, 1, 4096, 0, False, 4),       # few long requests: items cut into many pieces
    (40, 1, 16, 16, 0, 700, 0, False, 5),       # skewed, with zero-length requests
    (20, 2, 6, 32, 1, 900, 0, False, 6),        # two heads per CTA, 32-token blocks
    (10, 1, 3, 16, 1, 300, 0, False, 7),        # one head per CTA
    (16, 1, 16, 16, 1000, 2000, 1, False, 8),   # one-tile runs allowed: every CTA of the wave
    (16, 4, 16, 16, 1000, 2000, 64, False, 9),  # long runs: fewer CTAs, whole items
    (12, 8, 16, 16, 8, 600, 0, True, 10),       # causal rows, up to 8 per request
    (2048, 1, 16, 16, 1, 200, 0, False, 11),    # the most requests the schedule takes
    (1, 1, 16, 16, 3000, 3000, 0, False, 12),   # one request over the whole wave
])
def test_balanced_matches_oracle(oracle_lib, requests, rows, heads, block_size, min_len, max_len, min_tiles,
                                 causal, seed):
    o = ops()
    g = torch.Generator().manual_seed(seed)
    q_lens = [rows] * requests
    if causal:
        q_lens = [int(torch.randint(1, rows + 1, (1,), generator=g)) for _ in range(requests)]
    q, kc, vc, qsl, lens, table = random_case(num_reqs=requests, heads=heads, head_dim=64, block_size=block_size,
                                              max_len=max_len, min_len=min_len, dtype=torch.bfloat16,
                                              q_lens=q_lens, seed=seed)
    if causal:
        lens = torch.maximum(lens, torch.tensor(q_lens, dtype=torch.int32))
    meta = balanced_meta(lens, qsl, heads, block_size, causal, min_tiles)
    out = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
    o.attention_with_kv_cache(q.to(DEV), kc.to(DEV), vc.to(DEV), out, qsl.to(DEV), lens.to(DEV), 64 ** -0.5,
                              causal, table.to(DEV), meta)
    torch.cuda.synchronize()
    assert o.read_device_errors(DEV) == 0
    want = oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, 64 ** -0.5, causal)
    assert_attention_close(out.cpu(), want, torch.bfloat16, f"balanced seed {seed}")


def _call_native(meta, q, kc, vc, out, qsl, lens, table, ws):
    from vflorence_b200 import _native as N

    o = ops()
    plan = o.plan_of(meta)
    n = kc.shape[0]
    st = N.lib().vfl_attention_with_kv_cache(
        ctypes.byref(plan), q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(), n, out.data_ptr(),
        out.stride(0), qsl.data_ptr(), lens.data_ptr(), table.data_ptr(), table.stride(0), table.shape[1],
        ctypes.c_float(64 ** -0.5), ws.data_ptr(), ws.numel(), torch.cuda.current_stream(DEV).cuda_stream)
    N.check(st, "attention")


def test_balanced_ignores_stale_workspace(oracle_lib):
    """Every item's directory entry is written on every call: a workspace left by a call with
    other lengths, or filled with plausible piece counts, does not leak into the merge."""
    g = torch.Generator().manual_seed(21)
    ws = None
    for seed, (lo, hi) in ((22, (1500, 2000)), (23, (1, 300)), (24, (0, 40))):
        q, kc, vc, qsl, lens, table = random_case(num_reqs=24, heads=16, head_dim=64, block_size=16, max_len=hi,
                                                  min_len=lo, dtype=torch.bfloat16, q_lens=[2] * 24, seed=seed)
        meta = balanced_meta(lens, qsl, 16, 16)
        need = ops().plan_of(meta).workspace_bytes
        if ws is None or ws.numel() < need:
            ws = torch.randint(0, 5, (need // 4,), generator=g, dtype=torch.int32).to(DEV).view(torch.uint8)
        out = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
        _call_native(meta, q.to(DEV), kc.to(DEV), vc.to(DEV), out, qsl.to(DEV), lens.to(DEV), table.to(DEV), ws)
        torch.cuda.synchronize()
        assert ops().read_device_errors(DEV) == 0
        want = oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, 64 ** -0.5)
        assert_attention_close(out.cpu(), want, torch.bfloat16, f"stale workspace, seed {seed}")


@pytest.mark.parametrize("kind,seed,block_size,max_len,requests,min_tiles", [
    ("rows", 31, 16, 200, 40, 0), ("rows", 32, 16, 4000, 9, 0), ("rows", 33, 32, 1500, 17, 3),
    ("causal", 34, 16, 600, 12, 0), ("causal", 35, 32, 2000, 5, 1)])
def test_balanced_append_equals_append_then_attend(kind, seed, block_size, max_len, requests, min_tiles):
    """The fused append under the balanced schedule: the piece that holds a row's new position
    stores it before loading that tile; output and pools equal append-then-attend with the same
    plan, bit for bit."""
    o = ops()
    q, key, value, kc, vc, qsl, lens, table, slots = _appended_case(kind, seed, block_size, max_len, requests)
    causal = kind == "causal"
    meta = balanced_meta(lens, qsl, kc.shape[1], block_size, causal, min_tiles)
    assert o.attention_append_supported(meta)
    dq, dl, dt, ds = qsl.to(DEV), lens.to(DEV), table.to(DEV), slots.to(DEV)
    kc2, vc2 = kc.clone(), vc.clone()
    o.reshape_and_cache(key, value, kc2, vc2, ds)
    want = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
    o.attention_with_kv_cache(q, kc2, vc2, want, dq, dl, 64 ** -0.5, causal, dt, meta)
    got = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
    o.attention_with_kv_cache_append(q, key, value, kc, vc, got, ds, dq, dl, 64 ** -0.5, causal, dt, meta)
    torch.cuda.synchronize()
    assert o.read_device_errors(DEV) == 0
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(got, want)


def test_balanced_plan_in_a_cuda_graph_follows_the_lengths(oracle_lib):
    """A balanced call captured in a CUDA graph (the merge as a programmatic dependent launch in
    the graph) lays out its runs from the device lengths of each replay."""
    o = ops()
    q, kc, vc, qsl, lens, table = random_case(num_reqs=48, heads=16, head_dim=64, block_size=16, max_len=1024,
                                              min_len=1024, dtype=torch.bfloat16, q_lens=[3] * 48, seed=41,
                                              on_device=True)
    meta = balanced_meta(lens, qsl, 16, 16)
    dq, dl, dt = qsl.to(DEV), lens.to(DEV), table.to(DEV)
    out = torch.zeros_like(q)
    o.attention_with_kv_cache(q, kc, vc, out, dq, dl, 64 ** -0.5, False, dt, meta)  # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o.attention_with_kv_cache(q, kc, vc, out, dq, dl, 64 ** -0.5, False, dt, meta)
    g = torch.Generator().manual_seed(42)
    for step in range(3):
        new = torch.randint(0, 1025, (48,), generator=g, dtype=torch.int32)
        new[step::7] = 0
        dl.copy_(new)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert o.read_device_errors(DEV) == 0
        want = oracle_attn(oracle_lib, q.cpu(), kc.cpu(), vc.cpu(), qsl, new, table, 64 ** -0.5)
        assert_attention_close(out.cpu(), want, torch.bfloat16, f"graph replay {step}")
    del graph


def test_balanced_flags_bad_block_ids():
    """A block id outside the pool is reported and read as block 0, as in the item grid."""
    o = ops()
    from vflorence_b200 import _native

    q, kc, vc, qsl, lens, table = random_case(num_reqs=6, heads=16, head_dim=64, block_size=16, max_len=400,
                                              min_len=300, dtype=torch.bfloat16, seed=51, on_device=True)
    table[3, 2] = kc.shape[0] + 5
    meta = balanced_meta(lens, qsl, 16, 16)
    out = torch.empty_like(q)
    o.attention_with_kv_cache(q, kc, vc, out, qsl.to(DEV), lens.to(DEV), 64 ** -0.5, False, table.to(DEV), meta)
    assert o.read_device_errors(DEV) & _native.DEVERR_BLOCK_ID
    assert bool(torch.isfinite(out.float()).all())
