"""Paged attention on the GPU (through the C ABI) against the CPU oracle and the float64 fixtures.

Tolerances (assert_attention_close): float32 1e-5 relative (scaled to the output magnitude),
bfloat16 2e-2 absolute. At the BASELINE sweep's full size (1024 sequences, contexts up to 4096)
the oracle checks a sample of rows and size-independent properties cover the rest.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import assert_attention_close, case_tensors, load_attention_cases

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
CASES = load_attention_cases()


def ops():
    from vflorence_b200 import paged_ops

    return paged_ops


def kernel(q, kc, vc, qsl, lens, table, scale, causal=False, *, device_lens=None):
    o = ops()
    n, h, bs, d = kc.shape
    meta = o.get_scheduler_metadata(lens.numel(), h, h, d, lens, kc.dtype, qsl, causal, "sm100", bs)
    out = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
    o.attention_with_kv_cache(q.to(DEV), kc.to(DEV), vc.to(DEV), out, qsl.to(DEV),
                              (lens if device_lens is None else device_lens).to(DEV), scale, causal,
                              table.to(DEV), meta)
    return out.cpu(), o.plan_of(meta)


def oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, scale, causal=False):
    out = torch.empty_like(q)
    assert oracle_lib.attention(q, kc, vc, out, qsl, lens, scale, causal, table) == 0
    return out


def random_case(*, num_reqs, heads, head_dim, block_size, max_len, dtype, q_lens=None, seed=0,
                min_len=0, extra_blocks=3, on_device=False):
    """Seeded paged case: lengths U[min_len, max_len], block tables a random permutation of the
    pool, K/V/q N(0, 1) (drawn on the GPU; returned there when ``on_device``)."""
    g = torch.Generator().manual_seed(seed)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    lens = torch.randint(min_len, max_len + 1, (num_reqs,), generator=g, dtype=torch.int32)
    need = [max(1, math.ceil(int(n) / block_size)) for n in lens]
    nb = sum(need) + extra_blocks
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    table = torch.zeros(num_reqs, max(need), dtype=torch.int32)
    pos = 0
    for r, k in enumerate(need):
        table[r, :k] = perm[pos:pos + k]
        pos += k
    kc = torch.randn(nb, heads, block_size, head_dim, generator=gd, device=DEV, dtype=dtype)
    vc = torch.randn(nb, heads, block_size, head_dim, generator=gd, device=DEV, dtype=dtype)
    q_lens = q_lens or [1] * num_reqs
    qsl = torch.tensor([0] + list(torch.tensor(q_lens).cumsum(0).tolist()), dtype=torch.int32)
    q = torch.randn(int(qsl[-1]), heads, head_dim, generator=gd, device=DEV, dtype=dtype)
    if not on_device:
        q, kc, vc = q.cpu(), kc.cpu(), vc.cpu()
    return q, kc, vc, qsl, lens, table


def compact_sample(kc, vc, table, lens, rows, block_size):
    """CPU copies of only the blocks that ``rows`` read, with their table remapped."""
    need = [max(1, math.ceil(int(lens[r]) / block_size)) for r in rows.tolist()]
    ids = torch.cat([table[r, :k] for r, k in zip(rows.tolist(), need)]).long()
    uniq, inv = torch.unique(ids, return_inverse=True)
    sub = torch.zeros(len(need), max(need), dtype=torch.int32)
    pos = 0
    for i, k in enumerate(need):
        sub[i, :k] = inv[pos:pos + k].to(torch.int32)
        pos += k
    dev_ids = uniq.to(kc.device)
    return kc[dev_ids].cpu(), vc[dev_ids].cpu(), sub


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_fixture_cases(oracle_lib, case):
    t = case_tensors(case)
    dt = t["q"].dtype
    got, _ = kernel(t["q"], t["k_cache"], t["v_cache"], t["query_start_loc"], t["seq_lens"],
                    t["block_table"], case["scale"], bool(case["causal"]))
    assert_attention_close(got, t["expected"], dt, case["name"] + " vs float64")
    ref = oracle_attn(oracle_lib, t["q"], t["k_cache"], t["v_cache"], t["query_start_loc"],
                      t["seq_lens"], t["block_table"], case["scale"], bool(case["causal"]))
    assert_attention_close(got, ref, dt, case["name"] + " vs oracle")


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_fixture_cases_other_dtype(oracle_lib, case):
    other = torch.bfloat16 if case["dtype"] == "f32" else torch.float32
    t = case_tensors(case, other)
    got, _ = kernel(t["q"], t["k_cache"], t["v_cache"], t["query_start_loc"], t["seq_lens"],
                    t["block_table"], case["scale"], bool(case["causal"]))
    ref = oracle_attn(oracle_lib, t["q"], t["k_cache"], t["v_cache"], t["query_start_loc"],
                      t["seq_lens"], t["block_table"], case["scale"], bool(case["causal"]))
    assert_attention_close(got, ref, other, case["name"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("head_dim", [32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 512])
@pytest.mark.parametrize("block_size", [16, 32])
def test_head_dims_and_block_sizes(oracle_lib, dtype, head_dim, block_size):
    heads = 4 if head_dim <= 128 else 2
    q, kc, vc, qsl, lens, table = random_case(num_reqs=6, heads=heads, head_dim=head_dim,
                                              block_size=block_size, max_len=300, dtype=dtype,
                                              seed=head_dim + block_size)
    got, _ = kernel(q, kc, vc, qsl, lens, table, head_dim ** -0.5)
    ref = oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, head_dim ** -0.5)
    assert_attention_close(got, ref, dtype, f"D={head_dim} bs={block_size}")


@pytest.mark.parametrize("heads", [1, 2, 3, 12, 16])
def test_head_counts(oracle_lib, heads):
    q, kc, vc, qsl, lens, table = random_case(num_reqs=5, heads=heads, head_dim=64, block_size=16,
                                              max_len=200, dtype=torch.bfloat16, seed=heads)
    got, plan = kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert heads % plan.heads_per_cta == 0
    assert_attention_close(got, oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, 0.125),
                           torch.bfloat16, f"H={heads}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_grouped_rows_share_pages(oracle_lib, dtype):
    # beams of one request as several query rows (up to 9 -> three chunks of four)
    q_lens = [3, 1, 4, 9, 2, 5]
    q, kc, vc, qsl, lens, table = random_case(num_reqs=6, heads=12, head_dim=64, block_size=16,
                                              max_len=1024, min_len=300, dtype=dtype, q_lens=q_lens,
                                              seed=5)
    got, plan = kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert plan.queries_per_cta == (8 if dtype == torch.bfloat16 else 4)
    assert_attention_close(got, oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, 0.125), dtype,
                           "grouped")
    # grouped rows equal the per-row (repeated table) computation
    rows = torch.repeat_interleave(torch.arange(6), torch.tensor(q_lens))
    got_rows, _ = kernel(q, kc, vc, torch.arange(q.shape[0] + 1, dtype=torch.int32), lens[rows],
                         table[rows].contiguous(), 0.125)
    assert_attention_close(got_rows, got, dtype, "grouped vs per-row")


def test_causal_rows(oracle_lib):
    q, kc, vc, qsl, lens, table = random_case(num_reqs=4, heads=2, head_dim=64, block_size=16,
                                              max_len=90, min_len=1, dtype=torch.float32,
                                              q_lens=[1, 5, 3, 8], seed=9)
    got, _ = kernel(q, kc, vc, qsl, lens, table, 0.125, causal=True)
    ref = oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, 0.125, causal=True)
    assert_attention_close(got, ref, torch.float32, "causal")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_split_k_long_contexts(oracle_lib, dtype):
    # few long requests: the planner splits them; results must equal the unsplit oracle
    q, kc, vc, qsl, lens, table = random_case(num_reqs=3, heads=16, head_dim=64, block_size=16,
                                              max_len=4096, min_len=2000, dtype=dtype, seed=11)
    got, plan = kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert plan.num_splits > 1 and plan.workspace_bytes > 0
    assert_attention_close(got, oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, 0.125), dtype,
                           "split-K")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_split_plan_in_a_cuda_graph_follows_the_lengths(oracle_lib, dtype):
    """A split item-grid plan captured in a CUDA graph: the combine launch, the grid's programmatic
    dependent, becomes a programmatic edge of the graph. Replays with other device lengths (some
    zero, some too short to split) equal the oracle."""
    o = ops()
    q, kc, vc, qsl, lens, table = random_case(num_reqs=6, heads=16, head_dim=64, block_size=16, max_len=4096,
                                              min_len=4096, dtype=dtype, seed=12, on_device=True)
    meta = o.get_scheduler_metadata(6, 16, 16, 64, lens, dtype, qsl, False, "sm100", 16)
    plan = o.plan_of(meta)
    assert plan.schedule == o.SCHEDULE_ITEMS and plan.num_splits > 1
    dq, dl, dt = qsl.to(DEV), lens.to(DEV), table.to(DEV)
    out = torch.zeros_like(q)
    o.attention_with_kv_cache(q, kc, vc, out, dq, dl, 0.125, False, dt, meta)  # warm-up outside capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o.attention_with_kv_cache(q, kc, vc, out, dq, dl, 0.125, False, dt, meta)
    g = torch.Generator().manual_seed(13)
    for step in range(3):
        new = torch.randint(0, 4097, (6,), generator=g, dtype=torch.int32)
        new[step] = 0
        new[(step + 1) % 6] = 40
        dl.copy_(new)
        out.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        assert o.read_device_errors(DEV) == 0
        want = oracle_attn(oracle_lib, q.cpu(), kc.cpu(), vc.cpu(), qsl, new, table, 0.125)
        assert_attention_close(out.cpu(), want, dtype, f"graph replay {step}")
    del graph


def test_baseline_sweep_b256_against_oracle(oracle_lib):
    # BASELINE config 5 at batch 256: bf16, 16 heads x 64, block 16, contexts U[1, 4096]
    q, kc, vc, qsl, lens, table = random_case(num_reqs=256, heads=16, head_dim=64, block_size=16,
                                              max_len=4096, min_len=1, dtype=torch.bfloat16, seed=2)
    got, plan = kernel(q, kc, vc, qsl, lens, table, 0.125)
    ref = oracle_attn(oracle_lib, q, kc, vc, qsl, lens, table, 0.125)
    assert_attention_close(got, ref, torch.bfloat16, "cfg5 B=256")


def test_baseline_sweep_b1024_properties(oracle_lib):
    o = ops()
    H, D, bs = 16, 64, 16
    q, kc, vc, qsl, lens, table = random_case(num_reqs=1024, heads=H, head_dim=D, block_size=bs,
                                              max_len=4096, min_len=1, dtype=torch.bfloat16, seed=2,
                                              extra_blocks=0, on_device=True)
    got, plan = kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert plan.num_splits > 1
    # (1) a sample of rows against the oracle
    g = torch.Generator().manual_seed(0)
    rows = torch.randperm(1024, generator=g)[:48].sort().values
    kc_s, vc_s, tab_s = compact_sample(kc, vc, table, lens, rows, bs)
    ref = oracle_attn(oracle_lib, q[rows.to(DEV)].cpu().contiguous(), kc_s, vc_s,
                      torch.arange(49, dtype=torch.int32), lens[rows].contiguous(), tab_s, 0.125)
    assert_attention_close(got[rows], ref, torch.bfloat16, "cfg5 B=1024 sample")
    # (2) physical placement does not matter: relocate every block, results are bit-identical
    nb = kc.shape[0]
    perm = torch.randperm(nb, generator=g)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(nb)
    inv_d = inv.to(DEV)
    got2, _ = kernel(q, kc[inv_d], vc[inv_d], qsl, lens, perm[table.long()].to(torch.int32).contiguous(), 0.125)
    assert torch.equal(got, got2)
    # (3) deterministic: a second run gives the same bits
    got3, _ = kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert torch.equal(got, got3)
    assert o.read_device_errors(DEV) == 0


def test_constant_values_give_that_value(oracle_lib):
    q, kc, vc, qsl, lens, table = random_case(num_reqs=8, heads=4, head_dim=64, block_size=16,
                                              max_len=2000, min_len=1, dtype=torch.float32, seed=4)
    vc = torch.full_like(vc, 0.375)
    got, _ = kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert (got - 0.375).abs().max() <= 1e-6


def test_zero_length_rows_and_empty_batches():
    o = ops()
    q, kc, vc, qsl, lens, table = random_case(num_reqs=4, heads=2, head_dim=64, block_size=16,
                                              max_len=40, dtype=torch.bfloat16, seed=1)
    lens = torch.tensor([0, 5, 0, 40], dtype=torch.int32)
    got, _ = kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert torch.all(got[0] == 0) and torch.all(got[2] == 0) and torch.isfinite(got).all()
    # no requests at all: nothing launched, output untouched
    meta = o.get_scheduler_metadata(0, 2, 2, 64, torch.zeros(0, dtype=torch.int32), torch.bfloat16,
                                    None, False, "sm100", 16)
    out = torch.ones(0, 2, 64, dtype=torch.bfloat16, device=DEV)
    o.attention_with_kv_cache(out, kc.to(DEV), vc.to(DEV), out, torch.zeros(1, dtype=torch.int32, device=DEV),
                              torch.zeros(0, dtype=torch.int32, device=DEV), 0.125, False,
                              torch.zeros(0, 1, dtype=torch.int32, device=DEV), meta)


def test_strided_query_from_fused_projection(oracle_lib):
    # q/k/v chunks of a fused qkv projection: token stride 3 * H * D
    H, D = 4, 64
    q0, kc, vc, qsl, lens, table = random_case(num_reqs=7, heads=H, head_dim=D, block_size=16,
                                               max_len=130, dtype=torch.bfloat16, seed=8)
    qkv = torch.randn(7, 3 * H * D, dtype=torch.bfloat16, device=DEV)
    q = qkv[:, : H * D].reshape(7, H, D)
    assert q.stride(0) == 3 * H * D
    o = ops()
    meta = o.get_scheduler_metadata(7, H, H, D, lens, torch.bfloat16, qsl, False, "sm100", 16)
    out = torch.empty_like(q)
    o.attention_with_kv_cache(q, kc.to(DEV), vc.to(DEV), out, qsl.to(DEV), lens.to(DEV), 0.125, False,
                              table.to(DEV), meta)
    ref = oracle_attn(oracle_lib, q.cpu().contiguous(), kc, vc, qsl, lens, table, 0.125)
    assert_attention_close(out.cpu(), ref, torch.bfloat16, "strided q")


def test_bad_block_ids_are_flagged_not_dereferenced():
    o = ops()
    o.read_device_errors(DEV)
    q, kc, vc, qsl, lens, table = random_case(num_reqs=3, heads=2, head_dim=64, block_size=16,
                                              max_len=60, min_len=20, dtype=torch.bfloat16, seed=6)
    table = table.clone()
    table[1, 0] = kc.shape[0] + 1000
    table[2, 0] = -7
    kernel(q, kc, vc, qsl, lens, table, 0.125)
    assert o.read_device_errors(DEV) & 0x1  # VFL_DEVERR_BLOCK_ID
    assert o.read_device_errors(DEV) == 0   # cleared by the read


def test_device_lengths_beyond_the_plan_are_clamped_and_flagged(oracle_lib):
    o = ops()
    o.read_device_errors(DEV)
    q, kc, vc, qsl, lens, table = random_case(num_reqs=2, heads=2, head_dim=64, block_size=16,
                                              max_len=40, min_len=40, dtype=torch.float32, seed=7)
    planned = torch.tensor([20, 30], dtype=torch.int32)
    got, _ = kernel(q, kc, vc, qsl, planned, table, 0.125, device_lens=torch.tensor([20, 40], dtype=torch.int32))
    assert o.read_device_errors(DEV) & 0x4  # VFL_DEVERR_CONTEXT
    ref = oracle_attn(oracle_lib, q, kc, vc, qsl, planned, table, 0.125)
    assert_attention_close(got, ref, torch.float32, "clamped")


def beam_case(*, requests, beams, block_size, max_len, seed, heads=16, head_dim=64):
    """Beam-search self-attention: each request's rows (its beams) share a prefix of blocks and
    then diverge (copy-on-write forks); a request's rows see the same number of tokens."""
    g = torch.Generator().manual_seed(seed)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    counts = [int(torch.randint(1, beams + 1, (1,), generator=g)) for _ in range(requests)]
    lens = torch.randint(1, max_len + 1, (requests,), generator=g, dtype=torch.int32)
    nbs = [max(1, math.ceil(int(n) / block_size)) for n in lens]
    rows = sum(counts)
    width = max(nbs)
    table = torch.zeros(rows, width, dtype=torch.int32)
    next_block = 0
    row = 0
    for r, (c, nb) in enumerate(zip(counts, nbs)):
        base = torch.arange(next_block, next_block + nb, dtype=torch.int32)
        next_block += nb
        for b in range(c):
            t = base.clone()
            shared = int(torch.randint(0, nb + 1, (1,), generator=g)) if b else nb  # row 0 keeps all
            for j in range(shared, nb):
                t[j] = next_block
                next_block += 1
            if b and int(torch.randint(0, 3, (1,), generator=g)) == 0 and nb > 1:
                t[0] = table[row - 1, 0]  # also share with a sibling rather than row 0
            table[row, :nb] = t
            row += 1
    perm = torch.randperm(next_block + 3, generator=g).to(torch.int32)
    table = perm[table.long()] * (table >= 0)
    qsl = torch.tensor([0] + torch.tensor(counts).cumsum(0).tolist(), dtype=torch.int32)
    kc = torch.randn(next_block + 3, heads, block_size, head_dim, generator=gd, device=DEV, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(rows, heads, head_dim, generator=gd, device=DEV, dtype=torch.bfloat16)
    row_lens = torch.repeat_interleave(lens, torch.tensor(counts))
    return q, kc, vc, qsl, lens, row_lens, table


@pytest.mark.parametrize("requests,beams,block_size,max_len,seed", [
    (40, 3, 16, 150, 1), (12, 4, 16, 2500, 2), (7, 8, 32, 900, 3), (64, 5, 16, 60, 4), (3, 2, 16, 4096, 5),
    (6, 12, 16, 300, 6)])
def test_row_tables_match_per_row_requests(oracle_lib, requests, beams, block_size, max_len, seed):
    """One CTA serves the beams of a request with their own block tables (shared prefix, forked
    tails); the result equals attention with every beam as its own request."""
    o = ops()
    q, kc, vc, qsl, lens, row_lens, table = beam_case(requests=requests, beams=beams, block_size=block_size,
                                                      max_len=max_len, seed=seed)
    n, h, bs, d = kc.shape
    meta = o.get_scheduler_metadata(requests, h, h, d, lens, torch.bfloat16, qsl, False, "sm100", bs, row_tables=True)
    plan = o.plan_of(meta)
    assert plan.row_tables == 1 and plan.queries_per_cta == 8
    out = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
    o.attention_with_kv_cache(q, kc, vc, out, qsl.to(DEV), lens.to(DEV), d ** -0.5, False, table.to(DEV), meta)
    rows_qsl = torch.arange(q.shape[0] + 1, dtype=torch.int32)
    want = oracle_attn(oracle_lib, q.cpu(), kc.cpu(), vc.cpu(), rows_qsl, row_lens, table, d ** -0.5)
    assert_attention_close(out.cpu(), want, torch.bfloat16, f"row tables {requests}x{beams} bs{bs} len<={max_len}")
    # and the per-row kernel agrees
    per_row, _ = kernel(q, kc, vc, rows_qsl, row_lens, table, d ** -0.5)
    assert_attention_close(out.cpu(), per_row, torch.bfloat16, "row tables vs per-row kernel")
    assert o.read_device_errors(DEV) == 0
    if max_len >= 2500:
        assert plan.num_splits > 1  # the split path and its merge are exercised


def test_row_tables_refused_where_not_built():
    o = ops()
    from vflorence_b200._native import VflError

    lens = torch.tensor([10, 20], dtype=torch.int32)
    qsl = torch.tensor([0, 2, 4], dtype=torch.int32)
    with pytest.raises(VflError, match="row tables"):
        o.get_scheduler_metadata(2, 16, 16, 64, lens, torch.float32, qsl, False, "sm100", 16, row_tables=True)
    with pytest.raises(ValueError, match="causal"):
        o.get_scheduler_metadata(2, 16, 16, 64, lens, torch.bfloat16, qsl, True, "sm100", 16, row_tables=True)


# ------------------------------------------------------------- fused KV append + attention

def _appended_case(kind, seed, block_size, max_len, requests, dtype=torch.bfloat16, head_dim=64):
    """Pools, tables and one step's new tokens: every query row appends its newest token into
    a block of its own (after copy-on-write no row shares the block it writes)."""
    g = torch.Generator().manual_seed(seed)
    gd = torch.Generator(device=DEV).manual_seed(seed)
    H, D = 16, head_dim
    if kind == "beams":
        counts = [int(torch.randint(1, 5, (1,), generator=g)) for _ in range(requests)]
    elif kind == "causal":
        counts = [int(torch.randint(1, 9, (1,), generator=g)) for _ in range(requests)]
    else:
        counts = [1] * requests
    lens = torch.randint(1, max_len + 1, (requests,), generator=g, dtype=torch.int32)
    lens[::5] = torch.tensor([block_size * k + 1 for k in range(1, 1 + len(lens[::5]))], dtype=torch.int32)[
        : len(lens[::5])].clamp(max=max_len)  # some new tokens open a block
    if kind == "causal":
        lens = torch.maximum(lens, torch.tensor(counts, dtype=torch.int32))
    nbs = [math.ceil(int(n) / block_size) for n in lens]
    rows = sum(counts) if kind == "beams" else requests
    width = max(nbs)
    table = torch.zeros(rows, width, dtype=torch.int32)
    nxt, row = 0, 0
    for r, (c, nb) in enumerate(zip(counts, nbs)):
        base = torch.arange(nxt, nxt + nb, dtype=torch.int32)
        nxt += nb
        for b in range(c if kind == "beams" else 1):
            t = base.clone()
            if b:  # a forked beam: shared prefix, own blocks from a random point, always its own last
                first = int(torch.randint(0, nb, (1,), generator=g))
                for j in range(first, nb):
                    t[j] = nxt
                    nxt += 1
            table[row, :nb] = t
            row += 1
    pool = nxt + 4
    perm = torch.randperm(pool, generator=g).to(torch.int32)
    table = perm[table.long()]
    kc = torch.randn(pool, H, block_size, D, generator=gd, device=DEV, dtype=dtype)
    vc = torch.randn_like(kc)
    qsl = torch.tensor([0] + torch.tensor(counts).cumsum(0).tolist(), dtype=torch.int32)
    nq = int(qsl[-1])
    # the new tokens' slots: row i's newest position (causal: the request's last counts[r] positions)
    slots = torch.empty(nq, dtype=torch.int64)
    for r in range(requests):
        for j in range(int(qsl[r]), int(qsl[r + 1])):
            trow = j if kind == "beams" else r
            pos = int(lens[r]) - 1 if kind != "causal" else int(lens[r]) - (int(qsl[r + 1]) - j)
            slots[j] = int(table[trow, pos // block_size]) * block_size + pos % block_size
    fused = torch.randn(nq, 3 * H * D, generator=gd, device=DEV, dtype=dtype)  # a q/k/v projection
    q, key, value = (x.reshape(nq, H, D) for x in fused.chunk(3, dim=-1))
    return q, key, value, kc, vc, qsl, lens, table, slots


@pytest.mark.parametrize("kind,seed,block_size,max_len,requests,dtype,head_dim", [
    ("rows", 1, 16, 200, 40, torch.bfloat16, 64), ("rows", 2, 16, 4000, 9, torch.bfloat16, 64),
    ("rows", 3, 32, 1500, 17, torch.bfloat16, 64), ("beams", 4, 16, 300, 30, torch.bfloat16, 64),
    ("beams", 5, 16, 3000, 6, torch.bfloat16, 64), ("causal", 6, 16, 600, 12, torch.bfloat16, 64),
    ("causal", 7, 32, 2000, 5, torch.bfloat16, 64),
    # the CUDA-core kernel: float32 (BASELINE cfg 1's decoder), and bf16 at other head dims
    ("rows", 8, 16, 200, 40, torch.float32, 64), ("rows", 9, 16, 4000, 9, torch.float32, 64),
    ("rows", 10, 32, 1500, 17, torch.float32, 64), ("rows", 11, 16, 900, 12, torch.bfloat16, 128),
    ("rows", 12, 16, 700, 7, torch.float32, 32)], ids=lambda v: str(v).replace("torch.", ""))
def test_attention_append_equals_append_then_attend(kind, seed, block_size, max_len, requests, dtype, head_dim):
    """One launch that stores each row's new K/V and attends over it gives the output and the
    pools of reshape_and_cache followed by attention_with_kv_cache, bit for bit (the same plan
    reads the same bytes); long contexts exercise the split that holds the new position."""
    o = ops()
    q, key, value, kc, vc, qsl, lens, table, slots = _appended_case(kind, seed, block_size, max_len, requests,
                                                                    dtype, head_dim)
    n, h, bs, d = kc.shape
    causal = kind == "causal"
    meta = o.get_scheduler_metadata(requests, h, h, d, lens, dtype, qsl, causal, "sm100", bs,
                                    row_tables=kind == "beams")
    assert o.attention_append_supported(meta)
    dq, dl, dt, ds = qsl.to(DEV), lens.to(DEV), table.to(DEV), slots.to(DEV)
    kc2, vc2 = kc.clone(), vc.clone()
    o.reshape_and_cache(key, value, kc2, vc2, ds)
    want = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
    o.attention_with_kv_cache(q, kc2, vc2, want, dq, dl, d ** -0.5, causal, dt, meta)
    got = torch.full(q.shape, float("nan"), dtype=q.dtype, device=DEV)
    o.attention_with_kv_cache_append(q, key, value, kc, vc, got, ds, dq, dl, d ** -0.5, causal, dt, meta)
    torch.cuda.synchronize()
    assert o.read_device_errors(DEV) == 0
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(got, want)
    if max_len >= 3000:
        assert o.plan_of(meta).num_splits > 1


def test_attention_append_skips_padding_and_flags_bad_slots():
    o = ops()
    q, key, value, kc, vc, qsl, lens, table, slots = _appended_case("rows", 8, 16, 100, 6)
    n, h, bs, d = kc.shape
    lens[2] = 0          # a padding row: no token, no write
    slots[2] = -1
    slots[4] = n * bs    # one past the pool: skipped and flagged
    meta = o.get_scheduler_metadata(6, h, h, d, lens, torch.bfloat16, qsl, False, "sm100", bs)
    before_k, before_v = kc.clone(), vc.clone()
    out = torch.empty_like(q)
    o.attention_with_kv_cache_append(q, key, value, kc, vc, out, slots.to(DEV), qsl.to(DEV), lens.to(DEV),
                                     d ** -0.5, False, table.to(DEV), meta)
    from vflorence_b200 import _native

    assert o.read_device_errors(DEV) & _native.DEVERR_SLOT
    want_k, want_v = before_k.clone(), before_v.clone()
    keep = torch.tensor([i not in (2, 4) for i in range(6)])
    o.reshape_and_cache(key[keep.to(DEV)], value[keep.to(DEV)], want_k, want_v, slots[keep].to(DEV))
    assert torch.equal(kc, want_k) and torch.equal(vc, want_v)
    assert bool((out[2] == 0).all())  # a row with no tokens gives zeros


def test_attention_append_refused_where_not_built():
    o = ops()
    from vflorence_b200._native import VflError

    lens = torch.tensor([10, 20], dtype=torch.int32)
    f32 = o.get_scheduler_metadata(2, 16, 16, 64, lens, torch.float32, None, False, "sm100", 16)
    assert o.attention_append_supported(f32)  # one row per request: the CUDA-core kernel appends too
    f32_grouped = o.get_scheduler_metadata(2, 16, 16, 64, lens, torch.float32, torch.tensor([0, 2, 4], dtype=torch.int32),
                                           False, "sm100", 16)
    assert not o.attention_append_supported(f32_grouped)
    # several non-causal rows sharing one table would all write its newest position
    grouped = o.get_scheduler_metadata(2, 16, 16, 64, lens, torch.bfloat16, torch.tensor([0, 2, 4], dtype=torch.int32),
                                       False, "sm100", 16)
    assert not o.attention_append_supported(grouped)
    kc = torch.zeros(4, 16, 16, 64, device=DEV, dtype=torch.bfloat16)
    q = torch.zeros(4, 16, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(VflError, match="attention_append"):
        o.attention_with_kv_cache_append(q, q, q, kc, kc.clone(), torch.empty_like(q),
                                         torch.zeros(4, dtype=torch.int64, device=DEV),
                                         torch.tensor([0, 2, 4], dtype=torch.int32, device=DEV),
                                         lens.to(DEV), 0.125, False, torch.zeros(2, 2, dtype=torch.int32, device=DEV),
                                         grouped)
