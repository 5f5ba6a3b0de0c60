"""The C-ABI library without a GPU: it loads, exports exactly what include/vflorence_b200.h and
include/vflorence_b200_runtime.h declare, and its host-only entry points (get_isa, the planner,
argument validation) behave."""

from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

from conftest import REPO


def _declared():
    names = []
    for header in ("vflorence_b200.h", "vflorence_b200_runtime.h"):
        text = open(os.path.join(REPO, "include", header)).read()
        names += re.findall(r"^(?:int|void|size_t|const char\*)\s+(vfl_\w+)\(", text, flags=re.M)
    return names


def test_library_exports_every_declared_symbol(native):
    from vflorence_b200 import _native

    declared = _declared()
    assert sorted(declared) == sorted(_native.EXPORTS)
    for name in declared:
        assert hasattr(native, name), name
    assert native.vfl_abi_version() == _native.ABI_VERSION == 4


def test_bounded_wait_check_refuses_limits_on_the_host(native):
    """The wait limit must lie in (0, 2 s]; refused before any CUDA call."""
    for limit in (0, -5, 2_000_000_001):
        assert native.vfl_check_bounded_wait(0, limit, None) == 1
        assert b"limit_ns" in native.vfl_last_error_message()


def test_decode_linear_support_and_refusals(native):
    """Shapes the skinny linear kernel takes, and host-side refusals before any launch."""
    from vflorence_b200 import paged_ops as ops

    assert ops.decode_linear_supported(torch.float32, 8, 1024, 4096)
    assert ops.decode_linear_supported(torch.float32, 16, 50304, 1024)
    assert ops.decode_linear_supported(torch.float32, 1, 96, 256)
    for args in ((torch.bfloat16, 8, 1024, 1024), (torch.float32, 17, 1024, 1024), (torch.float32, 0, 1024, 1024),
                 (torch.float32, 8, 1000, 1024), (torch.float32, 8, 1024, 1000)):
        assert not ops.decode_linear_supported(*args)
    ptr = 1 << 20  # never dereferenced: every call below is refused on the host
    assert native.vfl_decode_linear(ptr, 1024, ptr, None, ptr, 1024, 8, 1024, 1024, 1, 0, None) == 2  # bf16
    assert native.vfl_decode_linear(ptr, 1024, ptr, None, ptr, 1024, 8, 1024, 1024, 0, 7, None) == 1  # activation
    assert native.vfl_decode_linear(None, 1024, ptr, None, ptr, 1024, 8, 1024, 1024, 0, 0, None) == 1
    assert native.vfl_decode_linear(ptr + 4, 1024, ptr, None, ptr, 1024, 8, 1024, 1024, 0, 0, None) == 1
    assert native.vfl_decode_linear(ptr, 1026, ptr, None, ptr, 1024, 8, 1024, 1024, 0, 0, None) == 1
    assert native.vfl_decode_linear(ptr, 1024, ptr, None, ptr, 1000, 8, 1024, 1024, 0, 0, None) == 1
    assert native.vfl_decode_linear(ptr, 1024, ptr, None, ptr, 1024, 20, 1024, 1024, 0, 0, None) == 2
    assert native.vfl_decode_linear(ptr, 1024, ptr, None, ptr, 1024, 0, 1024, 1024, 0, 0, None) == 0  # no rows


def test_status_strings(native):
    assert native.vfl_status_string(0) == b"ok"
    assert b"workspace" in native.vfl_status_string(3)
    assert b"capacity" in native.vfl_status_string(5)


def test_get_isa(native):
    from vflorence_b200 import paged_ops as ops

    for dt in (torch.float32, torch.bfloat16):
        for d in sorted(ops.HEAD_DIMS):
            assert ops.get_isa(dt, 16, d) == "sm100"
    assert ops.get_isa(torch.bfloat16, 32, 64) == "sm100"
    assert ops.get_isa(torch.float32, 16, 512) == "sm100"  # the reference's largest head_dim
    for args in ((torch.bfloat16, 16, 1024), (torch.bfloat16, 16, 40), (torch.bfloat16, 8, 64),
                 (torch.bfloat16, 24, 64)):
        with pytest.raises(ValueError):
            ops.get_isa(*args)
    with pytest.raises(ValueError):
        ops.get_isa(torch.float16, 16, 64)


def _plan(lens, qsl=None, heads=16, d=64, bs=16, dtype=torch.bfloat16, causal=False):
    from vflorence_b200 import paged_ops as ops

    meta = ops.get_scheduler_metadata(len(lens), heads, heads, d, torch.tensor(lens, dtype=torch.int32),
                                      dtype, None if qsl is None else torch.tensor(qsl, dtype=torch.int32),
                                      causal, "sm100", bs)
    return ops.plan_of(meta)


def test_plan_large_batch_splits_long_requests(native):
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator().manual_seed(2)
    lens = torch.randint(1, 4097, (1024,), generator=g).tolist()
    p = _plan(lens)
    assert (p.heads_per_cta, p.queries_per_cta) == (4, 8)   # bf16 x 64: tensor cores
    assert p.blocks_per_split == 64                # only the table slice (64 blocks) splits the grid
    assert p.num_splits == -(-max(lens) // 1024)
    assert p.total_q == 1024 and p.max_seq_len == max(lens)
    assert p.merge_in_kernel == 0          # bandwidth-bound: separate combine launch
    # skewed lengths over many waves of that grid: the balanced wave, with two stages
    assert (p.schedule, p.stages, p.balanced_ctas, p.min_tiles) == (ops.SCHEDULE_BALANCED, 2, 148 * 3, 8)
    recs = 148 * 3 * 2 * 4 * 8
    assert p.workspace_bytes == _r256(recs * 64 * 4) + _r256(recs * 2 * 4) + _r256(1024 * 4 * 16)


def test_plan_schedule_rule(native):
    """The item grid where it runs in at most one wave, where items are short, and for
    near-uniform lengths it runs unsplit over four waves or more; the balanced wave otherwise."""
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator().manual_seed(3)
    beams = lambda n, k: [min(k * r, k * n) for r in range(n + 1)]  # noqa: E731
    items = ops.SCHEDULE_ITEMS
    bal = ops.SCHEDULE_BALANCED
    cases = [
        (_plan([592] * 85, qsl=beams(85, 3)), items),          # the cfg-4 cross-attention wave: 0.77 waves
        (_plan([1024] * 32, qsl=beams(32, 4)), items),         # cfg 2: split 3 ways, 0.86 waves
        (_plan([128] * 256), items),                           # short items
        (_plan([592] * 1024), items),                          # near-uniform, unsplit, 9 waves
        (_plan([592] * 128), bal),                             # 2.3 waves
        (_plan(torch.randint(1, 2049, (32,), generator=g).tolist()), bal),  # skewed, split grid
        (_plan(torch.randint(1, 1025, (1024,), generator=g).tolist()), bal),  # skewed, 9 waves
        (_plan([577] * 200, heads=16, dtype=torch.float32), items),  # CUDA-core kernel: grid only
        (_plan([4096] * 32, d=128), items),
    ]
    for i, (p, want) in enumerate(cases):
        assert p.schedule == want, i


def test_plan_merges_splits_in_a_separate_launch(native):
    """Split partials always merge in a separate combine launch (measured faster than the
    in-kernel last-arriver merge in 1214 of 1220 swept cases); the workspace holds only the
    partials, no arrival counters."""
    from vflorence_b200 import paged_ops as ops

    g = torch.Generator().manual_seed(2)
    for n in (8, 256):
        lens = torch.randint(1, 4097, (n,), generator=g).to(torch.int32)
        meta = ops.get_scheduler_metadata(n, 16, 16, 64, lens, torch.bfloat16, None, False, "sm100", 16)
        p = ops.plan_of(ops.set_schedule(meta, ops.SCHEDULE_ITEMS))  # the item grid of the same call
        assert p.num_splits > 1 and p.merge_in_kernel == 0
        items = p.total_q * 16 * p.num_splits
        r256 = lambda x: -(-x // 256) * 256  # noqa: E731
        assert p.workspace_bytes == r256(items * 64 * 4) + r256(items * 2 * 4)


def test_plan_uniform_batches_are_not_split(native):
    # decode-step shapes (half a wave or more of near-uniform items): no split, and short items
    # run two-stage rings when they fill a wave
    p = _plan([592] * 85, qsl=[min(3 * r, 255) for r in range(86)])
    assert p.num_splits == 1 and p.workspace_bytes == 0
    q = _plan([100 + i % 60 for i in range(255)])
    assert q.num_splits == 1 and q.stages == 2
    # few near-uniform items: split to fill about 0.9 of a wave, items of at least 96 tokens
    few = _plan([2048] * 8)
    assert 4 <= few.num_splits <= 16 and few.blocks_per_split >= 6
    assert 8 * 4 * few.num_splits <= 148 * 3
    # items that would land between one and two waves back off to one wave: 32 requests x 2048
    # tokens split 3 ways (384 items), not 4 (512)
    one = _plan([2048] * 32)
    assert one.num_splits == 3
    # skewed lengths: pieces of about the total work over 1.5 waves (here ~820 tokens: 5 splits
    # of the longest request), never below 320 tokens
    g = torch.Generator().manual_seed(2)
    lens = torch.randint(1, 4097, (64,), generator=g).tolist()
    skew = _plan(lens)
    assert 4 <= skew.num_splits <= 8 and skew.blocks_per_split * 16 >= 320


def test_plan_single_long_request_fills_the_gpu(native):
    p = _plan([4096])
    ctas = (16 // p.heads_per_cta) * p.num_splits
    assert ctas >= 148


def test_plan_short_batch_needs_no_workspace(native):
    p = _plan([5, 17, 33], heads=2)
    assert p.num_splits == 1 and p.workspace_bytes == 0
    assert p.heads_per_cta == 2


def test_plan_grouped_rows(native):
    p = _plan([577, 577], qsl=[0, 3, 6], heads=12)
    assert p.queries_per_cta == 8 and p.total_q == 6 and p.max_q_len == 3   # tensor-core kernel
    assert p.heads_per_cta == 4
    # CUDA-core kernel (fp32, or other head dims): 1 row per CTA for decode, 4 for grouped rows
    f = _plan([577, 577], qsl=[0, 3, 6], heads=12, dtype=torch.float32)
    assert f.queries_per_cta == 4
    assert _plan([577, 577], heads=12, dtype=torch.float32).queries_per_cta == 1
    assert _plan([577, 577], heads=12, d=128).queries_per_cta == 1


def test_plan_f32_and_wide_heads(native):
    p = _plan([100], heads=16, d=256, dtype=torch.float32)
    assert 2 * p.heads_per_cta * 16 * 256 * 4 <= 32 * 1024
    assert p.stages >= 2


def test_plan_rejects_bad_input(native):
    from vflorence_b200 import paged_ops as ops
    from vflorence_b200._native import VflError

    with pytest.raises(VflError, match="grouped-query"):
        ops.get_scheduler_metadata(2, 16, 4, 64, torch.tensor([3, 4], dtype=torch.int32),
                                   torch.bfloat16, None, False, "sm100", 16)
    with pytest.raises(VflError, match="< 0"):
        _plan([3, -1])
    with pytest.raises(VflError, match="decreases"):
        _plan([3, 4], qsl=[0, 2, 1])
    with pytest.raises(ValueError):
        _plan([3, 4], qsl=[0, 1])


def _r256(x):
    return -(-x // 256) * 256


def test_plan_balanced_schedule(native):
    """vfl_plan_attention_schedule re-plans a call for one persistent wave: 148 SMs x 3 CTAs,
    at least 8 tiles per CTA by default, a workspace of partial records (2 per CTA, head and
    row) and the item directory; back to the item grid restores the grid's workspace."""
    from vflorence_b200 import paged_ops as ops

    lens = torch.full((85,), 592, dtype=torch.int32)
    qsl = torch.arange(0, 256, 3, dtype=torch.int32)
    meta = ops.get_scheduler_metadata(85, 16, 16, 64, lens, torch.bfloat16, qsl, False, "sm100", 16)
    ops.set_schedule(meta, ops.SCHEDULE_ITEMS)
    items_ws = ops.plan_of(meta).workspace_bytes
    ops.set_schedule(meta, ops.SCHEDULE_BALANCED)
    p = ops.plan_of(meta)
    assert (p.schedule, p.balanced_ctas, p.min_tiles) == (ops.SCHEDULE_BALANCED, 148 * 3, 8)
    recs = 148 * 3 * 2 * 4 * 8
    assert p.workspace_bytes == _r256(recs * 64 * 4) + _r256(recs * 2 * 4) + _r256(85 * 4 * 16)
    ops.set_schedule(meta, ops.SCHEDULE_BALANCED, 3)
    assert ops.plan_of(meta).min_tiles == 3
    ops.set_schedule(meta, ops.SCHEDULE_ITEMS)
    p = ops.plan_of(meta)
    assert (p.schedule, p.min_tiles, p.balanced_ctas, p.workspace_bytes) == (ops.SCHEDULE_ITEMS, 0, 0, items_ws)


def test_plan_balanced_schedule_refused_where_not_built(native):
    from vflorence_b200 import paged_ops as ops

    def meta(n=4, rows=1, d=64, dtype=torch.bfloat16, row_tables=False):
        lens = torch.full((n,), 300, dtype=torch.int32)
        qsl = torch.arange(0, n * rows + 1, rows, dtype=torch.int32)
        return ops.get_scheduler_metadata(n, 16, 16, d, lens, dtype, qsl, False, "sm100", 16, row_tables=row_tables)

    for m in (meta(dtype=torch.float32), meta(d=128), meta(rows=9), meta(n=2049), meta(rows=2, row_tables=True)):
        with pytest.raises(ValueError, match="balanced"):
            ops.set_schedule(m, ops.SCHEDULE_BALANCED)
        assert ops.plan_of(m).schedule == ops.SCHEDULE_ITEMS
    huge = ops.get_scheduler_metadata(2, 16, 16, 64, torch.tensor([1 << 24, 5], dtype=torch.int32), torch.bfloat16,
                                      None, False, "sm100", 16)  # the tile prefix would leave int32
    with pytest.raises(ValueError, match="balanced"):
        ops.set_schedule(huge, ops.SCHEDULE_BALANCED)
    with pytest.raises(ValueError, match="schedule"):
        ops.set_schedule(meta(), 2)
    with pytest.raises(ValueError, match="min_tiles"):
        ops.set_schedule(meta(), ops.SCHEDULE_BALANCED, -1)
    big = ops.set_schedule(meta(n=2048), ops.SCHEDULE_BALANCED)  # the most requests it takes
    assert ops.plan_of(big).num_reqs == 2048 and ops.plan_of(big).balanced_ctas >= 148


@pytest.mark.parametrize("field,value", [("schedule", 2), ("min_tiles", 0), ("balanced_ctas", 0),
                                         ("balanced_ctas", 148 * 3 + 1), ("workspace_bytes", 4096),
                                         ("row_tables", 1), ("max_q_len", 9)])
def test_attention_refuses_a_corrupted_balanced_plan_before_the_device(native, field, value):
    from vflorence_b200 import _native
    from vflorence_b200 import paged_ops as ops

    lens = torch.tensor([2048, 1000, 37], dtype=torch.int32)
    meta = ops.get_scheduler_metadata(3, 16, 16, 64, lens, torch.bfloat16, None, False, "sm100", 16)
    ops.set_schedule(meta, ops.SCHEDULE_BALANCED)
    plan = ops.plan_of(meta)
    setattr(plan, field, value)
    fake = 1 << 20  # never dereferenced: the call must fail before touching memory
    st = native.vfl_attention_with_kv_cache(ctypes.byref(plan), fake, 16 * 64, fake, fake, 1000, fake, 16 * 64,
                                            fake, fake, fake, 128, 128, 1.0, fake, 1 << 30, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT, native.vfl_last_error_message()
    assert b"plan" in native.vfl_last_error_message()


def test_attention_rejects_foreign_metadata_without_touching_the_gpu(native):
    from vflorence_b200 import _native

    plan = _native.AttentionPlan()
    st = native.vfl_attention_with_kv_cache(ctypes.byref(plan), None, 0, None, None, 0, None, 0, None,
                                            None, None, 0, 0, 1.0, None, 0, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT
    assert b"plan" in native.vfl_last_error_message()


@pytest.mark.parametrize("field,value", [("blocks_per_split", 65), ("blocks_per_split", 0), ("stages", 9),
                                         ("stages", 1), ("heads_per_cta", 3), ("num_splits", 1),
                                         ("workspace_bytes", 16), ("queries_per_cta", 2), ("merge_in_kernel", 2)])
def test_attention_refuses_a_corrupted_plan_before_the_device(native, field, value):
    """A plan is caller memory; every field the kernels rely on is re-checked on the host (a
    larger split than the shared-memory table slice would overrun it)."""
    from vflorence_b200 import _native

    plan = _plan([2048, 1000, 37])
    assert plan.num_splits > 1 and plan.blocks_per_split <= 64
    setattr(plan, field, value)
    fake = 1 << 20  # never dereferenced: the call must fail before touching memory
    st = native.vfl_attention_with_kv_cache(ctypes.byref(plan), fake, 16 * 64, fake, fake, 1000, fake, 16 * 64,
                                            fake, fake, fake, 128, 128, 1.0, fake, 1 << 30, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT, native.vfl_last_error_message()
    assert b"plan" in native.vfl_last_error_message()
    st = native.vfl_attention_with_kv_cache_no_alloc(ctypes.byref(plan), fake, 16 * 64, fake, fake, 1000, fake,
                                                     16 * 64, fake, fake, fake, 128, 128, 1.0, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT, native.vfl_last_error_message()


def test_copy_blocks_host_checks(native):
    from vflorence_b200 import paged_ops as ops

    assert ops.check_copy_pairs([(0, 2), (1, 3)], 4) == [(0, 2), (1, 3)]
    for bad in ([(0, 4)], [(0, 2), (1, 2)], [(0, 2), (2, 3)], [(-1, 0)]):
        with pytest.raises(ValueError):
            ops.check_copy_pairs(bad, 4)


def test_ops_refuse_cpu_tensors(native):
    from vflorence_b200 import paged_ops as ops

    kc = torch.zeros(4, 2, 16, 64)
    k = torch.zeros(1, 2, 64)
    with pytest.raises(ValueError, match="CUDA"):
        ops.reshape_and_cache(k, k, kc, kc, torch.zeros(1, dtype=torch.int64))
    with pytest.raises(ValueError, match="CUDA"):
        ops.copy_blocks([kc], [kc], [(0, 1)])


def test_add_layernorm_host_checks(native):
    """Which widths the fused add + LayerNorm is built for, and refusals before any launch."""
    from vflorence_b200 import _native

    bf16, f32 = _native.DTYPE_BF16, _native.DTYPE_F32
    for d in (256, 512, 768, 1024, 2048):
        assert native.vfl_add_layernorm_supported(bf16, d) == 1
    for d in (128, 640, 4096):
        assert native.vfl_add_layernorm_supported(bf16, d) == 0
    for d in (128, 768, 1024):
        assert native.vfl_add_layernorm_supported(f32, d) == 1
    assert native.vfl_add_layernorm_supported(f32, 2048) == 0
    assert native.vfl_add_layernorm_supported(7, 1024) == 0
    fake = ctypes.c_void_p(16)
    st = native.vfl_add_layernorm(fake, 640, fake, 640, fake, None, fake, 640, 4, 640, 1e-5, bf16, None)
    assert st == _native.VFL_ERR_UNSUPPORTED, native.vfl_last_error_message()
    st = native.vfl_add_layernorm(fake, 1024, fake, 1024, fake, None, fake, 1024, -1, 1024, 1e-5, bf16, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT
    st = native.vfl_add_layernorm(ctypes.c_void_p(18), 1024, fake, 1024, fake, None, fake, 1024, 4, 1024, 1e-5,
                                  bf16, None)  # misaligned rows
    assert st == _native.VFL_ERR_INVALID_ARGUMENT
    assert native.vfl_add_layernorm(None, 1024, None, 1024, None, None, None, 1024, 0, 1024, 1e-5, bf16, None) == 0


def test_attention_append_host_checks(native):
    """Which plans the fused append takes, and refusals before any launch."""
    from vflorence_b200 import _native
    from vflorence_b200 import paged_ops as ops

    def meta(lens, qsl=None, dtype=torch.bfloat16, causal=False, row_tables=False, d=64):
        q = None if qsl is None else torch.tensor(qsl, dtype=torch.int32)
        return ops.get_scheduler_metadata(len(lens), 16, 16, d, torch.tensor(lens, dtype=torch.int32), dtype, q,
                                          causal, "sm100", 16, row_tables=row_tables)

    assert ops.attention_append_supported(meta([100, 200]))                              # one row per request
    assert ops.attention_append_supported(meta([100, 200], [0, 3, 5], row_tables=True))  # beam groups
    assert ops.attention_append_supported(meta([100, 200], [0, 3, 5], causal=True))      # causal rows
    # more than 8 causal rows of a request span two CTAs, and later rows read earlier rows' tokens
    assert not ops.attention_append_supported(meta([100, 200], [0, 12, 14], causal=True))
    assert not ops.attention_append_supported(meta([100, 200], [0, 3, 5]))               # rows sharing a table
    # the CUDA-core kernel (float32, other head dims) appends for one row per request only
    assert ops.attention_append_supported(meta([100, 200], dtype=torch.float32))
    assert ops.attention_append_supported(meta([100, 200], d=128))
    assert not ops.attention_append_supported(meta([100, 200], [0, 3, 5], dtype=torch.float32))
    assert not ops.attention_append_supported(meta([100, 200], [0, 1, 3], causal=True, d=128))
    fake = ctypes.c_void_p(256)
    bad = ops.plan_of(meta([100, 200], [0, 3, 5], dtype=torch.float32))
    st = native.vfl_attention_with_kv_cache_append(ctypes.byref(bad), fake, 1024, fake, 1024, fake, 1024, fake, fake,
                                                   fake, 100, fake, 1024, fake, fake, fake, 16, 16, 0.125, None, 0,
                                                   None)
    assert st == _native.VFL_ERR_UNSUPPORTED, native.vfl_last_error_message()
    good = ops.plan_of(meta([100, 200]))
    st = native.vfl_attention_with_kv_cache_append(ctypes.byref(good), fake, 1024, None, 1024, fake, 1024, fake,
                                                   fake, fake, 100, fake, 1024, fake, fake, fake, 16, 16, 0.125, None,
                                                   0, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT and b"NULL" in native.vfl_last_error_message()
    st = native.vfl_attention_with_kv_cache_append(ctypes.byref(good), fake, 1024, ctypes.c_void_p(264), 1024, fake,
                                                   1024, fake, fake, fake, 100, fake, 1024, fake, fake, fake, 16, 16,
                                                   0.125, None, 0, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT  # a key not 16-byte aligned
    f32 = ops.plan_of(meta([100, 200], dtype=torch.float32))
    st = native.vfl_attention_with_kv_cache_append(ctypes.byref(f32), fake, 1024, fake, 1026, fake, 1024, fake,
                                                   fake, fake, 100, fake, 1024, fake, fake, fake, 16, 16, 0.125, None,
                                                   0, None)
    assert st == _native.VFL_ERR_INVALID_ARGUMENT  # a float32 key row stride of 1026 elements: not 16-byte


def test_cache_ops_refuse_bad_arguments_before_the_device(native):
    """reshape_and_cache, prepare_decode and paged_slots check sizes, dtypes, NULL pointers,
    alignment and strides on the host and return a status without a launch; empty work is a
    no-op. The addresses below are never dereferenced: every case fails a host check first."""
    from vflorence_b200 import _native as N

    A = 0x10000  # a 16-byte aligned stand-in address
    H, D, BS = 2, 64, 16

    def rc(key=A, value=A, kc=A, vc=A, slots=A, tokens=3, heads=H, head_dim=D, block_size=BS, blocks=8,
           kstride=H * D, vstride=H * D, dtype=N.DTYPE_BF16):
        return native.vfl_reshape_and_cache(key, value, kc, vc, slots, tokens, heads, head_dim, block_size,
                                            blocks, kstride, vstride, dtype, None)

    assert rc(dtype=7) == N.VFL_ERR_UNSUPPORTED
    assert rc(heads=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert rc(blocks=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert rc(tokens=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert rc(tokens=0, key=None, value=None, kc=None, vc=None, slots=None) == N.VFL_OK  # nothing to append
    assert rc(head_dim=6) == N.VFL_ERR_UNSUPPORTED  # 12-byte rows: not a 16-byte multiple
    assert rc(key=None) == N.VFL_ERR_INVALID_ARGUMENT
    assert rc(slots=None) == N.VFL_ERR_INVALID_ARGUMENT
    assert rc(kc=A + 8) == N.VFL_ERR_INVALID_ARGUMENT  # misaligned pool
    assert rc(kstride=H * D + 4) == N.VFL_ERR_INVALID_ARGUMENT  # 8-byte token stride step in bf16
    assert rc(vstride=H * D - 8) == N.VFL_ERR_INVALID_ARGUMENT  # shorter than a token
    assert b"reshape_and_cache" in native.vfl_last_error_message()

    def prep(table=A, stride=4, cols=4, positions=A, seqs=2, block_size=BS, slots=A):
        return native.vfl_prepare_decode(table, stride, cols, positions, seqs, block_size, slots, A, A, None)

    assert prep(seqs=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert prep(block_size=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert prep(stride=3) == N.VFL_ERR_INVALID_ARGUMENT  # stride below the column count
    assert prep(positions=None) == N.VFL_ERR_INVALID_ARGUMENT
    assert prep(table=None) == N.VFL_ERR_INVALID_ARGUMENT  # slots asked for without a table

    def slots(pages=A, stride=4, cols=4, reqs=2, seq_len=50, block_size=BS, out=A):
        return native.vfl_paged_slots(pages, stride, cols, reqs, seq_len, block_size, out, None)

    assert slots(reqs=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert slots(block_size=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert slots(stride=2) == N.VFL_ERR_INVALID_ARGUMENT
    assert slots(seq_len=0, pages=None, out=None) == N.VFL_OK  # no tokens
    assert slots(out=None) == N.VFL_ERR_INVALID_ARGUMENT


def test_selection_ops_refuse_bad_arguments_before_the_device(native):
    """row_topk, beam_merge and fork_token_rows check dtypes, sizes, k and NULL pointers on the
    host; empty work is a no-op. The stand-in addresses are never dereferenced."""
    from vflorence_b200 import _native as N

    A = 0x10000

    def topk(scores=A, dtype=N.DTYPE_BF16, rows=4, vocab=1000, stride=1000, k=4, values=A, indices=A):
        return native.vfl_row_topk(scores, dtype, rows, vocab, stride, 1, None, k, values, indices, None, 0, None)

    assert topk(dtype=9) == N.VFL_ERR_UNSUPPORTED
    assert topk(rows=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert topk(vocab=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert topk(stride=999) == N.VFL_ERR_INVALID_ARGUMENT  # rows overlap
    assert topk(k=0) == N.VFL_ERR_UNSUPPORTED
    assert topk(k=65) == N.VFL_ERR_UNSUPPORTED             # beyond the largest supported k
    assert topk(vocab=3, stride=3) == N.VFL_ERR_UNSUPPORTED  # k larger than the vocabulary
    assert topk(rows=0, scores=None, values=None, indices=None) == N.VFL_OK
    assert topk(values=None) == N.VFL_ERR_INVALID_ARGUMENT
    assert topk(scores=A + 1) == N.VFL_ERR_INVALID_ARGUMENT  # bf16 scores at an odd address
    # the merge workspace is needed only when few rows split each row across CTAs
    assert native.vfl_row_topk_workspace_size(255, 51289, 6) == 0
    assert native.vfl_row_topk_workspace_size(2, 51289, 6) > 0

    def merge(values=A, indices=A, rows=6, k=4, groups=A, ranks=A, num_groups=2, keep=4, out=A):
        return native.vfl_beam_merge(values, indices, rows, k, groups, ranks, num_groups, keep, out, None)

    assert merge(k=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert merge(keep=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert merge(num_groups=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert merge(num_groups=0, values=None, indices=None, groups=None, ranks=None, out=None) == N.VFL_OK
    assert merge(ranks=None) == N.VFL_ERR_INVALID_ARGUMENT

    def fork(tokens=A, stride=300, rows=8, width=257, born=A, num_born=3):
        return native.vfl_fork_token_rows(tokens, stride, rows, width, born, num_born, None)

    assert fork(width=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert fork(stride=256) == N.VFL_ERR_INVALID_ARGUMENT  # rows shorter than the width
    assert fork(num_born=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert fork(num_born=0, tokens=None, born=None) == N.VFL_OK
    assert fork(born=None) == N.VFL_ERR_INVALID_ARGUMENT


def test_kv_proj_paged_refuses_bad_arguments_before_the_device(native):
    """The fused encoder K/V projection checks its GEMM shape (hidden a multiple of 64, head_dim
    of 32, 2 x heads x head_dim of 128), pointers, alignment and the hidden row stride on the
    host; no tokens is a no-op. The stand-in addresses are never dereferenced."""
    from vflorence_b200 import _native as N

    A = 0x10000

    def proj(hidden=A, stride=1024, w=A, kc=A, vc=A, slots=A, tokens=590, hidden_dim=1024, heads=16, head_dim=64,
             block_size=16, blocks=64):
        return native.vfl_kv_proj_paged(hidden, stride, w, None, kc, vc, slots, tokens, hidden_dim, heads, head_dim,
                                        block_size, blocks, None)

    assert proj(hidden_dim=1000) == N.VFL_ERR_INVALID_ARGUMENT  # not a multiple of the 64-wide k-step
    assert proj(head_dim=48) == N.VFL_ERR_INVALID_ARGUMENT      # head slices are 32-column chunks
    assert proj(heads=1, head_dim=32) == N.VFL_ERR_UNSUPPORTED  # 2 x 1 x 32 = 64 features: not a 128 tile
    assert proj(tokens=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert proj(blocks=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert proj(tokens=0, hidden=None, w=None, kc=None, vc=None, slots=None) == N.VFL_OK
    assert proj(slots=None) == N.VFL_ERR_INVALID_ARGUMENT
    assert proj(w=A + 8) == N.VFL_ERR_INVALID_ARGUMENT          # TMA sources start on 16 bytes
    assert proj(stride=1028) == N.VFL_ERR_INVALID_ARGUMENT      # 2056-byte rows: not a 16-byte multiple
    assert proj(stride=512) == N.VFL_ERR_INVALID_ARGUMENT       # rows shorter than hidden_dim


def test_copy_blocks_c_entry_refuses_bad_arguments_before_the_device(native):
    """vfl_copy_blocks reads its per-layer pool pointers on the host and checks them (NULL,
    16-byte alignment), the layer limit and the block size before any launch; no pairs or no
    layers is a no-op. The stand-in pool addresses are never dereferenced."""
    from vflorence_b200 import _native as N

    A = 0x10000
    pairs = (ctypes.c_int64 * 2)(0, 1)

    def layers(*addrs):
        return (ctypes.c_void_p * len(addrs))(*addrs)

    def copy(k=None, v=None, num_layers=2, prs=pairs, num_pairs=1, blocks=8, block_bytes=32768):
        k = layers(A, A) if k is None else k
        v = layers(A, A) if v is None else v
        return native.vfl_copy_blocks(k, v, num_layers, prs, num_pairs, blocks, block_bytes, None)

    assert copy(num_pairs=-1) == N.VFL_ERR_INVALID_ARGUMENT
    assert copy(blocks=0) == N.VFL_ERR_INVALID_ARGUMENT
    assert copy(num_pairs=0, prs=None) == N.VFL_OK
    assert copy(num_layers=0) == N.VFL_OK
    big = layers(*([A] * (N.MAX_COPY_LAYERS + 1)))
    assert copy(k=big, v=big, num_layers=N.MAX_COPY_LAYERS + 1) == N.VFL_ERR_UNSUPPORTED
    assert copy(block_bytes=24) == N.VFL_ERR_INVALID_ARGUMENT
    assert copy(prs=None) == N.VFL_ERR_INVALID_ARGUMENT
    assert copy(k=layers(A, None)) == N.VFL_ERR_INVALID_ARGUMENT
    assert copy(v=layers(A, A + 4)) == N.VFL_ERR_INVALID_ARGUMENT
    assert b"layer 1" in native.vfl_last_error_message()
