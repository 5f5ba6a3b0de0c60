"""KV append, copy-on-write copies and per-step metadata on the GPU: bit-exact against the oracle
and against the reference engine's recorded steps (tests/golden/engine_trace.pt)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def ops():
    from vflorence_b200 import paged_ops

    return paged_ops


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("tokens", [1, 7, 256, 37440])  # decode steps ... a 64-request encoder group
def test_reshape_and_cache_matches_oracle(oracle_lib, dtype, tokens):
    g = torch.Generator().manual_seed(tokens)
    H, D, bs = 16, 64, 16
    nb = tokens // bs + 8
    kc = torch.randn(nb, H, bs, D, generator=g).to(dtype)
    vc = torch.randn(nb, H, bs, D, generator=g).to(dtype)
    qkv = torch.randn(tokens, 3 * H * D, generator=g).to(dtype)
    key = qkv[:, H * D: 2 * H * D].reshape(tokens, H, D)   # strided, as the decoder's fused qkv
    value = qkv[:, 2 * H * D:].reshape(tokens, H, D)
    slots = torch.randperm(nb * bs, generator=g)[:tokens]
    slots[:: 5] = -1                                      # padding tokens are skipped
    kd, vd = kc.to(DEV), vc.to(DEV)
    ops().reshape_and_cache(key.to(DEV), value.to(DEV), kd, vd, slots.to(DEV))
    assert oracle_lib.reshape_and_cache(key.contiguous(), value.contiguous(), kc, vc, slots) == 0
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)


def test_reshape_and_cache_flags_out_of_range_slots():
    o = ops()
    o.read_device_errors(DEV)
    kc = torch.zeros(2, 2, 16, 64, device=DEV)
    k = torch.ones(2, 2, 64, device=DEV)
    o.reshape_and_cache(k, k, kc, kc.clone(), torch.tensor([32, 3], device=DEV))
    assert o.read_device_errors(DEV) & 0x2  # VFL_DEVERR_SLOT
    assert kc[0, :, 3].eq(1).all() and kc.sum() == 2 * 64


def test_copy_on_write_copies_each_pair():
    # the reference's check (tests/test_engine.py:382-405) through the device kernel
    from vflorence_b200.kv_cache import PagedKVCache

    kv = PagedKVCache(num_layers=3, num_heads=2, head_dim=64, block_size=16, num_blocks=4,
                      num_cross_blocks=2, dtype=torch.float32, device=DEV)
    caches = kv.k_caches + kv.v_caches
    for c in caches:
        for b in range(4):
            c[b] = b
    kv.copy_blocks([(0, 2), (1, 3)])
    for c in caches:
        assert [c[b].unique().item() for b in range(4)] == [0, 1, 0, 1]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_copy_blocks_matches_oracle(oracle_lib, dtype):
    g = torch.Generator().manual_seed(1)
    L, N = 12, 96
    ks = [torch.randn(N, 16, 16, 64, generator=g).to(dtype) for _ in range(L)]
    vs = [torch.randn(N, 16, 16, 64, generator=g).to(dtype) for _ in range(L)]
    perm = torch.randperm(N, generator=g).tolist()
    pairs = list(zip(perm[:40], perm[40:80]))
    kd, vd = [k.to(DEV) for k in ks], [v.to(DEV) for v in vs]
    ops().copy_blocks(kd, vd, pairs)
    oracle_lib.copy_blocks(ks, vs, pairs)
    for a, b in zip(kd + vd, ks + vs):
        assert torch.equal(a.cpu(), b)


def test_copy_blocks_device_pairs_out_of_range_flagged():
    o = ops()
    o.read_device_errors(DEV)
    k = torch.arange(4.0, device=DEV).view(4, 1, 1, 1).expand(4, 1, 16, 64).contiguous()
    v = k.clone()
    o.copy_blocks([k], [v], torch.tensor([[0, 9], [1, 2]], device=DEV))
    assert o.read_device_errors(DEV) & 0x1
    assert k[2].unique().item() == 1.0 and k[3].unique().item() == 3.0


def test_prepare_decode_replays_reference_steps(engine_trace):
    from vflorence_b200.kv_cache import PagedKVCache

    for run in engine_trace["runs"]:
        kv = PagedKVCache(num_layers=1, num_heads=2, head_dim=64, block_size=run["block_size"],
                          num_blocks=run["num_blocks"], num_cross_blocks=4, dtype=torch.float32,
                          device=DEV)
        for step in run["steps"]:
            st = kv.prepare_decode(step["block_tables"], step["positions"])
            assert torch.equal(st.block_tables.cpu(), step["ctx_block_tables"])
            assert torch.equal(st.slot_mapping.cpu(), step["ctx_slot_mapping"])
            assert torch.equal(st.context_lens.cpu(), step["ctx_context_lens"])
            assert torch.equal(st.query_start_loc.cpu(), step["ctx_query_start_loc"])


def test_encoder_slots_replay_reference(engine_trace):
    from vflorence_b200.kv_cache import PagedKVCache

    for run in engine_trace["runs"]:
        kv = PagedKVCache(num_layers=1, num_heads=2, head_dim=64, block_size=run["block_size"],
                          num_blocks=4, num_cross_blocks=run["num_cross_blocks"], dtype=torch.float32,
                          device=DEV)
        clears = list(run["clears"])
        for enc in run["encodes"]:
            while kv.cross.free != enc["cross_free_before"]:
                kv.clear_request(clears.pop(0)[0])
            for (rids, n), want in zip(enc["groups"], enc["group_slots"]):
                assert torch.equal(kv.page_requests(rids, n).cpu(), want)


def test_prepare_flags_positions_beyond_the_table():
    o = ops()
    o.read_device_errors(DEV)
    table = torch.tensor([[3, 4]], dtype=torch.int32, device=DEV)
    slots = torch.empty(1, dtype=torch.int64, device=DEV)
    lens = torch.empty(1, dtype=torch.int32, device=DEV)
    qsl = torch.empty(2, dtype=torch.int32, device=DEV)
    o.prepare_decode(table, torch.tensor([40], dtype=torch.int32, device=DEV), 16, slots, lens, qsl)
    assert o.read_device_errors(DEV) & 0x4
    assert slots.item() == -1 and lens.item() == 41 and qsl.tolist() == [0, 1]
