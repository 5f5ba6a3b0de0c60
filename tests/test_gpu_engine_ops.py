"""The custom ops as the decoder calls them (vflorence::self_attention / cross_attention with a
per-step Context), on the reference engine's recorded attention calls and on seeded steps."""

from __future__ import annotations

import pytest
import torch

from conftest import assert_attention_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_recorded_attention_calls(engine_trace):
    from vflorence_b200 import paged_ops as ops

    n = 0
    for run in engine_trace["runs"]:
        for snap in run["attention_snapshots"]:
            kc, vc = snap["k_cache"], snap["v_cache"]
            _, h, bs, d = kc.shape
            meta = ops.get_scheduler_metadata(snap["seq_lens"].numel(), h, h, d, snap["seq_lens"], kc.dtype,
                                              snap["query_start_loc"], snap["causal"], "sm100", bs)
            out = torch.empty_like(snap["query"], device=DEV)
            ops.attention_with_kv_cache(snap["query"].to(DEV), kc.to(DEV), vc.to(DEV), out,
                                        snap["query_start_loc"].to(DEV), snap["seq_lens"].to(DEV),
                                        snap["scale"], snap["causal"], snap["block_table"].to(DEV), meta)
            assert_attention_close(out, snap["output"], torch.float32, f"{run['name']} call {snap['call']}")
            n += 1
    assert n >= 6


class _Attn:
    def __init__(self, heads, head_dim):
        self.num_heads, self.head_dim = heads, head_dim
        self.k_cache = self.v_cache = None


class _Layer:
    def __init__(self, heads, head_dim):
        self.self_attn = _Attn(heads, head_dim)
        self.encoder_attn = _Attn(heads, head_dim)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
def test_decode_step_through_custom_ops(oracle_lib, dtype):
    """One decoder step of 2 layers: CoW copies, append + paged self-attention, grouped cross-
    attention over encoder pages shared by beams - against the oracle doing the same per row."""
    from vflorence_b200.attention import decoder_cross_attention, decoder_self_attention
    from vflorence_b200.context import set_context
    from vflorence_b200.kv_cache import PagedKVCache

    g = torch.Generator().manual_seed(3)
    H, D, bs, L = 4, 64, 16, 2
    layers = [_Layer(H, D) for _ in range(L)]
    kv = PagedKVCache(num_layers=L, num_heads=H, head_dim=D, block_size=bs, num_blocks=64,
                      num_cross_blocks=80, dtype=dtype, device=DEV)
    kv.bind(layers)
    for c in kv.k_caches + kv.v_caches:
        c.copy_(torch.randn(c.shape, generator=g).to(dtype))
    # two requests: encoder lengths 70 and 33, beams 3 and 1
    enc = {0: 70, 1: 33}
    for rid, n in enc.items():
        slots = kv.page_requests([rid], n)
        for li in range(L):
            k = torch.randn(n, H, D, generator=g).to(dtype).to(DEV)
            v = torch.randn(n, H, D, generator=g).to(dtype).to(DEV)
            kv.write_encoder_kv(li, k, v, slots)
    rows_req = [0, 0, 0, 1]
    tables = [[5, 9, 2], [5, 9, 3], [5, 9, 4], [7]]   # beams share blocks 5, 9
    positions = [40, 40, 40, 6]
    copies = [(2, 11)]                                  # one CoW pair this step
    kv.copy_blocks(copies)
    step = kv.prepare_decode(tables, positions)
    staged = kv.stage_cross(layers, rows_req)
    assert staged[0][5].tolist() == [0, 3, 4]          # beams grouped: one request, three rows
    set_context(context_lens=step.context_lens, block_tables=step.block_tables,
                slot_mapping=step.slot_mapping, query_start_loc=step.query_start_loc,
                self_metadata=step.self_metadata, isa=kv.isa, cross_staged=staged)
    try:
        B = len(positions)
        outs = []
        host_caches = [(kc.cpu(), vc.cpu()) for kc, vc in zip(kv.k_caches, kv.v_caches)]
        inputs = []
        for li in range(L):
            qkv = torch.randn(B, 3 * H * D, generator=g).to(dtype).to(DEV)
            q, k, v = (t.reshape(B, H, D) for t in qkv.chunk(3, dim=-1))
            qc = torch.randn(B, H, D, generator=g).to(dtype).to(DEV)
            so = decoder_self_attention(q, k, v, layers[li].self_attn.k_cache, layers[li].self_attn.v_cache, D ** -0.5)
            co = decoder_cross_attention(qc, li, D ** -0.5)
            outs.append((so.cpu(), co.cpu()))
            inputs.append((q.cpu().contiguous(), k.cpu().contiguous(), v.cpu().contiguous(), qc.cpu()))
    finally:
        set_context()
    # oracle: same step on host copies
    tab = torch.tensor([t + [0] * (3 - len(t)) for t in tables], dtype=torch.int32)
    slots = torch.tensor([tables[i][p // bs] * bs + p % bs for i, p in enumerate(positions)])
    lens = torch.tensor([p + 1 for p in positions], dtype=torch.int32)
    qsl = torch.arange(B + 1, dtype=torch.int32)
    for li in range(L):
        kc, vc = host_caches[li]
        oracle_lib.copy_blocks([kc], [vc], copies)
        q, k, v, qc = inputs[li]
        oracle_lib.reshape_and_cache(k, v, kc, vc, slots)
        ref = torch.empty_like(q)
        oracle_lib.attention(q, kc, vc, ref, qsl, lens, D ** -0.5, False, tab)
        assert_attention_close(outs[li][0], ref, dtype, f"self layer {li}")
        assert torch.equal(kv.k_caches[li].cpu(), kc) and torch.equal(kv.v_caches[li].cpu(), vc)
        # cross: per-row tables repeat each request's pages (the reference's staging)
        ck, cv = kv.cross_k_caches[li].cpu(), kv.cross_v_caches[li].cpu()
        pages = [kv.cross.pages[r][0] for r in rows_req]
        ctab = torch.nn.utils.rnn.pad_sequence(pages, batch_first=True)
        clens = torch.tensor([enc[r] for r in rows_req], dtype=torch.int32)
        cref = torch.empty_like(qc)
        oracle_lib.attention(qc, ck, cv, cref, qsl, clens, D ** -0.5, False, ctab)
        assert_attention_close(outs[li][1], cref, dtype, f"cross layer {li}")
