"""The drop-in, shown: ``vflorence_b200.paged_ops`` bound as ``vllm_cpu_attn`` under the
reference's own op bodies, driven by every recorded step of the reference engine's trace
(tests/golden/engine_trace.pt) in the argument forms the reference passes, against the C oracle.

The reference's ops (vflorence/layers/attention.py) take host tensors: ``_prepare`` builds the
step's context lengths, zero-padded block tables, slot mapping and ``arange`` query_start_loc on
the CPU (vflorence/engine/model_runner.py:290-337), ``stage_cross`` pads each row's pages with
``pad_sequence`` and keeps host ``seq_lens`` in 5-tuples (attention.py:9-39). The three functions
below restate those op bodies line for line, with ``vllm_cpu_attn`` replaced by the B200 module;
the product ops (``torch.ops.vflorence.*`` of this package) are driven with the same Context.
"""

from __future__ import annotations

import pytest
import torch

import vflorence_b200.paged_ops as vllm_cpu_attn  # the drop-in import
from conftest import assert_attention_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


class _Attn:
    def __init__(self, k_cache, v_cache, num_heads, head_dim):
        self.k_cache, self.v_cache, self.num_heads, self.head_dim = k_cache, v_cache, num_heads, head_dim


class _Layer:
    def __init__(self, cross: _Attn):
        self.encoder_attn = cross


def reference_stage_cross(layers, pages, enc_lens, block_size, isa):
    """vflorence/layers/attention.py:9-39 with vllm_cpu_attn = vflorence_b200.paged_ops."""
    attn = layers[0].encoder_attn
    block_table = torch.nn.utils.rnn.pad_sequence(pages, batch_first=True)
    seq_lens = torch.tensor(enc_lens, dtype=torch.int32)
    metadata = vllm_cpu_attn.get_scheduler_metadata(
        num_reqs=len(pages), num_heads=attn.num_heads, num_kv_heads=attn.num_heads, head_dim=attn.head_dim,
        seq_lens=seq_lens, dtype=attn.k_cache.dtype, query_start_loc=torch.arange(len(pages) + 1, dtype=torch.int32),
        causal=False, isa=isa, block_size=block_size)
    return [(layer.encoder_attn.k_cache, layer.encoder_attn.v_cache, block_table, seq_lens, metadata)
            for layer in layers]


def reference_self_attention(query, key, value, k_cache, v_cache, scale, ctx):
    """The body of vflorence::self_attention (attention.py:53-73)."""
    vllm_cpu_attn.reshape_and_cache(key, value, k_cache, v_cache, ctx.slot_mapping, isa=ctx.isa)
    out = torch.empty_like(query)
    vllm_cpu_attn.attention_with_kv_cache(query, k_cache, v_cache, out, ctx.query_start_loc, ctx.context_lens,
                                          scale=scale, causal=False, block_table=ctx.block_tables,
                                          scheduler_metadata=ctx.self_metadata)
    return out


def reference_cross_attention(query, layer_idx, scale, ctx):
    """The body of vflorence::cross_attention (attention.py:94-110)."""
    k_cache, v_cache, block_table, seq_lens, metadata = ctx.cross_staged[layer_idx]
    out = torch.empty_like(query)
    vllm_cpu_attn.attention_with_kv_cache(query, k_cache, v_cache, out, ctx.query_start_loc, seq_lens,
                                          scale=scale, causal=False, block_table=block_table,
                                          scheduler_metadata=metadata)
    return out


def _reference_context(step, run, isa, layers, dtype=torch.float32):
    """The Context the reference's _prepare publishes for a recorded step: its own host tensors,
    the self metadata from model_runner.py:308-319, and the cross staging rebuilt from each row's
    pages (the recorded padded table's leading ceil(enc_len / bs) entries)."""
    from vflorence_b200.context import Context

    bs, H, D = run["block_size"], run["num_heads"], run["head_dim"]
    lens = step["ctx_context_lens"]
    meta = vllm_cpu_attn.get_scheduler_metadata(
        num_reqs=len(lens), num_heads=H, num_kv_heads=H, head_dim=D, seq_lens=lens, dtype=dtype,
        query_start_loc=step["ctx_query_start_loc"], causal=False, isa=isa, block_size=bs)
    enc = step["cross_seq_lens"].tolist()
    pages = [step["cross_block_table"][i, : -(-n // bs)].clone() for i, n in enumerate(enc)]
    staged = reference_stage_cross(layers, pages, enc, bs, isa)
    assert torch.equal(staged[0][2], step["cross_block_table"])  # pad_sequence gives the recorded table
    return Context(context_lens=lens, block_tables=step["ctx_block_tables"], slot_mapping=step["ctx_slot_mapping"],
                   query_start_loc=step["ctx_query_start_loc"], self_metadata=meta, isa=isa, cross_staged=staged)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("run_name", ["greedy", "beam2", "beam4"])
@pytest.mark.parametrize("ops", ["reference_bodies", "product_ops"])
def test_reference_call_forms_replay_trace(engine_trace, oracle_lib, run_name, ops, dtype):
    """Every recorded step: append + self-attention and cross-attention of one layer, with the
    reference's host metadata, on the GPU and on the oracle; outputs within the bar of the dtype
    and the pools bit-exact after every append. In bf16 (head_dim 64) the product's
    self-attention op takes the tensor-core kernel with the KV append fused into it, here fed
    the reference's host slot mapping, lengths and tables."""
    from vflorence_b200 import attention  # noqa: F401  (registers torch.ops.vflorence.*)
    from vflorence_b200.context import set_context

    run = next(r for r in engine_trace["runs"] if r["name"] == run_name)
    bs, H, D = run["block_size"], run["num_heads"], run["head_dim"]
    isa = vllm_cpu_attn.get_isa(dtype, bs, D)
    g = torch.Generator().manual_seed(3)
    rnd = lambda *shape: torch.randn(*shape, generator=g).to(dtype)  # noqa: E731
    shape = (run["num_blocks"], H, bs, D)
    k_host, v_host = rnd(*shape), rnd(*shape)
    cross = (run["num_cross_blocks"], H, bs, D)
    ck_host, cv_host = rnd(*cross), rnd(*cross)
    k_dev, v_dev = k_host.to(DEV), v_host.to(DEV)
    layers = [_Layer(_Attn(ck_host.to(DEV), cv_host.to(DEV), H, D))]
    scale = D ** -0.5
    for n, step in enumerate(run["steps"]):
        B = len(step["ctx_context_lens"])
        q, k, v, qc = (rnd(B, H, D) for _ in range(4))
        ctx = _reference_context(step, run, isa, layers, dtype)
        if ops == "reference_bodies":
            out = reference_self_attention(q.to(DEV), k.to(DEV), v.to(DEV), k_dev, v_dev, scale, ctx)
            out_c = reference_cross_attention(qc.to(DEV), 0, scale, ctx)
        else:  # this package's custom ops, with the reference's Context
            set_context(**{f: getattr(ctx, f) for f in ("context_lens", "block_tables", "slot_mapping",
                                                         "query_start_loc", "self_metadata", "isa", "cross_staged")})
            try:
                out = torch.ops.vflorence.self_attention(q.to(DEV), k.to(DEV), v.to(DEV), k_dev, v_dev, scale)
                out_c = torch.ops.vflorence.cross_attention(qc.to(DEV), 0, scale)
            finally:
                set_context()
        assert oracle_lib.reshape_and_cache(k, v, k_host, v_host, step["ctx_slot_mapping"]) == 0
        want = torch.empty_like(q)
        oracle_lib.attention(q, k_host, v_host, want, step["ctx_query_start_loc"], step["ctx_context_lens"], scale,
                             False, step["ctx_block_tables"])
        want_c = torch.empty_like(qc)
        oracle_lib.attention(qc, ck_host, cv_host, want_c, torch.arange(B + 1, dtype=torch.int32),
                             step["cross_seq_lens"], scale, False, step["cross_block_table"])
        assert_attention_close(out, want, dtype, f"{run_name} step {n} self")
        assert_attention_close(out_c, want_c, dtype, f"{run_name} step {n} cross")
        assert torch.equal(k_dev.cpu(), k_host) and torch.equal(v_dev.cpu(), v_host), f"step {n} pools"
    assert vllm_cpu_attn.read_device_errors(DEV) == 0


def test_recorded_snapshots_through_reference_forms(engine_trace):
    """The six attention calls the trace snapshotted (self and cross, greedy and beams) with the
    reference's own inputs and pools, in its keyword form; outputs equal the reference run's."""
    for run in engine_trace["runs"]:
        bs, D = run["block_size"], run["head_dim"]
        isa = vllm_cpu_attn.get_isa(torch.float32, bs, D)
        for s in run["attention_snapshots"]:
            lens, qsl = s["seq_lens"], s["query_start_loc"]
            meta = vllm_cpu_attn.get_scheduler_metadata(
                num_reqs=len(lens), num_heads=run["num_heads"], num_kv_heads=run["num_heads"], head_dim=D,
                seq_lens=lens, dtype=s["k_cache"].dtype, query_start_loc=qsl, causal=False, isa=isa, block_size=bs)
            q = s["query"].to(DEV)
            out = torch.empty_like(q)
            vllm_cpu_attn.attention_with_kv_cache(q, s["k_cache"].to(DEV), s["v_cache"].to(DEV), out, qsl, lens,
                                                  scale=s["scale"], causal=s["causal"], block_table=s["block_table"],
                                                  scheduler_metadata=meta)
            assert_attention_close(out, s["output"], torch.float32, f"{run['name']} call {s['call']}")


def test_host_metadata_is_not_read_after_the_call():
    """A host block table changed right after the call does not change the result: the upload is
    taken inside the call (pageable memory is staged, pinned memory waited for)."""
    g = torch.Generator().manual_seed(9)
    H, D, bs, nb = 2, 64, 16, 40
    kc = torch.randn(nb, H, bs, D, generator=g).to(DEV)
    vc = torch.randn(nb, H, bs, D, generator=g).to(DEV)
    q = torch.randn(3, H, D, generator=g).to(DEV)
    lens = torch.tensor([40, 17, 64], dtype=torch.int32)
    qsl = torch.arange(4, dtype=torch.int32)
    isa = vllm_cpu_attn.get_isa(torch.float32, bs, D)
    meta = vllm_cpu_attn.get_scheduler_metadata(3, H, H, D, lens, torch.float32, qsl, False, isa, bs)
    table = torch.randperm(nb, generator=g)[:12].to(torch.int32).view(3, 4)
    want = torch.empty_like(q)
    vllm_cpu_attn.attention_with_kv_cache(q, kc, vc, want, qsl.to(DEV), lens.to(DEV), D ** -0.5, False,
                                          table.to(DEV), meta)
    for pinned in (False, True):
        host = table.clone().pin_memory() if pinned else table.clone()
        out = torch.empty_like(q)
        vllm_cpu_attn.attention_with_kv_cache(q, kc, vc, out, qsl, lens, D ** -0.5, False, host, meta)
        host.zero_()  # the caller reuses its buffer at once
        torch.cuda.synchronize()
        assert torch.equal(out, want)
