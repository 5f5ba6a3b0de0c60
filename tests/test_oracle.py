"""Pins of the CPU oracle (test infrastructure) against fixtures it did not produce.

* attention: float64 softmax attention computed by torch on a dense gather of the pages
  (tests/golden/attention_cases.npz) - an implementation independent of the oracle.
* the reference engine run on the oracle reproduced HuggingFace ``generate`` tokens (checked
  when the trace was made and re-checked here from the stored tokens).
* per-step metadata, encoder slots and copy-on-write copies recorded from the unmodified
  reference engine (tests/golden/engine_trace.pt) - bit-exact.
"""

from __future__ import annotations

import pytest
import torch

from conftest import assert_attention_close, case_tensors, load_attention_cases

CASES = load_attention_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_attention_matches_float64(oracle_lib, case):
    dt = torch.float32 if case["dtype"] == "f32" else torch.bfloat16
    t = case_tensors(case)
    out = torch.empty_like(t["q"])
    bad = oracle_lib.attention(t["q"], t["k_cache"], t["v_cache"], out, t["query_start_loc"],
                               t["seq_lens"], case["scale"], bool(case["causal"]), t["block_table"])
    assert bad == 0
    assert_attention_close(out, t["expected"], dt, case["name"])


F32_CASES = [c for c in CASES if c["dtype"] == "f32" and int(max(c["seq_lens"])) >= 2]


@pytest.mark.parametrize("case", F32_CASES, ids=[c["name"] for c in F32_CASES])
@pytest.mark.parametrize("mistake", ["one_token_short", "scale_off_1pct"])
def test_planted_oracle_mistakes_fail_the_golden_check(oracle_lib, case, mistake):
    """A slip planted in the call of the oracle (one token short of each context, or a scale off
    by 1 %) fails the float64 golden check: the fixture and the fp32 bar can tell them apart."""
    t = case_tensors(case)
    lens, scale = t["seq_lens"].clone(), case["scale"]
    if mistake == "one_token_short":
        lens = (lens - 1).clamp(min=0)
    else:
        scale *= 1.01
    out = torch.empty_like(t["q"])
    oracle_lib.attention(t["q"], t["k_cache"], t["v_cache"], out, t["query_start_loc"], lens, scale,
                         bool(case["causal"]), t["block_table"])
    with pytest.raises(AssertionError):
        assert_attention_close(out, t["expected"], torch.float32, case["name"])


def test_engine_tokens_equal_hf_generate(engine_trace):
    for run in engine_trace["runs"]:
        assert run["tokens"] == run["hf_tokens"], run["name"]
        assert any(len(t) > 16 for t in run["tokens"]), "trace must cross block boundaries"
    assert sum(len(s["copies"]) for r in engine_trace["runs"] for s in r["steps"]) > 0


def test_engine_attention_snapshots(oracle_lib, engine_trace):
    n = 0
    for run in engine_trace["runs"]:
        for snap in run["attention_snapshots"]:
            out = torch.empty_like(snap["query"])
            oracle_lib.attention(snap["query"], snap["k_cache"], snap["v_cache"], out,
                                 snap["query_start_loc"], snap["seq_lens"], snap["scale"],
                                 snap["causal"], snap["block_table"])
            assert torch.equal(out, snap["output"])
            n += 1
    assert n >= 6


def test_prepare_matches_reference_steps(oracle_lib, engine_trace):
    from vflorence_b200.kv_cache import pack_decode_step

    for run in engine_trace["runs"]:
        bs = run["block_size"]
        for step in run["steps"]:
            b = len(step["positions"])
            host = pack_decode_step(step["block_tables"], step["positions"])
            width = host.size // b - 1
            table = torch.from_numpy(host[: b * width].reshape(b, width).copy())
            assert torch.equal(table, step["ctx_block_tables"])
            slots, lens, qsl = oracle_lib.prepare_decode(table, torch.tensor(step["positions"]), bs)
            assert torch.equal(slots, step["ctx_slot_mapping"])
            assert torch.equal(lens, step["ctx_context_lens"])
            assert torch.equal(qsl, step["ctx_query_start_loc"])


def test_encoder_slots_match_reference(oracle_lib, engine_trace):
    for run in engine_trace["runs"]:
        for enc in run["encodes"]:
            for (rids, n), slots in zip(enc["groups"], enc["group_slots"]):
                pages = torch.stack([enc["cross_pages"][rid][0] for rid in rids])
                assert torch.equal(oracle_lib.paged_slots(pages, n, run["block_size"]), slots)


def test_copy_on_write_copies_each_pair(oracle_lib):
    # the reference's own check (tests/test_engine.py:382-405): blocks filled with their index,
    # pairs (0, 2), (1, 3) -> every cache reads [0, 1, 0, 1]
    caches = [torch.zeros(4, 2, 16, 64) for _ in range(4)]
    for c in caches:
        for b in range(4):
            c[b] = b
    oracle_lib.copy_blocks(caches[:2], caches[2:], [(0, 2), (1, 3)])
    for c in caches:
        assert [c[b].unique().item() for b in range(4)] == [0, 1, 0, 1]


def test_reshape_and_cache_strided_and_padding(oracle_lib):
    g = torch.Generator().manual_seed(3)
    kc = torch.zeros(6, 2, 16, 64)
    vc = torch.zeros(6, 2, 16, 64)
    qkv = torch.randn(5, 3 * 2 * 64, generator=g)
    key = qkv[:, 128:256].reshape(5, 2, 64)  # token stride 384, like the decoder's fused qkv
    value = qkv[:, 256:].reshape(5, 2, 64)
    slots = torch.tensor([0, 17, -1, 95, 40])
    assert oracle_lib.reshape_and_cache(key, value, kc, vc, slots) == 0
    for t, s in enumerate(slots.tolist()):
        if s < 0:
            continue
        assert torch.equal(kc[s // 16, :, s % 16], key[t]) and torch.equal(vc[s // 16, :, s % 16], value[t])
    assert kc.count_nonzero() == 4 * 2 * 64
    assert oracle_lib.reshape_and_cache(key, value, kc, vc, torch.tensor([96, 0, 0, 0, 0])) == 1
