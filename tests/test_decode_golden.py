"""The decode-token fixture (tests/golden/decode_tokens.json) describes the workloads the GPU
parity tests run: the tiny Florence-2 rebuilds to the same weights on the CPU, and the BASELINE
entries were made with bench.py's own sampling parameters (plus the reference's "no forced EOS"
form) on bench.py's requests."""

from __future__ import annotations

import json
import os
import sys

import pytest
import torch

from conftest import GOLDEN, REPO

sys.path.insert(0, GOLDEN)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "decode_tokens.json")) as f:
        return json.load(f)


def test_tiny_florence2_rebuilds_to_the_fixture_weights(golden):
    import make_decode_golden as mk

    g = golden["florence2_tiny"]
    model = mk.build_tiny_florence2()
    assert mk.weights_checksum(model) == pytest.approx(g["weights_checksum"], rel=1e-12)
    with torch.no_grad():
        n = model.model.get_image_features(torch.zeros(1, 3, 64, 64)).pooler_output.shape[1]
    assert n == g["num_image_tokens"]
    reqs = mk.tiny_requests(n)
    assert [len(ids) for ids, _ in reqs] == [n + 2 + r["prompt_len"] for r in mk.TINY["requests"]]
    for run in g["runs"]:
        assert all(len(t) == run["params"]["max_tokens"] for t in run["tokens"])
        for k, v in run["params"].items():
            assert run["sampling"][k] == v


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg2_fp32", "cfg3_fp32", "cfg4_fp32"])
def test_bench_entries_use_bench_sampling(golden, name):
    import bench
    from vflorence_b200.engine import SamplingParams

    g, cfg = golden[name], bench.decode_config(name.split("_")[0])
    if name.endswith("_fp32"):
        cfg["dtype"] = torch.float32
    eff = SamplingParams.from_dict(g["sampling"])
    ours = SamplingParams.from_dict(cfg["params"])
    assert eff.forced_eos_token_id == [] and ours.forced_eos_token_id is None  # both: no forced EOS
    eff.forced_eos_token_id = None
    assert eff == ours
    assert g["dtype"] == str(cfg["dtype"]).replace("torch.", "")
    assert all(len(t) == cfg["params"]["max_tokens"] for t in g["tokens"])
    assert g["requests"] == (cfg["num_requests"] if name == "cfg1" else len(g["tokens"]))


def test_cfg1_weights_and_requests_rebuild(golden):
    """bench.py's cfg-1 model (CPU-seeded) has the checksum the reference ran with."""
    import bench
    import make_decode_golden as mk

    cfg, model, reqs = bench.decode_setup("cfg1", torch.device("cpu"))
    assert mk.weights_checksum(model) == pytest.approx(golden["cfg1"]["weights_checksum"], rel=1e-12)
    assert len(reqs) == 8 and all(200 <= len(r.input_ids) <= 1000 for r in reqs)
