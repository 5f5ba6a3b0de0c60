"""The engine around the paged path, replayed against the reference engine's golden trace
(tests/golden/engine_trace.pt): same random BART weights, fp32, block size 16, same requests
and sampling parameters. Greedy and beam tokens must be identical (the reference's tokens equal
HuggingFace generate), and every step's scheduling - positions, block tables, copy-on-write
pairs - must equal the reference's step for step."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _hf_model(trace):
    from transformers import BartConfig, BartForConditionalGeneration

    cfg = BartConfig(**{k: v for k, v in trace["runs"][0]["model_config"].items()
                        if k not in ("transformers_version", "architectures", "model_type")})
    model = BartForConditionalGeneration(cfg)
    model.load_state_dict(trace["model_state"])
    return model.to(DEV).eval()


@pytest.fixture(scope="module")
def hf_model(engine_trace):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return _hf_model(engine_trace)


@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "cuda_graphs"])
@pytest.mark.parametrize("run_name", ["greedy", "beam2", "beam4"])
def test_engine_replays_reference(engine_trace, hf_model, run_name, graphs):
    from vflorence_b200.engine import Engine, Request, SamplingParams

    run = next(r for r in engine_trace["runs"] if r["name"] == run_name)
    cfg = run["config"]
    params = SamplingParams.from_dict(run["sampling"])
    eng = Engine(hf_model, max_num_seqs=cfg["max_num_seqs"], max_decoder_len=cfg["max_decoder_len"],
                 max_encoder_len=hf_model.config.max_position_embeddings, block_size=16,
                 num_blocks=run["num_blocks"], record_steps=True, cuda_graphs=graphs)
    assert eng.kv.num_cross_blocks == run["num_cross_blocks"]
    tokens = eng.generate([Request(r) for r in run["requests"]], params)
    assert tokens == run["tokens"]
    assert tokens == run["hf_tokens"]
    assert len(eng.record) == len(run["steps"])
    for mine, ref in zip(eng.record, run["steps"]):
        assert mine["request_ids"] == ref["request_ids"]
        assert mine["positions"] == ref["positions"]
        assert mine["block_tables"] == ref["block_tables"]
        assert mine["copies"] == [tuple(c) for c in ref["copies"]]
    # everything released
    assert eng.blocks.num_free_blocks == eng.blocks.num_blocks and not any(eng.blocks.ref_counts)
    assert sorted(eng.kv.cross.free) == list(range(eng.kv.num_cross_blocks))
    from vflorence_b200 import paged_ops

    assert paged_ops.read_device_errors(DEV) == 0


def test_engine_bf16_tokens_same_length(engine_trace, hf_model):
    """bf16 may flip near-tie tokens (the reference accepts that, tests/verify_parity.py:59-67)
    but every request must still produce its full length under min_length."""
    from vflorence_b200.engine import Engine, Request, SamplingParams

    run = next(r for r in engine_trace["runs"] if r["name"] == "greedy")
    model = _hf_model(engine_trace).to(torch.bfloat16)
    eng = Engine(model, max_num_seqs=3, max_decoder_len=48, max_encoder_len=160)
    tokens = eng.generate([Request(r) for r in run["requests"]], SamplingParams.from_dict(run["sampling"]))
    assert [len(t) for t in tokens] == [len(t) for t in run["tokens"]]
    same = sum(a == b for t, u in zip(tokens, run["tokens"]) for a, b in zip(t, u))
    assert same >= 0.5 * sum(len(t) for t in tokens)


@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "cuda_graphs"])
def test_grouped_beams_match_row_by_row(engine_trace, graphs):
    """bf16 beam search with the beams of a request attending as one group (per-row block
    tables) decides exactly as row-by-row attention: each row's tiles are reduced in the same
    order, and a tile a row does not hold adds exact zeros."""
    from vflorence_b200.engine import Engine, Request, SamplingParams
    from vflorence_b200 import paged_ops

    run = next(r for r in engine_trace["runs"] if r["name"] == "beam4")
    cfg = run["config"]
    model = _hf_model(engine_trace).to(torch.bfloat16)
    results = []
    for group in ("always", False):
        eng = Engine(model, max_num_seqs=cfg["max_num_seqs"], max_decoder_len=cfg["max_decoder_len"],
                     max_encoder_len=model.config.max_position_embeddings, block_size=16,
                     num_blocks=run["num_blocks"], record_steps=True, cuda_graphs=graphs, group_beams=group)
        tokens = eng.generate([Request(r) for r in run["requests"]], SamplingParams.from_dict(run["sampling"]))
        results.append((tokens, eng.record))
    assert results[0][0] == results[1][0]
    assert results[0][1] == results[1][1]
    assert paged_ops.read_device_errors(DEV) == 0


def test_fused_encoder_kv_matches_gemm_then_append(engine_trace):
    """bf16: the encoder pages written by the fused projection + page write equal (to one bf16
    step) those of the projection GEMM followed by the append kernel."""
    from vflorence_b200.engine import Engine, Request, SamplingParams

    run = next(r for r in engine_trace["runs"] if r["name"] == "beam4")
    model = _hf_model(engine_trace).to(torch.bfloat16)
    pools = []
    for fused in (True, False):
        eng = Engine(model, max_num_seqs=16, max_decoder_len=8, max_encoder_len=model.config.max_position_embeddings,
                     fused_encoder_kv=fused)
        assert eng.fused_encoder_kv == fused
        params = SamplingParams.from_dict(dict(run["sampling"], max_tokens=2))
        for r in run["requests"]:
            eng.add_request(Request(r), params)
        eng.step()  # admits and encodes every request
        pools.append([torch.stack(c).float() for c in (eng.kv.cross_k_caches, eng.kv.cross_v_caches)])
    for a, b in zip(*pools):
        assert bool(((a - b).abs() <= 2e-2 + b.abs() * 2.0 ** -7).all())
        assert float((a == b).float().mean()) >= 0.99


def _tiny_florence2():
    """Florence-2-shaped model (DaViT vision tower + BART), random init, fp32: 64 x 64 images
    give 5 image tokens; head_dim 64."""
    from transformers import Florence2Config, Florence2ForConditionalGeneration

    text = dict(vocab_size=51290, d_model=128, encoder_layers=2, decoder_layers=2, encoder_attention_heads=2,
                decoder_attention_heads=2, encoder_ffn_dim=256, decoder_ffn_dim=256, max_position_embeddings=128,
                activation_function="gelu", decoder_start_token_id=2, eos_token_id=2, bos_token_id=0, pad_token_id=1)
    vision = dict(embed_dim=[32, 64, 96, 128], num_heads=[2, 2, 2, 4], num_groups=[2, 2, 2, 4], depths=[1, 1, 1, 1],
                  projection_dim=128)
    torch.manual_seed(0)
    with torch.device(DEV):
        model = Florence2ForConditionalGeneration(Florence2Config(text_config=text, vision_config=vision,
                                                                  image_token_id=51289))
    return model.eval()


def test_encoder_prepared_mask_matches_hf_padding_mask():
    """Ragged prompts with images, fp32: the engine's encoder (images copied one by one into the
    batch, the padding mask passed as a prepared 4-D mask, no host read of it) gives the hidden
    states of HuggingFace's own encoder with the 2-D padding mask, at every real position."""
    from vflorence_b200.engine.model import PagedSeq2Seq

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    hf = _tiny_florence2()
    m = PagedSeq2Seq(hf)
    g = torch.Generator().manual_seed(5)
    lens = [3, 8, 5, 8]
    ids = torch.full((len(lens), 5 + max(lens)), 1, dtype=torch.long)
    mask = torch.zeros_like(ids)
    for i, n in enumerate(lens):
        ids[i, :5 + n] = torch.tensor([51289] * 5 + torch.randint(4, 51289, (n,), generator=g).tolist())
        mask[i, :5 + n] = 1
    px = torch.randn(len(lens), 3, 64, 64, generator=g).to(DEV)
    ids, mask = ids.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        mine = m.encode(ids, px, mask)
        feats = hf.model.get_image_features(px).pooler_output
        emb = m.lm.get_input_embeddings()(ids)
        emb = emb.masked_scatter((ids == 51289).unsqueeze(-1).expand_as(emb), feats)
        ref = m.lm.encoder(inputs_embeds=emb, attention_mask=mask).last_hidden_state
    real = mask.bool()
    torch.testing.assert_close(mine[real], ref[real], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "cuda_graphs"])
def test_fused_layernorm_same_tokens(graphs):
    """fp32 Florence-2-shaped model: the decoder with each LayerNorm(h + x) in one launch
    generates the tokens of the decoder with the add and the torch modules."""
    from vflorence_b200.engine import Engine, Request, SamplingParams

    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    model = _tiny_florence2()
    g = torch.Generator().manual_seed(11)
    reqs = [Request([51289] * 5 + torch.randint(4, 51289, (n,), generator=g).tolist(),
                    torch.randn(3, 64, 64, generator=g)) for n in (3, 6, 4, 8, 5)]
    results = []
    for fused in (True, False):
        eng = Engine(model, max_num_seqs=6, max_decoder_len=24, max_encoder_len=32, cuda_graphs=graphs,
                     fused_layernorm=fused)
        assert eng.model.fused_layernorm == fused
        results.append(eng.generate(reqs, SamplingParams.from_dict(dict(max_tokens=20, num_beams=2,
                                                                        eos_token_id=[]))))
    assert results[0] == results[1]
    from vflorence_b200 import paged_ops

    assert paged_ops.read_device_errors(DEV) == 0
