"""Generate tests/golden/decode_tokens.json: token ids of the UNMODIFIED reference engine on
BASELINE-shaped decode workloads (run once, where the reference is checked out).

    python tests/golden/make_decode_golden.py --reference-root <vflorence checkout> \
        [--only florence2_tiny,cfg1,cfg2,cfg3,cfg4,cfg2_fp32,cfg3_fp32,cfg4_fp32] [--bf16-requests 4]

The reference engine (``vflorence.LLM``, block size 16, ``compile=False``) runs on this machine's
CPU with ``oracle/vllm_cpu_attn`` (the C restatement) standing in for the un-installable
``vllm_cpu_attn``. Weights are never stored: every model is random-init on the CPU from a seed
(bench.py's ``build_decode_model`` for configs 1-4, the seed below for the tiny Florence-2), and
the fixture keeps a checksum of the weights so a test can tell that it rebuilt the same model.

* ``florence2_tiny``: a small random Florence-2 (DaViT tower + BART, fp32), three image requests
  with prompts of different lengths, greedy / 2 beams / 4 beams over the checkpoint's generation
  defaults. The reference's tokens are asserted equal to HuggingFace ``generate`` before they are
  stored, as the reference's own test does (vflorence tests/test_florence2.py:108-130).
* ``cfg1``: BASELINE config 1 as ``bench.py --decode cfg1`` runs it (BART-large shape, fp32,
  greedy, 8 requests, 64 tokens, EOS disabled), all requests. Also each step's gap between the
  two best logits of every row (how far each greedy decision was from a tie).
* ``cfg2``..``cfg4``: the first ``--bf16-requests`` requests of BASELINE configs 2-4 (bf16, beam
  search) as bench.py builds them.
* ``cfg2_fp32``..``cfg4_fp32``: the same requests and weights with fp32 arithmetic, where token
  identity is the bar (bf16 runs on two machines may take different beam paths).

The bench configs disable EOS and carry no forced EOS, so the reference is given
``forced_eos_token_id=[]`` (its "none" form; the checkpoint's generation config would force EOS
at the last position otherwise); the effective parameters are recorded next to the tokens.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from tempfile import TemporaryDirectory

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "decode_tokens.json")

# tiny Florence-2: 64 x 64 images -> 5 image tokens; head_dim 64; vocabulary 51290 so the image
# token id 51289 is an embedding row
TINY = {
    "seed": 0,
    "text": dict(vocab_size=51290, d_model=128, encoder_layers=2, decoder_layers=2, encoder_attention_heads=2,
                 decoder_attention_heads=2, encoder_ffn_dim=256, decoder_ffn_dim=256, max_position_embeddings=128,
                 activation_function="gelu", decoder_start_token_id=2, eos_token_id=2, bos_token_id=0,
                 pad_token_id=1, init_std=0.2),
    "vision": dict(embed_dim=[32, 64, 96, 128], num_heads=[2, 2, 2, 4], num_groups=[2, 2, 2, 4],
                   depths=[1, 1, 1, 1], projection_dim=128),
    "image_token_id": 51289,
    "image_size": 64,
    "requests": [dict(prompt_len=3, image_seed=21), dict(prompt_len=7, image_seed=22), dict(prompt_len=5, image_seed=23)],
    "prompt_seed": 5,
    # each run: the checkpoint's generation defaults plus these (min_length keeps EOS out until
    # the forced EOS of the last position, so every request decodes all max_tokens)
    "runs": [dict(max_tokens=20, num_beams=1, min_length=21),
             dict(max_tokens=20, num_beams=2, no_repeat_ngram_size=3, length_penalty=2.0),
             dict(max_tokens=20, num_beams=4, min_length=21)],
}


def weights_checksum(model) -> float:
    """float64 sum over every 997th element of every parameter (order of ``parameters()``)."""
    return float(sum(p.detach().double().flatten()[::997].sum().item() for p in model.parameters()))


def build_tiny_florence2():
    from transformers import Florence2Config, Florence2ForConditionalGeneration

    torch.manual_seed(TINY["seed"])
    with torch.device("cpu"):
        model = Florence2ForConditionalGeneration(Florence2Config(
            text_config=TINY["text"], vision_config=TINY["vision"], image_token_id=TINY["image_token_id"]))
    return model.eval()


def tiny_requests(num_image_tokens: int):
    """(encoder ids, pixel values [3, S, S]) of the tiny Florence-2 requests: image tokens, BOS,
    prompt ids drawn from [4, 51289), EOS - the form of the reference's own test
    (tests/test_florence2.py:26-34)."""
    g = torch.Generator().manual_seed(TINY["prompt_seed"])
    text = TINY["text"]
    out = []
    for r in TINY["requests"]:
        prompt = torch.randint(4, TINY["image_token_id"], (r["prompt_len"],), generator=g).tolist()
        ids = [TINY["image_token_id"]] * num_image_tokens + [text["bos_token_id"]] + prompt + [text["eos_token_id"]]
        px = torch.randn(3, TINY["image_size"], TINY["image_size"], generator=torch.Generator().manual_seed(r["image_seed"]))
        out.append((ids, px))
    return out


def _reference(reference_root: str):
    sys.path.insert(0, os.path.join(REPO, "oracle"))  # the vllm_cpu_attn stand-in
    sys.path.insert(0, reference_root)
    import vllm_cpu_attn  # noqa: F401
    import vflorence.config as vconfig

    vconfig.AARCH64 = True  # block size 16, the BASELINE block size (only compile choices otherwise)
    import vflorence

    return vflorence


def _effective(llm, params) -> dict:
    eff = params.with_defaults(llm._sampling_params)
    return {f: getattr(eff, f) for f in eff.__slots__}


def florence2_tiny(vf) -> dict:
    torch.set_num_threads(os.cpu_count())
    model = build_tiny_florence2()
    with torch.no_grad():
        n_img = model.model.get_image_features(torch.zeros(1, 3, TINY["image_size"], TINY["image_size"])).pooler_output.shape[1]
    reqs = tiny_requests(n_img)
    runs = []
    with TemporaryDirectory() as path:
        model.save_pretrained(path)
        for run in TINY["runs"]:
            params = vf.SamplingParams(**run)
            llm = vf.LLM(path, max_num_seqs=8, compile=False, max_decoder_len=32, max_encoder_len=32)
            assert llm.config.block_size == 16
            outs = llm.generate([vf.Request(ids, px) for ids, px in reqs], params, use_tqdm=False)
            tokens = [o.completion_token_ids for o in outs]
            hf_tokens = []
            for ids, px in reqs:
                with torch.no_grad():
                    kw = {k: v for k, v in run.items() if k != "max_tokens"}
                    ref = model.generate(input_ids=torch.tensor([ids]), pixel_values=px[None],
                                         max_new_tokens=run["max_tokens"], do_sample=False, **kw)
                hf_tokens.append(ref[0].tolist()[1:])
            assert tokens == hf_tokens, (run, tokens, hf_tokens)
            print(f"florence2_tiny {run}: reference engine == HF generate: {tokens}", flush=True)
            runs.append({"params": run, "sampling": _effective(llm, params), "tokens": tokens})
    return {"model": TINY, "num_image_tokens": n_img, "weights_checksum": weights_checksum(model), "runs": runs}


def bench_config(vf, name: str, num_requests: int | None, dtype=None) -> dict:
    """The reference engine on a BASELINE config as bench.py --decode builds it (in ``dtype``
    instead of the config's when given)."""
    sys.path.insert(0, REPO)
    import bench

    torch.set_num_threads(os.cpu_count())
    # the reference's own Request type: the product package is never imported here (it registers
    # custom ops under the reference's op names)
    cfg, model, reqs = bench.decode_setup(name, torch.device("cpu"), dtype=torch.float32, request_cls=vf.Request)
    if dtype is not None:
        cfg["dtype"] = dtype
    assert "vflorence_b200" not in sys.modules
    checksum = weights_checksum(model)
    if num_requests:
        reqs = reqs[:num_requests]
    margins: list = []
    with TemporaryDirectory() as path:
        model.save_pretrained(path)
        del model
        if cfg["kind"] == "florence2":
            with open(os.path.join(path, "preprocessor_config.json"), "w") as f:
                json.dump({"image_seq_length": cfg["image_tokens"], "crop_size": {"height": 768, "width": 768}}, f)
        llm = vf.LLM(path, max_num_seqs=cfg["max_num_seqs"], dtype=cfg["dtype"], compile=False,
                     max_decoder_len=cfg["max_decoder_len"], max_encoder_len=cfg["max_encoder_len"])
        assert llm.config.block_size == 16
        params = vf.SamplingParams(**dict(cfg["params"], forced_eos_token_id=[]))
        if cfg["params"]["num_beams"] == 1:  # greedy: record how close each decision was to a tie
            runner = llm.runner
            orig = runner._sample

            def _sample(seqs, logits):
                top = logits.float().topk(2, dim=-1).values
                margins.append({s.request_id: float(t[0] - t[1]) for s, t in zip(seqs, top)})
                return orig(seqs, logits)

            runner._sample = _sample
        t0 = time.perf_counter()
        outs = llm.generate(reqs, params, use_tqdm=False)
        wall = time.perf_counter() - t0
        eff = _effective(llm, params)
    tokens = [o.completion_token_ids for o in outs]
    print(f"{name}: {len(reqs)} requests, {sum(map(len, tokens))} tokens in {wall:.1f} s", flush=True)
    res = {"config": name, "dtype": str(cfg["dtype"]).replace("torch.", ""), "requests": len(reqs),
           "of_requests": cfg["num_requests"], "weights_checksum": checksum, "sampling": eff, "tokens": tokens}
    if margins:
        # per request, per generated position: top-1 minus top-2 logit of the reference's step
        res["logit_margins"] = [[round(m[rid], 6) for m in margins if rid in m] for rid in range(len(reqs))]
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True, help="vflorence checkout")
    ap.add_argument("--only", default="florence2_tiny,cfg1,cfg2,cfg3,cfg4,cfg2_fp32,cfg3_fp32,cfg4_fp32")
    ap.add_argument("--bf16-requests", type=int, default=4)
    args = ap.parse_args()
    vf = _reference(args.reference_root)
    data = {}
    if os.path.exists(OUT):
        with open(OUT) as f:
            data = json.load(f)
    for name in args.only.split(","):
        if name == "florence2_tiny":
            data[name] = florence2_tiny(vf)
        elif name.endswith("_fp32"):  # a bf16 config's first requests with fp32 arithmetic
            data[name] = bench_config(vf, name[: -len("_fp32")], args.bf16_requests, torch.float32)
        else:
            data[name] = bench_config(vf, name, None if name == "cfg1" else args.bf16_requests)
        with open(OUT, "w") as f:
            json.dump(data, f, separators=(",", ":"))
    print(f"wrote {OUT}: {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
