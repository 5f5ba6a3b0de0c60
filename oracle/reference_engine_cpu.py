"""ORACLE — test infrastructure only: the reference's own CPU decode engine, timed.

    python oracle/reference_engine_cpu.py --reference-root <vflorence checkout> [--configs cfg1,cfg2]
                                          [--threads N] [--requests K]

Runs the UNMODIFIED vflorence engine (``vflorence.LLM``, imported from ``--reference-root``) on
this machine's CPU cores, with ``oracle/vllm_cpu_attn`` (the C restatement of the attention
library, whose SIMD build is not installable here) standing in for ``vllm_cpu_attn``. The
workloads are BASELINE configs 1-4 exactly as ``bench.py --decode cfgN`` builds them: the same
random-init weights of the configs' shapes (BART-large; Florence-2-base and -large with their
DaViT towers; seed 0), the same seeded requests and images, the same sampling (EOS disabled, so
every request decodes ``max_tokens``), block size 16. ``--requests K`` times the first K
requests of a config only (cfg 4's 512 image requests take long on a CPU). One JSON line per config:
decode tokens/s = completion tokens of all requests / wall time of the whole job (encoding
included), as the reference counts them (vflorence/engine/llm_engine.py:114-118), with the
thread count. A short warm-up job (two requests, 4 tokens) runs first.

``bench.py`` runs this script as a child process (its cpu-baseline leg) with the reference
installed under ``baseline/_ref``, which travels with the tree; the figure it prints is a
reported CPU baseline, not something the product calls.
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

BART_LARGE = dict(vocab_size=50265, d_model=1024, encoder_layers=12, decoder_layers=12,
                  encoder_attention_heads=16, decoder_attention_heads=16, encoder_ffn_dim=4096,
                  decoder_ffn_dim=4096, max_position_embeddings=1024, activation_function="gelu",
                  decoder_start_token_id=2, eos_token_id=2, bos_token_id=0, pad_token_id=1, init_std=0.02)

# BASELINE configs 1-4, as bench.py's decode_config defines them.
CONFIGS = {
    "cfg1": dict(dtype=torch.float32, num_requests=8, lens=(200, 1000), ids=(4, 50264), id_seed=0,
                 params=dict(max_tokens=64, num_beams=1, eos_token_id=[]),
                 max_num_seqs=8, max_decoder_len=64, max_encoder_len=1000),
    "cfg2": dict(dtype=torch.bfloat16, num_requests=32, lens=(300, 1024), ids=(4, 50264), id_seed=1,
                 params=dict(max_tokens=142, num_beams=4, length_penalty=2.0, no_repeat_ngram_size=3,
                             eos_token_id=[]),
                 max_num_seqs=128, max_decoder_len=144, max_encoder_len=1024),
    # Florence-2-base shape: DaViT tower on 768x768 images (577 image tokens) + 6+6 text layers
    "cfg3": dict(kind="florence2", dtype=torch.bfloat16, num_requests=64, prompt=(3, 10), ids=(4, 51289),
                 id_seed=3, params=dict(max_tokens=256, num_beams=3, eos_token_id=[]),
                 max_num_seqs=192, max_decoder_len=256, max_encoder_len=592),
    # Florence-2-large shape: DaViT-large tower + 12+12 text layers, 512 requests, max_num_seqs 256
    "cfg4": dict(kind="florence2-large", dtype=torch.bfloat16, num_requests=512, prompt=(3, 10), ids=(4, 51289),
                 id_seed=4, params=dict(max_tokens=256, num_beams=3, eos_token_id=[]),
                 max_num_seqs=256, max_decoder_len=1024, max_encoder_len=592),
}

FLORENCE2_BASE_TEXT = dict(BART_LARGE, vocab_size=51290, d_model=768, encoder_layers=6, decoder_layers=6,
                           encoder_attention_heads=12, decoder_attention_heads=12, encoder_ffn_dim=3072,
                           decoder_ffn_dim=3072)
FLORENCE2_BASE_VISION = dict(embed_dim=[128, 256, 512, 1024], num_heads=[4, 8, 16, 32], num_groups=[4, 8, 16, 32],
                             depths=[1, 1, 9, 1], projection_dim=768)
FLORENCE2_LARGE_TEXT = dict(BART_LARGE, vocab_size=51290)
FLORENCE2_LARGE_VISION = dict(embed_dim=[256, 512, 1024, 2048], num_heads=[8, 16, 32, 64],
                              num_groups=[8, 16, 32, 64], depths=[1, 1, 9, 1], projection_dim=1024)
SHAPES = {"florence2": (FLORENCE2_BASE_TEXT, FLORENCE2_BASE_VISION),
          "florence2-large": (FLORENCE2_LARGE_TEXT, FLORENCE2_LARGE_VISION)}
IMAGE_TOKEN_ID, IMAGE_TOKENS, IMAGE_SIZE = 51289, 577, 768


def requests_of(cfg):
    """The seeded requests of bench.py's decode_requests: (encoder ids, pixel values or None)."""
    g = torch.Generator().manual_seed(cfg["id_seed"])
    reqs = []
    for _ in range(cfg["num_requests"]):
        if cfg.get("kind", "bart") != "bart":
            n = int(torch.randint(cfg["prompt"][0], cfg["prompt"][1] + 1, (1,), generator=g))
            prompt = torch.randint(*cfg["ids"], (n,), generator=g).tolist()
            px = torch.randn(3, IMAGE_SIZE, IMAGE_SIZE, generator=g)
            reqs.append(([IMAGE_TOKEN_ID] * IMAGE_TOKENS + prompt, px))
        else:
            n = int(torch.randint(cfg["lens"][0], cfg["lens"][1] + 1, (1,), generator=g))
            reqs.append((torch.randint(*cfg["ids"], (n,), generator=g).tolist(), None))
    return reqs


def save_checkpoint(kind: str, path: str) -> None:
    """Random-init weights of the config's shape (seed 0, as bench.py builds them), saved as a
    local HF checkpoint; Florence-2 also gets the preprocessor facts the engine reads (image
    token count and size)."""
    torch.manual_seed(0)
    if kind == "bart":
        from transformers import BartConfig, BartForConditionalGeneration

        model = BartForConditionalGeneration(BartConfig(**BART_LARGE))
    else:
        from transformers import Florence2Config, Florence2ForConditionalGeneration

        text, vision = SHAPES[kind]
        model = Florence2ForConditionalGeneration(Florence2Config(
            text_config=text, vision_config=vision, image_token_id=IMAGE_TOKEN_ID))
        with open(os.path.join(path, "preprocessor_config.json"), "w") as f:
            json.dump({"image_seq_length": IMAGE_TOKENS,
                       "crop_size": {"height": IMAGE_SIZE, "width": IMAGE_SIZE}}, f)
    model.eval().save_pretrained(path)


def _cpu_name() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True, help="vflorence checkout")
    ap.add_argument("--configs", default="cfg1,cfg2")
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    ap.add_argument("--requests", type=int, default=0,
                    help="time only the first K requests of each config (0: all of them)")
    args = ap.parse_args()
    torch.set_num_threads(args.threads)

    sys.path.insert(0, HERE)                 # the vllm_cpu_attn stand-in (oracle/vllm_cpu_attn)
    sys.path.insert(0, args.reference_root)
    import vllm_cpu_attn  # noqa: F401
    import vflorence.config as vconfig

    vconfig.AARCH64 = True  # block size 16, the BASELINE block size
    from vflorence import LLM, Request, SamplingParams

    with TemporaryDirectory() as root:
        for name in args.configs.split(","):
            cfg = CONFIGS[name]
            kind = cfg.get("kind", "bart")
            path = os.path.join(root, kind)
            if not os.path.isdir(path):
                os.makedirs(path)
                save_checkpoint(kind, path)
            reqs = requests_of(cfg)
            if args.requests:
                reqs = reqs[: args.requests]
            llm = LLM(path, max_num_seqs=cfg["max_num_seqs"], dtype=cfg["dtype"], compile=False,
                      max_decoder_len=cfg["max_decoder_len"], max_encoder_len=cfg["max_encoder_len"])
            assert llm.config.block_size == 16
            # no forced EOS (the bench workload's rules; [] is the reference's "none" form, where
            # the checkpoint's generation config would force EOS at the last position)
            params = SamplingParams(**dict(cfg["params"], forced_eos_token_id=[]))
            # warm-up images are blank, so no timed image is already in the engine's embedding cache
            warm = [Request(ids, None if px is None else torch.zeros_like(px)) for ids, px in reqs[:2]]
            llm.generate(warm, SamplingParams(**dict(cfg["params"], max_tokens=4)), use_tqdm=False)
            t0 = time.perf_counter()
            outs = llm.generate([Request(ids, px) for ids, px in reqs], params, use_tqdm=False)
            wall = time.perf_counter() - t0
            tokens = sum(len(o.completion_token_ids) for o in outs)
            print(json.dumps({
                "metric": "decode tokens/s", "config": name, "value": tokens / wall, "unit": "tokens/s",
                "impl": "reference engine (vflorence, unmodified) + C restatement of vllm_cpu_attn",
                "threads": args.threads, "requests": len(reqs), "of_requests": cfg["num_requests"],
                "completion_tokens": tokens, "wall_s": wall, "params": cfg["params"],
                "dtype": str(cfg["dtype"]).replace("torch.", ""), "compile": False,
                "cpu": _cpu_name()}), flush=True)
            del llm


if __name__ == "__main__":
    main()
