"""Benchmark of the paged-KV attention path on B200 (the isolated kernel sweep).

    python bench.py [--gpus N --steps K --warmup W] [--batch B] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU; weak scaling)

One step = one decoder layer's paged attention for a batch of B sequences (bf16, 16 heads x 64,
block 16): the KV append of the step's token (reshape_and_cache), paged self-attention decode
over contexts drawn U[1, 4096] (seed 2; block tables a random permutation of the pool), and
cross-attention over 1024 encoder tokens per sequence. Synthetic inputs with the sweep's shapes
and distributions; the pools (about 13 GB at B=1024) are far larger than L2, so no L2 flush is
needed between steps.

``value`` = algorithmic HBM bytes per step / device time per step (GB/s), inputs resident in HBM.
``e2e``   = the same bytes over the time of the public API path with host buffers: every step
            uploads its inputs from pinned host memory, plans on the host, runs the ops and reads
            both outputs back - pipelined as a serving loop runs it (uploads and read-backs on
            their own streams with double buffers, overlapping the neighbouring steps' kernels;
            the host waits for each step's results one step later).
``roofline`` = the paged self-attention kernel (split partials merged as planned), timed with CUDA events in
            the timed region, against the measured HBM copy bandwidth.
``cpu_baseline`` = the C oracle (the restated vllm_cpu_attn arithmetic; the library itself cannot
            be installed) on the host cores, on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

H, D, BS, ENC_LEN, MAX_CTX = 16, 64, 16, 1024, 4096
DTYPE = torch.bfloat16
ELEM = 2
METRIC = "paged-attn HBM GB/s vs 8 TB/s"


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def _kernel_of(plan):
    """The attention kernel a plan launches."""
    if plan.schedule == 1:
        return "paged_attention_tc_balanced_kernel"
    return "paged_attention_tc_kernel" if plan.queries_per_cta == 8 else "paged_attention_kernel"


def _launches_of(plan):
    """Kernel launches of one attention call: the balanced wave and its merge, or the grid and
    its combine when the grid splits."""
    return 2 if plan.schedule == 1 else 1 + (plan.num_splits > 1)


def _plan_desc(plan):
    """The launch-shape fields of a plan, for the JSON lines."""
    d = {"kernel": _kernel_of(plan), "heads_per_cta": plan.heads_per_cta, "stages": plan.stages}
    if plan.schedule == 1:
        d.update(schedule="balanced", ctas=plan.balanced_ctas, min_tiles=plan.min_tiles)
    else:
        d.update(schedule="items", splits=plan.num_splits, blocks_per_split=plan.blocks_per_split)
    return d


def load_traffic():
    """dram bytes per algorithmic byte of the self-attention kernel, from the committed ncu
    summary (profiles/paged_decode_traffic.json), if one exists."""
    path = os.path.join(REPO, "profiles", "paged_decode_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


# ------------------------------------------------------------------------------------ workload

def make_workload(batch: int, seed: int, device):
    """Seeded synthetic step of the sweep (host-side metadata + device pools and inputs)."""
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, MAX_CTX + 1, (batch,), generator=g, dtype=torch.int32)
    nblk = (ctx + BS - 1) // BS
    n_self = int(nblk.sum())
    perm = torch.randperm(n_self, generator=g).to(torch.int32)
    width = int(nblk.max())
    table = torch.zeros(batch, width, dtype=torch.int32)
    offs = torch.cumsum(nblk, 0) - nblk
    for b in range(batch):
        table[b, : nblk[b]] = perm[offs[b]: offs[b] + nblk[b]]
    cw = math.ceil(ENC_LEN / BS)
    n_cross = batch * cw
    cross_table = torch.randperm(n_cross, generator=g).to(torch.int32).view(batch, cw).contiguous()
    pos = ctx - 1
    slots = table[torch.arange(batch), (pos // BS).long()].long() * BS + (pos % BS).long()
    w = dict(batch=batch, ctx=ctx, table=table, cross_table=cross_table, slots=slots,
             cross_lens=torch.full((batch,), ENC_LEN, dtype=torch.int32),
             qsl=torch.arange(batch + 1, dtype=torch.int32), n_self=n_self, n_cross=n_cross)
    if device is not None:
        gd = torch.Generator(device=device).manual_seed(seed)
        rnd = lambda *s: torch.randn(*s, generator=gd, device=device, dtype=DTYPE)  # noqa: E731
        w.update(k_cache=rnd(n_self, H, BS, D), v_cache=rnd(n_self, H, BS, D),
                 ck_cache=rnd(n_cross, H, BS, D), cv_cache=rnd(n_cross, H, BS, D),
                 q=rnd(batch, H, D), k_new=rnd(batch, H, D), v_new=rnd(batch, H, D), qc=rnd(batch, H, D))
    return w


def algorithmic_bytes(w) -> dict:
    """Minimum HBM bytes of one step (per op), as counted in the design notes."""
    B, ctx = w["batch"], w["ctx"].long()
    row = H * D * ELEM
    nblk = (ctx + BS - 1) // BS
    self_b = int(2 * ctx.sum()) * row + 2 * B * row + 4 * int(nblk.sum()) + 4 * B + 4 * (B + 1)
    append_b = 4 * B * row + 8 * B
    cross_b = 2 * B * ENC_LEN * row + 2 * B * row + 4 * B * math.ceil(ENC_LEN / BS) + 4 * B + 4 * (B + 1)
    return {"self": self_b, "append": append_b, "cross": cross_b, "total": self_b + append_b + cross_b}


# ---------------------------------------------------------------------------------- the step

class Step:
    """The three ops of one step through the public API (vflorence_b200.paged_ops)."""

    def __init__(self, w, device):
        from vflorence_b200 import paged_ops as ops

        self.ops, self.w, self.device = ops, w, device
        self.dev = {k: w[k].to(device) for k in ("table", "cross_table", "slots", "ctx", "cross_lens", "qsl")}
        self.meta_self = ops.get_scheduler_metadata(w["batch"], H, H, D, w["ctx"], DTYPE, w["qsl"], False,
                                                    "sm100", BS)
        self.meta_cross = ops.get_scheduler_metadata(w["batch"], H, H, D, w["cross_lens"], DTYPE, w["qsl"],
                                                     False, "sm100", BS)
        self.out = torch.empty_like(w["q"])
        self.out_c = torch.empty_like(w["qc"])
        plan_s, plan_c = ops.plan_of(self.meta_self), ops.plan_of(self.meta_cross)
        self.launches = 1 + _launches_of(plan_s) + _launches_of(plan_c)  # append + self + cross
        self.plans = (plan_s, plan_c)

    def append(self, k_new, v_new, slots):
        self.ops.reshape_and_cache(k_new, v_new, self.w["k_cache"], self.w["v_cache"], slots)

    def self_attn(self, q, out, meta, ctx, qsl, table):
        self.ops.attention_with_kv_cache(q, self.w["k_cache"], self.w["v_cache"], out, qsl, ctx, D ** -0.5,
                                         False, table, meta)

    def cross_attn(self, qc, out, meta, lens, qsl, table):
        self.ops.attention_with_kv_cache(qc, self.w["ck_cache"], self.w["cv_cache"], out, qsl, lens, D ** -0.5,
                                         False, table, meta)


# ------------------------------------------------------------------------------------ clocks

class ClockSampler:
    """Clock, power and throttle-reason samples of this GPU during a timed region: NVML read every
    5 ms by a thread (read-only queries), else nvidia-smi every 100 ms; either writes rows of the
    nvidia-smi trace format to one file, which ``summary`` reads."""

    # NVML clocks-event reason bits: hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap
    NVML_REASONS = (0x8, 0x40, 0x20, 0x4)
    INTERVAL_S = 0.005
    _count = 0

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        phys = device_index
        if vis:
            ids = [v.strip() for v in vis.split(",") if v.strip()]
            if device_index < len(ids) and ids[device_index].isdigit():
                phys = int(ids[device_index])
        self.phys = phys
        self.proc = None
        # the raw trace: VFL_CLOCKS_DIR when set (to keep it), else a temporary file
        out_dir = os.environ.get("VFL_CLOCKS_DIR") or tempfile.gettempdir()
        ClockSampler._count += 1  # one trace file per sampler of the process
        self.path = os.path.join(out_dir, f"vfl_clocks_gpu{phys}_{os.getpid()}_{ClockSampler._count}.csv")

    def _nvml_loop(self, nvml, handle):
        active = lambda bit: "Active" if self._reasons & bit else "Not Active"  # noqa: E731
        while not self._stop.is_set():
            try:
                sm = nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM)
                mx = nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM)
                pw = nvml.nvmlDeviceGetPowerUsage(handle) / 1000.0
                self._reasons = nvml.nvmlDeviceGetCurrentClocksThrottleReasons(handle)
            except Exception:  # a failed read drops the sample
                self._stop.wait(self.INTERVAL_S)
                continue
            self.fh.write(f"{sm}, {mx}, {pw:.2f}, {self._reasons:#x}, "
                          + ", ".join(active(b) for b in self.NVML_REASONS) + "\n")
            self._stop.wait(self.INTERVAL_S)

    def __enter__(self):
        import threading

        self.fh = open(self.path, "w")
        self._stop, self._thread, self._reasons = threading.Event(), None, 0
        try:
            import pynvml as nvml

            nvml.nvmlInit()
            handle = nvml.nvmlDeviceGetHandleByIndex(self.phys)
            self._thread = threading.Thread(target=self._nvml_loop, args=(nvml, handle), daemon=True)
            self._thread.start()
            self.proc = self._thread
            return self
        except Exception:
            self._thread = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.phys), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.fh.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["NVML and nvidia-smi unavailable"]}
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) != 8:
                    continue
                try:
                    rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
                except ValueError:
                    continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[3][1:]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "samples": len(rows), "power_w_max": max(r[2] for r in rows), "reasons": reasons}


# ------------------------------------------------------------------------------- CPU baseline

def host_threads() -> int:
    """Every host core this process may run on (torchrun exports OMP_NUM_THREADS=1; the CPU
    baseline deliberately ignores that)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(batch: int, seconds: float = 10.0, sample: int = 32):
    """The C oracle on the host cores over ``sample`` sequences of the same workload."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle

    oracle.build()
    w = make_workload(batch, 2, None)
    rows = torch.arange(sample)
    ctx = w["ctx"][rows]
    nblk = (ctx + BS - 1) // BS
    # compact host pools holding exactly the sampled sequences' blocks (values N(0, 1))
    g = torch.Generator().manual_seed(5)
    n_self = int(nblk.sum())
    kc = torch.randn(n_self, H, BS, D, generator=g).to(DTYPE)
    vc = torch.randn(n_self, H, BS, D, generator=g).to(DTYPE)
    # block tables: a random permutation of the sampled pool, as the GPU arm reads its pool
    perm = torch.randperm(n_self, generator=g).to(torch.int32)
    table = torch.zeros(sample, int(nblk.max()), dtype=torch.int32)
    pos = 0
    for i in range(sample):
        table[i, : nblk[i]] = perm[pos: pos + int(nblk[i])]
        pos += int(nblk[i])
    cw = math.ceil(ENC_LEN / BS)
    ck = torch.randn(sample * cw, H, BS, D, generator=g).to(DTYPE)
    cv = torch.randn(sample * cw, H, BS, D, generator=g).to(DTYPE)
    ctab = torch.randperm(sample * cw, generator=g).to(torch.int32).view(sample, cw)
    q = torch.randn(sample, H, D, generator=g).to(DTYPE)
    kn, vn = torch.randn(sample, H, D, generator=g).to(DTYPE), torch.randn(sample, H, D, generator=g).to(DTYPE)
    p = ctx.long() - 1
    slots = table[torch.arange(sample), (p // BS)].long() * BS + p % BS
    qsl = torch.arange(sample + 1, dtype=torch.int32)
    clens = torch.full((sample,), ENC_LEN, dtype=torch.int32)
    out, outc = torch.empty_like(q), torch.empty_like(q)
    threads = host_threads()
    sub = dict(batch=sample, ctx=ctx)
    nbytes = algorithmic_bytes(sub)["total"]
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.reshape_and_cache(kn, vn, kc, vc, slots)
        oracle.attention(q, kc, vc, out, qsl, ctx, D ** -0.5, False, table, threads)
        oracle.attention(q, ck, cv, outc, qsl, clens, D ** -0.5, False, ctab, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    full = algorithmic_bytes(w)["total"]
    return {"value": nbytes * reps / el / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "seconds_per_full_step": el / reps * full / nbytes,
            "sample": f"{sample} of the {batch} sequences (self ctx U[1,4096] + cross enc {ENC_LEN}; block "
                      f"tables a random permutation of the sampled pools), {reps} repetitions in {el:.1f} s",
            "seconds_per_step": el / reps}


def reference_engine_cpu(name: str, requests: int = 0, timeout: float = 1800.0) -> dict:
    """The reference's own decode engine timed on this host's cores: the unmodified vflorence
    installed under baseline/_ref, with the C restatement of vllm_cpu_attn standing in for the
    library, on the bench's decode workload (same weights, requests and sampling; first
    ``requests`` requests when > 0). A child process without the GPU: the reference registers
    the same custom-op names as this package, and it is a CPU figure."""
    root = os.path.join(REPO, "baseline", "_ref")
    if not os.path.isdir(os.path.join(root, "vflorence")):
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    threads = host_threads()
    cmd = [sys.executable, os.path.join(REPO, "oracle", "reference_engine_cpu.py"), "--reference-root", root,
           "--configs", name, "--threads", str(threads)] + (["--requests", str(requests)] if requests else [])
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS=str(threads))
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env, cwd=REPO)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"reference CPU engine did not finish within {timeout:.0f} s"}
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    if res.returncode != 0 or not lines:
        return {"unavailable": f"reference CPU engine exited {res.returncode}: {res.stderr.strip()[-200:]}"}
    r = json.loads(lines[-1])
    return {"value": r["value"], "unit": "tokens/s", "cores": r["threads"], "kind": "reference",
            "sample": f"{r['requests']} of the {r['of_requests']} requests, {r['completion_tokens']} tokens in "
                      f"{r['wall_s']:.1f} s (unmodified vflorence, C restatement of vllm_cpu_attn, compile=False)",
            "cpu": r.get("cpu")}


# -------------------------------------------------------------------------------------- sweep

def _cross_workload(batch, enc_len, seed, device):
    g = torch.Generator().manual_seed(seed)
    cw = math.ceil(enc_len / BS)
    table = torch.randperm(batch * cw, generator=g).to(torch.int32).view(batch, cw).contiguous()
    gd = torch.Generator(device=device).manual_seed(seed)
    rnd = lambda *s: torch.randn(*s, generator=gd, device=device, dtype=DTYPE)  # noqa: E731
    return dict(table=table, lens=torch.full((batch,), enc_len, dtype=torch.int32),
                k=rnd(batch * cw, H, BS, D), v=rnd(batch * cw, H, BS, D), q=rnd(batch, H, D))


def _graph_ms(body, reps):
    """Device time (ms) of one replay of a CUDA graph holding `reps` x body(), best of three."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        body()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(reps):
            body()
    graph.replay()
    torch.cuda.synchronize()
    best = None
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        best = a.elapsed_time(b) if best is None else min(best, a.elapsed_time(b))
    del graph
    return best


def _time_op(fn, reps, flush):
    """Mean device time (ms) of fn(), L2 flushed (a 256 MB write) before each call: CUDA-graph
    replays of reps x [flush, fn] minus reps x [flush], so no host time (Python, launches) lands
    inside the measurement - with eager launches it does for calls shorter than the host's
    per-call cost, which biases small calls (and split plans, whose combine is a second launch)."""
    reps = max(5, min(reps, 20))
    with_fn = _graph_ms(lambda: (flush.zero_(), fn()), reps)
    alone = _graph_ms(flush.zero_, reps)
    return max(with_fn - alone, 1e-6) / reps


def _cpu_attn_gbs(oracle, q, k, v, lens, table, nbytes, threads):
    qsl = torch.arange(lens.numel() + 1, dtype=torch.int32)
    out = torch.empty_like(q)
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.attention(q, k, v, out, qsl, lens, D ** -0.5, False, table, threads)
        reps += 1
        el = time.perf_counter() - t0
        if el > 0.5:
            return nbytes * reps / el / 1e9, el / reps


def run_sweep(args):
    """batch 1..1024, self ctx U[1,4096] and cross at 577 / 1024 tokens.
    One JSON line per point: device GB/s and us per call (L2 flushed before every call), the
    fraction of the measured HBM bandwidth, and the C oracle on the host cores (a sample of up
    to 16 sequences of the point)."""
    from vflorence_b200 import paged_ops as ops

    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle

    oracle.build()
    threads = host_threads()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    peak, _ = load_peaks()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    row = H * D * ELEM
    batches = [int(b) for b in args.sweep_batches.split(",")]
    for B in batches:
        w = make_workload(B, 2, device)
        nb = algorithmic_bytes(w)["self"]
        meta = ops.get_scheduler_metadata(B, H, H, D, w["ctx"], DTYPE, w["qsl"], False, "sm100", BS)
        d = {k: w[k].to(device) for k in ("table", "ctx", "qsl")}
        out = torch.empty_like(w["q"])
        fn = lambda: ops.attention_with_kv_cache(w["q"], w["k_cache"], w["v_cache"], out, d["qsl"],  # noqa: E731
                                                 d["ctx"], D ** -0.5, False, d["table"], meta)
        for _ in range(3):
            fn()
        reps = max(5, min(200, int(2e9 / max(nb, 1))))
        ms = _time_op(fn, reps, flush)
        # CPU oracle on a sample of the same sequences
        n = min(B, 16)
        rows = torch.arange(n)
        need = int(((w["ctx"][rows] + BS - 1) // BS).max())
        ids = w["table"][rows, :need]
        uniq, inv = torch.unique(ids.long(), return_inverse=True)
        kc, vc = w["k_cache"][uniq.to(device)].cpu(), w["v_cache"][uniq.to(device)].cpu()
        sub = dict(batch=n, ctx=w["ctx"][rows])
        cpu_gbs, cpu_s = _cpu_attn_gbs(oracle, w["q"][:n].cpu(), kc, vc, w["ctx"][rows].contiguous(),
                                       inv.to(torch.int32).contiguous(), algorithmic_bytes(sub)["self"], threads)
        plan = ops.plan_of(meta)
        print(json.dumps({"point": "self", "batch": B, "ctx": "U[1,4096]", "us": ms * 1e3,
                          "gbs": nb / ms / 1e6, "frac_of_measured_hbm": nb / ms / 1e6 / peak,
                          "plan": _plan_desc(plan),
                          "cpu_oracle_gbs": cpu_gbs, "cpu_threads": threads,
                          "cpu_sample_seqs": n}), flush=True)
        del w, kc, vc
        for enc in (577, 1024):
            c = _cross_workload(B, enc, 3, device)
            lens_d, table_d = c["lens"].to(device), c["table"].to(device)
            qsl = torch.arange(B + 1, dtype=torch.int32)
            meta_c = ops.get_scheduler_metadata(B, H, H, D, c["lens"], DTYPE, qsl, False, "sm100", BS)
            qsl_d = qsl.to(device)
            out_c = torch.empty_like(c["q"])
            fc = lambda: ops.attention_with_kv_cache(c["q"], c["k"], c["v"], out_c, qsl_d, lens_d,  # noqa: E731
                                                     D ** -0.5, False, table_d, meta_c)
            for _ in range(3):
                fc()
            nbc = 2 * B * enc * row + 2 * B * row + 4 * B * math.ceil(enc / BS) + 4 * B + 4 * (B + 1)
            ms_c = _time_op(fc, max(5, min(200, int(2e9 / nbc))), flush)
            n = min(B, 16)
            cw = math.ceil(enc / BS)
            ids = c["table"][:n].long().flatten()
            kc, vc = c["k"][ids.to(device)].cpu(), c["v"][ids.to(device)].cpu()
            tab = torch.arange(n * cw, dtype=torch.int32).view(n, cw)
            sub_b = 2 * n * enc * row + 2 * n * row
            cpu_gbs, _ = _cpu_attn_gbs(oracle, c["q"][:n].cpu(), kc, vc, c["lens"][:n].contiguous(), tab,
                                       sub_b, threads)
            print(json.dumps({"point": "cross", "batch": B, "enc_len": enc, "us": ms_c * 1e3,
                              "gbs": nbc / ms_c / 1e6, "frac_of_measured_hbm": nbc / ms_c / 1e6 / peak,
                              "cpu_oracle_gbs": cpu_gbs, "cpu_threads": threads, "cpu_sample_seqs": n}),
                  flush=True)
            del c, kc, vc
    # beams sharing a request's encoder pages (configs 2-4): R requests x beams query rows
    for R, beams, enc in ((64, 3, 587), (85, 3, 587), (256, 3, 587), (32, 4, 1024), (256, 4, 1024)):
        c = _cross_workload(R, enc, 4, device)
        q = torch.randn(R * beams, H, D, device=device, dtype=DTYPE)
        qsl = torch.arange(0, R * beams + 1, beams, dtype=torch.int32)
        meta_c = ops.get_scheduler_metadata(R, H, H, D, c["lens"], DTYPE, qsl, False, "sm100", BS)
        lens_d, table_d, qsl_d = c["lens"].to(device), c["table"].to(device), qsl.to(device)
        out_c = torch.empty_like(q)
        fb = lambda: ops.attention_with_kv_cache(q, c["k"], c["v"], out_c, qsl_d, lens_d,  # noqa: E731
                                                 D ** -0.5, False, table_d, meta_c)
        for _ in range(3):
            fb()
        nbb = 2 * R * enc * row + 2 * R * beams * row + 4 * R * math.ceil(enc / BS) + 4 * R + 4 * (R + 1)
        ms_b = _time_op(fb, 50, flush)
        print(json.dumps({"point": "cross_beams", "requests": R, "beams": beams, "enc_len": enc, "us": ms_b * 1e3,
                          "gbs": nbb / ms_b / 1e6, "frac_of_measured_hbm": nbb / ms_b / 1e6 / peak,
                          "rows_per_cta": ops.plan_of(meta_c).queries_per_cta}), flush=True)
        del c


def run_split_sweep(args):
    """The measurements behind the planner's split rule: for batch 8-1024 x 1, 3 or 4 query rows
    per request x context 128-2048 (near-uniform lengths U[3/4 ctx, ctx], and skewed U[1, ctx]
    from 1024 tokens), the planner's plan and every fixed split count x 2 or 4 stages x separate
    or in-kernel merge; then 16-512 requests at 3072-4096 tokens against split counts 4-24 (4
    stages, separate merge). Device time per call with L2 flushed. One JSON line per shape."""
    from vflorence_b200 import paged_ops as ops

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(192 * 1024 * 1024, dtype=torch.uint8, device=device)
    g = torch.Generator().manual_seed(0)

    def override(meta, splits, stages, merge):
        """Force a split count (as blocks per split), stage count and merge mode on a plan."""
        p = ops.plan_of(meta)
        max_blocks = -(-p.max_seq_len // BS)
        bps = -(-max_blocks // splits)
        p.blocks_per_split, p.num_splits = bps, -(-max_blocks // bps)
        p.stages, p.merge_in_kernel = stages, merge
        ws = 0
        if p.num_splits > 1:
            items = p.total_q * H * p.num_splits
            r256 = lambda x: -(-x // 256) * 256  # noqa: E731
            ws = r256(items * D * 4) + r256(items * 2 * 4)
            if merge:  # the arrival counters: one per (request, head group, query chunk), rounded up
                ws += r256(p.num_reqs * H * 4)
        p.workspace_bytes = ws
        return p.num_splits

    shapes = []  # (rows per request, requests, context, skewed, long): long shapes sweep fewer variants
    for rpr in (1, 3, 4):
        for R in (8, 32, 85, 128, 256, 1024):
            if rpr > 1 and R > 256:
                continue
            for ctx in (128, 592, 1024, 2048):
                for skew in (False, True):
                    if not (skew and ctx < 1024):
                        shapes.append((rpr, R, ctx, skew, False))
    shapes += [(1, R, ctx, skew, True) for R in (16, 32, 64, 128, 256, 512) for ctx in (3072, 4096)
               for skew in (False, True)]
    shapes += [(3, 32, 4096, True, True), (3, 85, 4096, True, True)]
    for rpr, R, ctx, skew, long_ctx in shapes:
        nb = -(-ctx // BS)
        if R * nb * BS * H * D * ELEM * 2 > (9e9 if long_ctx else 5e9):
            continue
        lens = torch.randint(1 if skew else max(1, ctx * 3 // 4), ctx + 1, (R,), generator=g).to(torch.int32)
        k = torch.randn(R * nb, H, BS, D, device=device, dtype=DTYPE)
        v = torch.randn_like(k)
        table = torch.randperm(R * nb, generator=g).to(torch.int32).view(R, nb).to(device)
        q = torch.randn(R * rpr, H, D, device=device, dtype=DTYPE)
        out = torch.empty_like(q)
        qsl = torch.arange(0, R * rpr + 1, rpr, dtype=torch.int32)
        lens_d, qsl_d = lens.to(device), qsl.to(device)
        mk = lambda: ops.get_scheduler_metadata(R, H, H, D, lens, DTYPE, qsl, False, "sm100", BS)  # noqa: E731

        def us(meta):
            call = lambda: ops.attention_with_kv_cache(q, k, v, out, qsl_d, lens_d, D ** -0.5,  # noqa: E731
                                                       False, table, meta)
            call()
            return round(_time_op(call, 10, flush) * 1e3, 2)

        base = mk()
        bp = ops.plan_of(base)
        row = {"point": "split_sweep", "rows_per_request": rpr, "requests": R, "ctx": ctx,
               "lengths": "U[1,ctx]" if skew else "U[3/4 ctx,ctx]",
               "plan": [bp.num_splits, bp.blocks_per_split, bp.stages, bp.merge_in_kernel],
               "plan_us": us(base)}
        var = {}
        counts = (4, 5, 6, 8, 10, 12, 16, 24) if long_ctx else (1, 2, 3, 4, 6, 8, 12, 16)
        for splits in sorted({max(-(-nb // 64), s_) for s_ in counts}):
            if splits > nb:
                break
            for stages in ((4,) if long_ctx else (2, 4)):
                for merge in ((0, 1) if splits > 1 and not long_ctx else (0,)):
                    m = mk()
                    ns = override(m, splits, stages, merge)
                    var[f"{ns}/{stages}/{merge}"] = us(m)
        best = min(var, key=var.get)
        row.update(best=[best, var[best]], plan_vs_best=round(row["plan_us"] / var[best], 3),
                   variants_splits_stages_merge=var)
        if ops.read_device_errors(device):
            raise RuntimeError(f"device error bits at {row}")
        print(json.dumps(row), flush=True)
        del k, v


def run_ring_sweep(args):
    """Under-filled attention shapes (few requests, the decode engine's cross-attention shapes)
    against the depth of the shared-memory ring: the planner's plan with 2, 4, 6 and 8 stages
    (device time per call, L2 flushed). One JSON line per shape."""
    from vflorence_b200 import paged_ops as ops

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(192 * 1024 * 1024, dtype=torch.uint8, device=device)
    g = torch.Generator().manual_seed(0)
    peak, _ = load_peaks()
    shapes = [("cross 32 requests x 4 beams x 1024", 32, 4, torch.full((32,), 1024, dtype=torch.int32)),
              ("cross 64 x 3 x 587", 64, 3, torch.full((64,), 587, dtype=torch.int32)),
              ("cross 85 x 3 x 592", 85, 3, torch.full((85,), 592, dtype=torch.int32)),
              ("self 8 x U[1,4096]", 8, 1, torch.randint(1, MAX_CTX + 1, (8,), generator=g).to(torch.int32)),
              ("self 32 x U[1,4096]", 32, 1, torch.randint(1, MAX_CTX + 1, (32,), generator=g).to(torch.int32)),
              ("self 32 x 2048", 32, 1, torch.full((32,), 2048, dtype=torch.int32))]
    for name, R, rpr, lens in shapes:
        nb = -(-int(lens.max()) // BS)
        k = torch.randn(R * nb, H, BS, D, device=device, dtype=DTYPE)
        v = torch.randn_like(k)
        table = torch.randperm(R * nb, generator=g).to(torch.int32).view(R, nb).to(device)
        q = torch.randn(R * rpr, H, D, device=device, dtype=DTYPE)
        out = torch.empty_like(q)
        qsl = torch.arange(0, R * rpr + 1, rpr, dtype=torch.int32)
        lens_d, qsl_d = lens.to(device), qsl.to(device)
        plan = ops.plan_of(ops.get_scheduler_metadata(R, H, H, D, lens, DTYPE, qsl, False, "sm100", BS))
        row = {"point": "ring_sweep", "shape": name, "plan": [plan.num_splits, plan.blocks_per_split, plan.stages]}
        for stages in (2, 4, 6, 8):
            meta = ops.get_scheduler_metadata(R, H, H, D, lens, DTYPE, qsl, False, "sm100", BS)
            ops.plan_of(meta).stages = stages
            call = lambda: ops.attention_with_kv_cache(q, k, v, out, qsl_d, lens_d, D ** -0.5,  # noqa: E731
                                                       False, table, meta)
            call()
            row[f"stages_{stages}_us"] = round(_time_op(call, 10, flush) * 1e3, 2)
        nbytes = int(lens.long().sum()) * H * D * ELEM * 2
        best = min(v_ for k_, v_ in row.items() if k_.startswith("stages_"))
        row["best_frac_of_hbm"] = round(nbytes / (best * 1e-6) / (peak * 1e9), 3)
        if ops.read_device_errors(device):
            raise RuntimeError(f"device error bits at {name}")
        print(json.dumps(row), flush=True)
        del k, v


def run_schedule_sweep(args):
    """The measurements behind the planner's choice of schedule: for 8-512 requests x 1, 3 or 4
    query rows x 128-4096 tokens (near-uniform U[3/4 ctx, ctx] and skewed U[1, ctx] lengths),
    the item grid of the planner's split rule against the balanced schedule at 2 and 4 stages x
    4-32 tiles per CTA at least. Device time per call with L2 flushed, bf16, 16 heads x 64,
    block 16, block tables a random permutation of the pool. One JSON line per shape."""
    from vflorence_b200 import paged_ops as ops

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    flush = torch.empty(192 * 1024 * 1024, dtype=torch.uint8, device=device)
    g = torch.Generator().manual_seed(0)
    peak, _ = load_peaks()
    shapes = []
    for rpr in (1, 3, 4):
        for R in (8, 32, 85, 128, 256, 512, 1024):
            if rpr > 1 and R > 256:
                continue
            for ctx in (128, 592, 1024, 2048, 4096):
                for skew in (False, True):
                    if not (skew and ctx < 1024) and (R * ctx <= 512 * 2048 or (R == 1024 and skew)):
                        shapes.append((rpr, R, ctx, skew))
    if args.sweep_shapes:
        keep = {tuple(int(x) for x in s.split("x")) for s in args.sweep_shapes.split(",")}
        shapes = [s for s in shapes if (s[0], s[1], s[2]) in keep]
    for rpr, R, ctx, skew in shapes:
        nb = -(-ctx // BS)
        lens = torch.randint(1 if skew else max(1, ctx * 3 // 4), ctx + 1, (R,), generator=g).to(torch.int32)
        k = torch.randn(R * nb, H, BS, D, device=device, dtype=DTYPE)
        v = torch.randn_like(k)
        table = torch.randperm(R * nb, generator=g).to(torch.int32).view(R, nb).to(device)
        q = torch.randn(R * rpr, H, D, device=device, dtype=DTYPE)
        out = torch.empty_like(q)
        qsl = torch.arange(0, R * rpr + 1, rpr, dtype=torch.int32)
        lens_d, qsl_d = lens.to(device), qsl.to(device)

        def us(meta):
            call = lambda: ops.attention_with_kv_cache(q, k, v, out, qsl_d, lens_d, D ** -0.5,  # noqa: E731
                                                       False, table, meta)
            call()
            return round(_time_op(call, 10, flush) * 1e3, 2)

        mk = lambda: ops.get_scheduler_metadata(R, H, H, D, lens, DTYPE, qsl, False, "sm100", BS)  # noqa: E731
        base = mk()
        bp = ops.plan_of(base)
        nbytes = int(lens.long().sum()) * H * D * ELEM * 2
        row = {"point": "schedule_sweep", "rows_per_request": rpr, "requests": R, "ctx": ctx,
               "lengths": "U[1,ctx]" if skew else "U[3/4 ctx,ctx]", "bytes": nbytes,
               "plan": [bp.schedule, bp.num_splits, bp.blocks_per_split, bp.stages, bp.min_tiles],
               "plan_us": us(base)}
        items = ops.set_schedule(mk(), ops.SCHEDULE_ITEMS)
        row["items_us"] = us(items)
        var = {}
        for stages in (2, 4):
            for min_tiles in (4, 8, 16, 32):
                m = mk()
                ops.plan_of(m).stages = stages
                ops.set_schedule(m, ops.SCHEDULE_BALANCED, min_tiles)
                var[f"{stages}/{min_tiles}"] = us(m)
        best = min(var, key=var.get)
        row.update(balanced_best=[best, var[best]], items_over_best_balanced=round(row["items_us"] / var[best], 3),
                   plan_frac_of_hbm=round(nbytes / (row["plan_us"] * 1e-6) / (peak * 1e9), 3),
                   balanced_stages_min_tiles=var)
        if ops.read_device_errors(device):
            raise RuntimeError(f"device error bits at {row}")
        print(json.dumps(row), flush=True)
        del k, v


def run_profile_topk(args):
    """The workload of the candidate-selection capture: three calls of the beam-search selection
    of a cfg-4 step (ROWS rows x the Florence-2 vocabulary of 51289, bf16 logits, k 6, log-softmax
    plus each row's cumulative log-prob), L2 flushed before each, checked against torch."""
    from vflorence_b200 import paged_ops as ops

    rows, vocab, k = args.profile_topk, 51289, 6
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator(device=device).manual_seed(0)
    logits = (torch.randn(rows, vocab, generator=g, device=device) * 3).to(DTYPE)
    cum = torch.randn(rows, generator=g, device=device)
    flush = torch.empty(192 * 1024 * 1024, dtype=torch.uint8, device=device)
    for _ in range(3):
        flush.zero_()
        vals, idx = ops.row_topk(logits, k, log_softmax=True, row_offset=cum)
    torch.cuda.synchronize()
    want_i = torch.sort(logits.float(), dim=1, descending=True, stable=True).indices[:, :k]
    want_v = torch.log_softmax(logits.float(), -1).gather(1, want_i) + cum[:, None]
    if not torch.equal(idx.long(), want_i) or float((vals - want_v).abs().max()) > 2e-5:
        raise RuntimeError("row_topk differs from torch")
    call = lambda: ops.row_topk(logits, k, log_softmax=True, row_offset=cum)  # noqa: E731
    print(json.dumps({"point": "profile_topk", "rows": rows, "vocab": vocab, "k": k,
                      "us_l2_flushed": round(_time_op(call, 10, flush) * 1e3, 2)}))


def run_profile_attn(args):
    """The workload of the attention captures: three calls of paged attention for R requests x
    ROWS query rows (beams sharing one request's pages, as the engine's cross-attention) over LEN
    tokens each, the planner's plan (bf16, 16 heads x 64, block 16, block tables a random
    permutation of the pool)."""
    from vflorence_b200 import paged_ops as ops

    R, rows, length = (int(x) for x in args.profile_attn.split(","))
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    g = torch.Generator().manual_seed(0)
    nb = -(-length // BS)
    k = torch.randn(R * nb, H, BS, D, device=device, dtype=DTYPE)
    v = torch.randn_like(k)
    table = torch.randperm(R * nb, generator=g).to(torch.int32).view(R, nb).to(device)
    q = torch.randn(R * rows, H, D, device=device, dtype=DTYPE)
    out = torch.empty_like(q)
    lens = torch.full((R,), length, dtype=torch.int32)
    qsl = torch.arange(0, R * rows + 1, rows, dtype=torch.int32)
    meta = ops.get_scheduler_metadata(R, H, H, D, lens, DTYPE, qsl, False, "sm100", BS)
    lens_d, qsl_d = lens.to(device), qsl.to(device)
    for _ in range(3):
        ops.attention_with_kv_cache(q, k, v, out, qsl_d, lens_d, D ** -0.5, False, table, meta)
    torch.cuda.synchronize()
    if ops.read_device_errors(device):
        raise RuntimeError("attention raised device error bits")
    p = ops.plan_of(meta)
    print(json.dumps({"point": "profile_attn", "requests": R, "rows": rows, "len": length,
                      "plan": [p.num_splits, p.blocks_per_split, p.stages, p.heads_per_cta]}))


def run_profile_step(args):
    """The workload of the decode-step launch list: the config's engine with CUDA graphs, one
    wave of requests, 120 steps (half of max_tokens for shorter jobs), then one step between
    torch.cuda.profiler.start() and stop() (capture it with ncu --profile-from-start off)."""
    from vflorence_b200.engine import Engine, SamplingParams

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg, model, reqs = decode_setup(args.profile_step, device)
    params = SamplingParams.from_dict(cfg["params"])
    reqs = reqs[: cfg["max_num_seqs"] // params.num_beams]
    eng = Engine(model, max_num_seqs=cfg["max_num_seqs"], max_decoder_len=cfg["max_decoder_len"],
                 max_encoder_len=cfg["max_encoder_len"], block_size=BS, cuda_graphs=True)
    eng.graphs.capture(cfg["max_num_seqs"], params.num_beams)
    for r in reqs:
        eng.add_request(r, params)
    with torch.inference_mode():
        for _ in range(min(120, params.max_tokens // 2)):
            eng.step()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        eng.step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
    print(json.dumps({"point": "profile_step", "config": args.profile_step, "rows": eng.rt.num_running}))


def run_profile_kv_proj(args):
    """The workload of the K/V projection captures: three calls of kv_proj_paged at the given
    token count (hidden 1024, 16 heads x 64, block 16, random slots; from 6144 tokens the 2-SM
    kernel)."""
    from vflorence_b200 import paged_ops as ops

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    T, K, heads = args.profile_kv_proj, 1024, 16
    g = torch.Generator(device=device).manual_seed(0)
    hidden = torch.randn(T, K, generator=g, device=device).to(torch.bfloat16)
    w = (torch.randn(2 * heads * D, K, generator=g, device=device) / K ** 0.5).to(torch.bfloat16)
    b = torch.randn(2 * heads * D, generator=g, device=device).to(torch.bfloat16)
    nb = -(-T // BS) + 1
    kc = torch.zeros(nb, heads, BS, D, device=device, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(nb * BS, generator=g, device=device)[:T].to(torch.int64)
    for _ in range(3):
        ops.kv_proj_paged(hidden, w, b, kc, vc, slots)
    torch.cuda.synchronize()
    if ops.read_device_errors(device):
        raise RuntimeError("kv_proj_paged raised device error bits")
    print(json.dumps({"point": "profile_kv_proj", "tokens": T}))


# ---------------------------------------------------------------------------- decode (engine)

def decode_config(name: str):
    """model shape, dtype, sampling and synthetic requests."""
    from transformers import BartConfig

    bart_large = dict(vocab_size=50265, d_model=1024, encoder_layers=12, decoder_layers=12,
                      encoder_attention_heads=16, decoder_attention_heads=16, encoder_ffn_dim=4096,
                      decoder_ffn_dim=4096, max_position_embeddings=1024, activation_function="gelu",
                      decoder_start_token_id=2, eos_token_id=2, bos_token_id=0, pad_token_id=1,
                      init_std=0.02)
    if name == "cfg1":
        return dict(kind="bart", text=bart_large, dtype=torch.float32, num_requests=8, lens=(200, 1000),
                    ids=(4, 50264), id_seed=0, params=dict(max_tokens=64, num_beams=1, eos_token_id=[]),
                    max_num_seqs=8, max_decoder_len=64, max_encoder_len=1000)
    if name == "cfg2":
        return dict(kind="bart", text=bart_large, dtype=torch.bfloat16, num_requests=32, lens=(300, 1024),
                    ids=(4, 50264), id_seed=1,
                    params=dict(max_tokens=142, num_beams=4, length_penalty=2.0, no_repeat_ngram_size=3,
                                eos_token_id=[]),
                    max_num_seqs=128, max_decoder_len=144, max_encoder_len=1024)
    florence_text = dict(bart_large, vocab_size=51290)
    if name == "cfg3":
        text = dict(florence_text, d_model=768, encoder_layers=6, decoder_layers=6, encoder_attention_heads=12,
                    decoder_attention_heads=12, encoder_ffn_dim=3072, decoder_ffn_dim=3072)
        vision = dict(embed_dim=[128, 256, 512, 1024], num_heads=[4, 8, 16, 32], num_groups=[4, 8, 16, 32],
                      depths=[1, 1, 9, 1], projection_dim=768)
        return dict(kind="florence2", text=text, vision=vision, dtype=torch.bfloat16, num_requests=64,
                    prompt=(3, 10), ids=(4, 51289), id_seed=3,
                    params=dict(max_tokens=256, num_beams=3, eos_token_id=[]),
                    max_num_seqs=192, max_decoder_len=256, max_encoder_len=592)
    if name == "cfg4":
        vision = dict(embed_dim=[256, 512, 1024, 2048], num_heads=[8, 16, 32, 64], num_groups=[8, 16, 32, 64],
                      depths=[1, 1, 9, 1], projection_dim=1024)
        return dict(kind="florence2", text=florence_text, vision=vision, dtype=torch.bfloat16, num_requests=512,
                    prompt=(3, 10), ids=(4, 51289), id_seed=4,
                    params=dict(max_tokens=256, num_beams=3, eos_token_id=[]),
                    max_num_seqs=256, max_decoder_len=1024, max_encoder_len=592)
    raise ValueError(name)


def build_decode_model(cfg, device, dtype=None):
    """Random-init weights of the config's shape: drawn on the CPU from seed 0 (so every device,
    and the reference engine's checkpoint of the same model, holds the same values), then moved
    to ``device`` and cast to ``dtype`` (default: the config's)."""
    from transformers import BartConfig, BartForConditionalGeneration

    torch.manual_seed(0)
    with torch.device("cpu"):
        if cfg["kind"] == "bart":
            model = BartForConditionalGeneration(BartConfig(**cfg["text"]))
        else:
            from transformers import Florence2Config, Florence2ForConditionalGeneration

            fc = Florence2Config(text_config=cfg["text"], vision_config=cfg["vision"], image_token_id=51289)
            model = Florence2ForConditionalGeneration(fc)
    return model.eval().to(device).to(dtype or cfg["dtype"])


def decode_setup(name: str, device, dtype=None, request_cls=None):
    """(config, model, requests) of a BASELINE decode config on ``device``; Florence-2 configs
    learn their image-token count from the built vision tower."""
    cfg = decode_config(name)
    model = build_decode_model(cfg, device, dtype)
    if cfg["kind"] == "florence2":
        with torch.inference_mode():
            px = torch.zeros(1, 3, 768, 768, device=device, dtype=dtype or cfg["dtype"])
            cfg["image_tokens"] = model.model.get_image_features(px).pooler_output.shape[1]
    return cfg, model, decode_requests(cfg, device, request_cls)


def decode_requests(cfg, device, request_cls=None):
    """The config's seeded requests as ``request_cls(input_ids, pixel_values)`` (default: the
    engine's Request)."""
    if request_cls is None:
        from vflorence_b200.engine import Request as request_cls

    Request = request_cls
    g = torch.Generator().manual_seed(cfg["id_seed"])
    reqs = []
    for i in range(cfg["num_requests"]):
        if cfg["kind"] == "bart":
            n = int(torch.randint(cfg["lens"][0], cfg["lens"][1] + 1, (1,), generator=g))
            reqs.append(Request(torch.randint(*cfg["ids"], (n,), generator=g).tolist()))
        else:
            n = int(torch.randint(cfg["prompt"][0], cfg["prompt"][1] + 1, (1,), generator=g))
            prompt = torch.randint(*cfg["ids"], (n,), generator=g).tolist()
            px = torch.randn(3, 768, 768, generator=g)
            reqs.append(Request([51289] * cfg["image_tokens"] + prompt, px))
    return reqs


def poisson_arrivals(n: int, rate: float, seed: int = 7) -> list[float]:
    """Arrival offsets (seconds) of ``n`` requests of a Poisson process with ``rate`` per second:
    cumulative sums of seeded exponential gaps."""
    g = torch.Generator().manual_seed(seed)
    gaps = torch.empty(n, dtype=torch.float64).exponential_(rate, generator=g)
    return torch.cumsum(gaps, 0).tolist()


def serve_arrivals(eng, reqs, params, arrivals):
    """Continuous batching with arrivals, as a server loop drives the reference's engine
    (vflorence/engine/llm_engine.py:34-63): each request is added when its arrival time has
    passed, a step runs whenever anything is admitted or waiting, and the loop idles only when
    nothing is. Returns (outputs in request order, per-request latency in seconds from arrival
    to the step that finished it)."""
    t0 = time.perf_counter()
    rid_of, arrived, latency = [], {}, {}
    i = 0
    try:
        while i < len(reqs) or not eng.is_finished():
            now = time.perf_counter() - t0
            while i < len(reqs) and arrivals[i] <= now:
                rid = eng.add_request(reqs[i], params)
                rid_of.append(rid)
                arrived[rid] = arrivals[i]
                i += 1
            if eng.is_finished():
                time.sleep(max(0.0, arrivals[i] - (time.perf_counter() - t0)))
                continue
            for rid in eng.step():
                latency[rid] = time.perf_counter() - t0 - arrived[rid]
    except BaseException:
        eng.abort()  # as Engine.generate does: no request is left half-served
        raise
    return [eng.outputs.pop(r) for r in rid_of], [latency[r] for r in rid_of]


def decode_generate(cfg, model, reqs, eager: bool = False, world: int = 1, arrivals=None, timer=None):
    """The engine's job on ``reqs`` as the decode leg times it: start-up warm-up, then every
    request encoded and decoded from scratch - all queued at the start, or added at their
    ``arrivals`` (seconds from the start). ``timer``: a PhaseTimer bracketing the job's phases.
    Returns (generated tokens per request, seconds, per-request latencies or None)."""
    from vflorence_b200.engine import Engine, SamplingParams

    for r in reqs:  # images wait in pinned host memory, as a pinned data loader hands them over
        if r.pixel_values is not None and not r.pixel_values.is_pinned():
            r.pixel_values = r.pixel_values.pin_memory()
    params = SamplingParams.from_dict(cfg["params"])
    eng = Engine(model, max_num_seqs=cfg["max_num_seqs"], max_decoder_len=cfg["max_decoder_len"],
                 max_encoder_len=cfg["max_encoder_len"], block_size=BS, cuda_graphs=not eager)
    # warm-up, as a server does at start-up: one wave of this rank's requests (the encoder and
    # library kernels for the batch shapes the run meets; first use of a kernel otherwise lands
    # in the timed region and cost up to seconds), 4 tokens each; graphs for every batch size
    # this run can reach are captured up front. The timed run then encodes and decodes every
    # request from scratch.
    wave = max(1, min(len(reqs), cfg["max_num_seqs"] // params.num_beams))
    eng.generate(reqs[:wave], SamplingParams.from_dict(dict(cfg["params"], max_tokens=4)))
    if eng.graphs is not None:
        eng.graphs.capture(min(cfg["max_num_seqs"], len(reqs) * params.num_beams), params.num_beams)
    eng.timer = timer
    barrier(world)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    latency = None
    with torch.inference_mode():
        if arrivals is None:
            outs = eng.generate(reqs, params)
        else:
            outs, latency = serve_arrivals(eng, reqs, params, arrivals)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    barrier(world)
    return outs, elapsed, latency


def decode_measure(name: str, world: int, rank: int, local: int, eager: bool = False,
                   arrival_rate: float = 0.0, setup=None) -> dict:
    """End-to-end decode tokens/s of the engine around the paged path on one BASELINE config:
    completion tokens of all requests / wall time of the whole job (max over ranks). The
    requests are dealt to the ranks whole (strong scaling: the job is fixed); with
    ``arrival_rate`` > 0 they arrive as a seeded Poisson process instead of all at the start, and
    the line adds per-request latency percentiles. ``per_rank`` splits each rank's job into the
    vision tower, text encoder, encoder K/V paging and decode steps (CUDA-event time), plus its
    start-up (weights, warm-up, graph capture). ``setup``: a ready (cfg, model, requests).
    Synthetic:
    random-init weights of the config's shape, seeded ids and N(0,1) images; EOS is disabled so
    every request decodes exactly max_tokens tokens (random weights have no natural stop)."""
    from vflorence_b200.engine.timing import PhaseTimer
    from vflorence_b200.sharding import assign_requests, gather_to_rank0, max_over_ranks, sum_over_ranks

    device = torch.device("cuda", local)
    t_start = time.perf_counter()
    cfg, model, reqs = setup if setup is not None else decode_setup(name, device)
    costs = [len(r.input_ids) + cfg["params"]["num_beams"] * cfg["params"]["max_tokens"] for r in reqs]
    shard = assign_requests(costs, world)[rank]
    mine = [reqs[i] for i in shard]
    arrivals = None
    if arrival_rate > 0:  # the job's arrival times; each rank serves its own requests as they arrive
        every = poisson_arrivals(len(reqs), arrival_rate)
        arrivals = [every[i] for i in shard]
    timer = PhaseTimer()
    outs, elapsed, latency = decode_generate(cfg, model, mine, eager, world, arrivals, timer)
    startup = time.perf_counter() - t_start - elapsed
    tokens = sum(len(o) for o in outs)
    phases = {k: round(v / 1e3, 4) if k != "steps" else v for k, v in timer.summary().items()}
    per_rank = gather_to_rank0({"rank": rank, "requests": len(mine), "tokens": tokens, "wall_s": round(elapsed, 4),
                                "startup_s": round(startup, 2), "phases_s": phases})
    total_tokens = sum_over_ranks(float(tokens))
    wall = max_over_ranks(elapsed)
    line = {"metric": "decode tokens/s", "config": name, "value": total_tokens / wall, "unit": "tokens/s",
            "n_gpus": world, "scaling": "strong", "requests": cfg["num_requests"],
            "completion_tokens": int(total_tokens), "wall_s": wall, "params": cfg["params"],
            "dtype": str(cfg["dtype"]).replace("torch.", ""), "max_num_seqs": cfg["max_num_seqs"],
            "cuda_graphs": not eager, "data": "synthetic (random-init weights)",
            "arrivals": (f"Poisson, {arrival_rate:g} requests/s (seed 7), dealt to ranks by request"
                         if arrivals is not None else "all queued at the start (offline)"),
            "per_rank": per_rank}
    if latency is not None:
        lat = sorted(x for r in gather_to_rank0(latency) or [] for x in r) if world > 1 else sorted(latency)
        if lat:
            line["latency_s"] = {"p50": lat[len(lat) // 2], "p90": lat[int(0.9 * (len(lat) - 1))], "max": lat[-1]}
    return line


def decode_legs(name: str, world: int, rank: int, local: int, eager: bool = False, arrival_rate: float = 0.0):
    """The offline job, then - with ``arrival_rate`` > 0 - the same requests arriving as a Poisson
    process, on the same weights (built once). One line; the Poisson job under ``poisson``."""
    if world > 1:  # ranks share the host's cores while they build their weights
        torch.set_num_threads(max(1, (os.cpu_count() or 8) // world))
    t0 = time.perf_counter()
    setup = decode_setup(name, torch.device("cuda", local))
    build_s = time.perf_counter() - t0
    line = decode_measure(name, world, rank, local, eager, setup=setup)
    if arrival_rate > 0:
        p = decode_measure(name, world, rank, local, eager, arrival_rate, setup=setup)
        line["poisson"] = {k: p[k] for k in ("value", "unit", "wall_s", "arrivals", "latency_s", "per_rank") if k in p}
    line["weights_build_s"] = round(build_s, 2)
    return line


def run_decode(args):
    world, rank, local = dist_setup()
    torch.cuda.set_device(torch.device("cuda", local))
    line = decode_legs(args.decode, world, rank, local, args.eager, args.arrival_rate or 0.0)
    if rank == 0 and args.cpu_engine:
        line["cpu_baseline"] = reference_engine_cpu(args.decode, args.cpu_engine_requests)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


# -------------------------------------------------------------------------------------- main

def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def run_reference(args, world, rank):
    if rank != 0:
        return
    cb = cpu_baseline(args.batch, seconds=max(1.0, 0.05 * (args.steps + args.warmup)), sample=args.cpu_sample)
    # ms_per_step: the sample's time per step scaled by bytes to the full step (not a timed full step)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["seconds_per_full_step"] * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": config_of(args, world),
            "cpu_baseline": dict({k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
                                 ms_per_step="the sample's time per step scaled by bytes to the full step"),
            "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_of(args, world):
    return {"workload": f"cfg5 paged-attention sweep point: {args.batch} seqs/GPU, self ctx U[1,{MAX_CTX}] "
                        f"+ append + cross enc {ENC_LEN}",
            "batch_per_gpu": args.batch, "heads": H, "head_dim": D, "block_size": BS,
            "cross_enc_len": ENC_LEN, "parallelism": f"request-sharded x{world} (no collective)",
            "l2": "inputs larger than L2 (pools ~13 GB per GPU at batch 1024), no flush"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--cpu-sample", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="BASELINE config-5 batch sweep, one line per point")
    ap.add_argument("--split-sweep", action="store_true",
                    help="the planner's split rule against every fixed split, one line per shape")
    ap.add_argument("--sweep-batches", default="1,2,4,8,16,32,64,128,256,512,1024")
    ap.add_argument("--ring-sweep", action="store_true",
                    help="under-filled attention shapes against 2-8 ring stages, one line per shape")
    ap.add_argument("--schedule-sweep", action="store_true",
                    help="item grid against the balanced schedule (attention), one line per shape")
    ap.add_argument("--sweep-shapes", default="",
                    help="--schedule-sweep: only these ROWSxREQUESTSxCTX shapes (comma-separated)")
    ap.add_argument("--profile-step", choices=["cfg1", "cfg2", "cfg3", "cfg4"], default=None,
                    help="one decode step of the config's engine inside a profiler range (for ncu)")
    ap.add_argument("--profile-attn", default=None, metavar="R,ROWS,LEN",
                    help="three paged-attention calls of R requests x ROWS rows over LEN tokens (for ncu)")
    ap.add_argument("--profile-topk", type=int, default=0, metavar="ROWS",
                    help="three cfg-4 candidate selections of ROWS rows (for ncu), then their time")
    ap.add_argument("--profile-kv-proj", type=int, default=0, metavar="TOKENS",
                    help="three encoder K/V projection calls at TOKENS tokens (for ncu)")
    ap.add_argument("--decode", choices=["cfg1", "cfg2", "cfg3", "cfg4"], default=None,
                    help="end-to-end decode tokens/s of the engine on a BASELINE config")
    ap.add_argument("--eager", action="store_true", help="decode without CUDA graphs")
    ap.add_argument("--cpu-engine", action="store_true",
                    help="--decode: also time the reference's own decode engine on the host cores")
    ap.add_argument("--cpu-engine-requests", type=int, default=0,
                    help="requests of the reference CPU engine timing (0: all with --cpu-engine; the "
                         "default run's decode leg uses 3)")
    ap.add_argument("--arrival-rate", type=float, default=None,
                    help="decode: also serve the requests arriving as a Poisson process at this many per "
                         "second (default run: 1000 for cfg4; --decode: off)")
    ap.add_argument("--decode-config", default="cfg4", choices=["cfg1", "cfg2", "cfg3", "cfg4", "none"],
                    help="engine config measured after the kernel leg of the default run ('none' skips it)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.sweep:
        run_sweep(args)
        return
    if args.split_sweep:
        run_split_sweep(args)
        return
    if args.ring_sweep:
        run_ring_sweep(args)
        return
    if args.schedule_sweep:
        run_schedule_sweep(args)
        return
    if args.profile_step:
        run_profile_step(args)
        return
    if args.profile_kv_proj:
        run_profile_kv_proj(args)
        return
    if args.profile_attn:
        run_profile_attn(args)
        return
    if args.profile_topk:
        run_profile_topk(args)
        return
    if args.decode:
        run_decode(args)
        return

    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return

    world, rank, local = dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from vflorence_b200 import paged_ops as ops
    from vflorence_b200.sharding import max_over_ranks, sum_over_ranks

    w = make_workload(args.batch, 2 + rank, device)
    step = Step(w, device)
    nb = algorithmic_bytes(w)
    stream = torch.cuda.current_stream(device)
    d = step.dev

    def device_step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        step.append(w["k_new"], w["v_new"], d["slots"])
        if ev is not None:
            ev[1].record(stream)
        step.self_attn(w["q"], step.out, step.meta_self, d["ctx"], d["qsl"], d["table"])
        if ev is not None:
            ev[2].record(stream)
        step.cross_attn(w["qc"], step.out_c, step.meta_cross, d["cross_lens"], d["qsl"], d["cross_table"])
        if ev is not None:
            ev[3].record(stream)

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize()
    assert ops.read_device_errors(device) == 0

    # ---- device-resident leg
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for i in range(args.steps):
            device_step(evs[i])
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    elapsed_ms = start.elapsed_time(end)
    t_self = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    t_append = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    t_cross = sum(e[2].elapsed_time(e[3]) for e in evs) / args.steps
    elapsed_max = max_over_ranks(elapsed_ms)
    total_bytes = sum_over_ranks(float(nb["total"] * args.steps))
    value = total_bytes / (elapsed_max / 1e3) / 1e9

    # ---- e2e leg: public API with host buffers (pinned inputs up, outputs down, host planning),
    # pipelined as a serving loop runs it: step i's inputs go up on a copy stream into one of two
    # device buffer sets while step i-1 computes, its outputs come down on another stream into
    # one of two pinned buffers, and the host waits for step i-1's results before issuing step
    # i+1. Every step still moves all of its bytes, and the host reads every result.
    host_in = {k: w[k].cpu().pin_memory() for k in ("q", "k_new", "v_new", "qc")}
    host_meta = {k: w[k].pin_memory() for k in ("table", "cross_table", "slots", "ctx", "cross_lens", "qsl")}
    host_all = {**host_in, **host_meta}
    dev_sets = [{k: torch.empty_like(t, device=device) for k, t in host_all.items()} for _ in range(2)]
    dev_outs = [(torch.empty_like(step.out), torch.empty_like(step.out_c)) for _ in range(2)]
    host_outs = [(torch.empty_like(host_in["q"]).pin_memory(), torch.empty_like(host_in["qc"]).pin_memory())
                 for _ in range(2)]
    h2d = sum(t.nbytes for t in host_all.values())
    d2h = host_outs[0][0].nbytes + host_outs[0][1].nbytes
    e2e_steps = max(3, min(args.steps, 100))
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def e2e_run(n, start_ev=None, end_ev=None):
        if start_ev is not None:
            start_ev.record(stream)
            copy_in.wait_event(start_ev)
        for i in range(n):
            b = i % 2
            dv, (o, oc), (ho, hoc) = dev_sets[b], dev_outs[b], host_outs[b]
            with torch.cuda.stream(copy_in):
                if i >= 2:
                    copy_in.wait_event(ev_done[b])  # step i-2 has finished reading set b
                for k, t in host_all.items():
                    dv[k].copy_(t, non_blocking=True)
                ev_in[b].record(copy_in)
            meta_s = ops.get_scheduler_metadata(args.batch, H, H, D, host_meta["ctx"], DTYPE, host_meta["qsl"],
                                                False, "sm100", BS)
            meta_c = ops.get_scheduler_metadata(args.batch, H, H, D, host_meta["cross_lens"], DTYPE,
                                                host_meta["qsl"], False, "sm100", BS)
            stream.wait_event(ev_in[b])
            if i >= 2:
                stream.wait_event(ev_out[b])  # step i-2's outputs have left buffer b
            step.append(dv["k_new"], dv["v_new"], dv["slots"])
            step.self_attn(dv["q"], o, meta_s, dv["ctx"], dv["qsl"], dv["table"])
            step.cross_attn(dv["qc"], oc, meta_c, dv["cross_lens"], dv["qsl"], dv["cross_table"])
            ev_done[b].record(stream)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(ev_done[b])
                ho.copy_(o, non_blocking=True)
                hoc.copy_(oc, non_blocking=True)
                ev_out[b].record(copy_out)
            if i >= 1:
                ev_out[(i - 1) % 2].synchronize()  # the caller reads step i-1's results
        if end_ev is not None:
            end_ev.record(copy_out)
        ev_out[(n - 1) % 2].synchronize()

    e2e_run(3)
    barrier(world)
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks_e2e:
        e2e_run(e2e_steps, s2, e2)
        torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))
    e2e_bytes = sum_over_ranks(float(nb["total"] * e2e_steps))
    e2e_value = e2e_bytes / (e2e_ms / 1e3) / 1e9
    assert ops.read_device_errors(device) == 0

    peak, peak_kind = load_peaks()
    achieved = nb["self"] / (t_self / 1e3) / 1e9
    traffic_info = load_traffic()
    traffic = None
    if traffic_info and traffic_info.get("dram_bytes_per_algorithmic_byte"):
        traffic = nb["self"] * float(traffic_info["dram_bytes_per_algorithmic_byte"])

    plan_s, plan_c = step.plans
    launches = step.launches * args.steps
    decode = None
    if args.decode_config != "none":
        del w, step, d, host_in, host_meta, host_all, dev_sets, dev_outs, host_outs
        torch.cuda.empty_cache()
        try:
            rate = args.arrival_rate if args.arrival_rate is not None else (1000.0 if args.decode_config == "cfg4" else 0.0)
            decode = decode_legs(args.decode_config, world, rank, local, arrival_rate=rate)
        except Exception as exc:  # the kernel line stands even if the engine leg fails
            decode = {"config": args.decode_config, "error": f"{type(exc).__name__}: {exc}"[:300]}

    cb = None
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and isinstance(decode, dict)
            and "error" not in decode):  # the reference's own engine beside the decode figure, N=1 only
        decode["cpu_baseline"] = reference_engine_cpu(args.decode_config, args.cpu_engine_requests or 3)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:  # reported at N=1 only
        cb = cpu_baseline(args.batch, seconds=args.cpu_seconds, sample=args.cpu_sample)
        cb.pop("seconds_per_step", None)
        cb.pop("seconds_per_full_step", None)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config_of(args, world),
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms / e2e_steps, "steps": e2e_steps, "clocks": clocks_e2e.summary()},
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "kernel": f"self decode: {_kernel_of(plan_s)} (bf16, head_dim 64) + merge",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                         else "fallback 6650 GB/s", "traffic": traffic,
                         "algorithmic_bytes_per_launch": nb["self"]},
            "ops_ms": {"append": t_append, "self_decode": t_self, "cross": t_cross},
            "ops_gbs": {"append": nb["append"] / t_append / 1e6, "self_decode": nb["self"] / t_self / 1e6,
                        "cross": nb["cross"] / t_cross / 1e6},
            "plans": {"self": _plan_desc(plan_s), "cross": _plan_desc(plan_c)},
            "clocks": clocks.summary(),
            "cpu_baseline": cb,
            "decode": decode,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
