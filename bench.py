#!/usr/bin/env python
"""Benchmark: Pplx-shaped Q4 encoder forward at 1024 tokens per GPU.

One step = one 28-layer forward of one 1024-token sequence on every GPU (weak scaling; ranks
process independent sequences, no collective on the data path).  `value` is device-timed with
inputs resident in HBM; `e2e` goes through the public API (Model.predict) with host token ids in
and the host embedding out.  Runs under torchrun for N > 1 (one process per GPU).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Pplx Q4 tokens/s @1024 tok (1/2/4/8 B200) + GEMM % roofline vs host-CPU ref"
CFG = dict(layers=28, hidden=1024, q_heads=16, kv_heads=8, head_dim=128, ffn=3072, vocab=151936, weight_bits=4)
TOKENS = 1024
SEED = 1234
L2_BYTES = 126 * 2 ** 20


def gemm_flops_per_token_layer(c):
    nq, nk = c["q_heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    d, f = c["hidden"], c["ffn"]
    return {"gemm_qkv": 2 * d * (nq + 2 * nk), "gemm_o": 2 * nq * d, "gemm_mlp_swiglu": 2 * d * 2 * f,
            "gemm_down": 2 * f * d}


def q4_weight_bytes(c):
    nq, nk = c["q_heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
    d, f = c["hidden"], c["ffn"]
    params = c["layers"] * (d * (nq + 2 * nk) + nq * d + 2 * d * f + f * d)
    return params * (0.5 + 4 / 64)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def ncu_traffic(summary: str = "gemm_i8_c2_encoder.md"):
    """DRAM bytes per GEMM launch from the committed ncu summary (profiles/), or None."""
    p = os.path.join(ROOT, "profiles", summary)
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        sm, mx, reasons = [], None, set()
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for i, n in enumerate(names):
                    if r[5 + i].lower().startswith("active"):
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        load = [s for s in sm if s > 0.5 * max(sm)]
        return {"sm_mhz": float(np.median(load)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline (oracle, test infrastructure)
_CPU_ENCODERS = {}


def _cpu_encoder(layers: int, vocab: int):
    """Oracle encoder with `layers` layers cycling through two distinct random layers (timing does
    not depend on the weight values; generating 28 distinct layers would dominate the run)."""
    from oracle import oracle
    key = (layers, vocab)
    if key not in _CPU_ENCODERS:
        c = dict(CFG, layers=layers, vocab=vocab)
        rng = np.random.default_rng(SEED)
        d, f = c["hidden"], c["ffn"]
        nq, nk = c["q_heads"] * 128, c["kv_heads"] * 128

        def bf(shape):
            return oracle.f32_to_bf16(rng.normal(0, 0.02, shape).astype(np.float32))

        w = {"embedding": bf((vocab, d))}
        for n, shape in (("q", (nq, d)), ("k", (nk, d)), ("v", (nk, d)), ("o", (d, nq)), ("gate", (f, d)),
                         ("up", (f, d)), ("down", (d, f))):
            two = [bf(shape) for _ in range(2)]
            w[n] = [two[i % 2] for i in range(layers)]
        for n, size in (("input_norm", d), ("post_norm", d), ("q_norm", 128), ("k_norm", 128)):
            w[n] = [np.ones(size, np.float32) for _ in range(layers)]
        w["final_norm"] = np.ones(d, np.float32)
        _CPU_ENCODERS[key] = oracle.Encoder(c, w)
    return _CPU_ENCODERS[key]


def cpu_sample(threads: int = 0, layers: int = 2, vocab: int = 4096, full_budget_s: float = 0.0):
    """Times the CPU restatement of the reference path (AVX2 rows<R,Q4> GEMMs, f32 attention) at
    1024 tokens on `layers` of the 28 layers, scaled to 28; when full_budget_s > 0 and the scaled
    estimate fits in it, times the full 28-layer forward instead.  Returns (tokens/s, info)."""
    from oracle import oracle
    if threads > 0:
        oracle.set_threads(threads)
    rng = np.random.default_rng(SEED + 1)
    ids = rng.integers(0, vocab, TOKENS).astype(np.int32)
    enc = _cpu_encoder(layers, vocab)
    enc.forward(ids[:64], mode=2)  # thread-pool warm-up
    t0 = time.perf_counter()
    enc.forward(ids, mode=2)
    dt = time.perf_counter() - t0
    est_full = dt / layers * CFG["layers"]
    if full_budget_s > 0 and est_full <= full_budget_s:
        enc = _cpu_encoder(CFG["layers"], vocab)
        t0 = time.perf_counter()
        enc.forward(ids, mode=2)
        dt = time.perf_counter() - t0
        return TOKENS / dt, {"cores": oracle.num_threads(), "seconds": dt,
                             "sample": "one full 28-layer 1024-token Q4 forward (oracle AVX2 path, f32 attention); "
                                       f"vocab {vocab} embedding table"}
    return TOKENS / est_full, {"cores": oracle.num_threads(), "seconds": dt,
                               "sample": f"{layers} of 28 layers of the 1024-token Q4 forward (oracle AVX2 path, "
                                         f"f32 attention), time scaled to 28 layers; vocab {vocab} embedding table"}


def host_cores() -> int:
    """Host threads this process may run on (torchrun's OMP_NUM_THREADS=1 does not apply to the
    CPU baseline, which is timed with every core the process can use)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args, rank):
    """The reference arm: the CPU restatement of the reference's native path (oracle, AVX2
    rows<R,Q4> GEMMs, int8.rs:448-480 / :526-585), one full 28-layer 1024-token forward per timed
    step, on every host core.  Warm-up steps are short forwards (thread pool and page warm-up)."""
    if rank != 0:
        return
    from oracle import oracle
    oracle.set_threads(host_cores())
    vocab = 4096
    enc = _cpu_encoder(CFG["layers"], vocab)
    rng = np.random.default_rng(SEED + 1)
    ids = rng.integers(0, vocab, TOKENS).astype(np.int32)
    for _ in range(max(args.warmup, 1)):
        enc.forward(ids[:64], mode=2)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        enc.forward(ids, mode=2)
        times.append(time.perf_counter() - t0)
    sec = float(np.median(times))
    value = TOKENS / sec
    sample = (f"one full 28-layer {TOKENS}-token Q4 forward per step (oracle AVX2 path, f32 attention), "
              f"median of {args.steps}; vocab {vocab} embedding table")
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "w4a8 int (f32 fma)",
            "data": "synthetic", "config": config_json(),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": oracle.num_threads(), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_json():
    return {"workload": "pplx-q4-encoder-1024tok (BASELINE config 2)", **CFG, "tokens_per_step_per_gpu": TOKENS,
            "group": 64, "weight_quant": "Q4 absmax g64 f32 scales", "activation_quant": "int8 g64 f32 scales",
            "l2": f"inputs larger than L2: {q4_weight_bytes(CFG) / 1e6:.0f} MB of Q4 weights streamed per step "
                  f"(L2 {L2_BYTES >> 20} MiB)"}


# ------------------------------------------------------------------ named shapes (driver-run evidence)
def _device_time_us(fn, reps, flush=None, sleep=200_000):
    """Median device time of fn() over reps launches (CUDA events on the current stream), each
    launch queued behind a short GPU sleep (no host latency timed) and, when given, an L2 flush."""
    import torch
    times = []
    for _ in range(reps):
        if flush is not None:
            flush.zero_()
        torch.cuda._sleep(sleep)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return float(np.median(times))


def shape_c1(db, reps=20, layout=None):
    """one W4A8 g64 GEMM, M=1024 K=1024 N=3072 (activations f16 N(0,1) seed 0,
    weights f32 N(0,0.02) seed 1 -> bf16 -> Q4), the exact int8 tensor-core path (or the given
    activation layout, e.g. the dequantised one, unpack pass included), L2 flushed per launch."""
    import torch
    from oracle import oracle
    m, k, n = 1024, 1024, 3072
    w = oracle.f32_to_bf16(np.random.default_rng(1).normal(0, 0.02, (n, k)).astype(np.float32))
    x = torch.from_numpy(np.random.default_rng(0).normal(0, 1, (m, k)).astype(np.float16)).cuda()
    codes, scales = db.pack_weights(torch.from_numpy(w.view(np.int16)).cuda(), 4)
    layout = db.CODES_NATURAL if layout is None else layout
    a, sa, _ = db.quantize_activations(x, bits=8, layout=layout)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    fn = lambda: db.gemm(a, layout, sa, codes, scales, m, n, k, 4, residual=y)
    for _ in range(3):
        fn()
    us = _device_time_us(fn, reps, flush)
    peak_tf, _, kind = measured_peaks()
    tf = 2.0 * m * n * k / us / 1e6
    return {"us": us, "tflops": tf, "frac_of_bf16_peak": tf / peak_tf, "peak_kind": kind,
            "timing": f"device, median of {reps}, L2 flushed"}


def shape_gemv(db, rows=(1, 4, 8), copies=16, reps=5):
    """Small-M decode GEMV on the C5 layers (hidden 2560, 32q/8kv x 128, FF 9728, Q4 g64), as a decode
    step runs it: `copies` distinct weight matrices of one shape (together larger than L2, so every
    launch streams its weights from HBM) launched back to back; time per launch = device time of
    the chain / copies (median of `reps` chains).  The roofline is the weight (+ scale) bytes per
    launch over the measured HBM copy bandwidth."""
    import torch
    hid, ff = 2560, 9728
    shapes = [("qkv", hid, 32 * 128 + 2 * 8 * 128), ("o", 32 * 128, hid), ("gate_up", hid, 2 * ff), ("down", ff, hid)]
    _, peak_gbs, kind = measured_peaks()
    out = {}
    for t, (name, k, n) in enumerate(shapes):
        mats = [db.pack_weights(db.synthetic_bf16(SEED, 100 + 16 * t + c, (n, k), 0.02), 4) for c in range(copies)]
        wbytes = mats[0][0].numel() + (k // 64) * n * 4
        for m in rows:
            x = torch.randn(m, k, device="cuda")
            a, sa, sums = db.quantize_activations(x, bits=8, layout=db.CODES_GEMV, sums=True)
            y = torch.empty((m, n), dtype=torch.float32, device="cuda")

            def chain():
                for codes, scales in mats:
                    db.gemm(a, db.CODES_GEMV, sa, codes, scales, m, n, k, 4, a_sums=sums, residual=y)
            chain()
            # the GPU sleep ahead of the chain (~2 ms) outlasts the host's enqueueing of the launches,
            # so the events time the kernels back to back, not the host's launch rate
            us = _device_time_us(chain, reps, sleep=4_000_000) / copies
            out[f"{name}_M{m}"] = {"us": us, "GB/s": wbytes / us / 1e3, "frac_of_hbm": wbytes / us / 1e3 / peak_gbs}
        del mats
    for m in rows:
        fr = [v["frac_of_hbm"] for kk, v in out.items() if kk.endswith(f"_M{m}")]
        out[f"mean_frac_M{m}"] = float(np.mean(fr))
    out["peak_kind"] = kind
    out["timing"] = (f"device time of {copies} back-to-back launches on distinct weights (> L2) / {copies}, "
                     f"median of {reps} chains")
    return out


def shape_c3(db, rank, world, local_rank, reps=3, dq=False):
    """the C2-shaped encoder with int8 (Q8 g64) weights on a ragged batch of 64
    sequences, lengths U(16, 1024) (seed 3), through the public predict_batch (packed passes).  At
    N > 1 the sequences are sharded by longest-processing-time (sharding.assign_lpt) and each rank
    runs its share; the time is the max over ranks and the outputs are gathered on rank 0."""
    import torch
    import torch.distributed as dist

    from decisive_b200 import sharding
    cfg = dict(CFG, weight_bits=8)
    model = db.Model.synthetic(db.EncoderConfig(**cfg, max_sequence_tokens=1024), seed=SEED, std=0.02,
                               device=local_rank)
    if dq:
        model.set_code_layout(db.CODES_DQ)
    rng = np.random.default_rng(3)
    lens = rng.integers(16, 1025, 64)
    reqs = [rng.integers(0, CFG["vocab"], int(L)).astype(np.int32) for L in lens]
    mine = sharding.assign_lpt([int(L) for L in lens], world)[rank]
    local = [reqs[i] for i in mine]
    model.predict_batch(local)  # warm-up (workspace sized)
    torch.cuda.synchronize()
    best = 1e30
    for _ in range(reps):
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        out = model.predict_batch(local)
        dt = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([dt], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        best = min(best, dt)
    ok = all(o.status == "success" for o in out)
    if world > 1:
        gathered = sharding.gather_ordered({i: np.asarray(o.result.response)[:4].tolist() for i, o in zip(mine, out)}, 64)
        ok = ok and (rank != 0 or len(gathered) == 64)
    loads = sharding.rank_loads(sharding.assign_lpt([int(L) for L in lens], world), [int(L) for L in lens])
    model.close()
    tokens = int(lens.sum())
    return {"tokens_per_s": tokens / best, "ms_per_batch": best * 1e3, "sequences": 64, "tokens": tokens,
            "numerics": "dequantised" if dq else "exact",
            "all_success": bool(ok), "lpt_max_over_mean_load": max(loads) / (sum(loads) / len(loads)),
            "timing": "host wall clock around predict_batch (host ids in, pooled embeddings out), best of "
                      f"{reps}, max over ranks"}


def c4_requests(vocab, n, seed=4):
    """BASELINE config 4 requests: a 384-token state and 8 choices of U(16..48) tokens each."""
    rng = np.random.default_rng(seed)
    return [(rng.integers(0, vocab, 384).astype(np.int32),
             [rng.integers(0, vocab, int(rng.integers(16, 49))).astype(np.int32) for _ in range(8)])
            for _ in range(n)]


def shape_c4(db, local_rank, requests=4):
    """BASELINE config 4 (shape): the Decima-shaped cross-encoder (12L, D=768, 12 heads, FF 3072,
    W8A8 blocks of 32), each request one 384-token state with 8 choices of 16..48 tokens scored as
    8 packed state+choice sequences -> 3-way logits, through the public score call."""
    cfg = db.BertConfig(layers=12, hidden=768, heads=12, ffn=3072, vocab=128100, max_positions=512, block=32)
    model = db.BertModel(cfg, seed=SEED, std=0.02, device=local_rank)
    reqs = c4_requests(cfg.vocab, requests)
    model.score(*reqs[0])
    t0 = time.perf_counter()
    for state, choices in reqs:
        model.score(state, choices)
    dt = time.perf_counter() - t0
    model.close()
    tokens = sum(8 * len(st) + sum(len(c) for c in ch) for st, ch in reqs)
    return {"tokens_per_s": tokens / dt, "requests_per_s": requests / dt, "ms_per_request": dt / requests * 1e3,
            "timing": "host wall clock around the public score call per request (state and choice ids in, "
                      "8 x 3 logits out)"}


def shape_c5(db, local_rank, requests=3, dq=False):
    """BASELINE config 5 (shape): the Qwen3-4B-shaped decoder (36L, D=2560, 32q/8kv, FF 9728, Q4),
    requests of a 512-token prefix and 4 continuations of 32 tokens scored by log-probability
    (LM head over the 151,936-token vocabulary), through the public score_continuations; cold
    (new prefix) and prefix-cached."""
    cfg = db.EncoderConfig(layers=36, hidden=2560, q_heads=32, kv_heads=8, head_dim=128, ffn=9728, vocab=151936,
                           weight_bits=4, max_sequence_tokens=1024, causal=True)
    model = db.Model.synthetic(cfg, seed=SEED, std=0.02, device=local_rank)
    if dq:
        model.set_code_layout(db.CODES_DQ)
    rng = np.random.default_rng(5)
    prefixes = rng.integers(0, cfg.vocab, (requests + 1, 512)).astype(np.int32)
    conts = rng.integers(0, cfg.vocab, (requests + 1, 4, 32)).astype(np.int32)
    cache = model.create_cache(db.CacheOptions(max_bytes=256 << 20, require_prefix=True))
    model.score_continuations(prefixes[requests], conts[requests], cache=cache)  # warm-up
    t0 = time.perf_counter()
    for i in range(requests):
        model.score_continuations(prefixes[i], conts[i], cache=cache)
    cold = (time.perf_counter() - t0) / requests
    t0 = time.perf_counter()
    for i in range(requests):
        model.score_continuations(prefixes[0], conts[i], cache=cache)
    hit = (time.perf_counter() - t0) / requests
    model.close()
    return {"ms_per_request": cold * 1e3, "ms_per_request_prefix_cached": hit * 1e3,
            "tokens_per_s": (512 + 128) / cold, "numerics": "dequantised" if dq else "exact",
            "timing": "host wall clock around the public call (ids in, 4 x 32 log-probs out)"}


def named_shapes(db, rank, world, local_rank, dq=False):
    """Every named BASELINE shape, short: each entry is independent (a failure is recorded, not
    raised).  C3 runs on every rank (sharded); the others on rank 0."""
    import torch
    import torch.distributed as dist
    out = {}

    def run(name, fn):
        try:
            out[name] = fn()
        except Exception as e:  # recorded in the line
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}

    run("c3_ragged_int8_batch", lambda: shape_c3(db, rank, world, local_rank, dq=dq))
    if rank == 0:
        run("c1_gemm", lambda: shape_c1(db))
        if dq:
            run("c1_gemm_dequantised", lambda: shape_c1(db, layout=db.CODES_DQ))
        run("gemv_c5_layers", lambda: shape_gemv(db))
        run("c4_decima_encoder", lambda: shape_c4(db, local_rank))
        run("c5_decoder_prefix", lambda: shape_c5(db, local_rank, dq=dq))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    return out


# ------------------------------------------------------------------ GPU arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import decisive_b200 as db

    torch.cuda.set_device(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local_rank))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg = db.EncoderConfig(**CFG, max_sequence_tokens=TOKENS)
    model = db.Model.synthetic(cfg, seed=SEED, std=0.02, device=local_rank)
    dq = args.numerics == "dq"
    if dq:
        # dequantised projections: f16(code * scale) operands, f32 accumulation over the whole K
        model.set_code_layout(db.CODES_DQ)
    # kernel selection (bitwise-equal tile configurations, fastest by >= 1 %), before any timing;
    # the dequantised GEMM has one configuration per shape
    tuning = None if (args.no_tune or dq) else {k: v["choice"] for k, v in model.tune(TOKENS).items()}
    if args.stream:
        model.set_streaming(True)  # weights in pinned host memory, two layers on the device
    rng = np.random.default_rng(SEED + rank)
    ids_host = torch.from_numpy(rng.integers(0, CFG["vocab"], TOKENS).astype(np.int32)).pin_memory()
    ids_dev = ids_host.cuda()
    out_dev = torch.empty(CFG["hidden"], dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream()

    for _ in range(args.warmup):
        model.forward_device(ids_dev, out_dev)
    torch.cuda.synchronize()

    gpu_index = local_rank
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        parts = vis.split(",")
        if local_rank < len(parts) and parts[local_rank].strip().isdigit():
            gpu_index = int(parts[local_rank])

    # ---- device-timed region: K forwards with inputs resident in HBM
    with ClockSampler(gpu_index) as clocks:
        barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            model.forward_device(ids_dev, out_dev)
        end.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = start.elapsed_time(end)
    # ---- per-kernel breakdown: the same K forwards again with a CUDA event pair around every
    # launch on the model's stream (kept out of the timed region above)
    model.profile(True)
    model.profile_read(reset=True)
    for _ in range(args.steps):
        model.forward_device(ids_dev, out_dev)
    torch.cuda.synchronize()
    prof = model.profile_read(reset=True)
    model.profile(False)
    ms_max = max_over_ranks(ms)
    assert np.all(np.isfinite(out_dev.cpu().numpy())), "non-finite embedding"
    assert db.device_error_word() == 0, "device wait expired"
    value = world * TOKENS * args.steps / (ms_max / 1e3)

    # ---- end to end through the public API: host ids in (pinned), host embedding out
    out_host = torch.empty(CFG["hidden"], dtype=torch.float32).pin_memory()
    ids_np, out_np = ids_host.numpy(), out_host.numpy()
    for _ in range(2):
        model.predict(ids_np, out=out_np)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        model.predict(ids_np, out=out_np)
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    barrier()
    e2e = world * TOKENS * args.steps / e2e_s

    # ---- roofline of the dominant kernel (the grouped GEMM, all four projection shapes)
    fl = gemm_flops_per_token_layer(CFG)
    gemm_ms = sum(prof[k][0] for k in fl)
    gemm_launches = sum(prof[k][1] for k in fl)
    gemm_flops = sum(fl.values()) * TOKENS * CFG["layers"] * args.steps
    achieved = gemm_flops / (gemm_ms / 1e3) / 1e12
    peak_tf, _, peak_kind = measured_peaks()
    traffic = ncu_traffic("gemm_dq_c2.md" if dq else "gemm_i8_c2_encoder.md")
    # profiled regions; in dequantised mode each projection's region holds two kernels (unpack, GEMM)
    launches = sum(v[1] for v in prof.values()) + (gemm_launches if dq else 0)

    extras = None if args.no_extras else named_shapes(db, rank, world, local_rank, dq=dq)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": ("w4a8 dequantised to f16 operands, f32 accumulation over K (kind::f16)" if dq
                          else "w4a8 int (kind::i8 exact int dots, f32 fma group fold)"),
                "numerics": ("dequantised: f16(code*scale) operands, full-K f32 sums; within the contract's "
                             "2e-3 x RMS per GEMM, C2 pooled cosine >= 0.9999 (tests)" if dq
                             else "exact: the reference's grouped fold bit for bit"),
                "data": "synthetic (seeded N(0,0.02) bf16 weights, uniform token ids)", "config": config_json(),
                "clocks": clocks.summary(),
                "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": TOKENS * 4,
                        "d2h_bytes_per_step": CFG["hidden"] * 4},
                "gpu_launches": launches,
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                             "frac": achieved / peak_tf, "traffic": traffic,
                             "kernel": ("unpack_weights_kernel + gemm_dq_kernel (all projection launches)" if dq
                                        else "gemm_i8_kernel (all projection launches)"),
                             "peak_kind": f"{peak_kind} bf16 dense burst",
                             "launches": gemm_launches, "avg_launch_us": gemm_ms / gemm_launches * 1e3,
                             "flops_per_launch": gemm_flops / gemm_launches},
                "kernel_ms_per_step": {k: v[0] / args.steps for k, v in prof.items()},
                "weights": "streamed: pinned host memory -> two device banks" if args.stream else "resident in HBM",
                "tile_configs": tuning}
        if extras is not None:
            line["named_shapes"] = extras
        if world == 1 and not args.no_cpu:
            cpu_v, info = cpu_sample(host_cores(), layers=args.cpu_layers, full_budget_s=30.0)
            line["cpu_baseline"] = {"value": cpu_v, "unit": "tokens/s", "cores": info["cores"], "kind": "port",
                                    "sample": info["sample"]}
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()


def run_gemm(args, local_rank):
    """Single grouped GEMM (BASELINE config 1 by default: M=1024, K=1024, N=3072, W4A8 g64): K
    device-timed launches on prepared activations, L2 flushed between launches."""
    import torch

    import decisive_b200 as db
    from oracle import oracle
    torch.cuda.set_device(local_rank)
    m, k, n = (int(v) for v in args.gemm_shape.split(","))
    rng = np.random.default_rng(1)
    w = oracle.f32_to_bf16(rng.normal(0, 0.02, (n, k)).astype(np.float32))
    x = np.random.default_rng(0).normal(0, 1, (m, k)).astype(np.float16)
    codes, scales = db.pack_weights(torch.from_numpy(w.view(np.int16)).cuda(), args.bits)
    xt = torch.from_numpy(x).cuda()
    layout = {"tc": db.CODES_TC, "dq": db.CODES_DQ}.get(args.layout, db.CODES_NATURAL)
    a, sa, _ = db.quantize_activations(xt, bits=8, layout=layout)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    cfg = db.GemmConfig(*(int(v) for v in args.gemm_config.split(","))) if args.gemm_config else None
    for _ in range(args.warmup):
        db.gemm(a, layout, sa, codes, scales, m, n, k, args.bits, residual=y, config=cfg)
    torch.cuda.synchronize()
    times = []
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda._sleep(200_000)  # the launch is queued before the start event fires
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        db.gemm(a, layout, sa, codes, scales, m, n, k, args.bits, residual=y, config=cfg)
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    us = float(np.mean(times)) * 1e3
    flops = 2.0 * m * n * k
    peak_tf, peak_gbs, kind = measured_peaks()
    out = {"workload": f"gemm W{args.bits}A8 g64 M={m} K={k} N={n}", "layout": args.layout,
           "config": args.gemm_config or "default", "us_per_launch": us,
           "tflops": flops / us / 1e6, "frac_of_bf16_peak": flops / us / 1e6 / peak_tf, "peak_kind": kind,
           "launches": args.steps, "l2": "flushed between launches"}
    print(json.dumps(out), flush=True)


def run_gemv(args, local_rank):
    """Small-M grouped GEMV (decode / scoring steps) on the C5-shaped layers, chained launches on
    distinct weights (see shape_gemv)."""
    import torch

    import decisive_b200 as db
    torch.cuda.set_device(local_rank)
    rows = tuple(int(v) for v in args.gemv_rows.split(","))
    print(json.dumps({"workload": f"gemv Q4 g64 C5-shaped layers", **shape_gemv(db, rows=rows)}), flush=True)


def run_decima(args, local_rank):
    """Decima int8 (C4 scheme: W8A8, blocks of 32, round-half-away division, bias) projections of a
    C4-shaped layer (D=768, FF=3072) on one request's tokens (8 sequences x 416 = 3328 rows):
    quantise + grouped GEMM + bias through db_decima_linear, device-timed, L2 flushed before every
    launch.  Reports microseconds and TFLOP/s per projection and the layer's linear time."""
    import torch

    import decisive_b200 as db
    torch.cuda.set_device(local_rank)
    m, d, ff, block = 3328, 768, 3072, 32
    shapes = [("qkv", d, 3 * d), ("o", d, d), ("ffn_in", d, ff), ("ffn_out", ff, d)]
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device="cuda")
    peak_tf, _, kind = measured_peaks()
    cases, total_us = [], 0.0
    for name, k, n in shapes:
        rng = np.random.default_rng(k * 3 + n)
        w = torch.from_numpy(rng.normal(0, 0.02, (n, k)).astype(np.float32)).cuda()
        codes, scales = db.decima_quantize_weights(w, block)
        x = torch.from_numpy(rng.normal(0, 1, (m, k)).astype(np.float32)).cuda()
        bias = torch.from_numpy(rng.normal(0, 0.1, n).astype(np.float32)).cuda()
        for _ in range(args.warmup):
            db.decima_linear(x, codes, scales, n, block, True, bias)
        torch.cuda.synchronize()
        times = []
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda._sleep(200_000)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            db.decima_linear(x, codes, scales, n, block, True, bias)
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        us = float(np.median(times)) * 1e3
        total_us += us
        tf = 2.0 * m * n * k / us / 1e6
        cases.append({"projection": name, "M": m, "K": k, "N": n, "us": us, "tflops": tf, "frac_of_bf16_peak": tf / peak_tf})
    print(json.dumps({"workload": f"decima W8A8 block {block} C4-shaped layer projections (quantise + GEMM + bias)",
                      "tokens": m, "layer_linear_us": total_us, "linear_tokens_per_s_per_layer": m / total_us * 1e6,
                      "peak_kind": kind, "l2": "flushed before every launch", "launches_per_case": args.steps,
                      "cases": cases}), flush=True)


def run_c5(args, local_rank):
    """C5 (Qwen3-4B-shaped decoder: 36 layers, D=2560, 32q/8kv x 128, FF 9728, Q4 g64, synthetic
    weights): requests of a 512-token prefix and 4 continuations of 32 tokens.  Each request runs
    the causal prefix pass once (keys/values kept per layer) and the 4 continuations batched after
    it, scored by log-probability through the public db_score_continuations call (host ids in,
    host per-token log-probs out).
    Requests have distinct prefixes, so nothing is reused across them; a second timing repeats one
    prefix to show the cached path."""
    import torch

    import decisive_b200 as db
    torch.cuda.set_device(local_rank)
    cfg = db.EncoderConfig(layers=36, hidden=2560, q_heads=32, kv_heads=8, head_dim=128, ffn=9728, vocab=151936,
                           weight_bits=4, max_sequence_tokens=1024, causal=True)
    model = db.Model.synthetic(cfg, seed=SEED, std=0.02, device=local_rank)
    if args.numerics == "dq":
        model.set_code_layout(db.CODES_DQ)
    rng = np.random.default_rng(5)
    n_req = max(args.steps, 1)
    prefixes = rng.integers(0, cfg.vocab, (n_req + args.warmup, 512)).astype(np.int32)
    conts = rng.integers(0, cfg.vocab, (n_req + args.warmup, 4, 32)).astype(np.int32)
    cache = model.create_cache(db.CacheOptions(max_bytes=256 << 20, require_prefix=True))
    for i in range(args.warmup):
        model.score_continuations(prefixes[n_req + i], conts[n_req + i], cache=cache)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(n_req):
        model.score_continuations(prefixes[i], conts[i], cache=cache)
    dt = time.perf_counter() - t0
    t1 = time.perf_counter()
    for i in range(n_req):
        model.score_continuations(prefixes[0], conts[i], cache=cache)  # same prefix: reused
    dt_hit = time.perf_counter() - t1
    tokens = 512 + 4 * 32
    print(json.dumps({"workload": "C5 decoder Q4 (36L, D=2560, 32q/8kv, FF 9728): 512-token prefix + 4 x 32 continuations scored by log-probability",
                      "requests": n_req, "requests_per_s": n_req / dt, "tokens_per_s": n_req * tokens / dt,
                      "ms_per_request": dt / n_req * 1e3, "ms_per_request_prefix_cached": dt_hit / n_req * 1e3,
                      "cache": cache.stats(), "timing": "host wall clock around the public call (ids in, log-probs out)",
                      "data": "synthetic (seeded N(0,0.02) bf16 weights, uniform token ids)"}), flush=True)
    model.close()


def run_c4(args, local_rank):
    """C4 (Decima-shaped cross-encoder: 12 layers, D=768, 12 heads, FF 3072, vocab 128100, W8A8 in
    blocks of 32, synthetic weights): requests of a 384-token state and 8 choices of U(16..48)
    tokens, one db_bert_score call each (8 packed sequences, 3-way logits out), host wall clock."""
    import torch

    import decisive_b200 as db
    torch.cuda.set_device(local_rank)
    cfg = db.BertConfig(layers=12, hidden=768, heads=12, ffn=3072, vocab=128100, max_positions=512, block=32,
                        mode=args.c4_mode)
    model = db.BertModel(cfg, seed=SEED, std=0.02, device=local_rank)
    n = max(args.steps, 1)
    reqs = c4_requests(cfg.vocab, n)
    for state, choices in reqs[:max(args.warmup, 1)]:
        model.score(state, choices)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for state, choices in reqs:
        model.score(state, choices)
    dt = time.perf_counter() - t0
    tokens = sum(8 * len(st) + sum(len(c) for c in ch) for st, ch in reqs)
    print(json.dumps({"workload": "C4 Decima-shaped cross-encoder (12L, D=768, FF 3072), "
                                  f"{'W8A32' if args.c4_mode else 'W8A8'} block 32, "
                                  "requests of a 384-token state + 8 choices of U(16..48) tokens -> 8 x 3 logits",
                      "requests": n, "tokens_per_s": tokens / dt, "requests_per_s": n / dt,
                      "ms_per_request": dt / n * 1e3,
                      "timing": "host wall clock around the public score call (ids in, logits out)",
                      "data": "synthetic (seeded N(0,0.02) bf16 weights, uniform token ids)"}), flush=True)
    model.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-layers", type=int, default=2)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the named BASELINE shapes in the line")
    ap.add_argument("--no-tune", action="store_true", help="skip kernel selection (default tile configurations)")
    ap.add_argument("--numerics", default="dq", choices=["dq", "exact"],
                    help="C2 projections: dequantised f16 operands with full-K f32 sums (default) or the "
                         "reference's exact grouped fold (kind::i8)")
    ap.add_argument("--stream", action="store_true",
                    help="stream layer weights from pinned host memory through two device banks")
    ap.add_argument("--workload", default="encoder", choices=["encoder", "gemm", "gemv", "decima", "c5", "c4"])
    ap.add_argument("--gemv-rows", default="1,4,8", help="activation rows (M) for --workload gemv")
    ap.add_argument("--gemm-shape", default="1024,1024,3072", help="M,K,N for --workload gemm")
    ap.add_argument("--bits", type=int, default=4)
    ap.add_argument("--layout", default="i8", choices=["i8", "tc", "dq"],
                    help="activation codes of --workload gemm: int8 (kind::i8 kernel), f16 codes (kind::f16 "
                         "kernel) or dequantised f16 (kind::f16 full-K kernel)")
    ap.add_argument("--gemm-config", default="", help="block_n,max_ctas,pair_ctas for --workload gemm")
    ap.add_argument("--c4-mode", type=int, default=0, choices=[0, 1], help="--workload c4: 0 W8A8, 1 W8A32")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.workload == "gemm":
        run_gemm(args, local_rank)
    elif args.workload == "gemv":
        run_gemv(args, local_rank)
    elif args.workload == "decima":
        run_decima(args, local_rank)
    elif args.workload == "c5":
        run_c5(args, local_rank)
    elif args.workload == "c4":
        run_c4(args, local_rank)
    elif args.impl == "reference":
        run_reference(args, rank)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
