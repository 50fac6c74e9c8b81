#!/usr/bin/env python3
"""Decode throughput of woolly's quantized forward on B200.

Workload (the metric's config): LLaMA-2-7B shape
(d 4096, 32 layers, 32 heads MHA, FFN 11008, vocab 32000), Q4_0 weights drawn
N(0, 0.02) from a seed, 16 sessions each prefilled with 512 random tokens,
then teacher-forced decode at batch 16 (headline) and at batch 1.  One step =
one batched decode step (16 tokens).  The weights (3.7 GB) and KV cache are
far larger than L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0).  At N = 1 the line also carries a `tp`
sub-record: the LLaMA-2-70B shape (all 80 layers,
Q4_0) decoded on one GPU (TP-1), the base of the tensor-parallel curve.  Under
torchrun (N > 1) the line's value is that 70B decode, tensor-parallel over
the N ranks (ncclAllReduce after attn_output and ffn_down), at batch 32
(strong scaling: the same batch on more GPUs), with batch 1 beside it;
timing is the max over ranks of the CUDA-event time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(hidden=4096, layers=32, heads=32, kv_heads=32, ff=11008, vocab=32000)
PREFILL = 512
BATCH = 16
SEED = 7
METRIC = "decode tok/s, 7B-shape Q4_0 (bs1/bs16); dequant-GEMV HBM GB/s vs peak"
WORKLOAD = "llama2-7b-shape Q4_0, 16 sessions x 512-token prefill, teacher-forced decode bs16 (and bs1)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def weight_bytes_7b():
    d, L, ff, V = CFG["hidden"], CFG["layers"], CFG["ff"], CFG["vocab"]
    per_layer = (4 * d * d + 3 * d * ff) // 32 * 18
    return L * per_layer + d * V // 32 * 18


def kv_bytes(ctx_lens):
    d, L = CFG["hidden"], CFG["layers"]
    return sum(L * 2 * c * d * 2 for c in ctx_lens)


class Clocks:
    """Samples SM clocks and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.dev = dev
        self.p = None
        self.lines = []

    def start(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.p = None

    def _read(self):
        for line in self.p.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.p:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=None)
    return ws, rank, local


def max_over_ranks(x, ws):
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def model_path(tmpdir, rank, ws):
    from woolly_b200.gguf import write_synthetic
    path = os.path.join(tmpdir, "llama7b_q4_0.gguf")
    if rank == 0 and not os.path.exists(path):
        write_synthetic(path, **CFG, weight_type=2, context_length=4096, seed=SEED)
    barrier(ws)
    return path


# ---------------------------------------------------------------- CPU baseline
def oracle_model_path(tmpdir):
    """The same seeded 7B-shape GGUF, written by the oracle's own writer
    (byte-identical to the product's), so the CPU legs never load the product
    library."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    path = os.path.join(tmpdir, "llama7b_q4_0.gguf")
    if not os.path.exists(path):
        O.synth_gguf(path, **CFG, weight_type=O.Q4_0, context_length=4096, seed=SEED)
    return path


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_step_time(path, threads, steps, ctx):
    """Seconds per 16-session decode step of the CPU oracle, extrapolated to
    32 layers from runs with 1 and 2 layers loaded (the per-layer cost is the
    difference; the rest is the embedding, final norm and LM head)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    times = {}
    for nl in (1, 2):
        m = O.Model(path, threads=threads, max_layers=nl)
        kvs = [m.new_kv(ctx + steps + 2) for _ in range(BATCH)]
        for i, kv in enumerate(kvs):
            kv.fill_synthetic(ctx, seed=i)
        ids = np.arange(BATCH, dtype=np.uint32)
        m.decode_batch(kvs, ids)  # warm
        t0 = time.perf_counter()
        for _ in range(steps):
            m.decode_batch(kvs, ids)
        times[nl] = (time.perf_counter() - t0) / steps
        for kv in kvs:
            kv.close()
        m.close()
    per_layer = max(times[2] - times[1], 1e-9)
    fixed = max(times[1] - per_layer, 0.0)
    return fixed + CFG["layers"] * per_layer


def cpu_baseline(path, steps=2, ctx=640):
    """Times the CPU oracle (plain-C restatement of woolly's forward, f32
    weights as woolly's dequantization cache holds them) on a bounded sample:
    16 sessions x `steps` decode steps at context `ctx`, with 1 and 2 of 32
    layers loaded, extrapolated to 32 layers; once with OpenMP over all host
    cores (the reported value) and once on one thread (woolly's QKV loops are
    single-threaded, tensor_utils_simd.rs:1050-1081)."""
    cores = os.cpu_count() or 1
    step = cpu_step_time(path, cores, steps, ctx)
    step1 = cpu_step_time(path, 1, 1, ctx)
    return {"value": BATCH / step, "unit": "tok/s", "cores": cores, "kind": "port",
            "cpu_model": cpu_model(), "single_thread_tok_s": BATCH / step1,
            "sample": f"{BATCH} sessions x {steps} decode steps (1 on one thread) at context {ctx} "
                      f"with 1 and 2 of 32 layers loaded, f32 weights; step time extrapolated to "
                      f"32 layers ({step * 1e3:.0f} ms/step on {cores} threads, "
                      f"{step1 * 1e3:.0f} ms/step on 1)"}


def run_reference(args):
    ws, rank, local = dist_init()
    if rank != 0:
        return
    os.makedirs(args.tmpdir, exist_ok=True)
    with tempfile.TemporaryDirectory(dir=args.tmpdir) as td:
        path = oracle_model_path(td)
        steps = max(1, min(args.steps, 3))
        res = None
        t0 = time.perf_counter()
        for _ in range(max(0, min(args.warmup, 1))):
            cpu_baseline(path, steps=1)
        samples = []
        for _ in range(max(1, min(args.steps, 2))):
            res = cpu_baseline(path, steps=steps)
            samples.append(res["value"])
        wall = time.perf_counter() - t0
    v = float(np.median(samples))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": BATCH / v * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "model": "llama2-7b-shape", "global_batch": BATCH,
                       "seq_len": PREFILL, "parallelism": "cpu"},
            "cpu_baseline": dict(res, value=v),
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": wall}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def gemv_roofline(torch, dev, reps=24):
    """Average duration of the layout-B Q4_0 GEMV at B=16 over the four 7B
    projection shapes (the launches of one decode layer), on the tiled decode
    copies the model runtime uses, weights rotated across copies totalling
    > 4x L2, launches captured in a CUDA graph and timed with CUDA events on
    the capturing stream."""
    from woolly_b200 import ops
    shapes = [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]
    res = {}
    tot_bytes, tot_ms = 0, 0.0
    for K, N in shapes:
        nbytes = K * N // 32 * 18
        copies = max(2, int(600e6 // nbytes) + 1)
        ws = [torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=dev) for _ in range(copies)]
        for w in ws:  # realistic f16 scales (0x2000 ~ 0.0078) in every block
            v = w.view(-1, 18)
            v[:, 0] = 0
            v[:, 1] = 0x20
        ws = [ops.qtile(w, 2, K, N) for w in ws]
        planes = ops.split_planes(torch.randn(BATCH, K, device=dev))
        y = torch.empty(BATCH, N, device=dev)
        s = torch.cuda.Stream(dev)
        with torch.cuda.stream(s):
            for i in range(3):
                ops.qgemv_tiled(ws[i % copies], 2, planes, N, out=y)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                ops.qgemv_tiled(ws[i % copies], 2, planes, N, out=y)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            g.replay()
            e1.record(s)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        alg = nbytes + 4 * BATCH * K + 4 * BATCH * N
        res[f"{K}x{N}"] = {"us": round(ms * 1e3, 2), "GBps": round(alg / ms / 1e6, 1)}
        tot_bytes += alg
        tot_ms += ms
        del ws, g
    return tot_bytes / tot_ms / 1e6, res


SWEEP_SHAPES = [(4096, 4096), (4096, 14336), (14336, 4096)]


def _rand_blocks(torch, dev, qt, K, N, copies):
    """Random GGUF blocks with finite, realistic scales (d ~ 0.0078; Q4_1 m
    too; Q4_K d 1.6e-4, dmin -0.02; Q6_K d 4.7e-4)."""
    S, E = {2: (18, 32), 3: (20, 32), 8: (34, 32), 12: (144, 256), 14: (210, 256)}[qt]
    nbytes = K * N // E * S
    ws = []
    for _ in range(copies):
        w = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device=dev)
        v = w.view(-1, S)
        if qt == 12:
            v[:, 12], v[:, 13], v[:, 14], v[:, 15] = 0x3E, 0x09, 0x1F, 0xA5
        elif qt == 14:
            v[:, 208], v[:, 209] = 0xB3, 0x0F
        else:
            v[:, 0] = 0
            v[:, 1] = 0x20
        if qt == 3:
            v[:, 2] = 0
            v[:, 3] = 0xA0  # m ~ -0.0078
        ws.append(w)
    return ws, nbytes


def _graph_time(torch, dev, fn, reps):
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(reps):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def gemv_gemm_sweep(torch, dev, hbm_peak, tc_peak):
    """The standalone sweep: layout-B GEMV (tiled decode copies) for
    Q4_0/Q4_1/Q8_0/Q4_K/Q6_K x three shapes x B in {1, 4, 16} (weights
    rotated over copies > 4x L2, CUDA-graph timed; GB/s of algorithmic bytes
    -- the GGUF bytes of the matrix; the K-quant tiled copies are 22/18 and
    40/26.25 of that -- and fraction of the measured HBM peak), and the
    tcgen05 prefill GEMM at M = 512 (useful TFLOP/s = 2*M*K*N / time, and the
    fraction of the measured bf16 dense peak it issues with its 3 exact MMAs)."""
    from woolly_b200 import ops
    out = {"gemv_layout_b": {}, "gemm_m512": {}}
    for qt, name in ((2, "q4_0"), (3, "q4_1"), (8, "q8_0"), (12, "q4_k"), (14, "q6_k")):
        for K, N in SWEEP_SHAPES:
            ws, nbytes = _rand_blocks(torch, dev, qt, K, N, 2)
            copies = max(2, int(600e6 // nbytes) + 1)
            ws += _rand_blocks(torch, dev, qt, K, N, copies - 2)[0]
            ws = [ops.qtile(w, qt, K, N) for w in ws]
            for B in (1, 4, 16):
                planes = ops.split_planes(torch.randn(B, K, device=dev))
                y = torch.empty(B, N, device=dev)
                ms = _graph_time(torch, dev, lambda i: ops.qgemv_tiled(ws[i % copies], qt, planes, N, out=y), 24)
                alg = nbytes + 4 * B * (K + N)
                gbs = alg / ms / 1e6
                out["gemv_layout_b"][f"{name} {K}x{N} B={B}"] = {
                    "us": round(ms * 1e3, 2), "GBps": round(gbs, 1), "frac": round(gbs / hbm_peak, 3)}
            del ws
        if qt != 2:
            continue
        for K, N in SWEEP_SHAPES:
            ws, _ = _rand_blocks(torch, dev, qt, K, N, 1)
            wt = ops.qtile(ws[0], qt, K, N)  # the GEMM reads the tiled copy, as in the runtime
            planes = ops.split_planes(torch.randn(512, K, device=dev))
            y = torch.empty(512, N, device=dev)
            for _ in range(3):
                ops.qgemm_tiled(wt, qt, planes, N, out=y)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                ops.qgemm_tiled(wt, qt, planes, N, out=y)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 10
            tf = 2 * 512 * K * N / ms / 1e9
            out["gemm_m512"][f"{name} {K}x{N}"] = {
                "us": round(ms * 1e3, 1), "TFLOPs_useful": round(tf, 1),
                "issued_frac_of_bf16_peak": round(3 * tf / tc_peak, 3) if tc_peak else None}
            del ws
    return out


def run_gpu(args):
    import torch
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from woolly_b200.model import CudaTransformer, Session
    hbm_peak, peak_kind = peaks()
    os.makedirs(args.tmpdir, exist_ok=True)
    td = args.tmpdir
    path = model_path(td, rank, ws)
    max_ctx = PREFILL + args.warmup + args.steps + args.bs1_steps + 8
    m = CudaTransformer(path, device=local, max_sessions=BATCH + 1, max_context=max_ctx,
                        max_batch=BATCH, max_prefill=PREFILL)
    rng = np.random.default_rng(SEED + 1_000_000 + rank)
    sess = [Session(m) for _ in range(BATCH)]
    # prompt throughput through the public API (tensor-core GEMMs and
    # attention; the first session is the warm-up, the other 15 are timed)
    for i, s in enumerate(sess):
        if i == 1:
            torch.cuda.synchronize()
            tp0 = time.perf_counter()
        s.infer_last(rng.integers(0, CFG["vocab"], PREFILL).tolist())
    torch.cuda.synchronize()
    prefill_tps = (BATCH - 1) * PREFILL / (time.perf_counter() - tp0)
    total = args.warmup + args.steps
    forced = torch.from_numpy(rng.integers(0, CFG["vocab"], (total, BATCH)).astype(np.int32)).to(dev)
    logits = torch.empty(BATCH, CFG["vocab"], device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for t in range(args.warmup):
        m.decode_step_device(sess, forced[t].data_ptr(), logits.data_ptr(), stream)
    torch.cuda.synchronize()
    barrier(ws)
    ctx0 = [len(s) for s in sess]
    clk = Clocks(local)
    clk.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for t in range(args.warmup, total):
        m.decode_step_device(sess, forced[t].data_ptr(), logits.data_ptr(), stream)
    e1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    ms_total = max_over_ranks(e0.elapsed_time(e1), ws)
    ms_step = ms_total / args.steps
    value = ws * BATCH * args.steps / (ms_total / 1e3)
    # algorithmic bytes of the timed steps: weights once per step + KV read
    kv = sum(kv_bytes([c + i + 1 for c in ctx0]) for i in range(args.steps)) / args.steps
    step_bytes = weight_bytes_7b() + kv
    step_gbs = step_bytes / (ms_step / 1e3) / 1e9
    barrier(ws)

    # ---- end to end through the public API: host ids in, host logits out ----
    e2e_steps = max(3, min(args.steps, 32))
    for s in sess:
        s.reset()
    for s in sess:
        s.infer_last(rng.integers(0, CFG["vocab"], PREFILL).tolist())
    # each step: the step's token ids host -> device, one decode step, the
    # server's sampling on the GPU (temperature 0.8, top-k 40, top-p 0.95,
    # host-drawn uniforms), the sampled ids device -> host
    host_ids = rng.integers(0, CFG["vocab"], (e2e_steps + 1, BATCH)).astype(np.uint32)
    draws = rng.random((e2e_steps + 1, BATCH), dtype=np.float32)
    m.decode_sample(sess, host_ids[0], 0.8, 40, 0.95, draws[0])
    torch.cuda.synchronize()
    barrier(ws)
    t0 = time.perf_counter()
    for t in range(1, e2e_steps + 1):
        nxt = m.decode_sample(sess, host_ids[t], 0.8, 40, 0.95, draws[t])
    e2e_s = max_over_ranks(time.perf_counter() - t0, ws)
    e2e_value = ws * BATCH * e2e_steps / e2e_s
    assert ((nxt >= 0) & (nxt < CFG["vocab"])).all()

    # ---- batch 1 ----
    s1 = Session(m)
    s1.infer_last(rng.integers(0, CFG["vocab"], PREFILL).tolist())
    ids1 = torch.from_numpy(rng.integers(0, CFG["vocab"], args.bs1_steps + 3).astype(np.int32)).to(dev)
    for t in range(3):
        m.decode_step_device([s1], ids1[t].data_ptr(), logits.data_ptr(), stream)
    torch.cuda.synchronize()
    e0.record()
    for t in range(3, args.bs1_steps + 3):
        m.decode_step_device([s1], ids1[t].data_ptr(), logits.data_ptr(), stream)
    e1.record()
    torch.cuda.synchronize()
    ms1 = max_over_ranks(e0.elapsed_time(e1), ws) / args.bs1_steps
    bs1 = {"value": ws * 1e3 / ms1, "unit": "tok/s", "ms_per_step": ms1,
           "hbm_frac_of_" + peak_kind: (weight_bytes_7b() + kv_bytes([PREFILL + 3])) / (ms1 / 1e3) / 1e9 / hbm_peak}
    launches = m.decode_kernel_count(BATCH) * args.steps
    s1.close()
    for s in sess:
        s.close()
    m.close()

    # ---- dominant kernel: the layout-B Q4_0 GEMV ----
    achieved, per_shape = gemv_roofline(torch, dev)
    sweep = None
    if not args.no_sweep and rank == 0:
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                tc_peak = float(json.load(f)["bf16_tflops"])
        except Exception:
            tc_peak = 1590.0
        sweep = gemv_gemm_sweep(torch, dev, hbm_peak, tc_peak)
    traffic = None  # dram bytes per launch, scaled from the committed ncu capture
    try:
        with open(os.path.join(ROOT, "profiles", "qgemv_b_q4_0_7b_decode.json")) as f:
            ratio = json.load(f)["traffic_ratio"]
        mean_alg = sum(K * N // 32 * 18 + 4 * BATCH * (K + N) for K, N in
                       [(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]) / 4
        traffic = ratio * mean_alg
    except Exception:
        pass

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 weights, f16 MMA operands, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, uniform random token ids)",
            "config": {"workload": WORKLOAD, "model": "llama2-7b-shape", "global_batch": BATCH * ws,
                       "seq_len": PREFILL, "parallelism": f"replicas x{ws}",
                       "l2": "inputs larger than L2 (3.7 GB weights + KV per step)"},
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": BATCH * (4 + 16),
                    "d2h_bytes_per_step": BATCH * 4,
                    "what": "CudaTransformer.decode_sample: host ids in, GPU-sampled ids out"},
            "bs1": bs1,
            "prefill": {"value": round(prefill_tps, 1), "unit": "tok/s",
                        "what": f"Session.infer_last of {PREFILL}-token prompts, 15 sessions, wall clock"},
            "step_roofline": {"bound": "hbm", "achieved": step_gbs, "peak": hbm_peak,
                              "unit": "GB/s", "frac": step_gbs / hbm_peak,
                              "bytes_per_step": step_bytes, "peak_kind": peak_kind},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": traffic,
                         "kernel": "k_qgemv_b<Q4_0, B=16, tiled copy>", "peak_kind": peak_kind,
                         "shapes": per_shape},
            "clocks": clocks,
            "gpu_launches": launches,
        }
        if sweep is not None:
            line["sweep"] = sweep
        if not args.no_cpu_baseline and ws == 1:
            line["cpu_baseline"] = cpu_baseline(path)
    if ws == 1 and not args.no_long:
        torch.cuda.empty_cache()
        line["long_context"] = long_context(args, local)
    if ws == 1 and not args.no_tp:
        torch.cuda.empty_cache()
        line["tp"] = tp_decode(args, 1, 0, local)
    if rank == 0:
        print(json.dumps(line), flush=True)
    barrier(ws)
    if ws > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


CFG_70B = dict(hidden=8192, heads=64, kv_heads=8, ff=28672, vocab=32000)
TP_METRIC = "decode tok/s, 70B-shape Q4_0 tensor-parallel (bs1/bs32)"


def weight_bytes_70b(layers):
    d, ff, V = CFG_70B["hidden"], CFG_70B["ff"], CFG_70B["vocab"]
    kv = d // 8
    per_layer = (2 * d * d + 2 * d * kv + 3 * d * ff) // 32 * 18
    return layers * per_layer + d * V // 32 * 18


def path_70b(tmpdir, layers, rank, ws):
    """Seeded 70B-shape Q4_0 GGUF (written once per box by rank 0, reused)."""
    from woolly_b200.gguf import write_synthetic
    path = os.path.join(tmpdir, f"llama70b_{layers}l_q4_0.gguf")
    if rank == 0 and not os.path.exists(path):
        tmp = path + ".part"
        write_synthetic(tmp, **CFG_70B, layers=layers, weight_type=2, context_length=4096, seed=SEED)
        os.replace(tmp, path)
    barrier(ws)
    return path


def tp_decode(args, ws, rank, local, steps=None, warmup=3):
    """LLaMA-2-70B shape (d 8192, 80 layers, 64 heads, 8
    KV heads, FFN 28672), Q4_0, tensor-parallel over the launch's ranks
    (column shards for q/k/v and gate/up, row shards for attn_output and
    ffn_down, ncclAllReduce after each row-parallel projection).  32 sessions
    each prefilled with `tp_prompt` random tokens, then teacher-forced decode
    at batch 32 and at batch 1, device time max over ranks.  Returns the
    per-batch results (rank 0) or None."""
    import torch
    import torch.distributed as dist
    from woolly_b200.model import CudaTransformer, Session, nccl_communicator, nccl_destroy
    dev = torch.device("cuda", local)
    hbm_peak, peak_kind = peaks()
    L, P, B = args.tp_layers, args.tp_prompt, 32
    os.makedirs(args.tmpdir, exist_ok=True)
    path = path_70b(args.tmpdir, L, rank, ws)
    comm = nccl_communicator(rank, ws) if ws > 1 else None
    steps = steps or args.tp_steps
    W = max(1, warmup)
    m = CudaTransformer(path, device=local, tp_rank=rank, tp_size=ws, nccl_comm=comm,
                        max_sessions=B, max_context=P + 2 * (steps + W) + 8, max_batch=B, max_prefill=P)
    rng = np.random.default_rng(SEED + 7)
    sess = [Session(m) for _ in range(B)]
    t0 = time.perf_counter()
    for s in sess:
        s.infer_last(rng.integers(0, CFG_70B["vocab"], P).tolist())
    prefill_s = time.perf_counter() - t0
    logits = torch.empty(B, CFG_70B["vocab"], device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    out = {}
    wb = weight_bytes_70b(L)
    launches = m.decode_kernel_count(B) * steps  # this library's kernels in the bs32 timed loop
    for nb in (B, 1):
        ids = torch.from_numpy(rng.integers(0, CFG_70B["vocab"], (steps + W, nb)).astype(np.int32)).to(dev)
        for t in range(W):
            m.decode_step_device(sess[:nb], ids[t].data_ptr(), logits.data_ptr(), stream)
        torch.cuda.synchronize()
        barrier(ws)
        ctx = [len(s) for s in sess[:nb]]
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for t in range(W, steps + W):
            m.decode_step_device(sess[:nb], ids[t].data_ptr(), logits.data_ptr(), stream)
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1), ws) / steps
        kvb = sum(L * 2 * (c + steps / 2) * (CFG_70B["hidden"] // 8) * 2 for c in ctx)
        per_gpu = (wb + kvb) / ws  # each GPU reads its shard of the weights and KV
        gbs = per_gpu / (ms / 1e3) / 1e9
        out[f"bs{nb}"] = {"tok_s": nb * 1e3 / ms, "ms_per_step": ms,
                          "per_gpu_GBps": gbs, "per_gpu_hbm_frac_of_" + peak_kind: gbs / hbm_peak}
    # end to end at batch 32 through the public API (host ids in, host logits out)
    e2e_steps = 8
    host_ids = rng.integers(0, CFG_70B["vocab"], (e2e_steps + 1, B)).astype(np.uint32)
    m.forward_sessions(sess, [[int(i)] for i in host_ids[0]])
    barrier(ws)
    t0 = time.perf_counter()
    for t in range(1, e2e_steps + 1):
        m.forward_sessions(sess, [[int(i)] for i in host_ids[t]])
    e2e = B * e2e_steps / max_over_ranks(time.perf_counter() - t0, ws)
    for s in sess:
        s.close()
    m.close()
    # share of a step spent in the collectives, estimated by timing the same
    # all-reduces (2 per layer, [B, d] f32) on the launch's NCCL group
    ar = None
    if ws > 1:
        x = torch.ones(B, CFG_70B["hidden"], device=dev)
        for _ in range(5):
            dist.all_reduce(x)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(2 * L):
            dist.all_reduce(x)
        e1.record()
        torch.cuda.synchronize()
        ar_ms = max_over_ranks(e0.elapsed_time(e1), ws)
        ar = {"allreduce_ms_per_step_bs32": ar_ms,
              "share_of_bs32_step": ar_ms / out[f"bs{B}"]["ms_per_step"],
              "how": "2 x layers ncclAllReduce of [32, 8192] f32 on the launch's group, CUDA events"}
    if comm is not None:
        nccl_destroy(comm)
    if rank != 0:
        return None
    return {"tp": ws, "layers": L, "prompt": P, "prefill_s": prefill_s, "timed_steps": steps,
            "gpu_launches_bs32": launches,
            "results": out, "e2e_bs32_tok_s": e2e, "collectives": ar,
            "workload": f"llama2-70b-shape Q4_0, {L} layers, TP{ws}, 32 sessions x {P}-token prefill, "
                        f"teacher-forced decode bs32 and bs1"}


CFG_MISTRAL = dict(hidden=4096, heads=32, kv_heads=8, ff=14336, vocab=32000)


def long_context(args, local):
    """Mistral-7B shape (d 4096, 32 heads, 8 KV heads, FFN
    14336, sliding window 4096), Q4_1, 8 sessions each prefilled to an
    8192-token f16 KV cache, then teacher-forced batch-8 decode (the split-K
    attention reads the last 4096 keys of every session)."""
    import torch
    from woolly_b200.gguf import write_synthetic
    from woolly_b200.model import CudaTransformer, Session
    dev = torch.device("cuda", local)
    hbm_peak, peak_kind = peaks()
    L, P, B, W, steps = args.long_layers, 8192, 8, 4096, args.long_steps
    path = os.path.join(args.tmpdir, f"mistral_{L}l_q4_1.gguf")
    if not os.path.exists(path):
        write_synthetic(path + ".part", **CFG_MISTRAL, layers=L, weight_type=3, sliding_window=W,
                        context_length=16384, seed=SEED)
        os.replace(path + ".part", path)
    m = CudaTransformer(path, device=local, max_sessions=B, max_context=P + steps + 8, max_batch=B,
                        max_prefill=2048)
    rng = np.random.default_rng(SEED + 3)
    sess = [Session(m) for _ in range(B)]
    t0 = time.perf_counter()
    for s in sess:
        s.infer_last(rng.integers(0, CFG_MISTRAL["vocab"], P).tolist())
    prefill_s = time.perf_counter() - t0
    ids = torch.from_numpy(rng.integers(0, CFG_MISTRAL["vocab"], (steps + 3, B)).astype(np.int32)).to(dev)
    logits = torch.empty(B, CFG_MISTRAL["vocab"], device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for t in range(3):
        m.decode_step_device(sess, ids[t].data_ptr(), logits.data_ptr(), stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for t in range(3, steps + 3):
        m.decode_step_device(sess, ids[t].data_ptr(), logits.data_ptr(), stream)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    for s in sess:
        s.close()
    m.close()
    d, ff, kv = CFG_MISTRAL["hidden"], CFG_MISTRAL["ff"], 1024
    wbytes = L * (2 * d * d + 2 * d * kv + 3 * d * ff) // 32 * 20 + d * CFG_MISTRAL["vocab"] // 32 * 20
    kvbytes = B * L * 2 * W * kv * 2  # the window's keys and values, f16
    gbs = (wbytes + kvbytes) / (ms / 1e3) / 1e9
    return {"workload": f"mistral-7b-shape Q4_1, {L} layers, window {W}, {B} sessions x {P}-token "
                        f"prefill, teacher-forced decode bs{B}",
            "tok_s": B * 1e3 / ms, "ms_per_step": ms, "prefill_s": prefill_s, "timed_steps": steps,
            "step_bytes": wbytes + kvbytes, "kv_bytes_per_step": kvbytes,
            "step_hbm_frac_of_" + peak_kind: gbs / hbm_peak}


def run_tp_headline(args):
    """N > 1: the 70B tensor-parallel decode is the line's value (batch 32)."""
    import torch
    ws, rank, local = dist_init()
    torch.cuda.set_device(local)
    clk = Clocks(local)
    clk.start()
    # the line times exactly the driver's K steps after its W warm-up steps
    r = tp_decode(args, ws, rank, local, steps=args.steps, warmup=args.warmup)
    clocks = clk.stop()
    if rank == 0:
        b32 = r["results"]["bs32"]
        print(json.dumps({
            "metric": TP_METRIC, "value": b32["tok_s"], "unit": "tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": b32["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4_0 weights, f16 MMA operands, f32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights, uniform random token ids)",
            "config": {"workload": r["workload"], "model": "llama2-70b-shape", "global_batch": 32,
                       "seq_len": args.tp_prompt, "parallelism": f"tp{ws}",
                       "l2": "inputs larger than L2 (weights + KV per step)"},
            "e2e": {"value": r["e2e_bs32_tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 32 * 12,
                    "d2h_bytes_per_step": 32 * CFG_70B["vocab"] * 4},
            "gpu_launches": r["gpu_launches_bs32"], "tp": r, "clocks": clocks}), flush=True)
    barrier(ws)
    import torch.distributed as dist
    if ws > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=253)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--bs1-steps", type=int, default=64)
    ap.add_argument("--impl", default="woolly_b200", choices=["woolly_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the GEMV/GEMM shape sweep")
    ap.add_argument("--tp-layers", type=int, default=80)
    ap.add_argument("--tp-prompt", type=int, default=1024)
    ap.add_argument("--tp-steps", type=int, default=32)
    ap.add_argument("--no-tp", action="store_true", help="N=1: skip the 70B TP-1 sub-record")
    ap.add_argument("--long-layers", type=int, default=32)
    ap.add_argument("--long-steps", type=int, default=32)
    ap.add_argument("--no-long", action="store_true", help="N=1: skip the long-context sub-record")
    ap.add_argument("--tmpdir", default=os.environ.get("WOOLLY_BENCH_DIR", "/tmp/woolly_bench"))
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_tp_headline(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
