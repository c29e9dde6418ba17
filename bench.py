"""Benchmark of the LEAP attention hot path on B200.

Headline (BASELINE.json metric "decode-attn KV GB/s (% HBM peak)", config 2):
Llama-3-8B-shaped decode attention (32 q heads, 8 kv heads, head_dim 128,
RoPE theta 500000), one query token at context 8192, FP32 KV cache.  One
step = one decode token through the attention of all 32 layers of an
8B-shaped model: 32 launches of the fused RoPE + append + split-KV decode
kernel, each over its own layer's 67 MB K+V cache (2.15 GB in total, so no
layer's cache is still in the 126 MB L2 when it is read again).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

N > 1 runs under torchrun, one process per GPU; every rank decodes its own
independent sequence (replicas, weak scaling, no collective on the data
path).  Times are CUDA-event device times, max over ranks.

value      : algorithmic KV-path bytes / s over all ranks (GB/s), with the
             inputs resident in HBM
e2e        : the same through the host-pointer C ABI entry point
             (leap_attn_decode_host, ctypes with prebound pointers): q/k/v
             in through pinned staging, kernel, output back, per layer,
             blocking
roofline   : dominant kernel (decode_attn_kernel) bytes per launch / mean
             launch time, against MEASURED_PEAKS.json hbm_gbs
cpu_baseline: the reference's own attention block (oracle/_ref, compiled
             from src/inference/FloatTransformer.cpp:404-662) on the host's
             cores over a bounded sample of the same workload
--impl reference: the reference's CPU block as the timed arm.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Config 2 shape at its largest context.
N_LAYERS = 32
N_HEADS, N_KV, HD = 32, 8, 128
CTX = 8192
THETA = 500000.0
SEED = 0


# The one JSON result line goes to the process's original stdout; everything
# else written to file descriptor 1 (NCCL's version banner, native libraries)
# is sent to stderr, so stdout carries exactly that line.
_RESULT_OUT = None


def emit(obj) -> None:
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def _keep_stdout_for_result() -> None:
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def algorithmic_bytes(n_heads, n_kv, hd, ctx):
    """Bytes one decode launch must move: K and V rows read (ctx rows), q in,
    new k/v in, new k/v appended, out written."""
    return 4 * (2 * n_kv * hd * ctx + n_heads * hd + 2 * n_kv * hd + 2 * n_kv * hd
                + n_heads * hd)


def read_traffic(ctx):
    """DRAM bytes (read + write) per decode launch from the committed ncu
    launch-list summary, or None when none was captured for this context."""
    p = os.path.join(ROOT, "profiles", "decode_attn_kernel_l8b_ctx8192.traffic.txt")
    if not os.path.exists(p):
        return None
    kv = {}
    with open(p) as f:
        for line in f:
            if "=" in line and not line.lstrip().startswith("#"):
                k, v = line.split("=", 1)
                kv[k.strip()] = v.strip()
    if int(kv.get("ctx", -1)) != ctx:
        return None
    return int(kv["bytes_per_launch"])


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU arms (test infrastructure: the reference's own code, or the C port)
# ---------------------------------------------------------------------------

def cpu_reference_step_time(min_seconds: float, threads: int | None = None):
    """Time the reference attention block at the config-2 shape on the host.

    Uses oracle/_ref (the reference's own block, compiled from its sources)
    when present, else the C restatement.  The block is called 32 times per
    step (one per layer) at ctx 8192, cycling over 4 distinct layer caches
    (each 67 MB, larger than the host's last-level cache).  Returns
    (seconds per step, kind, threads, steps timed)."""
    import oracle
    threads = threads or os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    kind = "reference" if oracle.has_ref() else "port"
    rng = np.random.default_rng(SEED)
    kv_dim = N_KV * HD
    caches = [(rng.standard_normal((CTX, kv_dim), dtype=np.float32),
               rng.standard_normal((CTX, kv_dim), dtype=np.float32)) for _ in range(4)]
    c, s = oracle.rope_table(CTX, HD, THETA)
    q = rng.standard_normal(N_HEADS * HD, dtype=np.float32)

    def step():
        for layer in range(N_LAYERS):
            kc, vc = caches[layer % 4]
            oracle.attn_block(q.copy(), kc, vc, CTX - 1, N_HEADS, N_KV, HD, c, s,
                              impl="ref" if kind == "reference" else "port", threads=threads)

    step()  # warm-up
    n = 0
    t0 = time.perf_counter()
    while True:
        step()
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return el / n, kind, threads, n


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # other ranks exit without work
    import oracle
    threads = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    kind = "reference" if oracle.has_ref() else "port"
    rng = np.random.default_rng(SEED)
    kv_dim = N_KV * HD
    caches = [(rng.standard_normal((CTX, kv_dim), dtype=np.float32),
               rng.standard_normal((CTX, kv_dim), dtype=np.float32)) for _ in range(4)]
    c, s = oracle.rope_table(CTX, HD, THETA)
    q = rng.standard_normal(N_HEADS * HD, dtype=np.float32)
    impl = "ref" if kind == "reference" else "port"

    def step():
        for layer in range(N_LAYERS):
            kc, vc = caches[layer % 4]
            oracle.attn_block(q.copy(), kc, vc, CTX - 1, N_HEADS, N_KV, HD, c, s, impl=impl,
                              threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    nbytes = algorithmic_bytes(N_HEADS, N_KV, HD, CTX) * N_LAYERS * args.steps
    value = nbytes / el / 1e9
    line = {
        "impl": "reference",
        "metric": "decode-attn KV GB/s", "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": kind,
                         "sample": f"{N_LAYERS} block calls per step at ctx {CTX} cycling over 4 "
                                   "distinct 67 MB layer caches (each larger than the host LLC)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    emit(line)


def workload_config(n, n_layers=N_LAYERS, ctx=CTX):
    mb = algorithmic_bytes(N_HEADS, N_KV, HD, ctx) / 1e6
    return {"workload": "config2: Llama-3-8B-shape GQA decode attention (32q/8kv/hd128, theta "
                        f"500000), 1 token at ctx {ctx}, one step = {n_layers} layers",
            "model": "llama3-8b-shape attention", "global_batch": n, "seq_len": ctx,
            "parallelism": f"replicas{n}" if n > 1 else "single",
            "l2": f"inputs > L2: {n_layers} distinct layer caches of {mb:.0f} MB "
                  f"({n_layers * mb / 1e3:.2f} GB) rotated"}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def run_gpu_arm(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from leap_b200 import AttentionContext

    n_layers, ctx_len = args.layers, args.ctx
    ctx = AttentionContext(n_layers, N_HEADS, N_KV, HD, ctx_len, device=local, theta=THETA)
    ctx.set_decode_impl(args.decode_impl)
    ctx.set_overlap(not args.no_overlap)
    cluster_cap = ctx.cluster_capacity()
    stream = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + rank)
    # resident synthetic caches, N(0,1), written through the ABI (rows
    # 0..ctx-2; row ctx-1 is the token being decoded)
    for layer in range(n_layers):
        kr = torch.randn(ctx_len - 1, N_KV, HD, device=dev, generator=g)
        vr = torch.randn(ctx_len - 1, N_KV, HD, device=dev, generator=g)
        ctx.kv_write(0, layer, 0, kr, vr)
        del kr, vr
    q = torch.randn(n_layers, N_HEADS, HD, device=dev, generator=g)
    kn = torch.randn(n_layers, N_KV, HD, device=dev, generator=g)
    vn = torch.randn(n_layers, N_KV, HD, device=dev, generator=g)
    out = torch.empty_like(q)
    ctx.sync()
    torch.cuda.synchronize(dev)
    pos = ctx_len - 1

    def step():
        for layer in range(n_layers):
            ctx.decode(layer, pos, q[layer], kn[layer], vn[layer], out[layer])

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # One step (n_layers launches) captured as a CUDA graph, so the timed
    # region measures the GPU rather than Python's launch rate.
    graph = None
    if not args.eager:
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            ctx.bind_torch_stream(side)
            step()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ctx.bind_torch_stream()  # the capture stream
            step()
        ctx.bind_torch_stream(stream)
        graph.replay()
        torch.cuda.synchronize(dev)

    # ---- timed region (device time, CUDA events on the launch stream) ------
    sampler = ClockSampler(local)
    sampler.start()
    barrier()
    torch.cuda.synchronize(dev)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step()
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ctx.sync()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_end))
    mean_launch_ms = elapsed_ms / (args.steps * n_layers)

    per_launch = algorithmic_bytes(N_HEADS, N_KV, HD, ctx_len)
    total_bytes = per_launch * n_layers * args.steps * world
    value = total_bytes / (elapsed_ms / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    achieved = per_launch / (mean_launch_ms / 1e3) / 1e9
    del graph

    # ---- end to end through the host-pointer entry point -------------------
    e2e = None
    if not args.no_e2e:
        # The C-ABI call an engine makes per layer (leap_attn_decode_host on
        # host buffers it owns), bound once through ctypes: q/k/v in through
        # pinned staging, kernel, output back, blocking.
        from leap_b200._native import lib as _lib
        hq = np.ascontiguousarray(q.cpu().numpy())
        hk = np.ascontiguousarray(kn.cpu().numpy())
        hv = np.ascontiguousarray(vn.cpu().numpy())
        hout = np.empty((N_HEADS, HD), np.float32)
        fn, handle = _lib().leap_attn_decode_host, ctx.handle
        ptrs = [(hq[l].ctypes.data, hk[l].ctypes.data, hv[l].ctypes.data)
                for l in range(n_layers)]
        op = hout.ctypes.data

        def host_step():
            for layer in range(n_layers):
                if fn(handle, layer, pos, *ptrs[layer], op) != 0:
                    raise RuntimeError("leap_attn_decode_host failed")

        ctx.sync()
        for _ in range(min(args.warmup, 2)):
            host_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            host_step()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        barrier()
        e2e = {"value": round(per_launch * n_layers * args.steps * world / e2e_s / 1e9, 2),
               "unit": "GB/s",
               "h2d_bytes_per_step": int(n_layers * (hq[0].nbytes + hk[0].nbytes
                                                     + hv[0].nbytes)),
               "d2h_bytes_per_step": int(n_layers * hq[0].nbytes),
               "ms_per_step": round(e2e_s / args.steps * 1e3, 4),
               "path": "leap_attn_decode_host per layer (host buffers, blocking)"}

    line = None
    if rank == 0:
        traffic = read_traffic(ctx_len)
        line = {
            "metric": "decode-attn KV GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(world, n_layers, ctx_len),
            "frac_of_hbm_peak": round(value / world / peak, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "kernel": ("decode_cluster_kernel<128,4,16>"
                                    if (args.decode_impl == 2 or (args.decode_impl == 0
                                        and cluster_cap >= N_KV))
                                    else "decode_attn_kernel<128,4>"),
                         "bytes_per_launch": per_launch,
                         "mean_launch_us": round(mean_launch_ms * 1e3, 3)},
            "e2e": e2e,
            "gpu_launches": n_layers * args.steps,
            "clocks": clocks,
        }
    ctx.close()
    del q, kn, vn, out
    torch.cuda.empty_cache()
    if not args.no_pipeline:
        # The split that shards: the Llama-3-8B-shape W8A8 model as N
        # layer-range stages, one per rank (BASELINE metric "tok/s
        # Llama-3-8B-shape W8A8 at 1/2/4/8 GPU"); outside the timed region of
        # the headline value.
        pl = measure_pipeline("llama3-8b-w8a8", world, rank, local, dev, steps=128)
        if rank == 0:
            pl["note"] = ("layer-range pipeline over the ranks (batch 1: stages run one after "
                          "another); timed separately from the headline value")
            line["pipeline"] = pl
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, kind, threads, n = cpu_reference_step_time(args.cpu_seconds)
        cpu_val = algorithmic_bytes(N_HEADS, N_KV, HD, CTX) * N_LAYERS / sec / 1e9
        line["cpu_baseline"] = {
            "value": round(cpu_val, 3), "unit": "GB/s", "cores": threads, "kind": kind,
            "sample": f"{n} steps of {N_LAYERS} reference-block calls at ctx {CTX} "
                      "(4 distinct 67 MB layer caches cycled)",
            "ms_per_step": round(sec * 1e3, 2)}
    if rank == 0:
        emit(line)


def run_prefill(args):
    """causal prefill, Llama-3-8B heads, batch 1, prompt
    length L.  One step = the prefill of L tokens of one layer (RoPE + append
    + causal attention), cycling 8 layers so K/V (8 x 8 x L x 1 KB) are not
    all L2-resident.  Metric: logical TFLOP/s, FLOP = 2*n_h*hd*L*(L+1)."""
    import torch
    from leap_b200 import AttentionContext
    dev = torch.device("cuda", 0)
    L, n_layers = args.prefill, 8
    ctx = AttentionContext(n_layers, N_HEADS, N_KV, HD, L, theta=THETA)
    ctx.set_prefill_impl(args.prefill_impl)
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    q = torch.randn(L, N_HEADS, HD, device=dev, generator=g)
    k = torch.randn(L, N_KV, HD, device=dev, generator=g)
    v = torch.randn(L, N_KV, HD, device=dev, generator=g)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    for i in range(max(args.warmup, 3)):
        ctx.prefill(0, i % n_layers, 0, q, k, v, out)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        ctx.prefill(0, i % n_layers, 0, q, k, v, out)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ctx.sync()
    ms = e0.elapsed_time(e1) / args.steps
    flop = 2.0 * N_HEADS * HD * L * (L + 1)
    tflops = flop / (ms / 1e3) / 1e12
    peak = 1622.9
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peak = float(json.load(f)["bf16_tflops"])
    line = {"metric": "causal prefill TFLOP/s (logical FP32)", "value": round(tflops, 2),
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True,
            "dtype": {1: "f32", 3: "f32 (TF32 + BF16 corrections)"}.get(args.prefill_impl,
                                                                        "f32 (3xTF32)"),
            "config": {"workload": f"config4: causal prefill L={L}, Llama-3-8B heads, batch 1",
                       "seq_len": L, "impl": {0: "tcgen05 3xTF32 pipelined", 1: "CUDA-core FP32",
                                2: "tcgen05 3xTF32 serial",
                                3: "tcgen05 TF32 + BF16 corrections pipelined"}[args.prefill_impl]},
            "roofline": {"bound": "tensor", "achieved": round(tflops, 2),
                         "tensor_tflops_issued": round(3 * tflops, 2)
                         if args.prefill_impl in (0, 2) else None,
                         "peak": peak, "peak_kind": "measured bf16 dense (TF32 is half)",
                         "unit": "TFLOP/s", "frac": round(tflops / peak, 4)}}
    ctx.close()
    emit(line)


# ---------------------------------------------------------------------------
# End-to-end models (BASELINE configs 1 and 5, and the metric's 8B W8A8 shape)
# ---------------------------------------------------------------------------

# name: (dim, hidden, layers, heads, kv heads, vocab, seq_len), W8A8?, theta,
#       prompt tokens, generated tokens
MODELS = {
    "tinyllama-fp32": ((2048, 5632, 22, 32, 4, 32000, 2048), False, 10000.0, 32, 256),
    "llama3-8b-w8a8": ((4096, 14336, 32, 32, 8, 128256, 8448), True, 500000.0, 8192, 256),
    "llama3-70b-w8a8": ((8192, 28672, 80, 64, 8, 128256, 8448), True, 500000.0, 8192, 256),
}


def model_bytes_per_token(shape, q8, ctx):
    """Bytes one decode token must move: every weight once (int8 + one FP32
    scale per 64, or FP32), the norms, and K/V rows 0..ctx of every layer."""
    dim, hid, L, nh, nkv, vocab, _ = shape
    kv = nkv * (dim // nh)
    per_w = (1 + 4 / 64) if q8 else 4
    layer_w = (dim * dim * 2 + 2 * kv * dim + 3 * hid * dim) * per_w + 2 * dim * 4
    cls = vocab * dim * per_w + dim * 4
    kv_bytes = L * 2 * kv * ctx * 4
    return L * layer_w + cls + kv_bytes


def hop_latency(comm, rank, dim, dev, iters=200):
    """One stage hop of the pipeline, measured: a ping-pong of one
    activation row x[dim] FP32 between ranks 0 and 1 through the stage
    transport, timed with CUDA events on rank 0's stream.  Returns the
    one-way time in microseconds on rank 0 (None elsewhere); ranks other
    than 0 and 1 take no part."""
    import torch
    if rank > 1:
        return None
    x = torch.zeros(dim, device=dev)
    stream = torch.cuda.current_stream(dev)

    def rounds(n):
        for _ in range(n):
            if rank == 0:
                comm.send(x, 1)
                comm.recv(x, 1)
            else:
                comm.recv(x, 0)
                comm.send(x, 0)

    rounds(20)
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    rounds(iters)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) * 1e3 / iters / 2 if rank == 0 else None


def measure_pipeline(model, world, rank, local, dev, prompt_len=None, steps=None, warm=3,
                     comm_kind="native", q8_gemv=None, want_e2e=False):
    """Prefill a random prompt, then greedy-decode, through `world` layer-range
    pipeline stages (1 = the single-GPU engine), on an already initialised
    process group.  Synthetic N(0, 0.02) weights (W8A8: quantized per group
    of 64) generated on the device; RMSNorm weights 1.0.  Decode tok/s is
    timed from the first generated token, as the reference's generate() does
    (main.cpp:100-107); times are CUDA events, max over ranks.

    Returns a dict on rank 0 (None elsewhere): decode tok/s, prefill seconds,
    each stage's layer compute per token, and the measured hop time."""
    import torch
    import torch.distributed as dist
    from leap_b200 import ModelConfig, Transformer
    from leap_b200.pipeline import PipelineStage, stage_range

    shape, q8, theta, p_len, gen = MODELS[model]
    prompt_len = prompt_len or p_len
    cfg = ModelConfig(*shape)
    lb, le = stage_range(cfg.n_layers, rank, world)
    chunk = 512
    if q8_gemv is not None:
        from leap_b200._native import check as _check, lib as _lib
        _check(_lib().leap_op_set_q8_gemv(q8_gemv))
    eng = Transformer.synthetic(cfg, q8, seed=SEED, device=local, rope_theta=theta,
                                layer_range=(lb, le), max_chunk=chunk)
    eng.bind_torch_stream()
    comm = None
    if world > 1:
        from leap_b200.pipeline import NativeComm, TorchComm
        comm = NativeComm(rank, world, local) if comm_kind == "native" else TorchComm()
    stage = PipelineStage(eng, cfg.dim, dev, max_chunk=chunk, rank=rank, world=world, comm=comm)
    prompt = [int(t) for t in np.random.default_rng(SEED).integers(0, cfg.vocab_size,
                                                                     prompt_len)]
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if world == 1:
            return [x]
        t = torch.zeros(world, device=dev, dtype=torch.float64)
        t[rank] = x
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return [float(v) for v in t.tolist()]

    def timed(fn):
        barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        r = fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        eng.sync()
        return r, max_over_ranks(e0.elapsed_time(e1) / 1e3)

    # warm-up: a short prompt and a few tokens, then a clean cache
    stage.prefill(prompt[:64], 0)
    stage.decode(64, warm)
    torch.cuda.synchronize(dev)
    eng.clear_kv_cache()

    _, prefill_s = timed(lambda: stage.prefill(prompt, 0))
    steps = steps or gen - 1 - warm
    stage.decode(prompt_len, warm)  # untimed decode steps, positions continue
    toks, decode_s = timed(lambda: stage.decode(prompt_len + warm, steps))
    ctx_mid = prompt_len + warm + steps // 2

    # each stage's own layer compute per decode token (no hand-off): the
    # same rows again, with this stage's layers alone
    x1 = torch.randn((1, cfg.dim), device=dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n_c = min(steps, 64)
    e0.record(stream)
    for i in range(n_c):
        eng.layers(prompt_len + warm + i, x1)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    stage_compute_us = sum_over_ranks(e0.elapsed_time(e1) * 1e3 / n_c)
    hop_us = hop_latency(comm, rank, cfg.dim, dev) if world > 1 else None

    e2e = None
    if world == 1 and want_e2e:
        # the reference-facing call: forward(token, pos) with the logits read
        # back to the host every step (Transformer.h:56)
        nxt = int(toks[-1].item())
        n_e2e = min(steps, 64)
        pos = prompt_len + warm + steps - n_e2e
        t0 = time.perf_counter()
        for i in range(n_e2e):
            eng.forward(nxt, pos + i)
            nxt = eng.last_token
        e2e_s = time.perf_counter() - t0
        e2e = {"value": round(n_e2e / e2e_s, 2), "unit": "tok/s",
               "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4 * cfg.vocab_size + 4,
               "path": "Transformer.forward(token, pos) -> host logits, per token"}
    eng.close()
    if comm is not None:
        torch.cuda.synchronize(dev)
        comm.close()
    barrier()
    if rank != 0:
        return None
    step_us = decode_s / steps * 1e6
    # per token: embedding; per layer 6 kernels (qkv with the RMSNorm (and the
    # quantize) in its prologue, attention, wo (W8A8: quantize prologue), w13
    # with its RMSNorm, silu(+quantize), w2); W8A8 with dim > 4096 forms the
    # norm/quantize in separate kernels (3 more); head: classifier (W8A8: with
    # the final norm in its prologue; FP32: after an RMSNorm launch), argmax
    fused_q8 = q8 and cfg.dim <= 4096
    per_layer = 6 + (3 if q8 and not fused_q8 else 0)
    head = (2 if fused_q8 else 3) if q8 else 3
    n_launch = 1 + per_layer * cfg.n_layers + head
    return {"model": model, "stages": [list(stage_range(cfg.n_layers, r, world))
                                       for r in range(world)],
            "decode_tok_s": round(steps / decode_s, 2), "decode_steps": steps,
            "decode_us_per_token": round(step_us, 2),
            "prefill_tokens": prompt_len, "prefill_s": round(prefill_s, 3),
            "prefill_tok_s": round(prompt_len / prefill_s, 1),
            "stage_compute_us_per_token": [round(v, 2) for v in stage_compute_us],
            "hand_off_us_per_token": round(step_us - sum(stage_compute_us), 2),
            "hops_per_token": world if world > 1 else 0,
            "hop_us_measured": None if hop_us is None else round(hop_us, 2),
            "bytes_per_token": int(model_bytes_per_token(shape, q8, ctx_mid)),
            "ctx_mid": ctx_mid, "q8": q8, "e2e": e2e, "gpu_launches": n_launch * steps,
            "stage_transport": ("leap_pp (NCCL p2p over NVLink)" if comm_kind == "native"
                                else "torch.distributed p2p") if world > 1 else None}


def run_model(args):
    """The --model line: measure_pipeline over N ranks (N = 1: the
    single-GPU engine)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        os.environ.setdefault("TORCH_NCCL_SHOW_EAGER_INIT_P2P_SERIALIZATION_WARNING", "false")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    shape, q8, theta, prompt_len, gen = MODELS[args.model]
    prompt_len = args.prompt or prompt_len
    sampler = ClockSampler(local)
    sampler.start()
    pl = measure_pipeline(args.model, world, rank, local, dev, prompt_len=prompt_len,
                          steps=args.steps if args.steps_given else None, warm=args.warmup,
                          comm_kind=args.comm, q8_gemv=args.q8_gemv,
                          want_e2e=not args.no_e2e)
    clocks = sampler.stop()
    line = None
    if rank == 0:
        tok_s = pl["decode_tok_s"]
        per_tok = pl["bytes_per_token"]
        peak, peak_kind = load_peaks()
        line = {
            "metric": f"decode tok/s ({args.model})", "value": tok_s, "unit": "tok/s",
            "n_gpus": world, "steps": pl["decode_steps"], "warmup": args.warmup,
            "ms_per_step": round(pl["decode_us_per_token"] / 1e3, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 x int8 -> f32" if q8
            else "f32", "data": "synthetic (seeded N(0,0.02) weights on device, random ids)",
            "config": {"workload": f"{args.model}: batch 1, {prompt_len}-token prompt prefilled, "
                                   f"then greedy decode", "model": args.model,
                       "global_batch": 1, "seq_len": prompt_len + args.warmup + pl["decode_steps"],
                       "parallelism": f"pp{world}" if world > 1 else "single",
                       "stage_transport": pl["stage_transport"], "stages": pl["stages"],
                       "l2": f"inputs > L2: {per_tok / 1e9:.2f} GB of weights and KV per token"},
            "prefill": {"tokens": prompt_len, "seconds": pl["prefill_s"],
                        "tok_s": pl["prefill_tok_s"]},
            "pipeline": {k: pl[k] for k in ("stage_compute_us_per_token", "hand_off_us_per_token",
                                            "hops_per_token", "hop_us_measured")},
            "roofline": {"bound": "hbm", "achieved": round(per_tok * tok_s / 1e9, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(per_tok * tok_s / 1e9 / peak, 4),
                         "bytes_per_token": int(per_tok), "traffic": None,
                         "note": "whole decode step (all kernels) against one GPU's HBM; "
                                 "stages run one after another for batch 1"},
            "e2e": pl["e2e"],
            "gpu_launches": pl["gpu_launches"],
            "clocks": clocks,
        }
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = model_cpu_baseline(args.model, prompt_len + args.warmup
                                                  + pl["decode_steps"] // 2, args.cpu_seconds)
    if rank == 0:
        emit(line)


def run_model_reference(args):
    """The reference engine's decode tok/s for --model on the host cores
    (rank 0 only; other ranks exit without work)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    shape, q8, theta, prompt_len, gen = MODELS[args.model]
    prompt_len = args.prompt or prompt_len
    cb = model_cpu_baseline(args.model, prompt_len + gen // 2, max(args.cpu_seconds, 5.0))
    if cb is None:
        emit({"impl": "reference", "unavailable": "oracle/_ref was not built"})
        return
    line = {"impl": "reference", "metric": f"decode tok/s ({args.model})",
            "value": cb["value"], "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": cb["ms_per_token"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 x int8 -> f32" if q8
            else "f32", "data": "synthetic",
            "config": {"workload": f"{args.model}: batch 1, decode at position "
                                   f"{prompt_len + gen // 2}", "model": args.model},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    emit(line)


def model_cpu_baseline(name, ctx, seconds):
    """The reference engine (oracle/_ref, Transformer::create + forward) on
    this host: decode tok/s at position `ctx`.  Attention cost does not
    depend on the cache contents, so forward(token, pos) is called at
    pos = ctx.. directly.  Models too large for a bounded sample are timed on
    1- and 3-layer files of the same shape and extrapolated linearly in the
    layer count (labelled)."""
    import oracle
    from leap_b200.modelfile import ModelConfig, write_timing_file
    if not oracle.has_ref_engine():
        return None
    shape, q8, theta, _, _ = MODELS[name]
    threads = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(threads)
    cfg = ModelConfig(*shape)
    cfg.seq_len = max(cfg.seq_len, ctx + 64)
    full = name == "tinyllama-fp32"
    layer_counts = [cfg.n_layers] if full else [1, 3]
    times = []
    with tempfile.TemporaryDirectory() as d:
        for nl in layer_counts:
            c = ModelConfig(cfg.dim, cfg.hidden_dim, nl, cfg.n_heads, cfg.n_kv_heads,
                            cfg.vocab_size, cfg.seq_len)
            path = os.path.join(d, f"m{nl}.bin")
            write_timing_file(path, c, q8)
            ref = oracle.RefEngine(path, theta_10k=(theta == 10000.0))
            ref.forward(1, ctx)  # warm-up (page-in of the mmapped weights)
            n, t0 = 0, time.perf_counter()
            while True:
                ref.forward(1 + n, ctx + 1 + n)
                n += 1
                if time.perf_counter() - t0 >= seconds / len(layer_counts) or n >= 64:
                    break
            times.append((time.perf_counter() - t0) / n)
            ref.close()
            os.unlink(path)
    if full:
        sec = times[0]
        sample = f"{len(layer_counts)} file: full model, forward() at pos {ctx}.."
    else:
        per_layer = (times[1] - times[0]) / 2
        sec = times[0] + (cfg.n_layers - 1) * per_layer
        sample = (f"extrapolated: 1- and 3-layer files of the same shape timed at pos {ctx}.., "
                  f"{times[0] * 1e3:.1f} / {times[1] * 1e3:.1f} ms per token, "
                  f"x{cfg.n_layers} layers")
    return {"value": round(1 / sec, 3), "unit": "tok/s", "cores": threads,
            "kind": "reference", "sample": sample, "ms_per_token": round(sec * 1e3, 2)}


def run_batched(args):
    """ragged batched decode, 64 sequences with contexts
    drawn uniform in [512, 8192] from seed 1 (numpy default_rng), Llama-3-8B
    heads, fused RoPE + append.  One step = one batched launch per layer over
    2 layers (each layer's caches hold 2.28 GB, far beyond L2).  Bytes per
    launch = the sum over sequences of the config-2 formula."""
    import torch
    from leap_b200 import AttentionContext
    dev = torch.device("cuda", 0)
    n_seq, n_layers = 64, 2
    ctxs = np.random.default_rng(1).integers(512, 8193, n_seq)
    max_seq = int(ctxs.max())
    ctx = AttentionContext(n_layers, N_HEADS, N_KV, HD, max_seq, max_batch=n_seq, theta=THETA)
    ctx.set_decode_impl(args.decode_impl)
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    for layer in range(n_layers):
        for i, c in enumerate(ctxs):
            kr = torch.randn(int(c) - 1, N_KV, HD, device=dev, generator=g)
            vr = torch.randn(int(c) - 1, N_KV, HD, device=dev, generator=g)
            ctx.kv_write(i, layer, 0, kr, vr)
    q = torch.randn(n_layers, n_seq, N_HEADS, HD, device=dev, generator=g)
    kn = torch.randn(n_layers, n_seq, N_KV, HD, device=dev, generator=g)
    vn = torch.randn(n_layers, n_seq, N_KV, HD, device=dev, generator=g)
    out = torch.empty_like(q)
    slots = np.arange(n_seq, dtype=np.int32)
    pos = (ctxs - 1).astype(np.int32)
    ctx.bind_torch_stream()
    stream = torch.cuda.current_stream(dev)

    def step():
        for layer in range(n_layers):
            ctx.decode_batched(layer, slots, pos, q[layer], kn[layer], vn[layer], out[layer])

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(0)
    sampler.start()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    ctx.sync()
    ms = e0.elapsed_time(e1) / args.steps
    per_launch = sum(algorithmic_bytes(N_HEADS, N_KV, HD, int(c)) for c in ctxs)
    value = per_launch * n_layers / (ms / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    line = {"metric": "batched decode-attn KV GB/s", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config3: 64 ragged sequences, ctx ~U[512,8192] seed 1, "
                                   "Llama-3-8B heads, fused RoPE + append",
                       "global_batch": n_seq, "seq_len": int(ctxs.max()),
                       "total_ctx": int(ctxs.sum()),
                       "l2": f"inputs > L2: {per_launch / 1e9:.2f} GB per launch"},
            "roofline": {"bound": "hbm", "achieved": round(value, 2), "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": round(value / peak, 4),
                         "bytes_per_launch": int(per_launch),
                         "mean_launch_us": round(ms / n_layers * 1e3, 2)},
            "gpu_launches": n_layers * args.steps, "clocks": clocks}
    ctx.close()
    emit(line)


def run_qgemm(args):
    """The W8A8 prompt-chunk GEMMs of one Llama-3-8B-shape layer (wq;wk;wv,
    wo, w1;w3, w2) over T tokens through leap_op_qmatmul, the product the
    engine's prefill runs per 512-token chunk (QuantizedTransformer.cpp:
    359-652 per token).  One step = the four GEMMs; the weights are random
    int8 with random group scales.  Metric: int8 TOP/s (2·n·d·T per GEMM).
    The CUDA-core dp4a kernel is timed beside the tcgen05 one."""
    import ctypes
    import torch
    from leap_b200._native import check, lib
    dev = torch.device("cuda", 0)
    T = args.qgemm
    shapes = [("wqkv", 4096, 6144), ("wo", 4096, 4096), ("w13", 4096, 28672),
              ("w2", 14336, 4096)]
    g = torch.Generator(device=dev)
    g.manual_seed(SEED)
    mats = []
    for _, n, d in shapes:
        wq = torch.randint(-127, 128, (d, n), dtype=torch.int8, device=dev, generator=g)
        ws = torch.rand(d, n // 64, device=dev, generator=g) * 1e-3
        xq = torch.randint(-127, 128, (T, n), dtype=torch.int8, device=dev, generator=g)
        xs = torch.rand(T, n // 64, device=dev, generator=g) * 1e-2
        mats.append((n, d, wq, ws, xq, xs, torch.empty(T, d, device=dev)))
    stream = torch.cuda.current_stream(dev)
    s = ctypes.c_void_p(stream.cuda_stream)

    def step():
        for n, d, wq, ws, xq, xs, y in mats:
            check(lib().leap_op_qmatmul(s, y.data_ptr(), xq.data_ptr(), xs.data_ptr(),
                                        wq.data_ptr(), ws.data_ptr(), n, d, T, 64, None))

    ops = sum(2.0 * n * d * T for _, n, d in shapes)
    per = {}
    clocks = None
    try:
        for impl, steps in ((0, max(2, args.steps // 10)), (1, args.steps)):
            check(lib().leap_op_set_q8_gemm(impl))
            for _ in range(max(args.warmup, 3)):
                step()
            torch.cuda.synchronize(dev)
            sampler = ClockSampler(0)
            if impl == 1:
                sampler.start()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(steps):
                step()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            if impl == 1:
                clocks = sampler.stop()
            per[impl] = e0.elapsed_time(e1) / steps
    finally:
        check(lib().leap_op_set_q8_gemm(1))
    ms = per[1]
    tops = ops / (ms / 1e3) / 1e12
    peak = 2 * 1622.9
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            peak = 2 * float(json.load(f)["bf16_tflops"])
    emit({"metric": "W8A8 prompt GEMM TOP/s (int8)", "value": round(tops, 1), "unit": "TOP/s",
          "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
          "higher_is_better": True, "dtype": "int8 x int8 -> s32, f32 chain",
          "data": "synthetic (random int8 weights and activations, random scales)",
          "config": {"workload": f"the 4 W8A8 GEMMs of one Llama-3-8B-shape layer over {T} "
                                 "prompt tokens (wqkv, wo, w13, w2)", "tokens": T,
                     "l2": "inputs > L2: 219 MB of int8 weights per step"},
          "cuda_core_dp4a": {"value": round(ops / (per[0] / 1e3) / 1e12, 1), "unit": "TOP/s",
                             "ms_per_step": round(per[0], 4)},
          "roofline": {"bound": "tensor", "achieved": round(tops, 1), "peak": peak,
                       "peak_kind": "2 x measured bf16 dense (int8 rate)", "unit": "TOP/s",
                       "frac": round(tops / peak, 4)},
          "gpu_launches": 4 * args.steps, "clocks": clocks})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["leap", "reference"], default="leap")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--eager", action="store_true", help="launch from Python, no CUDA graph")
    ap.add_argument("--decode-impl", type=int, default=0,
                    help="0 auto, 1 split-KV + last-CTA combine, 2 cluster kernel, "
                         "3 wide split-KV, 4 split-KV + combine launch")
    ap.add_argument("--no-overlap", action="store_true",
                    help="no programmatic dependent launch between layers")
    ap.add_argument("--prefill", type=int, default=0,
                    help="benchmark config 4 (causal prefill of this many tokens) instead")
    ap.add_argument("--prefill-impl", type=int, default=3,
                    help="0 tcgen05 3xTF32 pipelined, 1 CUDA-core FP32, 2 tcgen05 3xTF32 serial, "
                         "3 tcgen05 TF32 + BF16 corrections pipelined")
    ap.add_argument("--layers", type=int, default=N_LAYERS)
    ap.add_argument("--ctx", type=int, default=CTX)
    ap.add_argument("--batched", action="store_true",
                    help="benchmark config 3 (64 ragged sequences) instead")
    ap.add_argument("--model", choices=sorted(MODELS), default=None,
                    help="end-to-end decode of a whole model (pipeline over the ranks)")
    ap.add_argument("--prompt", type=int, default=0, help="prompt tokens for --model")
    ap.add_argument("--q8-gemv", type=int, default=None,
                    help="W8A8 GEMV kernel for --model: 0 sliced, 1 register-staged, "
                         "2 persistent bulk-copy (default: the library's, 2)")
    ap.add_argument("--comm", choices=["native", "torch"], default="native",
                    help="stage transport for --model on N > 1 ranks")
    ap.add_argument("--no-pipeline", action="store_true",
                    help="skip the 8B W8A8 layer-range pipeline of the default line")
    ap.add_argument("--qgemm", type=int, default=0,
                    help="benchmark the W8A8 prompt GEMMs of one 8B layer over this many tokens")
    args = ap.parse_args()
    _keep_stdout_for_result()
    args.steps_given = args.steps is not None
    if args.steps is None:
        args.steps = 20
    if args.warmup < 3 and args.impl == "leap":
        args.warmup = 3  # timing rule: at least 3 warm-up steps
    if args.impl == "reference":
        if args.model:
            run_model_reference(args)
        else:
            run_reference_arm(args)
    elif args.model:
        run_model(args)
    elif args.batched:
        run_batched(args)
    elif args.prefill:
        run_prefill(args)
    elif args.qgemm:
        run_qgemm(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
