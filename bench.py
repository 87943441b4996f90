"""Benchmark of the mxtorch hot path on B200.

Headline: int8d x int8d packed GEMM, M=N=K=4096,
block 128, seeded N(0,1) fp32 operands quantized on the device; output int16d
(requantized, packed).  At N GPUs the weight B is column-sharded and every
rank's GEMM epilogue writes its int16d tiles into all ranks' full outputs
over NVLink (the all-gather fused into the kernel; `--gather nccl` times
the NCCL all-gather + reorder instead).  Strong scaling: the total work is
fixed.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  `value` times the GEMM on operands already
resident in HBM; `e2e` times the user-facing call with host buffers (h2d of
the fp32 operands, quantize, matmul, d2h of the packed result).  Extra
sub-results (weight-only int4d GEMM / GEMV, quantize) go under `extra`.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = N = K = 4096
BLOCK = 128
L2_FLUSH_BYTES = 256 << 20


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.p is not None:
            time.sleep(0.2)
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                out, _ = self.p.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def graphed(fn, stream):
    """Capture fn (already warmed up) into a CUDA graph; returns a replay
    callable, or fn itself if capture is not possible."""
    g = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    try:
        with torch.cuda.graph(g):  # captured on torch's side stream
            fn()
    except Exception:  # noqa: BLE001 - fall back to eager launches
        torch.cuda.synchronize()
        return fn
    torch.cuda.synchronize()
    return g.replay


def time_steps(fn, steps, flush, stream=None):
    """Device time of each call (CUDA events on the launching stream); L2
    flushed before each timed call.  A short device-side sleep after the flush
    lets the host enqueue the call before the GPU reaches the start event, so
    the interval holds the call's kernels and not Python launch overhead."""
    st = stream or torch.cuda.current_stream()
    ts = []
    for _ in range(steps):
        flush()
        torch.cuda._sleep(1_000_000)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(st)
        fn()
        e1.record(st)
        ts.append((e0, e1))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ts]


def dist_setup(gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def profiled_traffic(key):
    """DRAM bytes per launch recorded from an ncu capture (profiles/traffic.txt)."""
    p = os.path.join(ROOT, "profiles", "traffic.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        f = line.split()
        if len(f) == 2 and f[0] == key:
            return int(f[1])
    return None


def make_inputs():
    torch.manual_seed(0)
    a = torch.randn(M, K)
    b = torch.randn(K, N)
    return a, b


# ── reference arm: the CPU oracle port on the host cores ─────────────────────
def cpu_baseline_sample(rows=256, reps=1):
    """Reference path on the host: quantize A-rows + B, packed int GEMM, requant
    (oracle port of mxtorch.py:1426-1463, 1299-1385) on a row sample of A."""
    from oracle import mx_oracle as O
    a, b = make_inputs()
    a = a[:rows].numpy()
    b = b.numpy()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        pa, sa, _ = O.quantize(a, 8, "int", BLOCK)
        pb, sb, _ = O.quantize(b, 8, "int", BLOCK)
        ca = O.unpack(pa, 8, a.size)
        cb = O.unpack(pb, 8, b.size)
        O.qscale_matmul(ca, sa, cb, sb, rows, K, N, BLOCK, 16)
        ts.append(time.perf_counter() - t0)
    t = min(ts)
    return 2.0 * rows * N * K / t / 1e12, t


def run_reference(args, world, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    rows = 128
    vals = []
    for i in range(args.warmup + args.steps):
        v, t = cpu_baseline_sample(rows)
        if i >= args.warmup:
            vals.append(v)
    v = statistics.median(vals)
    cores = os.cpu_count()
    line = {
        "metric": "int8d x int8d packed GEMM throughput (4096^3, block 128)",
        "value": v, "unit": "TOPS", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong", "dtype": "int8", "data": "synthetic",
        "config": {"workload": "int8d x int8d GEMM M=N=K=4096 block 128 (configs[1])",
                   "sample": f"{rows} rows of A x full B per step"},
        "cpu_baseline": {"value": v, "unit": "TOPS", "cores": cores, "kind": "port",
                         "sample": f"quantize {rows}x4096 A + 4096x4096 B, GEMM, requant"},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)


# ── our arm ──────────────────────────────────────────────────────────────────
def run_ours(args, world, rank, local):
    import qtpytorch_b200 as mxb
    from qtpytorch_b200 import _lib as L
    from qtpytorch_b200 import ops
    from qtpytorch_b200.parallel import (PeerOutputs, ShardedQGemmWeight, sharded_qgemm,
                                         sharded_qgemm_fused)

    dev = torch.device("cuda", local)
    lib = L.load()
    hbm, bf16, bf16s, peak_src = peaks()
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def flush():
        flush_buf.zero_()

    if args.only in ("gemv1", "gemv16", "wo2048", "quant", "dequant"):
        print(json.dumps(run_extras(args, dev, flush, torch.cuda.current_stream(dev), hbm, bf16)))
        return

    a_h, b_h = make_inputs()
    qa = mxb.mx_tensor.quantize(a_h.to(dev), mxb.int8d, BLOCK)
    qb = mxb.mx_tensor.quantize(b_h.to(dev), mxb.int8d, BLOCK)
    w = ShardedQGemmWeight(qb, world, rank)
    nl = w.n1 - w.n0
    # N > 1: each rank's GEMM epilogue writes its int16d tiles into every
    # rank's full output over NVLink (CUDA IPC peer mappings), then one
    # one-element all-reduce orders the ranks; no gather or reorder pass
    fused = world > 1 and args.gather == "fused"
    peers, fuse_note = None, None
    if fused:
        # all ranks map their peers' outputs; if any rank cannot, all use
        # the NCCL all-gather instead (decided together, so none waits alone)
        try:
            peers = PeerOutputs(M, N, BLOCK, world, rank, device=dev)
            ok = 1
        except Exception as e:  # noqa: BLE001 - reported in the JSON line
            fuse_note = f"peer mapping failed on rank {rank}: {e}"[:200]
            ok = 0
        import torch.distributed as dist
        flag = torch.tensor([ok], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0:
            fused = False
            fuse_note = fuse_note or "a peer rank could not map the outputs"

    def step():
        if fused:
            return sharded_qgemm_fused(qa, w, peers)
        return sharded_qgemm(qa, w)

    # GEMM kernel alone (fp32 C, no requantization) for the roofline
    c32 = torch.empty(M, nl, dtype=torch.float32, device=dev)
    wsb = lib.mxb_qgemm_workspace_size(M, K, nl, 8, BLOCK)
    ws = L.workspace(wsb, dev)
    cp = torch.empty(lib.mxb_packed_bytes(M * nl, 16, BLOCK) // 4, dtype=torch.int32, device=dev)
    cs = torch.empty(M * nl // BLOCK, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def gemm_only():
        rc = lib.mxb_qgemm(L.ptr(qa._mx_packed), L.ptr(qa._mx_scales), qa._mx_scales.numel(),
                           L.ptr(w.codes), L.ptr(w.scales), w.scales.numel(), M, K, nl, 8,
                           BLOCK, 16, L.ptr(cp), L.ptr(cs), None, L.ptr(ws), wsb,
                           torch.cuda.current_stream(dev).cuda_stream)
        L.check(rc, "mxb_qgemm")

    for _ in range(max(args.warmup, 3)):
        step()
        gemm_only()
    barrier(world)
    if args.only == "gemm":  # profiling case: the GEMM kernel alone, no timing
        for _ in range(args.steps):
            gemm_only()
        torch.cuda.synchronize()
        print(json.dumps({"only": "gemm", "device_error": lib.mxb_device_error(1)}))
        return

    # kernels of this library per step, counted on one eager step; the timed
    # steps replay the same launches from a CUDA graph
    n0 = lib.mxb_launch_count()
    step()
    launches = (lib.mxb_launch_count() - n0) * args.steps
    # N > 1: eager steps (the NCCL gather is not graph-captured here)
    step_g = graphed(step, stream) if world == 1 else step
    with Clocks(local) as clk:
        barrier(world)
        ts = time_steps(step_g, args.steps, flush, stream)
        barrier(world)
    step_ms = max_over_ranks(sum(ts) / len(ts), world)
    value = 2.0 * M * N * K / (step_ms * 1e-3) / 1e12

    check = check_result(step(), qa, qb, world)

    tg = time_steps(graphed(gemm_only, stream), args.steps, flush, stream)
    gemm_ms = max_over_ranks(sum(tg) / len(tg), world)
    int8_peak = 2.0 * bf16  # kind::i8 issues twice the bf16 rate on sm_100
    achieved = 2.0 * M * nl * K / (gemm_ms * 1e-3) / 1e12
    traffic = profiled_traffic("qgemm_int8_4096") if world == 1 else None

    # e2e: host fp32 operands -> public API -> host packed result
    a_pin = a_h.pin_memory()
    b_pin = b_h.pin_memory()

    # B's upload runs on a side stream while A is uploaded and quantized; the
    # packed result comes back into pinned host buffers.
    side = torch.cuda.Stream(dev)
    out_words = torch.empty(M * nl // 2 * world, dtype=torch.int32, pin_memory=True)
    out_scales = torch.empty(M * N // BLOCK, dtype=torch.float32, pin_memory=True)
    xa = torch.empty(M, K, dtype=torch.float32, device=dev)
    xb = torch.empty(K, N, dtype=torch.float32, device=dev)

    def e2e_step():
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            xb.copy_(b_pin, non_blocking=True)
        xa.copy_(a_pin, non_blocking=True)
        ea = mxb.mx_tensor.quantize(xa, mxb.int8d, BLOCK)
        torch.cuda.current_stream(dev).wait_stream(side)
        eb = mxb.mx_tensor.quantize(xb, mxb.int8d, BLOCK)
        ew = ShardedQGemmWeight(eb, world, rank)
        ec = sharded_qgemm_fused(ea, ew, peers) if fused else sharded_qgemm(ea, ew)
        out_words.copy_(ec._mx_packed, non_blocking=True)
        out_scales.copy_(ec._mx_scales, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return out_words, out_scales

    for _ in range(2):
        e2e_step()
    barrier(world)
    te = []
    for _ in range(args.steps):  # host wall clock: the caller's view of one call
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        pk, sc = e2e_step()
        te.append((time.perf_counter() - t0) * 1e3)
    e2e_ms = max_over_ranks(sum(te) / len(te), world)
    h2d = a_h.numel() * 4 + b_h.numel() * 4
    d2h = pk.numel() * pk.element_size() + sc.numel() * 4

    extra = {}
    if world == 1 and not args.no_extra:
        extra = run_extras(args, dev, flush, stream, hbm, bf16)

    if rank == 0:
        cpu = None
        if world == 1:
            torch.set_num_threads(os.cpu_count() or 1)
            v_cpu, t_cpu = cpu_baseline_sample(128)
            cpu = {"value": v_cpu, "unit": "TOPS", "cores": os.cpu_count(), "kind": "port",
                   "sample": "quantize 128x4096 A rows + 4096x4096 B, int GEMM, requant "
                             f"({t_cpu:.2f} s)"}
        line = {
            "metric": "int8d x int8d packed GEMM throughput (4096^3, block 128)",
            "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "int8d x int8d GEMM M=N=K=4096 block 128 -> int16d "
                                   "(configs[1])",
                       "global_batch": M,
                       "parallelism": f"N-sharded x{world}" + (
                           ", output gather fused into the GEMM epilogue (peer stores)"
                           if fused else (", NCCL all-gather" if world > 1 else "")
                           + (f" ({fuse_note})" if fuse_note else "")),
                       "l2": "flushed (256 MiB write) before every timed step"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak,
                         "unit": "TOPS", "frac": achieved / int8_peak, "traffic": traffic,
                         "kernel": "qgemm_tc_kernel (int16d requantization fused)",
                         "peak_note": f"2x {peak_src} bf16 burst {bf16} TFLOP/s"},
            "cpu_baseline": cpu,
            "e2e": {"value": 2.0 * M * N * K / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "check": check,
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "extra": extra,
        }
        print(json.dumps(line), flush=True)


def check_result(c, qa, qb, world):
    """Sampled rows of the (gathered) int16d C against a single-GPU matmul of
    the same rows of A with the whole B, on every rank (CUDA-core kernel for
    the 40-row sample, an implementation independent of the tcgen05 one);
    'ok' only if every rank agrees bit for bit."""
    from qtpytorch_b200 import ops
    torch.cuda.synchronize()
    dev = qa._mx_packed.device
    rows = np.concatenate([[0, M - 1], np.random.default_rng(7).choice(M - 2, 38, replace=False) + 1])
    r = torch.from_numpy(np.sort(rows)).to(dev)
    a_rows = qa._mx_packed[: M * K].view(M, K)[r].contiguous()
    s_rows = qa._mx_scales.view(M, K // BLOCK)[r].contiguous()
    words, scales, _ = ops.qgemm(a_rows, s_rows, qb._mx_packed, qb._mx_scales, len(rows), K, N,
                                 8, BLOCK, 16)
    ok = (torch.equal(c._mx_packed.view(M, N // 2)[r], words.view(len(rows), N // 2))
          and torch.equal(c._mx_scales.view(M, N // BLOCK)[r].view(torch.int32),
                          scales.view(len(rows), N // BLOCK).view(torch.int32)))
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return "ok" if int(flag.item()) == 1 else "mismatch"


def run_extras(args, dev, flush, stream, hbm, bf16):
    """Weight-only int4d and quantize/pack sub-results."""
    import qtpytorch_b200 as mxb
    from qtpytorch_b200 import ops
    out = {}
    steps = max(3, min(args.steps, 10))
    if args.only == "quant":  # profiling case: int4d quantize of 2^26 fp32 values
        x = torch.randn(1 << 26, device=dev)
        for _ in range(3 + args.steps):
            ops.quantize(x, mxb.int4d, 128)
        torch.cuda.synchronize()
        return {"only": "quant"}
    if args.only == "dequant":  # profiling case: int4d dequantize of 2^26 values
        x = torch.randn(1 << 26, device=dev)
        p_, s_, _ = ops.quantize(x, mxb.int4d, 128)
        for _ in range(3 + args.steps):
            ops.dequantize(p_, s_, mxb.int4d, 1 << 26, 128)
        torch.cuda.synchronize()
        return {"only": "dequant"}
    g = torch.Generator().manual_seed(1)
    W = torch.randn(11008, 4096, generator=g) * 0.02
    lin = torch.nn.Linear(4096, 11008, bias=False)
    with torch.no_grad():
        lin.weight.copy_(W)
    ml = mxb.mx_linear.from_linear(lin.to(dev), mxb.int4d, 128)
    wbytes = ml._mx_weight._mx_packed.numel() + ml._mx_weight._mx_scales.numel() * 4
    g2 = torch.Generator().manual_seed(2)
    only = {"gemv1": (1,), "gemv16": (16,), "wo2048": (2048,)}.get(args.only)
    for Mx in only or (1, 16, 128, 2048):
        x = torch.randn(Mx, 4096, generator=g2).bfloat16().to(dev)
        for _ in range(3):
            ml(x)
        if only:  # profiling case: untimed launches
            for _ in range(args.steps):
                ml(x)
            torch.cuda.synchronize()
            return {"only": args.only}
        fn = graphed(lambda: ml(x), stream)
        t = statistics.median(time_steps(fn, steps, flush, stream))
        flops = 2.0 * Mx * 4096 * 11008
        byts = wbytes + x.numel() * 2 + Mx * 11008 * 4
        out[f"wonly_int4d_M{Mx}"] = {"ms": t, "tflops": flops / t / 1e9,
                                     "gbs": byts / t / 1e6, "hbm_frac": byts / t / 1e6 / hbm,
                                     "tensor_frac_bf16": flops / t / 1e9 / bf16}
        if Mx >= 128:  # fast mode: weights rounded to bf16 once (one MMA per K step)
            ml.mode = "fast"
            ml(x)
            fn = graphed(lambda: ml(x), stream)
            t = statistics.median(time_steps(fn, steps, flush, stream))
            ml.mode = "parity"
            out[f"wonly_int4d_M{Mx}_fast"] = {"ms": t, "tflops": flops / t / 1e9,
                                              "tensor_frac_bf16": flops / t / 1e9 / bf16}
    for dt, n in (("int2d", 1 << 28), ("int4d", 1 << 28), ("float4d", 1 << 26)):
        x = torch.randn(n, device=dev)
        d = mxb.get_mx_dtype(dt)
        for _ in range(2):
            ops.quantize(x, d, 128)
        fn = graphed(lambda: ops.quantize(x, d, 128), stream)
        t = statistics.median(time_steps(fn, steps, flush, stream))
        byts = n * 4 + n * d.bits / 8 + n / 128 * 4
        out[f"quantize_{dt}_fp32_2^{n.bit_length() - 1}"] = {
            "ms": t, "gbs": byts / t / 1e6, "hbm_frac": byts / t / 1e6 / hbm}
        del x
    # configs[4] sweep (bounded): int2d / int1d / float4d, fp32 and bf16
    # N(0,1) inputs of 2^26 elements (larger than L2), block 32 and 128,
    # quantize then dequantize; GB/s = algorithmic bytes / device time
    sweep = {}
    n = 1 << 26
    for in_dt in (torch.float32, torch.bfloat16):
        x = torch.randn(n, device=dev).to(in_dt)
        ib = 4 if in_dt == torch.float32 else 2
        for dt in ("int2d", "int1d", "float4d", "int4d", "int8d"):
            d = mxb.get_mx_dtype(dt)
            for blk in ((32, 128) if dt in ("int2d", "int1d", "float4d") else (128,)):
                p_, s_, _ = ops.quantize(x, d, blk)
                fq = graphed(lambda: ops.quantize(x, d, blk), stream)
                tq = statistics.median(time_steps(fq, steps, flush, stream))
                fd = graphed(lambda: ops.dequantize(p_, s_, d, n, blk), stream)
                td = statistics.median(time_steps(fd, steps, flush, stream))
                qb = n * ib + n * d.bits / 8 + n / blk * 4
                db = n * d.bits / 8 + n / blk * 4 + n * 4
                key = f"{dt}_{'fp32' if ib == 4 else 'bf16'}_b{blk}"
                sweep[key] = {"q_gbs": round(qb / tq / 1e6, 1), "q_frac": round(qb / tq / 1e6 / hbm, 3),
                              "dq_gbs": round(db / td / 1e6, 1), "dq_frac": round(db / td / 1e6 / hbm, 3)}
                del p_, s_
        del x
    out["quant_dequant_sweep_2^26"] = sweep
    # configs[3] on one rank: int4dh weight-only linear, W 8192 x 8192 ~ N(0, 0.02)
    # with 8 outlier input channels x25, x bf16 [4096, 8192]; the sharded
    # linear at world 1 (GEMM + the 8192-point unrotation of y)
    from qtpytorch_b200 import parallel as P
    g3 = torch.Generator().manual_seed(3)
    W3 = torch.randn(8192, 8192, generator=g3) * 0.02
    W3[:, torch.randperm(8192, generator=g3)[:8]] *= 25.0
    lin3 = torch.nn.Linear(8192, 8192, bias=False)
    with torch.no_grad():
        lin3.weight.copy_(W3)
    ml3 = mxb.mx_linear.from_linear(lin3.to(dev), mxb.get_mx_dtype("int4dh"), 128)
    del W3, lin3
    x3 = torch.randn(4096, 8192, generator=torch.Generator().manual_seed(4)).bfloat16().to(dev)
    sw3 = P.ShardedLinearWeight.from_module(ml3, 1, 0)
    for _ in range(2):
        P.sharded_linear(x3, sw3)
    fn = graphed(lambda: P.sharded_linear(x3, sw3), stream)
    t = statistics.median(time_steps(fn, steps, flush, stream))
    flops = 2.0 * 4096 * 8192 * 8192
    out["wonly_int4dh_8192_M4096_g1"] = {"ms": t, "tflops": flops / t / 1e9,
                                         "tensor_frac_bf16": flops / t / 1e9 / bf16}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true")
    ap.add_argument("--gather", default="fused", choices=["fused", "nccl"],
                    help="N > 1: output gather fused into the GEMM kernel, or NCCL all-gather")
    ap.add_argument("--only", default=None, choices=["gemm", "gemv1", "gemv16", "wo2048", "quant", "dequant"],
                    help="run one kernel case untimed (for profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return
    world, rank, local = dist_setup(args.gpus)
    run_ours(args, world, rank, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
