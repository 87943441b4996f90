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


def time_steps(fn, steps, flush, stream=None, align=None):
    """Device time of each call (CUDA events on the launching stream); L2
    flushed before each timed call.  A short device-side sleep after the flush
    lets the host enqueue the call before the GPU reaches the start event, so
    the interval holds the call's kernels and not Python launch overhead.
    `align` (multi-rank) enqueues a device-side barrier across the ranks
    before the start event, so every rank's step starts at the same time and
    no rank's interval holds another rank's host launch delay."""
    st = stream or torch.cuda.current_stream()
    ts = []
    for _ in range(steps):
        flush()
        torch.cuda._sleep(1_000_000)
        if align is not None:
            align()
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


# ── reference arm: the reference's CPU path, as the torch-CPU port ──────────
def cpu_full_job():
    """The whole configs[1] job on the host cores: int8d quantize of A and B,
    the packed int matmul and the int16d requantize (oracle/port_torch.py: the
    reference's CPU algorithm on torch's multithreaded CPU kernels, bit-exact
    to the reference's output; in the survey container it took 0.82x the
    reference's own time for this job).  Returns (TOPS, seconds)."""
    from oracle import port_torch as PT
    a, b = make_inputs()
    t0 = time.perf_counter()
    PT.int8_job(a, b, BLOCK)
    t = time.perf_counter() - t0
    return 2.0 * M * N * K / t / 1e12, t


def run_reference(args, world, rank):
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    vals = []
    for i in range(args.warmup + args.steps):
        v, t = cpu_full_job()
        if i >= args.warmup:
            vals.append(v)
    v = statistics.median(vals)
    cores = torch.get_num_threads()
    line = {
        "metric": "int8d x int8d packed GEMM throughput (4096^3, block 128)",
        "value": v, "unit": "TOPS", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong", "dtype": "int8", "data": "synthetic",
        "config": {"workload": "int8d x int8d GEMM M=N=K=4096 block 128 (configs[1])",
                   "sample": "the whole job per step"},
        "cpu_baseline": {"value": v, "unit": "TOPS", "cores": cores, "kind": "port",
                         "sample": "whole configs[1] job per step: quantize A and B, matmul, "
                                   "requantize (torch-CPU port, 0.82x the reference's time "
                                   "in calibration)"},
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
                                         sharded_qgemm_fused, sharded_qgemm_pull)

    dev = torch.device("cuda", local)
    lib = L.load()
    hbm, bf16, bf16s, peak_src = peaks()
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def flush():
        flush_buf.zero_()

    if args.only in ("gemv1", "gemv16", "wo2048", "wo2048_fast", "quant", "quant_f4", "dequant",
                     "h"):
        print(json.dumps(run_extras(args, dev, flush, torch.cuda.current_stream(dev), hbm, bf16)))
        return
    if args.only == "sweep":  # the full configs[4] sweep (a few minutes), one JSON line
        print(json.dumps({"sweep": run_sweep(dev, flush, torch.cuda.current_stream(dev), hbm,
                                             max(3, min(args.steps, 10)))}))
        return

    if args.only == "gemm8192":  # traffic case: the GEMM at 8192^3 (output > L2), untimed
        g = torch.Generator().manual_seed(0)
        qa8 = mxb.mx_tensor.quantize(torch.randn(8192, 8192, generator=g).to(dev), mxb.int8d, BLOCK)
        qb8 = mxb.mx_tensor.quantize(torch.randn(8192, 8192, generator=g).to(dev), mxb.int8d, BLOCK)
        for _ in range(3 + args.steps):
            qa8 @ qb8
        torch.cuda.synchronize()
        print(json.dumps({"only": "gemm8192", "device_error": lib.mxb_device_error(1)}))
        return

    a_h, b_h = make_inputs()
    qa = mxb.mx_tensor.quantize(a_h.to(dev), mxb.int8d, BLOCK)
    qb = mxb.mx_tensor.quantize(b_h.to(dev), mxb.int8d, BLOCK)
    w = ShardedQGemmWeight(qb, world, rank)
    nl = w.n1 - w.n0
    # N > 1: each rank's GEMM epilogue writes its int16d tiles into every
    # rank's full output over NVLink (CUDA IPC peer mappings), then one
    # one-element all-reduce orders the ranks; no gather or reorder pass
    # "pull": each rank's GEMM writes only its own output, the ranks' SMs
    # then read the peers' shards (same peer mappings, same barrier kernel)
    fused = world > 1 and args.gather in ("fused", "pull")
    pull = fused and args.gather == "pull"
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
        if pull:
            return sharded_qgemm_pull(qa, w, peers)
        if fused:
            return sharded_qgemm_fused(qa, w, peers)
        return sharded_qgemm(qa, w)

    stream = torch.cuda.current_stream(dev)
    align = peers.barrier if fused else None
    # The GEMM kernel alone, for the roofline: at N = 1 the plain matmul
    # (int16d requantization fused); at N > 1 the kernel the step runs, its
    # epilogue storing into every rank's output, without the ordering barrier.
    wsb = lib.mxb_qgemm_workspace_size(M, K, nl, 8, BLOCK)
    ws = L.workspace(wsb, dev)
    cp = torch.empty(lib.mxb_packed_bytes(M * nl, 16, BLOCK) // 4, dtype=torch.int32, device=dev)
    cs = torch.empty(M * nl // BLOCK, dtype=torch.float32, device=dev)

    def gemm_only():
        if fused:
            import ctypes as C
            out = peers.next()
            rc = lib.mxb_qgemm_sharded(L.ptr(qa._mx_packed), L.ptr(qa._mx_scales),
                                       qa._mx_scales.numel(), L.ptr(w.codes), L.ptr(w.scales),
                                       w.scales.numel(), M, K, nl, 8, BLOCK, N, w.n0,
                                       1 if pull else world,
                                       C.cast((C.c_void_p * 1)(out["ptr_w"][rank]) if pull
                                              else out["ptr_w"], C.c_void_p),
                                       C.cast((C.c_void_p * 1)(out["ptr_s"][rank]) if pull
                                              else out["ptr_s"], C.c_void_p), L.ptr(ws), wsb,
                                       torch.cuda.current_stream(dev).cuda_stream)
            L.check(rc, "mxb_qgemm_sharded")
            return
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
    # the fused step (in-kernel barrier, no collective) replays from a CUDA
    # graph; the NCCL all-gather variant runs eagerly
    step_g = graphed(step, stream) if (world == 1 or fused) else step
    with Clocks(local) as clk:
        barrier(world)
        ts = time_steps(step_g, args.steps, flush, stream, align)
        barrier(world)
    step_ms = max_over_ranks(sum(ts) / len(ts), world)
    value = 2.0 * M * N * K / (step_ms * 1e-3) / 1e12

    check = check_result(step(), qa, qb, world)

    barrier(world)
    tg = time_steps(graphed(gemm_only, stream) if world == 1 else gemm_only, args.steps, flush,
                    stream, align)
    barrier(world)
    gemm_ms = max_over_ranks(sum(tg) / len(tg), world)
    int8_peak = 2.0 * bf16  # kind::i8 issues twice the bf16 rate on sm_100
    achieved = 2.0 * M * nl * K / (gemm_ms * 1e-3) / 1e12
    traffic = profiled_traffic("qgemm_int8_4096") if world == 1 else None
    # bytes this rank's epilogue stores into its peers' outputs per launch
    peer_bytes = (world - 1) * (M * nl * 2 + M * nl // BLOCK * 4) if fused else 0

    # e2e: host fp32 operands -> public API -> host packed result.  Each rank
    # uploads its rows of A and its columns of B (whole 128-column blocks),
    # quantizes them (row-sharded quantize, no communication), all-gathers
    # A's codes and every rank's B block scales (the reference's B-scale view
    # pairs a column with other rows' blocks), runs the sharded matmul and
    # reads back its rows of the replicated result.
    e2e_step, h2d, d2h = make_e2e_step(a_h, b_h, w, peers, fused, world, rank, dev, pull)
    for _ in range(2):
        e2e_step()
    barrier(world)
    te = []
    for _ in range(args.steps):  # host wall clock: the caller's view of one call
        barrier(world)
        t0 = time.perf_counter()
        e2e_step()
        te.append((time.perf_counter() - t0) * 1e3)
    e2e_ms = max_over_ranks(sum(te) / len(te), world)

    sharded3 = None
    if not args.no_extra:
        sharded3 = run_config3_sharded(args, world, rank, dev, flush, stream, bf16)

    extra = {}
    if world == 1 and not args.no_extra:
        extra = run_extras(args, dev, flush, stream, hbm, bf16)

    if rank == 0:
        cpu = None
        if world == 1:
            torch.set_num_threads(os.cpu_count() or 1)
            cpu_full_job()  # warm-up
            v_cpu, t_cpu = cpu_full_job()
            cpu = {"value": v_cpu, "unit": "TOPS", "cores": torch.get_num_threads(),
                   "kind": "port",
                   "sample": f"whole configs[1] job ({t_cpu:.2f} s): quantize A and B, matmul, "
                             "requantize (torch-CPU port of the reference's CPU path)"}
        line = {
            "metric": "int8d x int8d packed GEMM throughput (4096^3, block 128)",
            "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "int8d x int8d GEMM M=N=K=4096 block 128 -> int16d "
                                   "(configs[1])",
                       "global_batch": M,
                       "parallelism": f"N-sharded x{world}" + (
                           (", local GEMM, barrier kernel over peer flags, then every SM "
                            "pulls the peers' shards over NVLink" if pull else
                            ", output gather fused into the GEMM epilogue (peer stores, "
                            "completion barrier kernel over peer flags)")
                           if fused else (", NCCL all-gather" if world > 1 else "")
                           + (f" ({fuse_note})" if fuse_note else "")),
                       "l2": "flushed (256 MiB write) before every timed step"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak,
                         "unit": "TOPS", "frac": achieved / int8_peak, "traffic": traffic,
                         "traffic_note": ("DRAM bytes of one 4096^3 launch (ncu): the inputs "
                                          "read once; the 34 MB result drains from L2 after "
                                          "the launch" if traffic else None),
                         "kernel": "qgemm_tc_kernel (int16d requantization fused"
                                   + (", stores into every rank's output)" if fused and not pull
                                      else ")"),
                         "peak_note": f"2x {peak_src} bf16 burst {bf16} TFLOP/s"},
            "cpu_baseline": cpu,
            "e2e": {"value": 2.0 * M * N * K / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                    "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gemm_ms": gemm_ms,
            "nvlink": ({"peer_bytes_per_launch": peer_bytes,
                        "gbs_per_direction": peer_bytes / (gemm_ms * 1e-3) / 1e9,
                        "link_ref_gbs": 770.0} if fused and not pull else None),
            "config3_sharded": sharded3,
            "check": check,
            "gpu_launches": int(launches),
            "clocks": clk.summary(),
            "extra": extra,
        }
        print(json.dumps(line), flush=True)


def make_e2e_step(a_h, b_h, w, peers, fused, world, rank, dev, pull=False):
    """One call of the user-facing path from host buffers (see run_ours)."""
    import qtpytorch_b200 as mxb
    from qtpytorch_b200 import ops
    from qtpytorch_b200.parallel import (ShardedQGemmWeight, row_shard, sharded_qgemm,
                                         sharded_qgemm_fused, sharded_qgemm_pull)
    r0, r1 = [b * BLOCK // K for b in row_shard(M * K // BLOCK, world, rank)]  # rows of A
    n0, n1 = w.n0, w.n1
    nl = n1 - n0
    a_pin = a_h[r0:r1].contiguous().pin_memory()
    b_pin = b_h[:, n0:n1].contiguous().pin_memory()  # this rank's columns, prepared once
    xa = torch.empty(r1 - r0, K, dtype=torch.float32, device=dev)
    xb = torch.empty(K, nl, dtype=torch.float32, device=dev)
    side = torch.cuda.Stream(dev)
    rows_out = (r1 - r0)
    out_words = torch.empty(rows_out * N // 2, dtype=torch.int32, pin_memory=True)
    out_scales = torch.empty(rows_out * N // BLOCK, dtype=torch.float32, pin_memory=True)
    kbn = K // BLOCK
    shim = ShardedQGemmWeight.__new__(ShardedQGemmWeight)
    shim.K, shim.N, shim.world, shim.rank, shim.block = K, N, world, rank, BLOCK
    shim.dtype, shim.shards, shim.n0, shim.n1 = mxb.int8d, w.shards, n0, n1

    def gather(t):
        if world == 1:
            return t.unsqueeze(0)
        import torch.distributed as dist
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.contiguous())
        return out

    def e2e_step():
        cur = torch.cuda.current_stream(dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            xb.copy_(b_pin, non_blocking=True)
        xa.copy_(a_pin, non_blocking=True)
        pa, sa, _ = ops.quantize(xa, mxb.int8d, BLOCK)
        cur.wait_stream(side)
        pb, sb, _ = ops.quantize(xb, mxb.int8d, BLOCK)  # blocks = B's blocks of these columns
        ga, gs = gather(pa), gather(sa)
        qa = mxb.mx_tensor(ga.reshape(-1), gs.reshape(-1), mxb.int8d, (M, K), M * K, BLOCK)
        # B's scales of all blocks [K, N/128], rows of N/128 in rank order, then
        # this shard's slice of the [K/128, N] view
        sball = gather(sb.view(K, nl // BLOCK)).permute(1, 0, 2).reshape(-1)
        shim.codes = pb.view(K, nl)
        shim.scales = sball.view(kbn, N)[:, n0:n1].contiguous()
        c = ((sharded_qgemm_pull if pull else sharded_qgemm_fused)(qa, shim, peers) if fused
             else sharded_qgemm(qa, shim))
        out_words.copy_(c._mx_packed.view(M, N // 2)[r0:r1].reshape(-1), non_blocking=True)
        out_scales.copy_(c._mx_scales.view(M, N // BLOCK)[r0:r1].reshape(-1), non_blocking=True)
        cur.synchronize()
        return out_words, out_scales

    h2d = a_pin.numel() * 4 + b_pin.numel() * 4
    d2h = out_words.numel() * 4 + out_scales.numel() * 4
    return e2e_step, h2d, d2h


def run_config3_sharded(args, world, rank, dev, flush, stream, bf16):
    """the int4dh weight-only linear, W 8192 x 8192 ~ N(0, 0.02)
    with 8 outlier input channels x25, x bf16 [4096, 8192] replicated, W^T
    column-sharded over the ranks.  Times the rank's GEMM alone and the whole
    step (GEMM, per-shard transform, all-gather, cross-shard stage), max over
    ranks, and checks 16 sampled rows against the single-GPU module."""
    import math
    import qtpytorch_b200 as mxb
    from qtpytorch_b200 import _lib as L
    from qtpytorch_b200 import ops
    from qtpytorch_b200 import parallel as P
    g3 = torch.Generator().manual_seed(3)
    W3 = torch.randn(8192, 8192, generator=g3) * 0.02
    W3[:, torch.randperm(8192, generator=g3)[:8]] *= 25.0
    lin3 = torch.nn.Linear(8192, 8192, bias=False)
    with torch.no_grad():
        lin3.weight.copy_(W3)
    dt = mxb.get_mx_dtype("int4dh")
    ml3 = mxb.mx_linear.from_linear(lin3.to(dev), dt, 128)
    del W3, lin3
    x3 = torch.randn(4096, 8192, generator=torch.Generator().manual_seed(4)).bfloat16().to(dev)
    sw = P.ShardedLinearWeight.from_module(ml3, world, rank)
    nl = sw.n1 - sw.n0

    def gemm():
        ops.linear_wonly(x3, sw.codes, sw.scales, 8192, nl, dt, 128)

    def step():
        return P.sharded_linear(x3, sw)

    for _ in range(3):
        gemm()
        step()
    barrier(world)
    steps = max(3, min(args.steps, 10))
    tg = time_steps(graphed(gemm, stream), steps, flush, stream)
    barrier(world)
    ts = time_steps(graphed(step, stream) if world == 1 else step, steps, flush, stream)
    barrier(world)
    gemm_ms = max_over_ranks(statistics.median(tg), world)
    step_ms = max_over_ranks(statistics.median(ts), world)
    y = step()
    rows = torch.tensor([0, 1, 777, 1500, 2047, 2048, 3001, 4095, 5, 99, 1234, 2500, 3333, 3900,
                         4000, 4094], device=dev)
    ref = ml3(x3[rows])
    q = ml3._mx_weight
    D = ops.dequantize(q._mx_packed, q._mx_scales, dt.base, q._mx_n, 128, (8192, 8192))
    bound = (x3[rows].float().abs() @ D.abs()).sum(dim=1, keepdim=True) / math.sqrt(8192)
    ok = bool(torch.all((y[rows] - ref).abs() <= 2e-5 * bound)) and L.load().mxb_device_error(1) == 0
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    flops = 2.0 * 4096 * 8192 * 8192
    return {"workload": "int4dh W 8192x8192 (x25 outliers), x bf16 4096x8192, N-sharded "
                        f"x{world} (configs[3])",
            "gemm_ms": gemm_ms, "gemm_tflops": flops / world / gemm_ms / 1e9,
            "gemm_tflops_all_ranks": flops / gemm_ms / 1e9,
            "step_ms": step_ms, "tflops": flops / step_ms / 1e9,
            "tensor_frac_bf16": flops / world / gemm_ms / 1e9 / bf16,
            "unrotation": ("kronecker split" if sw.kron_split and world > 1 else
                           "full rows" + (" after the gather" if world > 1 else "")),
            "check": "ok" if int(flag.item()) == 1 else "mismatch"}


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
    if args.only in ("quant", "quant_f4"):  # profiling case: int4d (float4d) quantize of
        x = torch.randn(1 << 26, device=dev)  # 2^26 fp32 values
        dt = mxb.int4d if args.only == "quant" else mxb.get_mx_dtype("float4d")
        for _ in range(3 + args.steps):
            ops.quantize(x, dt, 128)
        torch.cuda.synchronize()
        return {"only": args.only}
    if args.only == "h":  # profiling case: int4dh quantize / dequantize of W^T 8192 x 8192
        # and the row unrotation of y 4096 x 8192
        dt = mxb.get_mx_dtype("int4dh")
        w = torch.randn(8192, 8192, device=dev) * 0.02
        y = torch.randn(4096, 8192, device=dev)
        for _ in range(3 + args.steps):
            p_, s_, n_ = ops.quantize(w, dt, 128)
            ops.dequantize(p_, s_, dt, n_, 128, (8192, 8192))
            ops.hadamard_rows(y, dt.hadamard_seed, True)
        torch.cuda.synchronize()
        return {"only": "h"}
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
    only = {"gemv1": (1,), "gemv16": (16,), "wo2048": (2048,), "wo2048_fast": (2048,)}.get(
        args.only)
    if args.only == "wo2048_fast":
        ml.mode = "fast"
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
    # Decode as a model runs it: one graph of 8 consecutive linears over 8
    # distinct int4d weights (8 x 24 MB > L2, so no flush is needed and each
    # weight streams from HBM); time per linear = graph time / 8.  The
    # single-call lines above also carry the fixed launch and event time.
    ws8 = []
    for _ in range(8):
        lin = torch.nn.Linear(4096, 11008, bias=False, device=dev)
        with torch.no_grad():
            lin.weight.normal_(0.0, 0.02)
        ws8.append(mxb.mx_linear.from_linear(lin, mxb.int4d, 128))
        del lin
    for Mx in (1, 16):
        x = torch.randn(Mx, 4096, generator=g2).bfloat16().to(dev)
        for m_ in ws8:
            m_(x)

        def chain(x=x):
            for m_ in ws8:
                m_(x)
        fn = graphed(chain, stream)
        t = statistics.median(time_steps(fn, steps, lambda: None, stream)) / 8
        byts = wbytes + x.numel() * 2 + Mx * 11008 * 4
        out[f"wonly_int4d_M{Mx}_stream8"] = {"ms": t, "gbs": byts / t / 1e6,
                                             "hbm_frac": byts / t / 1e6 / hbm,
                                             "note": "per linear in a graph of 8 over distinct weights (192 MB > L2)"}
    del ws8
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
    out.update(run_h_kernels(dev, flush, stream, hbm, steps))
    return out


def run_h_kernels(dev, flush, stream, hbm, steps):
    """The Hadamard-variant kernels at configs[3] sizes: int4dh quantize and
    dequantize of W^T 8192 x 8192 (fused 8192-point row WHT) and the row
    unrotation of y 4096 x 8192; GB/s of algorithmic bytes."""
    import qtpytorch_b200 as mxb
    from qtpytorch_b200 import ops
    out = {}
    dt = mxb.get_mx_dtype("int4dh")
    w = torch.randn(8192, 8192, device=dev) * 0.02
    n = w.numel()
    p_, s_, _ = ops.quantize(w, dt, 128)
    fq = graphed(lambda: ops.quantize(w, dt, 128), stream)
    tq = statistics.median(time_steps(fq, steps, flush, stream))
    fd = graphed(lambda: ops.dequantize(p_, s_, dt, n, 128, (8192, 8192)), stream)
    td = statistics.median(time_steps(fd, steps, flush, stream))
    qb = n * 4 + n / 2 + n / 128 * 4
    out["quantize_int4dh_8192x8192"] = {"ms": tq, "gbs": qb / tq / 1e6,
                                         "hbm_frac": qb / tq / 1e6 / hbm}
    out["dequantize_int4dh_8192x8192"] = {"ms": td, "gbs": qb / td / 1e6,
                                           "hbm_frac": qb / td / 1e6 / hbm}
    y = torch.randn(4096, 8192, device=dev)
    fr = graphed(lambda: ops.hadamard_rows(y, dt.hadamard_seed, True), stream)
    tr = statistics.median(time_steps(fr, steps, flush, stream))
    rb = y.numel() * 8
    out["hadamard_rows_4096x8192"] = {"ms": tr, "gbs": rb / tr / 1e6, "hbm_frac": rb / tr / 1e6 / hbm}
    return out


def run_sweep(dev, flush, stream, hbm, steps):
    """configs[4] in full: fp32 / bf16 N(0,1) of 2^20 .. 2^30 elements (x4)
    and a Student-t (nu = 3) tail at 2^26, quantized to int2d / int1d /
    float4d at blocks 32 and 128, then dequantized; GB/s of algorithmic
    bytes (quantize: input + codes + scales; dequantize: codes + scales +
    fp32 output).  Sizes under the L2 capacity are flushed between steps."""
    import qtpytorch_b200 as mxb
    from qtpytorch_b200 import ops
    res = {}
    cases = [(1 << e, "normal") for e in range(20, 31, 2)] + [(1 << 26, "student_t")]
    for n, dist_ in cases:
        torch.cuda.manual_seed(5)
        if dist_ == "normal":
            base = torch.randn(n, device=dev)
        else:
            base = torch.distributions.StudentT(torch.tensor(3.0, device=dev)).sample((n,))
        for in_dt in (torch.float32, torch.bfloat16):
            x = base.to(in_dt)
            ib = 4 if in_dt == torch.float32 else 2
            for dt in ("int2d", "int1d", "float4d"):
                d = mxb.get_mx_dtype(dt)
                for blk in (32, 128):
                    p_, s_, _ = ops.quantize(x, d, blk)
                    fq = graphed(lambda: ops.quantize(x, d, blk), stream)
                    tq = statistics.median(time_steps(fq, steps, flush, stream))
                    fd = graphed(lambda: ops.dequantize(p_, s_, d, n, blk), stream)
                    td = statistics.median(time_steps(fd, steps, flush, stream))
                    qb = n * ib + n * d.bits / 8 + n / blk * 4
                    db = n * d.bits / 8 + n / blk * 4 + n * 4
                    key = (f"2^{n.bit_length() - 1}_{dist_}_{'fp32' if ib == 4 else 'bf16'}_"
                           f"{dt}_b{blk}")
                    res[key] = {"q_gbs": round(qb / tq / 1e6, 1),
                                "q_frac": round(qb / tq / 1e6 / hbm, 3),
                                "dq_gbs": round(db / td / 1e6, 1),
                                "dq_frac": round(db / td / 1e6 / hbm, 3)}
                    del p_, s_
            del x
        del base
        torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-extra", action="store_true")
    ap.add_argument("--gather", default="fused", choices=["fused", "pull", "nccl"],
                    help="N > 1: output gather fused into the GEMM kernel (peer stores), "
                         "pulled by every SM after the local GEMM, or NCCL all-gather")
    ap.add_argument("--only", default=None, choices=["gemm", "gemm8192", "gemv1", "gemv16", "wo2048", "wo2048_fast", "quant",
                             "quant_f4", "dequant", "h",
                             "sweep"],
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
