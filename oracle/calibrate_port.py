"""Calibrate the CPU baseline: the ports (the numpy oracle, oracle/mx_oracle.py,
and the torch-CPU port bench.py times, oracle/port_torch.py) against the
reference's own CPU path (mxtorch), on the same inputs and threads.

    PYTHONHASHSEED=0 PYTHONDONTWRITEBYTECODE=1 python oracle/calibrate_port.py /path/to/qtpytorch

Test infrastructure: it needs the reference checked out (it does not travel
to the GPU box), so bench.py times the port there and this script records,
once, how the port's time relates to the reference's on the configs[1]
workload (int8d x int8d 4096^3, block 128).  Prints one JSON line.
"""
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def _best(fn, reps):
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return min(ts)


def main(ref_dir):
    if os.environ.get("PYTHONHASHSEED") != "0":
        raise SystemExit("run with PYTHONHASHSEED=0")
    sys.path.insert(0, ref_dir)
    import mxtorch as mx  # the reference
    from oracle import mx_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    M = N = K = 4096
    torch.manual_seed(0)
    a = torch.randn(M, K)
    b = torch.randn(K, N)
    dt = mx.get_mx_dtype("int8d")
    out = {"cores": os.cpu_count(), "torch": torch.__version__}
    # full-job pieces, reference: quantize A, quantize B, matmul of a row sample
    out["ref_quantize_A_s"] = _best(lambda: mx.mx_tensor.quantize(a, dt, 128), 2)
    qb = mx.mx_tensor.quantize(b, dt, 128)
    out["ref_quantize_B_s"] = _best(lambda: mx.mx_tensor.quantize(b, dt, 128), 2)
    for rows in (128, 512):
        qa = mx.mx_tensor.quantize(a[:rows], dt, 128)
        out[f"ref_matmul_{rows}rows_s"] = _best(lambda: qa @ qb, 2)
        pa, sa, _ = O.quantize(a[:rows].numpy(), 8, "int", 128)
        pb, sb, _ = O.quantize(b.numpy(), 8, "int", 128)
        ca, cb = O.unpack(pa, 8, rows * K), O.unpack(pb, 8, K * N)
        out[f"port_matmul_{rows}rows_s"] = _best(
            lambda: O.qscale_matmul(ca, sa, cb, sb, rows, K, N, 128, 16), 2)
    out["port_quantize_A_s"] = _best(lambda: O.quantize(a.numpy(), 8, "int", 128), 2)
    out["port_quantize_B_s"] = _best(lambda: O.quantize(b.numpy(), 8, "int", 128), 2)
    # one full reference matmul at 4096^3 (the configs[1] job)
    qa = mx.mx_tensor.quantize(a, dt, 128)
    out["ref_matmul_full_s"] = _best(lambda: qa @ qb, 1)
    for who in ("ref", "port"):
        per_row = out[f"{who}_matmul_512rows_s"] / 512
        full = out[f"{who}_quantize_A_s"] + out[f"{who}_quantize_B_s"] + per_row * M
        out[f"{who}_full_job_est_s"] = full
        out[f"{who}_full_job_tops"] = 2.0 * M * N * K / full / 1e12
    out["ref_full_job_measured_s"] = (out["ref_quantize_A_s"] + out["ref_quantize_B_s"]
                                      + out["ref_matmul_full_s"])
    out["port_over_ref_time"] = out["port_full_job_est_s"] / out["ref_full_job_measured_s"]
    # the torch-CPU port bench.py times: the whole job, same inputs
    from oracle import port_torch as PT
    out["torch_port_full_job_s"] = _best(lambda: PT.int8_job(a, b, 128), 2)
    out["torch_port_over_ref_time"] = out["torch_port_full_job_s"] / out["ref_full_job_measured_s"]
    print(json.dumps(out))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")
