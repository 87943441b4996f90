"""Worker of tests/test_gpu_dist.py, one process per GPU under torchrun:
the column-sharded int4dh weight-only linear (per-shard transforms, one
all-gather, the cross-shard stage) must agree with the single-GPU module
within the linear's bound, and the row-sharded h quantize must reassemble
the single-GPU codes bit for bit.  Prints OK on rank 0."""
import math
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import qtpytorch_b200 as mxb  # noqa: E402
from qtpytorch_b200 import ops  # noqa: E402
from qtpytorch_b200 import parallel as P  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl")
    dev = torch.device("cuda", torch.cuda.current_device())
    dt = mxb.get_mx_dtype("int4dh")
    K, N, M = 1024, 2048, 96
    g = torch.Generator().manual_seed(6)
    lin = torch.nn.Linear(K, N, bias=False)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
    ml = mxb.mx_linear.from_linear(lin.to(dev), dt, 128)
    x = torch.randn(M, K, generator=g).bfloat16().to(dev)
    sw = P.ShardedLinearWeight.from_module(ml, world, rank)
    assert sw.kron_split
    y = P.sharded_linear(x, sw)
    ref = ml(x)
    q = ml._mx_weight
    D = ops.dequantize(q._mx_packed, q._mx_scales, dt.base, q._mx_n, 128, (K, N)).double()
    bound = (x.double().abs() @ D.abs()).sum(dim=1, keepdim=True) / math.sqrt(N)
    err = (y.double() - ref.double()).abs()
    assert torch.all(err <= 2e-5 * bound), float((err / bound).max())
    # row-sharded quantize of an h tensor reassembles the full codes
    xr = torch.randn(40, 768, generator=g).to(dev)
    p, s, (b0, b1) = P.sharded_quantize(xr, dt, 128, world, rank)
    parts_p = [None] * world
    parts_s = [None] * world
    dist.all_gather_object(parts_p, p.cpu())
    dist.all_gather_object(parts_s, s.cpu())
    full = mxb.mx_tensor.quantize(xr, dt, 128)
    assert torch.equal(torch.cat(parts_p), full._mx_packed.cpu())
    assert torch.equal(torch.cat(parts_s), full._mx_scales.cpu())
    assert mxb._lib.load().mxb_device_error(1) == 0
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("OK")


if __name__ == "__main__":
    main()
