"""Worker of tests/test_gpu_dist.py, one process per GPU under torchrun:
the column-sharded int8 matmul with the output gather fused into the
kernel (peer stores), ordered by the in-kernel barrier or by an all-reduce
after the launch, or pulled by every rank after its local matmul, must
equal, bit for bit, the NCCL-gather version and the single-GPU matmul.  Prints OK on rank 0."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import qtpytorch_b200 as mxb  # noqa: E402
from qtpytorch_b200 import parallel as P  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl")
    dev = torch.device("cuda", torch.cuda.current_device())
    M, K, N = 256, 512, 128 * 3 * world + (128 if world > 1 else 0)  # uneven shards
    g = torch.Generator().manual_seed(5)
    a = torch.randn(M, K, generator=g).to(dev)
    b = torch.randn(K, N, generator=g).to(dev)
    qa = mxb.mx_tensor.quantize(a, mxb.int8d, 128)
    qb = mxb.mx_tensor.quantize(b, mxb.int8d, 128)
    w = P.ShardedQGemmWeight(qb, world, rank)
    peers = P.PeerOutputs(M, N, 128, world, rank, device=dev)
    ref_gather = P.sharded_qgemm(qa, w)
    full = qa @ qb
    for it in range(9):  # both output sets, reuse, both barrier kinds, then pulled
        if it < 6:
            c = P.sharded_qgemm_fused(qa, w, peers, in_kernel_barrier=it < 4)
        else:
            c = P.sharded_qgemm_pull(qa, w, peers)
        torch.cuda.synchronize()
        assert torch.equal(c._mx_packed, ref_gather._mx_packed.view(torch.int32)), it
        assert torch.equal(c._mx_scales, ref_gather._mx_scales), it
        assert torch.equal(c._mx_packed, full._mx_packed.view(torch.int32)), it
        assert torch.equal(c._mx_scales, full._mx_scales), it
    assert mxb._lib.load().mxb_device_error(1) == 0
    dist.barrier()
    peers.close()
    dist.destroy_process_group()
    if rank == 0:
        print("OK")


if __name__ == "__main__":
    main()
