"""torchrun worker for the multi-GPU peer-memory collective test."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from rational_optimizer_b200.parallel.dist import setup_distributed  # noqa: E402
from rational_optimizer_b200.parallel.p2p import Int8AllReduce, P2PCommunicator  # noqa: E402


def main():
    info = setup_distributed(timeout_s=60)
    rank, world, dev = info.rank, info.world_size, info.device
    n = 3_000_001
    comm = P2PCommunicator(dev, rank, world, 4 * n, timeout_s=10)
    flat = comm.float_view(n)
    for it in range(3):
        gen = torch.Generator(device="cuda").manual_seed(100 * it + rank)
        src = torch.randn(n, device=dev, generator=gen)
        flat.copy_(src)
        ref = src.clone()
        dist.all_reduce(ref)
        ref /= world
        comm.all_reduce_mean_(flat)
        torch.cuda.synchronize()
        comm.check()
        torch.testing.assert_close(flat, ref, rtol=1e-5, atol=1e-6)
        # replicas bitwise identical
        allv = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(allv, flat)
        for v in allv:
            assert torch.equal(v, allv[0])
    q = Int8AllReduce(dev, n)
    src = torch.randn(n, device=dev)
    out = torch.empty_like(src)
    q(src, out)
    torch.cuda.synchronize()
    q.comm.check()
    ref = src.clone()
    dist.all_reduce(ref)
    ref /= world
    rel = ((out - ref).norm() / ref.norm()).item()
    assert rel < 0.02, rel
    allv = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(allv, out)
    for v in allv:
        assert torch.equal(v, allv[0])
    comm.close()
    q.comm.close()
    dist.barrier()
    if rank == 0:
        print("COMM_OK", world, flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
