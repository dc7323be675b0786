"""Transport smoke test before admitting a node (behaviour of
experiments/protocol/smoke_nccl.py:1-44, extended to this package's peer-memory paths).

Run once per node, one process per GPU:

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m rational_optimizer_b200.protocol.smoke

Checks, with exact expected values (every rank fills with rank + 1):

* NCCL broadcast and all-reduce of a 256 MiB fp32 buffer;
* the reduce-to-owner kernels (:class:`~rational_optimizer_b200.parallel.owner_reduce.OwnerReduce`):
  every rank owns one segment, receives the others' copies over NVLink peer
  memory and must hold the mean;
* the owner weight pull (:class:`~rational_optimizer_b200.parallel.owner_gather.OwnerGather`):
  after a publish every rank must hold every owner's values.

Rank 0 prints one JSON line with the measured bus bandwidths (device time,
max over ranks) and ``passed``; any mismatch raises.  Every collective wait
inside the package's kernels is bounded (``RO_COMM_TIMEOUT_S``).
"""
from __future__ import annotations

import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

ELEMS = 64 * 1024 * 1024  # 256 MiB of fp32


def _time(fn, device, reps=3):
    fn()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    torch.cuda.synchronize(device)
    t = torch.tensor([start.elapsed_time(end) / reps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def nccl_checks(rank, world, device):
    value = torch.full((ELEMS,), float(rank + 1), device=device)
    dist.broadcast(value, src=0)
    if value[0].item() != 1.0 or value[-1].item() != 1.0:
        raise RuntimeError("NCCL broadcast returned the wrong value")
    value.fill_(float(rank + 1))
    dist.all_reduce(value)
    if value[0].item() != world * (world + 1) / 2:
        raise RuntimeError("NCCL all-reduce returned the wrong value")
    ms = _time(lambda: dist.all_reduce(value), device)
    return {"nccl_allreduce_ms": ms, "nccl_allreduce_busbw_gbs": 2 * (world - 1) / world * value.numel() * 4 / ms / 1e6}


def owner_checks(rank, world, device):
    from ..parallel.owner_reduce import OwnerReduce
    from ..parallel import owner_gather
    seg = ELEMS // world // 8 * 8
    flat = torch.full((seg * world,), float(rank + 1), device=device)
    red = OwnerReduce(flat, [(r * seg, seg) for r in range(world)], list(range(world)))
    red.begin()
    for layer in range(world):
        red.send(layer)
    red.reduce()
    torch.cuda.synchronize(device)
    red.check()
    mine = flat[rank * seg:(rank + 1) * seg]
    want = (world + 1) / 2
    if not torch.all(mine == want):
        raise RuntimeError(f"reduce-to-owner: rank {rank} holds {mine[0].item()}, expected {want}")

    def once():
        flat.fill_(float(rank + 1))
        red.begin()
        for layer in range(world):
            red.send(layer)
        red.reduce()

    ms_red = _time(once, device)
    red.close()
    raw, weights = owner_gather.shared_buffer(seg * world, device)
    weights.copy_(torch.arange(world, device=device, dtype=torch.float32).repeat_interleave(seg) + 1.0)
    weights[rank * seg:(rank + 1) * seg] = float(rank + 1)
    gather = owner_gather.OwnerGather(raw, weights, [(r * seg, (r + 1) * seg) for r in range(world)],
                                      [[] for _ in range(world)])
    weights.zero_()
    weights[rank * seg:(rank + 1) * seg] = float(rank + 1)
    gather.publish()
    gather.pending = False
    gather.pull()
    torch.cuda.current_stream(device).wait_stream(owner_gather.param_ready.side_stream(device))
    torch.cuda.synchronize(device)
    gather.check()
    expect = torch.arange(world, device=device, dtype=torch.float32).repeat_interleave(seg) + 1.0
    if not torch.equal(weights, expect):
        raise RuntimeError(f"weight pull: rank {rank} holds the wrong values")

    def pull_once():
        gather.publish()
        gather.pending = False
        gather.pull()
        torch.cuda.current_stream(device).wait_stream(owner_gather.param_ready.side_stream(device))

    ms_pull = _time(pull_once, device)
    gather.close()
    moved = (world - 1) * seg * 4  # bytes each rank receives
    return {"owner_reduce_ms": ms_red, "owner_reduce_ingress_gbs": moved / ms_red / 1e6,
            "owner_pull_ms": ms_pull, "owner_pull_ingress_gbs": moved / ms_pull / 1e6}


def main() -> int:
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    out = {"world_size": world, "bytes_per_collective": ELEMS * 4,
           "nccl_nvls_enable": os.environ.get("NCCL_NVLS_ENABLE"),
           "nccl_p2p_disable": os.environ.get("NCCL_P2P_DISABLE")}
    out.update(nccl_checks(rank, world, device))
    if world > 1:
        out.update(owner_checks(rank, world, device))
    dist.barrier()
    out["passed"] = True
    if rank == 0:
        print(json.dumps(out, sort_keys=True), flush=True)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
