"""Transport smoke test before admitting a node (behaviour of
experiments/protocol/smoke_nccl.py:1-44, extended to this package's peer-memory paths).

Run once per node, one process per GPU:

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m rational_optimizer_b200.protocol.smoke

Checks, with exact expected values (every rank fills with rank + 1):

* NCCL broadcast and all-reduce of a 256 MiB fp32 buffer;
* the reduce-to-owner kernels (:class:`~rational_optimizer_b200.parallel.owner_reduce.OwnerReduce`)
  in each transport format (fp32, bf16, int8 with per-256 scales): every
  rank owns one segment, receives the others' copies over NVLink peer memory
  and must hold the mean (exactly; int8 to one rounding of the scale);
* the owner weight pull (:class:`~rational_optimizer_b200.parallel.owner_gather.OwnerGather`):
  after a publish every rank must hold every owner's values.

Rank 0 prints one JSON line with the measured bandwidths (device time, max
over ranks): NCCL bus bandwidth, and for the peer-memory kernels the bytes
each rank receives per second and that figure as a fraction of the measured
770 GB/s per-direction NVLink peer-copy bandwidth; and ``passed``.  Any
mismatch raises.  Every collective wait
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


NVLINK_GBS = 770.0  # measured peer copy per direction per B200 on this class of node


def owner_checks(rank, world, device):
    from ..parallel import owner_gather
    from ..parallel.owner_reduce import OwnerReduce, slot_bytes
    seg = ELEMS // world // 256 * 256
    out = {}
    flat = torch.empty(seg * world, device=device)
    from ..parallel.owner_reduce import SEND_CTAS
    # the training configuration (few send CTAs, beside the backward's kernels)
    # and a wide one (about one CTA per SM), which bounds what the kernels reach
    # and the copy-engine fp32 send (no send CTAs)
    for transport, ctas, ce in (("f32", SEND_CTAS, False), ("bf16", SEND_CTAS, False),
                                ("int8", SEND_CTAS, False), ("f32", 128, False), ("bf16", 128, False),
                                ("int8", 128, False), ("f32", SEND_CTAS, True)):
        red = OwnerReduce(flat, [(r * seg, seg) for r in range(world)], list(range(world)), transport=transport,
                          send_ctas=ctas, copy_engine=ce)
        name = "f32_ce" if ce else (transport if ctas == SEND_CTAS else f"{transport}_ctas{ctas}")

        def once():
            flat.fill_(float(rank + 1))
            red.begin()
            for layer in range(world):
                red.send(layer)
            red.reduce()

        once()
        torch.cuda.synchronize(device)
        red.check()
        mine = flat[rank * seg:(rank + 1) * seg]
        want = torch.full_like(mine, (world + 1) / 2)
        if transport == "int8":  # one rounding of the per-block scale
            ok = torch.allclose(mine, want, rtol=1e-5, atol=0.0)
        else:
            ok = torch.equal(mine, want)
        if not ok:
            raise RuntimeError(f"reduce-to-owner ({name}): rank {rank} holds {mine[0].item()}, "
                               f"expected {(world + 1) / 2}")
        ms = _time(once, device)
        red.close()
        moved = (world - 1) * slot_bytes(seg, transport)  # bytes each rank receives (and sends)
        out[f"owner_reduce_{name}_ms"] = ms
        out[f"owner_reduce_{name}_ingress_gbs"] = moved / ms / 1e6
        out[f"owner_reduce_{name}_frac_nvlink"] = moved / ms / 1e6 / NVLINK_GBS
    out["send_ctas_training"] = SEND_CTAS
    raw, weights = owner_gather.shared_buffer(seg * world, device)
    gather = owner_gather.OwnerGather(raw, weights, [(r * seg, (r + 1) * seg) for r in range(world)],
                                      [[] for _ in range(world)])
    weights.zero_()
    weights[rank * seg:(rank + 1) * seg] = float(rank + 1)

    def pull_once():
        gather.publish()
        gather.pending = False
        gather.pull()
        torch.cuda.current_stream(device).wait_stream(owner_gather.param_ready.side_stream(device))

    pull_once()
    torch.cuda.synchronize(device)
    gather.check()
    expect = torch.arange(world, device=device, dtype=torch.float32).repeat_interleave(seg) + 1.0
    if not torch.equal(weights, expect):
        raise RuntimeError(f"weight pull: rank {rank} holds the wrong values")
    ms_pull = _time(pull_once, device)
    gather.close()
    moved = (world - 1) * seg * 4
    out.update(owner_pull_ms=ms_pull, owner_pull_ingress_gbs=moved / ms_pull / 1e6,
               owner_pull_frac_nvlink=moved / ms_pull / 1e6 / NVLINK_GBS)
    return out


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
