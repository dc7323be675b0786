"""torchrun worker (gloo, CPU): ownership and state replication of the layer-sharded Muon."""
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from rational_optimizer_b200.optim.muon import Muon, MuonShard  # noqa: E402
from rational_optimizer_b200.optim.tiller import shard_bounds  # noqa: E402


def main():
    dist.init_process_group("gloo")
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.manual_seed(0)
    layers = 5
    named = [(f"layers.{l}.{k}.weight", torch.nn.Parameter(torch.randn(8, 4))) for l in range(layers)
             for k in ("qkv", "out")]
    muon = Muon(named, lr=0.02)
    per_layer = [[p for n, p in named if n.startswith(f"layers.{l}.")] for l in range(layers)]
    shard = MuonShard(per_layer, world, rank)
    lo, hi = shard_bounds(layers, rank, world)
    assert shard.owned == {id(p) for l in range(lo, hi) for p in per_layer[l]}
    assert [shard.owner(l) for l in range(layers)] == [r for r in range(world)
                                                      for _ in range(*shard_bounds(layers, r, world))]
    shard.replicate_state(muon)  # before any step: nothing to replicate
    assert all("momentum_buffer" not in muon.state[p] for ps in per_layer for p in ps)
    for l in range(lo, hi):
        for p in per_layer[l]:
            muon.state[p]["momentum_buffer"] = torch.full_like(p, float(100 * rank + l))
    shard.replicate_state(muon)
    for l in range(layers):
        for p in per_layer[l]:
            want = float(100 * shard.owner(l) + l)
            assert torch.equal(muon.state[p]["momentum_buffer"], torch.full_like(p, want)), (rank, l)
    if rank == 0:
        print("MUON_STATE_OK", world, flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
