"""torchrun worker: data-parallel training paths agree across ranks and with each other.

Runs a 4-layer GRAIN+TILLER model for 10 steps per configuration: gradient
all-reduce during backward (per-layer buckets) or after it, TILLER sharded by
layer (deferred weight broadcasts) or replicated, one or two micro-batches;
then Muon replicated against Muon layer-sharded (reduce-to-owner gradients,
owner update, peer-memory weight pull), eager and graphed.
Every configuration must leave bitwise-identical replicas on all ranks, the
fully overlapped/sharded run must follow the plain run's loss curve, and the
same run with its forward/backward/reduction replayed from a CUDA graph must
reproduce it bit for bit.
"""
import os
import sys
from types import SimpleNamespace

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from rational_optimizer_b200.models.transformer import CausalTransformer, preset  # noqa: E402
from rational_optimizer_b200.optim.composite import configure_optimizer  # noqa: E402
from rational_optimizer_b200.parallel import param_ready  # noqa: E402
from rational_optimizer_b200.parallel.dist import setup_distributed  # noqa: E402
from rational_optimizer_b200.parallel.grad_sync import GradientSynchronizer  # noqa: E402
from rational_optimizer_b200.train.engine import TrainEngine  # noqa: E402
from rational_optimizer_b200.train.integrity import model_state_sha256  # noqa: E402


def run(info, *, overlap, shard, accum, graph=False, transport="nccl", weights="nccl", optimizer="tiller_v1",
        fused=False):
    os.environ["RO_FUSED_WGRAD_SEND"] = "1" if fused else "0"
    os.environ["RO_TILLER_SHARD"] = "1" if shard else "0"
    os.environ["RO_MUON_SHARD"] = "1" if shard else "0"
    os.environ["RO_WEIGHT_TRANSPORT"] = weights
    os.environ["RO_CUDA_GRAPH"] = "1" if graph else "0"
    torch.manual_seed(0)
    args = preset("18l_1024d", layers=4, seq_len=256, activation="grain")
    model = CausalTransformer(args, 50304).cuda()
    ns = SimpleNamespace(optimizer=optimizer, lr=3e-4, weight_decay=0.1, beta1=0.9, beta2=0.95, eps=1e-8,
                         muon_momentum=0.95, muon_ns_steps=5, muon_adjust_lr_fn="match_rms_adamw",
                         grad_accum=accum, layers=4, steps=100)
    opt = configure_optimizer(model, ns)
    if transport.startswith("owner"):
        from rational_optimizer_b200.optim.composite import owner_layers
        layers, owner_of = owner_layers(opt)
        sync = GradientSynchronizer(model, transport=transport, owner_layers=layers, layer_owner=owner_of)
        assert sync.transport == (transport if transport in ("owner-bf16", "owner-int8", "owner-ce")
                                  else "owner-f32")
        assert sync.fused_wgrad == fused
    else:
        sync = GradientSynchronizer(model, transport="nccl", overlap=overlap)
        assert sync.transport == ("nccl-overlap" if overlap else "nccl")
    eng = TrainEngine(model, opt, grad_clip=1.0, grad_accum=accum, synchronizer=sync)
    gen = torch.Generator().manual_seed(100 + info.rank)
    losses = []
    for _ in range(10):
        batches = []
        for _ in range(accum):
            x = torch.randint(0, 50304, (4 // accum, 257), generator=gen).cuda()
            batches.append((x[:, :-1], x[:, 1:]))
        losses.append(eng.step(batches, lr=3e-4))
    param_ready.wait_all()
    torch.cuda.synchronize()
    if sync.owner is not None:
        sync.owner.check()
    return [float(v) for v in losses], model_state_sha256(model)


def main():
    info = setup_distributed(timeout_s=120)
    configs = [dict(overlap=False, shard=False, accum=1), dict(overlap=True, shard=False, accum=1),
               dict(overlap=False, shard=True, accum=1), dict(overlap=True, shard=True, accum=1),
               dict(overlap=True, shard=True, accum=2), dict(overlap=True, shard=True, accum=1, graph=True),
               dict(overlap=False, shard=True, accum=1, transport="owner"),
               dict(overlap=False, shard=True, accum=1, transport="owner", graph=True),
               dict(overlap=False, shard=True, accum=1, transport="owner-bf16"),
               dict(overlap=False, shard=True, accum=1, transport="owner", weights="p2p"),
               dict(overlap=False, shard=True, accum=1, transport="owner", weights="p2p", graph=True),
               dict(overlap=True, shard=False, accum=1, optimizer="muon"),
               dict(overlap=False, shard=True, accum=1, transport="owner", weights="p2p", optimizer="muon"),
               dict(overlap=False, shard=True, accum=1, transport="owner", weights="p2p", graph=True,
                    optimizer="muon"),
               dict(overlap=False, shard=True, accum=1, transport="owner-int8", weights="p2p"),
               dict(overlap=False, shard=True, accum=1, transport="owner", weights="p2p", fused=True),
               dict(overlap=False, shard=True, accum=1, transport="owner", weights="p2p", fused=True, graph=True),
               dict(overlap=False, shard=True, accum=2, transport="owner", weights="p2p", fused=True),
               dict(overlap=False, shard=True, accum=1, transport="owner-ce"),
               dict(overlap=False, shard=True, accum=1, transport="owner-ce", graph=True)]
    runs = [run(info, **c) for c in configs]
    digests = [None] * info.world_size
    dist.all_gather_object(digests, [r[1] for r in runs])
    if info.rank == 0:
        equal = [len({d[k] for d in digests}) == 1 for k in range(len(configs))]
        for c, e, r in zip(configs, equal, runs):
            print("config", c, "replicas equal", e, "final loss", r[0][-1], flush=True)
        assert all(equal), equal
        rel = max(abs(x - y) / abs(y) for x, y in zip(runs[3][0], runs[0][0]))
        assert rel < 1e-2, (runs[3][0], runs[0][0])
        # the captured forward/backward/reduction replays the overlapped run exactly
        assert runs[5][0] == runs[3][0] and digests[0][5] == digests[0][3], (runs[5][0], runs[3][0])
        # reduce-to-owner (fp32 transport) follows the all-reduce runs; its graph replays it exactly;
        # bf16 transport stays close
        rel_owner = max(abs(x - y) / abs(y) for x, y in zip(runs[6][0], runs[0][0]))
        assert rel_owner < 1e-2, (runs[6][0], runs[0][0])
        assert runs[7][0] == runs[6][0] and digests[0][7] == digests[0][6], (runs[7][0], runs[6][0])
        rel_bf16 = max(abs(x - y) / abs(y) for x, y in zip(runs[8][0], runs[0][0]))
        assert rel_bf16 < 2e-2, (runs[8][0], runs[0][0])
        print("OWNER_OK max rel loss diff f32", rel_owner, "bf16", rel_bf16, flush=True)
        # weights pulled from their owners over peer memory: the same numbers as the
        # NCCL broadcasts, eagerly and from the step graph
        assert runs[9][0] == runs[6][0] and digests[0][9] == digests[0][6], (runs[9][0], runs[6][0])
        assert runs[10][0] == runs[6][0] and digests[0][10] == digests[0][6], (runs[10][0], runs[6][0])
        print("PULL_OK", flush=True)
        # layer-sharded Muon (reduce-to-owner, owner update, weight pull) follows the
        # replicated Muon; its graphed forward/backward replays it exactly
        rel_muon = max(abs(x - y) / abs(y) for x, y in zip(runs[12][0], runs[11][0]))
        assert rel_muon < 1e-2, (runs[12][0], runs[11][0])
        assert runs[13][0] == runs[12][0] and digests[0][13] == digests[0][12], (runs[13][0], runs[12][0])
        print("MUON_SHARD_OK max rel loss diff", rel_muon, flush=True)
        # int8 gradients with per-256 fp32 scales stay close to the fp32 transport
        rel_i8 = max(abs(x - y) / abs(y) for x, y in zip(runs[14][0], runs[0][0]))
        assert rel_i8 < 3e-2, (runs[14][0], runs[0][0])
        print("INT8_OK max rel loss diff", rel_i8, flush=True)
        # weight-gradient GEMMs storing their tiles straight into the owners' slots
        rel_fused = max(abs(x - y) / abs(y) for x, y in zip(runs[15][0], runs[9][0]))
        assert rel_fused < 1e-2, (runs[15][0], runs[9][0])
        assert runs[16][0] == runs[15][0] and digests[0][16] == digests[0][15], (runs[16][0], runs[15][0])
        rel_fused2 = max(abs(x - y) / abs(y) for x, y in zip(runs[17][0], runs[4][0]))
        assert rel_fused2 < 1e-2, (runs[17][0], runs[4][0])
        print("FUSED_WGRAD_OK max rel loss diff", rel_fused, rel_fused2, flush=True)
        # fp32 sends by copy engines deliver the same bytes as the send kernels
        assert runs[18][0] == runs[6][0] and digests[0][18] == digests[0][6], (runs[18][0], runs[6][0])
        assert runs[19][0] == runs[6][0] and digests[0][19] == digests[0][6], (runs[19][0], runs[6][0])
        print("COPY_ENGINE_OK", flush=True)
        print("TRAIN_OK", info.world_size, "max rel loss diff", rel, flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
