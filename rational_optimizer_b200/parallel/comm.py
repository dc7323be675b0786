"""In-kernel NVLink collectives (peer memory via CUDA IPC) - communicator factory.

``maybe_communicator(device)`` returns a communicator whose
``all_reduce_mean_(flat)`` runs the sm_100a peer-memory all-reduce when the
extension provides it and every rank can map its peers' buffers; otherwise
``None`` (callers then use NCCL through torch.distributed).
"""
from __future__ import annotations

from .. import _ext


def maybe_communicator(device, numel, group=None):
    if not _ext.available() or not hasattr(_ext.ext(), "comm_allreduce_f32"):
        return None
    from .p2p import P2PCommunicator
    return P2PCommunicator.create(device, numel, group=group)
