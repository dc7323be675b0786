"""Bounded waits of the peer-memory collectives (single GPU: a flag nobody sets)."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

from rational_optimizer_b200 import _ext


def test_wait_on_flag_nobody_sets_times_out_and_gpu_stays_usable():
    C = _ext.ext()
    dev = torch.cuda.current_device()
    buf = C.comm_alloc(1 << 16, dev)
    own_flags = C.comm_alloc(48 * 4, dev)
    fake_peer_flags = C.comm_alloc(48 * 4, dev)   # the "peer" never writes here
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    C.comm_wait_only([buf.data_ptr(), buf.data_ptr()], [own_flags.data_ptr(), fake_peer_flags.data_ptr()],
                     0, 1, err, int(50e6))
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert int(err.item()) == 3          # the "gathered" phase wait gave up
    assert elapsed < 5.0
    x = torch.randn(1000, device="cuda")  # context still healthy
    assert torch.isfinite(x.sum()).item()


def test_ipc_handle_roundtrip_in_process():
    C = _ext.ext()
    dev = torch.cuda.current_device()
    buf = C.comm_alloc(4096, dev)
    h = C.comm_handle(buf)
    assert isinstance(h, bytes) and len(h) == 64
