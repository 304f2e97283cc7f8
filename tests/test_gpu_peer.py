"""The peer-memory all-gather on one GPU: with world = 1 it gathers the
payload into the rank's own slot; and its wait is bounded -- given a second
region that no rank ever writes (a peer that never arrives), the wait gives
up after its time limit, records code 501 in the status word and returns,
leaving the context usable.  No fault, no trap: the flag is simply never
set."""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

from srswa import _lib as L  # noqa: E402
from srswa.peer import PeerAllGather  # noqa: E402


def test_peer_allgather_world1(cuda):
    ex = PeerAllGather(4096)
    for step in range(3):
        x = torch.arange(512, device=cuda, dtype=torch.int64) * (step + 1)
        y = ex(x)
        torch.cuda.synchronize()
        assert y.shape == (1, 512) and torch.equal(y[0], x)
    assert int(ex.counter.item()) == 3
    ex.check()
    ex.close()


def test_peer_wait_expires_with_status(cuda):
    lib = L.lib()
    size = C.c_size_t(0)
    assert lib.srswa_peer_region_size(2, 256, C.byref(size)) == 0
    regs = []
    for _ in range(2):
        p = C.c_void_p()
        assert lib.srswa_peer_region_alloc(size.value, C.byref(p)) == 0
        regs.append(p.value)
    # rank 0 of a 2-rank group whose rank 1 never pushes: flag 1 of the own
    # region is never set, so the wait must expire (2 s) with code 501
    regions = torch.tensor(regs, dtype=torch.int64, device=cuda)
    counter = torch.zeros(1, dtype=torch.int64, device=cuda)
    tickets = torch.zeros(2, dtype=torch.int32, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    peer = L.Peer(regions.data_ptr(), regs[0], 256, 0, 2, counter.data_ptr(), tickets.data_ptr(), status.data_ptr())
    x = torch.ones(64, device=cuda, dtype=torch.int32)
    rc = lib.srswa_peer_allgather(x.data_ptr(), 256, C.byref(peer), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 501
    assert int(counter.item()) == 1           # the epoch still advanced
    y = torch.ones(8, device=cuda) * 2        # the context is still usable
    assert float(y.sum().item()) == 16.0
    for p in regs:
        assert lib.srswa_peer_region_free(C.c_void_p(p)) == 0
