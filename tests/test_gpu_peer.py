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


@pytest.mark.parametrize("ll", [False, True])
@pytest.mark.parametrize("nsplit", [0, 1, 4])
def test_attend_push_world1_equals_plain(cuda, nsplit, ll):
    """srswa_decode_attend_push with a one-rank exchange: the partial o / lse
    land in the rank's own slot, equal to the plain attend's, and the
    log-sum-exp merge that waits on the exchange returns the same output;
    three calls in a row (the exchange's epochs advance)."""
    import math
    from srswa import ops
    g = torch.Generator(device=cuda).manual_seed(3)
    N, H, Hkv, D, BS, L_, K, nblk = 2, 10, 10, 128, 64, 8, 8, 512
    kc = torch.randn(nblk, BS, Hkv, D, device=cuda, generator=g).to(torch.bfloat16)
    vc = torch.randn(nblk, BS, Hkv, D, device=cuda, generator=g).to(torch.bfloat16)
    table = torch.randperm(nblk, device=cuda, generator=g).to(torch.int32)[None]
    kbar = torch.randn(nblk, 128, device=cuda, generator=g)
    q = torch.randn(N, H, D, device=cuda, generator=g).to(torch.bfloat16)
    iq = torch.randn(N, 128, device=cuda, generator=g).to(torch.bfloat16)
    S = nblk * BS - 5
    q_pos = torch.tensor([S - 2, S - 1], device=cuda, dtype=torch.int64)
    sel = ops.route(iq, kbar, block_table=table, q_pos=q_pos, rows_per_seq=N, want=("topi32", "bias"),
                    block_size=BS, local_blocks=L_, topk=K, topm=16, idx_scale=128 / math.sqrt(128), floor=1e-4,
                    sigma=1.0)
    kw = dict(block_size=BS, local_blocks=L_, sm_scale=1 / math.sqrt(D), block_table=table, q_pos=q_pos,
              rows_per_req=N, lse=True, nsplit=nsplit)
    ref_o, ref_l = ops.decode_attend(q, kc, vc, sel["topi32"], sel["bias"], out=torch.empty(N, H, D, device=cuda),
                                     **kw)
    n4 = -(-(N * H * D + N * H) // 4) * 4
    ex = PeerAllGather(n4 * 4 * (2 if ll else 1), ll=ll)
    for rep in range(3):
        # flag protocol: the local copy is this rank's own slot; LL: any buffer
        buf = torch.empty(n4, device=cuda) if ll else ex.own_slot((n4,), torch.float32)
        buf.zero_()
        o, lse = buf[:N * H * D].view(N, H, D), buf[N * H * D:N * H * D + N * H].view(N, H)
        ops.decode_attend(q, kc, vc, sel["topi32"], sel["bias"], out=o, lse_out=lse, push=ex.peer, **kw)
        if ll:
            merged = ops.lse_merge_exchange(ex.peer, 1, N, H, D, cuda)[0]
            # the attend that also exchanges and merges (one launch)
            fused = ops.decode_attend(q, kc, vc, sel["topi32"], sel["bias"], out=torch.empty_like(o),
                                      lse_out=torch.empty_like(lse), push=ex.peer,
                                      merged_out=torch.empty(N, H, D, device=cuda), **kw)
            torch.cuda.synchronize()
            assert torch.equal(fused, ref_o)
        else:
            parts = ex.slots((n4,), torch.float32)
            merged = ops.lse_merge(parts[:, :N * H * D].view(1, N, H, D),
                                   parts[:, N * H * D:N * H * D + N * H].view(1, N, H),
                                   out_dtype=torch.float32, wait=ex.peer)[0]
        torch.cuda.synchronize()
        assert torch.equal(o, ref_o) and torch.equal(lse, ref_l)
        torch.testing.assert_close(merged, ref_o, rtol=1e-6, atol=1e-6)
    assert int(ex.counter.item()) == (6 if ll else 3)   # ll: two exchanges per repetition
    ex.check()
    ex.close()
