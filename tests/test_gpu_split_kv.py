"""GPU parity of the split-KV decode pieces (the 1M-token configuration):
sharded router (per-shard top-M keys + merge) against the whole-row router,
bit for bit, and sharded attention (owned slots per shard, window on its
owner, log-sum-exp merge) against one attention call over all shards' data.
The shards run one after another on one GPU; the all-gather is a stack."""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from srswa import ops  # noqa: E402
from srswa.split_kv import ShardPlan, SplitKVDecode  # noqa: E402

RP = dict(block_size=64, local_blocks=8, topk=8, topm=16, idx_scale=128 / math.sqrt(128), floor=1e-4, sigma=1.0)


def _bounds(nblk, nshard):
    plan = [ShardPlan(nblk, nshard, r, nblk) for r in range(nshard)]
    return [p.bounds(p.rank) for p in plan]


@pytest.mark.parametrize("nblk,nshard,paged", [(16384, 8, False), (16384, 1, False), (5000, 3, True),
                                               (700, 4, True), (130, 2, False)])
def test_sharded_route_equals_whole_row(cuda, nblk, nshard, paged):
    g = torch.Generator(device="cuda").manual_seed(nblk + nshard)
    d, N = 128, 4
    kbar = torch.randn(1, nblk, d, device=cuda, generator=g)
    idx_q = torch.randn(N, d, device=cuda, generator=g).to(torch.bfloat16)
    S = nblk * 64
    q_pos = torch.tensor([S - 1, S - 2, S // 2 + 7, 3 * 64 + 5], device=cuda, dtype=torch.int64)
    if paged:
        perm = torch.randperm(nblk, device=cuda, generator=g).to(torch.int32)
        cache = torch.empty(nblk, d, device=cuda)
        cache[perm.long()] = kbar[0]
        table = perm[None].repeat(1, 1)
        full = ops.route(idx_q, cache, block_table=table, q_pos=q_pos, rows_per_seq=N,
                         want=("topi64", "bias", "valid"), **RP)
    else:
        full = ops.route(idx_q, kbar, q_pos=q_pos, rows_per_seq=N, want=("topi64", "bias", "valid"), **RP)
    keys = []
    for lo, hi in _bounds(nblk, nshard):
        if paged:
            keys.append(ops.route_shard_keys(idx_q, cache, block_offset=lo, nblk_local=hi - lo, nblk_total=nblk,
                                             q_pos=q_pos, rows_per_seq=N, block_table=table, **RP))
        else:
            keys.append(ops.route_shard_keys(idx_q, kbar[:, lo:hi], block_offset=lo, nblk_local=hi - lo,
                                             nblk_total=nblk, q_pos=q_pos, rows_per_seq=N, **RP))
    p = {k: v for k, v in RP.items() if k not in ("block_size", "local_blocks")}
    merged = ops.route_merge_keys(torch.stack(keys), nblk_total=nblk, want=("topi64", "bias", "valid"), **p)
    torch.cuda.synchronize()
    assert torch.equal(merged["topi64"], full["topi64"])
    assert torch.equal(merged["valid"], full["valid"])
    if nblk >= 512:
        # the whole-row router takes the same score arithmetic here (wide rows)
        assert torch.equal(merged["bias"], full["bias"])
    else:
        # rows under 512 blocks: the whole-row router is the one-warp-per-row
        # kernel, whose dot products round differently in the last bit
        torch.testing.assert_close(merged["bias"], full["bias"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("nblk,exchange", [(16384, None), (16384, "flag"), (16384, "ll"), (100, None),
                                            (100, "flag"), (100, "ll"), (3000, "flag"), (3000, "ll")])
def test_shard_select_equals_two_stages(cuda, nblk, exchange):
    """srswa_route_shard_select (one launch: shard keys, optional exchange of
    one rank, merge and epilogue) = shard keys + merge, bit for bit."""
    from srswa.peer import PeerAllGather
    g = torch.Generator(device="cuda").manual_seed(nblk + 3)
    d, N = 128, 3
    kbar = torch.randn(1, nblk, d, device=cuda, generator=g)
    idx_q = torch.randn(N, d, device=cuda, generator=g).to(torch.bfloat16)
    S = nblk * 64
    q_pos = torch.tensor([S - 1, S // 3, 9 * 64 + 1], device=cuda, dtype=torch.int64)
    p = {k: v for k, v in RP.items() if k not in ("block_size", "local_blocks")}
    own = (nblk // 4, nblk // 2)
    ex = None if exchange is None else PeerAllGather(N * RP["topm"] * 16, None, cuda, ll=exchange == "ll")
    for rep in range(3):   # the exchange's epochs advance from call to call
        keys = ops.route_shard_keys(idx_q, kbar, block_offset=0, nblk_local=nblk, nblk_total=nblk, q_pos=q_pos,
                                    rows_per_seq=N, **RP)
        two = ops.route_merge_keys(keys[None], nblk_total=nblk, own=own,
                                   want=("topi64", "topi32", "bias", "valid"), **p)
        one = ops.route_shard_select(idx_q, kbar, block_offset=0, nblk_local=nblk, nblk_total=nblk, q_pos=q_pos,
                                     rows_per_seq=N, own=own, want=("topi64", "topi32", "bias", "valid"),
                                     exchange=None if ex is None else ex.peer, **RP)
        torch.cuda.synchronize()
        for name in ("topi64", "topi32", "bias", "valid", "topi32_own"):
            assert torch.equal(one[name], two[name]), name
    if ex is not None:
        ex.check()
        ex.close()


def test_sharded_attend_equals_single_call(cuda):
    g = torch.Generator(device="cuda").manual_seed(11)
    nblk, BS, H, Hkv, D, d, nshard = 4096, 64, 10, 10, 128, 128, 4
    S = nblk * BS - 37                      # last block partly filled
    P = nblk
    k_cache = (torch.randn(P, BS, Hkv, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    v_cache = (torch.randn(P, BS, Hkv, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    table = torch.randperm(P, device=cuda, generator=g).to(torch.int32)[None]
    kbar = torch.randn(P, d, device=cuda, generator=g)
    N = 2                                    # two query rows of the sequence (decode_query_len 2)
    q = (torch.randn(N, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    idx_q = torch.randn(N, d, device=cuda, generator=g).to(torch.bfloat16)
    q_pos = torch.tensor([S - 2, S - 1], device=cuda, dtype=torch.int64)
    full_sel = ops.route(idx_q, kbar, block_table=table, q_pos=q_pos, rows_per_seq=N, want=("topi32", "bias"),
                         **RP)
    ref = torch.empty(N, H, D, device=cuda)
    ops.decode_attend(q, k_cache, v_cache, full_sel["topi32"], full_sel["bias"], block_size=BS,
                      local_blocks=RP["local_blocks"], sm_scale=1 / math.sqrt(D), out=ref, block_table=table,
                      q_pos=q_pos, rows_per_req=N)
    parts, lses = [], []
    for r in range(nshard):
        dec = SplitKVDecode(nblk_total=nblk, nblk_filled=nblk, sm_scale=1 / math.sqrt(D), rank=r, world=nshard,
                            **RP)
        lo, hi = dec.plan.lo, dec.plan.hi
        layer = dict(kbar=kbar, kbar_table=table, k_cache=k_cache, v_cache=v_cache, block_table=table)
        be = dec.backend
        keys = torch.stack([ops.route_shard_keys(idx_q, kbar, block_offset=a, nblk_local=b - a, nblk_total=nblk,
                                                 q_pos=q_pos, rows_per_seq=N, block_table=table, **RP)
                            for a, b in (ShardPlan(nblk, nshard, j, nblk).bounds(j) for j in range(nshard))])
        sel = be.merge_keys(keys, dec.plan, dec.rp)
        assert torch.equal(torch.where(sel["topi32"] >= 0, sel["topi32"], -1), full_sel["topi32"])
        own = sel["topi32_own"]
        assert bool(((own == -1) | ((own >= lo) & (own < hi))).all())
        owner = dec.window_owner(S - 1, S - 2)
        o, lse = be.attend(q, layer, own, sel["bias"], q_pos, block_size=BS, local_blocks=RP["local_blocks"],
                           sm_scale=1 / math.sqrt(D), skip_local=(r != owner))
        parts.append(o)
        lses.append(lse)
    out = ops.lse_merge(torch.stack(parts), torch.stack(lses))[0]
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), rtol=1e-4, atol=1e-5)


def test_split_decode_world1_matches_plain_path(cuda):
    """SplitKVDecode with one rank = route + attend of the whole sequence."""
    g = torch.Generator(device="cuda").manual_seed(5)
    nblk, BS, H, D, d = 1024, 64, 10, 128, 128
    k_cache = (torch.randn(nblk, BS, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    v_cache = (torch.randn(nblk, BS, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    table = torch.arange(nblk, device=cuda, dtype=torch.int32)[None]
    kbar = torch.randn(1, nblk, d, device=cuda, generator=g)
    q = (torch.randn(1, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    idx_q = torch.randn(1, d, device=cuda, generator=g).to(torch.bfloat16)
    S = nblk * BS
    q_pos = torch.tensor([S - 1], device=cuda, dtype=torch.int64)
    dec = SplitKVDecode(nblk_total=nblk, nblk_filled=nblk, sm_scale=1 / math.sqrt(D), **RP)
    out = dec.step(q, idx_q, q_pos, dict(kbar=kbar, k_cache=k_cache, v_cache=v_cache, block_table=table),
                   p_range=(S - 1, S - 1), out_dtype=torch.float32)
    sel = ops.route(idx_q, kbar, q_pos=q_pos, want=("topi32", "bias"), **RP)
    ref = torch.empty(1, H, D, device=cuda)
    ops.decode_attend(q, k_cache, v_cache, sel["topi32"], sel["bias"], block_size=BS,
                      local_blocks=RP["local_blocks"], sm_scale=1 / math.sqrt(D), out=ref, block_table=table,
                      q_pos=q_pos, rows_per_req=1)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), rtol=1e-5, atol=1e-6)
