"""Host logic of the split-KV decode on CPU: two gloo ranks, each holding half
of the blocks of one sequence, run SplitKVDecode.step with a NumPy backend
that restates the kernels' contracts (packed keys, owned-slot attention with
log-sum-exp).  The combined output and the merged selection must equal the
oracle's whole-sequence decode (_block_scores_infer + _infer_route_select +
_decode_attend)."""

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import srswa_oracle as O

from srswa.split_kv import ShardPlan, SplitKVDecode

BS, L, K, M = 64, 2, 4, 8
H, HKV, D, DI = 2, 1, 32, 32
IDX_SCALE, FLOOR, SIGMA = 128 / math.sqrt(128), 1e-4, 1.0
SCALE = 1 / math.sqrt(D)


def _problem(seed, nblk_filled, extra_tokens):
    rng = np.random.default_rng(seed)
    S = nblk_filled * BS + extra_tokens
    k = O.bf16_round(rng.standard_normal((HKV, S, D)).astype(np.float32))
    v = O.bf16_round(rng.standard_normal((HKV, S, D)).astype(np.float32))
    idx_k = O.bf16_round(rng.standard_normal((S, DI)).astype(np.float32))
    q = O.bf16_round(rng.standard_normal((2, H, D)).astype(np.float32))
    idx_q = O.bf16_round(rng.standard_normal((2, DI)).astype(np.float32))
    q_pos = np.array([S - 2, S - 1], np.int64)
    return dict(S=S, k=k, v=v, idx_k=idx_k, q=q, idx_q=idx_q, q_pos=q_pos)


def _pack(x, blk, cand):
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    ordered = np.where(u & 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)
    lo = ((0x7FFFFFFF - np.asarray(blk, np.uint64)) << np.uint64(1)) | np.asarray(cand, np.uint64)
    return (ordered << np.uint64(32)) | lo


def _unpack(k):
    hi = (k >> np.uint64(32)).astype(np.uint32)
    u = np.where(hi & 0x80000000, hi & 0x7FFFFFFF, (~hi) & 0xFFFFFFFF).astype(np.uint32)
    lo = (k & np.uint64(0xFFFFFFFF)).astype(np.int64)
    return u.view(np.float32), 0x7FFFFFFF - (lo >> 1), (lo & 1).astype(bool)


def _topm_keys(keys, m):
    order = np.argsort(keys, axis=-1)[..., ::-1][..., :m]
    out = np.take_along_axis(keys, order, -1)
    if out.shape[-1] < m:
        out = np.concatenate([out, np.zeros(out.shape[:-1] + (m - out.shape[-1],), np.uint64)], -1)
    return out


class NumpyBackend:
    """Restatement of the kernels' contracts on this rank's shard."""

    def __init__(self, world):
        self.world = world

    def shard_keys(self, idx_q, layer, plan, q_pos, rp):
        lo, hi = plan.lo, plan.hi
        kb = np.zeros((plan.nblk_total, DI), np.float32)
        cv = np.zeros(plan.nblk_total, bool)
        kb[lo:hi] = layer["kbar"]
        cv[lo:hi] = layer["chunk_valid"]
        sc = O.block_scores_headcls(idx_q[None], kb[None], cv[None], q_pos[None], BS, L)[0][:, lo:hi]
        remote = sc > O.SCORE_NEG * np.float32(0.5)
        x = np.where(remote, sc * np.float32(IDX_SCALE), np.float32(O.ENTMAX_NEG)).astype(np.float32)
        keys = _pack(x, np.arange(lo, hi)[None].repeat(len(x), 0), remote)
        return torch.from_numpy(_topm_keys(keys, M).view(np.int64).copy())

    def merge_keys(self, keys, plan, rp):
        ks = keys.numpy().view(np.uint64).transpose(1, 0, 2).reshape(keys.shape[1], -1)
        top = _topm_keys(ks, M)
        x, blk, cand = _unpack(top)
        topi, bias = np.zeros((len(top), K), np.int64), np.zeros((len(top), K), np.float32)
        for n in range(len(top)):
            p = O.entmax15(x[n])
            vld = cand[n, :K]
            logp = np.log(np.maximum(p[:K], np.float32(FLOOR))).astype(np.float32)
            mu = logp[vld].mean() if vld.any() else np.float32(0)
            bias[n] = np.where(vld, (logp - mu) / np.float32(SIGMA), 0)
            topi[n] = np.where(vld, blk[n, :K], -1)
        own = np.where((topi >= plan.lo) & (topi < plan.hi), topi, -1)
        return dict(topi32=topi, bias=bias, topi32_own=own)

    def attend(self, q, layer, topi, bias, q_pos, *, block_size, local_blocks, sm_scale, skip_local,
               out_dtype=None):
        lo_tok = layer["tok0"]
        k, v = layer["k"], layer["v"]          # this shard's tokens [HKV, ntok, D]
        N = len(q_pos)
        o = np.zeros((N, H, D), np.float32)
        lse = np.full((N, H), -np.inf, np.float32)
        lw = local_blocks * block_size
        for n in range(N):
            p = int(q_pos[n])
            ls = max(p - lw + 1, 0)
            keys, add = [], []
            for s in range(topi.shape[1]):
                b = int(topi[n, s])
                if b < 0:
                    continue
                for j in range(b * block_size, min((b + 1) * block_size, ls, p + 1)):
                    keys.append(j)
                    add.append(bias[n, s])
            if not skip_local:
                for j in range(ls, p + 1):
                    keys.append(j)
                    add.append(0.0)
            if not keys:
                continue
            idx = np.array(keys) - lo_tok
            for h in range(H):
                hk = h // (H // HKV)
                s_ = k[hk, idx] @ q[n, h] * np.float32(sm_scale) + np.array(add, np.float32)
                mx = s_.max()
                e = np.exp(s_ - mx)
                o[n, h] = e @ v[hk, idx] / e.sum()
                lse[n, h] = mx + np.log(e.sum())
        return torch.from_numpy(o), torch.from_numpy(lse)

    def gather_keys(self, keys, world):
        return self.all_gather(keys, world)

    def exchange_partials(self, o_part, lse_part, world):
        return self.all_gather(o_part, world), self.all_gather(lse_part, world)

    def lse_merge(self, o_all, lse_all, out_dtype):
        return torch.from_numpy(O.lse_merge(o_all.numpy(), lse_all.numpy())[0])

    def all_gather(self, x, world):
        if world == 1:
            return x.unsqueeze(0)
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x.contiguous())
        return torch.stack(parts)


def _reference(pb, nblk_total):
    S = pb["S"]
    kb, cv = O.kbar_contiguous(pb["idx_k"][None], np.zeros(DI, np.float32), BS, nblk_total)
    sc = O.block_scores_headcls(pb["idx_q"][None], kb, cv, pb["q_pos"][None], BS, L)
    topi, bias, valid = O.infer_route_select(sc, None, IDX_SCALE, FLOOR, SIGMA, K, M)
    kall = np.zeros((1, HKV, nblk_total * BS, D), np.float32)
    vall = np.zeros_like(kall)
    kall[0, :, :S] = pb["k"]
    vall[0, :, :S] = pb["v"]
    o = O.decode_attend(pb["q"].transpose(1, 0, 2)[None], kall, vall, topi, bias, valid, pb["q_pos"][None], BS,
                        L * BS, SCALE)[0].transpose(1, 0, 2)
    return o, np.where(valid[0], topi[0], -1), bias[0]


def _rank(rank, world, port, seed, nblk_filled, extra, nblk_total, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pb = _problem(seed, nblk_filled, extra)
        dec = SplitKVDecode(nblk_total=nblk_total, nblk_filled=nblk_filled, block_size=BS, local_blocks=L, topk=K,
                            topm=M, idx_scale=IDX_SCALE, floor=FLOOR, sigma=SIGMA, sm_scale=SCALE, rank=rank,
                            world=world, backend=NumpyBackend(world))
        lo, hi = dec.plan.lo, dec.plan.hi
        kb, cv = O.kbar_contiguous(pb["idx_k"][None], np.zeros(DI, np.float32), BS, nblk_total)
        S = pb["S"]
        t0, t1 = lo * BS, min(hi * BS, S)
        layer = dict(kbar=kb[0, lo:hi], chunk_valid=cv[0, lo:hi], k=pb["k"][:, t0:t1], v=pb["v"][:, t0:t1],
                     tok0=t0)
        out = dec.step(pb["q"], pb["idx_q"], pb["q_pos"], layer, p_range=(S - 2, S - 1))
        if rank == 0:
            ref, rtopi, rbias = _reference(pb, nblk_total)
            sel = dec.backend.merge_keys(
                dec.backend.all_gather(dec.backend.shard_keys(pb["idx_q"], layer, dec.plan, pb["q_pos"], None),
                                       world), dec.plan, None)
            result_q.put(("ok", float(np.abs(out.numpy() - ref).max()), bool(np.array_equal(sel["topi32"], rtopi)),
                          float(np.abs(sel["bias"] - rbias).max())))
        else:
            dec.backend.merge_keys(
                dec.backend.all_gather(dec.backend.shard_keys(pb["idx_q"], layer, dec.plan, pb["q_pos"], None),
                                       world), dec.plan, None)
    except Exception as e:  # reported to the parent, which fails the test
        result_q.put(("error", repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("nblk_filled,extra,nblk_total", [(40, 17, 41), (37, 0, 40)])
def test_split_kv_two_ranks_matches_oracle(nblk_filled, extra, nblk_total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_rank, args=(2, _free_port(), 3, nblk_filled, extra, nblk_total, q), nprocs=2, join=True,
                       start_method="spawn")
    msg = q.get(timeout=60)
    assert msg[0] == "ok", msg
    _, err, same_topi, bias_err = msg
    assert same_topi
    assert bias_err <= 1e-6
    assert err < 1e-5


def test_window_must_stay_on_one_shard():
    dec = SplitKVDecode(nblk_total=40, nblk_filled=40, block_size=BS, local_blocks=L, topk=K, topm=M,
                        idx_scale=IDX_SCALE, floor=FLOOR, sigma=SIGMA, sm_scale=SCALE, rank=0, world=2,
                        backend=NumpyBackend(2))
    assert dec.window_owner(40 * BS - 1, 40 * BS - 2) == 1
    with pytest.raises(ValueError):
        dec.window_owner(20 * BS + 3, 20 * BS + 3)    # window starts in block 18 (rank 0), ends in 20 (rank 1)


class _RecordingBackend:
    """Fails the test if the step reaches any launch or collective."""

    def __getattr__(self, name):
        raise AssertionError(f"backend.{name} called before the plan was checked")


def test_bad_plan_rejected_before_any_launch():
    dec = SplitKVDecode(nblk_total=40, nblk_filled=40, block_size=BS, local_blocks=L, topk=K, topm=M,
                        idx_scale=IDX_SCALE, floor=FLOOR, sigma=SIGMA, sm_scale=SCALE, rank=0, world=2,
                        backend=_RecordingBackend())
    p = 20 * BS + 3      # window straddles the two shards
    with pytest.raises(ValueError, match="spans two shards"):
        dec.step(None, None, None, {}, p_range=(p, p))
    with pytest.raises(ValueError, match="p_range"):
        dec.step(None, None, None, {}, p_range=None)   # positions must come from the host, not the device


def test_shard_plan_covers_blocks_once():
    for total, filled, world in ((16388, 16384, 8), (41, 40, 2), (10, 3, 4)):
        cover = []
        for r in range(world):
            lo, hi = ShardPlan(total, world, r, filled).bounds(r)
            cover.extend(range(lo, hi))
        assert cover == list(range(total))
