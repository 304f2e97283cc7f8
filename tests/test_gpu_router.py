"""GPU parity of the router kernels (a1 k_bar, a2 scores, a3 block max, a4
selection) against the reference's golden vectors and the CPU oracle.

Bar (north star): selected block-index sets identical except for fp32 score
ties.  Biases: within 2e-5 when both sides select from the same scores; within
5e-4 when the GPU recomputes the scores itself (fp32 summation-order noise of
~3e-7 is amplified by d log(p)/d score ~ idx_scale/sqrt(p) in the entmax
log-prior)."""

import math

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import srswa_oracle as O

pytestmark = pytest.mark.gpu

from srswa import dash_infer, ops, paged  # noqa: E402
from srswa.sparse_gather import triton_block_max_score  # noqa: E402


def T(x, dev, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dt is None else t.to(dt)


def ties_only(topi_a, topi_b, valid, scores, tol=1e-5):
    """number of rows whose selected sets differ by more than an fp32 tie"""
    bad = 0
    for idx in np.ndindex(topi_a.shape[:-1]):
        va = valid[idx]
        a, b = set(topi_a[idx][va].tolist()), set(topi_b[idx][va].tolist())
        if a != b:
            s = scores[idx]
            kth = min(s[i] for i in a | b)
            if max(abs(s[i] - kth) for i in a ^ b) > tol * max(1.0, abs(kth)):
                bad += 1
    return bad


class Router:
    def __init__(self, bs, L, hc, stage0="head_cls"):
        self.block_size, self.local_blocks, self.local_window = bs, L, L * bs
        self.head_cls, self.stage0 = hc, stage0


def test_kbar_contig_vs_oracle(cuda):
    rng = np.random.default_rng(0)
    for S, bs, dt in ((1000, 64, torch.bfloat16), (777, 32, torch.float32)):
        idx_k = O.bf16_round(rng.standard_normal((2, S, 128)).astype(np.float32))
        for hc in (np.zeros(128, np.float32), (rng.standard_normal(128) * 0.3).astype(np.float32)):
            nblk = (S + bs - 1) // bs
            ref, cv = O.kbar_contiguous(idx_k, hc, bs, nblk)
            kb, cvg = ops.kbar_contig(T(idx_k, cuda, dt), T(hc, cuda), bs)
            np.testing.assert_allclose(kb.cpu().numpy(), ref, rtol=1e-5, atol=2e-6)
            assert np.array_equal(cvg.cpu().numpy(), cv)


@pytest.mark.parametrize("tag", ["hc0", "hc1"])
def test_route_fused_golden(cuda, tag):
    g = golden("route")
    BS, L, K, M = (int(x) for x in g["params"])
    idx_scale, floor, sigma = (float(x) for x in g["fparams"])
    B, S, d = g["idx_k"].shape
    nblk = (S + BS - 1) // BS
    hc = torch.zeros(d) if tag == "hc0" else torch.from_numpy(g["hc1"])
    rt = Router(BS, L, hc.to(cuda))
    iq, ik, qp = T(g["idx_q"], cuda), T(g["idx_k"], cuda, torch.bfloat16), T(g["q_pos"], cuda)
    sc = dash_infer._block_scores_infer(rt, iq, ik, qp, nblk).cpu().numpy()
    np.testing.assert_allclose(sc, g[f"scores_{tag}"], rtol=2e-5, atol=2e-5)
    p = dict(idx_scale=idx_scale, floor=floor, sigma=sigma, K=K, topm=M)
    topi, bias, valid = (x.cpu().numpy() for x in dash_infer.route(rt, iq, ik, qp, nblk, None, p))
    np.testing.assert_array_equal(valid, g[f"valid_{tag}"])
    assert ties_only(topi, g[f"topi_{tag}"], valid, g[f"scores_{tag}"]) == 0
    # Here the scores are recomputed on the GPU (fp32, different summation
    # order than the reference's BLAS): ~3e-7 score differences reach the bias
    # amplified by d log(p)/d score ~ idx_scale/sqrt(p) (~300 for p ~ 1e-3),
    # hence 5e-4.  With identical scores (test_route_select_golden) the bias
    # matches to 2e-5.
    np.testing.assert_allclose(bias, g[f"bias_{tag}"], rtol=1e-5, atol=5e-4)


def test_route_select_golden(cuda):
    g = golden("route")
    BS, L, K, M = (int(x) for x in g["params"])
    idx_scale, floor, sigma = (float(x) for x in g["fparams"])
    sc = T(g["scores_hc0"], cuda)
    p = dict(idx_scale=idx_scale, floor=floor, sigma=sigma, K=K, topm=M)
    for cand, tag in ((None, "hc0"), (T(g["cand"], cuda), "cand")):
        topi, bias, valid = (x.cpu().numpy() for x in dash_infer._infer_route_select(sc, cand, p))
        np.testing.assert_array_equal(valid, g[f"valid_{tag}"])
        assert ties_only(topi, g[f"topi_{tag}"], valid, g["scores_hc0"]) == 0
        np.testing.assert_allclose(bias, g[f"bias_{tag}"], rtol=1e-5, atol=2e-5)
    s2, f2, sg2, K2, M2 = (float(x) for x in g["fparams2"])
    p2 = dict(idx_scale=s2, floor=f2, sigma=sg2, K=int(K2), topm=int(M2))
    topi, bias, valid = (x.cpu().numpy() for x in dash_infer._infer_route_select(sc, None, p2))
    np.testing.assert_array_equal(valid, g["valid_p2"])
    assert ties_only(topi, g["topi_p2"], valid, g["scores_hc0"]) == 0
    np.testing.assert_allclose(bias, g["bias_p2"], rtol=1e-5, atol=2e-5)


def test_route_indexer_golden(cuda):
    g = golden("route")
    BS, L, _, _ = (int(x) for x in g["params"])
    B, S, d = g["idx_k"].shape
    nblk = (S + BS - 1) // BS
    rt = Router(BS, L, None, stage0="indexer")
    sc = dash_infer._block_scores_infer(rt, T(g["idx_q"], cuda), T(g["idx_k"], cuda), T(g["q_pos"], cuda), nblk)
    np.testing.assert_allclose(sc.cpu().numpy(), g["scores_indexer"], rtol=2e-5, atol=2e-4)


def test_block_max_golden(cuda):
    g = golden("block_max")
    BS, LW, nblk = (int(x) for x in g["params"])
    for dt in (torch.float32, torch.bfloat16):
        out = triton_block_max_score(T(g["q"], cuda, dt), T(g["k"], cuda, dt), T(g["pos"], cuda),
                                     T(g["seg"], cuda), BS, nblk, LW).cpu().numpy()
        ref = g["out"]
        assert np.array_equal(np.isneginf(out), np.isneginf(ref))
        fin = np.isfinite(ref)
        np.testing.assert_allclose(out[fin], ref[fin], rtol=1e-5, atol=1e-4)


def test_paged_kbar_and_route_golden(cuda):
    g = golden("paged")
    BS, L, Kb, M = (int(x) for x in g["params"])
    idx_scale, floor, sigma, _ = (float(x) for x in g["fparams"])
    P, _, d = g["idx_cache"].shape
    cache = paged.KBarCache(P, d, cuda)
    bt, sl = T(g["block_table"], cuda), T(g["seq_lens"], cuda)
    cache.summarize(kv_cache=T(g["idx_cache"], cuda, torch.bfloat16), block_table=bt, seq_lens=sl,
                    head_cls=T(g["hc"], cuda), block_size=BS, tail_pages=0)
    R, W = g["block_table"].shape
    used = np.concatenate([g["block_table"][r, :(int(g["seq_lens"][r]) + BS - 1) // BS] for r in range(R)])
    np.testing.assert_allclose(cache.k_bar.cpu().numpy()[used], g["kbar"][used], rtol=1e-5, atol=2e-6)
    # the tail refresh recomputes the same values
    before = cache.k_bar.clone()
    cache.refresh_tail(kv_cache=T(g["idx_cache"], cuda, torch.bfloat16), block_table=bt, seq_lens=sl,
                       head_cls=T(g["hc"], cuda), block_size=BS, tail_pages=2)
    assert torch.equal(before, cache.k_bar)
    out_idx = torch.full((R, 8), 7, dtype=torch.int32, device=cuda)
    out_bias = torch.full((R, 8), 3.0, device=cuda)
    k = paged.route_decode(idx_q=T(g["idx_q"], cuda), k_bar=T(g["kbar"], cuda), block_table=bt, seq_lens=sl,
                           image_allow=None, out_idx=out_idx, out_bias=out_bias, max_block=W, block_size=BS,
                           local_blocks=L, decode_query_len=1, idx_scale=idx_scale, prior_floor=floor,
                           sigma=sigma, topm=M, budget=Kb)
    assert k == Kb
    oi, ob = out_idx.cpu().numpy(), out_bias.cpu().numpy()
    ref_i, ref_b = g["idx"][:, :Kb], g["bias"][:, :Kb]
    valid = ref_i >= 0
    assert np.array_equal(oi[:, :Kb] >= 0, valid)
    assert ties_only(oi[:, :Kb], ref_i, valid, g["scores"]) == 0
    np.testing.assert_allclose(ob[:, :Kb], ref_b, rtol=1e-5, atol=5e-4)
    assert (oi[:, Kb:] == -1).all() and (ob[:, Kb:] == 0).all()
    # buffers exactly K slots wide are written in place by the kernel: same values
    di = torch.full((R, Kb), 7, dtype=torch.int32, device=cuda)
    db = torch.full((R, Kb), 3.0, device=cuda)
    k2 = paged.route_decode(idx_q=T(g["idx_q"], cuda), k_bar=T(g["kbar"], cuda), block_table=bt, seq_lens=sl,
                            image_allow=None, out_idx=di, out_bias=db, max_block=W, block_size=BS,
                            local_blocks=L, decode_query_len=1, idx_scale=idx_scale, prior_floor=floor,
                            sigma=sigma, topm=M, budget=Kb)
    assert k2 == Kb
    assert np.array_equal(di.cpu().numpy(), oi[:, :Kb]) and np.array_equal(db.cpu().numpy(), ob[:, :Kb])


@pytest.mark.parametrize("S_list", [[16384, 131072, 50001, 700, 130]])
def test_route_decode_long_vs_oracle(cuda, S_list):
    """BASELINE decode shape (BS=64, L=8, K=8, M=16, d=128) at long contexts,
    paged k_bar cache with a shuffled page table, against the oracle."""
    rng = np.random.default_rng(2)
    BS, L, K, M, d = 64, 8, 8, 16, 128
    idx_scale, floor, sigma = 128.0 / math.sqrt(d), 1e-4, 1.0
    R = len(S_list)
    W = max((s + BS - 1) // BS for s in S_list)
    P = R * W
    perm = rng.permutation(P).astype(np.int32).reshape(R, W)
    kbar = rng.standard_normal((P, d)).astype(np.float32) * 0.1
    idx_q = O.bf16_round(rng.standard_normal((R, d)).astype(np.float32))
    sl = np.asarray(S_list, np.int32)
    r = ops.route(T(idx_q, cuda), T(kbar, cuda), block_size=BS, local_blocks=L, topk=K, topm=M,
                  idx_scale=idx_scale, floor=floor, sigma=sigma, seq_lens=T(sl, cuda), block_table=T(perm, cuda),
                  want=("topi64", "topi32", "bias", "valid", "scores"))
    sc = r["scores"].cpu().numpy()
    for i in range(R):
        nb = (S_list[i] + BS - 1) // BS
        qb = (S_list[i] - 1) // BS
        cv = np.arange(W) < nb
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[perm[i]][None], cv[None],
                                        np.array([[S_list[i] - 1]]), BS, L)[0, 0]
        np.testing.assert_allclose(sc[i], ref_sc, rtol=2e-5, atol=2e-5)
        topi, bias, valid = O.infer_route_select(ref_sc[None], None, idx_scale, floor, sigma, K, M)
        gv = r["valid"].cpu().numpy()[i]
        assert np.array_equal(gv, valid[0])
        assert ties_only(r["topi64"].cpu().numpy()[i][None], topi, valid, ref_sc[None]) == 0
        np.testing.assert_allclose(r["bias"].cpu().numpy()[i], bias[0], rtol=1e-5, atol=5e-4)
        t32 = r["topi32"].cpu().numpy()[i]
        assert np.array_equal(t32 >= 0, gv) and (t32[gv] <= qb - L).all()


def test_route_decode_short_rows_both_paths_vs_oracle(cuda):
    """Decode rows with fewer than 512 blocks take route_kernel when there are
    enough of them to give every SM a CTA (600 rows here) and the chunked
    score + select kernels when there are few (the first 40 rows alone).
    Both against the oracle on sampled rows, and against each other."""
    rng = np.random.default_rng(7)
    BS, L, K, M, d = 64, 8, 8, 16, 128
    idx_scale, floor, sigma = 11.3, 1e-4, 1.0
    R, few = 600, 40
    S_list = rng.integers(1500, 16000, R).tolist()
    W = max((s + BS - 1) // BS for s in S_list)
    P = R * W
    perm = rng.permutation(P).astype(np.int32).reshape(R, W)
    kbar = rng.standard_normal((P, d)).astype(np.float32) * 0.1
    idx_q = O.bf16_round(rng.standard_normal((R, d)).astype(np.float32))
    sl = np.asarray(S_list, np.int32)
    want = ("topi64", "bias", "valid", "scores")
    kw = dict(block_size=BS, local_blocks=L, topk=K, topm=M, idx_scale=idx_scale, floor=floor, sigma=sigma)
    r_all = ops.route(T(idx_q, cuda), T(kbar, cuda), seq_lens=T(sl, cuda), block_table=T(perm, cuda),
                      want=want, **kw)
    r_few = ops.route(T(idx_q[:few], cuda), T(kbar, cuda), seq_lens=T(sl[:few], cuda),
                      block_table=T(perm[:few], cuda), want=want, **kw)
    res = [{k: v.cpu().numpy() for k, v in r.items()} for r in (r_all, r_few)]
    rows = list(range(0, few, 3)) + list(range(few, R, 37))
    for i in rows:
        cv = np.arange(W) < (S_list[i] + BS - 1) // BS
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[perm[i]][None], cv[None],
                                        np.array([[S_list[i] - 1]]), BS, L)[0, 0]
        topi, bias, valid = O.infer_route_select(ref_sc[None], None, idx_scale, floor, sigma, K, M)
        for r in res:
            if i >= len(r["valid"]):
                continue
            np.testing.assert_allclose(r["scores"][i], ref_sc, rtol=2e-5, atol=2e-5)
            assert np.array_equal(r["valid"][i], valid[0])
            assert ties_only(r["topi64"][i][None], topi, valid, ref_sc[None]) == 0
            np.testing.assert_allclose(r["bias"][i], bias[0], rtol=1e-5, atol=5e-4)
    a, b = res
    assert np.array_equal(a["valid"][:few], b["valid"])
    assert ties_only(a["topi64"][:few], b["topi64"], b["valid"], a["scores"][:few]) == 0


def test_route_prefill_tiled_1024_blocks_vs_oracle(cuda):
    """Prefill rows of one 40000-token sequence (625 blocks): the tiled
    router's wide instantiation (32 keys per lane, up to 1024 blocks);
    sampled rows, early and late, against the oracle."""
    rng = np.random.default_rng(11)
    BS, L, K, M, d = 64, 8, 8, 16, 128
    idx_scale, floor, sigma = 11.3, 1e-4, 1.0
    T_ = 40000
    nblk = (T_ + BS - 1) // BS
    kbar = rng.standard_normal((1, nblk, d)).astype(np.float32) * 0.1
    idx_q = O.bf16_round(rng.standard_normal((T_, d)).astype(np.float32))
    r = ops.route(T(idx_q, cuda), T(kbar, cuda), block_size=BS, local_blocks=L, topk=K, topm=M,
                  idx_scale=idx_scale, floor=floor, sigma=sigma, seq_lens=T(np.array([T_], np.int32), cuda),
                  rows_per_seq=T_, want=("topi64", "bias", "valid", "scores"))
    rows = [0, 530, 577, 4000, 16383, 31000, 38911, T_ - 1]
    idx = torch.tensor(rows, device=cuda)
    got = {k: v[idx].cpu().numpy() for k, v in r.items()}
    cv = np.ones(nblk, bool)
    for j, i in enumerate(rows):
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[0][None], cv[None], np.array([[i]]), BS, L)[0, 0]
        np.testing.assert_allclose(got["scores"][j], ref_sc, rtol=2e-5, atol=2e-5)
        topi, bias, valid = O.infer_route_select(ref_sc[None], None, idx_scale, floor, sigma, K, M)
        assert np.array_equal(got["valid"][j], valid[0])
        assert ties_only(got["topi64"][j][None], topi, valid, ref_sc[None]) == 0
        np.testing.assert_allclose(got["bias"][j], bias[0], rtol=1e-5, atol=5e-4)


def test_route_prefill_long_rows_tiled_vs_oracle(cuda):
    """One 90000-token sequence (1407 blocks, past the one-pass tiled
    router's 1024): the long-row tiled router (512-block spans merged into a
    running top-M), contiguous k_bar, sampled rows against the oracle; then
    the same rows over a shuffled paged k_bar, which must give the same
    outputs bit for bit."""
    rng = np.random.default_rng(13)
    BS, L, K, M, d = 64, 8, 8, 16, 128
    idx_scale, floor, sigma = 11.3, 1e-4, 1.0
    T_ = 90000
    nblk = (T_ + BS - 1) // BS
    kbar = rng.standard_normal((1, nblk, d)).astype(np.float32) * 0.1
    idx_q = O.bf16_round(rng.standard_normal((T_, d)).astype(np.float32))
    kw = dict(block_size=BS, local_blocks=L, topk=K, topm=M, idx_scale=idx_scale, floor=floor, sigma=sigma,
              want=("topi64", "bias", "valid"))
    sl = T(np.array([T_], np.int32), cuda)
    r = ops.route(T(idx_q, cuda), T(kbar, cuda), seq_lens=sl, rows_per_seq=T_, **kw)
    rows = [0, 520, 535, 600, 33000, 32767, 65600, 77777, T_ - 1]
    idx = torch.tensor(rows, device=cuda)
    got = {k: v[idx].cpu().numpy() for k, v in r.items()}
    cv = np.ones(nblk, bool)
    for j, i in enumerate(rows):
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[0][None], cv[None], np.array([[i]]), BS, L)[0, 0]
        topi, bias, valid = O.infer_route_select(ref_sc[None], None, idx_scale, floor, sigma, K, M)
        assert np.array_equal(got["valid"][j], valid[0])
        assert ties_only(got["topi64"][j][None], topi, valid, ref_sc[None]) == 0
        np.testing.assert_allclose(got["bias"][j], bias[0], rtol=1e-5, atol=5e-4)
    perm = rng.permutation(nblk + 5)[:nblk].astype(np.int32)
    pool = np.zeros((nblk + 5, d), np.float32)
    pool[perm] = kbar[0]
    rp = ops.route(T(idx_q, cuda), T(pool, cuda), seq_lens=sl, rows_per_seq=T_, block_table=T(perm[None], cuda),
                   **kw)
    for k in r:
        assert torch.equal(r[k], rp[k]), k
    # a candidate mask (PageGate): ~20 % of the blocks; rows 520 and 65600
    # have none among their remote blocks and fall back to all of them
    cand = torch.rand(T_, nblk, device=cuda) < 0.2
    cand[520] = False
    cand[65600] = False
    rc = ops.route(T(idx_q, cuda), T(kbar, cuda), seq_lens=sl, rows_per_seq=T_, cand=cand, **kw)
    got = {k: v[idx].cpu().numpy() for k, v in rc.items()}
    cm = cand[idx].cpu().numpy()
    for j, i in enumerate(rows):
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[0][None], cv[None], np.array([[i]]), BS, L)[0, 0]
        topi, bias, valid = O.infer_route_select(ref_sc[None], cm[j][None], idx_scale, floor, sigma, K, M)
        assert np.array_equal(got["valid"][j], valid[0]), i
        assert ties_only(got["topi64"][j][None], topi, valid, ref_sc[None]) == 0, i
        np.testing.assert_allclose(got["bias"][j], bias[0], rtol=1e-5, atol=5e-4)


def test_route_prefill_ragged_batch_per_sequence(cuda):
    """Three sequences of 3000 rows (not a multiple of the 32-row tile): the
    tiled router runs once per sequence; against the same rows routed one
    sequence per call, bit for bit, and sampled rows against the oracle."""
    rng = np.random.default_rng(17)
    BS, L, K, M, d = 64, 8, 8, 16, 128
    idx_scale, floor, sigma = 11.3, 1e-4, 1.0
    B, T_ = 3, 3000
    nblk = (T_ + BS - 1) // BS
    kbar = rng.standard_normal((B, nblk, d)).astype(np.float32) * 0.1
    idx_q = O.bf16_round(rng.standard_normal((B * T_, d)).astype(np.float32))
    kw = dict(block_size=BS, local_blocks=L, topk=K, topm=M, idx_scale=idx_scale, floor=floor, sigma=sigma,
              want=("topi64", "bias", "valid", "scores"))
    sl = T(np.full(B, T_, np.int32), cuda)
    r = ops.route(T(idx_q, cuda), T(kbar, cuda), seq_lens=sl, rows_per_seq=T_, **kw)
    for b in range(B):
        rb = ops.route(T(idx_q[b * T_:(b + 1) * T_], cuda), T(kbar[b:b + 1], cuda), seq_lens=sl[b:b + 1],
                       rows_per_seq=T_, **kw)
        for k in rb:
            assert torch.equal(r[k][b * T_:(b + 1) * T_], rb[k]), (b, k)
    cv = np.ones(nblk, bool)
    for i in [0, 700, 2999, 3000, 4500, 8999]:
        b, t = divmod(i, T_)
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[b][None], cv[None], np.array([[t]]), BS, L)[0, 0]
        np.testing.assert_allclose(r["scores"][i].cpu().numpy(), ref_sc, rtol=2e-5, atol=2e-5)
        topi, bias, valid = O.infer_route_select(ref_sc[None], None, idx_scale, floor, sigma, K, M)
        assert np.array_equal(r["valid"][i].cpu().numpy(), valid[0])
        assert ties_only(r["topi64"][i].cpu().numpy()[None], topi, valid, ref_sc[None]) == 0


def test_route_prefill_beyond_65535_rows_vs_oracle(cuda):
    """One 66000-token sequence (1032 blocks, above the tiled prefill
    router's 512): the score pass takes its rows in launches of at most
    65535; rows on both sides of that boundary against the oracle."""
    rng = np.random.default_rng(9)
    BS, L, K, M, d = 64, 8, 8, 16, 128
    idx_scale, floor, sigma = 11.3, 1e-4, 1.0
    T_ = 66000
    nblk = (T_ + BS - 1) // BS
    kbar = rng.standard_normal((1, nblk, d)).astype(np.float32) * 0.1
    idx_q = O.bf16_round(rng.standard_normal((T_, d)).astype(np.float32))
    r = ops.route(T(idx_q, cuda), T(kbar, cuda), block_size=BS, local_blocks=L, topk=K, topm=M,
                  idx_scale=idx_scale, floor=floor, sigma=sigma, seq_lens=T(np.array([T_], np.int32), cuda),
                  rows_per_seq=T_, want=("topi64", "bias", "valid", "scores"))
    rows = [600, 40000, 65533, 65534, 65535, 65536, 65537, T_ - 1]
    idx = torch.tensor(rows, device=cuda)
    got = {k: v[idx].cpu().numpy() for k, v in r.items()}
    cv = np.ones(nblk, bool)
    for j, i in enumerate(rows):
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[0][None], cv[None], np.array([[i]]), BS, L)[0, 0]
        np.testing.assert_allclose(got["scores"][j], ref_sc, rtol=2e-5, atol=2e-5)
        topi, bias, valid = O.infer_route_select(ref_sc[None], None, idx_scale, floor, sigma, K, M)
        assert np.array_equal(got["valid"][j], valid[0])
        assert ties_only(got["topi64"][j][None], topi, valid, ref_sc[None]) == 0
        np.testing.assert_allclose(got["bias"][j], bias[0], rtol=1e-5, atol=5e-4)


def test_route_decode_cand_mask_vs_oracle(cuda):
    """Chunked decode router with a page-aware candidate mask; rows 1 and 3
    have an empty mask and fall back to every remote block."""
    rng = np.random.default_rng(4)
    BS, L, K, M, d = 64, 8, 8, 16, 128
    S_list = [40000, 52000, 33000, 60000, 45000]
    R = len(S_list)
    W = max((s + BS - 1) // BS for s in S_list)
    P = R * W
    perm = rng.permutation(P).astype(np.int32).reshape(R, W)
    kbar = rng.standard_normal((P, d)).astype(np.float32) * 0.1
    idx_q = O.bf16_round(rng.standard_normal((R, d)).astype(np.float32))
    cand = rng.random((R, W)) < 0.2
    cand[1] = False
    cand[3] = False
    sl = np.asarray(S_list, np.int32)
    r = ops.route(T(idx_q, cuda), T(kbar, cuda), block_size=BS, local_blocks=L, topk=K, topm=M,
                  idx_scale=11.3, floor=1e-4, sigma=1.0, seq_lens=T(sl, cuda), block_table=T(perm, cuda),
                  cand=T(cand, cuda), want=("topi64", "bias", "valid", "scores"))
    sc = r["scores"].cpu().numpy()
    for i in range(R):
        cv = np.arange(W) < (S_list[i] + BS - 1) // BS
        ref_sc = O.block_scores_headcls(idx_q[i][None, None], kbar[perm[i]][None], cv[None],
                                        np.array([[S_list[i] - 1]]), BS, L)[0, 0]
        np.testing.assert_allclose(sc[i], ref_sc, rtol=2e-5, atol=2e-5)
        topi, bias, valid = O.infer_route_select(ref_sc[None], cand[i][None], 11.3, 1e-4, 1.0, K, M)
        assert np.array_equal(r["valid"].cpu().numpy()[i], valid[0])
        assert ties_only(r["topi64"].cpu().numpy()[i][None], topi, valid, ref_sc[None]) == 0
        np.testing.assert_allclose(r["bias"].cpu().numpy()[i], bias[0], rtol=1e-5, atol=5e-4)
