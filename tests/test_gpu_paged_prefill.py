"""GPU parity of the SGLang prefill serving ops of srswa.paged (the names
install_sglang binds into the DASH backend): the varlen paged prefill attend
dash_sparse_attn (K8), the varlen router route_prefill_triton, the k_bar
refresh of an explicit page plan, and the decode scan window
win_bounds_decode (K14).  Checked against the reference wheel's own outputs
(tests/golden/paged_prefill.npz, interpreted Triton) and, at BASELINE head
shapes with long cached prefixes, against the oracle.

Bars: selections identical (sets; the wheel packs ascending ids, this
library score-descending); fp32 attend outputs within 1e-4, bf16 within
2e-2 abs / 1e-2 rel; k_bar within 1e-5; scan-window spans exact."""

import math

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import srswa_oracle as O

pytestmark = pytest.mark.gpu

from srswa import paged  # noqa: E402


def T(x, dev, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dt is None else t.to(dt)


def test_paged_prefill_ops_golden(cuda):
    g = golden("paged_prefill")
    BS, L, topm, budget, dql, tile = (int(x) for x in g["params"])
    idx_scale, floor, sigma, scale = (float(x) for x in g["fparams"])
    bt, seq, ctx, cu = (T(g[k], cuda) for k in ("block_table", "seq_lens", "context_lens", "cu_seqlens_q"))
    W = g["block_table"].shape[1]
    idx_cache = T(g["idx_cache"], cuda, torch.bfloat16)
    # k_bar refresh of the kbar_all_plan pages; untouched rows keep their values
    kbar = T(g["kbar_before"], cuda)
    paged.kbar_refresh_tail_triton(kv_cache=idx_cache, k_bar=kbar, block_table=bt, seq_lens=seq,
                                   head_cls=T(g["hc"], cuda), block_size=BS,
                                   plan=(T(g["plan_pages"], cuda), T(g["plan_tok"], cuda)))
    torch.cuda.synchronize()
    np.testing.assert_allclose(kbar.cpu().numpy(), g["kbar"], rtol=1e-5, atol=1e-5)
    # varlen router into caller-owned [N, topm] buffers (reference layout)
    N = g["idx_q"].shape[0]
    out_idx = torch.full((N, topm), -7, device=cuda, dtype=torch.int32)
    out_bias = torch.full((N, topm), 9.0, device=cuda)
    width, _, _ = paged.route_prefill_triton(
        idx_q=T(g["idx_q"], cuda, torch.bfloat16), k_bar=T(g["kbar"], cuda), block_table=bt, seq_lens=seq,
        cu_seqlens_q=cu, context_lens=ctx, row2req=T(g["row2req"], cuda), image_allow=T(g["allow"], cuda),
        out_idx=out_idx, out_bias=out_bias, max_block=W, block_size=BS, local_blocks=L, idx_scale=idx_scale,
        prior_floor=floor, sigma=sigma, topm=topm, budget=budget)
    oi, ob = out_idx.cpu().numpy(), out_bias.cpu().numpy()
    assert width >= budget
    for n in range(N):
        ref = {int(b): float(x) for b, x in zip(g["out_idx"][n], g["out_bias"][n]) if b >= 0}
        mine = {int(b): float(x) for b, x in zip(oi[n], ob[n]) if b >= 0}
        assert set(ref) == set(mine), n
        for b in ref:
            assert abs(ref[b] - mine[b]) < 1e-4, (n, b)
        assert (oi[n][len(mine):] == -1).all() and (ob[n][len(mine):] == 0).all()
    # paged prefill attend on the wheel's selection, stride-0 over kv heads
    Hkv = g["k_cache"].shape[2]
    ti = T(g["out_idx"][:, :budget], cuda).unsqueeze(0).expand(Hkv, -1, -1)
    tb = T(g["out_bias"][:, :budget], cuda).unsqueeze(0).expand(Hkv, -1, -1)
    out = torch.zeros(g["q"].shape, device=cuda)
    paged.dash_sparse_attn(T(g["q"], cuda), T(g["k_cache"], cuda, torch.bfloat16),
                           T(g["v_cache"], cuda, torch.bfloat16), ti, tb, bt, cu, seq, ctx,
                           int((g["cu_seqlens_q"][1:] - g["cu_seqlens_q"][:-1]).max()), Hkv, scale, out,
                           local_blocks=L, sparse_block_size=BS)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], rtol=1e-4, atol=1e-4)
    # decode scan window
    nd = len(g["lo"])
    lo = torch.zeros(nd, device=cuda, dtype=torch.int32)
    hi = torch.zeros(nd, device=cuda, dtype=torch.int32)
    fit = torch.zeros(nd, device=cuda, dtype=torch.int8)
    paged.win_bounds_decode(allow=T(g["dallow"], cuda), seq_lens=seq, lo=lo, hi=hi, fit=fit, max_block=W,
                            block_size=BS, local_blocks=L, decode_query_len=dql, tile=tile)
    torch.cuda.synchronize()
    assert (lo.cpu().numpy() == g["lo"]).all() and (hi.cpu().numpy() == g["hi"]).all()
    assert (fit.cpu().numpy() == g["fit"]).all()


def test_paged_prefill_long_prefix_vs_oracle(cuda):
    """BASELINE head layout (H = Hkv = 10, D = 128, 64-token pages, K = 8,
    LW = 512) with cached prefixes of 0 to 5000 tokens and one-row to
    700-row requests on a shuffled page pool: router (sets and biases) and
    bf16 attend against the oracle."""
    rng = np.random.default_rng(31)
    H = Hkv = 10
    D, d, BS, L, K, M = 128, 128, 64, 8, 8, 16
    ctx = np.array([5000, 0, 1200, 777], np.int32)
    qlen = np.array([1, 300, 700, 64], np.int32)
    seq = ctx + qlen
    R = len(ctx)
    W = int((seq.max() + BS - 1) // BS) + 2
    P = R * W + 7
    bt = rng.permutation(P)[:R * W].reshape(R, W).astype(np.int32)
    cu = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int32)
    N = int(cu[-1])
    kc = O.bf16_round(rng.standard_normal((P, BS, Hkv, D)).astype(np.float32))
    vc = O.bf16_round(rng.standard_normal((P, BS, Hkv, D)).astype(np.float32))
    ic = O.bf16_round(rng.standard_normal((P, BS, d)).astype(np.float32) * 0.5)
    q = O.bf16_round(rng.standard_normal((N, H, D)).astype(np.float32))
    iq = O.bf16_round(rng.standard_normal((N, d)).astype(np.float32) * 0.5)
    row2req = (np.searchsorted(cu, np.arange(N), side="right") - 1).astype(np.int32)
    # k_bar of every page in use (all pages: plan with the token count per page)
    pages = bt.reshape(-1).astype(np.int64)
    tok = np.clip(seq[:, None] - np.arange(W)[None] * BS, 0, BS).reshape(-1).astype(np.int32)
    kbar = torch.zeros(P, d, device=cuda)
    paged.kbar_refresh_tail(kv_cache=T(ic, cuda, torch.bfloat16), k_bar=kbar, block_table=T(bt, cuda),
                            seq_lens=T(seq, cuda), head_cls=torch.zeros(d, device=cuda), block_size=BS,
                            plan=(T(pages, cuda), T(tok, cuda)))
    out_idx = torch.empty(N, K, device=cuda, dtype=torch.int32)
    out_bias = torch.empty(N, K, device=cuda)
    idx_scale = 128 / math.sqrt(d)
    paged.route_prefill_triton(idx_q=T(iq, cuda, torch.bfloat16), k_bar=kbar, block_table=T(bt, cuda),
                               seq_lens=T(seq, cuda), cu_seqlens_q=T(cu, cuda), context_lens=T(ctx, cuda),
                               row2req=T(row2req, cuda), image_allow=None, out_idx=out_idx, out_bias=out_bias,
                               max_block=W, block_size=BS, local_blocks=L, idx_scale=idx_scale, prior_floor=1e-4,
                               sigma=1.0, topm=M, budget=K)
    out = torch.empty(N, H, D, device=cuda, dtype=torch.bfloat16)
    paged.dash_sparse_attn(T(q, cuda, torch.bfloat16), T(kc, cuda, torch.bfloat16), T(vc, cuda, torch.bfloat16),
                           out_idx.unsqueeze(0).expand(Hkv, -1, -1), out_bias.unsqueeze(0).expand(Hkv, -1, -1),
                           T(bt, cuda), T(cu, cuda), T(seq, cuda), T(ctx, cuda), int(qlen.max()), Hkv,
                           1 / math.sqrt(D), out, local_blocks=L, sparse_block_size=BS)
    torch.cuda.synchronize()
    oi, ob = out_idx.cpu().numpy(), out_bias.cpu().numpy()
    kb_all = kbar.cpu().numpy()
    rows = np.unique(np.concatenate([cu[:-1], cu[1:] - 1, rng.integers(0, N, 60)]))
    for n in rows:
        r = int(row2req[n])
        p = int(ctx[r]) + n - int(cu[r])
        cv = (np.arange(W) * BS < int(seq[r]))[None]
        sc = O.block_scores_headcls(iq[n][None, None], kb_all[bt[r]][None], cv, np.array([[p]]), BS, L)
        topi, bias, valid = O.infer_route_select(sc, None, idx_scale, 1e-4, 1.0, K, M)
        ref = {int(b): float(x) for b, x, v in zip(topi[0, 0], bias[0, 0], valid[0, 0]) if v}
        mine = {int(b): float(x) for b, x in zip(oi[n], ob[n]) if b >= 0}
        if set(ref) != set(mine):           # only an fp32 tie may differ
            x = sc[0, 0]
            kth = min(x[j] for j in set(ref) | set(mine))
            assert max(abs(x[j] - kth) for j in set(ref) ^ set(mine)) <= 1e-5 * max(1.0, abs(kth)), n
            continue
        for b in ref:
            assert abs(ref[b] - mine[b]) < 1e-4, (n, b)
    ref_o, _ = O.paged_prefill(q, kc, vc, oi[None], ob[None], bt, cu, ctx, 1 / math.sqrt(D), L, BS, rows=rows)
    np.testing.assert_allclose(out.float().cpu().numpy()[rows], ref_o[rows], rtol=1e-2, atol=2e-2)


def test_paged_prefill_tensor_core_equals_row_kernel(cuda):
    """dash_sparse_attn sends requests of at least paged.TC_MIN_ROWS rows
    through the tensor-core forward over the paged caches (prefixes not a
    multiple of 64, partial last pages) and shorter ones through the row
    kernel.  Against the row kernel on every row, within the bf16 bar.  The
    unused slots of each request's last page hold NaN: neither path may read
    them."""
    from srswa import ops
    rng = np.random.default_rng(5)
    H = Hkv = 10
    D, BS, L, K = 128, 64, 8, 8
    LW = L * BS
    ctx = [0, 1000, 4133, 0, 50, 640]
    qlen = [700, 1300, 257, 130, 20, 384]   # the last ends on a page boundary (no partial page)
    R = len(ctx)
    seq = [c + n for c, n in zip(ctx, qlen)]
    W = max((s + BS - 1) // BS for s in seq) + 1
    P = R * W + 3
    bt = rng.permutation(P)[:R * W].reshape(R, W).astype(np.int32)
    cu = np.concatenate([[0], np.cumsum(qlen)]).astype(np.int32)
    N = int(cu[-1])
    kc = torch.randn(P, BS, Hkv, D, device=cuda).to(torch.bfloat16)
    vc = torch.randn(P, BS, Hkv, D, device=cuda).to(torch.bfloat16)
    for r in range(R):
        last, used = (seq[r] - 1) // BS, seq[r] % BS
        if used:
            kc[int(bt[r, last]), used:] = float("nan")
            vc[int(bt[r, last]), used:] = float("nan")
    q = torch.randn(N, H, D, device=cuda).to(torch.bfloat16)
    sel = np.full((N, K), -1, np.int32)
    for r in range(R):
        for i in range(qlen[r]):
            p = ctx[r] + i
            nrem = max(p - LW + 1, 0) // BS + 1   # blocks holding remote keys (the last one partly)
            pick = rng.choice(nrem + 2, size=min(K, nrem + 2), replace=False) - 1   # -1 and one past: unused
            sel[cu[r] + i, :len(pick)] = pick
    sel[::7, 1] = sel[::7, 0]                                  # repeats count once
    bias = (rng.standard_normal((N, K)) * 0.5).astype(np.float32)
    ti = T(sel, cuda).unsqueeze(0).expand(Hkv, -1, -1)
    tb = T(bias, cuda).unsqueeze(0).expand(Hkv, -1, -1)
    out_tc = torch.empty(N, H, D, device=cuda, dtype=torch.bfloat16)
    paged.dash_sparse_attn(q, kc, vc, ti, tb, T(bt, cuda), T(cu, cuda), T(np.asarray(seq, np.int32), cuda),
                           T(np.asarray(ctx, np.int32), cuda), max(qlen), Hkv, 1 / math.sqrt(D), out_tc,
                           local_blocks=L, sparse_block_size=BS)
    out_row = ops.prefill_attend(q, kc, vc, ti, tb, block_table=T(bt, cuda), cu_seqlens_q=T(cu, cuda),
                                 prefix_lens=T(np.asarray(ctx, np.int32), cuda), block_size=BS, local_blocks=L,
                                 sm_scale=1 / math.sqrt(D))
    torch.cuda.synchronize()
    assert torch.isfinite(out_tc).all() and torch.isfinite(out_row).all()
    np.testing.assert_allclose(out_tc.float().cpu().numpy(), out_row.float().cpu().numpy(), rtol=1e-2, atol=2e-2)
