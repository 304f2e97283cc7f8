"""Parity at the BASELINE configurations' full sizes.

cfg2 (prefill: B=4, T=16384, K=8, LW=512, seed 1, N(0,1)*0.5) and cfg4
(training: B=8, T=32768, K=16, LW=1024, seed 3, N(0,1)) run exactly as the
benchmark runs them: the CUDA router picks the blocks, the tensor-core
gather-attention computes o (and, for cfg4, dQ / dK / dV / d_bias).  The
oracle cannot build the dense [T, T] masks at these sizes, so it checks
sampled query rows (o, lse, dQ, d_bias, and the router's selection for the
same rows) and sampled key blocks (dK, dV) of two batch elements, the first
and the last; the sampled rows include the block and window edges.

Bar (north star): selections identical except fp32 ties; bf16 outputs and
gradients within 2e-2 abs / 1e-2 rel of fp32 on the same bf16 values."""

import math

import numpy as np
import pytest
import torch

from oracle import srswa_oracle as O

pytestmark = pytest.mark.gpu

from srswa import dash_infer, ops  # noqa: E402
from srswa.sparse_gather_e2e import triton_gather_attention_e2e  # noqa: E402

RTOL, ATOL = 1e-2, 2e-2
BS, H, D, DI, M = 64, 10, 128, 128, 16
IDX_SCALE, FLOOR, SIGMA = 128 / math.sqrt(128), 1e-4, 1.0
CFG = {"cfg2": dict(B=4, T=16384, K=8, LW=512, seed=1, sc=0.5),
       "cfg4": dict(B=8, T=32768, K=16, LW=1024, seed=3, sc=1.0)}


def _rows(T, LW, rng, n=40):
    edges = [0, 1, BS - 1, BS, LW - 1, LW, LW + BS - 1, LW + BS, 2 * LW, T // 2, T // 2 + 1, T - BS - 1, T - BS,
             T - 2, T - 1]
    return np.unique(np.concatenate([edges, rng.integers(0, T, n)]))


def _setup(cuda, cfg):
    c = CFG[cfg]
    B, T, K, LW = c["B"], c["T"], c["K"], c["LW"]
    g = torch.Generator(device=cuda).manual_seed(c["seed"] * 100)
    mk = lambda *shape: (torch.randn(*shape, device=cuda, generator=g) * c["sc"]).to(torch.bfloat16)  # noqa: E731
    q, k, v = mk(B, H, T, D), mk(B, H, T, D), mk(B, H, T, D)
    iq = mk(B, T, DI).float()
    ik = mk(B, T, DI)
    router = type("R", (), dict(block_size=BS, local_blocks=LW // BS, local_window=LW,
                                head_cls=torch.zeros(DI, device=cuda), stage0="head_cls"))()
    pos = torch.arange(T, device=cuda)[None].expand(B, T).contiguous()
    topi, bias, valid = dash_infer.route(router, iq, ik, pos, T // BS, None,
                                         dict(idx_scale=IDX_SCALE, floor=FLOOR, sigma=SIGMA, K=K, topm=M))
    sel = torch.where(valid, topi, torch.full_like(topi, -1))[:, None]
    b = (bias * valid).float().contiguous()
    return dict(B=B, T=T, K=K, LW=LW, q=q, k=k, v=v, iq=iq, ik=ik, pos=pos, topi=topi, bias=bias, valid=valid,
                sel=sel, b=b)


def _np(x):
    return x.float().cpu().numpy()


def _check_router_rows(s, bi, rows):
    """The CUDA router's selection and bias at the sampled rows equal the
    oracle's _block_scores_infer + _infer_route_select (ties aside)."""
    T, K, LW = s["T"], s["K"], s["LW"]
    nblk = T // BS
    kb, cv = O.kbar_contiguous(_np(s["ik"][bi:bi + 1]), np.zeros(DI, np.float32), BS, nblk)
    sc = O.block_scores_headcls(_np(s["iq"][bi, rows])[None], kb, cv, rows[None], BS, LW // BS)
    topi, bias, valid = O.infer_route_select(sc, None, IDX_SCALE, FLOOR, SIGMA, K, M)
    g_topi, g_bias, g_valid = (x[bi, rows].cpu().numpy() for x in (s["topi"], s["bias"], s["valid"]))
    for i in range(len(rows)):
        a, r = set(g_topi[i][g_valid[i]].tolist()), set(topi[0, i][valid[0, i]].tolist())
        if a != r:   # only an fp32 tie may differ
            x = sc[0, i]
            kth = min(x[j] for j in a | r)
            assert max(abs(x[j] - kth) for j in a ^ r) <= 1e-5 * max(1.0, abs(kth)), (rows[i], a, r)
            continue
        order = {blk: j for j, blk in enumerate(topi[0, i])}
        ref_b = np.array([bias[0, i][order[blk]] for blk in g_topi[i][g_valid[i]]])
        np.testing.assert_allclose(g_bias[i][g_valid[i]], ref_b, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("cfg", ["cfg2", "cfg4"])
def test_full_size_sampled_rows_vs_oracle(cuda, cfg):
    s = _setup(cuda, cfg)
    T, LW = s["T"], s["LW"]
    nblk = T // BS
    scale = 1 / math.sqrt(D)
    qt, kt, vt = (x.transpose(1, 2) for x in (s["q"], s["k"], s["v"]))
    sel_p = ops.pack_selection(s["sel"], nblk)
    o, lse = ops.gather_fwd(qt, kt, vt, sel_p, s["b"], None, BS, scale, LW)
    # the public autograd drop-in runs the same kernels: bit-identical output
    o_pub = triton_gather_attention_e2e(s["q"], s["k"], s["v"], s["sel"], s["b"], s["pos"], None, BS, scale, LW)
    torch.cuda.synchronize()
    assert torch.equal(o_pub.transpose(1, 2), o)
    del o_pub
    train = cfg == "cfg4"
    if train:
        g = torch.Generator(device=cuda).manual_seed(77)
        do = torch.randn(s["B"], T, H, D, device=cuda, generator=g).to(torch.bfloat16)
        dq, dk, dv, db = ops.gather_bwd(qt, kt, vt, o, lse, do, sel_p, s["b"], None, BS, scale, LW)
        torch.cuda.synchronize()
    rng = np.random.default_rng(5)
    seg = np.zeros(T, np.int64)
    for bi in (0, s["B"] - 1):
        rows = _rows(T, LW, rng)
        _check_router_rows(s, bi, rows)
        q_b, k_b, v_b = (_np(x[bi]) for x in (qt, kt, vt))
        sel_b = s["sel"][bi, 0].cpu().numpy()
        bias_b = s["b"][bi].cpu().numpy()
        o_r, lse_r = O.gather_rows_fwd(q_b, k_b, v_b, sel_b, seg, rows, BS, scale, LW, bias_b)
        np.testing.assert_allclose(_np(o[bi, rows]), o_r, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(lse[bi, rows].cpu().numpy(), lse_r, rtol=1e-3, atol=1e-3)
        if not train:
            continue
        do_b = _np(do[bi])
        dq_r, db_r = O.gather_rows_bwd(q_b, k_b, v_b, do_b, sel_b, seg, rows, BS, scale, LW, bias_b)
        np.testing.assert_allclose(_np(dq[bi, rows]), dq_r, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(db[bi, rows].cpu().numpy(), db_r, rtol=1e-2, atol=5e-2)
        o_b, lse_b = _np(o[bi]), lse[bi].cpu().numpy()
        for c in (0, 1, LW // BS, nblk // 3, nblk - LW // BS - 2, nblk - 1):
            dk_r, dv_r = O.gather_block_bwd(q_b, k_b, v_b, do_b, o_b, lse_b, sel_b, seg, c, BS, scale, LW, bias_b)
            np.testing.assert_allclose(_np(dk[bi, c * BS:(c + 1) * BS]), dk_r, rtol=RTOL, atol=ATOL)
            np.testing.assert_allclose(_np(dv[bi, c * BS:(c + 1) * BS]), dv_r, rtol=RTOL, atol=ATOL)
