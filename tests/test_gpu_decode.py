"""GPU parity of the sparse decode attend (a8/a9) and the split-KV LSE merge,
against the reference's golden vectors (SGLang paged decode kernel, HF
_decode_attend) and the CPU oracle, including the edge cases of the
reference: -1 slots anywhere, repeated ids, a selected block overlapping the
window, requests shorter than the window, several decode rows per request,
GQA, head dims 64 and 128.

Bar: fp32 outputs from bf16 inputs within 1e-4 of the fp32 reference on the
same values; bf16 outputs within 2e-2 abs / 1e-2 rel (north star)."""

import math

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import srswa_oracle as O

pytestmark = pytest.mark.gpu

from srswa import dash_infer, ops, paged  # noqa: E402


def T(x, dev, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dt is None else t.to(dt)


def test_paged_decode_golden(cuda):
    g = golden("paged")
    BS, L, Kb, M = (int(x) for x in g["params"])
    sm_scale = float(g["fparams"][3])
    R, H, D = g["q"].shape
    Hkv = g["k_cache"].shape[2]
    out = torch.zeros(R, H, D, device=cuda, dtype=torch.float32)
    ti = T(g["idx"], cuda).unsqueeze(0).expand(Hkv, -1, -1)
    tb = T(g["bias"], cuda).unsqueeze(0).expand(Hkv, -1, -1)
    paged.dash_sparse_attn_decode(T(g["q"], cuda, torch.bfloat16), T(g["k_cache"], cuda, torch.bfloat16),
                                  T(g["v_cache"], cuda, torch.bfloat16), ti, tb, T(g["block_table"], cuda),
                                  T(g["seq_lens"], cuda), Hkv, sm_scale, out, 1, local_blocks=L,
                                  sparse_block_size=BS)
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], rtol=1e-4, atol=1e-4)


def test_decode_attend_golden(cuda):
    g = golden("decode_attend")
    BS, L, K, M = (int(x) for x in g["params"])
    out = dash_infer._decode_attend(T(g["q"], cuda, torch.bfloat16), T(g["k"], cuda, torch.bfloat16),
                                    T(g["v"], cuda, torch.bfloat16), T(g["topi"], cuda), T(g["bias"], cuda),
                                    T(g["valid"], cuda), T(g["q_pos"], cuda), BS, L * BS, float(g["scale"]))
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], rtol=1e-4, atol=1e-4)


def _paged_case(rng, R, H, Hkv, D, BS, L, K, seqs, dql=1, extra_pages=5):
    W = max((s + BS - 1) // BS for s in seqs)
    P = R * W + extra_pages
    bt = rng.permutation(P)[: R * W].astype(np.int32).reshape(R, W)
    kc = O.bf16_round(rng.standard_normal((P, BS, Hkv, D)).astype(np.float32))
    vc = O.bf16_round(rng.standard_normal((P, BS, Hkv, D)).astype(np.float32))
    q = O.bf16_round(rng.standard_normal((R * dql, H, D)).astype(np.float32))
    idx = np.full((R * dql, K), -1, np.int64)
    bias = (rng.standard_normal((R * dql, K)) * 0.7).astype(np.float32)
    for n in range(R * dql):
        r = n // dql
        p = seqs[r] - dql + n % dql
        qb = p // BS
        cands = np.arange(max(qb - L + 1, 0))           # strictly remote
        if len(cands):
            pick = rng.choice(cands, size=min(K, len(cands)), replace=False)
            idx[n, : len(pick)] = pick
        if len(cands) > 2:
            idx[n, -1] = idx[n, 0]                       # repeated id
            idx[n, 1] = -1                               # hole in the middle
        if K > 3 and qb - L >= 0:
            idx[n, 2] = qb - L                           # block overlapping the window
    return bt, kc, vc, q, idx, bias


@pytest.mark.parametrize("D,H,Hkv,BS,L,K,dql", [(128, 10, 10, 64, 8, 8, 1), (128, 8, 2, 64, 4, 6, 2),
                                                 (64, 4, 4, 32, 3, 5, 1), (128, 4, 4, 16, 2, 4, 1)])
def test_paged_decode_edge_cases_vs_oracle(cuda, D, H, Hkv, BS, L, K, dql):
    rng = np.random.default_rng(D + H + BS)
    seqs = [5 * BS + 7, BS * L - 3, 1, 40 * BS, 12 * BS + 1, 3]
    R = len(seqs)
    bt, kc, vc, q, idx, bias = _paged_case(rng, R, H, Hkv, D, BS, L, K, seqs, dql)
    sm_scale = 1.0 / math.sqrt(D)
    seqs = np.asarray(seqs, np.int32)
    # oracle: repeated ids count once (HF dense block map semantics)
    idx_o = O.dedup_rows(idx)
    ref, ref_lse = O.paged_decode(q, kc, vc, idx_o[None], bias[None], bt, seqs, sm_scale, dql, L, BS)
    for nsplit in (0, 1, 2, 4, 8):
        out, lse = ops.decode_attend(T(q, cuda, torch.bfloat16), T(kc, cuda, torch.bfloat16),
                                     T(vc, cuda, torch.bfloat16), T(idx, cuda).to(torch.int32), T(bias, cuda),
                                     block_size=BS, local_blocks=L, sm_scale=sm_scale,
                                     out=torch.empty(q.shape, device=cuda), block_table=T(bt, cuda),
                                     seq_lens=T(seqs, cuda), rows_per_req=dql, lse=True, nsplit=nsplit)
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)
        l = lse.cpu().numpy()
        fin = np.isfinite(ref_lse)
        assert np.array_equal(np.isfinite(l), fin)
        np.testing.assert_allclose(l[fin], ref_lse[fin], rtol=1e-5, atol=1e-4)


def test_decode_bf16_output_tolerance(cuda):
    rng = np.random.default_rng(7)
    seqs = [3000, 9000, 800]
    bt, kc, vc, q, idx, bias = _paged_case(rng, 3, 10, 10, 128, 64, 8, 8, seqs)
    ref, _ = O.paged_decode(q, kc, vc, O.dedup_rows(idx)[None], bias[None], bt, np.asarray(seqs), 0.088, 1, 8, 64)
    out = ops.decode_attend(T(q, cuda, torch.bfloat16), T(kc, cuda, torch.bfloat16), T(vc, cuda, torch.bfloat16),
                            T(idx, cuda), T(bias, cuda), block_size=64, local_blocks=8, sm_scale=0.088,
                            block_table=T(bt, cuda), seq_lens=T(np.asarray(seqs, np.int32), cuda))
    assert out.dtype == torch.bfloat16
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=1e-2, atol=2e-2)


def test_lse_merge_vs_oracle(cuda):
    rng = np.random.default_rng(3)
    C, N, H, D = 5, 7, 3, 128
    o = rng.standard_normal((C, N, H, D)).astype(np.float32)
    lse = (rng.standard_normal((C, N, H)) * 3).astype(np.float32)
    lse[1, 2] = -np.inf
    lse[:, 4, 1] = -np.inf
    ref_o, ref_l = O.lse_merge(o, lse)
    out, l = ops.lse_merge(T(o, cuda), T(lse, cuda))
    np.testing.assert_allclose(out.cpu().numpy(), ref_o, rtol=1e-5, atol=1e-5)
    assert np.isneginf(l.cpu().numpy()[4, 1])
    fin = np.isfinite(ref_l)
    np.testing.assert_allclose(l.cpu().numpy()[fin], ref_l[fin], rtol=1e-5, atol=1e-5)



@pytest.mark.parametrize("R", [32, 70, 256])
def test_decode_many_rows_split_last_wave(cuda, R):
    """Enough (row, head) items for several waves of CTAs: the rows of a
    nearly empty last wave are attended split over clusters (the split left
    open), the others unsplit.  R = 32 (320 items: one wave unsplit, not
    2-way split) takes the light-load instantiation (5 CTAs per SM, 2-way
    split).  Same outputs and lse as every row unsplit
    (fp32, within 1e-5) and as the oracle on a sample of rows (1e-4).  Two
    KV heads and short requests keep the host-side cache small."""
    rng = np.random.default_rng(R)
    H, Hkv, D, BS, L, K = 10, 2, 128, 64, 8, 8
    seqs = list(rng.integers(520, 800, R))
    bt, kc, vc, q, idx, bias = _paged_case(rng, R, H, Hkv, D, BS, L, K, seqs, extra_pages=0)
    args = [T(q, cuda, torch.bfloat16), T(kc, cuda, torch.bfloat16), T(vc, cuda, torch.bfloat16), T(idx, cuda),
            T(bias, cuda)]
    kw = dict(block_size=BS, local_blocks=L, sm_scale=0.088, block_table=T(bt, cuda),
              seq_lens=T(np.asarray(seqs, np.int32), cuda), lse=True)
    out_auto, lse_auto = ops.decode_attend(*args, out=torch.empty(R, H, D, device=cuda), **kw)
    out_one, lse_one = ops.decode_attend(*args, out=torch.empty(R, H, D, device=cuda), nsplit=1, **kw)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out_auto.cpu().numpy(), out_one.cpu().numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse_auto.cpu().numpy(), lse_one.cpu().numpy(), rtol=1e-5, atol=1e-5)
    rows = np.unique(np.concatenate([np.arange(5), np.arange(R - 30, R)]))
    ref, _ = O.paged_decode(q[rows], kc, vc, O.dedup_rows(idx[rows])[None], bias[rows][None], bt[rows],
                            np.asarray(seqs)[rows], 0.088, 1, L, BS)
    np.testing.assert_allclose(out_auto.cpu().numpy()[rows], ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("R,nsplit", [(32, 0), (256, 0), (40, 2)])
def test_decode_overlap_after_router_equals_plain(cuda, R, nsplit):
    """overlap=True (the attend launched to start on its window keys while
    the router ahead of it on the stream finishes) gives the same bits as the
    plain launch.  The newest K/V row of every request is written on a side
    stream behind a long kernel and joined by an event just before the
    attend: the early window reads must still see it."""
    rng = np.random.default_rng(R + 7)
    H, Hkv, D, BS, L, K, d = 10, 2, 128, 64, 8, 8, 128
    seqs = list(rng.integers(2000, 6000, R))
    bt, kc, vc, q, _, _ = _paged_case(rng, R, H, Hkv, D, BS, L, K, seqs, extra_pages=0)
    P = kc.shape[0]
    kbar = T(rng.standard_normal((P, d)).astype(np.float32), cuda)
    iq = T(rng.standard_normal((R, d)).astype(np.float32), cuda, torch.bfloat16)
    bt_t, sl_t = T(bt, cuda), T(np.asarray(seqs, np.int32), cuda)
    k_t, v_t = T(kc, cuda, torch.bfloat16), T(vc, cuda, torch.bfloat16)
    qt = T(q, cuda, torch.bfloat16)
    last = [(int(bt[r, (s - 1) // BS]), (s - 1) % BS) for r, s in enumerate(seqs)]
    pg = torch.tensor([a for a, _ in last], device=cuda)
    ps = torch.tensor([b for _, b in last], device=cuda)
    new_k, new_v = k_t[pg, ps].clone(), v_t[pg, ps].clone()
    rp = dict(block_size=BS, local_blocks=L, topk=K, topm=16, idx_scale=128 / math.sqrt(d), floor=1e-4, sigma=1.0)
    kw = dict(block_size=BS, local_blocks=L, sm_scale=0.088, block_table=bt_t, seq_lens=sl_t, nsplit=nsplit)
    side = torch.cuda.Stream()
    ev = torch.cuda.Event()
    busy = torch.randn(4096, 4096, device=cuda)
    outs = []
    for overlap in (False, True):
        k_t[pg, ps] = 0
        v_t[pg, ps] = 0
        torch.cuda.synchronize()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(8):        # keeps the side stream busy well past the router
                busy = busy @ busy * 1e-3
            k_t[pg, ps] = new_k
            v_t[pg, ps] = new_v
            ev.record(side)
        sel = ops.route(iq, kbar, block_table=bt_t, seq_lens=sl_t, want=("topi32", "bias"), **rp)
        torch.cuda.current_stream().wait_event(ev)
        outs.append(ops.decode_attend(qt, k_t, v_t, sel["topi32"], sel["bias"], overlap=overlap,
                                      out=torch.empty(R, H, D, device=cuda), **kw))
        torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    rows = np.arange(min(R, 6))
    sel_np = {k: v.cpu().numpy() for k, v in sel.items()}
    ref, _ = O.paged_decode(q[rows], kc, vc, O.dedup_rows(sel_np["topi32"][rows])[None], sel_np["bias"][rows][None],
                            bt[rows], np.asarray(seqs)[rows], 0.088, 1, L, BS)
    np.testing.assert_allclose(outs[1].cpu().numpy()[rows], ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("fp8", [torch.float8_e4m3fn, torch.float8_e5m2])
@pytest.mark.parametrize("D", [128, 64])
def test_decode_fp8_cache_equals_bf16_of_same_values(cuda, fp8, D):
    """FP8 K/V caches (the reference's use_fp8 path, attend_triton.py:545,626:
    the cache is cast to the query dtype before the dots): the attend on fp8
    caches equals, bit for bit, the attend on the same values held in bf16
    (fp8 -> bf16 is exact), decode and paged prefill alike; and the oracle on
    the dequantised values."""
    rng = np.random.default_rng(D + (3 if fp8 == torch.float8_e4m3fn else 5))
    R, H, Hkv, BS, L, K = 6, 8, 4, 64, 8, 8
    seqs = list(rng.integers(700, 3000, R))
    bt, kc, vc, q, idx, bias = _paged_case(rng, R, H, Hkv, D, BS, L, K, seqs)
    k8 = T(kc, cuda).to(fp8)
    v8 = T(vc, cuda).to(fp8)
    kb, vb = k8.to(torch.bfloat16), v8.to(torch.bfloat16)
    args = dict(block_size=BS, local_blocks=L, sm_scale=0.1, block_table=T(bt, cuda),
                seq_lens=T(np.asarray(seqs, np.int32), cuda))
    qt, it, bt_ = T(q, cuda, torch.bfloat16), T(idx, cuda), T(bias, cuda)
    o8 = ops.decode_attend(qt, k8, v8, it, bt_, out=torch.empty(R, H, D, device=cuda), **args)
    ob = ops.decode_attend(qt, kb, vb, it, bt_, out=torch.empty(R, H, D, device=cuda), **args)
    # paged prefill (K8 op): the last 3 positions of each request as rows
    cu = torch.arange(0, 3 * R + 1, 3, device=cuda, dtype=torch.int32)
    pre = T(np.asarray(seqs, np.int32) - 3, cuda)
    qp = torch.repeat_interleave(qt, 3, dim=0)
    ip = torch.repeat_interleave(it, 3, dim=0)
    bp = torch.repeat_interleave(bt_, 3, dim=0)
    p8 = ops.prefill_attend(qp, k8, v8, ip, bp, block_table=T(bt, cuda), cu_seqlens_q=cu, prefix_lens=pre,
                            block_size=BS, local_blocks=L, sm_scale=0.1, out=torch.empty(3 * R, H, D, device=cuda))
    pb = ops.prefill_attend(qp, kb, vb, ip, bp, block_table=T(bt, cuda), cu_seqlens_q=cu, prefix_lens=pre,
                            block_size=BS, local_blocks=L, sm_scale=0.1, out=torch.empty(3 * R, H, D, device=cuda))
    torch.cuda.synchronize()
    assert torch.equal(o8, ob)
    assert torch.equal(p8, pb)
    ref, _ = O.paged_decode(q, k8.float().cpu().numpy(), v8.float().cpu().numpy(), O.dedup_rows(idx)[None],
                            bias[None], bt, np.asarray(seqs), 0.1, 1, L, BS)
    np.testing.assert_allclose(o8.cpu().numpy(), ref, rtol=1e-4, atol=1e-4)
