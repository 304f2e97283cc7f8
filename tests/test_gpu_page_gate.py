"""PageGate on the GPU (through the C ABI): page-aware ids, block candidate
masks and the decode allow mask, against the reference's own outputs (golden
fixture) and, at sizes spanning many 2048-token scan chunks, against the
pinned CPU oracle.  Integer work: every comparison is exact."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import page_gate as PG

pytestmark = pytest.mark.gpu

IMG, MARK = 128815, 128827


class Indexer:
    """The attributes of DeepseekV2Indexer the PageGate methods read."""

    def __init__(self, bs, per_page, constraint=True):
        self.block_size = bs
        self.per_page_image_tokens = per_page
        self.image_bucket_constraint = constraint
        self.image_token_id = IMG
        self.page_token_id = MARK


class Cache:
    def __init__(self, n):
        self.n = n

    def get_seq_length(self):
        return self.n


def long_rows(seed, B, S, per_page):
    """Seeded documents: <PAGE>-marked pages of 50-400 image tokens plus text,
    an instruction, then marked response pages (row 1: an unmarked image run
    in per-page mode; row 2: images before the first marker)."""
    rng = np.random.default_rng(seed)
    out = np.full((B, S), 5, np.int64)
    for b in range(B):
        r = [0]
        if b % 3 == 1:
            r += [IMG] * (per_page * 37 + 11) + list(rng.integers(0, 1000, 40))
        else:
            if b % 3 == 2:
                r += [IMG] * 300 + list(rng.integers(0, 1000, 9))
            while len(r) < S * 0.7:
                r += [MARK] + [IMG] * int(rng.integers(50, 400)) + list(rng.integers(0, 1000, int(rng.integers(0, 6))))
            r += list(rng.integers(0, 1000, 100))
        while len(r) < S:
            r += [MARK] + list(rng.integers(0, 1000, int(rng.integers(100, 600))))
        out[b] = np.asarray(r[:S])
    return out


def t(x, dev):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev)


def test_page_ids_golden(cuda):
    from srswa import page_gate as P
    g = golden("page_gate")
    _, _, per_page = (int(x) for x in g["params"])
    ids = t(g["ids"], cuda)
    S = ids.shape[1]
    saved = P._PAGE_SCOPE_PREFILL
    try:
        for scope in (0, 1):
            P._PAGE_SCOPE_PREFILL = bool(scope)
            for tag, kl in (("full", S), ("trunc", S - 37), ("pad", S + 50)):
                itm, ipi, qpi = P._build_page_aware_ids(Indexer(16, per_page), ids, IMG, MARK, kl)
                assert itm.dtype == torch.bool and ipi.dtype == torch.int64 and qpi.dtype == torch.int64
                np.testing.assert_array_equal(itm.cpu().numpy(), g[f"itm_s{scope}_{tag}"])
                np.testing.assert_array_equal(ipi.cpu().numpy(), g[f"ipi_s{scope}_{tag}"])
                np.testing.assert_array_equal(qpi.cpu().numpy(), g[f"qpi_s{scope}_{tag}"])
        assert P._build_page_aware_ids(Indexer(16, per_page), ids[3:], IMG, MARK, S) == (None, None, None)
        assert P._build_page_aware_ids(Indexer(16, per_page), ids, IMG, None, S) == (None, None, None)
    finally:
        P._PAGE_SCOPE_PREFILL = saved
    flat = P._build_flat_image_token_mask(Indexer(16, per_page), ids, IMG, S)
    np.testing.assert_array_equal(flat.cpu().numpy(), g["flat_itm"])


@pytest.mark.parametrize("bs", [16, 64])
def test_candidate_mask_golden(cuda, bs):
    from srswa import page_gate as P
    g = golden("page_gate")
    _, _, per_page = (int(x) for x in g["params"])
    B, S = g["ids"].shape
    nblk = -(-S // bs)
    pos = torch.arange(S, device=cuda)[None].expand(B, S).contiguous()
    itm, ipi, qpi, flat = (t(g[k], cuda) for k in ("itm_s1_full", "ipi_s1_full", "qpi_s1_full", "flat_itm"))
    for constraint in (1, 0):
        ix = Indexer(bs, per_page, bool(constraint))
        for ptag, pp in (("all", pos), ("chunk", t(g["pos_chunk"], cuda))):
            c = P._build_kl_candidate_mask(ix, pp, nblk, itm if constraint else flat, B, pp.shape[1],
                                           image_token_page_ids=ipi if constraint else None,
                                           query_token_page_ids=qpi if constraint else None)
            assert c.shape == (B, 1, pp.shape[1], nblk)
            np.testing.assert_array_equal(c[:, 0].cpu().numpy(), g[f"cand_bs{bs}_c{constraint}_{ptag}"])
    c = P._build_kl_candidate_mask(Indexer(bs, per_page, False), pos, nblk, None, B, S)
    np.testing.assert_array_equal(c[:, 0].cpu().numpy(), g[f"cand_bs{bs}_none"])
    # the DASH overlay's per-query domain: one launch for all queries
    dc = P._dash_block_cand(None, Indexer(bs, per_page), None, pos, itm, ipi, qpi, nblk, B, S)
    np.testing.assert_array_equal(dc.cpu().numpy(), g[f"cand_bs{bs}_c1_all"])
    # without the fallback (the reference's _build_page_aware_image_block_mask)
    raw = P._build_page_aware_image_block_mask(Indexer(bs, per_page), ipi, qpi, pos, nblk, S)
    ref = PG.page_aware_block_mask(g["ipi_s1_full"], g["qpi_s1_full"], pos.cpu().numpy(), nblk, bs)
    np.testing.assert_array_equal(raw[:, 0].cpu().numpy(), ref)
    blk = P._build_image_block_allow_mask(Indexer(bs, per_page), flat, nblk)
    np.testing.assert_array_equal(blk.cpu().numpy(), PG.image_block_allow(g["flat_itm"], nblk, bs))


@pytest.mark.parametrize("bs", [16, 64])
def test_decode_allow_golden(cuda, bs):
    from srswa import page_gate as P
    g = golden("page_gate")
    _, _, per_page = (int(x) for x in g["params"])
    ids = t(g["ids"], cuda)
    ix = Indexer(bs, per_page)
    cache = Cache(ids.shape[1])
    assert P._uocr_dash_decode_allow(ix, ids, cache) is None
    st = cache._uocr_pg
    for k in ("bmin", "bmax", "pp"):
        np.testing.assert_array_equal(st[k].cpu().numpy(), g[f"dec_bs{bs}_{k}"])
    np.testing.assert_array_equal(st["mcum"].cpu().numpy(), g[f"dec_bs{bs}_mcum0"])
    steps = t(g[f"dec_bs{bs}_steps"], cuda)
    for k, nb in enumerate(g[f"dec_bs{bs}_nblk"]):
        a = P._uocr_dash_decode_allow(ix, steps[:, k:k + 1], cache)
        cache.n += 1
        assert a.shape == (ids.shape[0], nb)
        np.testing.assert_array_equal(a.cpu().numpy(), g[f"dec_bs{bs}_allow"][k][:, :nb])
    assert P._uocr_dash_decode_allow(ix, steps[:, :1], Cache(5)) is None   # no prefill state


@pytest.mark.parametrize("bs,per_page", [(64, 273), (32, 5)])
def test_page_gate_long_rows_vs_oracle(cuda, bs, per_page):
    """Rows of 50 000 tokens (25 scan chunks): ids, candidates of a query
    subset, and a decode-allow sequence, bit-exact against the oracle."""
    from srswa import page_gate as P
    B, S = 3, 50000
    ids_np = long_rows(7 + bs, B, S, per_page)
    ids = t(ids_np, cuda)
    saved = P._PAGE_SCOPE_PREFILL
    try:
        for scope in (True, False):
            P._PAGE_SCOPE_PREFILL = scope
            for kl in (S, S - 1234, S + 777):
                itm, ipi, qpi = P._build_page_aware_ids(Indexer(bs, per_page), ids, IMG, MARK, kl)
                r_itm, r_ipi, r_qpi = PG.page_aware_ids(ids_np, IMG, MARK, kl, per_page, scope)
                np.testing.assert_array_equal(itm.cpu().numpy(), r_itm)
                np.testing.assert_array_equal(ipi.cpu().numpy(), r_ipi)
                np.testing.assert_array_equal(qpi.cpu().numpy(), r_qpi)
    finally:
        P._PAGE_SCOPE_PREFILL = saved
    nblk = -(-S // bs)
    rng = np.random.default_rng(3)
    pos_np = np.sort(rng.integers(-5, S + 5, (B, 600)), axis=1)     # out-of-range positions are clamped
    pos = t(pos_np, cuda)
    for constraint in (True, False):
        c = P._build_kl_candidate_mask(Indexer(bs, per_page, constraint), pos, nblk, itm, B, 600,
                                       image_token_page_ids=ipi, query_token_page_ids=qpi)
        ref = PG.kl_candidate_mask(pos_np, nblk, r_itm, bs, constraint, r_ipi, r_qpi)
        np.testing.assert_array_equal(c[:, 0].cpu().numpy(), ref)
    ix = Indexer(bs, per_page)
    cache = Cache(S)
    P._uocr_dash_decode_allow(ix, ids, cache)
    st = PG.decode_allow_prefill(ids_np, IMG, MARK, per_page, bs)
    for k in ("bmin", "bmax", "pp", "mcum"):
        np.testing.assert_array_equal(cache._uocr_pg[k].cpu().numpy(), st[k])
    new = rng.integers(0, 1000, (B, 70))
    new[:, 10] = MARK
    new[1, 40] = MARK
    for k in range(new.shape[1]):
        a = P._uocr_dash_decode_allow(ix, t(new[:, k:k + 1], cuda), cache)
        cache.n += 1
        ra, st = PG.decode_allow_step(st, new[:, k], MARK, cache.n, bs)
        np.testing.assert_array_equal(a.cpu().numpy(), ra)


def test_wide_block_page_sets(cuda):
    """Page ids built elsewhere may spread a block over 64 or more pages; such
    blocks are tested token by token."""
    from srswa import ops
    B, S, bs = 2, 640, 64
    rng = np.random.default_rng(5)
    ipi = np.full((B, S), -1, np.int64)
    ipi[0, 0:64] = np.arange(64) * 3          # one block over pages 0..189
    ipi[0, 64:100] = 7
    ipi[1, 128:192] = rng.integers(0, 500, 64)
    ipi[1, 300:310] = 499
    qpi = rng.integers(-1, 500, (B, S))
    qpi[0, :70] = np.arange(70) * 3 % 200
    pos = np.broadcast_to(np.arange(S), (B, S)).copy()
    nblk = S // bs
    desc = ops.page_block_desc(nblk, bs, ipi=t(ipi, cuda))
    for fb in (True, False):
        c = ops.page_cand_mask(desc, bs, pos=t(pos, cuda), qpi=t(qpi, cuda), ipi=t(ipi, cuda), fallback=fb)
        ref = PG.page_aware_block_mask(ipi, qpi, pos, nblk, bs)
        if fb:
            ref = ref | ~ref.any(-1, keepdims=True)
        np.testing.assert_array_equal(c.cpu().numpy(), ref)


def test_route_with_page_candidates(cuda):
    """The candidate mask feeds the fused router: its selections stay inside
    each query's candidates (or its fallback) and equal the oracle router with
    the same mask."""
    import math

    from oracle import srswa_oracle as O
    from srswa import dash_infer
    from srswa import page_gate as P
    B, S, bs, L, K, M, d = 1, 4096, 64, 4, 6, 12, 128
    ids_np = long_rows(11, B, S, 273)
    ids = t(ids_np, cuda)
    itm, ipi, qpi = P._build_page_aware_ids(Indexer(bs, 273), ids, IMG, MARK, S)
    nblk = S // bs
    pos = torch.arange(S, device=cuda)[None].contiguous()
    cand = P._dash_block_cand(None, Indexer(bs, 273), None, pos, itm, ipi, qpi, nblk, B, S)
    rng = np.random.default_rng(1)
    iq = O.bf16_round(rng.standard_normal((B, S, d)).astype(np.float32))
    ik = O.bf16_round(rng.standard_normal((B, S, d)).astype(np.float32))
    router = type("R", (), dict(block_size=bs, local_blocks=L, local_window=L * bs,
                                head_cls=torch.zeros(d, device=cuda), stage0="head_cls"))()
    p = dict(idx_scale=128 / math.sqrt(d), floor=1e-4, sigma=1.0, K=K, topm=M)
    topi, bias, valid = dash_infer.route(router, t(iq, cuda), t(ik, cuda), pos, nblk, cand, p)
    kb = O.kbar_summary(ik.reshape(B, nblk, bs, d), np.ones((B, nblk, bs), bool), np.zeros(d, np.float32))
    sc = O.block_scores_headcls(iq, kb, np.ones((B, nblk), bool), np.arange(S)[None], bs, L)
    r_topi, _, r_valid = O.infer_route_select(sc, cand.cpu().numpy(), p["idx_scale"], p["floor"], p["sigma"], K, M)
    ti, va, cn = topi.cpu().numpy(), valid.cpu().numpy(), cand.cpu().numpy()
    mism = 0
    for q in range(S):
        got = set(ti[0, q][va[0, q]].tolist())
        mism += got != set(r_topi[0, q][r_valid[0, q]].tolist())
        remote = sc[0, q] > -5e8
        allowed = remote & cn[0, q] if (remote & cn[0, q]).any() else remote
        assert all(allowed[c] for c in got)
    assert mism <= 2   # fp32 score ties only
