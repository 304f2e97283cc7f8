"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures under tests/golden/ were written by tests/golden/make_golden.py,
which runs the reference's PyTorch SR-SWA functions, its Triton kernels under
the Triton CPU interpreter, and the SGLang serving ops from the reference wheel.
These tests need no GPU and no reference checkout.
"""

import numpy as np
import pytest

from conftest import golden
from oracle import srswa_oracle as O


def _sets_equal_except_ties(topi_a, topi_b, valid, scores, tol=1e-5):
    """Selected index sets per row must match; a mismatch is allowed only when
    the differing blocks' scores tie (within tol) with the row's boundary."""
    bad = 0
    for idx in np.ndindex(topi_a.shape[:-1]):
        va = valid[idx]
        a = set(topi_a[idx][va].tolist())
        b = set(topi_b[idx][va].tolist())
        if a != b:
            s = scores[idx]
            diff = [s[i] for i in (a ^ b)]
            kth = min(s[i] for i in a | b)
            if max(abs(x - kth) for x in diff) > tol * max(1.0, abs(kth)):
                bad += 1
    return bad


def test_entmax_golden():
    g = golden("entmax")
    y = O.entmax15(g["x"])
    np.testing.assert_allclose(y, g["y"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("tag", ["hc0", "hc1"])
def test_route_headcls_golden(tag):
    g = golden("route")
    BS, L, K, M = (int(x) for x in g["params"])
    idx_scale, floor, sigma = (float(x) for x in g["fparams"])
    hc = np.zeros(128, np.float32) if tag == "hc0" else g["hc1"]
    B, S, d = g["idx_k"].shape
    nblk = (S + BS - 1) // BS
    kb, cv = O.kbar_contiguous(g["idx_k"], hc, BS, nblk)
    sc = O.block_scores_headcls(g["idx_q"], kb, cv, g["q_pos"], BS, L)
    ref = g[f"scores_{tag}"]
    np.testing.assert_allclose(sc, ref, rtol=2e-5, atol=2e-5)
    topi, bias, valid = O.infer_route_select(ref, None, idx_scale, floor, sigma, K, M)
    np.testing.assert_array_equal(valid, g[f"valid_{tag}"])
    assert _sets_equal_except_ties(topi, g[f"topi_{tag}"], valid, ref) == 0
    np.testing.assert_allclose(bias, g[f"bias_{tag}"], rtol=1e-5, atol=1e-5)


def test_route_cand_and_params_golden():
    g = golden("route")
    BS, L, K, M = (int(x) for x in g["params"])
    idx_scale, floor, sigma = (float(x) for x in g["fparams"])
    sc = g["scores_hc0"]
    topi, bias, valid = O.infer_route_select(sc, g["cand"], idx_scale, floor, sigma, K, M)
    np.testing.assert_array_equal(valid, g["valid_cand"])
    assert _sets_equal_except_ties(topi, g["topi_cand"], valid, sc) == 0
    np.testing.assert_allclose(bias, g["bias_cand"], rtol=1e-5, atol=1e-5)
    s2, f2, sg2, K2, M2 = g["fparams2"]
    topi, bias, valid = O.infer_route_select(sc, None, s2, f2, sg2, int(K2), int(M2))
    np.testing.assert_array_equal(valid, g["valid_p2"])
    assert _sets_equal_except_ties(topi, g["topi_p2"], valid, sc) == 0
    np.testing.assert_allclose(bias, g["bias_p2"], rtol=1e-5, atol=1e-5)


def test_route_indexer_golden():
    g = golden("route")
    BS, L, _, _ = (int(x) for x in g["params"])
    B, S, d = g["idx_k"].shape
    nblk = (S + BS - 1) // BS
    sc = O.block_scores_indexer(g["idx_q"], g["idx_k"], g["q_pos"], nblk, BS, L * BS)
    np.testing.assert_allclose(sc, g["scores_indexer"], rtol=2e-5, atol=2e-4)


def test_decode_attend_golden():
    g = golden("decode_attend")
    BS, L, K, M = (int(x) for x in g["params"])
    out = O.decode_attend(g["q"], g["k"], g["v"], g["topi"], g["bias"], g["valid"],
                          g["q_pos"], BS, L * BS, float(g["scale"]))
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=1e-5)


def test_decode_step_golden():
    """full HF decode step (k_bar + scores + select + attend) on the oracle."""
    g = golden("decode_attend")
    BS, L, K, M = (int(x) for x in g["params"])
    d = g["idx_k"].shape[-1]
    out, topi, bias, valid = O.decode_step_reference(
        g["q"], g["k"], g["v"], g["idx_q"], g["idx_k"], np.zeros(d, np.float32), g["q_pos"],
        BS, L, K, M, 128.0 / np.sqrt(d), 1e-4, 1.0, float(g["scale"]))
    assert _sets_equal_except_ties(topi, g["topi"], valid, g["scores"]) == 0
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=1e-5)


def _sel_from_topi(topi, valid):
    return np.where(valid, topi, -1)[:, None]


def test_forward_dense_golden():
    g = golden("forward_dense")
    BS, L = (int(x) for x in g["params"])
    q, k, v = (np.swapaxes(g[n], 1, 2) for n in ("q", "k", "v"))  # -> [B,T,H,D]
    sel = _sel_from_topi(g["topi"], g["valid"])
    B, T = sel.shape[0], sel.shape[2]
    seg = np.zeros((B, T), np.int64)
    bias = np.where(g["valid"], g["bias"], 0).astype(np.float32)
    o, lse = O.gather_attention_fwd(q, k, v, sel, seg, BS, float(g["scale"]), L * BS, bias)
    np.testing.assert_allclose(np.swapaxes(o, 1, 2), g["o"], rtol=1e-4, atol=2e-5)
    do = np.swapaxes(g["do"], 1, 2)
    dq, dk, dv, db = O.gather_attention_bwd(q, k, v, do, sel, seg, BS, float(g["scale"]), L * BS, bias)
    for name, mine in (("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(np.swapaxes(mine, 1, 2), g[name], rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(np.where(g["valid"], db, 0), np.where(g["valid"], g["dbias"], 0),
                               rtol=1e-3, atol=1e-4)


def test_gather_triton_golden():
    g = golden("gather_triton")
    BS, LW = (int(x) for x in g["params"])
    q, k, v = (np.swapaxes(g[n], 1, 2) for n in ("q", "k", "v"))
    T = q.shape[1]
    seg = (np.arange(T)[None, :] - g["pos"]).astype(np.int64)
    sel = O.dedup_rows(g["sel"])
    o, lse = O.gather_attention_fwd(q, k, v, sel, seg, BS, float(g["scale"]), LW)
    np.testing.assert_allclose(np.swapaxes(o, 1, 2), g["o"], rtol=1e-4, atol=2e-5)
    do = np.swapaxes(g["do"], 1, 2)
    dq, dk, dv, _ = O.gather_attention_bwd(q, k, v, do, sel, seg, BS, float(g["scale"]), LW)
    for name, mine in (("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(np.swapaxes(mine, 1, 2), g[name], rtol=1e-3, atol=1e-4)


def test_gather_e2e_golden():
    g = golden("gather_e2e")
    BS, LW = (int(x) for x in g["params"])
    q, k, v = (np.swapaxes(g[n], 1, 2) for n in ("q", "k", "v"))
    B, T = q.shape[:2]
    sel = O.dedup_rows(g["sel"])
    seg = np.zeros((B, T), np.int64)
    o, _ = O.gather_attention_fwd(q, k, v, sel, seg, BS, float(g["scale"]), LW, g["bias"])
    np.testing.assert_allclose(np.swapaxes(o, 1, 2), g["o"], rtol=1e-4, atol=2e-5)
    do = np.swapaxes(g["do"], 1, 2)
    dq, dk, dv, db = O.gather_attention_bwd(q, k, v, do, sel, seg, BS, float(g["scale"]), LW, g["bias"])
    for name, mine in (("dq", dq), ("dk", dk), ("dv", dv)):
        np.testing.assert_allclose(np.swapaxes(mine, 1, 2), g[name], rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(db, g["dbias"], rtol=1e-3, atol=1e-4)


def test_block_max_golden():
    g = golden("block_max")
    BS, LW, nblk = (int(x) for x in g["params"])
    out = O.block_max_score(g["q"], g["k"], g["pos"], g["seg"], BS, nblk, LW)
    ref = g["out"]
    assert np.array_equal(np.isneginf(out), np.isneginf(ref))
    fin = np.isfinite(ref)
    np.testing.assert_allclose(out[fin], ref[fin], rtol=1e-5, atol=1e-4)


def test_paged_golden():
    g = golden("paged")
    BS, L, Kb, M = (int(x) for x in g["params"])
    idx_scale, floor, sigma, sm_scale = (float(x) for x in g["fparams"])
    R, W = g["block_table"].shape
    d = g["idx_q"].shape[-1]
    # k_bar of every page in use
    for r in range(R):
        n = int(g["seq_lens"][r])
        nb = (n + BS - 1) // BS
        pages = g["block_table"][r, :nb]
        pos = np.arange(nb)[:, None] * BS + np.arange(BS)[None, :]
        kb = O.kbar_summary(g["idx_cache"][pages], pos < n, g["hc"])
        np.testing.assert_allclose(kb, g["kbar"][pages], rtol=1e-5, atol=1e-6)
    # decode scores off the page cache
    qpos = g["seq_lens"].astype(np.int64) - 1
    kb_rows = g["kbar"][g["block_table"]]                      # [R,W,d]
    cv = (np.arange(W)[None, :] * BS) < g["seq_lens"][:, None]
    sc = O.block_scores_headcls(g["idx_q"][:, None], kb_rows, cv, qpos[:, None], BS, L)[:, 0]
    np.testing.assert_allclose(sc, g["scores"], rtol=2e-5, atol=2e-5)
    topi, bias, valid = O.infer_route_select(sc, None, idx_scale, floor, sigma, Kb, M)
    ref_idx = g["idx"][:, :Kb]
    mine = np.where(valid, topi, -1)
    assert _sets_equal_except_ties(mine, ref_idx, valid, sc) == 0
    np.testing.assert_allclose(bias, g["bias"][:, :Kb], rtol=1e-5, atol=1e-5)
    out, _ = O.paged_decode(g["q"], g["k_cache"], g["v_cache"], g["idx"][None], g["bias"][None],
                            g["block_table"], g["seq_lens"], sm_scale, 1, L, BS)
    np.testing.assert_allclose(out, g["out"], rtol=1e-4, atol=2e-5)


def test_lse_merge_matches_single_pass():
    rng = np.random.default_rng(0)
    s = rng.standard_normal((3, 50)).astype(np.float32)
    v = rng.standard_normal((50, 8)).astype(np.float32)
    parts_o, parts_l = [], []
    for lo, hi in ((0, 20), (20, 20), (20, 50)):
        if hi == lo:
            parts_o.append(np.zeros((3, 8), np.float32))
            parts_l.append(np.full(3, -np.inf, np.float32))
            continue
        ss = s[:, lo:hi]
        m = ss.max(-1, keepdims=True)
        e = np.exp(ss - m)
        parts_o.append((e @ v[lo:hi]) / e.sum(-1, keepdims=True))
        parts_l.append((m + np.log(e.sum(-1, keepdims=True)))[:, 0])
    o, lse = O.lse_merge(np.stack(parts_o), np.stack(parts_l))
    e = np.exp(s - s.max(-1, keepdims=True))
    np.testing.assert_allclose(o, (e @ v) / e.sum(-1, keepdims=True), rtol=1e-5, atol=1e-6)


# ---------------------------------------------------------------- PageGate
def test_page_gate_ids_golden():
    from oracle import page_gate as PG
    g = golden("page_gate")
    img, mark, per_page = (int(x) for x in g["params"])
    ids = g["ids"]
    S = ids.shape[1]
    for scope in (0, 1):
        for tag, kl in (("full", S), ("trunc", S - 37), ("pad", S + 50)):
            itm, ipi, qpi = PG.page_aware_ids(ids, img, mark, kl, per_page, bool(scope))
            np.testing.assert_array_equal(itm, g[f"itm_s{scope}_{tag}"])
            np.testing.assert_array_equal(ipi, g[f"ipi_s{scope}_{tag}"])
            np.testing.assert_array_equal(qpi, g[f"qpi_s{scope}_{tag}"])
    assert g["none_text_only"].all() and PG.page_aware_ids(ids[3:], img, mark, S, per_page, True) is None
    np.testing.assert_array_equal(PG.flat_image_token_mask(ids, img, S), g["flat_itm"])


@pytest.mark.parametrize("bs", [16, 64])
def test_page_gate_cand_golden(bs):
    from oracle import page_gate as PG
    g = golden("page_gate")
    B, S = g["ids"].shape
    nblk = -(-S // bs)
    pos = np.broadcast_to(np.arange(S), (B, S))
    for constraint in (1, 0):
        for ptag, pp in (("all", pos), ("chunk", g["pos_chunk"])):
            c = PG.kl_candidate_mask(pp, nblk, g["itm_s1_full"] if constraint else g["flat_itm"], bs,
                                     bool(constraint), g["ipi_s1_full"] if constraint else None,
                                     g["qpi_s1_full"] if constraint else None)
            np.testing.assert_array_equal(c, g[f"cand_bs{bs}_c{constraint}_{ptag}"])
    np.testing.assert_array_equal(PG.kl_candidate_mask(pos, nblk, None, bs, False), g[f"cand_bs{bs}_none"])


@pytest.mark.parametrize("bs", [16, 64])
def test_page_gate_decode_allow_golden(bs):
    from oracle import page_gate as PG
    g = golden("page_gate")
    img, mark, per_page = (int(x) for x in g["params"])
    ids = g["ids"]
    st = PG.decode_allow_prefill(ids, img, mark, per_page, bs)
    for k in ("bmin", "bmax", "pp"):
        np.testing.assert_array_equal(st[k], g[f"dec_bs{bs}_{k}"])
    np.testing.assert_array_equal(st["mcum"], g[f"dec_bs{bs}_mcum0"])
    n = ids.shape[1]
    for k, nb in enumerate(g[f"dec_bs{bs}_nblk"]):
        allow, st = PG.decode_allow_step(st, g[f"dec_bs{bs}_steps"][:, k], mark, n + 1, bs)
        n += 1
        assert allow.shape[1] == nb
        np.testing.assert_array_equal(allow, g[f"dec_bs{bs}_allow"][k][:, :nb])


# ---------------------------------------------------------------- page2d RoPE
def _bf16_bits(a):
    return (np.asarray(a).astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_page_rope_pos_golden():
    from oracle import page_rope as PR
    g = golden("page_rope")
    ids = g["ids"]
    S = ids.shape[1]
    for span in (0, 64):
        for tag, kl in (("full", S), ("trunc", S - 20), ("pad", S + 30)):
            tok, page, pf, n_pg = PR.page_rope_pos(ids, 128815, 128827, kl, span)
            np.testing.assert_array_equal(tok, g[f"tok_sp{span}_{tag}"])
            np.testing.assert_array_equal(page, g[f"page_sp{span}_{tag}"])
            np.testing.assert_array_equal(pf, g[f"pfcnt_sp{span}_{tag}"])
    assert g["bail"].all()
    assert PR.page_rope_pos(g["bail_ids"], 128815, 128827, S) is None
    assert PR.page_rope_pos(g["text_ids"], 128815, 128827, S) is None


def test_page_rope_tables_and_apply_golden():
    from oracle import page_rope as PR
    g = golden("page_rope")
    tok, page, sub = g["tok_sp0_full"], g["page_sp0_full"], g["rot_sub"]
    for ci, (bt, bp, pairs, mode, pmod) in enumerate(((10000.0, 256.0, 1, "resample", 2),
                                                      (500000.0, 256.0, 8, "truncate", 0))):
        it, ip = PR.rotary2d_inv_freq(128, bt, bp, pairs, mode)
        np.testing.assert_allclose(it, g[f"rot{ci}_inv_tok"], rtol=2e-6)
        np.testing.assert_allclose(ip, g[f"rot{ci}_inv_page"], rtol=2e-6)
        cos, sin = PR.rotary2d_cos_sin(tok, page, g[f"rot{ci}_inv_tok"], g[f"rot{ci}_inv_page"], pmod)
        np.testing.assert_allclose(cos[:, sub, :64], g[f"rot{ci}_cos_f32"], atol=2e-6)
        np.testing.assert_allclose(sin[:, sub, :64], g[f"rot{ci}_sin_f32"], atol=2e-6)
        np.testing.assert_allclose(cos[:, sub, :64], _bf16_bits(g[f"rot{ci}_cos_bf16"]), atol=4e-3)
    cos, sin = PR.rotary2d_cos_sin(tok, page, g["rot0_inv_tok"], g["rot0_inv_page"], 2)
    P = g["qx"].shape[2]
    q = PR.apply_rotary(_bf16_bits(g["qx"]), cos[:, :P], sin[:, :P])
    np.testing.assert_allclose(q, _bf16_bits(g["qe"]), atol=2e-2, rtol=1e-2)


def test_page_rope_decode_golden():
    from oracle import page_rope as PR
    g = golden("page_rope")
    st = dict(page=g["dec_page0"], tok=g["dec_tok0"], pf_cnt=g["dec_pfcnt"], n_pg=int(g["dec_npg"]))
    tok, page, pf, n_pg = PR.page_rope_pos(g["ids"], 128815, 128827, g["ids"].shape[1])
    np.testing.assert_array_equal(st["page"], page[:, -1])
    np.testing.assert_array_equal(st["tok"], tok[:, -1])
    assert n_pg == st["n_pg"]
    for k in range(g["dec_steps"].shape[1]):
        st = PR.decode_coords_step(st, g["dec_steps"][:, k], 128827)
        np.testing.assert_array_equal(st["tok"], g["dec_tok"][k])
        np.testing.assert_array_equal(st["page"], g["dec_page"][k])


def _prefill_router_rows(g):
    """The oracle's HF router (_block_scores_infer + _infer_route_select) on
    the varlen prefill rows of the paged_prefill fixture."""
    BS, L, topm, budget = (int(x) for x in g["params"][:4])
    idx_scale, floor, sigma = (float(x) for x in g["fparams"][:3])
    bt, seq, ctx, cu = g["block_table"], g["seq_lens"], g["context_lens"], g["cu_seqlens_q"]
    W = bt.shape[1]
    N = int(cu[-1])
    out = []
    for n in range(N):
        r = int(g["row2req"][n])
        p = int(ctx[r]) + n - int(cu[r])
        kb = g["kbar"][bt[r]][None]
        cv = (np.arange(W) * BS < int(seq[r]))[None]
        sc = O.block_scores_headcls(g["idx_q"][n][None, None], kb, cv, np.array([[p]]), BS, L)
        cand = g["allow"][n, :W][None, None].astype(bool)
        topi, bias, valid = O.infer_route_select(sc, cand, idx_scale, floor, sigma, budget, topm)
        out.append((topi[0, 0], bias[0, 0], valid[0, 0]))
    return out


def test_paged_prefill_golden():
    """SGLang prefill serving ops (interpreted from the wheel): the varlen
    paged attend K8, the k_bar refresh of a kbar_all_plan, the decode scan
    window K14, and the varlen router, whose selected sets equal the HF
    router's (with W <= topm the entmax runs over every candidate in both, so
    the biases agree too)."""
    g = golden("paged_prefill")
    BS, L, topm, budget, dql, tile = (int(x) for x in g["params"])
    scale = float(g["fparams"][3])
    ti, tb = g["out_idx"][:, :budget], g["out_bias"][:, :budget]
    out, _ = O.paged_prefill(g["q"], g["k_cache"], g["v_cache"], ti[None], tb[None], g["block_table"],
                             g["cu_seqlens_q"], g["context_lens"], scale, L, BS)
    np.testing.assert_allclose(out, g["out"], rtol=1e-5, atol=1e-5)
    kb = g["kbar_before"].copy()
    for pg, tk in zip(g["plan_pages"], g["plan_tok"]):
        if tk > 0:
            kb[pg] = O.kbar_summary(g["idx_cache"][pg][None], (np.arange(BS) < tk)[None], g["hc"])[0]
    np.testing.assert_allclose(kb, g["kbar"], rtol=1e-6, atol=1e-6)
    lo, hi, fit = O.win_bounds_decode(g["dallow"], g["seq_lens"], len(g["lo"]), g["block_table"].shape[1], BS, L,
                                      dql, tile)
    assert (lo == g["lo"]).all() and (hi == g["hi"]).all() and (fit == g["fit"]).all()
    for n, (topi, bias, valid) in enumerate(_prefill_router_rows(g)):
        ref = {int(b): float(x) for b, x in zip(g["out_idx"][n], g["out_bias"][n]) if b >= 0}
        mine = {int(b): float(x) for b, x, v in zip(topi, bias, valid) if v}
        assert set(ref) == set(mine), n
        for b in ref:
            assert abs(ref[b] - mine[b]) < 1e-4, (n, b)


def test_gather_kl_golden():
    """DSA sparse-stage KL distillation (_kl_chunk_core, one index head) and
    its gradients to the index q / k: the oracle restatement against the
    reference's own bf16 outputs (packed batch included)."""
    g = golden("gather_kl")
    BS, LW = (int(x) for x in g["params"])
    kl, valid, dq, dk = O.gather_kl(g["idx_q"], g["idx_k"], g["q_main"], g["k_main"], g["sel"], g["pos"], g["seg"],
                                    BS, LW, float(g["scaling"]), bf16_logits=True, g=g["gout"])
    np.testing.assert_allclose(kl, g["kl"], rtol=1e-3, atol=1e-4)
    assert (g["kl"][~valid] == 0).all()
    # the reference's gradients pass through bf16 casts: bf16 tolerance
    np.testing.assert_allclose(dq, g["d_idx_q"], rtol=1e-2, atol=2e-2)
    np.testing.assert_allclose(dk, g["d_idx_k"], rtol=1e-2, atol=2e-2)
