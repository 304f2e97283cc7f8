"""CPU oracle for the SR-SWA hot path -- TEST INFRASTRUCTURE ONLY.

This module is a plain-numpy restatement of the reference's SR-SWA math
(Unlimited-OCR 2, ``hf-model-code/`` plus the SGLang serving ops shipped in the
reference wheel).  It exists to *check* the CUDA library, never to stand in for
it: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
/ reference arm may import it.  The product path (``srswa``) never imports it and
fails loudly when its CUDA library is missing.

Parity pin: every function here is checked against golden vectors produced by
running the reference's own PyTorch functions and its Triton kernels under the
Triton CPU interpreter (``tests/golden/make_golden.py``; fixtures in
``tests/golden/*.npz``; test ``tests/test_oracle_golden.py``).

Numerics: inputs are float32 arrays (callers pass bf16-rounded values upcast to
fp32 when the GPU runs bf16).  Arithmetic is fp32 wherever the reference is fp32;
the entmax cumulative sums accumulate in float64 and round each prefix to fp32,
which is what torch's CPU ``cumsum`` does for fp32 tensors.

Reference citations use paths inside the reference project; ``whl:`` paths are
files inside ``wheel/sglang-0.5.20.dev10+g8d62f5fb9c-py3-none-any.whl``.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32

# Finite sentinels of the reference (hf-model-code/dash_attention.py:740-754,
# modeling_deepseekv2.py:65).
SCORE_NEG = F32(-1.0e9)
MASK_NEG = F32(-1.0e9)
ENTMAX_NEG = F32(-1.0e4)
ACT_CLAMP = F32(1.0e4)
LOG2E = 1.4426950408889634


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 -> fp32 (bit-exact with torch)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    u = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    # NaN stays NaN
    return np.where(np.isnan(x), x, out)


# ---------------------------------------------------------------------------
# a1: k-bar block summary
# ---------------------------------------------------------------------------
def kbar_summary(keys: np.ndarray, valid: np.ndarray, head_cls: np.ndarray) -> np.ndarray:
    """head_cls masked-softmax summary of each block of index keys.

    keys [..., bs, d] fp32, valid [..., bs] bool, head_cls [d] -> k_bar [..., d].

    Follows ``_block_scores_infer`` head_cls branch
    (hf-model-code/modeling_deepseekv2.py:391-408), identical to
    ``DashAttention._block_scores_headcls`` Stage 0
    (hf-model-code/dash_attention.py:1079-1119) and SGLang ``_summary_keys``
    (whl:sglang/srt/layers/attention/unlimited_dash_ops/dash_stage0.py:25-41):
    aw = clamp(k.hc / sqrt(d)); row max over VALID tokens only (0 for an empty
    block); e = exp(aw - max) * valid; w = e / max(sum e, 1e-6); k_bar = sum w k;
    non-finite -> 0.
    """
    keys = keys.astype(F32, copy=False)
    d = keys.shape[-1]
    inv_sqrt_d = F32(1.0 / math.sqrt(d))
    aw = (keys * head_cls.astype(F32)).sum(-1, dtype=F32) * inv_sqrt_d
    aw = np.clip(aw, -ACT_CLAMP, ACT_CLAMP)
    neg = np.finfo(F32).min
    row_max = np.where(valid, aw, neg).max(-1, keepdims=True)
    row_max = np.where(valid.any(-1, keepdims=True), row_max, F32(0.0))
    e = np.exp(aw - row_max).astype(F32) * valid.astype(F32)
    w = e / np.maximum(e.sum(-1, keepdims=True, dtype=F32), F32(1e-6))
    kb = (w[..., None] * keys).sum(-2, dtype=F32)
    return np.where(np.isfinite(kb), kb, F32(0.0)).astype(F32)


def kbar_contiguous(idx_k: np.ndarray, head_cls: np.ndarray, block_size: int, nblk: int):
    """[B,S,d] index keys -> (k_bar [B,nblk,d], block_has_tokens [B,nblk]).

    Pads S up to nblk*block_size with invalid tokens
    (hf-model-code/modeling_deepseekv2.py:391-399)."""
    B, S, d = idx_k.shape
    Sp = nblk * block_size
    kk = np.zeros((B, Sp, d), F32)
    n = min(S, Sp)
    kk[:, :n] = idx_k[:, :n]
    real = np.zeros((B, Sp), bool)
    real[:, :n] = True
    kk = kk.reshape(B, nblk, block_size, d)
    vm = real.reshape(B, nblk, block_size)
    return kbar_summary(kk, vm, head_cls), vm.any(-1)


# ---------------------------------------------------------------------------
# a2: remote block scores (head_cls) and the "indexer" token block-max variant
# ---------------------------------------------------------------------------
def block_scores_headcls(idx_q, k_bar, chunk_valid, q_pos, block_size, local_blocks):
    """[B,Lq,d] x [B,nblk,d] -> [B,Lq,nblk] remote-only scores.

    hf-model-code/modeling_deepseekv2.py:409-417: z = clamp(q.k_bar / sqrt(d));
    kept iff block c <= q_pos//bs - local_blocks and the block holds a token;
    SCORE_NEG elsewhere."""
    d = idx_q.shape[-1]
    inv_sqrt_d = F32(1.0 / math.sqrt(d))
    z = np.matmul(idx_q.astype(F32), np.swapaxes(k_bar, -1, -2).astype(F32)) * inv_sqrt_d
    z = np.clip(z, -ACT_CLAMP, ACT_CLAMP)
    nblk = k_bar.shape[1]
    qblk = q_pos.astype(np.int64) // block_size
    blk = np.arange(nblk)
    keep = (blk[None, None, :] <= (qblk[:, :, None] - local_blocks)) & chunk_valid[:, None, :]
    return np.where(keep, z, SCORE_NEG).astype(F32)


def block_scores_indexer(idx_q, idx_k, q_pos, nblk, block_size, local_window):
    """stage0 == "indexer": block max of token scores over remote keys.

    hf-model-code/modeling_deepseekv2.py:418-430 (same as
    DashAttention._block_scores, dash_attention.py:1036-1050): raw q.k (no
    1/sqrt(d)), clamp, future and local keys -> SCORE_NEG, pad to whole blocks
    with SCORE_NEG, amax per block."""
    B, S, d = idx_k.shape
    sc = np.matmul(idx_q.astype(F32), np.swapaxes(idx_k, -1, -2).astype(F32))
    sc = np.clip(sc, -ACT_CLAMP, ACT_CLAMP)
    kpos = np.arange(S)
    pos = q_pos.astype(np.int64)[:, :, None]
    future = kpos[None, None, :] > pos
    local = (kpos[None, None, :] > (pos - local_window)) & ~future
    sc = np.where(future | local, SCORE_NEG, sc)
    Sp = nblk * block_size
    if Sp > S:
        sc = np.concatenate([sc, np.full(sc.shape[:-1] + (Sp - S,), SCORE_NEG, F32)], -1)
    return sc[..., :Sp].reshape(B, sc.shape[1], nblk, block_size).max(-1).astype(F32)


def block_max_score(q, k, pos, seg, block_size, num_key_blocks, local_window):
    """``triton_block_max_score`` semantics (hf-model-code/sparse_gather_triton.py:445-524).

    q [B,C,D], k [B,Sk,D], pos/seg [B,C] -> [B,C,nblk] fp32 = max over keys j of
    the block with seg <= j < max(pos - LW + 1, 0) and j < Sk of q.k (unscaled);
    -inf where no key qualifies."""
    B, C, D = q.shape
    Sk = k.shape[1]
    lw = block_size if local_window is None else max(1, int(local_window))
    sc = np.matmul(q.astype(F32), np.swapaxes(k, -1, -2).astype(F32))  # [B,C,Sk]
    j = np.arange(Sk)
    ls = np.maximum(pos.astype(np.int64) - (lw - 1), 0)
    ok = (j[None, None, :] < ls[:, :, None]) & (j[None, None, :] >= seg.astype(np.int64)[:, :, None])
    sc = np.where(ok, sc, -np.inf).astype(F32)
    out = np.full((B, C, num_key_blocks), -np.inf, F32)
    for c in range(num_key_blocks):
        lo, hi = c * block_size, min((c + 1) * block_size, Sk)
        if lo < hi:
            out[:, :, c] = sc[:, :, lo:hi].max(-1)
    return out


# ---------------------------------------------------------------------------
# a4: candidacy + top-M 1.5-entmax + hard top-K + centred log-prior bias
# ---------------------------------------------------------------------------
def entmax15(x: np.ndarray) -> np.ndarray:
    """Exact sort-based 1.5-entmax over the last axis.

    hf-model-code/dash_attention.py:772-800 (same math in
    whl:.../unlimited_dash_ops/dash_router.py:28-52): X = (x - max)/2; sort
    descending; tau_rho = mean_rho - sqrt(max(0, (1 - rho*(meansq_rho -
    mean_rho^2))/rho)); support = #(tau_rho <= X_sorted_rho) clamped >= 1;
    p = max(X - tau_support, 0)^2.  Prefix sums accumulate in float64 and
    round to fp32 (torch CPU cumsum semantics for fp32)."""
    x = x.astype(F32)
    X = (x - x.max(-1, keepdims=True)) / F32(2.0)
    Xs = -np.sort(-X, axis=-1)
    n = X.shape[-1]
    rho = np.arange(1, n + 1, dtype=F32)
    cs = np.cumsum(Xs.astype(np.float64), -1).astype(F32)
    cs2 = np.cumsum((Xs * Xs).astype(F32).astype(np.float64), -1).astype(F32)
    mean = cs / rho
    mean_sq = cs2 / rho
    ss = rho * (mean_sq - mean * mean)
    delta = (F32(1.0) - ss) / rho
    tau = mean - np.sqrt(np.maximum(delta, F32(0.0)))
    support = (tau <= Xs).sum(-1, keepdims=True)
    support = np.maximum(support, 1)
    tau_star = np.take_along_axis(tau, support - 1, -1)
    p = np.maximum(X - tau_star, F32(0.0))
    return (p * p).astype(F32)


def topk_desc(x: np.ndarray, k: int):
    """Top-k along the last axis, descending; ties keep the lower index first."""
    order = np.argsort(-x, axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(x, order, -1), order


def infer_route_select(block_scores, block_cand, idx_scale, floor, sigma, K, topm):
    """``_infer_route_select`` (hf-model-code/modeling_deepseekv2.py:339-362).

    Returns (topi int64 [B,Lq,K], bias fp32 [B,Lq,K], valid bool [B,Lq,K]).
    remote = score > SCORE_NEG/2; cand = remote & block_cand (falls back to
    remote on rows where that is empty); x = cand ? score*idx_scale : -1e4;
    top-M by x, entmax15 over those M, keep the first K; bias = (log(max(p,
    floor)) - mean over valid)/sigma on valid slots, 0 elsewhere."""
    sc = block_scores.astype(F32)
    remote = sc > SCORE_NEG * F32(0.5)
    cand = remote if block_cand is None else (remote & block_cand.astype(bool))
    empty = ~cand.any(-1, keepdims=True)
    cand = np.where(empty, remote, cand)
    x = np.where(cand, sc * F32(idx_scale), ENTMAX_NEG).astype(F32)
    x = np.where(np.isfinite(x), x, ENTMAX_NEG)
    nblk = x.shape[-1]
    M = max(1, min(int(topm), nblk)) if int(topm) > 0 else nblk
    xv, xi = topk_desc(x, M)
    prior = entmax15(xv)
    is_cand = np.take_along_axis(cand, xi, -1)
    KK = max(1, min(int(K), M))
    xi, prior, valid = xi[..., :KK], prior[..., :KK], is_cand[..., :KK]
    logp = np.log(np.maximum(prior, F32(floor))).astype(F32)
    cnt = np.maximum(valid.sum(-1, keepdims=True), 1).astype(F32)
    mu = np.where(valid, logp, F32(0.0)).sum(-1, keepdims=True, dtype=F32) / cnt
    bias = np.where(valid, (logp - mu) * F32(1.0 / sigma), F32(0.0)).astype(F32)
    return xi.astype(np.int64), bias, valid


# ---------------------------------------------------------------------------
# a5: dedup of repeated block ids inside a row
# ---------------------------------------------------------------------------
def dedup_rows(sel: np.ndarray) -> np.ndarray:
    """Repeated non-negative ids inside a row -> -1, keeping the first slot.

    hf-model-code/sparse_gather_triton.py:418-427 and
    sparse_gather_e2e_triton.py:387-394 (the reference keeps one occurrence
    per id; which slot survives is left to its sort, this keeps the lowest)."""
    sel = sel.astype(np.int64).copy()
    flat = sel.reshape(-1, sel.shape[-1])
    for r in range(flat.shape[0]):
        seen = set()
        for s in range(flat.shape[1]):
            v = flat[r, s]
            if v < 0:
                continue
            if v in seen:
                flat[r, s] = -1
            else:
                seen.add(v)
    return sel


# ---------------------------------------------------------------------------
# a6/a7/a8: gather-attention over (selected blocks, keys < local start) U window
# ---------------------------------------------------------------------------
def _key_masks(T, Sk, sel_row_blocks, seg, lw, block_size):
    """Boolean [T,Sk] masks (remote-kept, local-kept) and the slot owning each
    remote key ([T,Sk] int, -1 if none) for one (b, index head)."""
    t = np.arange(T)[:, None]
    j = np.arange(Sk)[None, :]
    seg = seg.astype(np.int64)[:, None]
    ls = np.maximum(t - lw + 1, seg)
    causal = (j <= t) & (j >= seg)
    local = causal & (j >= ls)
    slot_of = np.full((T, Sk), -1, np.int64)
    kb = j // block_size
    for s in range(sel_row_blocks.shape[1]):
        blk = sel_row_blocks[:, s][:, None]
        hit = (blk >= 0) & (kb == blk) & (slot_of < 0)
        slot_of = np.where(hit, s, slot_of)
    remote = causal & (j < ls) & (slot_of >= 0)
    return remote, local, np.where(remote, slot_of, -1)


def gather_attention_fwd(q, k, v, sel, seg, block_size, scale, local_window, bias=None):
    """Forward of the fused gather-attention (K1 / K5 semantics).

    q [B,T,HQ,D], k/v [B,Sk,Hkv,D], sel [B,HI,T,S] (deduped, -1 pad),
    seg [B,T] segment start (zeros when unpacked), bias [B,T,S] per-slot remote
    bias or None.  Returns (o [B,T,HQ,D] fp32, lse [B,T,HQ] natural log).

    hf-model-code/sparse_gather_triton.py:35-122 and
    sparse_gather_e2e_triton.py:36-121: per query t the kept keys are the
    local window [ls, t] with ls = max(t - LW + 1, seg_t) and the keys of the
    selected blocks that lie in [seg_t, ls); logits scale*q.k, plus the slot's
    bias on remote keys; one softmax over the union; empty rows give o = 0 and
    lse = -inf.  Equal to the dense masks of DashAttention._forward_dense
    (dash_attention.py:1230-1260) and build_block_mask + eager softmax
    (_sparse_base_impl.py:3518-3557, 1803-1836)."""
    B, T, HQ, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    HI = sel.shape[1]
    lw = block_size if local_window is None else max(1, int(local_window))
    G = HQ // Hkv
    o = np.zeros((B, T, HQ, v.shape[-1]), F32)
    lse = np.full((B, T, HQ), -np.inf, F32)
    for b in range(B):
        for hi in range(HI):
            remote, local, slot_of = _key_masks(T, Sk, sel[b, hi], seg[b], lw, block_size)
            keep = remote | local
            add = np.zeros((T, Sk), F32)
            if bias is not None:
                bsl = bias[b].astype(F32)  # [T,S]
                add = np.where(remote, np.take_along_axis(bsl, np.maximum(slot_of, 0), 1), F32(0.0))
            for hq in range(HQ):
                if (hq * HI) // HQ != hi:
                    continue
                hk = hq // G
                s = (q[b, :, hq].astype(F32) @ k[b, :, hk].astype(F32).T) * F32(scale) + add
                s = np.where(keep, s, -np.inf)
                m = s.max(-1, keepdims=True)
                ms = np.where(np.isfinite(m), m, F32(0.0))
                p = np.exp(s - ms).astype(F32)
                l = p.sum(-1, keepdims=True, dtype=F32)
                ls_ = np.where(l > 0, l, F32(1.0))
                o[b, :, hq] = (p @ v[b, :, hk].astype(F32)) / ls_
                lse[b, :, hq] = np.where(l[:, 0] > 0, (ms + np.log(ls_))[:, 0], -np.inf)
    return o, lse


def gather_attention_bwd(q, k, v, do, sel, seg, block_size, scale, local_window, bias=None):
    """Analytic backward of ``gather_attention_fwd``.

    Returns (dq, dk, dv, d_bias [B,T,S] or None), fp32.  Same math as the
    reference's autograd kernels K2/K3 (sparse_gather_triton.py:125-279) and
    K6/K7 (sparse_gather_e2e_triton.py:124-275): P = softmax, dV = P^T dO,
    dP = dO V^T, Delta = rowsum(O*dO), dS = P(dP - Delta), dQ = scale dS K,
    dK = scale dS^T Q, d_bias[t, slot] = sum over heads and the slot's remote
    keys of dS."""
    B, T, HQ, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    S = sel.shape[-1]
    HI = sel.shape[1]
    lw = block_size if local_window is None else max(1, int(local_window))
    G = HQ // Hkv
    dq = np.zeros_like(q, dtype=F32)
    dk = np.zeros(k.shape, F32)
    dv = np.zeros(v.shape, F32)
    dbias = np.zeros((B, T, S), F32) if bias is not None else None
    for b in range(B):
        for hi in range(HI):
            remote, local, slot_of = _key_masks(T, Sk, sel[b, hi], seg[b], lw, block_size)
            keep = remote | local
            add = np.zeros((T, Sk), F32)
            if bias is not None:
                add = np.where(remote, np.take_along_axis(bias[b].astype(F32), np.maximum(slot_of, 0), 1), F32(0.0))
            for hq in range(HQ):
                if (hq * HI) // HQ != hi:
                    continue
                hk = hq // G
                qh = q[b, :, hq].astype(F32)
                kh = k[b, :, hk].astype(F32)
                vh = v[b, :, hk].astype(F32)
                s = (qh @ kh.T) * F32(scale) + add
                s = np.where(keep, s, -np.inf)
                m = s.max(-1, keepdims=True)
                ms = np.where(np.isfinite(m), m, F32(0.0))
                p = np.exp(s - ms).astype(F32)
                l = p.sum(-1, keepdims=True, dtype=F32)
                p = p / np.where(l > 0, l, F32(1.0))
                oh = p @ vh
                doh = do[b, :, hq].astype(F32)
                dv[b, :, hk] += p.T @ doh
                dp = doh @ vh.T
                delta = (oh * doh).sum(-1, keepdims=True, dtype=F32)
                ds = p * (dp - delta)
                dq[b, :, hq] = F32(scale) * (ds @ kh)
                dk[b, :, hk] += F32(scale) * (ds.T @ qh)
                if dbias is not None:
                    dsr = np.where(remote, ds, F32(0.0))
                    for s_ in range(S):
                        dbias[b, :, s_] += np.where(slot_of == s_, dsr, F32(0.0)).sum(-1, dtype=F32)
    return dq, dk, dv, dbias


# ---------------------------------------------------------------------------
# a6/a7 at full size: the same math for a few sampled query rows or key blocks
# of one (b, index head = 0), so that the oracle finishes in seconds where the
# dense [T, Sk] masks above would not fit (T = 16k .. 32k).
# ---------------------------------------------------------------------------
def gather_row_keys(t, sel_row, seg_t, block_size, local_window, Sk):
    """Keys attended by query t and the slot of each one's remote block (-1:
    local key).  Row t of ``_key_masks``: remote keys are those of the
    selected blocks in [seg_t, ls) with ls = max(t - LW + 1, seg_t), local keys
    [ls, t]; a repeated block keeps its first slot
    (sparse_gather_e2e_triton.py:82-98, dash_attention.py:1230-1260)."""
    lw = block_size if local_window is None else max(1, int(local_window))
    t, seg_t = int(t), int(seg_t)
    ls = max(t - lw + 1, seg_t)
    keys, slots, seen = [], [], set()
    for s_, c in enumerate(np.asarray(sel_row).tolist()):
        if c < 0 or c in seen:
            continue
        seen.add(c)
        j = np.arange(c * block_size, min((c + 1) * block_size, Sk))
        j = j[(j >= seg_t) & (j < ls) & (j <= t)]
        keys.append(j)
        slots.append(np.full(len(j), s_, np.int64))
    loc = np.arange(ls, min(t + 1, Sk))
    keys.append(loc)
    slots.append(np.full(len(loc), -1, np.int64))
    return np.concatenate(keys).astype(np.int64), np.concatenate(slots)


def _row_probs(qr, kk, keys_slot, bias_row, scale, G):
    """Softmax row of one query over its keys: qr [HQ,D], kk [n,Hkv,D] ->
    (p [HQ,n], s [HQ,n], lse [HQ]) with the slot bias on remote keys."""
    kq = np.repeat(kk, G, axis=1) if G > 1 else kk            # [n, HQ, D]
    s = np.einsum("hd,nhd->hn", qr.astype(F32), kq.astype(F32)).astype(F32) * F32(scale)
    if bias_row is not None:
        add = np.where(keys_slot >= 0, np.asarray(bias_row, F32)[np.maximum(keys_slot, 0)], F32(0.0))
        s = s + add[None, :]
    if s.shape[1] == 0:
        return s, s, np.full(qr.shape[0], -np.inf, F32)
    m = s.max(-1, keepdims=True)
    p = np.exp(s - m).astype(F32)
    l = p.sum(-1, keepdims=True, dtype=F32)
    return p / l, s, (m + np.log(l))[:, 0].astype(F32)


def gather_rows_fwd(q_b, k_b, v_b, sel_b, seg_b, rows, block_size, scale, local_window, bias_b=None):
    """Forward of ``gather_attention_fwd`` for the sampled query rows of one
    batch element with one index head.  q_b [T,HQ,D], k_b/v_b [Sk,Hkv,D],
    sel_b [T,S] (-1 pad), seg_b [T], bias_b [T,S] or None ->
    (o [R,HQ,D], lse [R,HQ]) fp32."""
    HQ, Hkv = q_b.shape[1], k_b.shape[1]
    G = HQ // Hkv
    o = np.zeros((len(rows), HQ, v_b.shape[-1]), F32)
    lse = np.full((len(rows), HQ), -np.inf, F32)
    for i, t in enumerate(rows):
        keys, slot = gather_row_keys(t, sel_b[t], seg_b[t], block_size, local_window, k_b.shape[0])
        if len(keys) == 0:
            continue
        p, _, lse[i] = _row_probs(q_b[t], k_b[keys], slot, None if bias_b is None else bias_b[t], scale, G)
        vq = np.repeat(v_b[keys], G, axis=1) if G > 1 else v_b[keys]
        o[i] = np.einsum("hn,nhd->hd", p, vq.astype(F32))
    return o, lse


def gather_rows_bwd(q_b, k_b, v_b, do_b, sel_b, seg_b, rows, block_size, scale, local_window, bias_b=None):
    """dQ and d_bias of ``gather_attention_bwd`` for sampled query rows (one
    batch element, one index head): -> (dq [R,HQ,D], d_bias [R,S] or None)."""
    HQ, Hkv = q_b.shape[1], k_b.shape[1]
    G = HQ // Hkv
    S = sel_b.shape[-1]
    dq = np.zeros((len(rows), HQ, q_b.shape[-1]), F32)
    db = np.zeros((len(rows), S), F32) if bias_b is not None else None
    for i, t in enumerate(rows):
        keys, slot = gather_row_keys(t, sel_b[t], seg_b[t], block_size, local_window, k_b.shape[0])
        if len(keys) == 0:
            continue
        p, _, _ = _row_probs(q_b[t], k_b[keys], slot, None if bias_b is None else bias_b[t], scale, G)
        kq = (np.repeat(k_b[keys], G, axis=1) if G > 1 else k_b[keys]).astype(F32)
        vq = (np.repeat(v_b[keys], G, axis=1) if G > 1 else v_b[keys]).astype(F32)
        o = np.einsum("hn,nhd->hd", p, vq)
        dor = do_b[t].astype(F32)
        dp = np.einsum("hd,nhd->hn", dor, vq)
        delta = (o * dor).sum(-1, keepdims=True, dtype=F32)
        ds = p * (dp - delta)
        dq[i] = F32(scale) * np.einsum("hn,nhd->hd", ds, kq)
        if db is not None:
            dsum = ds.sum(0, dtype=F32)
            for s_ in range(S):
                db[i, s_] = dsum[slot == s_].sum(dtype=F32)
    return dq, db


def gather_block_bwd(q_b, k_b, v_b, do_b, o_b, lse_b, sel_b, seg_b, c, block_size, scale, local_window,
                     bias_b=None):
    """dK and dV of ``gather_attention_bwd`` for the keys of key block c (one
    batch element, one index head), given the forward's o [T,HQ,D] and lse
    [T,HQ] (natural log) -- the tensors the reference's autograd saves and
    hands its dK/dV kernels (K3 / K7, sparse_gather_e2e_triton.py:209-275).
    Every query whose key set holds a key of block c contributes:
    dV_j = sum_t P_tj dO_t, dK_j = scale sum_t dS_tj q_t, with P from lse and
    dS = P (dP - Delta), Delta = rowsum(o * dO).  -> (dk, dv) [n, Hkv, D]."""
    T, HQ = q_b.shape[0], q_b.shape[1]
    Hkv = k_b.shape[1]
    G = HQ // Hkv
    Sk = k_b.shape[0]
    lw = block_size if local_window is None else max(1, int(local_window))
    j0, j1 = c * block_size, min((c + 1) * block_size, Sk)
    kj = k_b[j0:j1].astype(F32)
    vj = v_b[j0:j1].astype(F32)
    dk = np.zeros_like(kj)
    dv = np.zeros_like(vj)
    cand = set(range(j0, min(T, j1 + lw)))
    cand.update(np.nonzero((sel_b == c).any(-1))[0].tolist())
    for t in sorted(cand):
        if t < j0:
            continue
        keys, slot = gather_row_keys(t, sel_b[t], seg_b[t], block_size, lw, Sk)
        inb = (keys >= j0) & (keys < j1)
        if not inb.any():
            continue
        kk, ks = keys[inb] - j0, slot[inb]
        s = np.einsum("hd,nhd->hn", q_b[t].astype(F32), np.repeat(kj[kk], G, axis=1)).astype(F32) * F32(scale)
        if bias_b is not None:
            s = s + np.where(ks >= 0, np.asarray(bias_b[t], F32)[np.maximum(ks, 0)], F32(0.0))[None, :]
        p = np.exp(s - lse_b[t][:, None]).astype(F32)                     # [HQ, n]
        dor = do_b[t].astype(F32)
        dp = np.einsum("hd,nhd->hn", dor, np.repeat(vj[kk], G, axis=1))
        delta = (o_b[t].astype(F32) * dor).sum(-1, keepdims=True, dtype=F32)
        ds = p * (dp - delta)
        for hq in range(HQ):
            hk = hq // G
            dv[kk, hk] += p[hq][:, None] * dor[hq][None, :]
            dk[kk, hk] += F32(scale) * ds[hq][:, None] * q_b[t, hq].astype(F32)[None, :]
    return dk, dv


# ---------------------------------------------------------------------------
# f4: DSA gather-KL distillation (training stage "sparse", one index head)
# ---------------------------------------------------------------------------
def _kl_row_keys(sel_row, pos, seg, block_size, local_window, Sk):
    """Keys of one query row in the KL: the selected blocks' keys (a repeated
    block counts once) below the local window start and not in the future,
    same segment: the token-level keep of _kl_chunk_core
    (_sparse_base_impl.py:2071-2120) for keep_block = the row's blocks."""
    ls = max(int(pos) - (int(local_window) - 1), 0)
    out, seen = [], set()
    for b in np.asarray(sel_row).tolist():
        if b < 0 or b in seen:
            continue
        seen.add(b)
        j = np.arange(b * block_size, min((b + 1) * block_size, Sk))
        out.append(j[(j <= pos) & (j < ls) & (j >= seg)])
    return np.concatenate(out).astype(np.int64) if out else np.zeros(0, np.int64)


def _bf16_if(x, flag):
    return bf16_round(x) if flag else x


def gather_kl(idx_q, idx_k, q_main, k_main, sel, pos, seg, block_size, local_window, scaling, bf16_logits=True,
              g=None):
    """Per-row KL(P_teacher || P_student) over each query row's selected
    remote keys, and (with g, dLoss/dkl per row) its gradients to the index
    q / k.  _kl_chunk_core and the gather branch of select_and_kl_loss
    (hf-model-code/_sparse_base_impl.py:2071-2137, 3397-3450):
      student s_j = idx_q . idx_k[j] (bf16 matmul output when the index
      tensors are bf16), log-softmax over the row's kept keys;
      teacher t_hj = (q_main[h] . k_main[j, h // group]) (bf16 output) *
      scaling, softmax per head over the same keys, averaged over the heads;
      kl = sum_j p_j (log max(p_j, 1e-12) - log p_idx_j); valid = any key.
    idx_q [B,C,d], idx_k [B,Sk,d], q_main [B,C,H,D], k_main [B,Sk,Hkv,D],
    sel [B,C,S] (-1 pad), pos / seg [B,C] (global position, segment start).
    Returns (kl [B,C], valid [B,C]) or, with g [B,C], also (d_idx_q
    [B,C,d], d_idx_k [B,Sk,d]): ds_j = g (P p_idx_j - p_j) on kept keys,
    P = sum of p over them."""
    B, C, d = idx_q.shape
    Sk = idx_k.shape[1]
    H, Hkv = q_main.shape[2], k_main.shape[2]
    G = H // Hkv
    kl = np.zeros((B, C), F32)
    valid = np.zeros((B, C), bool)
    dq = np.zeros(idx_q.shape, F32) if g is not None else None
    dk = np.zeros(idx_k.shape, F32) if g is not None else None
    for b in range(B):
        for c in range(C):
            keys = _kl_row_keys(sel[b, c], pos[b, c], 0 if seg is None else seg[b, c], block_size, local_window, Sk)
            if len(keys) == 0:
                continue
            valid[b, c] = True
            s = _bf16_if((idx_k[b, keys].astype(F32) @ idx_q[b, c].astype(F32)).astype(F32), bf16_logits)
            lse_s = s.max() + np.log(np.exp(s - s.max()).sum(dtype=F32))
            logp_idx = (s - lse_s).astype(F32)
            p = np.zeros(len(keys), F32)
            for h in range(H):
                t = _bf16_if((k_main[b, keys, h // G].astype(F32) @ q_main[b, c, h].astype(F32)).astype(F32),
                             bf16_logits) * F32(scaling)
                e = np.exp(t - t.max()).astype(F32)
                p += e / e.sum(dtype=F32)
            p /= F32(H)
            kl[b, c] = (p * (np.log(np.maximum(p, F32(1e-12))) - logp_idx)).sum(dtype=F32)
            if g is not None:
                p_idx = np.exp(logp_idx).astype(F32)
                ds = (F32(g[b, c]) * (p.sum(dtype=F32) * p_idx - p)).astype(F32)
                dq[b, c] = ds @ idx_k[b, keys].astype(F32)
                np.add.at(dk[b], keys, ds[:, None] * idx_q[b, c].astype(F32)[None, :])
    if g is None:
        return kl, valid
    return kl, valid, dq, dk


def decode_attend(q, k_all, v_all, topi, bias, valid, q_pos, block_size, local_window, scale):
    """``_decode_attend`` (hf-model-code/modeling_deepseekv2.py:455-481), fp32.

    q [B,H,Lq,D], k_all/v_all [B,Hkv,S,D], topi/bias/valid [B,Lq,K],
    q_pos [B,Lq] -> [B,H,Lq,D].  Selected blocks (valid slots) add their bias
    to causal keys outside the window; the window (q_pos - LW, q_pos] is
    unbiased and wins on overlap; everything else is dropped."""
    B, H, Lq, D = q.shape
    Hkv, S = k_all.shape[1], k_all.shape[2]
    nblk = (S + block_size - 1) // block_size
    kpos = np.arange(S)
    out = np.zeros((B, H, Lq, v_all.shape[-1]), F32)
    for b in range(B):
        for i in range(Lq):
            blk = np.full(nblk, MASK_NEG, F32)
            for s in range(topi.shape[-1]):
                blk[int(topi[b, i, s])] = bias[b, i, s] if valid[b, i, s] else MASK_NEG
            base = blk[kpos // block_size]
            p = int(q_pos[b, i])
            causal = kpos <= p
            local = causal & (kpos > p - local_window)
            keep = causal & (local | (base > MASK_NEG * F32(0.5)))
            madd = np.where(local, F32(0.0), base)
            madd = np.where(keep, madd, -np.inf).astype(F32)
            for h in range(H):
                hk = h // (H // Hkv)
                s_ = (k_all[b, hk].astype(F32) @ q[b, h, i].astype(F32)) * F32(scale) + madd
                mx = s_.max()
                e = np.exp(s_ - mx).astype(F32)
                out[b, h, i] = (e / e.sum(dtype=F32)) @ v_all[b, hk].astype(F32)
    return out


# ---------------------------------------------------------------------------
# a9: paged decode (SGLang dash_sparse_attn_decode) + LSE merge
# ---------------------------------------------------------------------------
def paged_decode(q, k_cache, v_cache, topk_idx, blk_bias, block_table, seq_lens,
                 sm_scale, decode_query_len, local_blocks, block_size):
    """``dash_sparse_attn_decode`` semantics
    (whl:sglang/srt/layers/attention/unlimited_dash_ops/attend_triton.py:307-518,
    600-715, merge common.py:43-89).

    q [R*dql,H,D]; k_cache/v_cache [P,BS,Hkv,D]; topk_idx/blk_bias [Hkv or 1,
    R*dql,K] (slot -1 = unused, skipped wherever it sits); block_table [R,W];
    seq_lens [R].  Query row n of request r sits at p = seq_len - dql + n%dql;
    remote keys of a selected block: pos < min(p+1, p-LW+1 .. ) i.e.
    pos <= p and pos < max(0, p - LW + 1), biased; local keys: blocks
    p//BS - j (j = 0..L), max(0, p-LW+1) <= pos <= p, unbiased.
    Returns (out [R*dql,H,D] fp32, lse [R*dql,H] natural log)."""
    N = q.shape[0]
    dql = decode_query_len
    req = np.arange(N) // dql
    pos = np.asarray(seq_lens, np.int64)[req] - dql + np.arange(N) % dql
    return _paged_rows(q, k_cache, v_cache, topk_idx, blk_bias, block_table, req, pos, sm_scale, local_blocks,
                       block_size)


def paged_prefill(q, k_cache, v_cache, topk_idx, blk_bias, block_table, cu_seqlens_q, prefix_lens, sm_scale,
                  local_blocks, block_size, rows=None):
    """``dash_sparse_attn`` semantics, one program per query token
    (whl:sglang/srt/layers/attention/unlimited_dash_ops/attend_triton.py:88-292,
    523-597): row i of request r (cu_seqlens_q[r] <= i < cu_seqlens_q[r+1])
    sits at p = prefix_lens[r] + i - cu_seqlens_q[r]; remote keys of its
    selected blocks below the window start (pos <= p - LW), biased; local
    keys [p - LW + 1, p], unbiased.  The reference walks the first
    count(slot >= 0) slots, so valid slots must come first (as its router
    packs them).  rows: compute only these rows (the others stay 0 / -inf).
    Returns (out [N,H,D] fp32, lse [N,H] natural log)."""
    cu = np.asarray(cu_seqlens_q, np.int64)
    N = int(cu[-1])
    req = np.searchsorted(cu, np.arange(N), side="right") - 1
    pos = np.asarray(prefix_lens, np.int64)[req] + np.arange(N) - cu[req]
    return _paged_rows(q, k_cache, v_cache, topk_idx, blk_bias, block_table, req, pos, sm_scale, local_blocks,
                       block_size, rows)


def _paged_rows(q, k_cache, v_cache, topk_idx, blk_bias, block_table, req, pos_of_row, sm_scale, local_blocks,
                block_size, rows=None):
    """One softmax per (row, head) over the row's remote keys (selected
    blocks, pos <= p and pos < p - LW + 1, slot bias) and window keys."""
    N, H, D = q.shape
    Hkv = k_cache.shape[2]
    G = H // Hkv
    lw = local_blocks * block_size
    out = np.zeros((N, H, v_cache.shape[-1]), F32)
    lse = np.full((N, H), -np.inf, F32)
    for n in (range(N) if rows is None else rows):
        r = int(req[n])
        p = int(pos_of_row[n])
        lws = max(0, p - lw + 1)
        for h in range(H):
            hk = h // G
            ti = topk_idx[min(hk, topk_idx.shape[0] - 1), n]
            bb = None if blk_bias is None else blk_bias[min(hk, blk_bias.shape[0] - 1), n]
            keys, vals, adds = [], [], []
            for s, blk in enumerate(ti):
                blk = int(blk)
                if blk < 0:
                    continue
                page = int(block_table[r, blk])
                for i in range(block_size):
                    pos = blk * block_size + i
                    if pos <= p and pos < lws:
                        keys.append(k_cache[page, i, hk])
                        vals.append(v_cache[page, i, hk])
                        adds.append(0.0 if bb is None else float(bb[s]))
            qb = p // block_size
            for j in range(local_blocks + 1):
                blk = qb - j
                if blk < 0:
                    continue
                page = int(block_table[r, blk])
                for i in range(block_size):
                    pos = blk * block_size + i
                    if lws <= pos <= p:
                        keys.append(k_cache[page, i, hk])
                        vals.append(v_cache[page, i, hk])
                        adds.append(0.0)
            if not keys:
                continue
            K_ = np.stack(keys).astype(F32)
            V_ = np.stack(vals).astype(F32)
            s_ = (K_ @ q[n, h].astype(F32)) * F32(sm_scale) + np.asarray(adds, F32)
            mx = s_.max()
            e = np.exp(s_ - mx).astype(F32)
            l = e.sum(dtype=F32)
            out[n, h] = (e @ V_) / l
            lse[n, h] = mx + np.log(l)
    return out, lse


def win_bounds_decode(allow, seq_lens, nd, max_block, block_size, local_blocks, decode_query_len, tile):
    """Remote page span of each decode row from its allow mask [nd, WQ]
    (whl:.../unlimited_dash_ops/route_triton.py:466-526): (lo, hi) = first
    and one past the last allowed block among the live remote blocks
    (c <= q_blk - L, c * bs < seq_len, c < min(W, WQ)); with none, (0, 0)
    when the row has no remote block at all, else (0, live width
    min(W, max(nblk, 1))); fit = hi - lo <= tile.  q_blk truncates toward
    zero (Triton integer division).  -> lo, hi int32 [nd], fit int8 [nd]."""
    W, WQ = int(max_block), allow.shape[1]
    lo = np.zeros(nd, np.int32)
    hi = np.zeros(nd, np.int32)
    fit = np.zeros(nd, np.int8)
    for row in range(nd):
        seq = int(seq_lens[row // decode_query_len])
        q_pos = seq - decode_query_len + row % decode_query_len
        q_blk = int(q_pos / block_size)            # truncation toward zero
        off = np.arange(min(W, WQ))
        keep = (allow[row, :len(off)] != 0) & (off <= q_blk - local_blocks) & (off * block_size < seq)
        nb = (seq + block_size - 1) // block_size
        if keep.any():
            lo_v, hi_v = int(off[keep].min()), int(off[keep].max()) + 1
        else:
            no_remote = seq <= 0 or (q_blk - local_blocks) < 0
            lo_v, hi_v = 0, (0 if no_remote else min(W, max(nb, 1)))
        lo[row], hi[row], fit[row] = lo_v, hi_v, int(hi_v - lo_v <= tile)
    return lo, hi, fit


def lse_merge(o_parts, lse_parts):
    """Merge split-KV partials: o = sum_c w_c o_c / sum_c w_c with
    w_c = exp(lse_c - max lse); parts with lse = -inf weigh 0
    (whl:.../unlimited_dash_ops/common.py:43-89, natural-log form).
    o_parts [C,...,D], lse_parts [C,...] -> (o [...,D], lse [...])."""
    mx = lse_parts.max(0)
    mxs = np.where(np.isfinite(mx), mx, F32(0.0))
    w = np.where(np.isfinite(lse_parts), np.exp(lse_parts - mxs), F32(0.0)).astype(F32)
    den = w.sum(0)
    o = (w[..., None] * o_parts).sum(0) / np.where(den > 0, den, F32(1.0))[..., None]
    lse = np.where(den > 0, mxs + np.log(np.where(den > 0, den, F32(1.0))), -np.inf)
    return o.astype(F32), lse.astype(F32)


def decode_attend_one(q, k_all, v_all, topi, bias, valid, p, block_size, local_window, scale):
    """``_decode_attend`` for one request and one query row, vectorised over
    heads (the CPU-baseline unit; same math as ``decode_attend``).
    q [H,D], k_all/v_all [Hkv,S,D], topi/bias/valid [K] -> [H,D]."""
    H, D = q.shape
    Hkv, S, _ = k_all.shape
    nblk = (S + block_size - 1) // block_size
    blk = np.full(nblk, MASK_NEG, F32)
    for s in range(topi.shape[0]):
        blk[int(topi[s])] = bias[s] if valid[s] else MASK_NEG
    kpos = np.arange(S)
    base = blk[kpos // block_size]
    causal = kpos <= p
    local = causal & (kpos > p - local_window)
    keep = causal & (local | (base > MASK_NEG * F32(0.5)))
    madd = np.where(keep, np.where(local, F32(0.0), base), -np.inf).astype(F32)
    G = H // Hkv
    qg = q.reshape(Hkv, G, D).astype(F32)
    s_ = np.matmul(qg, np.swapaxes(k_all, 1, 2).astype(F32)) * F32(scale) + madd   # [Hkv,G,S]
    s_ = s_ - s_.max(-1, keepdims=True)
    e = np.exp(s_).astype(F32)
    e /= e.sum(-1, keepdims=True, dtype=F32)
    return np.matmul(e, v_all.astype(F32)).reshape(H, -1)


# ---------------------------------------------------------------------------
# composite: one decode step of the HF inference path (CPU baseline unit)
# ---------------------------------------------------------------------------
def decode_step_reference(q, k_all, v_all, idx_q, idx_k, head_cls, q_pos, block_size,
                          local_blocks, K, topm, idx_scale, floor, sigma, scale):
    """_block_scores_infer -> _infer_route_select -> _decode_attend
    (hf-model-code/modeling_deepseekv2.py:520-529), the reference's CPU decode
    step: k_bar is recomputed over every block and the attend is dense over the
    whole cache."""
    S = idx_k.shape[1]
    nblk = (S + block_size - 1) // block_size
    kb, cv = kbar_contiguous(idx_k, head_cls, block_size, nblk)
    sc = block_scores_headcls(idx_q, kb, cv, q_pos, block_size, local_blocks)
    topi, bias, valid = infer_route_select(sc, None, idx_scale, floor, sigma, K, topm)
    out = decode_attend(q, k_all, v_all, topi, bias, valid, q_pos, block_size,
                        local_blocks * block_size, scale)
    return out, topi, bias, valid
