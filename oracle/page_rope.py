"""CPU oracle for the page2d (two-axis) RoPE coordinates -- TEST INFRASTRUCTURE ONLY.

Plain-numpy restatement of the reference's page-aware rotary coordinates
(Unlimited-OCR 2, ``hf-model-code/_sparse_base_impl.py``): token ids ->
(token-in-page, page) coordinates, the two-axis rotary angles, their
application to q / k, and the decode-time coordinate update.  Only ``tests/``
may import it; the product path (``srswa.page_rope``) runs CUDA kernels.

Parity pin: ``tests/golden/make_golden.py`` (case ``page_rope``) runs the
reference's own methods and ``tests/test_oracle_golden.py`` checks this file
against them.
"""

from __future__ import annotations

import numpy as np

I64 = np.int64


def page_rope_pos(ids, img_id, page_id, key_length, span=0):
    """(tok_pos, page_pos, pf_cnt, n_pg) or None.

    Follows ``_build_page_rope_pos`` + ``_page_rope_offsets``
    (``_sparse_base_impl.py:2511-2570``): page = cum (prefill: up to the row's
    last image token) or cum - n_pages (response), n_pages = markers up to the
    last image token (every row needs one, else None); tok = running count of
    the token's page bucket minus one; pf_cnt[b, p] = prefill tokens of page p;
    span > 0 maps each page's prefill onto span steps (page 0 stays raw)."""
    t = np.asarray(ids, I64)[:, :key_length]
    if t.shape[1] < key_length:
        t = np.pad(t, ((0, 0), (0, key_length - t.shape[1])), constant_values=-1)
    B, S = t.shape
    img = t == img_id
    mk = t == page_id
    if not img.any() or not mk.any():
        return None
    cum = np.cumsum(mk, axis=1, dtype=I64)
    ar = np.arange(S, dtype=I64)
    last = (img.astype(I64) * (ar + 1)).max(axis=1) - 1
    npg = cum[np.arange(B), np.maximum(last, 0)] * (last >= 0)
    if not (npg > 0).all():
        return None
    pre = ar[None, :] <= last[:, None]
    page = np.maximum(np.where(pre, cum, cum - npg[:, None]), 0)
    n_pg = int(page.max()) + 1
    tok = np.zeros((B, S), I64)
    pf_cnt = np.zeros((B, n_pg), I64)
    for b in range(B):
        cnt = np.zeros(n_pg, I64)
        for j in range(S):
            p = page[b, j]
            cnt[p] += 1
            tok[b, j] = cnt[p] - 1
            if pre[b, j]:
                pf_cnt[b, p] += 1
    if span > 0:
        pf_k = np.take_along_axis(pf_cnt, page, axis=1)
        tf = tok.astype(np.float32)
        pre_v = np.rint(tf * np.float32(span) / np.maximum(pf_k, 1).astype(np.float32))
        post_v = np.float32(span) + (tok - pf_k).astype(np.float32)
        scaled = np.where(pre, pre_v, post_v).astype(I64)
        tok = np.where(page > 0, scaled, tok)
    return tok, page, pf_cnt, n_pg


def rotary2d_inv_freq(dim, base_tok, base_page, page_pairs, tok_freq_mode="resample"):
    """(inv_tok, inv_page) fp32 (``DeepseekV2IndexerRotary2D.__init__``,
    ``_sparse_base_impl.py:2019-2041``)."""
    half = dim // 2
    n_tok = half - page_pairs
    ar = np.arange(n_tok, dtype=np.float32)
    if tok_freq_mode == "truncate":
        inv_tok = 1.0 / (np.float32(base_tok) ** (ar * 2 / dim))
    else:
        inv_tok = 1.0 / (np.float32(base_tok) ** (ar / n_tok))
    inv_page = 1.0 / (np.float32(base_page) ** (np.arange(page_pairs, dtype=np.float32) / page_pairs))
    return inv_tok.astype(np.float32), inv_page.astype(np.float32)


def rotary2d_cos_sin(tok, page, inv_tok, inv_page, page_mod=0):
    """cos, sin [B, S, dim] fp32 (``DeepseekV2IndexerRotary2D.forward``,
    ``_sparse_base_impl.py:2043-2058``): angles tok * inv_tok on the first
    n_tok pairs, (page mod page_mod) * inv_page on the rest, concatenated
    twice."""
    p = np.asarray(page, I64)
    if page_mod > 0:
        p = np.mod(p, page_mod)
    a_tok = np.asarray(tok, I64).astype(np.float32)[:, :, None] * inv_tok[None, None, :]
    a_page = p.astype(np.float32)[:, :, None] * inv_page[None, None, :]
    ang = np.concatenate([a_tok, a_page], axis=-1)
    emb = np.concatenate([ang, ang], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def apply_rotary(x, cos, sin):
    """x [B, H, S, D] with cos / sin [B, S, D]: x * cos + rotate_half(x) * sin
    (transformers ``apply_rotary_pos_emb`` with unsqueeze_dim = 1)."""
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return x * cos[:, None] + rot * sin[:, None]


def decode_coords_step(state, new_ids, page_id):
    """Decode branch of ``_main_rope_coords`` (``_sparse_base_impl.py:1482-1489``):
    a <PAGE> token moves to the next page (clamped to n_pg - 1) and restarts
    the token axis at that page's prefill count; any other token advances it."""
    is_pg = np.asarray(new_ids, I64) == page_id
    page = np.where(is_pg, np.minimum(state["page"] + 1, state["n_pg"] - 1), state["page"])
    pg_start = np.take_along_axis(state["pf_cnt"], np.maximum(page, 0)[:, None], axis=1)[:, 0]
    tok = np.where(is_pg, pg_start, state["tok"] + 1)
    return dict(state, page=page, tok=tok)
