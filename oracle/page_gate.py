"""CPU oracle for the PageGate candidate masks -- TEST INFRASTRUCTURE ONLY.

Plain-numpy restatement of the reference's page-aware remote-candidate logic
(Unlimited-OCR 2, ``hf-model-code/``): token ids -> per-token page ids ->
per-query "same-page image block" candidate masks for the prefill router, and
the decode-side allow mask.  Only ``tests/`` and ``bench.py``'s reference arm
may import it; the product path (``srswa.page_gate``) runs CUDA kernels and
never imports this file.

Parity pin: ``tests/golden/make_golden.py`` (case ``page_gate``) runs the
reference's own methods on seeded token sequences and
``tests/test_oracle_golden.py`` checks every function here against them.

All integer arithmetic is int64, as in the reference (torch ``long``).
"""

from __future__ import annotations

import numpy as np

I64 = np.int64


def _fit(token_ids: np.ndarray, key_length: int) -> np.ndarray:
    """Truncate or right-pad (with -1) token ids to key_length columns
    (``_sparse_base_impl.py:2415-2417``, ``:2620-2623``)."""
    t = np.asarray(token_ids, dtype=I64)[:, :key_length]
    if t.shape[1] < key_length:
        t = np.pad(t, ((0, 0), (0, key_length - t.shape[1])), constant_values=-1)
    return t


def page_aware_ids(token_ids, img_id, page_id, key_length, per_page_image_tokens, page_scope_prefill):
    """(image_token_mask bool, image_token_page_ids int64, query_token_page_ids
    int64), each [B, key_length], or None when the row set has no image token
    or no query with a page.

    Follows ``DeepseekV2Indexer._build_page_aware_ids``
    (``hf-model-code/_sparse_base_impl.py:2404-2497``):
      cum   = inclusive count of <PAGE> markers;
      run   = inclusive count of image tokens;
      last  = index of the row's last image token (-1: none);
      pp    = cum[last] if last >= 0 else 0 (prompt pages); marker mode = pp > 0;
      image page  = marker mode ? cum - 1 : (run - 1) // per_page  (image tokens; else -1);
      query page  = j <= last ? (page_scope_prefill ? cum - 1 : -1)
                              : cum - 1 - (marker mode ? pp : 0);  negatives -> -1.
    """
    t = _fit(token_ids, key_length)
    B, S = t.shape
    img = t == img_id
    cum = np.cumsum(t == page_id, axis=1, dtype=I64)
    ar = np.arange(S, dtype=I64)
    last = (img.astype(I64) * (ar + 1)).max(axis=1, initial=0) - 1              # [B]
    pp = cum[np.arange(B), np.maximum(last, 0)] * (last >= 0)
    marker = (pp > 0)[:, None]
    per_page = max(1, int(per_page_image_tokens))
    run = np.cumsum(img, axis=1, dtype=I64) - 1
    ipi = np.where(marker, cum - 1, np.floor_divide(run, per_page))
    ipi = np.where(img, ipi, -1)
    raw = cum - 1
    resp = raw - np.where(marker, pp[:, None], 0)
    in_prefill = ar[None, :] <= last[:, None]
    qpi = np.where(in_prefill, raw, resp)
    if not page_scope_prefill:
        qpi = np.where(in_prefill, -1, qpi)
    qpi = np.where(qpi < 0, -1, qpi)
    if img.sum() == 0 or (qpi >= 0).sum() == 0:
        return None
    return img, ipi.astype(I64), qpi.astype(I64)


def flat_image_token_mask(token_ids, img_id, key_length):
    """``_build_flat_image_token_mask`` (``_sparse_base_impl.py:2609-2627``):
    [B, key_length] bool, or None without an image token."""
    m = _fit(token_ids, key_length) == img_id
    return None if m.sum() == 0 else m


def image_block_allow(image_token_mask, nblk, block_size):
    """``_build_image_block_allow_mask`` (``_sparse_base_impl.py:2392-2402``):
    [B, nblk] -- block holds an image token (padding / truncation to
    nblk * block_size tokens)."""
    m = np.asarray(image_token_mask, bool)
    B, S = m.shape
    n = nblk * block_size
    m = np.pad(m, ((0, 0), (0, max(0, n - S))))[:, :n]
    return m.reshape(B, nblk, block_size).any(-1)


def page_aware_block_mask(ipi, qpi, pos, nblk, block_size):
    """``_build_page_aware_image_block_mask`` (``_sparse_base_impl.py:2629-2648``):
    [B, C, nblk] -- block holds an image token whose page equals the query's
    page (query page = qpi[b, clamp(pos, 0, S_q - 1)], pages < 0 never match)."""
    ipi = np.asarray(ipi, I64)
    qpi = np.asarray(qpi, I64)
    pos = np.asarray(pos, I64)
    B, K = ipi.shape
    n = nblk * block_size
    kp = np.pad(ipi, ((0, 0), (0, max(0, n - K))), constant_values=-1)[:, :n].reshape(B, nblk, block_size)
    qp = np.take_along_axis(qpi, np.clip(pos, 0, qpi.shape[1] - 1), axis=1)       # [B, C]
    out = np.zeros((B, pos.shape[1], nblk), bool)
    for b in range(B):
        for c in np.unique(qp[b]):
            if c < 0:
                continue
            out[b, qp[b] == c] = (kp[b] == c).any(-1)
    return out


def kl_candidate_mask(pos, nblk, image_token_mask, block_size, image_bucket_constraint, ipi=None, qpi=None):
    """``_build_kl_candidate_mask`` (``_sparse_base_impl.py:2697-2730``):
    [B, C, nblk] bool (the reference's [B, 1, C, nblk] without the head axis).

    Same-page image blocks when the constraint is on and page ids exist, else
    all image blocks when an image-token mask exists, else all blocks; a query
    with no candidate anywhere falls back to all blocks."""
    pos = np.asarray(pos, I64)
    B, C = pos.shape
    if image_bucket_constraint and ipi is not None and qpi is not None:
        cand = page_aware_block_mask(ipi, qpi, pos, nblk, block_size)
    elif image_token_mask is not None:
        cand = np.broadcast_to(image_block_allow(image_token_mask, nblk, block_size)[:, None, :],
                               (B, C, nblk)).copy()
    else:
        cand = np.ones((B, C, nblk), bool)
    empty = ~cand.any(-1, keepdims=True)
    return cand | empty


def decode_allow_prefill(ids, img_id, page_id, per_page_image_tokens, block_size):
    """Prefill half of ``_uocr_dash_decode_allow``
    (``hf-model-code/modeling_unlimitedocr.py:497-514``): per KV block the
    [min, max] image page it holds (-1, -1 without image tokens), the prompt
    page count pp and the marker count.  Image page of a token:
    cum > 0 ? cum - 1 : (run - 1) // per_page."""
    ids = np.asarray(ids, I64)
    B, L = ids.shape
    img = ids == img_id
    cum = np.cumsum(ids == page_id, axis=1, dtype=I64)
    run = np.cumsum(img, axis=1, dtype=I64)
    per_page = max(1, int(per_page_image_tokens))
    page = np.where(cum > 0, cum - 1, np.floor_divide(run - 1, per_page))
    page = np.where(img, page, -1)
    pp = np.maximum.accumulate(np.where(img, cum, 0), axis=1)[:, -1]
    nblk = -(-L // block_size)
    pg = np.pad(page, ((0, 0), (0, nblk * block_size - L)), constant_values=-1).reshape(B, nblk, block_size)
    bmax = pg.max(-1)
    bmin = np.where(pg >= 0, pg, 1 << 30).min(-1)
    bmin = np.where(bmax >= 0, bmin, -1)
    return dict(bmin=bmin.astype(I64), bmax=bmax.astype(I64), pp=pp.astype(I64), mcum=cum[:, -1].copy())


def decode_allow_step(state, last_ids, page_id, total_len, block_size):
    """Decode half of ``_uocr_dash_decode_allow``
    (``modeling_unlimitedocr.py:515-528``): advances the marker count by the
    new token, derives the query's page (response pages restart at 0) and
    returns (allow [B, nblk] bool, new state); nblk = ceil(total_len / bs)."""
    mcum = state["mcum"] + (np.asarray(last_ids, I64) == page_id)
    qp = mcum - 1 - state["pp"]
    qp = np.where(qp >= 0, qp, -1)[:, None]
    nblk = -(-int(total_len) // block_size)
    bmin, bmax = state["bmin"], state["bmax"]
    same = (bmin >= 0) & (bmin <= qp) & (bmax >= qp) & (qp >= 0)
    open_row = (qp[:, 0] < 0) | ~same.any(-1)
    allow = np.zeros((bmin.shape[0], nblk), bool)
    n0 = min(nblk, same.shape[1])
    allow[:, :n0] = same[:, :n0]
    st = dict(state)
    st["mcum"] = mcum
    return allow | open_row[:, None], st
