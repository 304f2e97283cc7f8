"""Drop-ins for the PageGate candidate logic of the reference: which remote key
blocks a query may select (image blocks of its own page), on CUDA kernels.

Indexer methods (``hf-model-code/_sparse_base_impl.py``, class
DeepseekV2Indexer; ``self`` is the indexer, only block_size,
per_page_image_tokens, image_bucket_constraint and q_proj are read):

* ``_build_page_aware_ids(self, source_input_ids, img_context_token_id,
  page_token_id, key_length)``                                   (:2404-2497)
* ``_build_flat_image_token_mask(self, source_input_ids,
  img_context_token_id, key_length)``                            (:2609-2627)
* ``_build_image_block_allow_mask(self, image_token_mask,
  num_key_blocks)``                                              (:2392-2402)
* ``_build_page_aware_image_block_mask(self, image_token_page_ids,
  query_token_page_ids, pos_chunk, num_key_blocks, cq)``         (:2629-2648)
* ``_build_kl_candidate_mask(self, pos_chunk, num_key_blocks,
  image_token_mask, batch, cq, image_token_page_ids=None,
  query_token_page_ids=None)``                                   (:2697-2730)

DASH overlay functions:

* ``_dash_block_cand(self, idx, router, pos_ids, itm, ipi, qpi, nblk, bsz,
  q_len)`` (``modeling_deepseekv2.py:108-122``): one launch for every query
  instead of the reference's q_chunk loop; same [B, S, nblk] result.
* ``_uocr_dash_decode_allow(indexer, input_ids, cache)``
  (``modeling_unlimitedocr.py:482-528``): the prefill call records the
  per-block page range in ``cache._uocr_pg`` and returns None; each decode
  call returns the [B, nblk] allow mask (the marker count advances in place).
  The block size must divide 2048.

Same return values and ``None`` cases as the reference.  The page-scope
switch for prefill queries is the reference's ``_PAGE_SCOPE_PREFILL`` (env
``PAGE_SCOPE_PREFILL``); after ``srswa.dropin.install`` it is read from the
reference module, so ``configure_dash_inference`` keeps controlling it.
"""

from __future__ import annotations

import os

import torch

from . import ops

_PAGE_SCOPE_PREFILL = os.environ.get("PAGE_SCOPE_PREFILL", "0") == "1"
_scope_source = None   # module whose _PAGE_SCOPE_PREFILL is authoritative (set by dropin.install)


def _scope() -> bool:
    if _scope_source is not None and hasattr(_scope_source, "_PAGE_SCOPE_PREFILL"):
        return bool(_scope_source._PAGE_SCOPE_PREFILL)
    return _PAGE_SCOPE_PREFILL


def _device(self, fallback: torch.Tensor) -> torch.device:
    qp = getattr(self, "q_proj", None)
    w = getattr(qp, "weight", None)
    if w is not None and w.is_cuda:
        return w.device
    if fallback.is_cuda:
        return fallback.device
    return torch.device("cuda", torch.cuda.current_device())


@torch.no_grad()
def _build_page_aware_ids(self, source_input_ids, img_context_token_id, page_token_id, key_length):
    """(image_token_mask bool, image_token_page_ids int64, query_token_page_ids
    int64), each [B, key_length], or (None, None, None)."""
    if source_input_ids is None or img_context_token_id is None or page_token_id is None:
        return None, None, None
    if source_input_ids.ndim != 2:
        return None, None, None
    ids = source_input_ids.to(device=_device(self, source_input_ids))
    itm, ipi, qpi, flags = ops.page_ids(ids, img_context_token_id, page_token_id, int(key_length),
                                        max(1, int(self.per_page_image_tokens)), _scope())
    has_img, has_page = flags.tolist()   # the reference's `.sum() == 0` tests read the device too
    if not has_img or not has_page:
        return None, None, None
    return itm, ipi, qpi


@torch.no_grad()
def _build_flat_image_token_mask(self, source_input_ids, img_context_token_id, key_length):
    """[B, key_length] bool image-token mask, or None."""
    if source_input_ids is None or img_context_token_id is None:
        return None
    if source_input_ids.ndim != 2:
        return None
    ids = source_input_ids[..., :key_length].to(device=_device(self, source_input_ids))
    if ids.shape[-1] < key_length:
        ids = torch.nn.functional.pad(ids, (0, key_length - ids.shape[-1]), value=-1)
    mask = ids == img_context_token_id
    if not bool(mask.any()):
        return None
    return mask


@torch.no_grad()
def _build_image_block_allow_mask(self, image_token_mask, num_key_blocks):
    """[B, num_key_blocks] bool: the block holds an image token."""
    desc = ops.page_block_desc(int(num_key_blocks), int(self.block_size), itm=image_token_mask)
    return desc[..., 0] >= 0


@torch.no_grad()
def _build_page_aware_image_block_mask(self, image_token_page_ids, query_token_page_ids, pos_chunk,
                                       num_key_blocks, cq):
    """[B, 1, cq, nblk] bool: the block holds an image token of the query's
    page (no fallback)."""
    bs = int(self.block_size)
    desc = ops.page_block_desc(int(num_key_blocks), bs, ipi=image_token_page_ids)
    return ops.page_cand_mask(desc, bs, pos=pos_chunk, qpi=query_token_page_ids, ipi=image_token_page_ids,
                              fallback=False)[:, None]


@torch.no_grad()
def _build_kl_candidate_mask(self, pos_chunk, num_key_blocks, image_token_mask, batch, cq,
                             image_token_page_ids=None, query_token_page_ids=None):
    """[B, 1, cq, nblk] bool remote candidates with the per-query fallback."""
    bs = int(self.block_size)
    nblk = int(num_key_blocks)
    if self.image_bucket_constraint and image_token_page_ids is not None and query_token_page_ids is not None:
        desc = ops.page_block_desc(nblk, bs, ipi=image_token_page_ids)
        cand = ops.page_cand_mask(desc, bs, pos=pos_chunk, qpi=query_token_page_ids, ipi=image_token_page_ids)
    elif image_token_mask is not None:
        desc = ops.page_block_desc(nblk, bs, itm=image_token_mask)
        cand = ops.page_cand_mask(desc, bs, flat=True, cq=int(cq))
    else:
        return torch.ones(batch, 1, cq, nblk, dtype=torch.bool, device=pos_chunk.device)
    return cand[:, None]


@torch.no_grad()
def _dash_block_cand(self, idx, router, pos_ids, itm, ipi, qpi, nblk, bsz, q_len):
    """Per-query candidate domain [B, S, nblk] (same-page image blocks with the
    per-query fallback), or None without image information."""
    if itm is None and (ipi is None or qpi is None):
        return None
    return _build_kl_candidate_mask(idx, pos_ids, nblk, itm, bsz, q_len,
                                    image_token_page_ids=ipi, query_token_page_ids=qpi)[:, 0]


@torch.no_grad()
def _uocr_dash_decode_allow(indexer, input_ids, cache):
    """Prefill (q_len > 1): records the decode state, returns None.  Decode
    (q_len == 1): [B, nblk] bool allow mask of the new query, or None."""
    img_id, pg_id = indexer.image_token_id, indexer.page_token_id
    if img_id is None or pg_id is None:
        return None
    bs = int(indexer.block_size)
    B, Lq = input_ids.shape
    if Lq > 1:
        ids = input_ids.to(device=_device(indexer, input_ids))
        cache._uocr_pg = ops.decode_allow_state(ids, img_id, pg_id, max(1, int(indexer.per_page_image_tokens)), bs)
        return None
    st = getattr(cache, "_uocr_pg", None)
    if st is None:
        return None
    total = int(cache.get_seq_length()) + Lq
    nblk = -(-total // bs)
    return ops.decode_allow(st, input_ids.to(device=st["bmin"].device), pg_id, nblk)
