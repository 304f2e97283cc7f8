"""Drop-ins for the page2d (two-axis) RoPE of the indexer and main branch, on
CUDA kernels (``hf-model-code/_sparse_base_impl.py``).

* ``_build_page_rope_pos(self, source_input_ids, key_length)`` -- the
  DeepseekV2Indexer method (:2511-2570, with ``_page_rope_offsets``):
  (tok_pos, page_pos) [B, key_length] int64 or None; sets
  ``self._page_rope_meta = {'pf_cnt', 'n_pg'}``.  Reads image_token_id,
  page_token_id, rope_page_span and q_proj of ``self``.
* ``rotary2d_forward(self, x, tok_pos, page_pos)`` --
  ``DeepseekV2IndexerRotary2D.forward`` (:2043-2058): cos / sin [B, S, dim]
  in x's dtype.  ``self`` is the rotary module (inv_tok, inv_page,
  page_mod).
* ``apply_rotary2d_(x, tok_pos, page_pos, rot)`` -- the table and its
  application (``apply_rotary_pos_emb``) fused, in place on x [B, H, S, D] (or
  [B, S, H, D] with ``heads_first=False``), without materialising the tables.
* ``_main_rope_coords(self, q_len, past_kv)`` -- the SlidingWindowLlamaAttention
  method (:1451-1489): prefill coordinates and the per-layer decode state;
  each decode token updates the state on the device.

Same ``None`` cases as the reference (no image token or <PAGE> marker, or a
row without prompt pages).
"""

from __future__ import annotations

import torch

from . import ops


def _device(self, fallback: torch.Tensor) -> torch.device:
    w = getattr(getattr(self, "q_proj", None), "weight", None)
    if w is not None and w.is_cuda:
        return w.device
    if fallback.is_cuda:
        return fallback.device
    return torch.device("cuda", torch.cuda.current_device())


def _bail(self, reason):
    fn = getattr(self, "_page_rope_bail", None)
    return fn(reason) if callable(fn) else None


@torch.no_grad()
def _build_page_rope_pos(self, source_input_ids, key_length):
    """(tok_pos, page_pos) [B, key_length] int64, or None to fall back to 1D."""
    if source_input_ids is None or getattr(source_input_ids, "ndim", 0) != 2:
        return _bail(self, "no source_input_ids")
    if self.image_token_id is None or self.page_token_id is None:
        return _bail(self, "image_token_id / page_token_id unavailable")
    ids = source_input_ids.to(device=_device(self, source_input_ids))
    tok, page, pf, flags = ops.rope2d_pos(ids, self.image_token_id, self.page_token_id, int(key_length),
                                          int(getattr(self, "rope_page_span", 0) or 0))
    has_img, has_mark, no_pages, n_pg = flags.tolist()   # the reference's .any() tests read the device too
    if not has_img or not has_mark:
        return _bail(self, "row has no image token / no <PAGE> marker")
    if no_pages:
        return _bail(self, "non-marker mode (prompt carries no <PAGE>)")
    self._page_rope_meta = {"pf_cnt": pf[:, :n_pg], "n_pg": int(n_pg)}
    return tok, page


def _freqs(rot):
    inv_page = getattr(rot, "inv_page", None)
    return rot.inv_tok, inv_page, int(getattr(rot, "page_mod", 0) or 0)


@torch.no_grad()
def rotary2d_forward(self, x, tok_pos, page_pos):
    """cos / sin [B, S, dim] in x's dtype for coordinates tok_pos / page_pos [B, S]."""
    inv_tok, inv_page, page_mod = _freqs(self)
    dev = x.device if x.is_cuda else tok_pos.device
    return ops.rope2d_table(tok_pos.to(dev), page_pos.to(dev), inv_tok, inv_page, page_mod, dtype=x.dtype)


@torch.no_grad()
def apply_rotary2d_(x, tok_pos, page_pos, rot, heads_first=True, table_dtype=None):
    """x <- x * cos + rotate_half(x) * sin in place, the tables of ``rot`` at
    (tok_pos, page_pos) rounded to x's dtype (as the reference casts them);
    features beyond the table's dim are not allowed.  Returns x."""
    inv_tok, inv_page, page_mod = _freqs(rot)
    v = x.transpose(1, 2) if heads_first else x
    ops.rope2d_apply_(v, tok_pos, page_pos, inv_tok, inv_page, page_mod, table_dtype=table_dtype)
    return x


@torch.no_grad()
def _main_rope_coords(self, q_len, past_kv):
    """Prefill: full-sequence coordinates (recording the decode state when a
    cache is given); decode: the per-layer state advanced by the new token.
    Returns (tok, page) or None (fall back to 1D)."""
    if self.indexer is None:
        return None
    if q_len > 1:
        coords = getattr(self, "_main_rope_pos_2d", None)
        if coords is None:
            coords = self.indexer._build_page_rope_pos(getattr(self, "_sparse_source_input_ids", None), q_len)
            self._main_rope_pos_2d = coords
        if coords is None or coords[0].shape[-1] != q_len:
            return None
        if past_kv is not None:
            meta = getattr(self.indexer, "_page_rope_meta", None)
            if meta is not None:
                st = getattr(past_kv, "_page_rope_state", None)
                if st is None:
                    st = {}
                    past_kv._page_rope_state = st
                st[self.layer_idx] = {"page": coords[1][:, -1].clone(), "tok": coords[0][:, -1].clone(),
                                      "pf_cnt": meta["pf_cnt"], "n_pg": meta["n_pg"]}
        return coords
    st = getattr(past_kv, "_page_rope_state", None) if past_kv is not None else None
    st = st.get(self.layer_idx) if st else None
    ids = getattr(self, "_sparse_source_input_ids", None)
    if st is None or ids is None or ids.shape[-1] < 1:
        return _bail(self.indexer, "decode without page-rope state")
    page, tok = st["page"].clone(), st["tok"].clone()   # fresh tensors per step, as the reference's
    ops.rope2d_decode_(ids.to(page.device), self.indexer.page_token_id, page, tok, st["pf_cnt"], st["n_pg"])
    st["page"], st["tok"] = page, tok
    return tok[:, None], page[:, None]
