"""Drop-in for the reference module ``sparse_gather_e2e_triton``.

``triton_gather_attention_e2e`` keeps the signature and contract of
hf-model-code/sparse_gather_e2e_triton.py:355-407: it returns ``None`` for an
attention mask, more than one index head, a prefix cache (Sk != T) or
position_ids that are not ``arange`` (packing), and gradients flow to q, k, v
and ``blk_bias_slots``.  The per-slot bias is consumed directly (the reference
scatters it into a dense [B, T, nblk] map first); a repeated block id keeps its
first slot, whose gradient is the block's, and the repeats get zero gradient.
``SPARSE_E2E_SENTINEL`` (:33) is exported for modeling_unlimitedocr.py.
"""

from __future__ import annotations

import weakref

import torch

from . import ops
from .sparse_gather import _btHd, _check_head_dim, _GatherAttnFn

SPARSE_E2E_SENTINEL = 1


_arange_check = None  # (weak reference to the position_ids tensor, its version, result)


def _positions_are_arange(position_ids, T):
    """position_ids == arange(T) on every row (the reference's packing test,
    which reads the device).  The model passes one position_ids tensor to every
    layer of a forward, so the answer is kept for that tensor object while its
    in-place version counter is unchanged; a new or modified tensor is tested
    again (a weak reference: a freed tensor can never match)."""
    global _arange_check
    c = _arange_check
    if c is not None and c[0]() is position_ids and c[1] == position_ids._version:
        return c[2]
    ar = torch.arange(T, device=position_ids.device)
    res = bool((position_ids == ar).all())
    _arange_check = (weakref.ref(position_ids), position_ids._version, res)
    return res


def triton_gather_attention_e2e(query_states, key_states, value_states, block_indices, blk_bias_slots,
                                position_ids, attention_mask, block_size, scale, local_window=None):
    """Fused gather-attention with a differentiable per-slot bias on remote
    keys; [B,HQ,T,D] or None (caller falls back)."""
    if attention_mask is not None:
        return None
    if block_indices.shape[1] != 1:
        return None
    B, HQ, T, D = query_states.shape
    if key_states.shape[2] != T:
        return None
    if position_ids is None or position_ids.dim() != 2 or position_ids.shape[-1] != T:
        return None
    if not _positions_are_arange(position_ids, T):
        return None
    _check_head_dim(query_states)
    nblk = (T + block_size - 1) // block_size
    sel = ops.pack_selection(block_indices, nblk)
    bias = blk_bias_slots
    if bias.dtype != torch.float32:
        bias = bias.float()
    if not bias.is_contiguous():
        bias = bias.contiguous()
    q, k, v = _btHd(query_states), _btHd(key_states), _btHd(value_states)
    if k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    o = _GatherAttnFn.apply(q, k, v, sel, None, bias, block_size, float(scale), local_window)
    return o.transpose(1, 2)
