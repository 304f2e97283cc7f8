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

import torch

from . import ops
from .sparse_gather import _btHd, _check_head_dim, _GatherAttnFn

SPARSE_E2E_SENTINEL = 1


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
    ar = torch.arange(T, device=position_ids.device)
    if not bool((position_ids == ar).all()):
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
