"""Drop-in for the reference module ``sparse_gather_triton``.

Same names, arguments, return contract and autograd behaviour as
hf-model-code/sparse_gather_triton.py:

* ``triton_gather_attention`` (:379-434) returns ``None`` for shapes the fused
  path does not take (attention mask given, index heads not dividing the head
  layout, prefix cache Sk != T, malformed position_ids) so the caller falls back;
  raises ``NotImplementedError`` for unsupported head dims / dtypes (the caller
  wraps it in try/except, _sparse_base_impl.py:1751-1763);
* ``triton_block_max_score`` (:488-524) returns fp32 [B, C, nblk];
* ``SPARSE_BLOCK_SIZE_SENTINEL`` (:32) is exported for the top-level import of
  modeling_unlimitedocr.py.

The work runs in libsrswa.so (sm_100a CUDA); there is no CPU path.
"""

from __future__ import annotations

import torch

from . import ops

SPARSE_BLOCK_SIZE_SENTINEL = 128


def _check_head_dim(q):
    D = q.shape[-1]
    if D not in (64, 128):
        raise NotImplementedError(f"head_dim {D} not supported (64 or 128)")
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError(f"dtype {q.dtype} not supported (bf16 / fp16)")


def _btHd(x):
    """[B,H,T,D] -> [B,T,H,D] view (no copy) with D contiguous."""
    y = x.transpose(1, 2)
    if y.stride(-1) != 1 or any(s % 8 for s in y.stride()[:3]):
        y = y.contiguous()
    return y


class _GatherAttnFn(torch.autograd.Function):
    """Autograd wrapper: saves (q, k, v, sel, seg, o, lse) like the reference's
    _TritonGatherAttnFn (sparse_gather_triton.py:356-376)."""

    @staticmethod
    def forward(ctx, q, k, v, sel, seg, bias, block_size, scale, local_window):
        o, lse = ops.gather_fwd(q, k, v, sel, bias, seg, block_size, scale, local_window)
        ctx.save_for_backward(q, k, v, sel, seg, o, lse, bias)
        ctx.block_size, ctx.scale, ctx.local_window = block_size, scale, local_window
        ctx.has_bias = bias is not None
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, sel, seg, o, lse, bias = ctx.saved_tensors
        if not ctx.has_bias:
            bias = None
        dq, dk, dv, dbias = ops.gather_bwd(q, k, v, o, lse, do, sel, bias, seg, ctx.block_size,
                                           ctx.scale, ctx.local_window)
        return dq, dk, dv, None, None, dbias, None, None, None


def triton_gather_attention(query_states, key_states, value_states, block_indices, position_ids,
                            attention_mask, block_size, scale, local_window=None):
    """Fused gather-attention; [B,HQ,T,D] or None (caller falls back).

    Per query t: local window [max(t-LW+1, seg_t), t] plus the keys of its
    selected blocks (block_indices [B,HI,T,S], -1 = pad, repeats deduped) in
    [seg_t, t-LW+1); seg_t = t - position_ids[b,t] isolates packed samples."""
    if attention_mask is not None:
        return None
    B, HQ, T, D = query_states.shape
    HI = block_indices.shape[1]
    Hkv = key_states.shape[1]
    if HI < 1 or HQ % HI != 0 or Hkv % HI != 0:
        return None
    if key_states.shape[2] != T:
        return None
    if position_ids is None or position_ids.dim() != 2 or position_ids.shape[-1] != T:
        return None
    _check_head_dim(query_states)
    ar = torch.arange(T, device=position_ids.device)
    seg = (ar[None, :] - position_ids).to(torch.int32).expand(B, T).contiguous()
    nblk = (T + block_size - 1) // block_size
    sel = ops.pack_selection(block_indices, nblk)
    q, k, v = _btHd(query_states), _btHd(key_states), _btHd(value_states)
    if k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    o = _GatherAttnFn.apply(q, k, v, sel, seg, None, block_size, float(scale), local_window)
    return o.transpose(1, 2)


def triton_block_max_score(q, k, pos, seg, block_size, num_key_blocks, local_window=None):
    """Block max of q.k over non-local causal same-segment keys (unscaled,
    -inf where a block has no such key); q [B,C,D], k [B,Sk,D] -> [B,C,nblk]."""
    assert q.dim() == 3 and k.dim() == 3, "expects [B, C, D] / [B, Sk, D]"
    D = q.shape[-1]
    if D > 256:
        raise NotImplementedError(f"index dim D={D} > 256 not supported")
    lw = block_size if local_window is None else max(1, int(local_window))
    return ops.block_max_score(q, k, pos, seg, block_size, num_key_blocks, lw, mode=0)
