"""DSA training extras (stage "sparse"): the gather-KL distillation of the
index branch against the main attention, and the select_and_kl_loss drop-in.

``gather_kl`` is differentiable in idx_q / idx_k (the teacher side is
detached, as in the reference) and runs srswa_gather_kl_fwd / _bwd.  It is
the KL of hf-model-code/_sparse_base_impl.py select_and_kl_loss's gather
branch (:3397-3450) and of _kl_chunk_core (:2071-2137): per query row, over
the keys of its selected blocks below the local window.

``select_and_kl_loss`` replaces DeepseekV2Indexer.select_and_kl_loss
(:3240-3516) for one index head on CUDA with unpacked rows: block-max scores
(srswa_block_max_score), the page-aware candidate mask and its per-row
fallback, top-k, then ``gather_kl`` over all query rows at once (the
reference's kl_chunk_size loop only bounds its dense memory).  Other cases
(several index heads, CPU tensors, packed rows) call the reference's own
method, saved at install time.  The Anchor / Reuse block-index cache of the
reference (:1698-1727, 3992-4055) is model plumbing around this call and
stays the reference's: an Anchor layer's block_indices are what this
function returns.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L


def _desc(iq, ik, qm, km, S, block_size, local_window, scaling, logits_bf16):
    B, Cq, d = iq.shape
    Sk = ik.shape[1]
    H, D = qm.shape[2], qm.shape[3]
    Hkv = km.shape[2]
    return L.KlDesc(B, Cq, Sk, H, Hkv, D, d, S, int(block_size), int(local_window), float(scaling),
                    1 if logits_bf16 else 0, L.dtype_code(iq), L.dtype_code(ik), L.dtype_code(qm), L.dtype_code(km),
                    iq.stride(0), iq.stride(1), ik.stride(0), ik.stride(1), qm.stride(0), qm.stride(1), qm.stride(2),
                    km.stride(0), km.stride(1), km.stride(2))


def _feat_contig(x):
    return x if x.stride(-1) == 1 else x.contiguous()


class _GatherKLFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, iq, ik, qm, km, sel, pos, seg, block_size, local_window, scaling, logits_bf16,
                save_teacher):
        iq, ik, qm, km = (_feat_contig(x) for x in (iq, ik, qm, km))
        B, Cq, _ = iq.shape
        S = sel.shape[-1]
        g = _desc(iq, ik, qm, km, S, block_size, local_window, scaling, logits_bf16)
        kl = torch.empty(B, Cq, device=iq.device, dtype=torch.float32)
        valid = torch.empty(B, Cq, device=iq.device, dtype=torch.uint8)
        # save_teacher: keep the averaged teacher probabilities [B, C, S * BS]
        # (fp32) so that the backward does not gather every head's main keys again
        teacher = torch.empty(B, Cq, S * int(block_size), device=iq.device, dtype=torch.float32) \
            if save_teacher else None
        rc = L.lib().srswa_gather_kl_fwd_save(C.byref(g), iq.data_ptr(), ik.data_ptr(), qm.data_ptr(),
                                              km.data_ptr(), sel.data_ptr(), pos.data_ptr(), L.ptr(seg),
                                              kl.data_ptr(), valid.data_ptr(), L.ptr(teacher), L.stream_of(iq))
        L.check(rc, "srswa_gather_kl_fwd")
        if teacher is not None:   # the main tensors are not needed again
            qm, km = qm.new_empty(0), km.new_empty(0)
        ctx.teacher = teacher
        ctx.main_shapes = (g.H, g.Hkv, g.D)
        ctx.save_for_backward(iq, ik, qm, km, sel, pos, seg if seg is not None else pos.new_empty(0))
        ctx.has_seg = seg is not None
        ctx.cfg = (block_size, local_window, scaling, logits_bf16)
        ctx.mark_non_differentiable(valid)
        return kl, valid.view(torch.bool)

    @staticmethod
    def backward(ctx, gkl, _gvalid):
        iq, ik, qm, km, sel, pos, seg = ctx.saved_tensors
        seg = seg if ctx.has_seg else None
        block_size, local_window, scaling, logits_bf16 = ctx.cfg
        teacher = ctx.teacher
        if teacher is not None:   # descriptor of the main tensors without them (only their shapes count)
            H, Hkv, D = ctx.main_shapes
            B, Cq, _ = iq.shape
            g = L.KlDesc(B, Cq, ik.shape[1], H, Hkv, D, iq.shape[2], sel.shape[-1], int(block_size),
                         int(local_window), float(scaling), 1 if logits_bf16 else 0, L.dtype_code(iq),
                         L.dtype_code(ik), L.dtype_code(iq), L.dtype_code(ik), iq.stride(0), iq.stride(1),
                         ik.stride(0), ik.stride(1), 0, 0, 0, 0, 0, 0)
        else:
            g = _desc(iq, ik, qm, km, sel.shape[-1], block_size, local_window, scaling, logits_bf16)
        lib = L.lib()
        gr = gkl.float().contiguous()
        diq = torch.empty(iq.shape, device=iq.device, dtype=torch.float32)
        dik = torch.empty(ik.shape, device=ik.device, dtype=torch.float32)
        ws_n = lib.srswa_gather_kl_bwd_workspace_size(C.byref(g))
        ws = torch.empty(max(ws_n, 1), device=iq.device, dtype=torch.uint8)
        if teacher is not None:
            rc = lib.srswa_gather_kl_bwd_saved(C.byref(g), iq.data_ptr(), ik.data_ptr(), sel.data_ptr(),
                                               pos.data_ptr(), L.ptr(seg), teacher.data_ptr(), gr.data_ptr(),
                                               diq.data_ptr(), dik.data_ptr(), ws.data_ptr(), ws_n,
                                               L.stream_of(iq))
            ctx.teacher = None
        else:
            rc = lib.srswa_gather_kl_bwd(C.byref(g), iq.data_ptr(), ik.data_ptr(), qm.data_ptr(), km.data_ptr(),
                                         sel.data_ptr(), pos.data_ptr(), L.ptr(seg), gr.data_ptr(), diq.data_ptr(),
                                         dik.data_ptr(), ws.data_ptr(), ws_n, L.stream_of(iq))
        L.check(rc, "srswa_gather_kl_bwd")
        return diq.to(iq.dtype), dik.to(ik.dtype), None, None, None, None, None, None, None, None, None, None


def gather_kl(idx_q, idx_k, q_main, k_main, sel, pos, seg=None, *, block_size, local_window, scaling,
              logits_bf16=None, save_teacher=True):
    """Per-row KL (and row validity) of the DSA distillation.
    idx_q [B,C,d], idx_k [B,Sk,d] (differentiable), q_main [B,C,H,D], k_main
    [B,Sk,Hkv,D] (detached teacher; [B,H,C,D] tensors go in as
    .transpose(1, 2) views), sel [B,C,S] block ids (-1 pad), pos / seg [B,C]
    (global positions, segment starts).  logits_bf16 defaults to the index
    tensors being bf16 (the reference rounds its matmul outputs to them).
    save_teacher: keep the rows' averaged teacher probabilities ([B, C, S *
    block_size] fp32) from the forward for the backward, which then skips
    the teacher's gather of every head's main keys (same gradients, bit for
    bit); False recomputes them."""
    if logits_bf16 is None:
        logits_bf16 = idx_q.dtype == torch.bfloat16
    sel32 = sel.to(torch.int32).contiguous()
    pos64 = pos.to(device=idx_q.device, dtype=torch.int64).contiguous()
    seg64 = None if seg is None else seg.to(device=idx_q.device, dtype=torch.int64).contiguous()
    return _GatherKLFn.apply(idx_q, idx_k, q_main.detach(), k_main.detach(), sel32, pos64, seg64, int(block_size),
                             int(local_window), float(scaling), bool(logits_bf16), bool(save_teacher))


_ORIGINAL = {}   # indexer class -> the reference's select_and_kl_loss


def _is_arange(position_ids):
    ar = torch.arange(position_ids.shape[-1], device=position_ids.device)
    return bool((position_ids == ar).all())


def select_and_kl_loss(self, hidden_states, query_states, key_states, position_embeddings, position_ids, scaling,
                       image_token_mask=None, image_token_page_ids=None, query_token_page_ids=None):
    """Drop-in for DeepseekV2Indexer.select_and_kl_loss (one index head, CUDA,
    unpacked rows): returns (block_indices [B,1,C,topk] long, -1 = none; the
    KL loss, sum over valid rows / (count + 1e-6))."""
    orig = _ORIGINAL.get(type(self))
    if self.num_heads != 1 or not hidden_states.is_cuda or not _is_arange(position_ids):
        if orig is None:
            raise NotImplementedError("select_and_kl_loss: this case needs the reference's own method")
        return orig(self, hidden_states, query_states, key_states, position_embeddings, position_ids, scaling,
                    image_token_mask=image_token_mask, image_token_page_ids=image_token_page_ids,
                    query_token_page_ids=query_token_page_ids)
    from .sparse_gather import triton_block_max_score
    batch, q_len, _ = hidden_states.shape
    idx_q, idx_k = self._project_index_qk(hidden_states.detach(), position_ids, None)   # [B,1,C,d], [B,1,Sk,d]
    k_len = idx_k.shape[2]
    nkb = -(-k_len // self.block_size)
    topk = self._remote_topk(nkb)
    pos = position_ids.to(torch.int64)
    if topk == 0:
        bi = idx_q.new_empty((batch, 1, q_len, 0), dtype=torch.long)
        return bi, idx_q.new_zeros((), dtype=torch.float32)
    with torch.no_grad():
        block_scores = triton_block_max_score(idx_q[:, 0], idx_k[:, 0], pos, torch.zeros_like(pos), self.block_size,
                                              nkb, local_window=self.local_window)[:, None]   # [B,1,C,nblk]
        candidate = self._build_kl_candidate_mask(pos, nkb, image_token_mask, batch, q_len,
                                                  image_token_page_ids=image_token_page_ids,
                                                  query_token_page_ids=query_token_page_ids)
        scores_c = block_scores.masked_fill(~candidate.expand_as(block_scores), float("-inf"))
        need = (scores_c > float("-inf")).sum(-1, keepdim=True) < topk   # per-row fallback to all blocks
        scores_c = torch.where(need, block_scores, scores_c)
        top_s, top_i = scores_c.topk(topk, dim=-1)
        bi = top_i.masked_fill(top_s == float("-inf"), -1)
    kl, valid = gather_kl(idx_q[:, 0], idx_k[:, 0], query_states.transpose(1, 2), key_states.transpose(1, 2),
                          bi[:, 0], pos, None, block_size=self.block_size, local_window=self.local_window,
                          scaling=scaling)
    v = valid.float()
    return bi, (kl * v).sum() / (v.sum() + 1e-6)
