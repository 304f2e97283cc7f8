"""Drop-ins for the router/decode functions of the DASH inference overlay
(hf-model-code/modeling_deepseekv2.py) plus a fused prefill/decode router.

* ``_block_scores_infer(router, idx_q, idx_k, q_pos, nblk)``   (:381-430)
* ``_infer_route_select(block_scores, block_cand, p)``         (:339-362)
* ``_decode_attend(q, k_all, v_all, topi, bias, valid, q_pos, block_size,
  local_window, scale)``                                        (:455-481)
* ``route(router, idx_q, idx_k, q_pos, nblk, block_cand, p)`` -- the first two
  fused (k_bar -> scores -> top-M entmax -> top-K bias) without materialising
  the [B, Lq, nblk] score tensor; same outputs as calling them in sequence.

``router`` is the reference's DashAttention (only block_size, local_blocks,
local_window, head_cls, stage0 are read); ``p`` is its ``_infer_params`` dict.
"""

from __future__ import annotations

import torch

from . import ops


def _stage0(router):
    return str(getattr(router, "stage0", "head_cls")).lower()


_seq_lens_cache = {}


def _seq_lens(B, S, dev):
    """[B] int32 tensor of S, read-only: kept per (B, S, device), so that
    every layer of a forward does not allocate and fill its own."""
    key = (B, S, dev)
    t = _seq_lens_cache.get(key)
    if t is None:
        if len(_seq_lens_cache) > 64:
            _seq_lens_cache.clear()
        t = _seq_lens_cache[key] = torch.full((B,), S, device=dev, dtype=torch.int32)
    return t


@torch.no_grad()
def _block_scores_infer(router, idx_q, idx_k, q_pos, nblk):
    """[B,Lq,nblk] fp32 remote block scores (SCORE_NEG = -1e9 elsewhere)."""
    B, S, d = idx_k.shape
    Lq = idx_q.shape[1]
    bs = int(router.block_size)
    if _stage0(router) == "head_cls":
        kb, _ = ops.kbar_contig(idx_k, router.head_cls.detach(), bs)
        if kb.shape[1] < nblk:
            kb = torch.cat([kb, kb.new_zeros(B, nblk - kb.shape[1], d)], 1)
        r = ops.route(idx_q.reshape(B * Lq, d), kb[:, :nblk].contiguous(), block_size=bs,
                      local_blocks=int(router.local_blocks), topk=1, topm=1, idx_scale=1.0,
                      floor=1.0, sigma=1.0, q_pos=q_pos.reshape(-1), seq_lens=_seq_lens(B, S, idx_k.device),
                      rows_per_seq=Lq, want=("scores",), nblk=nblk)
        return r["scores"].view(B, Lq, nblk)
    # stage0 "indexer": block max of token scores over remote keys
    pos = q_pos.expand(B, Lq) if q_pos.shape[0] != B else q_pos
    return ops.block_max_score(idx_q, idx_k, pos, None, bs, nblk, int(router.local_window), mode=1)


@torch.no_grad()
def _infer_route_select(block_scores, block_cand, p):
    """(topi int64 [B,Lq,K], bias fp32 [B,Lq,K], valid bool [B,Lq,K])."""
    r = ops.route_select(block_scores, block_cand, topk=p["K"], topm=p["topm"], idx_scale=p["idx_scale"],
                         floor=p["floor"], sigma=p["sigma"])
    return r["topi64"], r["bias"], r["valid"]


@torch.no_grad()
def route(router, idx_q, idx_k, q_pos, nblk, block_cand, p):
    """Fused _block_scores_infer + _infer_route_select (head_cls stage 0)."""
    B, S, d = idx_k.shape
    Lq = idx_q.shape[1]
    bs = int(router.block_size)
    if _stage0(router) != "head_cls":
        return _infer_route_select(_block_scores_infer(router, idx_q, idx_k, q_pos, nblk), block_cand, p)
    kb, _ = ops.kbar_contig(idx_k, router.head_cls.detach(), bs, chunk_valid=False)
    if kb.shape[1] < nblk:
        kb = torch.cat([kb, kb.new_zeros(B, nblk - kb.shape[1], d)], 1)
    r = ops.route(idx_q.reshape(B * Lq, d), kb[:, :nblk].contiguous(), block_size=bs,
                  local_blocks=int(router.local_blocks), topk=p["K"], topm=p["topm"], idx_scale=p["idx_scale"],
                  floor=p["floor"], sigma=p["sigma"], q_pos=q_pos.reshape(-1),
                  seq_lens=_seq_lens(B, S, idx_k.device), rows_per_seq=Lq, cand=block_cand, nblk=nblk)
    K = r["topi64"].shape[-1]
    return r["topi64"].view(B, Lq, K), r["bias"].view(B, Lq, K), r["valid"].view(B, Lq, K)


@torch.no_grad()
def _decode_attend(q, k_all, v_all, topi, bias, valid, q_pos, block_size, local_window, scale):
    """Bias-aware block-sparse attention for decode queries -> fp32 [B,H,Lq,D].

    Reads only the selected blocks and the window (the reference's dense
    version reads the whole cache)."""
    B, H, Lq, D = q.shape
    Hkv, S = k_all.shape[1], k_all.shape[2]
    if local_window % block_size:
        raise NotImplementedError("local_window must be a multiple of block_size")
    if k_all.stride(-1) != 1 or k_all.stride() != v_all.stride():
        k_all, v_all = k_all.contiguous(), v_all.contiguous()
    dt = k_all.dtype
    qq = q.permute(0, 2, 1, 3).reshape(B * Lq, H, D).to(dt).contiguous()
    nblk = (S + block_size - 1) // block_size
    K = topi.shape[-1]
    out = torch.empty(B * Lq, H, D, device=q.device, dtype=torch.float32)
    ops.decode_attend(qq, k_all, v_all, topi.reshape(B * Lq, K), bias.reshape(B * Lq, K).float(),
                      block_size=block_size, local_blocks=local_window // block_size, sm_scale=scale,
                      out=out, q_pos=q_pos.reshape(-1), rows_per_req=Lq, valid=valid.reshape(B * Lq, K),
                      kv_layout=(B, nblk, k_all.stride(0), k_all.stride(2), k_all.stride(1), Hkv))
    return out.view(B, Lq, H, D).permute(0, 2, 1, 3)
