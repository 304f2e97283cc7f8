"""Timed CPU baseline: the reference's CPU PyTorch SR-SWA path, restated in
torch -- TEST AND BENCHMARK INFRASTRUCTURE ONLY.

The reference runs its SR-SWA path on the host cores as plain PyTorch
(``hf-model-code/modeling_deepseekv2.py:339-481`` for the decode step,
``dash_attention.py:1230-1260`` for the dense prefill / training forward).
Its source cannot travel to the GPU host, so this module restates the same
sequence of torch operations (dense masked-softmax summaries of every block,
one matmul for the block scores, torch.topk, the sort / cumsum 1.5-entmax,
the dense masked attention over the whole cache) so that the benchmark times
the reference's algorithm at the reference's speed on the box's own cores.
Only ``tests/`` and ``bench.py``'s CPU-baseline / reference arm use it; the
product path (``srswa``) never imports it.  ``tests/test_oracle_torch.py``
pins it to the golden fixtures the reference produced."""

from __future__ import annotations

import math
import os

import torch

SCORE_NEG = -1.0e9
MASK_NEG = -1.0e9
ENTMAX_NEG = -1.0e4
ACT_CLAMP = 1.0e4


def host_info() -> dict:
    """Threads torch uses and the host CPU model (from /proc/cpuinfo)."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"threads": torch.get_num_threads(), "logical_cpus": os.cpu_count(), "cpu_model": model}


def entmax15(x: torch.Tensor) -> torch.Tensor:
    """Sort-based exact 1.5-entmax over the last axis (dash_attention.py:772-800):
    X <- (X - max) / 2; tau from the cumulative moments of the sorted row,
    support clamped >= 1; p = clamp(X - tau*, 0)^2."""
    x = (x - x.max(dim=-1, keepdim=True).values) / 2
    xs = torch.sort(x, dim=-1, descending=True).values
    rho = torch.arange(1, x.shape[-1] + 1, device=x.device, dtype=x.dtype)
    mean = xs.cumsum(-1) / rho
    msq = (xs * xs).cumsum(-1) / rho
    tau = mean - torch.sqrt(torch.clamp((1 - rho * (msq - mean * mean)) / rho, min=0))
    sup = (tau <= xs).sum(-1, keepdim=True).clamp(min=1)
    return torch.clamp(x - tau.gather(-1, sup - 1), min=0) ** 2


def route_select(scores, cand, idx_scale, floor, sigma, K, topm):
    """_infer_route_select (modeling_deepseekv2.py:339-362): candidacy with
    per-row fallback, top-M, entmax over the window, first K, centred
    log-prior bias -> (topi int64, bias fp32, valid bool) [..., K]."""
    remote = scores > SCORE_NEG * 0.5
    c = remote if cand is None else remote & cand
    c = torch.where(c.any(-1, keepdim=True), c, remote)
    x = torch.where(c, scores * idx_scale, torch.full_like(scores, ENTMAX_NEG))
    x = torch.nan_to_num(x, nan=ENTMAX_NEG, posinf=ENTMAX_NEG, neginf=ENTMAX_NEG)
    nblk = x.shape[-1]
    M = max(1, min(int(topm), nblk)) if int(topm) > 0 else nblk
    xv, xi = x.topk(M, dim=-1)
    prior = entmax15(xv)
    K = max(1, min(int(K), M))
    valid = c.gather(-1, xi)[..., :K]
    xi, prior = xi[..., :K], prior[..., :K]
    logp = torch.log(prior.clamp_min(floor))
    mu = torch.where(valid, logp, torch.zeros_like(logp)).sum(-1, keepdim=True) / valid.sum(-1, keepdim=True).clamp(min=1)
    return xi, torch.where(valid, (logp - mu) / sigma, torch.zeros_like(logp)).float(), valid


def block_scores(idx_q, idx_k, head_cls, q_pos, block_size, local_blocks):
    """_block_scores_infer, head_cls stage 0 (modeling_deepseekv2.py:381-417):
    the masked-softmax summary of EVERY block of idx_k [B,S,d], then one
    matmul against idx_q [B,Lq,d]; non-remote blocks -> SCORE_NEG."""
    B, S, d = idx_k.shape
    nblk = -(-S // block_size)
    pad = nblk * block_size - S
    if pad:
        kk = torch.nn.functional.pad(idx_k, (0, 0, 0, pad)).view(B, nblk, block_size, d)
        real = torch.nn.functional.pad(torch.ones(B, S, dtype=torch.bool), (0, pad)).view(B, nblk, block_size)
    else:   # whole blocks: views, no copy
        kk = idx_k.view(B, nblk, block_size, d)
        real = torch.ones(B, nblk, block_size, dtype=torch.bool)
    aw = ((kk * head_cls.view(1, 1, 1, d)).sum(-1) / math.sqrt(d)).clamp(-ACT_CLAMP, ACT_CLAMP)
    mx = torch.where(real, aw, torch.full_like(aw, torch.finfo(aw.dtype).min)).amax(-1, keepdim=True)
    mx = torch.where(real.any(-1, keepdim=True), mx, torch.zeros_like(mx))
    e = torch.exp(aw - mx) * real
    w = e / e.sum(-1, keepdim=True).clamp_min(1e-6)
    kbar = torch.nan_to_num((w.unsqueeze(-1) * kk).sum(2), nan=0.0, posinf=0.0, neginf=0.0)
    z = (idx_q @ kbar.transpose(-1, -2) / math.sqrt(d)).clamp(-ACT_CLAMP, ACT_CLAMP)
    blk = torch.arange(nblk)
    keep = (blk[None, None] <= (q_pos[:, :, None] // block_size - local_blocks)) & real.any(-1)[:, None]
    return z.masked_fill(~keep, SCORE_NEG)


def decode_attend(q, k_all, v_all, topi, bias, valid, q_pos, block_size, local_window, scale):
    """_decode_attend (modeling_deepseekv2.py:455-481): dense over the whole
    cache; selected blocks carry their bias, the window [p - LW + 1, p] none
    and wins on overlap -> [B,H,Lq,D] fp32."""
    B, H, Lq, D = q.shape
    S = k_all.shape[2]
    nblk = -(-S // block_size)
    kpos = torch.arange(S)
    src = torch.where(valid, bias, torch.full_like(bias, MASK_NEG))
    blk = torch.full((B, Lq, nblk), MASK_NEG).scatter(-1, topi.long(), src.float())
    base = blk.index_select(-1, kpos // block_size)
    qp = q_pos[:, :, None]
    causal = kpos[None, None] <= qp
    local = causal & (kpos[None, None] > qp - local_window)
    keep = causal & (local | (base > MASK_NEG * 0.5))
    m = torch.where(local, torch.zeros_like(base), base).masked_fill(~keep, float("-inf"))
    s = q.float() @ k_all.float().transpose(-1, -2) * scale + m[:, None]
    return torch.softmax(s, dim=-1) @ v_all.float()


def decode_step(q, k_all, v_all, idx_q, idx_k, head_cls, q_pos, block_size, local_blocks, K, topm, idx_scale,
                floor, sigma, scale):
    """One HF DASH decode step on the CPU (scores of every block, selection,
    dense attend), as _dash_decode_forward runs it (modeling_deepseekv2.py:483-530)."""
    with torch.no_grad():
        sc = block_scores(idx_q, idx_k, head_cls, q_pos, block_size, local_blocks)
        topi, bias, valid = route_select(sc, None, idx_scale, floor, sigma, K, topm)
        return decode_attend(q, k_all, v_all, topi, bias, valid, q_pos, block_size, local_blocks * block_size,
                             scale), topi, valid


def dense_forward(q, k, v, topi, bias, valid, block_size, local_window, scale, q_chunk=2048, q_rows=None,
                  q_start=0):
    """DashAttention._forward_dense (dash_attention.py:1230-1260): per query
    chunk, the [B,1,Lq,S] additive mask (0 on the window, the slot bias on
    selected remote blocks, MASK_NEG elsewhere) and one SDPA; q [B,H,T,D],
    k / v [B,H,S,D]; topi / bias / valid [B,T,K].  q_start / q_rows: compute
    only query rows [q_start, q_rows) (a timed sub-slice; keys stay [0, S))."""
    B, H, T, D = q.shape
    S = k.shape[2]
    nblk = -(-S // block_size)
    kidx = torch.arange(S)
    kb = kidx // block_size
    src = torch.where(valid, bias, torch.full_like(bias, MASK_NEG))
    logp = torch.full((B, bias.shape[1], nblk), MASK_NEG, dtype=bias.dtype).scatter(-1, topi, src)
    n = T if q_rows is None else min(T, int(q_rows))
    outs = []
    for qs in range(int(q_start), n, q_chunk):
        qe = min(qs + q_chunk, n)
        qi = torch.arange(qs, qe)
        base = logp[:, qs:qe].index_select(-1, kb)[:, None]
        causal = (kidx[None] <= qi[:, None])[None, None]
        local = (causal[0, 0] & (kidx[None] > qi[:, None] - local_window))[None, None]
        keep = causal & (local | (base > MASK_NEG * 0.5))
        mask = torch.where(local, torch.zeros_like(base), base).masked_fill(~keep, MASK_NEG)
        outs.append(torch.nn.functional.scaled_dot_product_attention(
            q[:, :, qs:qe], k, v, attn_mask=mask.clamp_min(MASK_NEG).to(q.dtype), scale=scale))
    return torch.cat(outs, dim=2)
