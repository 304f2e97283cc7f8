"""Paged-KV serving ops with the SGLang DASH signatures
(whl:sglang/srt/layers/attention/unlimited_dash_ops/):

* ``dash_sparse_attn_decode`` (attend_triton.py:600-715): split-KV decode with
  the merge done on-chip (thread-block cluster) instead of a second kernel;
  writes ``output`` in place.
* ``kbar_refresh_tail`` (route_triton.py:706-726) and ``KBarCache``
  (dash_stage0.py:106-150): one fp32 head_cls summary per KV page.
* ``route_decode`` (route_triton.py:729-847): fused scores over the k_bar cache
  + top-M entmax + top-K + bias into caller-owned ``out_idx`` / ``out_bias``
  (score-descending slots, -1 / 0 on unused slots).
"""

from __future__ import annotations

import torch

from . import ops

SPARSE_BLOCK_SIZE = 128


@torch.no_grad()
def dash_sparse_attn_decode(q, k_cache, v_cache, topk_idx, blk_bias, block_table, seq_lens, num_kv_heads,
                            sm_scale, output, decode_query_len, local_blocks=0,
                            sparse_block_size=SPARSE_BLOCK_SIZE, chunk_width=None, cg_rows=None):
    """Bias-aware block-sparse decode.  q [R*dql, H, D]; caches [P, BS, Hkv, D];
    topk_idx/blk_bias [Hkv, R*dql, K] (stride 0 over heads allowed); output
    [R*dql, H, D] written in place.  chunk_width / cg_rows are accepted for
    signature compatibility (no scratch geometry to pre-allocate)."""
    total_q = q.shape[0]
    assert total_q == seq_lens.shape[0] * decode_query_len
    assert k_cache.shape[2] == num_kv_heads
    ops.decode_attend(q, k_cache, v_cache, topk_idx, blk_bias, block_size=sparse_block_size,
                      local_blocks=local_blocks, sm_scale=sm_scale, out=output, block_table=block_table,
                      seq_lens=seq_lens, rows_per_req=decode_query_len)


class KBarCache:
    """One fp32 head_cls summary per KV page of a paged index-key cache."""

    def __init__(self, num_pages: int, dim: int, device, dtype=torch.float32):
        self.k_bar = torch.zeros(num_pages, dim, dtype=dtype, device=device)

    @torch.no_grad()
    def summarize(self, *, kv_cache, block_table, seq_lens, head_cls, block_size: int, tail_pages: int = 0):
        """Summaries of the last ``tail_pages`` pages of every request (all pages
        in use when tail_pages <= 0), computed from ``kv_cache`` [P, BS, d]."""
        assert kv_cache.shape[1] == block_size
        ops.kbar_paged(kv_cache, head_cls, block_table, seq_lens, self.k_bar, tail_pages)

    def refresh_tail(self, *, kv_cache, block_table, seq_lens, head_cls, block_size: int, tail_pages: int = 2):
        self.summarize(kv_cache=kv_cache, block_table=block_table, seq_lens=seq_lens, head_cls=head_cls,
                       block_size=block_size, tail_pages=tail_pages)


@torch.no_grad()
def kbar_refresh_tail(*, kv_cache, k_bar, block_table, seq_lens, head_cls, block_size: int, tail_pages: int = 1,
                      plan=None):
    del plan
    ops.kbar_paged(kv_cache, head_cls, block_table, seq_lens, k_bar, tail_pages)


@torch.no_grad()
def route_decode(*, idx_q, k_bar, block_table, seq_lens, image_allow, out_idx, out_bias, max_block: int,
                 block_size: int, local_blocks: int, decode_query_len: int, idx_scale: float, prior_floor: float,
                 sigma: float, topm: int, budget: int | None = None, out_slots: int | None = None, **_unused):
    """Route decode rows idx_q [R*dql, d] against the k_bar cache.  Writes the
    first K = min(budget, topm) slots of out_idx (int32, -1 unused) and
    out_bias (fp32, 0 unused); remaining slots are set to -1 / 0.  Returns the
    slot width written.  Contiguous buffers exactly K slots wide are written
    by the kernel directly (no copies)."""
    W = min(int(max_block), int(block_table.shape[1]))
    K = max(1, min(int(budget or topm), int(topm)))
    Ke, _ = ops.effective_km(K, topm, W)
    direct = (out_idx.dtype == torch.int32 and out_bias.dtype == torch.float32 and out_idx.is_contiguous()
              and out_bias.is_contiguous() and out_idx.shape[-1] == Ke and out_bias.shape[-1] == Ke)
    r = ops.route(idx_q, k_bar, block_size=block_size, local_blocks=local_blocks, topk=K, topm=topm,
                  idx_scale=idx_scale, floor=prior_floor, sigma=sigma, seq_lens=seq_lens,
                  rows_per_seq=max(1, int(decode_query_len)), block_table=block_table[:, :W],
                  cand=image_allow, want=("topi32", "bias"), nblk=W,
                  out={"topi32": out_idx, "bias": out_bias} if direct else None)
    k = r["topi32"].shape[-1]
    if direct:   # written in place: buffers exactly K slots wide
        return out_slots or k
    out_idx[:, :k].copy_(r["topi32"])
    out_bias[:, :k].copy_(r["bias"])
    if out_idx.shape[-1] > k:
        out_idx[:, k:].fill_(-1)
        out_bias[:, k:].zero_()
    return out_slots or k

