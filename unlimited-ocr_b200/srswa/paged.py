"""Paged-KV serving ops with the SGLang DASH signatures
(whl:sglang/srt/layers/attention/unlimited_dash_ops/):

* ``dash_sparse_attn_decode`` (attend_triton.py:600-715): split-KV decode with
  the merge done on-chip (thread-block cluster) instead of a second kernel;
  writes ``output`` in place.
* ``dash_sparse_attn`` (attend_triton.py:523-597): varlen paged prefill
  attend, one row per query token; writes ``output`` in place.
* ``kbar_refresh_tail`` / ``kbar_refresh_tail_triton`` (route_triton.py:706-726)
  and ``KBarCache`` (dash_stage0.py:106-150): one fp32 head_cls summary per KV
  page, for the tail pages or for an explicit (pages, tokens) plan.
* ``route_decode`` / ``route_decode_triton`` (route_triton.py:729-847) and
  ``route_prefill_triton`` (:624-680): fused scores over the k_bar cache +
  top-M entmax + top-K + bias into caller-owned ``out_idx`` / ``out_bias``
  (score-descending slots, -1 / 0 on unused slots).  The slots hold the
  reference HF router's selection (top-M exact entmax); the wheel's
  bisection entmax over every candidate selects the same set (the attend
  reads the slots as a set), its bias can differ when the entmax support
  exceeds M.
* ``win_bounds_decode`` (route_triton.py:466-526): each decode row's remote
  page span from its allow mask.  The router here scans the whole live
  width in one pass, so the span is an output for the caller only.
"""

from __future__ import annotations

import torch

from . import _lib as L
from . import ops

SPARSE_BLOCK_SIZE = 128


@torch.no_grad()
def dash_sparse_attn_decode(q, k_cache, v_cache, topk_idx, blk_bias, block_table, seq_lens, num_kv_heads,
                            sm_scale, output, decode_query_len, local_blocks=0,
                            sparse_block_size=SPARSE_BLOCK_SIZE, chunk_width=None, cg_rows=None,
                            overlap_router=False):
    """Bias-aware block-sparse decode.  q [R*dql, H, D]; caches [P, BS, Hkv, D];
    topk_idx/blk_bias [Hkv, R*dql, K] (stride 0 over heads allowed); output
    [R*dql, H, D] written in place.  chunk_width / cg_rows are accepted for
    signature compatibility (no scratch geometry to pre-allocate).
    overlap_router: called right after route_decode on the same stream (as
    the SGLang backend's _forward does), with q, the caches, block_table and
    seq_lens written before it: the window keys are attended while the
    router finishes (ops.decode_attend's overlap)."""
    total_q = q.shape[0]
    assert total_q == seq_lens.shape[0] * decode_query_len
    assert k_cache.shape[2] == num_kv_heads
    ops.decode_attend(q, k_cache, v_cache, topk_idx, blk_bias, block_size=sparse_block_size,
                      local_blocks=local_blocks, sm_scale=sm_scale, out=output, block_table=block_table,
                      seq_lens=seq_lens, rows_per_req=decode_query_len, overlap=overlap_router)


@torch.no_grad()
def dash_sparse_attn_decode_after_router(*args, **kwargs):
    """dash_sparse_attn_decode with overlap_router=True: for a caller that
    issues it right after route_decode on the same stream."""
    kwargs.setdefault("overlap_router", True)
    return dash_sparse_attn_decode(*args, **kwargs)


@torch.no_grad()
def dash_sparse_attn(q, k_cache, v_cache, topk_idx, blk_bias, block_table, cu_seqlens_q, seq_lens, prefix_lens,
                     max_query_len, num_kv_heads, sm_scale, output, local_blocks=0,
                     sparse_block_size=SPARSE_BLOCK_SIZE):
    """Bias-aware block-sparse prefill attention over the paged cache.  q
    [total_q, H, D]; row i of request r (cu_seqlens_q[r] <= i < cu_seqlens_q[r+1])
    sits at position prefix_lens[r] + i - cu_seqlens_q[r]; topk_idx / blk_bias
    [Hkv, total_q, K] (stride 0 over heads allowed; -1 = unused slot).
    seq_lens and max_query_len are accepted for signature compatibility (the
    rows carry their positions; no grid is sized on the host)."""
    del seq_lens, max_query_len
    assert k_cache.shape[2] == num_kv_heads
    if blk_bias is not None:
        assert blk_bias.shape == topk_idx.shape and blk_bias.dtype == torch.float32
    rest = _tc_prefill(q, k_cache, v_cache, topk_idx, blk_bias, block_table, cu_seqlens_q, prefix_lens, sm_scale,
                       output, local_blocks, sparse_block_size)
    if rest is None:  # the tensor-core path does not apply: every row on the row kernel
        ops.prefill_attend(q, k_cache, v_cache, topk_idx, blk_bias, block_table=block_table,
                           cu_seqlens_q=cu_seqlens_q, prefix_lens=prefix_lens, block_size=sparse_block_size,
                           local_blocks=local_blocks, sm_scale=sm_scale, out=output)
        return
    for r, a, b, ctx in rest:  # short requests: one row-kernel launch each
        dev = q.device
        ops.prefill_attend(q[a:b], k_cache, v_cache, topk_idx[:, a:b], None if blk_bias is None else blk_bias[:, a:b],
                           block_table=block_table[r:r + 1],
                           cu_seqlens_q=torch.tensor([0, b - a], dtype=torch.int32, device=dev),
                           prefix_lens=torch.tensor([ctx], dtype=torch.int32, device=dev),
                           block_size=sparse_block_size, local_blocks=local_blocks, sm_scale=sm_scale,
                           out=output[a:b])


# Requests with at least this many rows take the tensor-core forward.
TC_MIN_ROWS = 128


def _tc_prefill(q, k_cache, v_cache, topk_idx, blk_bias, block_table, cu_seqlens_q, prefix_lens, sm_scale, output,
                local_blocks, block_size):
    """Runs every request of at least TC_MIN_ROWS rows through the
    tensor-core gather forward over the paged caches (srswa_gather_fwd_paged:
    one launch sequence per request, its rows after a prefix of
    prefix_lens[r] tokens) and returns the other requests as (r, first row,
    end row, prefix); None when the path does not apply to this call (dtype,
    head dim, 64-token pages, a selection or bias that differs per head, no
    local window, or inside a CUDA graph capture).  Reads cu_seqlens_q and
    prefix_lens on the host."""
    if torch.cuda.is_current_stream_capturing():  # no host reads inside a CUDA graph capture
        return None
    if (q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16 or output.dtype != torch.bfloat16
            or q.shape[-1] != 128 or block_size != 64 or k_cache.shape[1] != 64 or local_blocks <= 0
            or k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1 or q.stride(-1) != 1
            or output.stride(-1) != 1):
        return None
    ti = topk_idx.unsqueeze(0) if topk_idx.dim() == 2 else topk_idx
    if ti.shape[0] > 1 and ti.stride(0) != 0:
        return None
    bb = None
    if blk_bias is not None:
        bb = blk_bias.unsqueeze(0) if blk_bias.dim() == 2 else blk_bias
        if bb.shape[0] > 1 and bb.stride(0) != 0:
            return None
        bb = bb[0]
    ti = ti[0]
    cu = cu_seqlens_q.tolist()
    ctxs = prefix_lens.tolist()
    if not any(cu[r + 1] - cu[r] >= TC_MIN_ROWS for r in range(len(ctxs))):
        return None
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    rest = []
    for r, ctx in enumerate(ctxs):
        a, b = cu[r], cu[r + 1]
        if b - a < TC_MIN_ROWS:
            if b > a:
                rest.append((r, a, b, ctx))
            continue
        nblk = (ctx + b - a + block_size - 1) // block_size
        if nblk > bt.shape[1]:  # the block table must cover every key block
            rest.append((r, a, b, ctx))
            continue
        sel = ops.pack_selection(ti[a:b].unsqueeze(0), nblk)
        bias = None if bb is None else bb[a:b].contiguous()
        pages = bt[r].contiguous()
        try:
            ops.gather_fwd_paged(q[a:b], k_cache, v_cache, sel, bias, pages, ctx, block_size, sm_scale,
                                 local_blocks * block_size, output[a:b])
        except NotImplementedError:
            rest.append((r, a, b, ctx))
    return rest


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
    """Refresh k_bar of the last ``tail_pages`` pages of every request, or of
    the pages of ``plan`` = (pages, tokens) when given (the reference's
    kbar_tail_plan / kbar_all_plan output; entries with no token are
    skipped)."""
    assert kv_cache.shape[1] == block_size
    if plan is not None:
        pages, tok = plan
        ops.kbar_pages(kv_cache, head_cls, pages, tok, k_bar)
        return
    ops.kbar_paged(kv_cache, head_cls, block_table, seq_lens, k_bar, tail_pages)


kbar_refresh_tail_triton = kbar_refresh_tail


@torch.no_grad()
def win_bounds_decode(*, allow, seq_lens, lo, hi, fit, max_block: int, block_size: int, local_blocks: int,
                      decode_query_len: int, tile: int):
    """Fill lo / hi / fit (int32 / int32 / int8 [nd]) in place from the
    per-decode-row allow mask [>= nd, WQ] (bool or uint8)."""
    nd = int(lo.numel())
    if nd <= 0:
        return
    a = allow.view(torch.uint8) if allow.dtype == torch.bool else allow
    if a.dtype not in (torch.uint8, torch.int8):
        a = (a != 0).to(torch.uint8)
    if a.stride(-1) != 1:
        a = a.contiguous()
    for t, dt in ((lo, torch.int32), (hi, torch.int32), (fit, torch.int8)):
        if t.dtype != dt or not t.is_contiguous():
            raise ValueError("win_bounds_decode: lo / hi must be contiguous int32, fit contiguous int8")
    sl = seq_lens if (seq_lens.dtype == torch.int32 and seq_lens.is_contiguous()) else \
        seq_lens.to(torch.int32).contiguous()
    rc = L.lib().srswa_win_bounds_decode(a.data_ptr(), a.stride(0), a.shape[1], sl.data_ptr(), nd, int(max_block),
                                         int(block_size), int(local_blocks), max(1, int(decode_query_len)),
                                         int(tile), lo.data_ptr(), hi.data_ptr(), fit.data_ptr(),
                                         L.stream_of(lo))
    L.check(rc, "srswa_win_bounds_decode")


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


def route_decode_triton(*, idx_q, k_bar, block_table, seq_lens, image_allow, out_idx, out_bias, max_block: int,
                        block_size: int, local_blocks: int, decode_query_len: int, idx_scale: float,
                        prior_floor: float, sigma: float, topm: int, score_buf=None, budget: int | None = None,
                        out_slots: int | None = None, entmax_base=None, entmax_fit=None, entmax_width: int = 0,
                        score_buf_win=None, bounds=None):
    """The reference's decode router signature.  score_buf and the scan-window
    arguments (bounds, entmax_base / fit / width, score_buf_win) only choose
    how the reference's kernels tile the scan; the selection does not depend
    on them, and the kernels here scan the live width in one pass."""
    del score_buf, entmax_base, entmax_fit, entmax_width, score_buf_win, bounds
    return route_decode(idx_q=idx_q, k_bar=k_bar, block_table=block_table, seq_lens=seq_lens,
                        image_allow=image_allow, out_idx=out_idx, out_bias=out_bias, max_block=max_block,
                        block_size=block_size, local_blocks=local_blocks, decode_query_len=decode_query_len,
                        idx_scale=idx_scale, prior_floor=prior_floor, sigma=sigma, topm=topm, budget=budget,
                        out_slots=out_slots)


# A request with at least this many rows is routed on its own by the tiled
# routers (32 rows share each k_bar chunk; past 12288 blocks of a paged
# k_bar the library takes its per-row pass for such a call).
ROUTE_TILE_MIN_ROWS = 64


def _route_by_request(idx_q, k_bar, bt, seq_lens, cu_seqlens_q, row2req, q_pos, cand, out_idx, out_bias, kw):
    """Routes each request of at least ROUTE_TILE_MIN_ROWS rows with its own
    call (the tiled router; the varlen per-row score pass would read the
    request's k_bar once per row) and the remaining rows with one varlen
    call on their gathered rows.  Same results as one varlen call.  Returns
    False (nothing done) when no request is long enough or a CUDA graph is
    being captured.  Reads cu_seqlens_q on the host."""
    if torch.cuda.is_current_stream_capturing():  # no host reads inside a CUDA graph capture
        return False
    cu = cu_seqlens_q.tolist()
    R = len(cu) - 1
    long_r = [r for r in range(R) if cu[r + 1] - cu[r] >= ROUTE_TILE_MIN_ROWS]
    if not long_r:
        return False
    dev = idx_q.device
    sl = seq_lens.to(device=dev, dtype=torch.int32)
    per_row = cand is not None and cand.dim() == 2 and cand.shape[0] == idx_q.shape[0] and cand.shape[0] > 1

    def rows_of(m, sel):  # a per-row mask follows its rows; a shared row stays as it is
        return None if m is None else (m[sel] if per_row else m)

    for r in long_r:
        a, b = cu[r], cu[r + 1]
        ops.route(idx_q[a:b], k_bar, seq_lens=sl[r:r + 1], q_pos=q_pos[a:b], rows_per_seq=b - a,
                  block_table=bt[r:r + 1], cand=rows_of(cand, slice(a, b)),
                  out={"topi32": out_idx[a:b], "bias": out_bias[a:b]}, **kw)
    short = [torch.arange(cu[r], cu[r + 1]) for r in range(R)
             if 0 < cu[r + 1] - cu[r] < ROUTE_TILE_MIN_ROWS]
    if short:
        idx = torch.cat(short).to(dev)
        res = ops.route(idx_q[idx], k_bar, seq_lens=sl, q_pos=q_pos[idx], row_seq=row2req[idx], block_table=bt,
                        cand=rows_of(cand, idx), **kw)
        out_idx.index_copy_(0, idx, res["topi32"])
        out_bias.index_copy_(0, idx, res["bias"])
    return True


@torch.no_grad()
def route_prefill_triton(*, idx_q, k_bar, block_table, seq_lens, cu_seqlens_q, context_lens, row2req, image_allow,
                         out_idx, out_bias, max_block: int, block_size: int, local_blocks: int, idx_scale: float,
                         prior_floor: float, sigma: float, topm: int, budget: int | None = None,
                         q_chunk: int = 2048, out_slots: int | None = None, score_buf=None):
    """Route varlen prefill rows idx_q [total_q, d]: row i of request
    r = row2req[i] sits at position context_lens[r] + i - cu_seqlens_q[r].
    Writes out_idx / out_bias like route_decode; returns (slot width, None,
    0): no q_chunk loop, so no last score chunk to hand back.  Requests of
    at least ROUTE_TILE_MIN_ROWS rows are routed one by one by the tiled
    routers, the other rows in one varlen launch."""
    del q_chunk, score_buf
    dev = idx_q.device
    N = int(idx_q.shape[0])
    W = min(int(max_block), int(block_table.shape[1]))
    K = max(1, min(int(budget or topm), int(topm)))
    Ke, _ = ops.effective_km(K, topm, W)
    width = out_slots or Ke
    if N == 0:
        return width, None, 0
    r = row2req.to(device=dev, dtype=torch.int64)
    rows = torch.arange(N, device=dev, dtype=torch.int64)
    q_pos = (context_lens.to(device=dev, dtype=torch.int64)[r] + rows
             - cu_seqlens_q.to(device=dev, dtype=torch.int64)[r])
    direct = (out_idx.dtype == torch.int32 and out_bias.dtype == torch.float32 and out_idx.is_contiguous()
              and out_bias.is_contiguous() and tuple(out_idx.shape) == (N, Ke) and tuple(out_bias.shape) == (N, Ke))
    kw = dict(block_size=block_size, local_blocks=local_blocks, topk=K, topm=topm, idx_scale=idx_scale,
              floor=prior_floor, sigma=sigma, want=("topi32", "bias"), nblk=W)
    if direct and _route_by_request(idx_q, k_bar, block_table[:, :W], seq_lens,
                                                                   cu_seqlens_q, row2req, q_pos, image_allow,
                                                                   out_idx, out_bias, kw):
        return width, None, 0
    res = ops.route(idx_q, k_bar, block_size=block_size, local_blocks=local_blocks, topk=K, topm=topm,
                    idx_scale=idx_scale, floor=prior_floor, sigma=sigma, seq_lens=seq_lens, q_pos=q_pos,
                    row_seq=row2req, block_table=block_table[:, :W], cand=image_allow, want=("topi32", "bias"),
                    nblk=W, out={"topi32": out_idx, "bias": out_bias} if direct else None)
    if not direct:
        k = res["topi32"].shape[-1]
        out_idx[:N, :k].copy_(res["topi32"])
        out_bias[:N, :k].copy_(res["bias"])
        if out_idx.shape[-1] > k:
            out_idx[:N, k:].fill_(-1)
            out_bias[:N, k:].zero_()
    return width, None, 0

