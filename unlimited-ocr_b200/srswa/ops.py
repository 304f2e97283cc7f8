"""Thin torch-facing wrappers over the C ABI (one function per entry point).

Every function takes CUDA tensors, allocates its outputs (and any workspace)
through torch's caching allocator, launches on the current stream and returns.
"""

from __future__ import annotations

import ctypes as C
import math
import os

import torch

from . import _lib as L


def _cand_args(cand, N, nblk):
    if cand is None:
        return None, 0
    c = cand
    if c.dtype == torch.bool:
        c = c.view(torch.uint8)
    elif c.dtype != torch.uint8:
        c = c.to(torch.uint8)
    if c.dim() == 1:
        return c.contiguous(), 0
    if c.dim() == 2 and c.shape[1] > nblk:
        c = c[:, :nblk]          # a mask wider than the scored blocks (the serving [rows, WQ] layout)
    else:
        c = c.reshape(-1, nblk)
    if c.shape[0] == 1:
        return c.contiguous(), 0
    if c.stride(-1) != 1:
        c = c.contiguous()
    assert c.shape[0] == N
    return c, c.stride(0)


def _route_params(block_size, local_blocks, topk, topm, idx_scale, floor, sigma):
    return L.RouteParams(int(block_size), int(local_blocks), int(topk), int(topm),
                         float(idx_scale), float(floor), float(sigma))


def _check_rows(N, rows_per_seq, kbar, block_table, nblk):
    """Every query row must map to an existing sequence of the k_bar source
    (row n belongs to sequence n // rows_per_seq), and a block table must
    cover the blocks scored; checked here because the C interface takes no
    sequence count."""
    nseq = -(-N // int(rows_per_seq))
    if block_table is None:
        if kbar.shape[0] < nseq:
            raise ValueError(f"{N} rows at {rows_per_seq} per sequence need {nseq} k_bar sequences, "
                             f"got {kbar.shape[0]}")
    elif block_table.shape[0] < nseq or block_table.shape[1] < nblk:
        raise ValueError(f"block_table {tuple(block_table.shape)} does not cover {nseq} sequences x {nblk} blocks")


def effective_km(topk, topm, nblk):
    M = max(1, min(int(topm), nblk)) if int(topm) > 0 else nblk
    K = max(1, min(int(topk), M))
    return K, M


def kbar_contig(idx_k: torch.Tensor, head_cls: torch.Tensor, block_size: int, out=None, chunk_valid=True):
    """[B,S,d] index keys -> (kbar [B,nblk,d] fp32, chunk_valid [B,nblk] bool).
    out: a caller's [B, nblk, d] fp32 tensor with contiguous rows (written in
    place, e.g. a slice of a larger k_bar); chunk_valid=False skips that output
    (returned as None)."""
    B, S, d = idx_k.shape
    if idx_k.stride(-1) != 1:
        idx_k = idx_k.contiguous()
    nblk = (S + block_size - 1) // block_size
    if out is None:
        out = torch.empty(B, nblk, d, device=idx_k.device, dtype=torch.float32)
    elif (out.shape != (B, nblk, d) or out.dtype != torch.float32 or out.stride(2) != 1
          or out.stride(1) != d or (B > 1 and out.stride(0) != nblk * d)):
        raise ValueError("out must be a [B, nblk, d] fp32 tensor laid out contiguously")
    cv = torch.empty(B, nblk, device=idx_k.device, dtype=torch.uint8) if chunk_valid else None
    hc = head_cls if (head_cls.dtype == torch.float32 and head_cls.is_contiguous()
                      and head_cls.device == idx_k.device) else \
        head_cls.to(device=idx_k.device, dtype=torch.float32).contiguous()
    rc = L.lib().srswa_kbar_contig(idx_k.data_ptr(), L.dtype_code(idx_k), idx_k.stride(0), idx_k.stride(1),
                                   B, S, d, block_size, hc.data_ptr(), out.data_ptr(), L.ptr(cv),
                                   L.stream_of(idx_k))
    L.check(rc, "srswa_kbar_contig")
    return out, (cv.view(torch.bool) if cv is not None else None)


def kbar_paged(idx_cache, head_cls, block_table, seq_lens, kbar_cache, tail_pages=0):
    """Refresh k_bar of the last `tail_pages` pages per request (all when <= 0)."""
    P, BS, d = idx_cache.shape
    assert idx_cache.stride(-1) == 1 and kbar_cache.stride(-1) == 1
    bt = block_table.to(torch.int32).contiguous()
    sl = seq_lens.to(torch.int32).contiguous()
    hc = head_cls.to(device=idx_cache.device, dtype=torch.float32).contiguous()
    rc = L.lib().srswa_kbar_paged(idx_cache.data_ptr(), L.dtype_code(idx_cache), idx_cache.stride(0),
                                  idx_cache.stride(1), d, BS, bt.data_ptr(), bt.stride(0), bt.shape[1],
                                  sl.data_ptr(), sl.shape[0], int(tail_pages), hc.data_ptr(),
                                  kbar_cache.data_ptr(), kbar_cache.stride(0), L.stream_of(idx_cache))
    L.check(rc, "srswa_kbar_paged")


def kbar_pages(idx_cache, head_cls, pages, tok, kbar_cache):
    """k_bar of an explicit page plan: pages [n] (page ids), tok [n] (tokens
    in use; <= 0: skipped) -> kbar_cache rows written in place."""
    P, BS, d = idx_cache.shape
    assert idx_cache.stride(-1) == 1 and kbar_cache.stride(-1) == 1
    pg = pages.to(device=idx_cache.device, dtype=torch.int64).contiguous().view(-1)
    tk = tok.to(device=idx_cache.device, dtype=torch.int32).contiguous().view(-1)
    assert pg.numel() == tk.numel()
    hc = head_cls.to(device=idx_cache.device, dtype=torch.float32).contiguous()
    rc = L.lib().srswa_kbar_pages(idx_cache.data_ptr(), L.dtype_code(idx_cache), idx_cache.stride(0),
                                  idx_cache.stride(1), d, BS, pg.data_ptr(), tk.data_ptr(), pg.numel(),
                                  hc.data_ptr(), kbar_cache.data_ptr(), kbar_cache.stride(0),
                                  L.stream_of(idx_cache))
    L.check(rc, "srswa_kbar_pages")


def route(idx_q, kbar, *, block_size, local_blocks, topk, topm, idx_scale, floor, sigma,
          q_pos=None, seq_lens=None, rows_per_seq=1, block_table=None, cand=None,
          want=("topi64", "bias", "valid"), nblk=None, out=None, row_seq=None):
    """Fused scores + selection for query rows idx_q [N, d].

    kbar: contiguous [B, nblk, d] (block_table None) or paged cache [P, d].
    Row n belongs to sequence n // rows_per_seq, or row_seq[n] (int32 [N],
    varlen prefill rows; needs q_pos).
    Returns a dict with the requested outputs among topi64, topi32, bias,
    valid, scores.  out: caller-owned tensors for some of them (contiguous,
    [N, K] or [N, nblk], the output's dtype), written in place."""
    N, d = idx_q.shape
    if idx_q.stride(-1) != 1:
        idx_q = idx_q.contiguous()
    dev = idx_q.device
    if block_table is None:
        B, nb, _ = kbar.shape
        s_b, s_c = kbar.stride(0), kbar.stride(1)
        bt = None
        nblk = nb if nblk is None else nblk
    else:
        s_b, s_c = 0, kbar.stride(0)
        bt = block_table.to(torch.int32).contiguous()
        nblk = bt.shape[1] if nblk is None else nblk
    if row_seq is None:
        _check_rows(N, rows_per_seq, kbar, bt, nblk)
    else:
        if q_pos is None:
            raise ValueError("route: varlen rows (row_seq) need q_pos")
        row_seq = row_seq.to(device=dev, dtype=torch.int32).contiguous()
    K, M = effective_km(topk, topm, nblk)
    given = out or {}
    out = {}
    for name, dt, shape in (("topi64", torch.int64, (N, K)), ("topi32", torch.int32, (N, K)),
                            ("bias", torch.float32, (N, K)), ("valid", torch.uint8, (N, K)),
                            ("scores", torch.float32, (N, nblk))):
        t = given.get(name)
        if t is not None:
            if t.dtype != dt or tuple(t.shape) != shape or not t.is_contiguous() or t.device != dev:
                raise ValueError(f"route: out[{name!r}] must be a contiguous {dt} {shape} tensor on {dev}")
            out[name] = t
        else:
            out[name] = torch.empty(shape, device=dev, dtype=dt) if name in want else None
    qp = None if q_pos is None else q_pos.to(device=dev, dtype=torch.int64).contiguous().view(-1)
    sl = None if seq_lens is None else seq_lens.to(device=dev, dtype=torch.int32).contiguous()
    cnd, s_cand = _cand_args(cand, N, nblk)
    p = _route_params(block_size, local_blocks, topk, topm, idx_scale, floor, sigma)
    lib = L.lib()
    ws_n = lib.srswa_route_workspace_size(N, nblk, d, p, 1 if cnd is not None else 0)

    def call(ws, n):
        return lib.srswa_route(idx_q.data_ptr(), L.dtype_code(idx_q), idx_q.stride(0), N, d,
                               kbar.data_ptr(), s_b, s_c, nblk, L.ptr(bt), 0 if bt is None else bt.stride(0),
                               L.ptr(sl), int(rows_per_seq), L.ptr(row_seq), L.ptr(qp), L.ptr(cnd), s_cand, p,
                               L.ptr(out["topi64"]), L.ptr(out["topi32"]), L.ptr(out["bias"]),
                               L.ptr(out["valid"]), L.ptr(out["scores"]), L.ptr(ws), n, L.stream_of(idx_q))

    rc = L.EWORKSPACE
    if ws_n and row_seq is None and int(rows_per_seq) >= 32:
        # prefill-shaped rows usually take the tiled routers, which need no
        # workspace: try without (nothing is launched when the call needs one)
        rc = call(None, 0)
    if rc == L.EWORKSPACE:
        rc = call(torch.empty(ws_n, device=dev, dtype=torch.uint8) if ws_n else None, ws_n)
    L.check(rc, "srswa_route")
    if out["valid"] is not None:
        out["valid"] = out["valid"].view(torch.bool)  # 0 / 1 bytes: no copy
    return {k: v for k, v in out.items() if v is not None}


def route_shard_keys(idx_q, kbar, *, block_offset, nblk_local, nblk_total, block_size, local_blocks, topk, topm,
                     idx_scale, floor, sigma, q_pos=None, seq_lens=None, rows_per_seq=1, block_table=None,
                     out=None, push=None, workspace=None):
    """Split-KV router stage 1: packed top-M keys [N, M] (int64 storage of
    the uint64 keys) of the blocks this shard owns, global ids
    [block_offset, block_offset + nblk_local).  kbar: the shard's contiguous
    [B, nblk_local, d], or a paged cache [P, d] with block_table [R, >=
    nblk_total] indexed by global block id."""
    N, d = idx_q.shape
    if idx_q.stride(-1) != 1:
        idx_q = idx_q.contiguous()
    dev = idx_q.device
    if block_table is None:
        s_b, s_c, bt = kbar.stride(0), kbar.stride(1), None
    else:
        s_b, s_c = 0, kbar.stride(0)
        bt = block_table if block_table.dtype == torch.int32 and block_table.is_contiguous() else \
            block_table.to(torch.int32).contiguous()
    _check_rows(N, rows_per_seq, kbar, bt, nblk_total)
    if bt is None and kbar.shape[1] < nblk_local:
        raise ValueError(f"k_bar holds {kbar.shape[1]} blocks, shard has {nblk_local}")
    _, M = effective_km(topk, topm, nblk_total)
    if out is None:
        out = torch.empty(N, M, device=dev, dtype=torch.int64)
    qp = None if q_pos is None else q_pos.to(device=dev, dtype=torch.int64).contiguous().view(-1)
    sl = None if seq_lens is None else seq_lens.to(device=dev, dtype=torch.int32).contiguous()
    p = _route_params(block_size, local_blocks, topk, topm, idx_scale, floor, sigma)
    lib = L.lib()
    ws_n = lib.srswa_route_shard_workspace_size(N, int(nblk_local), p)
    ws = _workspace(ws_n, dev, workspace) if ws_n else None
    rc = lib.srswa_route_shard_keys(idx_q.data_ptr(), L.dtype_code(idx_q), idx_q.stride(0), N, d,
                                    kbar.data_ptr(), s_b, s_c, int(nblk_local), int(block_offset),
                                    int(nblk_total), L.ptr(bt), 0 if bt is None else bt.stride(0), L.ptr(sl),
                                    int(rows_per_seq), L.ptr(qp), p, out.data_ptr(), L.ptr(ws), ws_n,
                                    None if push is None else C.byref(push), L.stream_of(idx_q))
    L.check(rc, "srswa_route_shard_keys")
    return out


def route_shard_select(idx_q, kbar, *, block_offset, nblk_local, nblk_total, block_size, local_blocks, topk, topm,
                       idx_scale, floor, sigma, q_pos=None, seq_lens=None, rows_per_seq=1, block_table=None,
                       own=None, want=("topi64", "bias", "valid"), exchange=None, workspace=None):
    """Both split-KV router stages in one launch (srswa_route_shard_select):
    this shard's keys, then -- alone, or merged with every rank's keys through
    the peer exchange ``exchange`` (an srswa_peer; every rank calls) -- the
    selection of the whole row, outputs as route_merge_keys."""
    N, d = idx_q.shape
    if idx_q.stride(-1) != 1:
        idx_q = idx_q.contiguous()
    dev = idx_q.device
    if block_table is None:
        s_b, s_c, bt = kbar.stride(0), kbar.stride(1), None
    else:
        s_b, s_c = 0, kbar.stride(0)
        bt = block_table if block_table.dtype == torch.int32 and block_table.is_contiguous() else \
            block_table.to(torch.int32).contiguous()
    _check_rows(N, rows_per_seq, kbar, bt, nblk_total)
    if bt is None and kbar.shape[1] < nblk_local:
        raise ValueError(f"k_bar holds {kbar.shape[1]} blocks, shard has {nblk_local}")
    K, _ = effective_km(topk, topm, nblk_total)
    out = {}
    for name, dt in (("topi64", torch.int64), ("topi32", torch.int32), ("bias", torch.float32),
                     ("valid", torch.uint8), ("topi32_own", torch.int32)):
        req = name in want or (name == "topi32_own" and own is not None)
        out[name] = torch.empty(N, K, device=dev, dtype=dt) if req else None
    lo, hi = own if own is not None else (0, 0)
    qp = None if q_pos is None else q_pos.to(device=dev, dtype=torch.int64).contiguous().view(-1)
    sl = None if seq_lens is None else seq_lens.to(device=dev, dtype=torch.int32).contiguous()
    p = _route_params(block_size, local_blocks, topk, topm, idx_scale, floor, sigma)
    lib = L.lib()
    ws_n = lib.srswa_route_shard_workspace_size(N, int(nblk_local), p)
    ws = _workspace(ws_n, dev, workspace) if ws_n else None
    rc = lib.srswa_route_shard_select(idx_q.data_ptr(), L.dtype_code(idx_q), idx_q.stride(0), N, d,
                                      kbar.data_ptr(), s_b, s_c, int(nblk_local), int(block_offset),
                                      int(nblk_total), L.ptr(bt), 0 if bt is None else bt.stride(0), L.ptr(sl),
                                      int(rows_per_seq), L.ptr(qp), p, L.ptr(out["topi64"]), L.ptr(out["topi32"]),
                                      L.ptr(out["bias"]), L.ptr(out["valid"]), int(lo), int(hi),
                                      L.ptr(out["topi32_own"]), L.ptr(ws), ws_n,
                                      None if exchange is None else C.byref(exchange), L.stream_of(idx_q))
    L.check(rc, "srswa_route_shard_select")
    if out["valid"] is not None:
        out["valid"] = out["valid"].view(torch.bool)
    return {k: v for k, v in out.items() if v is not None}


def route_merge_keys(keys, *, nblk_total, topk, topm, idx_scale, floor, sigma, own=None,
                     want=("topi64", "bias", "valid"), wait=None):
    """Split-KV router stage 2: keys [nlists, N, M] (the all-gathered stage-1
    outputs) -> the selection of the whole row, as srswa_route.  own =
    (lo, hi) adds "topi32_own": topi32 with -1 outside the owned range."""
    nl, N, M = keys.shape
    assert keys.stride(2) == 1
    dev = keys.device
    K, _ = effective_km(topk, topm, nblk_total)
    out = {}
    for name, dt in (("topi64", torch.int64), ("topi32", torch.int32), ("bias", torch.float32),
                     ("valid", torch.uint8), ("topi32_own", torch.int32)):
        req = name in want or (name == "topi32_own" and own is not None)
        out[name] = torch.empty(N, K, device=dev, dtype=dt) if req else None
    lo, hi = own if own is not None else (0, 0)
    p = _route_params(1, 0, topk, topm, idx_scale, floor, sigma)
    rc = L.lib().srswa_route_merge_keys(keys.data_ptr(), nl, keys.stride(0), keys.stride(1), N, int(nblk_total), p,
                                        L.ptr(out["topi64"]), L.ptr(out["topi32"]), L.ptr(out["bias"]),
                                        L.ptr(out["valid"]), int(lo), int(hi), L.ptr(out["topi32_own"]),
                                        None if wait is None else C.byref(wait), L.stream_of(keys))
    L.check(rc, "srswa_route_merge_keys")
    if out["valid"] is not None:
        out["valid"] = out["valid"].view(torch.bool)  # 0 / 1 bytes: no copy
    return {k: v for k, v in out.items() if v is not None}


def route_select(scores, cand, *, topk, topm, idx_scale, floor, sigma, want=("topi64", "bias", "valid")):
    """Selection from given scores [..., nblk] (fp32)."""
    shape = scores.shape
    nblk = shape[-1]
    sc = scores.reshape(-1, nblk)
    if sc.dtype != torch.float32 or sc.stride(-1) != 1:
        sc = sc.float().contiguous()
    N = sc.shape[0]
    K, M = effective_km(topk, topm, nblk)
    dev = sc.device
    out = {}
    for name, dt in (("topi64", torch.int64), ("topi32", torch.int32), ("bias", torch.float32),
                     ("valid", torch.uint8)):
        out[name] = torch.empty((N, K), device=dev, dtype=dt) if name in want else None
    cnd, s_cand = _cand_args(cand, N, nblk)
    p = _route_params(1, 0, topk, topm, idx_scale, floor, sigma)
    rc = L.lib().srswa_route_select(sc.data_ptr(), sc.stride(0), N, nblk, L.ptr(cnd), s_cand, p,
                                    L.ptr(out["topi64"]), L.ptr(out["topi32"]), L.ptr(out["bias"]),
                                    L.ptr(out["valid"]), L.stream_of(sc))
    L.check(rc, "srswa_route_select")
    res = {}
    for k, v in out.items():
        if v is None:
            continue
        v = v.view(*shape[:-1], K)
        res[k] = v.view(torch.bool) if k == "valid" else v
    return res


def block_max_score(q, k, pos, seg, block_size, num_key_blocks, local_window, mode):
    B, Cq, D = q.shape
    Sk = k.shape[1]
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    out = torch.empty(B, Cq, num_key_blocks, device=q.device, dtype=torch.float32)
    pos = pos.to(torch.int64).contiguous()
    seg = None if seg is None else seg.to(torch.int64).contiguous()
    rc = L.lib().srswa_block_max_score(q.data_ptr(), L.dtype_code(q), q.stride(0), q.stride(1),
                                       k.data_ptr(), L.dtype_code(k), k.stride(0), k.stride(1),
                                       pos.data_ptr(), L.ptr(seg), B, Cq, Sk, D, block_size,
                                       num_key_blocks, int(local_window), int(mode), out.data_ptr(),
                                       L.stream_of(q))
    L.check(rc, "srswa_block_max_score")
    return out


def pack_selection(sel, nblk):
    """int32 copy of sel with ids outside [0, nblk) and repeats inside a row -> -1."""
    s = sel.contiguous()
    is64 = 1 if s.dtype == torch.int64 else 0
    if s.dtype not in (torch.int64, torch.int32):
        s = s.to(torch.int64)
        is64 = 1
    out = torch.empty(s.shape, device=s.device, dtype=torch.int32)
    if s.numel() == 0:
        return out
    S = s.shape[-1]
    rows = s.numel() // max(S, 1)
    rc = L.lib().srswa_pack_selection(s.data_ptr(), is64, rows, S, int(nblk), out.data_ptr(), L.stream_of(s))
    L.check(rc, "srswa_pack_selection")
    return out


def _gather_desc(q, k, v, sel, block_size, scale, local_window):
    B, T, HQ, D = q.shape
    Hkv = k.shape[2]
    HI, S = sel.shape[1], sel.shape[-1]
    lw = block_size if local_window is None else max(1, int(local_window))
    return L.GatherDesc(B, T, HQ, Hkv, HI, D, S, int(block_size), lw, float(scale), L.dtype_code(q),
                        q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
                        v.stride(0), v.stride(1), v.stride(2))


_CHECK_STATUS = os.environ.get("SRSWA_CHECK_STATUS", "0") not in ("", "0")


def workspace_status(ws) -> int:
    """Status word of the last gather call made with workspace ``ws`` (a
    uint8 CUDA tensor): 0, or the code of a tensor-core kernel's bounded wait
    that expired.  Waits for the current stream."""
    v = C.c_int(0)
    L.check(L.lib().srswa_workspace_status(ws.data_ptr(), C.byref(v), L.stream_of(ws)), "srswa_workspace_status")
    return v.value


def _workspace(n, dev, given):
    if given is None:
        return torch.empty(max(n, 1), device=dev, dtype=torch.uint8)
    if given.dtype != torch.uint8 or given.numel() < n or not given.is_contiguous():
        raise ValueError(f"workspace must be a contiguous uint8 tensor of at least {n} bytes")
    return given


def _after_gather(ws, what):
    # opt-in (SRSWA_CHECK_STATUS=1): wait for the call and raise on an expired wait
    if _CHECK_STATUS:
        code = workspace_status(ws)
        if code:
            raise L.SrswaError(f"{what}: a bounded wait expired in a tensor-core kernel (code {code})")


def gather_fwd(q, k, v, sel, bias, seg, block_size, scale, local_window, workspace=None):
    """q/k/v [B,T,H,D] (D contiguous), sel [B,HI,T,S] int32 packed, bias [B,T,S]
    fp32 or None, seg [B,T] int32 or None -> (o [B,T,HQ,D] q.dtype, lse [B,T,HQ]).
    workspace: optional caller uint8 tensor (srswa_gather_fwd_workspace_size
    bytes); its first 4 bytes hold the call's status word afterwards."""
    B, T, HQ, D = q.shape
    o = torch.empty(B, T, HQ, D, device=q.device, dtype=q.dtype)
    lse = torch.empty(B, T, HQ, device=q.device, dtype=torch.float32)
    g = _gather_desc(q, k, v, sel, block_size, scale, local_window)
    lib = L.lib()
    ws_n = lib.srswa_gather_fwd_workspace_size(C.byref(g))
    ws = _workspace(ws_n, q.device, workspace)
    rc = lib.srswa_gather_fwd(C.byref(g), q.data_ptr(), k.data_ptr(), v.data_ptr(), sel.data_ptr(),
                              L.ptr(bias), L.ptr(seg), o.data_ptr(), L.dtype_code(o), o.stride(0),
                              o.stride(1), o.stride(2), lse.data_ptr(), ws.data_ptr(), ws_n, L.stream_of(q))
    L.check(rc, "srswa_gather_fwd")
    _after_gather(ws, "srswa_gather_fwd")
    return o, lse


def gather_bwd(q, k, v, o, lse, do, sel, bias, seg, block_size, scale, local_window, workspace=None):
    """Gradients (dq, dk, dv, d_bias or None) of gather_fwd; workspace as there."""
    g = _gather_desc(q, k, v, sel, block_size, scale, local_window)
    lib = L.lib()
    if do.stride() != o.stride():
        do = do.contiguous()
        o = o.contiguous()
        assert do.stride() == o.stride()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    assert dq.stride() == q.stride() and dk.stride() == k.stride() and dv.stride() == v.stride()
    d_bias = None
    if bias is not None:
        d_bias = torch.empty(bias.shape, device=q.device, dtype=torch.float32)
    ws_n = lib.srswa_gather_bwd_workspace_size(C.byref(g))
    ws = _workspace(ws_n, q.device, workspace)
    rc = lib.srswa_gather_bwd(C.byref(g), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                              o.stride(0), o.stride(1), o.stride(2), do.data_ptr(), lse.data_ptr(),
                              sel.data_ptr(), L.ptr(bias), L.ptr(seg), dq.data_ptr(), dk.data_ptr(),
                              dv.data_ptr(), L.ptr(d_bias), ws.data_ptr(), ws_n, L.stream_of(q))
    L.check(rc, "srswa_gather_bwd")
    _after_gather(ws, "srswa_gather_bwd")
    return dq, dk, dv, d_bias


def decode_attend(q, k_cache, v_cache, topk_idx, bias, *, block_size, local_blocks, sm_scale,
                  out=None, block_table=None, seq_lens=None, q_pos=None, rows_per_req=1,
                  valid=None, lse=False, nsplit=0, kv_layout=None, skip_local=False, lse_out=None,
                  overlap=False, push=None, merged_out=None, merged_lse=None):
    """Sparse decode attend.  q [N,H,D]; paged k/v caches [P, BS, Hkv, D] (any
    strides with D contiguous) indexed by block_table [R,W].  With
    block_table None, kv_layout = (R, W, s_req, s_pos, s_head, Hkv) describes
    one contiguous cache per request (block blk of request r at r*s_req +
    blk*BS*s_pos).  topk_idx [Hkv or 1 (stride 0 ok), N, K] or [N, K]; bias
    like topk_idx or None.  skip_local: attend the selected remote blocks
    only (a split-KV shard that does not own the window).  overlap: the
    attend starts on the window keys while the kernel just before it on the
    stream (the router that made topk_idx / bias) finishes; q, the caches,
    block_table, seq_lens and q_pos must have been written before that
    kernel began (srswa_decode_desc.overlap).  Same results either way.
    push (an srswa_peer): out / lse_out are fp32 views of this rank's own
    slot of that exchange and the results are also stored into every peer's
    region (srswa_decode_attend_push).  merged_out (with an LL push): the
    attend also waits for every rank's partial and writes their log-sum-exp
    merge there (and to merged_lse), srswa_decode_attend_exchange; raises
    NotImplementedError (ETOOLARGE, nothing launched) when the grid would not
    be resident at once."""
    N, H, D = q.shape
    assert k_cache.stride() == v_cache.stride()
    if block_table is not None:
        P, BS, Hkv, _ = k_cache.shape
        assert BS == block_size
        s_page, s_pos, s_head = k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
        s_req = 0
    else:
        _, _, s_req, s_pos, s_head, Hkv = kv_layout
        s_page = block_size * s_pos
    if topk_idx.dim() == 2:
        topk_idx = topk_idx.unsqueeze(0)
    ti = topk_idx
    if ti.stride(-1) != 1:
        ti = ti.contiguous()
    s_ti_h = ti.stride(0) if ti.shape[0] > 1 else 0
    b = None
    s_b_h = s_b_n = 0
    if bias is not None:
        b = bias.unsqueeze(0) if bias.dim() == 2 else bias
        if b.dtype != torch.float32 or b.stride(-1) != 1:
            b = b.float().contiguous()
        s_b_h = b.stride(0) if b.shape[0] > 1 else 0
        s_b_n = b.stride(1)
    vd = None
    if valid is not None:
        vd = (valid.unsqueeze(0) if valid.dim() == 2 else valid).to(torch.uint8)
        vd = vd.expand(ti.shape).contiguous() if vd.shape != ti.shape else vd.contiguous()
        if vd.stride() != ti.stride():
            ti = ti.contiguous()
            vd = vd.contiguous()
            s_ti_h = ti.stride(0) if ti.shape[0] > 1 else 0
    if out is None:
        out = torch.empty(N, H, D, device=q.device, dtype=q.dtype)
    lse_t = None
    if lse:
        lse_t = lse_out if lse_out is not None else torch.empty(N, H, device=q.device, dtype=torch.float32)
        assert lse_t.shape == (N, H) and lse_t.is_contiguous() and lse_t.dtype == torch.float32
    bt = None if block_table is None else block_table.to(torch.int32).contiguous()
    sl = None if seq_lens is None else seq_lens.to(device=q.device, dtype=torch.int32).contiguous()
    qp = None if q_pos is None else q_pos.to(device=q.device, dtype=torch.int64).contiguous().view(-1)
    if bt is not None:
        R, W = bt.shape
    else:
        R, W = kv_layout[0], kv_layout[1]
    # an input converted here was written by a kernel right before the attend:
    # then the window may not be read early
    early = all(x is None or (x.data_ptr() == y.data_ptr() and x.dtype == y.dtype)
                for x, y in ((bt, block_table), (sl, seq_lens), (qp, q_pos)))
    d = L.DecodeDesc(N, H, Hkv, D, ti.shape[-1], block_size, local_blocks, float(sm_scale),
                     L.dtype_code(q), L.dtype_code(k_cache), L.dtype_code(out), q.stride(0), q.stride(1),
                     s_page, s_pos, s_head, out.stride(0), out.stride(1),
                     R, W, s_req, rows_per_req, 1 if ti.dtype == torch.int64 else 0,
                     s_ti_h, ti.stride(1), s_b_h, s_b_n, int(nsplit), 1 if skip_local else 0,
                     1 if (overlap and early) else 0)
    if ti.dtype not in (torch.int32, torch.int64):
        raise NotImplementedError("topk_idx must be int32 or int64")
    if merged_out is not None:
        assert merged_out.is_contiguous() and merged_out.shape == (N, H, D)
        rc = L.lib().srswa_decode_attend_exchange(C.byref(d), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                                  L.ptr(bt), L.ptr(sl), L.ptr(qp), ti.data_ptr(), L.ptr(b),
                                                  L.ptr(vd), out.data_ptr(), L.ptr(lse_t), C.byref(push),
                                                  merged_out.data_ptr(), L.dtype_code(merged_out),
                                                  L.ptr(merged_lse), L.stream_of(q))
        L.check(rc, "srswa_decode_attend_exchange")
        return merged_out
    if push is not None:
        rc = L.lib().srswa_decode_attend_push(C.byref(d), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                              L.ptr(bt), L.ptr(sl), L.ptr(qp), ti.data_ptr(), L.ptr(b), L.ptr(vd),
                                              out.data_ptr(), L.ptr(lse_t), C.byref(push), L.stream_of(q))
        L.check(rc, "srswa_decode_attend_push")
        return (out, lse_t) if lse else out
    rc = L.lib().srswa_decode_attend(C.byref(d), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                     L.ptr(bt), L.ptr(sl), L.ptr(qp), ti.data_ptr(), L.ptr(b), L.ptr(vd),
                                     out.data_ptr(), L.ptr(lse_t), L.stream_of(q))
    L.check(rc, "srswa_decode_attend")
    return (out, lse_t) if lse else out


def gather_fwd_paged(q, k_cache, v_cache, sel, bias, pages, qoff, block_size, scale, local_window, out,
                     workspace=None):
    """Tensor-core forward of one sequence over paged K / V: q [T, HQ, D]
    (its rows at positions qoff .. qoff + T - 1), caches [P, 64, Hkv, D],
    pages [>= ceil((qoff + T) / 64)] int32 (key block j is page pages[j]),
    sel [HI, T, S] int32 packed (pack_selection), bias [T, S] fp32 or None,
    out [T, HQ, D] written in place.  Raises NotImplementedError where the
    tensor-core path does not apply (shape, dtype, alignment)."""
    T_, HQ, D = q.shape
    P, BS, Hkv, _ = k_cache.shape
    if k_cache.stride() != v_cache.stride():
        raise NotImplementedError("k and v caches must share strides")
    HI, S = sel.shape[0], sel.shape[-1]
    lw = block_size if local_window is None else max(1, int(local_window))
    g = L.GatherDesc(1, T_, HQ, Hkv, HI, D, S, int(block_size), lw, float(scale), L.dtype_code(q),
                     0, q.stride(0), q.stride(1), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
                     v_cache.stride(0), v_cache.stride(1), v_cache.stride(2))
    lib = L.lib()
    ws_n = lib.srswa_gather_fwd_paged_workspace_size(C.byref(g), int(qoff))
    if ws_n == 0:
        raise NotImplementedError("gather_fwd_paged: not a tensor-core shape")
    ws = _workspace(ws_n, q.device, workspace)
    rc = lib.srswa_gather_fwd_paged(C.byref(g), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), P,
                                    pages.data_ptr(), int(qoff), sel.data_ptr(), L.ptr(bias), out.data_ptr(),
                                    0, out.stride(0), out.stride(1), None, ws.data_ptr(), ws_n, L.stream_of(q))
    L.check(rc, "srswa_gather_fwd_paged")
    _after_gather(ws, "srswa_gather_fwd_paged")
    return out


def prefill_attend(q, k_cache, v_cache, topk_idx, bias, *, block_table, cu_seqlens_q, prefix_lens, block_size,
                   local_blocks, sm_scale, out=None, lse=False):
    """Paged varlen prefill attend: q [total_q, H, D]; caches [P, BS, Hkv, D];
    rows of request r are cu_seqlens_q[r] .. cu_seqlens_q[r+1]-1 at positions
    prefix_lens[r] + i; topk_idx / bias [Hkv or 1 (stride 0 ok), total_q, K]
    or [total_q, K] (-1 = unused slot)."""
    N, H, D = q.shape
    assert k_cache.stride() == v_cache.stride()
    P, BS, Hkv, _ = k_cache.shape
    assert BS == block_size
    ti = topk_idx.unsqueeze(0) if topk_idx.dim() == 2 else topk_idx
    if ti.dtype not in (torch.int32, torch.int64):
        raise NotImplementedError("topk_idx must be int32 or int64")
    if ti.stride(-1) != 1:
        ti = ti.contiguous()
    s_ti_h = ti.stride(0) if ti.shape[0] > 1 else 0
    b = None
    s_b_h = s_b_n = 0
    if bias is not None:
        b = bias.unsqueeze(0) if bias.dim() == 2 else bias
        if b.dtype != torch.float32 or b.stride(-1) != 1:
            b = b.float().contiguous()
        s_b_h = b.stride(0) if b.shape[0] > 1 else 0
        s_b_n = b.stride(1)
    if out is None:
        out = torch.empty(N, H, D, device=q.device, dtype=q.dtype)
    lse_t = torch.empty(N, H, device=q.device, dtype=torch.float32) if lse else None
    bt = block_table.to(torch.int32).contiguous()
    cu = cu_seqlens_q.to(device=q.device, dtype=torch.int32).contiguous()
    pl = prefix_lens.to(device=q.device, dtype=torch.int32).contiguous()
    R, W = bt.shape
    d = L.DecodeDesc(N, H, Hkv, D, ti.shape[-1], block_size, local_blocks, float(sm_scale),
                     L.dtype_code(q), L.dtype_code(k_cache), L.dtype_code(out), q.stride(0), q.stride(1),
                     k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), out.stride(0), out.stride(1),
                     R, W, 0, 1, 1 if ti.dtype == torch.int64 else 0, s_ti_h, ti.stride(1), s_b_h, s_b_n, 0, 0)
    rc = L.lib().srswa_prefill_attend(C.byref(d), q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                      bt.data_ptr(), cu.data_ptr(), pl.data_ptr(), ti.data_ptr(), L.ptr(b),
                                      out.data_ptr(), L.ptr(lse_t), L.stream_of(q))
    L.check(rc, "srswa_prefill_attend")
    return (out, lse_t) if lse else out


def lse_merge_exchange(exchange, world, N, H, D, device, out_dtype=torch.float32, out=None, lse=None):
    """Log-sum-exp merge of the world ranks' partials that
    srswa_decode_attend_push stored as LL words into this rank's region of
    ``exchange`` (an LL srswa_peer): waits for them itself (bounded)."""
    if out is None:
        out = torch.empty(N, H, D, device=device, dtype=out_dtype)
    assert out.is_contiguous()
    if lse is None:
        lse = torch.empty(N, H, device=device, dtype=torch.float32)
    rc = L.lib().srswa_lse_merge(None, None, int(world), N, H, D, 0, 0, out.data_ptr(), L.dtype_code(out),
                                 lse.data_ptr(), C.byref(exchange), L.stream_of(out))
    L.check(rc, "srswa_lse_merge")
    return out, lse


def lse_merge(o_parts, lse_parts, out_dtype=torch.float32, out=None, lse=None, wait=None):
    """o_parts [C,N,H,D], lse_parts [C,N,H] fp32 (each part contiguous; the
    parts may be strided, e.g. views into one packed all-gather buffer) ->
    (out [N,H,D] out_dtype, lse [N,H])."""
    Cn, N, H, D = o_parts.shape
    copy_o = o_parts.dtype != torch.float32 or o_parts[0].stride() != (H * D, D, 1)
    copy_l = lse_parts.dtype != torch.float32 or lse_parts[0].stride() != (H, 1)
    if wait is not None and (copy_o or copy_l):
        # the parts arrive from peers during the kernel's own wait: no copy may read them earlier
        raise ValueError("lse_merge with wait: parts must be fp32 views with contiguous parts")
    if copy_o:
        o_parts = o_parts.float().contiguous()
    if copy_l:
        lse_parts = lse_parts.float().contiguous()
    if out is None:
        out = torch.empty(N, H, D, device=o_parts.device, dtype=out_dtype)
    assert out.is_contiguous()
    if lse is None:
        lse = torch.empty(N, H, device=o_parts.device, dtype=torch.float32)
    rc = L.lib().srswa_lse_merge(o_parts.data_ptr(), lse_parts.data_ptr(), Cn, N, H, D, o_parts.stride(0),
                                 lse_parts.stride(0), out.data_ptr(), L.dtype_code(out), lse.data_ptr(),
                                 None if wait is None else C.byref(wait), L.stream_of(o_parts))
    L.check(rc, "srswa_lse_merge")
    return out, lse


INV_SQRT = lambda d: 1.0 / math.sqrt(d)  # noqa: E731


# ------------------------------------------------------------------ PageGate
def _ids64(ids: torch.Tensor) -> torch.Tensor:
    if ids.dtype != torch.int64 or ids.stride(-1) != 1:
        ids = ids.to(torch.int64).contiguous()
    return ids


def page_ids(ids, img_id, page_id, key_length, per_page, page_scope_prefill):
    """ids [B, n] int -> (itm bool [B, key_length], ipi int64, qpi int64,
    flags int32 [2] on the device: any image token, any query page)."""
    ids = _ids64(ids)
    B, n = ids.shape
    dev = ids.device
    itm = torch.empty(B, key_length, device=dev, dtype=torch.bool)
    ipi = torch.empty(B, key_length, device=dev, dtype=torch.int64)
    qpi = torch.empty(B, key_length, device=dev, dtype=torch.int64)
    flags = torch.empty(2, device=dev, dtype=torch.int32)
    wsb = L.lib().srswa_page_scan_workspace_size(B, key_length)
    ws = torch.empty(max(wsb, 16), device=dev, dtype=torch.uint8)
    rc = L.lib().srswa_page_ids(ids.data_ptr(), ids.stride(0), B, n, key_length, int(img_id), int(page_id),
                                int(per_page), 1 if page_scope_prefill else 0, itm.data_ptr(), ipi.data_ptr(),
                                qpi.data_ptr(), flags.data_ptr(), ws.data_ptr(), wsb, L.stream_of(ids))
    L.check(rc, "srswa_page_ids")
    return itm, ipi, qpi, flags


def page_block_desc(nblk, block_size, ipi=None, itm=None):
    """Block descriptors [B, nblk, 4] int32 from page ids ipi [B, n] int64 or
    (flat) an image-token mask itm [B, n] bool."""
    src = ipi if ipi is not None else itm
    if (ipi is None) == (itm is None):
        raise ValueError("page_block_desc: pass exactly one of ipi / itm")
    if ipi is not None:
        src = ipi = _ids64(ipi)
    else:
        src = itm = (itm if itm.dtype == torch.bool else itm.bool()).contiguous()
    B, n = src.shape
    desc = torch.empty(B, nblk, 4, device=src.device, dtype=torch.int32)
    rc = L.lib().srswa_page_block_desc(L.ptr(ipi), None if itm is None else itm.view(torch.uint8).data_ptr(),
                                       src.stride(0), B, n, int(block_size), int(nblk), desc.data_ptr(),
                                       L.stream_of(src))
    L.check(rc, "srswa_page_block_desc")
    return desc


def page_cand_mask(desc, block_size, pos=None, qpi=None, ipi=None, flat=False, fallback=True, out=None, cq=None):
    """Candidate mask [B, cq, nblk] bool: block c of row b is a candidate for
    query i when it holds an image token of page qpi[b, clamp(pos[b, i])]
    (flat: any image token, cq rows); fallback: a query without one gets
    every block."""
    B, nblk, _ = desc.shape
    if flat:
        cq = int(cq) if cq is not None else (pos.shape[1] if pos is not None else 1)
        pos = qpi = ipi = None
        n_tok = n_q = 0
        s_ipi = s_qpi = s_pos = 0
    else:
        pos, qpi, ipi = _ids64(pos), _ids64(qpi), _ids64(ipi)
        cq, n_q, n_tok = pos.shape[1], qpi.shape[1], ipi.shape[1]
        s_ipi, s_qpi, s_pos = ipi.stride(0), qpi.stride(0), pos.stride(0)
    if out is None:
        out = torch.empty(B, cq, nblk, device=desc.device, dtype=torch.bool)
    assert out.is_contiguous() and out.shape == (B, cq, nblk)
    rc = L.lib().srswa_page_cand_mask(desc.data_ptr(), L.ptr(ipi), s_ipi, n_tok, int(block_size), B, nblk,
                                      L.ptr(qpi), s_qpi, n_q, L.ptr(pos), s_pos, cq, 1 if flat else 0,
                                      1 if fallback else 0, out.view(torch.uint8).data_ptr(), L.stream_of(desc))
    L.check(rc, "srswa_page_cand_mask")
    return out


def decode_allow_state(ids, img_id, page_id, per_page, block_size):
    """Prefill ids [B, L] -> dict(bmin, bmax [B, ceil(L/bs)] int64, pp, mcum [B] int64)."""
    ids = _ids64(ids)
    B, Lk = ids.shape
    dev = ids.device
    nblk = -(-Lk // int(block_size))
    st = dict(bmin=torch.empty(B, nblk, device=dev, dtype=torch.int64),
              bmax=torch.empty(B, nblk, device=dev, dtype=torch.int64),
              pp=torch.empty(B, device=dev, dtype=torch.int64), mcum=torch.empty(B, device=dev, dtype=torch.int64))
    wsb = L.lib().srswa_page_scan_workspace_size(B, Lk)
    ws = torch.empty(max(wsb, 16), device=dev, dtype=torch.uint8)
    rc = L.lib().srswa_decode_allow_state(ids.data_ptr(), ids.stride(0), B, Lk, int(img_id), int(page_id),
                                          int(per_page), int(block_size), st["bmin"].data_ptr(),
                                          st["bmax"].data_ptr(), st["pp"].data_ptr(), st["mcum"].data_ptr(),
                                          ws.data_ptr(), wsb, L.stream_of(ids))
    L.check(rc, "srswa_decode_allow_state")
    return st


def decode_allow(state, last_ids, page_id, nblk, out=None):
    """One decode token per request: advances state['mcum'] in place and
    returns allow [B, nblk] bool."""
    last_ids = _ids64(last_ids.reshape(last_ids.shape[0], -1))
    bmin, bmax = state["bmin"], state["bmax"]
    B = bmin.shape[0]
    if out is None:
        out = torch.empty(B, nblk, device=bmin.device, dtype=torch.bool)
    rc = L.lib().srswa_decode_allow(last_ids[:, -1:].data_ptr(), last_ids.stride(0), B, int(page_id),
                                    bmin.data_ptr(), bmax.data_ptr(), bmin.stride(0), bmin.shape[1],
                                    state["pp"].data_ptr(), state["mcum"].data_ptr(), int(nblk),
                                    out.view(torch.uint8).data_ptr(), L.stream_of(bmin))
    L.check(rc, "srswa_decode_allow")
    return out


# --------------------------------------------------------------- page2d RoPE
def rope2d_pos(ids, img_id, page_id, key_length, span=0):
    """ids [B, n] -> (tok, page [B, key_length] int64, pf_cnt [B, key_length + 1]
    int64, flags int32 [4] on the device: image seen, marker seen, rows
    without prompt pages, page count)."""
    ids = _ids64(ids)
    B, n = ids.shape
    dev = ids.device
    tok = torch.empty(B, key_length, device=dev, dtype=torch.int64)
    page = torch.empty(B, key_length, device=dev, dtype=torch.int64)
    pf = torch.empty(B, key_length + 1, device=dev, dtype=torch.int64)
    flags = torch.empty(4, device=dev, dtype=torch.int32)
    wsb = L.lib().srswa_rope2d_pos_workspace_size(B, key_length)
    ws = torch.empty(max(wsb, 16), device=dev, dtype=torch.uint8)
    rc = L.lib().srswa_rope2d_pos(ids.data_ptr(), ids.stride(0), B, n, key_length, int(img_id), int(page_id),
                                  int(span), tok.data_ptr(), page.data_ptr(), pf.data_ptr(), key_length + 1,
                                  flags.data_ptr(), ws.data_ptr(), wsb, L.stream_of(ids))
    L.check(rc, "srswa_rope2d_pos")
    return tok, page, pf, flags


def _rope_freqs(inv_tok, inv_page):
    it = inv_tok.float().contiguous()
    ip = inv_page.float().contiguous() if inv_page is not None and inv_page.numel() else None
    return it, ip, (0 if ip is None else ip.numel())


def rope2d_table(tok, page, inv_tok, inv_page, page_mod=0, dtype=torch.float32):
    """cos, sin [B, S, 2 * (n_tok + page_pairs)] of coordinates tok / page [B, S]."""
    tok, page = _ids64(tok), _ids64(page)
    assert tok.stride(0) == page.stride(0)
    B, S = tok.shape
    it, ip, pairs = _rope_freqs(inv_tok.to(tok.device), None if inv_page is None else inv_page.to(tok.device))
    dim = 2 * (it.numel() + pairs)
    cos = torch.empty(B, S, dim, device=tok.device, dtype=dtype)
    sin = torch.empty_like(cos)
    rc = L.lib().srswa_rope2d_table(tok.data_ptr(), page.data_ptr(), tok.stride(0), B, S, it.data_ptr(), it.numel(),
                                    L.ptr(ip), pairs, int(page_mod), cos.data_ptr(), sin.data_ptr(),
                                    L.dtype_code(cos), L.stream_of(tok))
    L.check(rc, "srswa_rope2d_table")
    return cos, sin


def rope2d_apply_(x, tok, page, inv_tok, inv_page, page_mod=0, table_dtype=None):
    """In place x <- x * cos + rotate_half(x) * sin on x [B, S, H, D] (any
    strides with D contiguous; a [B, H, S, D] tensor goes in as
    x.transpose(1, 2)); the tables are rounded to table_dtype (default:
    x's dtype, as the reference casts them)."""
    tok, page = _ids64(tok), _ids64(page)
    assert tok.stride(0) == page.stride(0) and x.stride(-1) == 1
    B, S, H, D = x.shape
    it, ip, pairs = _rope_freqs(inv_tok.to(x.device), None if inv_page is None else inv_page.to(x.device))
    td = L.dtype_code(x if table_dtype is None else torch.empty(0, dtype=table_dtype))
    rc = L.lib().srswa_rope2d_apply(x.data_ptr(), L.dtype_code(x), B, S, H, D, x.stride(0), x.stride(1), x.stride(2),
                                    tok.data_ptr(), page.data_ptr(), tok.stride(0), it.data_ptr(), it.numel(),
                                    L.ptr(ip), pairs, int(page_mod), td, L.stream_of(x))
    L.check(rc, "srswa_rope2d_apply")
    return x


def rope2d_decode_(new_ids, page_id, page, tok, pf_cnt, n_pg):
    """One new token per row: updates page [B] and tok [B] (int64) in place."""
    new_ids = _ids64(new_ids.reshape(new_ids.shape[0], -1))
    assert page.dtype == torch.int64 and tok.dtype == torch.int64 and pf_cnt.dtype == torch.int64
    rc = L.lib().srswa_rope2d_decode(new_ids[:, -1:].data_ptr(), new_ids.stride(0), page.shape[0], int(page_id),
                                     page.data_ptr(), tok.data_ptr(), pf_cnt.data_ptr(), pf_cnt.stride(0),
                                     int(n_pg), L.stream_of(page))
    L.check(rc, "srswa_rope2d_decode")
