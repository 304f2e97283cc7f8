"""Host-side contract of the Python boundary (no GPU needed): the same
None-return cases as the reference wrappers, effective K/M, loud failure on
CPU tensors (no CPU fallback)."""

import pytest
import torch

from srswa import _lib as L
from srswa import ops
from srswa.sparse_gather import SPARSE_BLOCK_SIZE_SENTINEL, triton_gather_attention
from srswa.sparse_gather_e2e import SPARSE_E2E_SENTINEL, triton_gather_attention_e2e


def _qkv(B=1, H=2, T=64, D=64):
    q = torch.zeros(B, H, T, D, dtype=torch.bfloat16)
    return q, q.clone(), q.clone()


def test_sentinels():
    assert SPARSE_BLOCK_SIZE_SENTINEL == 128 and SPARSE_E2E_SENTINEL == 1


def test_gather_returns_none_like_reference():
    q, k, v = _qkv()
    sel = torch.zeros(1, 1, 64, 2, dtype=torch.int32)
    pos = torch.arange(64)[None]
    # sparse_gather_triton.py:400-412
    assert triton_gather_attention(q, k, v, sel, pos, torch.zeros(1), 32, 0.1) is None
    assert triton_gather_attention(q, k, v, torch.zeros(1, 3, 64, 2, dtype=torch.int32), pos, None, 32, 0.1) is None
    assert triton_gather_attention(q, k[:, :, :32], v[:, :, :32], sel, pos, None, 32, 0.1) is None
    assert triton_gather_attention(q, k, v, sel, None, None, 32, 0.1) is None
    assert triton_gather_attention(q, k, v, sel, pos[0], None, 32, 0.1) is None


def test_gather_e2e_returns_none_like_reference():
    q, k, v = _qkv()
    sel = torch.zeros(1, 1, 64, 2, dtype=torch.int32)
    b = torch.zeros(1, 64, 2)
    pos = torch.arange(64)[None]
    # sparse_gather_e2e_triton.py:370-381
    assert triton_gather_attention_e2e(q, k, v, sel, b, pos, torch.zeros(1), 32, 0.1) is None
    assert triton_gather_attention_e2e(q, k, v, torch.zeros(1, 2, 64, 2), b, pos, None, 32, 0.1) is None
    assert triton_gather_attention_e2e(q, k[:, :, :32], v[:, :, :32], sel, b, pos, None, 32, 0.1) is None
    packed = pos.clone()
    packed[0, 40:] = torch.arange(24)
    assert triton_gather_attention_e2e(q, k, v, sel, b, packed, None, 32, 0.1) is None


def test_unsupported_head_dim_raises():
    q, k, v = _qkv(D=96)
    sel = torch.zeros(1, 1, 64, 2, dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        triton_gather_attention(q, k, v, sel, torch.arange(64)[None], None, 32, 0.1)


def test_cpu_tensors_fail_loudly():
    x = torch.zeros(4, 128)
    with pytest.raises(L.SrswaError):
        ops.route_select(x, None, topk=2, topm=4, idx_scale=1.0, floor=1e-4, sigma=1.0)


@pytest.mark.parametrize("topk,topm,nblk,K,M", [(8, 16, 100, 8, 16), (8, 16, 5, 5, 5), (12, 4, 50, 4, 4),
                                                 (0, 16, 50, 1, 16), (3, 0, 20, 3, 20)])
def test_effective_km(topk, topm, nblk, K, M):
    # _infer_route_select: M = max(1, min(topm, nblk)) if topm > 0 else nblk; K = max(1, min(K, M))
    assert ops.effective_km(topk, topm, nblk) == (K, M)


def test_arange_check_follows_tensor_and_version():
    """The packing test of triton_gather_attention_e2e is kept per position_ids
    tensor object and re-run after an in-place change or for a new tensor."""
    import torch
    from srswa.sparse_gather_e2e import _positions_are_arange
    p = torch.arange(10)[None].repeat(2, 1)
    assert _positions_are_arange(p, 10)
    assert _positions_are_arange(p, 10)          # same object, same version
    p[1, 3] = 0                                  # in place: the version counter moves
    assert not _positions_are_arange(p, 10)
    v = p[1:]                                    # a view shares the version counter
    assert not _positions_are_arange(v, 10)
    p[1, 3] = 3
    assert _positions_are_arange(p, 10)
    q = torch.arange(10)[None].repeat(2, 1) * 2  # another tensor
    assert not _positions_are_arange(q, 10)


def test_install_sglang_reaches_the_backend(monkeypatch):
    """The SGLang backend imports the ops by `from ... import` at its own
    import (whl:.../unlimited_ocr_v2_backend.py:18-52); after install_sglang
    both the ops modules and the backend's copies are srswa.paged's."""
    import sys
    import types

    from srswa import dropin, paged
    pre = "sglang.srt.layers.attention.unlimited_dash_ops"
    ref = lambda *a, **k: "reference"  # noqa: E731
    at = types.ModuleType(pre + ".attend_triton")
    rt = types.ModuleType(pre + ".route_triton")
    for m, names in ((at, ("dash_sparse_attn", "dash_sparse_attn_decode")),
                     (rt, ("route_decode_triton", "route_prefill_triton", "kbar_refresh_tail_triton",
                           "win_bounds_decode", "kbar_tail_plan"))):
        for n in names:
            setattr(m, n, ref)
    be = types.ModuleType("sglang.srt.layers.attention.unlimited_ocr_v2_backend")
    for n in ("dash_sparse_attn", "dash_sparse_attn_decode", "route_decode_triton", "route_prefill_triton",
              "kbar_refresh_tail_triton", "win_bounds_decode", "kbar_tail_plan"):
        setattr(be, n, ref)        # the backend's own `from ... import` copies
    for m in (at, rt, be):
        monkeypatch.setitem(sys.modules, m.__name__, m)
    done = dropin.install_sglang()
    for n in ("dash_sparse_attn", "dash_sparse_attn_decode", "route_decode_triton", "route_prefill_triton",
              "kbar_refresh_tail_triton", "win_bounds_decode"):
        # the backend issues its decode attend right after its router: the overlapping variant
        want = paged.dash_sparse_attn_decode_after_router if n == "dash_sparse_attn_decode" else getattr(paged, n)
        assert getattr(be, n) is want, n
        mod = at if hasattr(at, n) else rt
        assert getattr(mod, n) is getattr(paged, n), n
    assert be.kbar_tail_plan is ref          # torch-only planning helpers stay the reference's
    assert len(done) == 12
    dropin.install_sglang(overlap_router=False)
    assert be.dash_sparse_attn_decode is paged.dash_sparse_attn_decode


def _no_capture(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: False)


def test_paged_prefill_dispatch_per_request(monkeypatch):
    """dash_sparse_attn: requests of >= TC_MIN_ROWS rows go to the
    tensor-core forward over the paged caches (one call each, their prefix
    as the query offset), shorter ones to the row kernel one by one; a
    request whose block table is too narrow, or a selection that differs per
    head, keeps the row kernel."""
    from srswa import paged
    _no_capture(monkeypatch)
    calls = []
    monkeypatch.setattr(ops, "pack_selection", lambda sel, nblk: sel.to(torch.int32))
    monkeypatch.setattr(ops, "gather_fwd_paged",
                        lambda q, kc, vc, sel, bias, pages, qoff, bs, sc, lw, out:
                        calls.append(("tc", q.shape[0], qoff, pages.shape[0], lw, out.shape[0])))
    monkeypatch.setattr(ops, "prefill_attend",
                        lambda q, kc, vc, ti, b, **kw:
                        calls.append(("row", q.shape[0], kw["prefix_lens"].tolist(), kw["block_table"].shape[0])))
    H, D, K = 2, 128, 4
    qlen, ctx = [200, 50, 130], [0, 100, 5000]
    N = sum(qlen)
    cu = torch.tensor([0, 200, 250, 380], dtype=torch.int32)
    pre = torch.tensor(ctx, dtype=torch.int32)
    q = torch.zeros(N, H, D, dtype=torch.bfloat16)
    kc = torch.zeros(4, 64, H, D, dtype=torch.bfloat16)
    ti = torch.zeros(N, K, dtype=torch.int32).unsqueeze(0).expand(H, -1, -1)
    tb = torch.zeros(N, K).unsqueeze(0).expand(H, -1, -1)
    out = torch.zeros(N, H, D, dtype=torch.bfloat16)

    def run(bt, ti_, tb_):
        calls.clear()
        paged.dash_sparse_attn(q, kc, kc.clone(), ti_, tb_, bt, cu, cu, pre, 200, H, 0.1, out,
                               local_blocks=8, sparse_block_size=64)
        return sorted(calls)

    bt = torch.zeros(3, 90, dtype=torch.int32)           # covers ceil((5000 + 130) / 64) = 81 blocks
    assert run(bt, ti, tb) == sorted([("tc", 200, 0, 90, 512, 200), ("tc", 130, 5000, 90, 512, 130),
                                      ("row", 50, [100], 1)])
    bt = torch.zeros(3, 60, dtype=torch.int32)           # too narrow for the 5130-token request
    assert run(bt, ti, tb) == sorted([("tc", 200, 0, 60, 512, 200), ("row", 130, [5000], 1),
                                      ("row", 50, [100], 1)])
    per_head = torch.zeros(H, N, K, dtype=torch.int32)   # a selection per KV head: all on the row kernel
    assert run(bt, per_head, tb) == [("row", N, ctx, 3)]


def test_route_prefill_dispatch_per_request(monkeypatch):
    """route_prefill_triton: each request of >= ROUTE_TILE_MIN_ROWS rows is
    routed by a call of its own (one sequence, the tiled routers), the other
    rows by one varlen call on their gathered rows, whose results land in the
    caller's rows."""
    from srswa import paged
    _no_capture(monkeypatch)
    calls = []

    masks = []

    def fake_route(idx_q, kbar, **kw):
        n = idx_q.shape[0]
        calls.append((n, kw.get("rows_per_seq"), kw.get("row_seq") is not None))
        if kw.get("cand") is not None:
            masks.append(tuple(kw["cand"].shape))
        if kw.get("out") is not None:
            kw["out"]["topi32"].fill_(7)
            kw["out"]["bias"].fill_(0.5)
            return kw["out"]
        return {"topi32": torch.full((n, 4), 3, dtype=torch.int32), "bias": torch.full((n, 4), 0.25)}

    monkeypatch.setattr(ops, "route", fake_route)
    qlen = [100, 30, 100]
    N = sum(qlen)
    cu = torch.tensor([0, 100, 130, 230], dtype=torch.int32)
    row2req = torch.repeat_interleave(torch.arange(3, dtype=torch.int32), torch.tensor(qlen))
    out_idx = torch.zeros(N, 4, dtype=torch.int32)
    out_bias = torch.zeros(N, 4)
    paged.route_prefill_triton(idx_q=torch.zeros(N, 128), k_bar=torch.zeros(200, 128),
                               block_table=torch.zeros(3, 50, dtype=torch.int32),
                               seq_lens=torch.tensor([100, 130, 300], dtype=torch.int32), cu_seqlens_q=cu,
                               context_lens=torch.tensor([0, 100, 200], dtype=torch.int32), row2req=row2req,
                               image_allow=None, out_idx=out_idx, out_bias=out_bias, max_block=50, block_size=64,
                               local_blocks=8, idx_scale=11.3, prior_floor=1e-4, sigma=1.0, topm=16, budget=4)
    assert sorted(calls, key=str) == sorted([(100, 100, False), (100, 100, False), (30, None, True)], key=str)
    assert (out_idx[:100] == 7).all() and (out_idx[130:] == 7).all() and (out_idx[100:130] == 3).all()
    assert (out_bias[100:130] == 0.25).all() and (out_bias[:100] == 0.5).all()
    # image_allow: a per-row mask follows its rows, a shared row is passed as is
    for allow, want in ((torch.ones(N, 60, dtype=torch.bool), [(100, 60), (100, 60), (30, 60)]),
                        (torch.ones(60, dtype=torch.bool), [(60,)] * 3)):
        masks.clear()
        paged.route_prefill_triton(idx_q=torch.zeros(N, 128), k_bar=torch.zeros(200, 128),
                                   block_table=torch.zeros(3, 50, dtype=torch.int32),
                                   seq_lens=torch.tensor([100, 130, 300], dtype=torch.int32), cu_seqlens_q=cu,
                                   context_lens=torch.tensor([0, 100, 200], dtype=torch.int32), row2req=row2req,
                                   image_allow=allow, out_idx=out_idx, out_bias=out_bias, max_block=50,
                                   block_size=64, local_blocks=8, idx_scale=11.3, prior_floor=1e-4, sigma=1.0,
                                   topm=16, budget=4)
        assert sorted(masks) == sorted(want)
