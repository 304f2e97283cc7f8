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
