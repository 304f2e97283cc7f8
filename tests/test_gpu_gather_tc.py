"""GPU parity of the tensor-core (tcgen05/TMEM) gather-attention forward and
backward: band pass + block-major remote pass over inverted selection lists.
Taken for bf16, head dim 128, 64-token blocks; compared with the CPU oracle
and, at larger sizes, with the CUDA-core kernels (selected here by asking for
an fp32 forward output, or fp16 inputs for the backward, which the
tensor-core path does not take).

Bar (north star): bf16 outputs within 2e-2 abs / 1e-2 rel."""

import ctypes as C
import math

import numpy as np
import pytest
import torch

from oracle import srswa_oracle as O

pytestmark = pytest.mark.gpu

from srswa import _lib as L  # noqa: E402
from srswa import ops  # noqa: E402

RTOL, ATOL = 1e-2, 2e-2


@pytest.fixture(autouse=True)
def check_call_status(monkeypatch):
    """Every gather call in these tests waits for itself and raises if a
    bounded wait of a tensor-core kernel expired (the call's status word)."""
    monkeypatch.setattr(ops, "_CHECK_STATUS", True)


def T(x, dev, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dt is None else t.to(dt)


def _inputs(rng, B, T_, H, Hkv, K, scale=0.5):
    D, BS = 128, 64
    q = O.bf16_round(rng.standard_normal((B, T_, H, D)).astype(np.float32) * scale)
    k = O.bf16_round(rng.standard_normal((B, T_, Hkv, D)).astype(np.float32) * scale)
    v = O.bf16_round(rng.standard_normal((B, T_, Hkv, D)).astype(np.float32) * scale)
    nblk = (T_ + BS - 1) // BS
    sel = np.full((B, 1, T_, K), -1, np.int64)
    for b in range(B):
        for t in range(T_):
            cands = np.arange(max(t // BS - 1, 0))
            if len(cands):
                pick = rng.choice(cands, size=min(K, len(cands)), replace=False)
                sel[b, 0, t, :len(pick)] = pick
    bias = (rng.standard_normal((B, T_, K)) * 0.7).astype(np.float32)
    return q, k, v, sel, bias, nblk


@pytest.mark.parametrize("B,T_,H,Hkv,K,LW,packed,use_bias", [
    (1, 256, 2, 2, 0, 128, False, False),      # band only
    (2, 700, 4, 4, 6, 256, False, True),       # T not a multiple of 128, bias
    (1, 1000, 4, 2, 8, 512, True, False),      # GQA + packed segments
    (1, 1536, 10, 10, 8, 512, False, True),    # BASELINE head layout
    (1, 2560, 10, 10, 16, 1024, False, True),  # cfg4 selection geometry: K = 16, LW = 1024
    (2, 1100, 4, 4, 16, 1024, True, True),     # K = 16, LW = 1024 with packing and T % 128 != 0
    (1, 1800, 4, 2, 20, 256, False, True),     # K = 20 slots, GQA, LW = 256
])
def test_tc_forward_vs_oracle(cuda, B, T_, H, Hkv, K, LW, packed, use_bias):
    rng = np.random.default_rng(T_ + K)
    Kk = max(K, 1)
    q, k, v, sel, bias, nblk = _inputs(rng, B, T_, H, Hkv, Kk)
    if K == 0:
        sel = sel[..., :0]
        bias = bias[..., :0]
    pos = np.tile(np.arange(T_), (B, 1))
    if packed:
        pos[0, 400:] = np.arange(T_ - 400)
    seg = (np.arange(T_)[None] - pos).astype(np.int64)
    scale = 1 / math.sqrt(128)
    sel_p = ops.pack_selection(T(sel, cuda), nblk)
    o, lse = ops.gather_fwd(T(q, cuda, torch.bfloat16), T(k, cuda, torch.bfloat16), T(v, cuda, torch.bfloat16),
                            sel_p, T(bias, cuda) if use_bias else None,
                            T(seg, cuda).to(torch.int32) if packed else None, 64, scale, LW)
    torch.cuda.synchronize()
    ref_o, ref_lse = O.gather_attention_fwd(q, k, v, sel, seg, 64, scale, LW, bias if use_bias else None)
    np.testing.assert_allclose(o.float().cpu().numpy(), ref_o, rtol=RTOL, atol=ATOL)
    fin = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse.cpu().numpy()[fin], ref_lse[fin], rtol=1e-3, atol=1e-3)


def test_tc_forward_vs_row_kernel_large(cuda):
    """cfg2-like shape (one batch element): tensor-core path vs the CUDA-core
    row kernel on identical inputs and selections from the CUDA router."""
    g = torch.Generator(device="cuda").manual_seed(1)
    B, T_, H, D, BS, LW, K = 1, 8192, 10, 128, 64, 512, 8
    q = (torch.randn(B, T_, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, T_, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, T_, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    iq = (torch.randn(B, T_, 128, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    from srswa import dash_infer
    router = type("R", (), dict(block_size=BS, local_blocks=LW // BS, local_window=LW,
                                head_cls=torch.zeros(128, device=cuda), stage0="head_cls"))()
    pos = torch.arange(T_, device=cuda)[None]
    topi, bias, valid = dash_infer.route(router, iq.float(), iq, pos, T_ // BS, None,
                                         dict(idx_scale=11.3, floor=1e-4, sigma=1.0, K=K, topm=16))
    sel = ops.pack_selection(torch.where(valid, topi, torch.full_like(topi, -1))[:, None], T_ // BS)
    b = (bias * valid).float()
    o_tc, lse_tc = ops.gather_fwd(q, k, v, sel, b, None, BS, 1 / math.sqrt(D), LW)
    # CUDA-core rows: same entry point with an fp32 output
    g_desc = ops._gather_desc(q, k, v, sel, BS, 1 / math.sqrt(D), LW)
    o_rows = torch.empty(B, T_, H, D, device=cuda, dtype=torch.float32)
    lse_rows = torch.empty(B, T_, H, device=cuda)
    rc = L.lib().srswa_gather_fwd(C.byref(g_desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), sel.data_ptr(),
                                  b.data_ptr(), None, o_rows.data_ptr(), L.F32, o_rows.stride(0), o_rows.stride(1),
                                  o_rows.stride(2), lse_rows.data_ptr(), None, 0,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    np.testing.assert_allclose(o_tc.float().cpu().numpy(), o_rows.cpu().numpy(), rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(lse_tc.cpu().numpy(), lse_rows.cpu().numpy(), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("layout", ["fused_qkv", "padded_heads"])
def test_tc_forward_strided_q(cuda, layout):
    """q as a view of a larger buffer (a fused q|k|v projection, or heads
    padded to D + 8) gives the contiguous-q result bit for bit: the remote
    pass gathers q rows through the caller's strides."""
    g = torch.Generator(device="cuda").manual_seed(7)
    B, T_, H, D, BS, LW, K = 2, 1536, 4, 128, 64, 256, 6
    q = (torch.randn(B, T_, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, T_, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, T_, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    rng = np.random.default_rng(3)
    _, _, _, sel, bias, nblk = _inputs(rng, B, T_, 1, 1, K)
    sel_p = ops.pack_selection(T(sel, cuda), nblk)
    bias_t = T(bias, cuda)
    if layout == "fused_qkv":
        buf = torch.cat([q, k, v], dim=2)           # [B, T, 3H, D]
        qs = buf[:, :, :H]
    else:
        buf = torch.zeros(B, T_, H, D + 8, device=cuda, dtype=torch.bfloat16)
        buf[..., :D] = q
        qs = buf[..., :D]
    o_ref, lse_ref = ops.gather_fwd(q, k, v, sel_p, bias_t, None, BS, 1 / math.sqrt(D), LW)
    o, lse = ops.gather_fwd(qs, k, v, sel_p, bias_t, None, BS, 1 / math.sqrt(D), LW)
    torch.cuda.synchronize()
    assert torch.equal(o, o_ref)
    assert torch.equal(lse, lse_ref)


def _route_case(cuda, seed, B, T_, H, Hkv, K, LW, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    D, BS = 128, 64
    q = (torch.randn(B, T_, H, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    k = (torch.randn(B, T_, Hkv, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    v = (torch.randn(B, T_, Hkv, D, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    do = torch.randn(B, T_, H, D, device=cuda, generator=g).to(torch.bfloat16)
    iq = (torch.randn(B, T_, 128, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    from srswa import dash_infer
    router = type("R", (), dict(block_size=BS, local_blocks=LW // BS, local_window=LW,
                                head_cls=torch.zeros(128, device=cuda), stage0="head_cls"))()
    pos = torch.arange(T_, device=cuda)[None].repeat(B, 1)
    nblk = (T_ + BS - 1) // BS
    topi, bias, valid = dash_infer.route(router, iq.float(), iq, pos, nblk, None,
                                         dict(idx_scale=11.3, floor=1e-4, sigma=1.0, K=K, topm=16))
    sel = ops.pack_selection(torch.where(valid, topi, torch.full_like(topi, -1))[:, None], nblk)
    b = (bias * valid).float().contiguous()
    return q, k, v, do, sel, b


@pytest.mark.parametrize("B,T_,H,Hkv,K,LW,packed,use_bias", [
    (1, 256, 2, 2, 0, 128, False, False),      # band only
    (2, 700, 4, 4, 6, 256, False, True),       # T not a multiple of 128, bias
    (1, 1000, 4, 2, 8, 512, True, False),      # GQA + packed segments
    (1, 1536, 10, 10, 8, 512, False, True),    # BASELINE head layout
    (1, 2560, 10, 10, 16, 1024, False, True),  # cfg4 selection geometry: K = 16, LW = 1024
    (2, 1100, 4, 4, 16, 1024, True, True),     # K = 16, LW = 1024 with packing and T % 128 != 0
])
def test_tc_backward_vs_oracle(cuda, B, T_, H, Hkv, K, LW, packed, use_bias):
    rng = np.random.default_rng(100 + T_ + K)
    Kk = max(K, 1)
    q, k, v, sel, bias, nblk = _inputs(rng, B, T_, H, Hkv, Kk)
    if K == 0:
        sel = sel[..., :0]
        bias = bias[..., :0]
    do = O.bf16_round(rng.standard_normal((B, T_, H, 128)).astype(np.float32))
    pos = np.tile(np.arange(T_), (B, 1))
    if packed:
        pos[0, 400:] = np.arange(T_ - 400)
    seg = (np.arange(T_)[None] - pos).astype(np.int64)
    scale = 1 / math.sqrt(128)
    sel_p = ops.pack_selection(T(sel, cuda), nblk)
    qd, kd, vd = (T(x, cuda, torch.bfloat16) for x in (q, k, v))
    bd = T(bias, cuda) if use_bias else None
    segd = T(seg, cuda).to(torch.int32) if packed else None
    o, lse = ops.gather_fwd(qd, kd, vd, sel_p, bd, segd, 64, scale, LW)
    dq, dk, dv, db = ops.gather_bwd(qd, kd, vd, o, lse, T(do, cuda, torch.bfloat16), sel_p, bd, segd, 64,
                                    scale, LW)
    torch.cuda.synchronize()
    rq, rk, rv, rb = O.gather_attention_bwd(q, k, v, do, sel, seg, 64, scale, LW, bias if use_bias else None)
    np.testing.assert_allclose(dq.float().cpu().numpy(), rq, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(dk.float().cpu().numpy(), rk, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(dv.float().cpu().numpy(), rv, rtol=RTOL, atol=ATOL)
    if use_bias:
        # d_bias sums dS over a block's 64 keys and all heads: absolute error
        # grows with that count, hence the wider absolute bound
        np.testing.assert_allclose(db.cpu().numpy(), rb, rtol=1e-2, atol=5e-2)


def test_tc_backward_vs_cuda_core_large(cuda):
    """Long-sequence shape: tensor-core backward (bf16) vs the CUDA-core
    backward run on the same values in fp16 (exact for these magnitudes)."""
    B, T_, H, Hkv, K, LW = 1, 8192, 10, 10, 8, 512
    q, k, v, do, sel, b = _route_case(cuda, 5, B, T_, H, Hkv, K, LW)
    scale = 1 / math.sqrt(128)
    o, lse = ops.gather_fwd(q, k, v, sel, b, None, 64, scale, LW)
    dq, dk, dv, db = ops.gather_bwd(q, k, v, o, lse, do, sel, b, None, 64, scale, LW)
    h = [x.to(torch.float16) for x in (q, k, v, o, do)]
    dq2, dk2, dv2, db2 = ops.gather_bwd(h[0], h[1], h[2], h[3], lse, h[4], sel, b, None, 64, scale, LW)
    torch.cuda.synchronize()
    for a, r in ((dq, dq2), (dk, dk2), (dv, dv2)):
        np.testing.assert_allclose(a.float().cpu().numpy(), r.float().cpu().numpy(), rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(db.cpu().numpy(), db2.cpu().numpy(), rtol=1e-2, atol=5e-2)


def test_tc_backward_deterministic(cuda):
    """Two calls give bit-identical gradients (fixed-order pair lists and
    partial sums; no floating-point atomics)."""
    q, k, v, do, sel, b = _route_case(cuda, 7, 2, 3000, 4, 2, 8, 512)
    scale = 1 / math.sqrt(128)
    o, lse = ops.gather_fwd(q, k, v, sel, b, None, 64, scale, 512)
    r1 = ops.gather_bwd(q, k, v, o, lse, do, sel, b, None, 64, scale, 512)
    r2 = ops.gather_bwd(q, k, v, o, lse, do, sel, b, None, 64, scale, 512)
    torch.cuda.synchronize()
    for a, c in zip(r1, r2):
        assert torch.isfinite(a).all()
        assert torch.equal(a, c)
