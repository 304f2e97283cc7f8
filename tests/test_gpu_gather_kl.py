"""GPU parity of the DSA gather-KL distillation (srswa_gather_kl_fwd / _bwd,
through srswa.dsa.gather_kl): per-row KL and validity, and the gradients to
the index q / k, against the reference's own outputs
(tests/golden/gather_kl.npz, _kl_chunk_core in bf16 with autograd; a packed
batch included) and against the oracle at the BASELINE head layout (H = 10,
D = d = 128, 64-token blocks, 16 blocks per row, window 1024) with repeated
and empty selections.  The backward is deterministic (two runs equal bit
for bit).

Bars: kl within 1e-3 rel / 1e-4 abs of the reference (fp32 softmaxes of the
same bf16 logits); gradients within the bf16 bar 2e-2 abs / 1e-2 rel."""

import math

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import srswa_oracle as O

pytestmark = pytest.mark.gpu

from srswa import dsa  # noqa: E402


def T(x, dev, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dt is None else t.to(dt)


def _run(cuda, iq, ik, qm, km, sel, pos, seg, BS, LW, scaling, gout):
    qi = T(iq, cuda, torch.bfloat16).requires_grad_(True)
    ki = T(ik, cuda, torch.bfloat16).requires_grad_(True)
    kl, valid = dsa.gather_kl(qi, ki, T(qm, cuda, torch.bfloat16), T(km, cuda, torch.bfloat16), T(sel, cuda),
                              T(pos, cuda), None if seg is None else T(seg, cuda), block_size=BS, local_window=LW,
                              scaling=scaling)
    kl.backward(T(gout, cuda))
    torch.cuda.synchronize()
    return kl.detach().cpu().numpy(), valid.cpu().numpy(), qi.grad.float().cpu().numpy(), \
        ki.grad.float().cpu().numpy()


def test_gather_kl_golden(cuda):
    g = golden("gather_kl")
    BS, LW = (int(x) for x in g["params"])
    kl, valid, dq, dk = _run(cuda, g["idx_q"], g["idx_k"], g["q_main"], g["k_main"], g["sel"], g["pos"], g["seg"],
                             BS, LW, float(g["scaling"]), g["gout"])
    np.testing.assert_allclose(kl, g["kl"], rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(dq, g["d_idx_q"], rtol=1e-2, atol=2e-2)
    np.testing.assert_allclose(dk, g["d_idx_k"], rtol=1e-2, atol=2e-2)


def test_gather_kl_baseline_heads_vs_oracle(cuda):
    rng = np.random.default_rng(41)
    B, Cq, H, Hkv, D, d, BS, LW, S = 1, 1500, 10, 10, 128, 128, 64, 1024, 16
    iq = O.bf16_round((rng.standard_normal((B, Cq, d)) * 0.08).astype(np.float32))
    ik = O.bf16_round(rng.standard_normal((B, Cq, d)).astype(np.float32))
    qm = O.bf16_round(rng.standard_normal((B, Cq, H, D)).astype(np.float32))
    km = O.bf16_round(rng.standard_normal((B, Cq, Hkv, D)).astype(np.float32))
    nblk = (Cq + BS - 1) // BS
    sel = np.full((B, Cq, S), -1, np.int32)
    for c in range(Cq):
        cands = np.arange(max(c // BS - 1, 0))
        if len(cands):
            pick = rng.choice(cands, size=min(S, len(cands)), replace=False)
            sel[0, c, :len(pick)] = pick
    sel[0, 1400, 3] = sel[0, 1400, 1]            # repeat
    sel[0, 1300, :] = -1                          # no selection
    pos = np.arange(Cq)[None].astype(np.int64)
    gout = rng.standard_normal((B, Cq)).astype(np.float32)
    scaling = 1 / math.sqrt(D)
    kl, valid, dq, dk = _run(cuda, iq, ik, qm, km, sel, pos, None, BS, LW, scaling, gout)
    rk, rv, rdq, rdk = O.gather_kl(iq, ik, qm, km, sel, pos, None, BS, LW, scaling, bf16_logits=True, g=gout)
    assert (valid == rv).all() and not valid[0, 1300]
    np.testing.assert_allclose(kl, rk, rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(dq, rdq, rtol=1e-2, atol=2e-2)
    np.testing.assert_allclose(dk, rdk, rtol=1e-2, atol=2e-2)
    # deterministic backward
    _, _, dq2, dk2 = _run(cuda, iq, ik, qm, km, sel, pos, None, BS, LW, scaling, gout)
    assert np.array_equal(dq, dq2) and np.array_equal(dk, dk2)


def test_gather_kl_saved_teacher_equals_recompute(cuda):
    """The backward that reads the forward's saved teacher probabilities
    (srswa_gather_kl_fwd_save / _bwd_saved) gives the recomputing backward's
    gradients bit for bit."""
    rng = np.random.default_rng(43)
    B, Cq, H, Hkv, D, d, BS, LW, S = 1, 1200, 10, 10, 128, 128, 64, 512, 8
    iq = (rng.standard_normal((B, Cq, d)) * 0.08).astype(np.float32)
    ik = rng.standard_normal((B, Cq, d)).astype(np.float32)
    qm = rng.standard_normal((B, Cq, H, D)).astype(np.float32)
    km = rng.standard_normal((B, Cq, Hkv, D)).astype(np.float32)
    pos = np.arange(Cq)[None]
    nrem = np.maximum(pos - LW + 1, 0) // BS
    sel = np.where(np.arange(S) < nrem[..., None], (rng.random((B, Cq, S)) * nrem[..., None]).astype(np.int64), -1)
    gout = rng.standard_normal((B, Cq)).astype(np.float32)
    res = []
    for save in (True, False):
        qi = T(iq, cuda, torch.bfloat16).requires_grad_(True)
        ki = T(ik, cuda, torch.bfloat16).requires_grad_(True)
        kl, _ = dsa.gather_kl(qi, ki, T(qm, cuda, torch.bfloat16), T(km, cuda, torch.bfloat16), T(sel, cuda),
                              T(pos, cuda), block_size=BS, local_window=LW, scaling=1 / math.sqrt(D),
                              save_teacher=save)
        kl.backward(T(gout, cuda))
        torch.cuda.synchronize()
        res.append((kl.detach(), qi.grad, ki.grad))
    for a, b in zip(*res):
        assert torch.equal(a, b)
