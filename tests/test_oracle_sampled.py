"""The sampled-row / sampled-block oracle (used by the full-size GPU parity
tests) equals the dense oracle, which the golden fixtures pin to the
reference: same rows of o / lse / dQ / d_bias and the same dK / dV of a key
block, with packing, repeats, -1 slots, GQA and a window wider than a block."""

import numpy as np
import pytest

from oracle import srswa_oracle as O


@pytest.mark.parametrize("T,HQ,Hkv,S,LW,packed", [(700, 4, 2, 6, 256, True), (900, 2, 2, 16, 512, False)])
def test_sampled_oracle_equals_dense(T, HQ, Hkv, S, LW, packed):
    rng = np.random.default_rng(T + S)
    D, BS = 32, 64
    q = rng.standard_normal((1, T, HQ, D)).astype(np.float32)
    k = rng.standard_normal((1, T, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((1, T, Hkv, D)).astype(np.float32)
    do = rng.standard_normal((1, T, HQ, D)).astype(np.float32)
    nblk = (T + BS - 1) // BS
    sel = O.dedup_rows(rng.integers(-1, nblk, (1, 1, T, S)))
    bias = rng.standard_normal((1, T, S)).astype(np.float32)
    pos = np.arange(T)[None].copy()
    if packed:
        pos[0, 300:] = np.arange(T - 300)
    seg = (np.arange(T)[None] - pos).astype(np.int64)
    scale = 0.17
    o, lse = O.gather_attention_fwd(q, k, v, sel, seg, BS, scale, LW, bias)
    dq, dk, dv, db = O.gather_attention_bwd(q, k, v, do, sel, seg, BS, scale, LW, bias)
    rows = np.array([0, 1, 63, 64, 299, 300, 301, T // 2, T - 2, T - 1])
    args = (q[0], k[0], v[0])
    o_r, lse_r = O.gather_rows_fwd(*args, sel[0, 0], seg[0], rows, BS, scale, LW, bias[0])
    np.testing.assert_allclose(o_r, o[0, rows], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lse_r, lse[0, rows], rtol=1e-5, atol=1e-5)
    dq_r, db_r = O.gather_rows_bwd(*args, do[0], sel[0, 0], seg[0], rows, BS, scale, LW, bias[0])
    np.testing.assert_allclose(dq_r, dq[0, rows], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(db_r, db[0, rows], rtol=1e-4, atol=1e-5)
    for c in (0, 3, nblk - 1):
        dk_c, dv_c = O.gather_block_bwd(*args, do[0], o[0], lse[0], sel[0, 0], seg[0], c, BS, scale, LW, bias[0])
        np.testing.assert_allclose(dk_c, dk[0, c * BS:(c + 1) * BS], rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(dv_c, dv[0, c * BS:(c + 1) * BS], rtol=1e-4, atol=1e-5)
