"""GPU parity of the fused gather-attention forward/backward (a6/a7), the
selection packing (a5) and the DASH window/reference merge (a8), against the
reference's golden vectors (Triton kernels K1-K7 under the interpreter and
DashAttention._forward_dense autograd) and the CPU oracle.

Bar (north star): bf16 outputs and gradients within 2e-2 abs / 1e-2 rel of
the fp32 reference on the same (bf16-representable) inputs."""

import math

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import srswa_oracle as O

pytestmark = pytest.mark.gpu

from srswa import dash_infer, ops  # noqa: E402
from srswa.sparse_gather import triton_gather_attention  # noqa: E402
from srswa.sparse_gather_e2e import triton_gather_attention_e2e  # noqa: E402

RTOL, ATOL = 1e-2, 2e-2


def T(x, dev, dt=None):
    t = torch.from_numpy(np.ascontiguousarray(x)).to(dev)
    return t if dt is None else t.to(dt)


def leaf(x, dev):
    return T(x, dev, torch.bfloat16).requires_grad_(True)


def close(a, b, rtol=RTOL, atol=ATOL):
    np.testing.assert_allclose(a.detach().float().cpu().numpy(), b, rtol=rtol, atol=atol)


def test_pack_selection(cuda):
    sel = np.array([[3, 3, -1, 5, 9, 5, 0], [1, 2, 3, 4, 5, 6, 7]], np.int64)
    out = ops.pack_selection(T(sel, cuda), nblk=7).cpu().numpy()
    np.testing.assert_array_equal(out, [[3, -1, -1, 5, -1, -1, 0], [1, 2, 3, 4, 5, 6, -1]])


def test_gather_golden_fwd_bwd(cuda):
    g = golden("gather_triton")
    BS, LW = (int(x) for x in g["params"])
    q, k, v = leaf(g["q"], cuda), leaf(g["k"], cuda), leaf(g["v"], cuda)
    o = triton_gather_attention(q, k, v, T(g["sel"], cuda), T(g["pos"], cuda), None, BS, float(g["scale"]), LW)
    close(o, g["o"])
    o.backward(T(g["do"], cuda, torch.bfloat16))
    close(q.grad, g["dq"])
    close(k.grad, g["dk"])
    close(v.grad, g["dv"])


def test_gather_e2e_golden_fwd_bwd(cuda):
    g = golden("gather_e2e")
    BS, LW = (int(x) for x in g["params"])
    q, k, v = leaf(g["q"], cuda), leaf(g["k"], cuda), leaf(g["v"], cuda)
    b = T(g["bias"], cuda).requires_grad_(True)
    T_ = g["q"].shape[2]
    pos = torch.arange(T_, device=cuda)[None].repeat(g["q"].shape[0], 1)
    o = triton_gather_attention_e2e(q, k, v, T(g["sel"], cuda), b, pos, None, BS, float(g["scale"]), LW)
    close(o, g["o"])
    o.backward(T(g["do"], cuda, torch.bfloat16))
    close(q.grad, g["dq"])
    close(k.grad, g["dk"])
    close(v.grad, g["dv"])
    close(b.grad, g["dbias"], rtol=1e-2, atol=5e-2)


def test_forward_dense_golden(cuda):
    """DASH merge semantics (dash_attention.py:1230-1260) through the fused
    e2e entry: selected blocks overlapping the window, invalid slots."""
    g = golden("forward_dense")
    BS, L = (int(x) for x in g["params"])
    valid = g["valid"]
    sel = np.where(valid, g["topi"], -1)[:, None]
    bias = np.where(valid, g["bias"], 0).astype(np.float32)
    q, k, v = leaf(g["q"], cuda), leaf(g["k"], cuda), leaf(g["v"], cuda)
    b = T(bias, cuda).requires_grad_(True)
    B, H, S, D = g["q"].shape
    pos = torch.arange(S, device=cuda)[None].repeat(B, 1)
    o = triton_gather_attention_e2e(q, k, v, T(sel, cuda), b, pos, None, BS, float(g["scale"]), L * BS)
    close(o, g["o"])
    o.backward(T(g["do"], cuda, torch.bfloat16))
    close(q.grad, g["dq"])
    close(k.grad, g["dk"])
    close(v.grad, g["dv"])
    close(b.grad * T(valid, cuda), np.where(valid, g["dbias"], 0), rtol=1e-2, atol=5e-2)


@pytest.mark.parametrize("B,T_,H,Hkv,D,BS,LW,K,packed", [(2, 1536, 4, 4, 128, 64, 512, 8, False),
                                                          (1, 2560, 10, 10, 128, 64, 1024, 16, False),  # cfg4
                                                          (1, 1000, 4, 2, 128, 64, 200, 6, True),
                                                          (2, 700, 2, 2, 64, 32, 96, 4, False)])
def test_gather_vs_oracle_router_selection(cuda, B, T_, H, Hkv, D, BS, LW, K, packed):
    """End-to-end: selections from the CUDA router, attention fwd + bwd vs the
    oracle on the same bf16 values (T not a multiple of BS, GQA, packing)."""
    rng = np.random.default_rng(T_)
    q = O.bf16_round(rng.standard_normal((B, T_, H, D)).astype(np.float32) * 0.5)
    k = O.bf16_round(rng.standard_normal((B, T_, Hkv, D)).astype(np.float32) * 0.5)
    v = O.bf16_round(rng.standard_normal((B, T_, Hkv, D)).astype(np.float32) * 0.5)
    do = O.bf16_round(rng.standard_normal((B, T_, H, D)).astype(np.float32))
    idx = O.bf16_round(rng.standard_normal((B, T_, 128)).astype(np.float32))
    nblk = (T_ + BS - 1) // BS
    L = LW // BS
    router = type("R", (), dict(block_size=BS, local_blocks=L, local_window=LW,
                                head_cls=torch.zeros(128, device=cuda), stage0="head_cls"))()
    pos = np.tile(np.arange(T_), (B, 1))
    if packed:
        pos[0, 600:] = np.arange(T_ - 600)
    p = dict(idx_scale=128 / math.sqrt(128), floor=1e-4, sigma=1.0, K=K, topm=16)
    topi, bias_t, valid = dash_infer.route(router, T(idx, cuda), T(idx, cuda, torch.bfloat16),
                                           T(np.tile(np.arange(T_), (B, 1)), cuda), nblk, None, p)
    sel = torch.where(valid, topi, torch.full_like(topi, -1))[:, None]
    qg, kg, vg = (leaf(np.swapaxes(x, 1, 2), cuda) for x in (q, k, v))
    if packed:
        o = triton_gather_attention(qg, kg, vg, sel, T(pos, cuda), None, BS, 1 / math.sqrt(D), LW)
        bias = None
    else:
        bias = (bias_t * valid).float().requires_grad_(True)
        o = triton_gather_attention_e2e(qg, kg, vg, sel, bias, T(pos, cuda), None, BS, 1 / math.sqrt(D), LW)
    o.backward(T(np.swapaxes(do, 1, 2), cuda, torch.bfloat16))
    seg = (np.arange(T_)[None] - pos).astype(np.int64)
    sel_np = sel.cpu().numpy()
    bias_np = None if bias is None else bias.detach().cpu().numpy()
    ref_o, _ = O.gather_attention_fwd(q, k, v, sel_np, seg, BS, 1 / math.sqrt(D), LW, bias_np)
    dq, dk, dv, db = O.gather_attention_bwd(q, k, v, do, sel_np, seg, BS, 1 / math.sqrt(D), LW, bias_np)
    close(o.transpose(1, 2), ref_o)
    close(qg.grad.transpose(1, 2), dq)
    close(kg.grad.transpose(1, 2), dk)
    close(vg.grad.transpose(1, 2), dv)
    if bias is not None:
        close(bias.grad, db, rtol=1e-2, atol=5e-2)


def test_gather_backward_deterministic(cuda):
    rng = np.random.default_rng(9)
    B, T_, H, D, BS, LW, K = 1, 900, 2, 128, 64, 256, 4
    q, k, v = (T(O.bf16_round(rng.standard_normal((B, H, T_, D)).astype(np.float32)), cuda, torch.bfloat16)
               for _ in range(3))
    nblk = (T_ + BS - 1) // BS
    sel = torch.randint(-1, nblk, (B, 1, T_, K), device=cuda)
    bias = torch.randn(B, T_, K, device=cuda)
    pos = torch.arange(T_, device=cuda)[None]
    do = torch.randn(B, H, T_, D, device=cuda, dtype=torch.bfloat16)
    grads = []
    for _ in range(2):
        qq, kk, vv, bb = (x.clone().requires_grad_(True) for x in (q, k, v, bias))
        o = triton_gather_attention_e2e(qq, kk, vv, sel, bb, pos, None, BS, 0.09, LW)
        o.backward(do)
        grads.append([x.grad.clone() for x in (qq, kk, vv, bb)])
    for a, b in zip(*grads):
        assert torch.equal(a, b)
