"""The torch CPU baseline (oracle/torch_cpu.py, the reference's CPU PyTorch
path restated for timing) reproduces the reference's own outputs: the golden
fixtures of _infer_route_select, _decode_attend, the full decode step and
DashAttention._forward_dense (with its autograd gradients)."""

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import torch_cpu as TC

t = torch.from_numpy


def test_torch_entmax_golden():
    g = golden("entmax")
    np.testing.assert_allclose(TC.entmax15(t(g["x"])).numpy(), g["y"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("tag", ["hc0", "hc1"])
def test_torch_route_golden(tag):
    g = golden("route")
    BS, L, K, M = (int(x) for x in g["params"])
    idx_scale, floor, sigma = (float(x) for x in g["fparams"])
    hc = torch.zeros(128) if tag == "hc0" else t(g["hc1"])
    sc = TC.block_scores(t(g["idx_q"]), t(g["idx_k"]), hc, t(g["q_pos"]), BS, L)
    np.testing.assert_allclose(sc.numpy(), g[f"scores_{tag}"], rtol=1e-5, atol=1e-5)
    topi, bias, valid = TC.route_select(t(g[f"scores_{tag}"]), None, idx_scale, floor, sigma, K, M)
    assert (valid.numpy() == g[f"valid_{tag}"]).all()
    assert (np.where(g[f"valid_{tag}"], topi.numpy(), -1) == np.where(g[f"valid_{tag}"], g[f"topi_{tag}"], -1)).all()
    np.testing.assert_allclose(bias.numpy(), g[f"bias_{tag}"], rtol=1e-5, atol=1e-5)


def test_torch_decode_golden():
    g = golden("decode_attend")
    BS, L, K, M = (int(x) for x in g["params"])
    out = TC.decode_attend(t(g["q"]), t(g["k"]), t(g["v"]), t(g["topi"]), t(g["bias"]), t(g["valid"]),
                           t(g["q_pos"]), BS, L * BS, float(g["scale"]))
    np.testing.assert_allclose(out.numpy(), g["out"], rtol=1e-4, atol=1e-5)
    d = g["idx_k"].shape[-1]
    out2, topi, valid = TC.decode_step(t(g["q"]), t(g["k"]), t(g["v"]), t(g["idx_q"]), t(g["idx_k"]), torch.zeros(d),
                                       t(g["q_pos"]), BS, L, K, M, 128.0 / np.sqrt(d), 1e-4, 1.0, float(g["scale"]))
    assert (np.where(valid.numpy(), topi.numpy(), -1) == np.where(g["valid"], g["topi"], -1)).all()
    np.testing.assert_allclose(out2.numpy(), g["out"], rtol=1e-4, atol=1e-5)


def test_torch_forward_dense_golden():
    g = golden("forward_dense")
    BS, L = (int(x) for x in g["params"])
    q, k, v = (t(g[n]).requires_grad_(True) for n in ("q", "k", "v"))
    bias = t(g["bias"]).requires_grad_(True)
    o = TC.dense_forward(q, k, v, t(g["topi"]), bias, t(g["valid"]), BS, L * BS, float(g["scale"]), q_chunk=100)
    np.testing.assert_allclose(o.detach().numpy(), g["o"], rtol=1e-4, atol=2e-5)
    o.backward(t(g["do"]))
    for name, x in (("dq", q), ("dk", k), ("dv", v)):
        np.testing.assert_allclose(x.grad.numpy(), g[name], rtol=1e-3, atol=1e-4)
    np.testing.assert_allclose(np.where(g["valid"], bias.grad.numpy(), 0), np.where(g["valid"], g["dbias"], 0),
                               rtol=1e-3, atol=1e-4)
