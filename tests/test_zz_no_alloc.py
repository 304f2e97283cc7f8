"""The gather-attention backward entry point that allocates nothing.

srswa_gather_bwd_noalloc serves callers that cannot allocate device memory
(a runtime that pre-reserves all device memory, a plugin/FFI host that hands
over only input and output buffers): its scratch is an array inside the
library instead of a caller workspace.  This test calls it through the C ABI
twice in a row and checks each result against the workspace entry point
srswa_gather_bwd on the same inputs (the second call also checks that the
shared scratch left by the first call does not leak into the result).  Both
entry points run the same deterministic kernels, so the results must be equal
bit for bit.  Before the compared calls, a backward of another shape fills
the shared array with unrelated data.  It runs last (file name) so a failure
here cannot hide the other tests, and it passes both alone in a fresh process
and after the rest of the suite."""

import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu

from srswa import _lib as L  # noqa: E402
from srswa import ops  # noqa: E402


def _case(dev, seed, T=900, B=2, H=4, Hkv=2, D=128, BS=64, LW=256, S=6):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B, T, Hkv, D, generator=g).to(torch.bfloat16).to(dev)
    do = torch.randn(B, T, H, D, generator=g).to(torch.bfloat16).to(dev)
    nblk = (T + BS - 1) // BS
    sel = ops.pack_selection(torch.randint(-1, nblk, (B, 1, T, S), generator=g).to(dev), nblk)
    bias = torch.randn(B, T, S, generator=g).to(dev)
    o, lse = ops.gather_fwd(q, k, v, sel, bias, None, BS, 0.088, LW)
    desc = ops._gather_desc(q, k, v, sel, BS, 0.088, LW)
    return q, k, v, o, lse, do, sel, bias, desc


def _call(lib, name, desc, q, k, v, o, lse, do, sel, bias, ws=None):
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    db = torch.empty(bias.shape, device=q.device, dtype=torch.float32)
    stream = torch.cuda.current_stream().cuda_stream
    args = [C.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), o.stride(0), o.stride(1),
            o.stride(2), do.data_ptr(), lse.data_ptr(), sel.data_ptr(), bias.data_ptr(), None,
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), db.data_ptr()]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    rc = getattr(lib, name)(*args, stream)
    assert rc == 0, (name, rc, L.status_text(rc))
    torch.cuda.synchronize()
    return dq, dk, dv, db


def _noalloc_status(lib):
    v = C.c_int(-1)
    assert lib.srswa_gather_bwd_noalloc_status(C.byref(v), torch.cuda.current_stream().cuda_stream) == 0
    return v.value


def test_noalloc_backward_matches_workspace_backward(cuda):
    lib = L.lib()
    assert lib.srswa_gather_bwd_noalloc_max_scratch() == 32 << 20
    # a different shape first, so the shared array holds stale, unrelated data
    junk = _case(cuda, 9, T=1300, B=1, H=2, Hkv=2, S=8)
    _call(lib, "srswa_gather_bwd_noalloc", junk[-1], *junk[:-1])
    for seed in (1, 2):  # two calls in a row, different inputs
        q, k, v, o, lse, do, sel, bias, desc = _case(cuda, seed)
        ws_n = lib.srswa_gather_bwd_workspace_size(C.byref(desc))
        assert 0 < ws_n <= lib.srswa_gather_bwd_noalloc_max_scratch()
        ws = torch.empty(ws_n, dtype=torch.uint8, device=cuda)
        ref = _call(lib, "srswa_gather_bwd", desc, q, k, v, o, lse, do, sel, bias, ws)
        assert ops.workspace_status(ws) == 0
        got = _call(lib, "srswa_gather_bwd_noalloc", desc, q, k, v, o, lse, do, sel, bias)
        assert _noalloc_status(lib) == 0
        for a, b in zip(got, ref):
            assert torch.isfinite(a).all()
            assert torch.equal(a, b)


def test_noalloc_rejects_oversized_problem(cuda):
    lib = L.lib()
    q, k, v, o, lse, do, sel, bias, desc = _case(cuda, 3, T=256)
    desc.T = 1 << 22  # scratch for 4M tokens exceeds the 32 MiB array; rejected before any launch
    dq = torch.empty_like(q)
    rc = lib.srswa_gather_bwd_noalloc(C.byref(desc), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                      o.stride(0), o.stride(1), o.stride(2), do.data_ptr(), lse.data_ptr(),
                                      sel.data_ptr(), bias.data_ptr(), None, dq.data_ptr(), dq.data_ptr(),
                                      dq.data_ptr(), bias.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == L.ETOOLARGE
