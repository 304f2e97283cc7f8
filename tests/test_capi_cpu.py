"""C ABI checks that need no GPU: libsrswa.so loads, exports every function
declared in include/srswa.h, and rejects invalid arguments before launching
anything (these calls never reach a CUDA API)."""

import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import ROOT

from srswa import _lib as L

HEADER = os.path.join(ROOT, "include", "srswa.h")


def declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"SRSWA_API\s+[\w\s\*]+?\b(srswa_\w+)\s*\(", txt)))


def test_library_loads_and_version():
    lib = L.lib()
    assert lib.srswa_version() >= 100


def test_every_declared_symbol_exported():
    names = declared()
    assert len(names) >= 14
    lib = L.lib()
    for n in names:
        assert hasattr(lib, n), n
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (srswa_\w+)", out))
    assert set(names) <= exported
    assert set(names) == set(L.exported_symbols())


def test_no_cuda_runtime_dependency():
    """cudart is static: the library loads on a host without the CUDA toolkit."""
    out = subprocess.run(["ldd", L.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in out


def test_status_strings():
    assert L.status_text(0) == "ok"
    assert "invalid" in L.status_text(L.EINVAL)
    assert "workspace" in L.status_text(L.EWORKSPACE)


def test_invalid_arguments_rejected_without_launch():
    lib = L.lib()
    # NULL pointers -> EINVAL before any CUDA call
    assert lib.srswa_kbar_contig(None, 1, 0, 0, 1, 1, 128, 64, None, None, None, None) == L.EINVAL
    p = L.RouteParams(64, 8, 8, 16, 11.3, 1e-4, 1.0)
    assert lib.srswa_route(None, 0, 128, 1, 128, None, 0, 0, 1, None, 0, None, 1, None, None, None, 0, p,
                           None, None, None, None, None, None, 0, None) == L.EINVAL
    assert lib.srswa_route_workspace_size(256, 2048, 128, p, 0) > 0      # decode rows: chunked router
    assert lib.srswa_route_workspace_size(65536, 256, 128, p, 0) == 0    # prefill rows: no scratch
    assert lib.srswa_lse_merge(None, None, 1, 1, 1, 1, 0, 0, None, 0, None, None, None) == L.EINVAL
    d = L.DecodeDesc()
    assert lib.srswa_decode_attend(C.byref(d), None, None, None, None, None, None, None, None, None, None,
                                   None, None) == L.EINVAL
    g = L.GatherDesc(1, 16, 10, 10, 1, 96, 8, 64, 512, 0.1, L.BF16, 0, 0, 0, 0, 0, 0, 0, 0, 0)
    assert lib.srswa_gather_fwd(C.byref(g), None, None, None, None, None, None, None, 1, 0, 0, 0, None,
                                None, 0, None) == L.EUNSUPPORTED  # head dim 96
    g.D = 128
    g.HQ = 7
    assert lib.srswa_gather_fwd(C.byref(g), None, None, None, None, None, None, None, 1, 0, 0, 0, None,
                                None, 0, None) == L.EINVAL  # HQ not divisible
    g.HQ = 10
    assert lib.srswa_gather_bwd_workspace_size(C.byref(g)) > 0


def test_paged_gather_forward_checks_without_launch():
    """srswa_gather_fwd_paged (the tensor-core forward of one request over
    paged K / V): unsupported shapes and bad arguments are refused before
    any CUDA call, and the workspace query reports 0 for them."""
    lib = L.lib()
    # one 1000-row request after a 5000-token prefix, 64-token pages [P, 64, 10, 128]
    g = L.GatherDesc(1, 1000, 10, 10, 1, 128, 8, 64, 512, 0.088, L.BF16, 0, 1280, 128,
                     64 * 1280, 1280, 128, 64 * 1280, 1280, 128)
    assert lib.srswa_gather_fwd_paged_workspace_size(C.byref(g), 5000) > 0
    assert lib.srswa_gather_fwd_paged_workspace_size(C.byref(g), -1) == 0   # negative prefix
    fake = C.c_void_p(1 << 20)  # never dereferenced: every call below is refused first
    args = (fake, fake, fake, 100, None, 5000, fake, None, fake, 0, 1280, 128, None, fake, 1 << 30, None)
    assert lib.srswa_gather_fwd_paged(C.byref(g), *args) == L.EINVAL          # no page table
    g.B = 2
    assert lib.srswa_gather_fwd_paged_workspace_size(C.byref(g), 5000) == 0
    args = (fake, fake, fake, 100, fake, 5000, fake, None, fake, 0, 1280, 128, None, fake, 1 << 30, None)
    assert lib.srswa_gather_fwd_paged(C.byref(g), *args) == L.EUNSUPPORTED   # one sequence per call
    g.B, g.dtype = 1, L.F16
    assert lib.srswa_gather_fwd_paged(C.byref(g), *args) == L.EUNSUPPORTED   # bf16 only


def test_route_topm_limit():
    lib = L.lib()
    p = L.RouteParams(64, 8, 8, 64, 11.3, 1e-4, 1.0)  # M = 64 > 32 unsupported
    dummy = 16
    rc = lib.srswa_route_select(dummy, 128, 1, 128, None, 0, p, None, None, None, None, None)
    assert rc == L.EUNSUPPORTED


def test_page_gate_arguments_rejected_without_launch():
    lib = L.lib()
    assert lib.srswa_page_scan_workspace_size(2, 5000) == 2 * 3 * 16     # 16 B per 2048-token chunk and row
    assert lib.srswa_page_ids(None, 0, 1, 1, 1, 1, 2, 7, 1, None, None, None, None, None, 0, None) == L.EINVAL
    assert lib.srswa_page_block_desc(None, None, 0, 1, 1, 64, 1, 16, None) == L.EINVAL   # neither source
    assert lib.srswa_page_block_desc(16, 16, 0, 1, 1, 64, 1, 16, None) == L.EINVAL       # both sources
    assert lib.srswa_page_block_desc(16, None, 0, 1, 1, 64, 1, 24, None) == L.EALIGN     # desc not 16-aligned
    assert lib.srswa_page_cand_mask(16, None, 0, 1, 64, 1, 1, None, 0, 0, None, 0, 1, 0, 1, 16,
                                    None) == L.EINVAL                                     # page mode without qpi
    # decode state: the block size must divide the 2048-token scan chunk
    assert lib.srswa_decode_allow_state(16, 100, 1, 100, 1, 2, 7, 96, 16, 16, 16, 16, 16, 16,
                                        None) == L.EUNSUPPORTED
    assert lib.srswa_decode_allow(None, 1, 1, 2, None, None, 1, 1, None, None, 1, None, None) == L.EINVAL
