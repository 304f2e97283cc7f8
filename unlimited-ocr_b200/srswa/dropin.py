"""Install srswa behind the reference's own module names.

    import srswa.dropin
    srswa.dropin.install("uocr_ref")   # the package holding hf-model-code

After ``install``:
  * ``<pkg>.sparse_gather_triton``      -> ``srswa.sparse_gather``
  * ``<pkg>.sparse_gather_e2e_triton``  -> ``srswa.sparse_gather_e2e``
  * ``<pkg>.modeling_deepseekv2._block_scores_infer / _infer_route_select /
    _decode_attend`` -> ``srswa.dash_infer`` (when that module is loaded)
so DashAttention._forward_triton, SlidingWindowLlamaAttention's sparse branch,
the DSA indexer and the DASH inference overlay call the CUDA kernels without a
source change.  ``install_sglang()`` does the same for the SGLang ops modules.
"""

from __future__ import annotations

import sys

from . import dash_infer, paged, sparse_gather, sparse_gather_e2e


def install(pkg: str) -> None:
    sys.modules[f"{pkg}.sparse_gather_triton"] = sparse_gather
    sys.modules[f"{pkg}.sparse_gather_e2e_triton"] = sparse_gather_e2e
    parent = sys.modules.get(pkg)
    if parent is not None:
        setattr(parent, "sparse_gather_triton", sparse_gather)
        setattr(parent, "sparse_gather_e2e_triton", sparse_gather_e2e)
    md = sys.modules.get(f"{pkg}.modeling_deepseekv2")
    if md is not None:
        for name in ("_block_scores_infer", "_infer_route_select", "_decode_attend"):
            setattr(md, name, getattr(dash_infer, name))


def install_sglang(prefix: str = "sglang.srt.layers.attention.unlimited_dash_ops") -> None:
    at = sys.modules.get(f"{prefix}.attend_triton")
    if at is not None:
        at.dash_sparse_attn_decode = paged.dash_sparse_attn_decode
    rt = sys.modules.get(f"{prefix}.route_triton")
    if rt is not None:
        rt.kbar_refresh_tail_triton = paged.kbar_refresh_tail
