"""Install srswa behind the reference's own module names.

    import srswa.dropin
    srswa.dropin.install("uocr_ref")   # the package holding hf-model-code

After ``install``:
  * ``<pkg>.sparse_gather_triton``      -> ``srswa.sparse_gather``
  * ``<pkg>.sparse_gather_e2e_triton``  -> ``srswa.sparse_gather_e2e``
  * ``<pkg>.modeling_deepseekv2._block_scores_infer / _infer_route_select /
    _decode_attend`` -> ``srswa.dash_infer`` (when that module is loaded)
  * the PageGate candidate methods of ``<pkg>._sparse_base_impl.DeepseekV2Indexer``,
    ``modeling_deepseekv2._dash_block_cand`` and
    ``modeling_unlimitedocr._uocr_dash_decode_allow`` -> ``srswa.page_gate``
  * ``DeepseekV2Indexer._build_page_rope_pos``, ``DeepseekV2IndexerRotary2D.forward``
    and ``SlidingWindowLlamaAttention._main_rope_coords`` -> ``srswa.page_rope``
so DashAttention._forward_triton, SlidingWindowLlamaAttention's sparse branch,
the DSA indexer and the DASH inference overlay call the CUDA kernels without a
source change.  ``install_sglang()`` does the same for the SGLang ops modules.
"""

from __future__ import annotations

import sys

from . import dash_infer, page_gate, page_rope, paged, sparse_gather, sparse_gather_e2e

_INDEXER_METHODS = ("_build_page_aware_ids", "_build_flat_image_token_mask", "_build_image_block_allow_mask",
                    "_build_page_aware_image_block_mask", "_build_kl_candidate_mask")


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
        md._dash_block_cand = page_gate._dash_block_cand
    base = sys.modules.get(f"{pkg}._sparse_base_impl")
    if base is not None:
        ix = getattr(base, "DeepseekV2Indexer", None)
        if ix is not None:
            for name in _INDEXER_METHODS:
                setattr(ix, name, getattr(page_gate, name))
        page_gate._scope_source = base      # _PAGE_SCOPE_PREFILL stays the reference's switch
        if ix is not None:
            ix._build_page_rope_pos = page_rope._build_page_rope_pos
        rot = getattr(base, "DeepseekV2IndexerRotary2D", None)
        if rot is not None:
            rot.forward = page_rope.rotary2d_forward
        attn = getattr(base, "SlidingWindowLlamaAttention", None)
        if attn is not None:
            attn._main_rope_coords = page_rope._main_rope_coords
    mu = sys.modules.get(f"{pkg}.modeling_unlimitedocr")
    if mu is not None:
        mu._uocr_dash_decode_allow = page_gate._uocr_dash_decode_allow


def install_sglang(prefix: str = "sglang.srt.layers.attention.unlimited_dash_ops") -> None:
    at = sys.modules.get(f"{prefix}.attend_triton")
    if at is not None:
        at.dash_sparse_attn_decode = paged.dash_sparse_attn_decode
    rt = sys.modules.get(f"{prefix}.route_triton")
    if rt is not None:
        rt.kbar_refresh_tail_triton = paged.kbar_refresh_tail
