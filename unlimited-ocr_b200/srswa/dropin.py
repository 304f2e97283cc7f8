"""Install srswa behind the reference's own module names.

    import srswa.dropin
    srswa.dropin.install("uocr_ref")   # the package holding hf-model-code

After ``install``:
  * ``<pkg>.sparse_gather_triton``      -> ``srswa.sparse_gather``
  * ``<pkg>.sparse_gather_e2e_triton``  -> ``srswa.sparse_gather_e2e``
  * ``<pkg>.modeling_deepseekv2._block_scores_infer / _infer_route_select /
    _decode_attend`` -> ``srswa.dash_infer`` (when that module is loaded)
  * ``DeepseekV2Indexer.select_and_kl_loss`` -> ``srswa.dsa`` (one index
    head on CUDA; other cases keep the reference's method)
  * the PageGate candidate methods of ``<pkg>._sparse_base_impl.DeepseekV2Indexer``,
    ``modeling_deepseekv2._dash_block_cand`` and
    ``modeling_unlimitedocr._uocr_dash_decode_allow`` -> ``srswa.page_gate``
  * ``DeepseekV2Indexer._build_page_rope_pos``, ``DeepseekV2IndexerRotary2D.forward``
    and ``SlidingWindowLlamaAttention._main_rope_coords`` -> ``srswa.page_rope``
so DashAttention._forward_triton, SlidingWindowLlamaAttention's sparse branch,
the DSA indexer and the DASH inference overlay call the CUDA kernels without a
source change.  ``install_sglang()`` does the same for the SGLang ops modules
and for the DASH attention backend's own imported copies of them.
"""

from __future__ import annotations

import sys

from . import dash_infer, dsa, page_gate, page_rope, paged, sparse_gather, sparse_gather_e2e

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
            if ix.select_and_kl_loss is not dsa.select_and_kl_loss:   # the reference's, for the cases it keeps
                dsa._ORIGINAL[ix] = ix.select_and_kl_loss
            ix.select_and_kl_loss = dsa.select_and_kl_loss
        rot = getattr(base, "DeepseekV2IndexerRotary2D", None)
        if rot is not None:
            rot.forward = page_rope.rotary2d_forward
        attn = getattr(base, "SlidingWindowLlamaAttention", None)
        if attn is not None:
            attn._main_rope_coords = page_rope._main_rope_coords
    mu = sys.modules.get(f"{pkg}.modeling_unlimitedocr")
    if mu is not None:
        mu._uocr_dash_decode_allow = page_gate._uocr_dash_decode_allow


# SGLang names this library provides, per reference module that defines them
_SGLANG_OPS = {
    "attend_triton": ("dash_sparse_attn", "dash_sparse_attn_decode"),
    "route_triton": ("route_decode_triton", "route_prefill_triton", "kbar_refresh_tail_triton",
                     "win_bounds_decode"),
}
_SGLANG_BACKEND = "sglang.srt.layers.attention.unlimited_ocr_v2_backend"


def install_sglang(prefix: str = "sglang.srt.layers.attention.unlimited_dash_ops",
                   backend: str = _SGLANG_BACKEND, overlap_router: bool = True) -> list[str]:
    """Point SGLang's DASH serving ops at ``srswa.paged``.

    The backend binds the ops by ``from ... import`` when it is imported
    (whl:sglang/srt/layers/attention/unlimited_ocr_v2_backend.py:18-52), so the
    names are rebound both in the ops modules and in the already-imported
    backend module, which holds its own copies.  A module imported later picks
    up the ops modules' (already rebound) attributes.  The torch-only planning
    helpers (kbar_tail_plan, kbar_all_plan, prefill_row2req) stay the
    reference's.  overlap_router: the backend's own dash_sparse_attn_decode
    becomes paged.dash_sparse_attn_decode_after_router, since its _forward
    issues the attend right after route_decode_triton with only views in
    between, and writes q and the caches before routing
    (unlimited_ocr_v2_backend.py:1412-1448); the ops module keeps the plain
    op for other callers.  Returns the qualified names rebound."""
    done = []
    for mod_name, names in _SGLANG_OPS.items():
        mod = sys.modules.get(f"{prefix}.{mod_name}")
        if mod is None:
            continue
        for name in names:
            setattr(mod, name, getattr(paged, name))
            done.append(f"{mod.__name__}.{name}")
    be = sys.modules.get(backend)
    if be is not None:
        for names in _SGLANG_OPS.values():
            for name in names:
                if hasattr(be, name):
                    op = getattr(paged, name)
                    if overlap_router and name == "dash_sparse_attn_decode":
                        op = paged.dash_sparse_attn_decode_after_router
                    setattr(be, name, op)
                    done.append(f"{be.__name__}.{name}")
    return done
