"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs only where a read-only checkout of the reference is available; its
location must be given in ``SRSWA_REFERENCE`` (the script refuses to guess).  It
imports the reference's own code -- the HF PyTorch SR-SWA path, its Triton
kernels under the Triton CPU interpreter, and the SGLang serving ops from the
reference's wheel -- runs them on small seeded inputs and writes
``tests/golden/<case>.npz`` (inputs + outputs + version metadata).  GPU runs
never execute this script; the tests there read the committed ``.npz`` files.

Usage:  SRSWA_REFERENCE=<reference checkout> python tests/golden/make_golden.py [case ...]
"""

from __future__ import annotations

import importlib
import importlib.util
import json
import math
import os
import shutil
import sys
import tempfile
import types
import zipfile

os.environ["TRITON_INTERPRET"] = "1"
os.environ.setdefault("CODE_STAMP_LOG", "0")

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF = os.environ.get("SRSWA_REFERENCE", "")
# what the fixtures record as their source: the project, not a machine path
REF_NAME = "dongf9527/Unlimited-OCR (hf-model-code/, wheel/sglang-0.5.20.dev10)"
OUT = os.path.dirname(os.path.abspath(__file__))
WHEEL = "wheel/sglang-0.5.20.dev10+g8d62f5fb9c-py3-none-any.whl"


def _shim_transformers():
    """Four attributes the reference expects from transformers 4.52 (its pin);
    the container has transformers 5.x where they moved or were removed."""
    import transformers.pytorch_utils as pu
    import transformers.utils as tu
    import transformers.utils.import_utils as iu
    iu.is_torch_fx_available = lambda: False
    pu.is_torch_greater_or_equal_than_1_13 = True
    pu.ALL_LAYERNORM_LAYERS = []
    tu.is_flash_attn_greater_or_equal_2_10 = lambda *a, **k: False


def import_reference():
    """Copy hf-model-code to a temp package (it uses relative imports) and
    import the modules the SR-SWA path lives in."""
    _shim_transformers()
    tmp = tempfile.mkdtemp(prefix="uocr_ref_")
    pkg = os.path.join(tmp, "uocr_ref")
    shutil.copytree(os.path.join(REF, "hf-model-code"), pkg,
                    ignore=shutil.ignore_patterns("tokenizer*", "*.json", "*.md"))
    open(os.path.join(pkg, "__init__.py"), "w").close()
    sys.path.insert(0, tmp)
    mods = {}
    for name in ("modeling_deepseekv2", "dash_attention", "sparse_gather_triton",
                 "sparse_gather_e2e_triton"):
        mods[name] = importlib.import_module(f"uocr_ref.{name}")
    return mods


def import_sglang_ops():
    """Load the SGLang DASH ops from the reference wheel with stub parent
    packages (the rest of SGLang is not needed for these files)."""
    tmp = tempfile.mkdtemp(prefix="uocr_sgl_")
    sub = "sglang/srt/layers/attention/unlimited_dash_ops/"
    with zipfile.ZipFile(os.path.join(REF, WHEEL)) as z:
        for n in z.namelist():
            if n.startswith(sub) and n.endswith(".py"):
                z.extract(n, tmp)
    for pk in ("sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.attention",
               "sglang.srt.layers.attention.unlimited_dash_ops"):
        m = types.ModuleType(pk)
        m.__path__ = [os.path.join(tmp, *pk.split("."))]
        sys.modules[pk] = m
    out = {}
    for name in ("common", "dash_router", "dash_stage0", "attend_triton", "route_triton"):
        full = f"sglang.srt.layers.attention.unlimited_dash_ops.{name}"
        spec = importlib.util.spec_from_file_location(full, os.path.join(tmp, sub, name + ".py"))
        mod = importlib.util.module_from_spec(spec)
        sys.modules[full] = mod
        spec.loader.exec_module(mod)
        out[name] = mod
    # CPU interpreter: no PDL, no graph capture
    out["common"]._PDL_SUPPORTED = False
    out["attend_triton"]._arch_supports_pdl = lambda: False
    torch.cuda.is_current_stream_capturing = lambda: False
    return out


def bf16r(t):
    return t.to(torch.bfloat16).to(torch.float32)


def save(name, **arrs):
    meta = dict(torch=torch.__version__, numpy=np.__version__,
                transformers=__import__("transformers").__version__,
                triton=__import__("triton").__version__, triton_interpret=True,
                reference=REF_NAME, shim="transformers 4-symbol shim (see import_reference)")
    arrs = {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v))
            for k, v in arrs.items()}
    np.savez_compressed(os.path.join(OUT, name + ".npz"), meta=json.dumps(meta), **arrs)
    print("wrote", name, {k: v.shape for k, v in arrs.items()})


def router_ns(block_size, local_blocks, head_cls, stage0="head_cls", q_chunk=2048):
    return types.SimpleNamespace(block_size=block_size, local_blocks=local_blocks,
                                 local_window=local_blocks * block_size,
                                 head_cls=head_cls, stage0=stage0, q_chunk=q_chunk)


def case_route(m):
    """_block_scores_infer (head_cls + indexer) and _infer_route_select."""
    md = m["modeling_deepseekv2"]
    g = torch.Generator().manual_seed(11)
    B, S, d, BS, L = 2, 700, 128, 64, 2
    nblk = (S + BS - 1) // BS
    idx_q = bf16r(torch.randn(B, S, d, generator=g))
    idx_k = bf16r(torch.randn(B, S, d, generator=g))
    hc0 = torch.zeros(d)
    hc1 = torch.randn(d, generator=g) * 0.3
    q_pos = torch.arange(S)[None].expand(B, S).contiguous()
    p = dict(idx_scale=128.0 / math.sqrt(d), floor=1e-4, sigma=1.0, K=4, topm=6)
    outs = {}
    for tag, hc in (("hc0", hc0), ("hc1", hc1)):
        sc = md._block_scores_infer(router_ns(BS, L, hc), idx_q, idx_k, q_pos, nblk)
        topi, bias, valid = md._infer_route_select(sc, None, p)
        outs[f"scores_{tag}"] = sc
        outs[f"topi_{tag}"] = topi
        outs[f"bias_{tag}"] = bias
        outs[f"valid_{tag}"] = valid
    # page-aware candidate mask (with rows whose mask empties -> fallback)
    cand = torch.rand(B, S, nblk, generator=g) < 0.3
    cand[:, 500:560] = False
    sc = outs["scores_hc0"]
    topi, bias, valid = md._infer_route_select(sc, cand, p)
    outs.update(cand=cand, topi_cand=topi, bias_cand=bias, valid_cand=valid)
    # sigma != 1, different K/M
    p2 = dict(idx_scale=3.0, floor=1e-2, sigma=0.7, K=8, topm=16)
    topi, bias, valid = md._infer_route_select(sc, None, p2)
    outs.update(topi_p2=topi, bias_p2=bias, valid_p2=valid)
    # indexer stage0 (token block-max)
    sci = md._block_scores_infer(router_ns(BS, L, hc0, stage0="indexer"), idx_q, idx_k, q_pos, nblk)
    outs["scores_indexer"] = sci
    save("route", idx_q=idx_q, idx_k=idx_k, hc1=hc1, q_pos=q_pos,
         params=np.array([BS, L, p["K"], p["topm"]]),
         fparams=np.array([p["idx_scale"], p["floor"], p["sigma"]]),
         fparams2=np.array([p2["idx_scale"], p2["floor"], p2["sigma"], p2["K"], p2["topm"]]),
         **outs)


def case_entmax(m):
    da = m["dash_attention"]
    g = torch.Generator().manual_seed(12)
    x = torch.randn(64, 16, generator=g) * 8.0
    x[5:9, 10:] = -1.0e4
    x[20] = -1.0e4
    x[30, :3] = 3.0
    y = da.entmax15(x, dim=-1)
    save("entmax", x=x, y=y)


def case_decode_attend(m):
    """_decode_attend, with selections from the reference router."""
    md = m["modeling_deepseekv2"]
    g = torch.Generator().manual_seed(13)
    B, H, D, S, BS, L, d = 2, 2, 64, 1100, 64, 3, 128
    nblk = (S + BS - 1) // BS
    q = bf16r(torch.randn(B, H, 2, D, generator=g))
    k = bf16r(torch.randn(B, H, S, D, generator=g))
    v = bf16r(torch.randn(B, H, S, D, generator=g))
    idx_q = bf16r(torch.randn(B, 2, d, generator=g))
    idx_k = bf16r(torch.randn(B, S, d, generator=g))
    q_pos = torch.tensor([[S - 2, S - 1], [700, 1003]])
    sc = md._block_scores_infer(router_ns(BS, L, torch.zeros(d)), idx_q, idx_k, q_pos, nblk)
    p = dict(idx_scale=128.0 / math.sqrt(d), floor=1e-4, sigma=1.0, K=5, topm=8)
    topi, bias, valid = md._infer_route_select(sc, None, p)
    scale = 1.0 / math.sqrt(D)
    out = md._decode_attend(q, k, v, topi, bias, valid, q_pos, BS, L * BS, scale)
    save("decode_attend", q=q, k=k, v=v, idx_q=idx_q, idx_k=idx_k, q_pos=q_pos,
         scores=sc, topi=topi, bias=bias, valid=valid, out=out,
         params=np.array([BS, L, p["K"], p["topm"]]), scale=np.array(scale))


def case_forward_dense(m):
    """DashAttention._forward_dense fwd + autograd grads (the DASH merge
    semantics, incl. selected blocks overlapping the window)."""
    da = m["dash_attention"]
    md = m["modeling_deepseekv2"]
    g = torch.Generator().manual_seed(14)
    B, H, S, D, BS, L, K = 2, 2, 256, 64, 32, 2, 4
    nblk = (S + BS - 1) // BS
    q = bf16r(torch.randn(B, H, S, D, generator=g))
    k = bf16r(torch.randn(B, H, S, D, generator=g))
    v = bf16r(torch.randn(B, H, S, D, generator=g))
    # selection: random distinct blocks <= qblk (some overlap the window, some
    # are purely remote); invalid slots marked by valid=False
    topi = torch.zeros(B, S, K, dtype=torch.long)
    valid = torch.zeros(B, S, K, dtype=torch.bool)
    for b in range(B):
        for t in range(S):
            qb = t // BS
            perm = torch.randperm(qb + 1, generator=g)[:K]
            n = perm.numel()
            topi[b, t, :n] = perm
            valid[b, t, :n] = True
            if n < K:
                # invalid slots point at blocks not selected by a valid slot
                rest = [c for c in range(nblk) if c not in perm.tolist()][:K - n]
                topi[b, t, n:] = torch.tensor(rest)
    bias = (torch.randn(B, S, K, generator=g) * 0.5).requires_grad_(True)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    self_ = types.SimpleNamespace(block_size=BS, q_chunk=128, local_window=L * BS,
                                  _scale=1.0 / math.sqrt(D))
    o = da.DashAttention._forward_dense(self_, qg, kg, vg, topi, bias, valid, S, nblk, None)
    do = torch.randn(o.shape, generator=g)
    (o * do).sum().backward()
    save("forward_dense", q=q, k=k, v=v, topi=topi, valid=valid, bias=bias.detach(),
         o=o.detach(), do=do, dq=qg.grad, dk=kg.grad, dv=vg.grad, dbias=bias.grad,
         params=np.array([BS, L]), scale=np.array(1.0 / math.sqrt(D)))
    del md


def case_gather_triton(m):
    """triton_gather_attention (K1-K3) under the Triton CPU interpreter:
    packing (seg), two index heads, duplicate ids and -1 padding."""
    sg = m["sparse_gather_triton"]
    g = torch.Generator().manual_seed(15)
    B, HQ, Hkv, T, D, BS, S, LW = 2, 4, 2, 224, 64, 32, 4, 72
    # bf16-representable fp32 inputs: the GPU runs bf16 on exactly these values
    q = bf16r(torch.randn(B, HQ, T, D, generator=g))
    k = bf16r(torch.randn(B, Hkv, T, D, generator=g))
    v = bf16r(torch.randn(B, Hkv, T, D, generator=g))
    nb = (T + BS - 1) // BS
    pos = torch.arange(T)[None].repeat(B, 1)
    pos[1, 90:] = torch.arange(T - 90)         # packed: 2nd sample starts at 90
    # The reference K1 has no NaN-safe running max (sparse_gather_triton.py:90-94):
    # a leading selected block with no kept key gives NaN.  Its callers only
    # select remote blocks, so slot 0 holds a block with >= 1 key in
    # [seg, t - LW + 1) whenever one exists; later slots are random (window
    # blocks, future blocks, -1) and slot 1 repeats slot 0 (dedup).
    sel = torch.randint(-1, nb, (B, 2, T, S), generator=g)
    for b in range(B):
        for t in range(T):
            seg = t - int(pos[b, t])
            ls = max(t - LW + 1, seg)
            rem = [c for c in range(nb) if max(c * BS, seg) < min((c + 1) * BS, ls)]
            for hi in range(2):
                if rem:
                    sel[b, hi, t, 0] = rem[int(torch.randint(len(rem), (1,), generator=g))]
                else:
                    # no remote key at all: only -1 or future blocks (skipped)
                    row = sel[b, hi, t]
                    sel[b, hi, t] = torch.where((row >= 0) & (row * BS <= t), -1, row)
    sel[:, :, :, 1] = sel[:, :, :, 0]          # duplicates
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = sg.triton_gather_attention(qg, kg, vg, sel, pos, None, BS, 0.3, LW)
    do = torch.randn(o.shape, generator=g)
    (o * do).sum().backward()
    save("gather_triton", q=q, k=k, v=v, sel=sel, pos=pos, o=o.detach(), do=do,
         dq=qg.grad, dk=kg.grad, dv=vg.grad, params=np.array([BS, LW]), scale=np.array(0.3))


def case_gather_e2e(m):
    """triton_gather_attention_e2e (K5-K7) under the interpreter, with grads
    to q/k/v and the per-slot bias."""
    se = m["sparse_gather_e2e_triton"]
    g = torch.Generator().manual_seed(16)
    B, H, T, D, BS, S, LW = 2, 2, 200, 64, 32, 3, 64
    q = bf16r(torch.randn(B, H, T, D, generator=g))
    k = bf16r(torch.randn(B, H, T, D, generator=g))
    v = bf16r(torch.randn(B, H, T, D, generator=g))
    nb = (T + BS - 1) // BS
    sel = torch.full((B, 1, T, S), -1, dtype=torch.long)
    for b in range(B):
        for t in range(T):
            cand = torch.randperm(t // BS + 1, generator=g)[:S]
            sel[b, 0, t, :cand.numel()] = cand
    sel[0, 0, 150, 2] = sel[0, 0, 150, 0]      # one duplicate
    bias = (torch.randn(B, T, S, generator=g) * 0.5).requires_grad_(True)
    pos = torch.arange(T)[None].repeat(B, 1)
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (q, k, v))
    o = se.triton_gather_attention_e2e(qg, kg, vg, sel, bias, pos, None, BS, 0.25, LW)
    do = torch.randn(o.shape, generator=g)
    (o * do).sum().backward()
    save("gather_e2e", q=q, k=k, v=v, sel=sel, bias=bias.detach(), o=o.detach(), do=do,
         dq=qg.grad, dk=kg.grad, dv=vg.grad, dbias=bias.grad,
         params=np.array([BS, LW]), scale=np.array(0.25))
    del nb


def case_block_max(m):
    sg = m["sparse_gather_triton"]
    g = torch.Generator().manual_seed(17)
    B, C, Sk, D, BS, LW = 2, 90, 200, 64, 16, 40
    q = bf16r(torch.randn(B, C, D, generator=g))
    k = bf16r(torch.randn(B, Sk, D, generator=g))
    pos = torch.arange(Sk - C, Sk)[None].repeat(B, 1)
    seg = torch.zeros(B, C, dtype=torch.long)
    seg[1, 40:] = 150
    nblk = (Sk + BS - 1) // BS
    out = sg.triton_block_max_score(q, k, pos, seg, BS, nblk, LW)
    save("block_max", q=q, k=k, pos=pos, seg=seg, out=out, params=np.array([BS, LW, nblk]))


def case_paged(sgl):
    """SGLang KBarCache summaries, torch decode scores + route_and_select, and
    the dash_sparse_attn_decode kernel (interpreter) on a shuffled page pool."""
    at, st, dr = sgl["attend_triton"], sgl["dash_stage0"], sgl["dash_router"]
    g = torch.Generator().manual_seed(18)
    R, H, Hkv, D, d, BS, L, W = 3, 2, 2, 64, 64, 32, 2, 12
    P = R * W + 3
    seq = torch.tensor([350, 47, 161], dtype=torch.int32)
    perm = torch.randperm(P, generator=g)[: R * W].view(R, W).to(torch.int32)
    k_cache = bf16r(torch.randn(P, BS, Hkv, D, generator=g))
    v_cache = bf16r(torch.randn(P, BS, Hkv, D, generator=g))
    idx_cache = bf16r(torch.randn(P, BS, d, generator=g))
    q = bf16r(torch.randn(R, H, D, generator=g))
    idx_q = bf16r(torch.randn(R, d, generator=g))
    hc = torch.randn(d, generator=g) * 0.2
    cache = st.KBarCache(P, d, "cpu")
    # summaries of every page in use
    for r in range(R):
        nb = (int(seq[r]) + BS - 1) // BS
        pages = perm[r, :nb].long()
        pos = torch.arange(nb)[:, None] * BS + torch.arange(BS)[None, :]
        cache.put(pages, st._summary_keys(idx_cache[pages].float(), pos < int(seq[r]), hc,
                                          1.0 / math.sqrt(d)))
    kbar = cache.k_bar.clone()
    sc = st.headcls_scores_decode(idx_q=idx_q, cache=cache, block_table=perm, seq_lens=seq,
                                  max_block=W, block_size=BS, local_blocks=L, decode_query_len=1)
    router = dr.DashRouterMath(index_dim=d, block_size=BS, local_blocks=L, topk_blocks=8,
                               scaling_factor=5.0, sigma=1.0, prior_floor=1e-3,
                               budget_remote=3, topm=4)
    idx, bias = router.route_and_select(sc[0], W)
    out = torch.zeros(R, H, D)
    ti = idx.unsqueeze(0).expand(Hkv, -1, -1)
    tb = bias.unsqueeze(0).expand(Hkv, -1, -1)
    at.dash_sparse_attn_decode(q, k_cache, v_cache, ti, tb, perm, seq, Hkv, 0.2, out, 1,
                               local_blocks=L, sparse_block_size=BS)
    save("paged", q=q, k_cache=k_cache, v_cache=v_cache, idx_cache=idx_cache, idx_q=idx_q,
         hc=hc, block_table=perm, seq_lens=seq, kbar=kbar, scores=sc[0], idx=idx, bias=bias,
         out=out, params=np.array([BS, L, 3, 4]), fparams=np.array([5.0 / math.sqrt(d), 1e-3, 1.0, 0.2]))


def case_paged_prefill(sgl):
    """SGLang prefill serving ops on a shuffled page pool of three requests
    with cached prefixes: the k_bar refresh driven by kbar_all_plan, the
    varlen router route_prefill_triton (with an image-allow mask) and the
    paged prefill attend dash_sparse_attn (K8) on its selection, plus the
    decode scan window win_bounds_decode (K14) -- all interpreted."""
    at, rt, st = sgl["attend_triton"], sgl["route_triton"], sgl["dash_stage0"]
    g = torch.Generator().manual_seed(23)
    R, H, Hkv, D, d, BS, L, W = 3, 4, 2, 64, 64, 32, 2, 14
    P = R * W + 5
    ctx = torch.tensor([0, 70, 20], dtype=torch.int32)
    qlen = torch.tensor([90, 40, 130], dtype=torch.int32)
    seq = ctx + qlen
    cu = torch.zeros(R + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(qlen, 0)
    N = int(cu[-1])
    perm = torch.randperm(P, generator=g)[: R * W].view(R, W).to(torch.int32)
    k_cache = bf16r(torch.randn(P, BS, Hkv, D, generator=g))
    v_cache = bf16r(torch.randn(P, BS, Hkv, D, generator=g))
    idx_cache = bf16r(torch.randn(P, BS, d, generator=g))
    q = bf16r(torch.randn(N, H, D, generator=g))
    idx_q = bf16r(torch.randn(N, d, generator=g))
    hc = torch.randn(d, generator=g) * 0.2
    # summaries of the prefix pages (as a previous step left them), then the
    # refresh of the pages this prefill step writes, driven by kbar_all_plan
    cache = st.KBarCache(P, d, "cpu")
    for r in range(R):
        nb = (int(ctx[r]) + BS - 1) // BS
        if nb:
            pages = perm[r, :nb].long()
            pos = torch.arange(nb)[:, None] * BS + torch.arange(BS)[None, :]
            cache.put(pages, st._summary_keys(idx_cache[pages].float(), pos < int(ctx[r]), hc,
                                              1.0 / math.sqrt(d)))
    kbar_before = cache.k_bar.clone()
    plan = rt.kbar_all_plan(block_table=perm, seq_lens=seq, context_lens=ctx, block_size=BS, max_block=W,
                            max_query_len=int(qlen.max()), device="cpu")
    rt.kbar_refresh_tail_triton(kv_cache=idx_cache, k_bar=cache.k_bar, block_table=perm, seq_lens=seq,
                                head_cls=hc, block_size=BS, plan=plan)
    kbar = cache.k_bar.clone()
    row2req = rt.prefill_row2req(cu_seqlens_q=cu, device="cpu")
    # image-allow mask [N, WQ] (WQ > W)
    WQ = W + 2
    allow = torch.rand(N, WQ, generator=g) < 0.6
    topm, budget = 16, 4
    out_idx = torch.full((N, topm), -7, dtype=torch.int32)
    out_bias = torch.full((N, topm), 9.0)
    width, _, _ = rt.route_prefill_triton(
        idx_q=idx_q, k_bar=kbar, block_table=perm, seq_lens=seq, cu_seqlens_q=cu, context_lens=ctx,
        row2req=row2req, image_allow=allow, out_idx=out_idx, out_bias=out_bias, max_block=W, block_size=BS,
        local_blocks=L, idx_scale=5.0, prior_floor=1e-3, sigma=1.0, topm=topm, budget=budget)
    # the wheel packs the active blocks at the front of out_idx
    ti = out_idx[:, :budget].contiguous()
    tb = out_bias[:, :budget].contiguous()
    out = torch.zeros(N, H, D)
    at.dash_sparse_attn(q, k_cache, v_cache, ti.unsqueeze(0).expand(Hkv, -1, -1),
                        tb.unsqueeze(0).expand(Hkv, -1, -1), perm, cu, seq, ctx, int(qlen.max()), Hkv, 0.125,
                        out, local_blocks=L, sparse_block_size=BS)
    # decode scan window over decode rows of the same requests (2 per request)
    dql = 2
    dallow = torch.rand(R * dql, WQ, generator=g) < 0.3
    dallow[1] = False                      # a row with no allowed block
    lo = torch.zeros(R * dql, dtype=torch.int32)
    hi = torch.zeros(R * dql, dtype=torch.int32)
    fit = torch.zeros(R * dql, dtype=torch.int8)
    rt.win_bounds_decode(allow=dallow, seq_lens=seq, lo=lo, hi=hi, fit=fit, max_block=W, block_size=BS,
                         local_blocks=L, decode_query_len=dql, tile=4)
    save("paged_prefill", q=q, k_cache=k_cache, v_cache=v_cache, idx_cache=idx_cache, idx_q=idx_q, hc=hc,
         block_table=perm, seq_lens=seq, context_lens=ctx, cu_seqlens_q=cu, row2req=row2req,
         plan_pages=plan[0], plan_tok=plan[1], kbar_before=kbar_before, kbar=kbar, allow=allow,
         out_idx=out_idx, out_bias=out_bias, width=np.array(width), out=out, dallow=dallow, lo=lo, hi=hi,
         fit=fit, params=np.array([BS, L, topm, budget, dql, 4]), fparams=np.array([5.0, 1e-3, 1.0, 0.125]))


def case_gather_kl(m):
    """DSA sparse-stage KL distillation: _kl_chunk_core (the KL of
    select_and_kl_loss over the selected blocks, one index head) in bf16 with
    its autograd gradients to the index q / k; batch 0 unpacked, batch 1
    packed (two samples, cross-sample keys dropped through same_seg)."""
    sb = importlib.import_module("uocr_ref._sparse_base_impl")
    g = torch.Generator().manual_seed(31)
    B, C, H, Hkv, D, d, BS, LW, S = 2, 300, 4, 2, 32, 32, 16, 48, 5
    nblk = (C + BS - 1) // BS
    q_main = torch.randn(B, H, C, D, generator=g).to(torch.bfloat16)
    k_main = torch.randn(B, Hkv, C, D, generator=g).to(torch.bfloat16)
    idx_q = (torch.randn(B, 1, C, d, generator=g) * 0.3).to(torch.bfloat16)
    idx_k = (torch.randn(B, 1, C, d, generator=g) * 0.3).to(torch.bfloat16)
    pos = torch.arange(C)[None].repeat(B, 1)
    seg_start = torch.zeros(B, C, dtype=torch.long)
    seg_start[1, 170:] = 170                      # batch 1: a second sample from token 170
    sel = torch.full((B, C, S), -1, dtype=torch.long)
    for b in range(B):
        for c in range(C):
            cands = torch.arange(0, max(c // BS, 0))
            if len(cands):
                pick = cands[torch.randperm(len(cands), generator=g)[:S]]
                sel[b, c, :len(pick)] = pick
    sel[0, 200, 2] = sel[0, 200, 0]              # a repeated block counts once
    keep_block = torch.zeros(B, 1, C, nblk + 1, dtype=torch.bool)
    keep_block.scatter_(-1, sel.masked_fill(sel < 0, nblk)[:, None], True)
    keep_block = keep_block[..., :nblk]
    kpos = torch.arange(C)
    same_seg = (kpos[None, None, :] >= seg_start[:, :, None])[:, None]    # [B,1,C,Sk]
    scaling = 1.0 / math.sqrt(D)
    qi = idx_q.clone().requires_grad_(True)
    ki = idx_k.clone().requires_grad_(True)
    kl = sb._kl_chunk_core(qi, ki, q_main, k_main, keep_block, pos, BS, scaling, H, H // Hkv, LW, same_seg)
    gout = torch.randn(kl.shape, generator=g)
    kl.backward(gout)
    save("gather_kl", idx_q=idx_q.float()[:, 0], idx_k=idx_k.float()[:, 0], q_main=q_main.float().transpose(1, 2),
         k_main=k_main.float().transpose(1, 2), sel=sel, pos=pos, seg=seg_start, kl=kl.detach()[:, 0],
         gout=gout[:, 0], d_idx_q=qi.grad.float()[:, 0], d_idx_k=ki.grad.float()[:, 0],
         params=np.array([BS, LW]), scaling=np.array(scaling))


PAGE_IMG, PAGE_MARK = 128815, 128827   # config.json image_token_id, page_token_id


def page_gate_rows(g, per_page, text_vocab=1000):
    """Seeded token rows covering the PageGate cases: <PAGE>-marked prompt
    pages (marker mode) with an instruction and response pages; an unmarked
    image run split every per_page tokens (per-page mode) with a marked
    response; image tokens before the first marker; a text-only row."""
    def txt(n):
        return torch.randint(0, text_vocab, (n,), generator=g).tolist()

    def img(n):
        return [PAGE_IMG] * n

    rows = []
    r = [0]                                                   # marker mode
    for _ in range(5):
        r += [PAGE_MARK] + img(int(torch.randint(20, 90, (1,), generator=g))) + txt(3)
    r += txt(40)
    for _ in range(4):
        r += [PAGE_MARK] + txt(int(torch.randint(10, 60, (1,), generator=g)))
    rows.append(r)
    r = [0] + img(per_page * 4 + 5) + txt(30)                 # per-page mode
    for _ in range(3):
        r += [PAGE_MARK] + txt(int(torch.randint(10, 70, (1,), generator=g)))
    rows.append(r)
    r = [0] + img(37) + txt(5) + [PAGE_MARK] + img(50) + [PAGE_MARK] + img(41) + txt(20)   # images before markers
    r += [PAGE_MARK] + txt(33) + [PAGE_MARK] + txt(25)
    rows.append(r)
    rows.append([0] + txt(300))                               # text only
    S = max(len(x) for x in rows)
    ids = torch.full((len(rows), S), 7, dtype=torch.long)
    for i, x in enumerate(rows):
        ids[i, :len(x)] = torch.tensor(x)
    return ids


def case_page_gate(m):
    """PageGate: _build_page_aware_ids, _build_flat_image_token_mask,
    _build_kl_candidate_mask (both constraint settings) and
    _uocr_dash_decode_allow (prefill state + decode steps)."""
    base = importlib.import_module("uocr_ref._sparse_base_impl")
    for name, attrs in (("easydict", {"EasyDict": dict}), ("addict", {"Dict": dict})):
        if name not in sys.modules:      # vision-encoder deps, not on this path
            mod = types.ModuleType(name)
            for k_, v_ in attrs.items():
                setattr(mod, k_, v_)
            sys.modules[name] = mod
    mu = importlib.import_module("uocr_ref.modeling_unlimitedocr")
    Ix = base.DeepseekV2Indexer
    g = torch.Generator().manual_seed(21)
    per_page = 7
    ids = page_gate_rows(g, per_page)
    B, S = ids.shape
    outs = dict(ids=ids, params=np.array([PAGE_IMG, PAGE_MARK, per_page]))

    def indexer(bs, constraint):
        ns = types.SimpleNamespace(block_size=bs, per_page_image_tokens=per_page, layer_idx=0,
                                   image_bucket_constraint=constraint, _page_aware_diag_logged=True,
                                   image_token_id=PAGE_IMG, page_token_id=PAGE_MARK,
                                   q_proj=types.SimpleNamespace(weight=torch.zeros(1)))
        for fn in ("_build_page_aware_ids", "_build_flat_image_token_mask", "_build_image_block_allow_mask",
                   "_build_page_aware_image_block_mask", "_build_kl_candidate_mask"):
            setattr(ns, fn, types.MethodType(getattr(Ix, fn), ns))
        return ns

    saved = base._PAGE_SCOPE_PREFILL
    for scope in (0, 1):
        base._PAGE_SCOPE_PREFILL = bool(scope)
        for kl, tag in ((S, "full"), (S - 37, "trunc"), (S + 50, "pad")):
            itm, ipi, qpi = indexer(16, True)._build_page_aware_ids(ids, PAGE_IMG, PAGE_MARK, kl)
            outs[f"itm_s{scope}_{tag}"], outs[f"ipi_s{scope}_{tag}"], outs[f"qpi_s{scope}_{tag}"] = itm, ipi, qpi
    base._PAGE_SCOPE_PREFILL = saved
    # a text-only batch gives (None, None, None)
    none = indexer(16, True)._build_page_aware_ids(ids[3:], PAGE_IMG, PAGE_MARK, S)
    outs["none_text_only"] = np.array([x is None for x in none])
    outs["flat_itm"] = indexer(16, False)._build_flat_image_token_mask(ids, PAGE_IMG, S)

    # candidate masks: scope-1 page ids, two block sizes, a query chunk with an
    # offset and positions beyond the page-id length (clamped by the reference)
    itm, ipi, qpi = outs["itm_s1_full"], outs["ipi_s1_full"], outs["qpi_s1_full"]
    pos = torch.arange(S)[None].expand(B, S).contiguous()
    pos_chunk = (torch.arange(150) + S - 120)[None].expand(B, 150).contiguous()
    outs["pos_chunk"] = pos_chunk
    for bs in (16, 64):
        nblk = -(-S // bs)
        for constraint in (True, False):
            ix = indexer(bs, constraint)
            flat = outs["flat_itm"]
            for ptag, pp_ in (("all", pos), ("chunk", pos_chunk)):
                cq = pp_.shape[1]
                cm = ix._build_kl_candidate_mask(pp_, nblk, itm if constraint else flat, B, cq,
                                                 image_token_page_ids=ipi if constraint else None,
                                                 query_token_page_ids=qpi if constraint else None)
                outs[f"cand_bs{bs}_c{int(constraint)}_{ptag}"] = cm[:, 0]
        cm = indexer(bs, False)._build_kl_candidate_mask(pos, nblk, None, B, S)
        outs[f"cand_bs{bs}_none"] = cm[:, 0]

    # decode allow: prefill state, then decode steps (a <PAGE> marker on step 2
    # of row 0 and step 4 of row 1 advances that row's page)
    for bs in (16, 64):
        ix = indexer(bs, True)
        cache = types.SimpleNamespace(n=S)
        cache.get_seq_length = lambda c=cache: c.n
        assert mu._uocr_dash_decode_allow(ix, ids, cache) is None
        st = cache._uocr_pg
        outs[f"dec_bs{bs}_bmin"], outs[f"dec_bs{bs}_bmax"] = st["bmin"].clone(), st["bmax"].clone()
        outs[f"dec_bs{bs}_pp"], outs[f"dec_bs{bs}_mcum0"] = st["pp"].clone(), st["mcum"].clone()
        steps = torch.randint(0, 1000, (B, 12), generator=g)
        steps[0, 2] = PAGE_MARK
        steps[1, 4] = PAGE_MARK
        steps[2, 0] = PAGE_MARK
        allows = []
        for k_ in range(steps.shape[1]):
            a = mu._uocr_dash_decode_allow(ix, steps[:, k_:k_ + 1], cache)
            cache.n += 1
            allows.append(a)
        outs[f"dec_bs{bs}_steps"] = steps
        width = max(a.shape[1] for a in allows)
        outs[f"dec_bs{bs}_allow"] = torch.stack(
            [torch.nn.functional.pad(a, (0, width - a.shape[1])) for a in allows])
        outs[f"dec_bs{bs}_nblk"] = np.array([a.shape[1] for a in allows])
    save("page_gate", **outs)


def case_page_rope(m):
    """page2d RoPE: _build_page_rope_pos (+ _page_rope_offsets, span 0 / 64),
    DeepseekV2IndexerRotary2D.forward (bf16 and fp32 tables, two configs),
    the rotary application of the DASH router, and the decode branch of
    SlidingWindowLlamaAttention._main_rope_coords."""
    base = importlib.import_module("uocr_ref._sparse_base_impl")
    Ix, Rot, Attn = base.DeepseekV2Indexer, base.DeepseekV2IndexerRotary2D, base.SlidingWindowLlamaAttention
    g = torch.Generator().manual_seed(31)
    rows = page_gate_rows(g, 7)
    # marker-mode rows only (the reference bails on a batch with a row without
    # prompt markers): row 0, row 2, and a row whose response has more pages
    # than its prompt
    r3 = [0] + [PAGE_MARK] + [PAGE_IMG] * 40 + [PAGE_MARK] + [PAGE_IMG] * 33 + [5] * 30
    for _ in range(8):
        r3 += [PAGE_MARK] + [9] * int(torch.randint(5, 40, (1,), generator=g))
    S = max(rows.shape[1], len(r3))
    ids = torch.full((3, S), 7, dtype=torch.long)
    ids[0, :rows.shape[1]] = rows[0]
    ids[1, :rows.shape[1]] = rows[2]
    ids[2, :len(r3)] = torch.tensor(r3)
    outs = dict(ids=ids, bail_ids=rows[:2].clone(), text_ids=rows[3:].clone())

    def indexer(span):
        rot = Rot(128, 10000.0, 256.0, 1, tok_freq_mode="resample", page_mod=2)
        ns = types.SimpleNamespace(image_token_id=PAGE_IMG, page_token_id=PAGE_MARK, rope_page_span=span,
                                   rotary_emb_2d=rot, layer_idx=0, _page_rope_diag_logged=True,
                                   _page_rope_bail_logged=True,
                                   q_proj=types.SimpleNamespace(weight=torch.zeros(1)))
        for fn in ("_build_page_rope_pos", "_page_rope_offsets", "_page_rope_bail"):
            setattr(ns, fn, types.MethodType(getattr(Ix, fn), ns))
        return ns

    for span in (0, 64):
        for tag, kl in (("full", S), ("trunc", S - 20), ("pad", S + 30)):
            ix = indexer(span)
            tok, page = ix._build_page_rope_pos(ids, kl)
            outs[f"tok_sp{span}_{tag}"], outs[f"page_sp{span}_{tag}"] = tok, page
            outs[f"pfcnt_sp{span}_{tag}"] = ix._page_rope_meta["pf_cnt"]
    outs["bail"] = np.array([indexer(0)._build_page_rope_pos(outs["bail_ids"], S) is None,
                             indexer(0)._build_page_rope_pos(outs["text_ids"], S) is None])
    # rotary tables (two configs, bf16 and fp32) and the router's application
    # (tables at every 5th position, first half only: the second repeats it;
    # bf16 values stored as their 16-bit patterns)
    tok, page = outs["tok_sp0_full"], outs["page_sp0_full"]
    sub = torch.arange(0, S, 5)
    b16 = lambda x: x.contiguous().view(torch.int16)  # noqa: E731
    outs["rot_sub"] = sub
    for ci, (bt, bp, pairs, mode, pmod) in enumerate(((10000.0, 256.0, 1, "resample", 2),
                                                      (500000.0, 256.0, 8, "truncate", 0))):
        rot = Rot(128, bt, bp, pairs, tok_freq_mode=mode, page_mod=pmod)
        outs[f"rot{ci}_inv_tok"], outs[f"rot{ci}_inv_page"] = rot.inv_tok.clone(), rot.inv_page.clone()
        for dt in (torch.bfloat16, torch.float32):
            cos, sin = rot(torch.zeros(1, dtype=dt), tok, page)
            cos, sin = cos[:, sub, :64], sin[:, sub, :64]
            if dt == torch.bfloat16:
                outs[f"rot{ci}_cos_bf16"], outs[f"rot{ci}_sin_bf16"] = b16(cos), b16(sin)
            else:
                outs[f"rot{ci}_cos_f32"], outs[f"rot{ci}_sin_f32"] = cos, sin
    cos, sin = Rot(128, 10000.0, 256.0, 1, tok_freq_mode="resample", page_mod=2)(
        torch.zeros(1, dtype=torch.bfloat16), tok, page)
    P = 200                                  # the router's application on the first 200 positions
    qx = torch.randn(3, 2, P, 128, generator=g).to(torch.bfloat16)
    kx = torch.randn(3, 1, P, 128, generator=g).to(torch.bfloat16)
    qe, ke = base._llama_apply_rotary_pos_emb(qx, kx, cos[:, :P], sin[:, :P])
    outs.update(qx=b16(qx), kx=b16(kx), qe=b16(qe), ke=b16(ke))
    # decode coordinates: prefill state, then 20 tokens (markers at steps 3, 9, 10)
    ix = indexer(0)
    attn = types.SimpleNamespace(indexer=ix, layer_idx=0, _main_rope_pos_2d=None, _sparse_source_input_ids=ids)
    kv = types.SimpleNamespace()
    coords = Attn._main_rope_coords(attn, S, kv)
    st0 = kv._page_rope_state[0]
    outs.update(dec_page0=st0["page"].clone(), dec_tok0=st0["tok"].clone(), dec_pfcnt=st0["pf_cnt"],
                dec_npg=np.array(st0["n_pg"]))
    steps = torch.randint(0, 1000, (3, 20), generator=g)
    steps[:, 3] = PAGE_MARK
    steps[0, 9] = PAGE_MARK
    steps[1, 10] = PAGE_MARK
    steps[2, 9:15] = PAGE_MARK           # past the last page: clamped to n_pg - 1
    toks, pages = [], []
    for k_ in range(steps.shape[1]):
        attn._sparse_source_input_ids = steps[:, k_:k_ + 1]
        t_, p_ = Attn._main_rope_coords(attn, 1, kv)
        toks.append(t_[:, 0].clone())
        pages.append(p_[:, 0].clone())
    outs.update(dec_steps=steps, dec_tok=torch.stack(toks), dec_page=torch.stack(pages))
    save("page_rope", **outs)


# cases run on the SGLang ops of the wheel; all others on the HF modules
_SGL_CASES = {"paged", "paged_prefill"}
_ORDER = ("route", "entmax", "decode_attend", "forward_dense", "gather_triton", "gather_e2e", "block_max",
          "paged", "paged_prefill", "page_gate", "page_rope", "gather_kl")


def main():
    if not REF or not os.path.isdir(REF):
        sys.exit("set SRSWA_REFERENCE to a checkout of the reference (hf-model-code/ and wheel/ inside)")
    names = sys.argv[1:] or list(_ORDER)   # e.g. `make_golden.py page_gate` regenerates one case
    m = import_reference()
    sgl = import_sglang_ops() if any(n in _SGL_CASES for n in names) else None
    torch.manual_seed(0)
    for name in names:
        globals()[f"case_{name}"](sgl if name in _SGL_CASES else m)


if __name__ == "__main__":
    main()
