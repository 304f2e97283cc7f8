#!/usr/bin/env python
"""SR-SWA decode benchmark on 1..8 B200s.

One step = one SR-SWA decode step of every request in the batch:
  k_bar tail-page refresh (a1) -> fused scores + top-M entmax + top-K + bias
  over the paged k_bar cache (a2+a4) -> block-sparse paged attend of the
  selected blocks + the 512-token window (a9),
for 256 concurrent requests with S_r ~ U[16384, 131072] (seeded), page = block
= 64 tokens, 10 heads x 128, index dim 128, K = 8, M = 16, LW = 512.  Requests
are sharded across ranks (greedy balance of sum S_r); no collective on the
data path (strong scaling: the 256 requests are split).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl srswa|reference]

`value` = algorithmic HBM bytes of all ranks' steps / (max-over-ranks device
time per step), GB/s.  Algorithmic bytes per step: the unique attended keys'
K and V rows (Hkv*D*2 B each), the k_bar rows of every remote candidate block
(d*4 B), block-table entries, the refreshed tail pages, q and the outputs.
The KV cache is resident (~100 GB at N=1); L2 is flushed between timed steps.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "unlimited-ocr_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = json.load(open(os.path.join(ROOT, "BASELINE.json")))["metric"]
BS, H, HKV, D, DI, L, K, M = 64, 10, 10, 128, 128, 8, 8, 16
IDX_SCALE, FLOOR, SIGMA = 128.0 / math.sqrt(DI), 1e-4, 1.0
SM_SCALE = 1.0 / math.sqrt(D)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="srswa", choices=["srswa", "reference"])
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--smin", type=int, default=16384)
    ap.add_argument("--smax", type=int, default=131072)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="decode: skip the cfg2 / cfg4 / cfg5 results that ride along in the line")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "train", "route", "longctx", "pagegate", "rope", "kl",
                                                     "paged-prefill"],
                    help="decode = cfg3 (default, the headline); prefill = cfg2; train = cfg4 fwd+bwd; "
                         "route = the cfg3 router alone (k_bar cache + block table, no KV; for profiling); "
                         "longctx = cfg5 attention share (12 layers, one 1M-token sequence, split-KV); "
                         "pagegate = PageGate candidate masks of a cfg2-shaped prefill; "
                         "rope = page2d RoPE coordinates + fused rotary of a cfg2-shaped prefill; "
                         "paged-prefill = SGLang extend: route_prefill_triton + dash_sparse_attn (K8)")
    ap.add_argument("--layers", type=int, default=12, help="longctx: decoder layers")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "p2p-flag", "p2p-launch", "nccl"],
                    help="longctx with N > 1: peer-memory exchange fused into the router / attend / merge "
                         "kernels with LL words (default) or with flags, the flag exchange as separate push + "
                         "wait launches, or NCCL all-gathers")
    ap.add_argument("--batch", type=int, default=0, help="prefill/train batch override (smaller cases)")
    ap.add_argument("--seq", type=int, default=0, help="prefill/train sequence override")
    return ap.parse_args()


# ---------------------------------------------------------------------------
def workload(args):
    """Seeded request lengths (drawn first from the seed-2 generator)."""
    g = torch.Generator().manual_seed(2)
    S = torch.randint(args.smin, args.smax + 1, (args.requests,), generator=g).tolist()
    return S, g


def request_cost(s):
    """Algorithmic bytes of one request's decode step: the attend reads about
    the same keys for every request (the window + K selected blocks, K and V
    of every kv head), the router one k_bar row and one block-table entry per
    remote candidate block (O(S_r))."""
    attend = (L * BS + K * BS) * HKV * D * 2 * 2
    route = max(0, (s - 1) // BS - L + 1) * (DI * 4 + 4)
    return attend + route


def shard(S, world):
    """Greedy balance (largest first) of the per-request step cost over ranks:
    request counts stay even (the attend's constant part dominates) and the
    router's O(S_r) part is spread."""
    cost = [request_cost(s) for s in S]
    order = sorted(range(len(S)), key=lambda i: -cost[i])
    load = [0] * world
    parts = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], len(parts[j])))
        parts[r].append(i)
        load[r] += cost[i]
    return [sorted(p) for p in parts]


def step_bytes(S_local, topi):
    """Algorithmic bytes of one decode step for these requests, counted from
    the emitted selection topi [R, K] (int32, -1 unused)."""
    attend = route = kbar = 0
    for r, s in enumerate(S_local):
        p = s - 1
        lws = max(0, p - L * BS + 1)
        remote = 0
        seen = set()
        for blk in topi[r].tolist():
            if blk < 0 or blk in seen:
                continue
            seen.add(blk)
            lo, hi = blk * BS, min((blk + 1) * BS, p + 1, lws)
            remote += max(0, hi - lo)
        n_keys = remote + (p + 1 - lws)
        attend += n_keys * HKV * D * 2 * 2 + 2 * H * D * 2          # K+V rows, q, out
        cand = max(0, p // BS - L + 1)
        route += cand * (DI * 4 + 4) + DI * 4 + K * 8                # k_bar rows, table, idx_q, outputs
        ntok = s - (math.ceil(s / BS) - 1) * BS
        kbar += ntok * DI * 2 + DI * 4 + 8                          # tail page keys, summary
    return attend, route, kbar


# ---------------------------------------------------------------------------
class Clocks:
    """nvidia-smi sampler for the timed region (clocks + throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-i", str(self.idx), "-lms", "50"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=10)
        except Exception:
            self.p.kill()
            return None
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def peaks():
    try:
        p = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic_ratio():
    """DRAM bytes per algorithmic byte of the attend kernel, from the committed
    ncu summary (a capture of a smaller case of the same kernel)."""
    path = os.path.join(ROOT, "profiles", "decode_attend_cfg3.txt")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_algorithmic_byte:"):
                return float(line.split(":")[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
def fill_from_pool(t, pool, gen):
    """Fill a bf16 tensor with windows of a seeded N(0,1) pool at seeded random
    offsets (generating ~100 GB of fresh normals would dominate the run)."""
    flat = t.view(-1)
    n = flat.numel()
    chunk = pool.numel() // 2
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        off = int(torch.randint(0, pool.numel() - (e - s) + 1, (1,), generator=gen))
        flat[s:e].copy_(pool[off:off + (e - s)])


def build_rank(S_local, seed, dev):
    from srswa import ops
    gen = torch.Generator().manual_seed(seed)
    nb = [math.ceil(s / BS) for s in S_local]
    R = len(S_local)
    W = max(nb)
    P = sum(nb)
    perm = torch.randperm(P, generator=gen)
    bt = torch.zeros(R, W, dtype=torch.int32)
    o = 0
    for r, n in enumerate(nb):
        bt[r, :n] = perm[o:o + n].to(torch.int32)
        o += n
    gdev = torch.Generator(device=dev).manual_seed(seed)
    pool = torch.randn(1 << 27, device=dev, dtype=torch.bfloat16, generator=gdev)
    k_cache = torch.empty(P, BS, HKV, D, device=dev, dtype=torch.bfloat16)
    v_cache = torch.empty_like(k_cache)
    idx_cache = torch.empty(P, BS, DI, device=dev, dtype=torch.bfloat16)
    for t in (k_cache, v_cache, idx_cache):
        fill_from_pool(t, pool, gen)
    del pool
    st = dict(
        bt=bt.to(dev), sl=torch.tensor(S_local, dtype=torch.int32, device=dev),
        k=k_cache, v=v_cache, idx=idx_cache,
        kbar=torch.zeros(P, DI, device=dev, dtype=torch.float32),
        hc=torch.zeros(DI, device=dev),
        q=torch.randn(R, H, D, generator=gen).to(torch.bfloat16).to(dev),
        iq=torch.randn(R, DI, generator=gen).to(torch.bfloat16).float().to(dev),
        out=torch.empty(R, H, D, device=dev, dtype=torch.bfloat16),
    )
    ops.kbar_paged(st["idx"], st["hc"], st["bt"], st["sl"], st["kbar"], tail_pages=0)   # prefill summaries
    torch.cuda.synchronize()
    return st


STEP_LAUNCHES = 5   # k_bar tail refresh, router scores, router selection, attend (last-wave rows, the rest)


def count_launches(fn, default):
    """Kernels of this library (names in the srswa namespace) that one call
    of fn launches, counted by the profiler on an untimed call; `default` if
    the profiler is unavailable."""
    try:
        from torch.autograd import DeviceType
        from torch.profiler import ProfilerActivity, profile
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        n = sum(1 for e in prof.events() if e.device_type == DeviceType.CUDA and "srswa::" in e.name)
        return n if n > 0 else default
    except Exception:
        return default


def fork_kbar_refresh(st, fn):
    """Run this step's k_bar tail-page refresh on a second stream.  The tail
    page holds the newest token, so it is inside the local window and never a
    remote candidate of this step's router: the refresh only has to land
    before the next step, and its latency-bound launch overlaps the router's
    score pass.  Returns the stream to join at the end of the step."""
    main = torch.cuda.current_stream()
    side = st.setdefault("side", torch.cuda.Stream())
    side.wait_stream(main)
    with torch.cuda.stream(side):
        fn()
    return side


def run_step(st):
    """One decode step through the library (device-resident inputs)."""
    from srswa import ops
    side = fork_kbar_refresh(st, lambda: ops.kbar_paged(st["idx"], st["hc"], st["bt"], st["sl"], st["kbar"],
                                                        tail_pages=1))
    r = ops.route(st["iq"], st["kbar"], block_size=BS, local_blocks=L, topk=K, topm=M, idx_scale=IDX_SCALE,
                  floor=FLOOR, sigma=SIGMA, seq_lens=st["sl"], block_table=st["bt"], want=("topi32", "bias"))
    st["topi"], st["bias"] = r["topi32"], r["bias"]
    run_attend(st, overlap=True)   # starts on the window keys while the router finishes
    torch.cuda.current_stream().wait_stream(side)


def run_step_public(st, q, iq, kv_ready=None, before_refresh=None):
    """The same decode step through the public paged API (SGLang signatures):
    kbar_refresh_tail, route_decode, dash_sparse_attn_decode.  kv_ready: a
    stream whose work (q and the new K/V rows) the attend must wait for;
    before_refresh: work the k_bar refresh depends on (the new index-key row),
    run on the refresh's stream."""
    from srswa import paged
    if "idx_buf" not in st:   # K slots wide: route_decode writes them in place
        st["idx_buf"] = torch.empty(q.shape[0], K, dtype=torch.int32, device=q.device)
        st["bias_buf"] = torch.empty(q.shape[0], K, dtype=torch.float32, device=q.device)
    def refresh():
        if before_refresh is not None:
            before_refresh()
        paged.kbar_refresh_tail(kv_cache=st["idx"], k_bar=st["kbar"], block_table=st["bt"], seq_lens=st["sl"],
                                head_cls=st["hc"], block_size=BS, tail_pages=1)

    side = fork_kbar_refresh(st, refresh)
    w = paged.route_decode(idx_q=iq, k_bar=st["kbar"], block_table=st["bt"], seq_lens=st["sl"], image_allow=None,
                           out_idx=st["idx_buf"], out_bias=st["bias_buf"], max_block=st["bt"].shape[1],
                           block_size=BS, local_blocks=L, decode_query_len=1, idx_scale=IDX_SCALE,
                           prior_floor=FLOOR, sigma=SIGMA, topm=M, budget=K)
    ti = st["idx_buf"][:, :w].unsqueeze(0).expand(HKV, -1, -1)
    tb = st["bias_buf"][:, :w].unsqueeze(0).expand(HKV, -1, -1)
    if kv_ready is not None:
        torch.cuda.current_stream().wait_stream(kv_ready)
    paged.dash_sparse_attn_decode(q, st["k"], st["v"], ti, tb, st["bt"], st["sl"], HKV, SM_SCALE, st["out"], 1,
                                  local_blocks=L, sparse_block_size=BS, overlap_router=True)
    torch.cuda.current_stream().wait_stream(side)


def run_attend(st, overlap=False):
    from srswa import ops
    ops.decode_attend(st["q"], st["k"], st["v"], st["topi"], st["bias"], block_size=BS, local_blocks=L,
                      sm_scale=SM_SCALE, out=st["out"], block_table=st["bt"], seq_lens=st["sl"], overlap=overlap)


def timed_graph(fn, steps, warmup, flush, use_graph=True):
    """Per-step device times (ms) of fn, L2 flushed before each step."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(max(warmup, 1)):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = None
    if use_graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        torch.cuda.synchronize()
    run = g.replay if g is not None else fn
    for _ in range(max(warmup, 1)):
        run()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for a, b in ev:
        flush.zero_()
        a.record()
        run()
        b.record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev], g


# ---------------------------------------------------------------------------
def cpu_decode_sample(S, budget_s=20.0, max_req=4):
    """The reference's CPU decode step (_block_scores_infer ->
    _infer_route_select -> _decode_attend: summaries of every block, scores,
    selection, dense masked attend over the whole cache; fp32 torch on all
    host cores, oracle/torch_cpu.py) on a bounded sample of the workload's
    requests.  Returns (GB/s of the step's algorithmic bytes, host info,
    sample, seconds)."""
    from oracle import torch_cpu as TC
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(2)
    t_all, bytes_all, lens = 0.0, 0, []
    for s_ in S[:max_req]:
        q = torch.randn(1, H, 1, D, generator=g)
        k = torch.randn(1, HKV, s_, D, generator=g)
        v = torch.randn(1, HKV, s_, D, generator=g)
        iq = torch.randn(1, 1, DI, generator=g)
        ik = torch.randn(1, s_, DI, generator=g)
        pos = torch.tensor([[s_ - 1]])
        TC.decode_step(q, k, v, iq, ik, torch.zeros(DI), pos, BS, L, K, M, IDX_SCALE, FLOOR, SIGMA, SM_SCALE)
        t0 = time.perf_counter()
        _, topi, valid = TC.decode_step(q, k, v, iq, ik, torch.zeros(DI), pos, BS, L, K, M, IDX_SCALE, FLOOR,
                                        SIGMA, SM_SCALE)
        t_all += time.perf_counter() - t0
        sel = torch.where(valid[0, 0], topi[0, 0], torch.full_like(topi[0, 0], -1))[None].to(torch.int32)
        a, r_, kk = step_bytes([s_], sel)
        bytes_all += a + r_ + kk
        lens.append(s_)
        if t_all > budget_s:
            break
    return bytes_all / t_all / 1e9, TC.host_info(), lens, t_all


def cpu_cfg1_ms(reps=20):
    """BASELINE config 1 on the host: one fp32 decode step, B=1, S=8192
    (32 pages x 256 tokens), seed 0, through the same CPU path."""
    from oracle import torch_cpu as TC
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    S0 = 8192
    q, k, v = (torch.randn(1, H, n, D, generator=g) for n in (1, S0, S0))
    iq, ik = torch.randn(1, 1, DI, generator=g), torch.randn(1, S0, DI, generator=g)
    pos = torch.tensor([[S0 - 1]])
    args = (q, k, v, iq, ik, torch.zeros(DI), pos, BS, L, K, M, IDX_SCALE, FLOOR, SIGMA, SM_SCALE)
    TC.decode_step(*args)
    t0 = time.perf_counter()
    for _ in range(reps):
        TC.decode_step(*args)
    return (time.perf_counter() - t0) / reps * 1e3


# ---------------------------------------------------------------------------
def attend_flops(T, LW, sel, BS, t0=0):
    """Exact forward flops of the gather-attention: 4*D per (query, head,
    attended key); attended keys = window + unique remote keys of the
    selection (sel [B, T - t0, K] int for queries t0 .. T-1, -1 unused)."""
    B = sel.shape[0]
    t = torch.arange(t0, T, device=sel.device)
    ls = (t - LW + 1).clamp(min=0)
    n = (t - ls + 1).to(torch.float64).sum() * B
    s = sel.clone()
    valid = s >= 0
    lo = s * BS
    hi = torch.minimum(torch.minimum((s + 1) * BS, (t + 1)[None, :, None]), ls[None, :, None])
    cnt = (hi - lo).clamp(min=0) * valid
    # repeated ids were removed by the router (distinct top-k)
    n = n + cnt.to(torch.float64).sum()
    return float(n) * 4 * D * H


def init_dist(dev, world):
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)


def rank_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def bf16_peak():
    try:
        pk = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(pk["bf16_tflops"]) * 1e12, "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except Exception:
        return 1.59e15, "fallback 1.59 PFLOP/s"


def dense_setup(train, B, T, rank, dev):
    """cfg2 / cfg4 inputs as the benchmark draws them (seeded N(0,1) * scale,
    bf16) and the router's selection of them (head_cls = 0)."""
    from srswa import dash_infer
    Kk, LW, seed, sc = (16, 1024, 3, 1.0) if train else (8, 512, 1, 0.5)
    g = torch.Generator(device=dev).manual_seed(seed * 100 + rank)
    mk = lambda *shape: (torch.randn(*shape, device=dev, generator=g) * sc).to(torch.bfloat16)  # noqa: E731
    x = dict(q=mk(B, H, T, D), k=mk(B, HKV, T, D), v=mk(B, HKV, T, D))
    x["iq"] = mk(B, T, DI).float()
    x["ik"] = mk(B, T, DI)
    # upstream gradient in the memory layout a model's o_proj hands back
    # (attn_output.transpose(1, 2).reshape(B, T, H * D) -> [B, T, H, D] memory)
    x["do"] = (torch.randn(B, T, H, D, device=dev, generator=g).to(torch.bfloat16).transpose(1, 2)
               if train else None)
    x["router"] = type("R", (), dict(block_size=BS, local_blocks=LW // BS, local_window=LW,
                                     head_cls=torch.zeros(DI, device=dev), stage0="head_cls"))()
    x["pos"] = torch.arange(T, device=dev)[None].expand(B, T).contiguous()
    x["p"] = dict(idx_scale=IDX_SCALE, floor=FLOOR, sigma=SIGMA, K=Kk, topm=M)
    x.update(K=Kk, LW=LW, nblk=T // BS, dash_infer=dash_infer)
    return x


def dense_step(x, train, q=None, k=None, v=None, iq=None, ik=None, do=None, outs=None):
    """One cfg2 / cfg4 step through the public drop-ins: route
    (_block_scores_infer + _infer_route_select fused) -> triton_gather_attention_e2e
    forward (and backward with autograd for cfg4)."""
    from srswa.sparse_gather_e2e import triton_gather_attention_e2e
    q = x["q"] if q is None else q
    k = x["k"] if k is None else k
    v = x["v"] if v is None else v
    iq = x["iq"] if iq is None else iq
    ik = x["ik"] if ik is None else ik
    topi, bias, valid = x["dash_infer"].route(x["router"], iq, ik, x["pos"], x["nblk"], None, x["p"])
    sel = torch.where(valid, topi, torch.full_like(topi, -1))[:, None]
    b = (bias * valid).float()
    if train:
        qq, kk, vv, bb = (t.detach().requires_grad_(True) for t in (q, k, v, b))
        o = triton_gather_attention_e2e(qq, kk, vv, sel, bb, x["pos"], None, BS, SM_SCALE, x["LW"])
        o.backward(x["do"] if do is None else do)
        res = (o, qq.grad, kk.grad, vv.grad)
    else:
        o = triton_gather_attention_e2e(q, k, v, sel, b, x["pos"], None, BS, SM_SCALE, x["LW"])
        res = (o,)
    x["sel"], x["b"] = sel, b
    if outs is not None:
        for dst, src in zip(outs, res):
            dst.copy_(src, non_blocking=True)
    return res


def dense_check(x, train, res):
    """Correctness of the timed workload, outside the timed region: a few
    query rows of the first and last batch element (o, and dQ for cfg4)
    against the CPU oracle on the same bf16 values and selection."""
    from oracle import srswa_oracle as O
    T, LW = x["q"].shape[2], x["LW"]
    rows = np.array([0, BS, LW, T // 2 + 7, T - 1])
    err, worst = 0.0, 0.0
    for bi in (0, x["q"].shape[0] - 1):
        qb, kb, vb = (t[bi].transpose(0, 1).float().cpu().numpy() for t in (x["q"], x["k"], x["v"]))
        sel = x["sel"][bi, 0].cpu().numpy()
        bias = x["b"][bi].cpu().numpy()
        seg = np.zeros(T, np.int64)
        o_r, _ = O.gather_rows_fwd(qb, kb, vb, sel, seg, rows, BS, SM_SCALE, LW, bias)
        got = res[0][bi][:, rows].transpose(0, 1).detach().float().cpu().numpy()
        d = np.abs(got - o_r)
        err = max(err, float(d.max()))
        worst = max(worst, float((d / (2e-2 + 1e-2 * np.abs(o_r))).max()))
        if train:
            dob = x["do"][bi].transpose(0, 1).float().cpu().numpy()
            dq_r, _ = O.gather_rows_bwd(qb, kb, vb, dob, sel, seg, rows, BS, SM_SCALE, LW, bias)
            got = res[1][bi][:, rows].transpose(0, 1).detach().float().cpu().numpy()
            d = np.abs(got - dq_r)
            err = max(err, float(d.max()))
            worst = max(worst, float((d / (2e-2 + 1e-2 * np.abs(dq_r))).max()))
    ok = worst <= 1.0
    if not ok:
        raise SystemExit(f"bench correctness check failed: max abs err {err} (tolerance ratio {worst})")
    return {"rows": int(len(rows) * 2), "outputs": "o, dq" if train else "o", "max_abs_err": err,
            "tolerance": "2e-2 abs + 1e-2 rel vs the CPU oracle", "ok": ok}


def dense_cpu_baseline(x, train, budget_rows):
    """The reference's CPU path on a sub-slice of batch element 0: routing of
    the last `budget_rows` queries (block summaries of every block, scores,
    selection) and DashAttention._forward_dense for them, fp32 on the host
    cores (oracle/torch_cpu.py restates the reference's torch ops); cfg4 adds
    the autograd backward.  Reported as TFLOP/s of the same attended work."""
    from oracle import torch_cpu as TC
    torch.set_num_threads(os.cpu_count() or 1)
    T, LW, Kk = x["q"].shape[2], x["LW"], x["K"]
    q0 = T - budget_rows
    q, k, v = (t[:1].float().cpu() for t in (x["q"], x["k"], x["v"]))
    iq, ik = x["iq"][:1].float().cpu(), x["ik"][:1].float().cpu()
    pos = torch.arange(T)[None]
    t0 = time.perf_counter()
    with torch.set_grad_enabled(train):
        sc = TC.block_scores(iq[:, q0:], ik, torch.zeros(DI), pos[:, q0:], BS, LW // BS)
        topi, bias, valid = TC.route_select(sc, None, IDX_SCALE, FLOOR, SIGMA, Kk, M)
        full = lambda t_, fill: torch.cat([torch.full((1, q0, t_.shape[-1]), fill, dtype=t_.dtype), t_], 1)  # noqa
        topi, bias, valid = full(topi, 0), full(bias, 0.0), full(valid, False)
        if train:
            q, k, v, bias = (t_.requires_grad_(True) for t_ in (q, k, v, bias))
        o = TC.dense_forward(q, k, v, topi, bias, valid, BS, LW, SM_SCALE, q_start=q0)
        if train:
            o.backward(torch.ones_like(o))
    dt = time.perf_counter() - t0
    sel = torch.where(valid[:, q0:], topi[:, q0:], torch.full_like(topi[:, q0:], -1))
    fl = attend_flops(T, LW, sel, BS, t0=q0) * (3.5 if train else 1.0)
    info = __import__("oracle.torch_cpu", fromlist=["host_info"]).host_info()
    return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "cores": info["threads"], "kind": "port",
            "cpu_model": info["cpu_model"], "seconds": dt,
            "sample": f"batch element 0, last {budget_rows} of {T} queries (all {T} keys): routing + "
                      f"_forward_dense{' + autograd backward' if train else ''}, fp32 torch on the host cores"}


def dense_e2e(x, train, steps, warmup):
    """The step through the public API from pinned host buffers: H2D of the
    step's inputs (q, k, v, idx_q, idx_k; dO for cfg4), the step, D2H of its
    results (o; dq, dk, dv for cfg4), every step."""
    dev = x["q"].device
    names = ["q", "k", "v", "iq", "ik"] + (["do"] if train else [])
    # dO travels in the memory layout it has on the device ([B, T, H, D])
    src = {n: (x[n].transpose(1, 2) if n == "do" else x[n]) for n in names}
    host = {n: torch.empty(src[n].shape, dtype=src[n].dtype).pin_memory() for n in names}
    for n in names:
        host[n].copy_(src[n])
    devb = {n: torch.empty(src[n].shape, dtype=src[n].dtype, device=dev) for n in names}
    out_shapes = [x["q"].shape] + ([x["q"].shape, x["k"].shape, x["v"].shape] if train else [])
    houts = [torch.empty(s_, dtype=torch.bfloat16).pin_memory() for s_ in out_shapes]
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = sum(t.numel() * t.element_size() for t in houts)

    def step():
        for n in names:
            devb[n].copy_(host[n], non_blocking=True)
        res = dense_step(x, train, q=devb["q"], k=devb["k"], v=devb["v"], iq=devb["iq"], ik=devb["ik"],
                         do=devb["do"].transpose(1, 2) if train else None)
        for dst, src in zip(houts, res):
            dst.copy_(src, non_blocking=True)

    for _ in range(max(warmup, 1)):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, h2d, d2h


def dense_measure(args, train, extras=True):
    """cfg2 prefill (route + gather fwd) or cfg4 training (route + gather fwd
    + bwd), one GPU per rank, batch sharded across ranks (weak: per-rank work
    fixed).  Returns this workload's result dict (rank 0) or None."""
    import torch.distributed as dist
    world, rank, local = rank_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_dist(dev, world)
    B, T = (8, 32768) if train else (4, 16384)
    if args.batch:
        B = args.batch
    if args.seq:
        T = args.seq
    Bl = max(1, B // world)
    x = dense_setup(train, Bl, T, rank, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for _ in range(max(args.warmup, 3)):
        res = dense_step(x, train)
    torch.cuda.synchronize()
    check = dense_check(x, train, res) if (extras and rank == 0) else None
    del res
    fl = attend_flops(T, x["LW"], x["sel"][:, 0], BS) * (3.5 if train else 1.0)  # fwd 4, bwd 10 per D
    if world > 1:
        dist.barrier()
    clocks = Clocks(local)
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a_, b_ in ev:
        flush.zero_()
        a_.record()
        dense_step(x, train)
        b_.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = sum(a_.elapsed_time(b_) for a_, b_ in ev) / args.steps
    e2e_ms, h2d, d2h = dense_e2e(x, train, args.steps, args.warmup) if extras else (0.0, 0, 0)
    vec = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
    tot = torch.tensor([fl, h2d, d2h], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vec, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    ms, e2e_ms = vec.tolist()
    fl_all, h2d, d2h = tot.tolist()
    cpu = None
    if extras and rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = dense_cpu_baseline(x, train, 256 if train else 2048)
    peak, src = bf16_peak()
    del x
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    out = {"value": fl_all / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "n_gpus": world,
           "steps": args.steps, "scaling": "weak", "dtype": "bf16",
           "config": {"workload": ("cfg4 train: route + gather-attention e2e fwd+bwd" if train else
                                   "cfg2 prefill: route + gather-attention fwd"),
                      "global_batch": Bl * world, "seq_len": T, "K": x_k(train), "LW": 1024 if train else 512,
                      "parallelism": f"batch/dp{world}", "l2": "flushed before every timed step",
                      "flops_per_step": fl_all,
                      **({"dO_layout": "[B,T,H,D] memory (as from o_proj)"} if train else {})},
           "roofline": {"bound": "tensor", "achieved": fl_all / world / (ms * 1e-3) / 1e12, "peak": peak / 1e12,
                        "unit": "TFLOP/s", "frac": fl_all / world / (ms * 1e-3) / peak, "peak_source": src,
                        "traffic": None},
           "clocks": clk}
    if extras:
        out["check"] = check
        out["cpu_baseline"] = cpu
        out["e2e"] = {"value": fl_all / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                      "how": "pinned H2D of q, k, v, idx_q, idx_k" + (", dO" if train else "") +
                             " -> route + triton_gather_attention_e2e" + (" fwd + bwd" if train else "") +
                             " -> D2H of o" + (", dq, dk, dv" if train else "") + ", every step",
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
    return out


def x_k(train):
    return 16 if train else 8


def main_dense(args):
    world, rank, _ = rank_env()
    r = dense_measure(args, args.workload == "train")
    if rank == 0:
        line = {"metric": METRIC, **r, "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
                "data": "synthetic seeded N(0,1)"}
        line["n_gpus"] = world
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main_route(args):
    """The cfg3 decode router alone (fused scores + selection over the paged
    k_bar cache of 256 requests), for profiling at full size without the KV."""
    from srswa import ops
    dev = torch.device("cuda", 0)
    S, _ = workload(args)
    gen = torch.Generator().manual_seed(1000)
    nb = [math.ceil(s / BS) for s in S]
    R, W, P = len(S), max(nb), sum(nb)
    perm = torch.randperm(P, generator=gen)
    bt = torch.zeros(R, W, dtype=torch.int32)
    o = 0
    for r, n in enumerate(nb):
        bt[r, :n] = perm[o:o + n].to(torch.int32)
        o += n
    bt, sl = bt.to(dev), torch.tensor(S, dtype=torch.int32, device=dev)
    kbar = torch.randn(P, DI, generator=gen).to(dev) * 0.1
    iq = torch.randn(R, DI, generator=gen).to(torch.bfloat16).float().to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    fn = lambda: ops.route(iq, kbar, block_size=BS, local_blocks=L, topk=K, topm=M, idx_scale=IDX_SCALE,  # noqa: E731
                           floor=FLOOR, sigma=SIGMA, seq_lens=sl, block_table=bt, want=("topi32", "bias"))
    times, g = timed_graph(fn, args.steps, args.warmup, flush, not args.no_graph)
    ms = sum(times) / len(times)
    byts = sum(max(0, (s - 1) // BS - L + 1) * (DI * 4 + 4) + DI * 4 + K * 8 for s in S)
    print(json.dumps({"workload": "cfg3 router alone", "us": ms * 1e3, "bytes": byts,
                      "GB/s": byts / (ms * 1e-3) / 1e9}), flush=True)
    del g
    return 0


def page_doc(B, T, seed, per_page=273, img=128815, mark=128827):
    """Seeded document token rows: <PAGE> + per_page image tokens + a few text
    tokens per prompt page (Base mode), an instruction, then <PAGE>-marked
    response pages of 200-600 text tokens."""
    rng = np.random.default_rng(seed)
    out = np.full((B, T), 5, np.int64)
    for b in range(B):
        r = [0]
        while len(r) < T * 0.6:
            r += [mark] + [img] * per_page + list(rng.integers(0, 1000, int(rng.integers(2, 8))))
        r += list(rng.integers(0, 1000, 60))
        while len(r) < T:
            r += [mark] + list(rng.integers(0, 1000, int(rng.integers(200, 600))))
        out[b] = np.asarray(r[:T])
    return out


def main_kl(args):
    """DSA gather-KL distillation (srswa.dsa.gather_kl, the select_and_kl_loss
    KL of the reference's sparse stage) forward + backward at the cfg4 per-
    element shape: T = 32768 rows, index d = 128, main H = Hkv = 10 x 128,
    16 selected 64-token blocks per row below a 1024-token window.  The
    selection is seeded random blocks of each row's remote range (the
    router's output stands in).  The kernels gather the selected keys' index
    and main rows from L2 (idx_k + k_main = 92 MB here): the figure is the
    gathered bytes per second, bound by L2, not HBM.  One GPU (each rank its
    own copy under torchrun)."""
    from srswa import dsa
    world, rank, local = rank_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_dist(dev, world)
    T_ = args.seq or 32768
    H_, Dm, d_, BS_, LW_, S_ = 10, 128, 128, 64, 1024, 16
    g = torch.Generator(device=dev).manual_seed(7 + rank)
    iq = (torch.randn(1, T_, d_, device=dev, generator=g) * 0.08).to(torch.bfloat16).requires_grad_(True)
    ik = torch.randn(1, T_, d_, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
    qm = torch.randn(1, T_, H_, Dm, device=dev, generator=g).to(torch.bfloat16)
    km = torch.randn(1, T_, H_, Dm, device=dev, generator=g).to(torch.bfloat16)
    pos = torch.arange(T_, device=dev)[None]
    nrem = ((pos - LW_ + 1).clamp(min=0) // BS_)                     # remote blocks of each row: [0, nrem)
    r = torch.rand(1, T_, S_, device=dev, generator=g)
    sel = (r * nrem[..., None]).long()
    sel = torch.where(torch.arange(S_, device=dev) < nrem[..., None], sel, torch.full_like(sel, -1)).to(torch.int32)
    gout = torch.randn(1, T_, device=dev, generator=g)
    kept = int(((sel >= 0).sum()).item()) * BS_                       # gathered keys (upper bound: repeats)

    def step():
        iq.grad = None
        ik.grad = None
        kl, _ = dsa.gather_kl(iq, ik, qm, km, sel, pos, block_size=BS_, local_window=LW_, scaling=1 / math.sqrt(Dm))
        kl.backward(gout)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    clocks = Clocks(local)
    clocks.start()
    times, g_ = timed_graph(step, args.steps, max(args.warmup, 3), flush, False)
    clk = clocks.stop()
    ms = sum(times) / len(times)
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    # gathered bytes: forward reads each kept key's index row and its main
    # rows of every head; the backward reads them again and writes a logit
    # gradient per key slot
    byts = kept * (d_ + H_ * Dm) * 2 * 2 + kept * 4
    if rank == 0:
        print(json.dumps({"metric": "DSA gather-KL forward + backward (cfg4 shape)", "value": T_ * world / (ms * 1e-3),
                          "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
                          "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "bf16", "data": "synthetic seeded N(0,1), seeded random remote selections",
                          "config": {"workload": "gather-KL fwd+bwd", "rows": T_, "heads": H_, "head_dim": Dm,
                                     "index_dim": d_, "blocks_per_row": S_, "block": BS_, "window": LW_,
                                     "l2": "flushed before every timed step (the gathered rows then stay in L2)"},
                          "gathered_gb_s": byts / (ms * 1e-3) / 1e9, "bound": "L2 gather", "clocks": clk}),
              flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main_pagegate(args):
    """PageGate candidate masks for a prefill of cfg2's shape (B=4, T=16384,
    block 64): page-aware ids -> block descriptors -> per-query candidate
    mask [B, T, nblk], the router's input.  HBM-bound (the mask write)."""
    from srswa import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, T = (args.batch or 4), (args.seq or 16384)
    nblk = T // BS
    ids_np = page_doc(B, T, 5)
    ids = torch.from_numpy(ids_np).to(dev)
    pos = torch.arange(T, device=dev)[None].expand(B, T).contiguous()
    state = {}

    def step():
        itm, ipi, qpi, _ = ops.page_ids(ids, 128815, 128827, T, 273, True)
        desc = ops.page_block_desc(nblk, BS, ipi=ipi)
        state["cand"] = ops.page_cand_mask(desc, BS, pos=pos, qpi=qpi, ipi=ipi)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    times, g = timed_graph(step, args.steps, args.warmup, flush, not args.no_graph)
    ms = sum(times) / len(times)
    # dominant kernel alone
    itm, ipi, qpi, _ = ops.page_ids(ids, 128815, 128827, T, 273, True)
    desc = ops.page_block_desc(nblk, BS, ipi=ipi)
    out = torch.empty(B, T, nblk, device=dev, dtype=torch.bool)
    ct, g2 = timed_graph(lambda: ops.page_cand_mask(desc, BS, pos=pos, qpi=qpi, ipi=ipi, out=out),
                         args.steps, args.warmup, flush, not args.no_graph)
    cms = sum(ct) / len(ct)
    cand_bytes = B * T * nblk + B * T * 16 + B * nblk * 16          # mask write, pos + qpi reads, descriptors
    step_bytes = B * T * (8 + 8) + B * T * 17 + B * T * 8 + B * nblk * 16 + cand_bytes  # ids x2, outputs, ipi
    peak, src = peaks()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import page_gate as PG
        reps, t0 = 0, time.time()
        while reps == 0 or time.time() - t0 < 3.0:
            r_itm, r_ipi, r_qpi = PG.page_aware_ids(ids_np[:1], 128815, 128827, T, 273, True)
            ref = PG.kl_candidate_mask(np.arange(T)[None], nblk, r_itm, BS, True, r_ipi, r_qpi)
            reps += 1
        tc = (time.time() - t0) / reps
        assert (ref == state["cand"][:1].cpu().numpy()).all()
        cpu = {"value": step_bytes / B / tc / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"1 of {B} rows (numpy restatement of _build_page_aware_ids + _build_kl_candidate_mask), "
                         f"{reps} repetitions, {tc * 1e3:.1f} ms each"}
    print(json.dumps({
        "metric": "PageGate candidate masks (prefill): GB/s vs HBM", "value": step_bytes / (ms * 1e-3) / 1e9,
        "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "us_per_step": ms * 1e3, "higher_is_better": True, "dtype": "int64/u8", "data": "synthetic token ids",
        "config": {"workload": "PageGate: page ids + block descriptors + [B,T,nblk] candidate mask",
                   "global_batch": B, "seq_len": T, "block": BS, "per_page_image_tokens": 273,
                   "l2": "flushed before every timed step", "bytes_per_step": step_bytes},
        "roofline": {"bound": "hbm", "kernel": "page_cand_kernel", "achieved": cand_bytes / (cms * 1e-3) / 1e9,
                     "peak": peak, "unit": "GB/s", "frac": cand_bytes / (cms * 1e-3) / 1e9 / peak,
                     "peak_source": src, "us": cms * 1e3, "algorithmic_bytes_per_launch": cand_bytes},
        "cpu_baseline": cpu, "gpu_launches": 4 * args.steps}), flush=True)
    del g, g2
    return 0


def main_rope(args):
    """page2d RoPE of a cfg2-shaped prefill (B=4, T=16384, 10 heads x 128 and
    the single-head index projections): page-bucket coordinates from the
    token ids, then the two-axis rotary applied in place to q, k, idx_q and
    idx_k (bf16, tables rounded to bf16 as the reference casts them).
    HBM-bound: every activation is read and written once."""
    from srswa import ops
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, T = (args.batch or 4), (args.seq or 16384)
    ids = torch.from_numpy(page_doc(B, T, 5)).to(dev)
    g = torch.Generator(device=dev).manual_seed(6)
    mk = lambda h: torch.randn(B, h, T, D, device=dev, generator=g).to(torch.bfloat16)  # noqa: E731
    q, k, iq, ik = mk(H), mk(HKV), mk(1), mk(1)
    inv_tok = (1.0 / (10000.0 ** (torch.arange(63, dtype=torch.float32) / 63))).to(dev)
    inv_page = torch.ones(1, device=dev)
    state = {}

    def coords():
        tok, page, _, _ = ops.rope2d_pos(ids, 128815, 128827, T)
        state["tok"], state["page"] = tok, page

    def step():
        coords()
        for x in (q, k, iq, ik):
            ops.rope2d_apply_(x.transpose(1, 2), state["tok"], state["page"], inv_tok, inv_page, 2)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    times, g1 = timed_graph(step, args.steps, args.warmup, flush, not args.no_graph)
    ms = sum(times) / len(times)
    at, g2 = timed_graph(lambda: ops.rope2d_apply_(q.transpose(1, 2), state["tok"], state["page"], inv_tok,
                                                   inv_page, 2), args.steps, args.warmup, flush, not args.no_graph)
    ams = sum(at) / len(at)
    act = sum(x.numel() * 2 for x in (q, k, iq, ik))
    step_bytes = 2 * act + B * T * (8 * 3 + 16)          # activations read + written; ids, tok, page
    q_bytes = 2 * q.numel() * 2 + B * T * 16
    peak, src = peaks()
    print(json.dumps({
        "metric": "page2d RoPE (prefill): GB/s vs HBM", "value": step_bytes / (ms * 1e-3) / 1e9, "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "us_per_step": ms * 1e3,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic token ids and activations",
        "config": {"workload": "page2d RoPE: coordinates + fused rotary of q, k, idx_q, idx_k",
                   "global_batch": B, "seq_len": T, "heads": H, "head_dim": D,
                   "l2": "flushed before every timed step", "bytes_per_step": step_bytes},
        "roofline": {"bound": "hbm", "kernel": "rope2d_apply_kernel (q)", "achieved": q_bytes / (ams * 1e-3) / 1e9,
                     "peak": peak, "unit": "GB/s", "frac": q_bytes / (ams * 1e-3) / 1e9 / peak,
                     "peak_source": src, "us": ams * 1e3, "algorithmic_bytes_per_launch": q_bytes},
        "gpu_launches": 7 * args.steps}), flush=True)
    del g1, g2
    return 0


def main_longctx(args):
    world, rank, _ = rank_env()
    r = longctx_measure(args)
    if rank == 0:
        print(json.dumps({"metric": METRIC, **r, "warmup": max(args.warmup, 3), "higher_is_better": True,
                          "vs_baseline": None, "data": "synthetic seeded N(0,1) (pooled)"}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def longctx_measure(args):
    """cfg5 attention share: one decode step of a 1M-token sequence through
    the SR-SWA attention of 12 layers, split-KV over the ranks (rank g owns a
    contiguous block range of every layer's K/V, index keys and k_bar; the
    last rank also owns the window).  Per layer: shard router keys ->
    all-gather -> merged selection -> owned-slot attention -> all-gather of
    partials -> log-sum-exp merge; the owner of the newest page refreshes its
    k_bar.  The non-attention layers of the model (MoE, norms, LM head) are
    not part of this path."""
    import torch.distributed as dist
    from srswa import ops
    from srswa.split_kv import SplitKVDecode
    world, rank, local = rank_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_dist(dev, world)
    S0 = (args.seq if args.workload == "longctx" and args.seq else 0) or 1_048_576
    nblk_filled = S0 // BS
    nblk_total = nblk_filled + 4                     # room for 256 decoded tokens
    p = S0 - 1                                       # the step decodes the last position
    nl = args.layers
    gen = torch.Generator().manual_seed(4 * 100 + rank)
    decs, layers = [], []
    backend = None
    if world > 1 and args.exchange != "nccl":
        from srswa.split_kv import PeerBackend
        backend = PeerBackend(rows=1, topm=M, heads=H, head_dim=D,   # one for all layers
                              mode={"p2p": "ll", "p2p-flag": "flag", "p2p-launch": "launch"}[args.exchange])
    pool = torch.randn(64 << 20, generator=gen).to(torch.bfloat16).to(dev)
    hc = torch.zeros(DI, device=dev)
    for _ in range(nl):
        dec = SplitKVDecode(nblk_total=nblk_total, nblk_filled=nblk_filled, block_size=BS, local_blocks=L, topk=K,
                            topm=M, idx_scale=IDX_SCALE, floor=FLOOR, sigma=SIGMA, sm_scale=SM_SCALE, rank=rank,
                            world=world, backend=backend)
        lo, hi = dec.plan.lo, dec.plan.hi
        nloc = hi - lo
        kc = torch.empty(nloc, BS, HKV, D, device=dev, dtype=torch.bfloat16)
        vc = torch.empty_like(kc)
        ic = torch.empty(nloc, BS, DI, device=dev, dtype=torch.bfloat16)
        for t in (kc, vc, ic):
            fill_from_pool(t, pool, gen)
        filled = max(0, min(nloc, nblk_filled - lo))   # pages holding tokens on this rank
        kbar = torch.zeros(1, nloc, DI, device=dev)
        if filled:
            kbar[:, :filled] = ops.kbar_contig(ic[:filled].view(1, filled * BS, DI), hc, BS)[0]
        table = torch.zeros(1, nblk_total, device=dev, dtype=torch.int32)
        table[0, lo:hi] = torch.arange(nloc, device=dev, dtype=torch.int32)
        layers.append(dict(kbar=kbar, k_cache=kc, v_cache=vc, block_table=table, idx=ic))
        decs.append(dec)
    del pool
    qs = (torch.randn(nl, 1, H, D, generator=gen) * 0.5).to(torch.bfloat16).to(dev)
    iqs = (torch.randn(nl, 1, DI, generator=gen) * 0.5).to(torch.bfloat16).to(dev)
    q_pos = torch.tensor([p], device=dev, dtype=torch.int64)
    tail = p // BS
    own_tail = decs[0].plan.lo <= tail < decs[0].plan.hi
    t_loc = tail - decs[0].plan.lo
    outs = []
    side = torch.cuda.Stream()

    def step():
        outs.clear()
        for li in range(nl):
            lay = layers[li]
            if own_tail:   # k_bar of the page receiving the new token (read by later steps' routing)
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    ops.kbar_contig(lay["idx"][t_loc:t_loc + 1], hc, BS, out=lay["kbar"][:, t_loc:t_loc + 1],
                                    chunk_valid=False)
            outs.append(decs[li].step(qs[li], iqs[li], q_pos, lay, p_range=(p, p)))
        if own_tail:   # join the side stream only where it was forked (graph capture)
            torch.cuda.current_stream().wait_stream(side)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def waits_expired():
        """Any rank's bounded peer wait expired (collective: every rank
        decides the same way)."""
        if backend is None:
            return False
        torch.cuda.synchronize()
        bad = torch.tensor([int(int(backend.keys_x.status.item()) != 0 or int(backend.part_x.status.item()) != 0)],
                           device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)
        return bool(bad.item())

    def failed(why):
        if backend is not None:
            backend.close()            # collective: every rank
        del layers[:], decs[:], outs[:]
        torch.cuda.empty_cache()
        return None if rank != 0 else {"error": why, "n_gpus": world}

    if world > 1:
        dist.barrier()
        step()                         # one eager step first: a peer that never arrives shows here
        if waits_expired():
            return failed("a bounded peer wait expired in the first step; not timed")
    clocks = Clocks(local)
    clocks.start()
    times, g = timed_graph(step, args.steps, max(args.warmup, 3), flush, not args.no_graph)
    clk = clocks.stop()
    ms = sum(times) / len(times)
    if waits_expired():
        if g is not None:
            del g
        return failed("a bounded peer wait expired during the timed steps")
    # algorithmic bytes of this rank: k_bar of its remote-candidate blocks,
    # the K/V rows of the keys it attends (its selected blocks + the window
    # on its owner), q and o; the selection is recomputed once, untimed, with
    # the same collectives on every rank
    plan0 = decs[0].plan
    ncand = max(0, min(plan0.hi, p // BS - L + 1) - plan0.lo)
    keys_att = 0
    for li in range(nl):
        be = decs[li].backend
        kk = be.shard_keys(iqs[li], layers[li], decs[li].plan, q_pos, decs[li].rp)
        sel = be.merge_keys(be.all_gather(kk, world), decs[li].plan, decs[li].rp)
        keys_att += int((sel["topi32_own"] >= 0).sum()) * BS + (L * BS if own_tail else 0)
    byts = nl * ncand * DI * 4 + keys_att * HKV * D * 2 * 2 + nl * H * D * 2 * 2
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    b = torch.tensor([float(byts)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(b, op=dist.ReduceOp.SUM)
    ms, byts = t.item(), b.item()
    hbm = peaks()[0]
    if g is not None:
        del g
    if backend is not None:
        backend.close()            # collective: every rank (waits checked above)
    del layers, decs, outs
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {"value": byts / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "ms_per_step": ms, "us_per_step": ms * 1e3, "scaling": "strong", "dtype": "bf16",
            "config": {"workload": "cfg5 attention share: 12-layer split-KV decode, one 1M-token sequence",
                       "seq_len": S0, "layers": nl, "K": K, "LW": L * BS, "parallelism": f"split-kv{world}",
                       "exchange": ({"ll": "peer memory (CUDA IPC over NVLink), LL words stored and polled by the "
                                           "router / attend / merge kernels",
                                     "flag": "peer memory (CUDA IPC over NVLink), payload + released flags in the "
                                             "router / attend / merge kernels",
                                     "launch": "peer memory (CUDA IPC over NVLink), push + flag-wait launches"}
                                    [backend.mode]
                                    if backend is not None else ("NCCL all-gather" if world > 1 else "none")),
                       "l2": "flushed before every timed step", "graph": not args.no_graph},
            "roofline": {"bound": "latency", "achieved": byts / (ms * 1e-3) / 1e9, "peak": hbm * world,
                         "unit": "GB/s", "frac": byts / (ms * 1e-3) / 1e9 / (hbm * world), "traffic": None},
            "clocks": clk}


def main_paged_prefill(args):
    """SGLang serving prefill (extend) through the paged drop-ins:
    route_prefill_triton (the varlen router over the k_bar page cache) +
    dash_sparse_attn (K8, the paged prefill attend) for 4 requests that each
    extend 4096 tokens after cached prefixes of 0, 4096, 16384 and 60000
    tokens, on a shuffled page pool (BASELINE head layout, K = 8, LW = 512);
    with --seq S one request extends 8192 rows after an S-token prefix.
    TFLOP/s counts 4 * D * H flops per attended (row, key) at window +
    selected keys per row.  One GPU (each rank its own copy under torchrun)."""
    from srswa import paged
    world, rank, local = rank_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_dist(dev, world)
    g = torch.Generator(device=dev).manual_seed(41 + rank)
    # --seq S: one request extending 8192 rows after an S-token prefix instead
    ctx_l, qlen_l = ([args.seq], [8192]) if args.seq else ([0, 4096, 16384, 60000], [4096] * 4)
    ctx = torch.tensor(ctx_l, dtype=torch.int32, device=dev)
    qlen = torch.tensor(qlen_l, dtype=torch.int32, device=dev)
    seq = ctx + qlen
    R = len(ctx_l)
    W = (max(c + q for c, q in zip(ctx_l, qlen_l)) + BS - 1) // BS + 1
    P = R * W
    bt = torch.randperm(P, device=dev, generator=g).to(torch.int32).view(R, W)
    cu = torch.zeros(R + 1, dtype=torch.int32, device=dev)
    cu[1:] = torch.cumsum(qlen, 0)
    N = sum(qlen_l)
    kc = torch.randn(P, BS, HKV, D, device=dev, generator=g).to(torch.bfloat16)
    vc = torch.randn(P, BS, HKV, D, device=dev, generator=g).to(torch.bfloat16)
    kbar = torch.randn(P, DI, device=dev, generator=g) * 0.1
    q = torch.randn(N, H, D, device=dev, generator=g).to(torch.bfloat16)
    iq = (torch.randn(N, DI, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    row2req = (torch.searchsorted(cu, torch.arange(N, device=dev, dtype=torch.int32), right=True) - 1).to(torch.int32)
    out_idx = torch.empty(N, K, device=dev, dtype=torch.int32)
    out_bias = torch.empty(N, K, device=dev)
    out = torch.empty(N, H, D, device=dev, dtype=torch.bfloat16)

    def step():
        paged.route_prefill_triton(idx_q=iq, k_bar=kbar, block_table=bt, seq_lens=seq, cu_seqlens_q=cu,
                                   context_lens=ctx, row2req=row2req, image_allow=None, out_idx=out_idx,
                                   out_bias=out_bias, max_block=W, block_size=BS, local_blocks=L,
                                   idx_scale=IDX_SCALE, prior_floor=FLOOR, sigma=SIGMA, topm=M, budget=K)
        paged.dash_sparse_attn(q, kc, vc, out_idx.unsqueeze(0).expand(HKV, -1, -1),
                               out_bias.unsqueeze(0).expand(HKV, -1, -1), bt, cu, seq, ctx, max(qlen_l), HKV,
                               SM_SCALE, out, local_blocks=L, sparse_block_size=BS)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    clocks = Clocks(local)
    clocks.start()
    times, _ = timed_graph(step, args.steps, max(args.warmup, 3), flush, False)
    clk = clocks.stop()
    ms = sum(times) / len(times)
    fl = 4.0 * D * H * N * (L * BS + K * BS)
    if rank == 0:
        print(json.dumps({"metric": "SGLang paged prefill (route_prefill_triton + dash_sparse_attn)",
                          "value": fl * world / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world,
                          "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                          "data": "synthetic seeded N(0,1), shuffled page pool",
                          "config": {"workload": (f"paged prefill: 1 request x 8192 new tokens after {args.seq}"
                                                  if args.seq else "paged prefill: 4 requests x 4096 new tokens, "
                                                  "prefixes 0 / 4096 / 16384 / 60000"),
                                     "rows": N, "K": K, "LW": L * BS,
                                     "l2": "flushed before every timed step"},
                          "clocks": clk}), flush=True)
    return 0


def main():
    args = parse()
    if args.workload == "route":
        return main_route(args)
    if args.workload == "longctx":
        return main_longctx(args)
    if args.workload == "pagegate":
        return main_pagegate(args)
    if args.workload == "rope":
        return main_rope(args)
    if args.workload == "kl":
        return main_kl(args)
    if args.workload == "paged-prefill":
        return main_paged_prefill(args)
    if args.workload != "decode" and args.impl != "reference":
        return main_dense(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    S, _ = workload(args)

    if args.impl == "reference":
        if rank != 0:
            return 0
        # the reference's CPU path (its torch ops restated), one request per step
        order = S[: max(1, args.steps + args.warmup)]
        per, byts = [], []
        for i in range(args.warmup + args.steps):
            gbs, info, lens, t = cpu_decode_sample([order[i % len(order)]], budget_s=1e9, max_req=1)
            if i >= args.warmup:
                per.append(t)
                byts.append(gbs * t * 1e9)
        val = sum(byts) / sum(per) / 1e9
        cores = info["threads"]
        line = {"impl": "reference", "metric": METRIC, "value": val, "unit": "GB/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(per) / len(per),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded N(0,1))",
                "config": {"workload": "cfg3 decode step per request (CPU: HF _block_scores_infer -> "
                                       "_infer_route_select -> _decode_attend, dense over the cache)",
                           "requests_per_step": 1, "parallelism": "host cores"},
                "cpu_baseline": {"value": val, "unit": "GB/s", "cores": cores, "kind": "port",
                                 "cpu_model": info["cpu_model"],
                                 "sample": f"{args.steps} request decode steps, S from the cfg3 draw: "
                                           "the reference's fp32 torch CPU path (oracle/torch_cpu.py)"},
                "e2e": {"value": val, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch.distributed as dist
    from srswa import ops  # noqa: F401  (fails loudly without libsrswa.so)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_dist(dev, world)
    parts = shard(S, world)
    mine = parts[rank]
    S_local = [S[i] for i in mine]
    st = build_rank(S_local, 1000 + rank, dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    # warm-up and selection for byte accounting
    run_step(st)
    torch.cuda.synchronize()
    a_b, r_b, k_b = step_bytes(S_local, st["topi"].cpu())
    bytes_rank = a_b + r_b + k_b

    clocks = Clocks(local if "CUDA_VISIBLE_DEVICES" not in os.environ else
                    os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local])
    # soak so the clock sampler sees the loaded state, then the timed steps
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    t_soak = time.time()
    while time.time() - t_soak < 1.5:
        run_step(st)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    times, graph = timed_graph(lambda: run_step(st), args.steps, args.warmup, flush, not args.no_graph)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    step_ms = sum(times) / len(times)

    # dominant kernel alone (attend), same stream discipline
    att_times, g2 = timed_graph(lambda: run_attend(st), args.steps, args.warmup, flush, not args.no_graph)
    att_ms = sum(att_times) / len(att_times)
    rt_times, g3 = timed_graph(lambda: ops.route(st["iq"], st["kbar"], block_size=BS, local_blocks=L, topk=K,
                                                  topm=M, idx_scale=IDX_SCALE, floor=FLOOR, sigma=SIGMA,
                                                  seq_lens=st["sl"], block_table=st["bt"],
                                                  want=("topi32", "bias")),
                               args.steps, args.warmup, flush, not args.no_graph)
    rt_ms = sum(rt_times) / len(rt_times)

    launches = count_launches(lambda: run_step(st), STEP_LAUNCHES)

    # e2e: host buffers through the public API, copies inside the timed region
    e2e = None
    if not args.no_e2e:
        e2e = e2e_measure(st, S_local, args, dev)

    # reduce across ranks: max time, sum bytes
    vec = torch.tensor([step_ms, att_ms, rt_ms, e2e["ms"] if e2e else 0.0], device=dev, dtype=torch.float64)
    tot = torch.tensor([bytes_rank, a_b, e2e["h2d"] if e2e else 0, e2e["d2h"] if e2e else 0, launches],
                       device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(vec, op=dist.ReduceOp.MAX)
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
    step_ms, att_ms, rt_ms, e2e_ms = vec.tolist()
    bytes_all, att_bytes_all, h2d_all, d2h_all, launches_all = tot.tolist()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        gbs, info, lens, t = cpu_decode_sample(S)
        cfg1_ms = cpu_cfg1_ms()
        cpu = {"value": gbs, "unit": "GB/s", "cores": info["threads"], "kind": "port",
               "cpu_model": info["cpu_model"], "logical_cpus": info["logical_cpus"],
               "sample": f"{len(lens)} of {len(S)} requests (S={lens}): the HF CPU decode step in fp32 torch "
                         f"(k_bar of every block, scores, top-M entmax, dense attend over the cache), {t:.1f} s",
               "cfg1_ms_per_step": cfg1_ms,
               "cfg1": "BASELINE config 1: one decode step at S=8192 (B=1, H=10, D=128, K=8, LW=512), fp32"}

    peak, src = peaks()
    att_gbs = (a_b / (att_ms * 1e-3)) / 1e9     # this rank's attend kernel
    ratio = ncu_traffic_ratio()
    if graph is not None:
        del graph, g2, g3
    if rank == 0:
        line = {
            "metric": METRIC, "value": bytes_all / (step_ms * 1e-3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
            "us_per_step": step_ms * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic: seeded request lengths U[16384,131072]; K/V/index keys N(0,1) bf16 "
                    "(windows of a seeded randn pool); q, idx_q seeded randn",
            "config": {"workload": "cfg3 paged SR-SWA decode: 256 requests, S~U[16384,131072], page=block 64, "
                                   "H=Hkv=10, D=128, index d=128, K=8, M=16, LW=512; per step k_bar tail "
                                   "refresh + fused route + sparse attend (CUDA graph)",
                       "global_batch": len(S), "seq_len": "U[16384,131072]", "parallelism": f"requests/dp{world}",
                       "l2": "flushed (256 MiB write) before every timed step",
                       "bytes_per_step": bytes_all},
            "breakdown_us": {"attend": att_ms * 1e3, "route": rt_ms * 1e3},
            "roofline": {"bound": "hbm", "kernel": "attend_rows_kernel<128,bf16>",
                         "achieved": att_gbs, "peak": peak, "unit": "GB/s", "frac": att_gbs / peak,
                         "peak_source": src,
                         "traffic": (ratio * a_b) if ratio else None,
                         "algorithmic_bytes_per_launch": a_b},
            "cpu_baseline": cpu,
            "e2e": None if e2e is None else {
                "value": bytes_all / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                "how": "pinned H2D of the step's inputs (router's inputs first; q and the new K/V rows "
                       "on a second stream beside the router), cache append, kbar_refresh_tail + "
                       "route_decode + dash_sparse_attn_decode, D2H of the output; one CUDA graph per step",
                "h2d_bytes_per_step": h2d_all, "d2h_bytes_per_step": d2h_all},
            "gpu_launches": int(launches_all) * args.steps,   # all ranks, counted on one profiled step
            "clocks": clk,
        }
    # the metric's other half and the long-context config, measured after the
    # headline (the decode state is freed first): cfg2 prefill and cfg4
    # training TFLOP/s against the bf16 peak, the cfg5 split-KV step
    st.clear()
    del st
    torch.cuda.empty_cache()
    extras = {}
    if not args.no_extras:
        # a failed extra is reported in its key; the headline line still prints
        for key, fn in (("prefill", lambda: dense_measure(args, False)), ("train", lambda: dense_measure(args, True)),
                        ("longctx", lambda: longctx_measure(args))):
            try:
                extras[key] = fn()
            except Exception as e:  # noqa: BLE001
                extras[key] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
                torch.cuda.empty_cache()
    if rank == 0:
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        try:
            dist.barrier()
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001  (a rank whose extra failed in a collective)
            pass
    return 0


def e2e_measure(st, S_local, args, dev):
    """Per step: the H2D copies of this step's inputs from pinned host
    buffers, the append of the new token to the paged caches, the decode step
    through the public paged API, and the D2H copy of the output; the step is
    captured once in a CUDA graph (as a serving loop's decode step) and
    replayed, copies included.  The inputs travel in two packed copies: the
    router's (idx_q, the new index-key row, the cache slots) first, then q
    and the new K / V rows on a second stream, appended while the router
    runs and joined before the attend."""
    R = len(S_local)
    g = torch.Generator().manual_seed(77)
    hq = torch.randn(R, H, D, generator=g).to(torch.bfloat16)
    hiq = torch.randn(R, DI, generator=g).to(torch.bfloat16).float()
    hk = torch.randn(R, HKV, D, generator=g).to(torch.bfloat16)
    hv = torch.randn(R, HKV, D, generator=g).to(torch.bfloat16)
    hik = torch.randn(R, DI, generator=g).to(torch.bfloat16)
    bt = st["bt"].cpu()
    page = torch.tensor([int(bt[r, (s - 1) // BS]) for r, s in enumerate(S_local)], dtype=torch.int64)
    slot = torch.tensor([(s - 1) % BS for s in S_local], dtype=torch.int64)
    hslot = torch.stack([page, slot])

    def pack(parts):
        raw = [x.contiguous().view(-1).view(torch.uint8) for x in parts]
        hbuf = torch.cat(raw).pin_memory()
        dbuf = torch.empty_like(hbuf, device=dev)
        views, o = [], 0
        for x, r_ in zip(parts, raw):
            views.append(dbuf[o:o + r_.numel()].view(x.dtype).view(x.shape))
            o += r_.numel()
        return hbuf, dbuf, views

    ha, da, (iq, nik, sl_) = pack([hiq, hik, hslot])   # the router's inputs
    hb, db, (q, nk, nv) = pack([hq, hk, hv])           # the attend's inputs
    hout = torch.empty(R, H, D, dtype=torch.bfloat16).pin_memory()
    h2d = ha.numel() + hb.numel()
    d2h = hout.numel() * hout.element_size()
    kv_stream = torch.cuda.Stream()

    def step():
        main = torch.cuda.current_stream()
        da.copy_(ha, non_blocking=True)
        kv_stream.wait_stream(main)
        with torch.cuda.stream(kv_stream):
            db.copy_(hb, non_blocking=True)
            st["k"][sl_[0], sl_[1]] = nk
            st["v"][sl_[0], sl_[1]] = nv
        def append_index_key():   # only the k_bar refresh reads it: off the router's path
            st["idx"][sl_[0], sl_[1]] = nik

        run_step_public(st, q, iq, kv_ready=kv_stream, before_refresh=append_index_key)
        hout.copy_(st["out"], non_blocking=True)

    s_ = torch.cuda.Stream()
    s_.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s_):
        for _ in range(max(args.warmup, 1)):
            step()
    torch.cuda.current_stream().wait_stream(s_)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(args.warmup, 1)):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    del graph
    return {"ms": ms, "h2d": h2d, "d2h": d2h}


if __name__ == "__main__":
    sys.exit(main())
