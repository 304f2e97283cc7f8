// SR-SWA router kernels: block summaries (a1), fused remote scores + top-M
// 1.5-entmax + top-K + centred log-prior bias (a2 + a4), token block-max
// scores (a3) and selection packing (a5).
//
// All arithmetic that decides the selection is IEEE fp32 (this file must not
// be built with fast-math: divisions and square roots of the entmax threshold
// have to round like the reference's CPU path).

#include "common.cuh"
#include "peer.cuh"

namespace srswa {

// ============================================================================
// a1: head_cls block summaries
// (hf-model-code/modeling_deepseekv2.py:391-408; dash_attention.py:1079-1119;
//  whl:.../unlimited_dash_ops/dash_stage0.py:25-41, route_triton.py:36-72)
// One warp per block; lane l owns features [4l, 4l+4) (d <= 128).
// ============================================================================
constexpr int kMaxBlockSize = 256;

struct KbarArgs {
  const void* keys;
  int dtype;
  int64_t d, bs;
  const float* hc;
  float* out;
  uint8_t* chunk_valid;
  // contiguous
  int64_t sb, st, S, nblk, B;
  // paged
  const int32_t* block_table;
  const int32_t* seq_lens;
  int64_t s_page, s_bt, W, R, tail, s_kbar;
  int paged;  // 0 contiguous, 1 block table (all / tail pages), 2 explicit page plan
  // page plan (paged == 2): item i summarizes page plan_pages[i] from its
  // first plan_tok[i] tokens; items with no token store nothing
  const int64_t* plan_pages;
  const int32_t* plan_tok;
  int64_t plan_n;
};

__device__ __forceinline__ void load4(const void* p, int64_t i, int dtype, float* o) {
  if (dtype == SRSWA_F32) {
    float4 f = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
    o[0] = f.x; o[1] = f.y; o[2] = f.z; o[3] = f.w;
  } else if (dtype == SRSWA_BF16) {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const unsigned short*>(p) + i));
    o[0] = bf16_lo(u.x); o[1] = bf16_hi(u.x); o[2] = bf16_lo(u.y); o[3] = bf16_hi(u.y);
  } else {
    uint2 u = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p) + i));
    float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y;
  }
}

// One CTA (128 threads) per block/page: the block's tokens are staged in
// shared memory as fp32 [bs][d+1] with every 16-byte global load of the block
// issued before any arithmetic (8 per thread for a 64 x 128 bf16 page), then
// thread i scores token i, warp 0 forms the masked softmax weights, and
// thread f accumulates feature f of k_bar.
constexpr int kKbarThreads = 128;

__device__ __forceinline__ void kbar_item(const KbarArgs& a, int64_t item, int64_t& base, int64_t& ntok,
                                          int64_t& out_row) {
  ntok = -1;
  if (!a.paged) {
    if (item >= a.B * a.nblk) return;
    const int64_t b = item / a.nblk, c = item % a.nblk;
    base = b * a.sb + c * a.bs * a.st;
    ntok = min(a.bs, a.S - c * a.bs);
    out_row = item * a.d;
  } else if (a.paged == 2) {
    if (item >= a.plan_n) return;
    const int64_t nt = min(a.bs, static_cast<int64_t>(a.plan_tok[item]));
    if (nt <= 0) return;  // not a page slot of the plan (padding): store nothing
    const int64_t page = a.plan_pages[item];
    base = page * a.s_page;
    out_row = page * a.s_kbar;
    ntok = nt;
  } else {
    const int64_t per = a.tail > 0 ? a.tail : a.W;
    if (item >= a.R * per) return;
    const int64_t r = item / per, j = item % per;
    const int64_t sl = a.seq_lens[r];
    const int64_t nb = (sl + a.bs - 1) / a.bs;
    const int64_t blk = a.tail > 0 ? nb - 1 - j : j;
    if (blk < 0 || blk >= nb || blk >= a.W) return;
    const int64_t nt = min(a.bs, sl - blk * a.bs);
    if (nt <= 0) return;  // not a page in use: never clobber another request's summary
    const int64_t page = a.block_table[r * a.s_bt + blk];
    base = page * a.s_page;
    out_row = page * a.s_kbar;
    ntok = nt;
  }
}

__global__ void __launch_bounds__(kKbarThreads) kbar_kernel(const KbarArgs a) {
  extern __shared__ __align__(16) float kb_smem[];  // [bs][d+1] then w[bs]
  const int tid = threadIdx.x;
  const int64_t item = blockIdx.x;
  int64_t base = 0, ntok = -1, out_row = 0;
  kbar_item(a, item, base, ntok, out_row);
  if (ntok < 0) return;  // CTA-uniform
  if (!a.paged && a.chunk_valid && tid == 0) a.chunk_valid[item] = ntok > 0;
  const int d = static_cast<int>(a.d);
  const int dp = d + 1;
  float* ks = kb_smem;
  float* w = kb_smem + a.bs * dp;
  // stage: 16-byte pieces (8 elements of a 16-bit type, 4 of fp32), all loads
  // of an 8-piece batch issued before any shared-memory store
  const int vec = a.dtype == SRSWA_F32 ? 4 : 8;
  const int ppt = d / vec;  // pieces per token
  const int pieces = static_cast<int>(ntok) * ppt;
  float* hcs = w + a.bs;
  for (int f = tid; f < d; f += kKbarThreads) hcs[f] = a.hc[f];
  for (int i0 = tid; i0 < pieces; i0 += kKbarThreads * 8) {
    float v[8][8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kKbarThreads;
      if (i < pieces) {
        const int t = i / ppt, f = (i % ppt) * vec;
        if (vec == 8) load8(a.keys, base + static_cast<int64_t>(t) * a.st + f, a.dtype, v[u]);
        else load4(a.keys, base + static_cast<int64_t>(t) * a.st + f, a.dtype, v[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * kKbarThreads;
      if (i < pieces) {
        const int t = i / ppt, f = (i % ppt) * vec;
        for (int e = 0; e < vec; ++e) ks[t * dp + f + e] = v[u][e];
      }
    }
  }
  __syncthreads();
  const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(d));
  for (int t = tid; t < ntok; t += kKbarThreads) {
    float acc = 0.f;
    for (int f = 0; f < d; ++f) acc = fmaf(ks[t * dp + f], hcs[f], acc);
    w[t] = fminf(fmaxf(acc * inv_sqrt_d, -kActClamp), kActClamp);
  }
  __syncthreads();
  if (tid < 32) {
    // masked softmax over the valid tokens (row max over valid tokens only)
    float mx = -INFINITY;
    for (int t = tid; t < ntok; t += 32) mx = fmaxf(mx, w[t]);
    mx = warp_max(mx);
    if (ntok <= 0) mx = 0.f;
    float den = 0.f;
    for (int t = tid; t < ntok; t += 32) {
      const float e = expf(w[t] - mx);
      w[t] = e;
      den += e;
    }
    den = warp_sum(den);
    const float dn = fmaxf(den, 1e-6f);
    __syncwarp();
    for (int t = tid; t < ntok; t += 32) w[t] = w[t] / dn;
  }
  __syncthreads();
  for (int f = tid; f < d; f += kKbarThreads) {
    float acc = 0.f;
    for (int t = 0; t < ntok; ++t) acc = fmaf(w[t], ks[t * dp + f], acc);
    a.out[out_row + f] = isfinite(acc) ? acc : 0.f;
  }
}

static int kbar_launch(const KbarArgs& a, int64_t items, cudaStream_t st) {
  const size_t smem = (static_cast<size_t>(a.bs) * (a.d + 1) + a.bs + a.d) * sizeof(float);
  if (smem > 227 * 1024) return SRSWA_ETOOLARGE;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kbar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  if (items >= (1ll << 31)) return SRSWA_ETOOLARGE;
  kbar_kernel<<<static_cast<unsigned>(items), kKbarThreads, smem, st>>>(a);
  return srswa_last_launch_status();
}

// ============================================================================
// a2 + a4: fused scores + selection
// ============================================================================
constexpr int kRouteThreads = 256;
constexpr int kMaxTopM = 32;

struct RouteArgs {
  // score source: 0 = dots against k_bar, 1 = given scores
  int from_scores;
  const void* q;
  int q_dtype;
  int64_t s_q, d;
  const float* kbar;
  int64_t s_kbar_b, s_kbar_c;
  const int32_t* block_table;
  int64_t s_bt;
  const int32_t* seq_lens;
  int64_t rows_per_seq;
  const int32_t* row_seq;  // sequence of each row (varlen prefill rows); NULL = n / rows_per_seq
  const int64_t* q_pos;
  const float* scores_in;
  int64_t s_sc;
  const uint8_t* cand;
  int64_t s_cand;
  int64_t N, nblk;
  int64_t BS, L, K, M;
  float idx_scale, floor_, inv_sigma;
  int64_t* topi64;
  int32_t* topi32;
  float* bias;
  uint8_t* valid;
  float* scores_out;
  int rows_per_cta;
};

__device__ __forceinline__ int64_t route_row_seq(const RouteArgs& a, int64_t n) {
  return a.row_seq ? static_cast<int64_t>(a.row_seq[n]) : n / a.rows_per_seq;
}

struct Best {
  float v;
  int i;
};
__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
  return v1 > v2 || (v1 == v2 && i1 < i2);
}

// dot products of one query row against k_bar rows [c_lo, c_hi), written to xs[c]
// as clamped fp32 scores.  ws warps of the row cooperate (wr = rank among them).
template <int LPB>
__device__ void route_dots(const RouteArgs& a, int64_t n, int64_t seq, int64_t c_hi, float* zs,
                           int wr, int ws, int lane) {
  constexpr int RPI = 32 / LPB;  // k_bar rows per warp instruction
  constexpr int BPG = RPI * 8;   // blocks per group (8 loads per lane)
  const int g = lane / LPB, u = lane % LPB;
  float qv[4];
  load4(a.q, n * a.s_q + 4 * u, a.q_dtype, qv);
  const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(a.d));
  const int64_t ngroups = (c_hi + BPG - 1) / BPG;
  for (int64_t gi = wr; gi < ngroups; gi += ws) {
    const int64_t c0 = gi * BPG;
    float part[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t c = c0 + i * RPI + g;
      float kv[4] = {0.f, 0.f, 0.f, 0.f};
      if (c < c_hi) {
        int64_t off;
        if (a.block_table) off = static_cast<int64_t>(a.block_table[seq * a.s_bt + c]) * a.s_kbar_c;
        else off = seq * a.s_kbar_b + c * a.s_kbar_c;
        const float4 f = __ldg(reinterpret_cast<const float4*>(a.kbar + off + 4 * u));
        kv[0] = f.x; kv[1] = f.y; kv[2] = f.z; kv[3] = f.w;
      }
      part[i] = qv[0] * kv[0] + qv[1] * kv[1] + qv[2] * kv[2] + qv[3] * kv[3];
    }
    const float s = transpose_reduce8<LPB>(part, u);
    const int my = 4 * ((u & (LPB / 2)) != 0) + 2 * ((u & (LPB / 4)) != 0) + ((u & (LPB / 8)) != 0);
    const int64_t c = c0 + my * RPI + g;
    if ((u & (LPB / 8 - 1)) == 0 && c < c_hi) {
      float z = s * inv_sqrt_d;
      z = fminf(fmaxf(z, -kActClamp), kActClamp);  // NaN propagates (fmin/fmax drop it) -> handled below
      if (s != s) z = s;
      zs[c] = z;
    }
  }
}

// Exact 1.5-entmax over the M sorted top values held one per lane (lane j <
// M holds the j-th largest x, its block sel_i and whether it is a candidate),
// then the first K slots and their centred log-prior bias, written for row n.
// Called by one warp.
// kCompact: short loops instead of unrolled gathers, for a single run from
// a cold instruction cache (once per row of a few-row kernel); the unrolled
// form keeps shuffle latency out of the sums for kernels that loop over rows.
template <bool kCompact = false>
__device__ __forceinline__ void route_epilogue(const RouteArgs& a, int64_t n, int lane, float sel_v, int sel_i,
                                               bool sel_cand) {
  const int M = static_cast<int>(a.M);
  // ---- exact 1.5-entmax over the M sorted values
  // (hf-model-code/dash_attention.py:772-800): X = (x - max)/2; prefix sums in
  // float64 rounded to fp32 per prefix (torch CPU cumsum of fp32); tau_rho =
  // mean - sqrt(max(0, (1 - rho(meansq - mean^2))/rho)); support = #(tau <= X)
  const float xmax = __shfl_sync(0xffffffffu, sel_v, 0);
  const float X = (sel_v - xmax) / 2.0f;
  // every lane runs the same left-to-right float64 sums
  double acc1 = 0.0, acc2 = 0.0;
  float my_cs = 0.f, my_cs2 = 0.f;
  if (kCompact) {
#pragma unroll 1
    for (int j = 0; j < M; ++j) {
      const float xj = __shfl_sync(0xffffffffu, X, j);
      acc1 += static_cast<double>(xj);
      acc2 += static_cast<double>(xj * xj);
      if (lane == j) { my_cs = static_cast<float>(acc1); my_cs2 = static_cast<float>(acc2); }
    }
  } else {  // 8 values gathered at a time (independent shuffles)
    for (int j0 = 0; j0 < M; j0 += 8) {
      float xs[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) xs[e] = __shfl_sync(0xffffffffu, X, (j0 + e) & 31);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (j0 + e < M) {
          acc1 += static_cast<double>(xs[e]);
          acc2 += static_cast<double>(xs[e] * xs[e]);
          if (lane == j0 + e) { my_cs = static_cast<float>(acc1); my_cs2 = static_cast<float>(acc2); }
        }
      }
    }
  }
  const float rho = static_cast<float>(lane + 1);
  const float mean = my_cs / rho;
  const float mean_sq = my_cs2 / rho;
  const float ss = rho * (mean_sq - mean * mean);
  const float delta = (1.0f - ss) / rho;
  const float tau = mean - sqrtf(fmaxf(delta, 0.0f));
  const unsigned sup_mask = __ballot_sync(0xffffffffu, lane < M && tau <= X);
  int support = __popc(sup_mask);
  if (support < 1) support = 1;
  const float tau_star = __shfl_sync(0xffffffffu, tau, support - 1);
  const float pm = fmaxf(X - tau_star, 0.0f);
  const float prior = pm * pm;

  // ---- first K slots, centred log-prior bias ----
  const int K = static_cast<int>(a.K);
  const bool vld = lane < K && sel_cand;
  const float logp = logf(fmaxf(prior, a.floor_));
  float sum = 0.f;
  int cnt = 0;
  const unsigned vmask = __ballot_sync(0xffffffffu, vld);
  if (kCompact) {
#pragma unroll 1
    for (int j = 0; j < K; ++j) {
      const float lj = __shfl_sync(0xffffffffu, logp, j);
      if ((vmask >> j) & 1u) { sum += lj; ++cnt; }
    }
  } else {
    for (int j0 = 0; j0 < K; j0 += 8) {
      float ls[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) ls[e] = __shfl_sync(0xffffffffu, logp, (j0 + e) & 31);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (j0 + e < K && ((vmask >> (j0 + e)) & 1u)) { sum += ls[e]; ++cnt; }
      }
    }
  }
  const float mu = sum / static_cast<float>(cnt > 0 ? cnt : 1);
  const float bias = vld ? (logp - mu) * a.inv_sigma : 0.f;
  if (lane < K) {
    const int64_t o = n * K + lane;
    if (a.topi64) a.topi64[o] = sel_i;
    if (a.topi32) a.topi32[o] = vld ? sel_i : -1;
    if (a.bias) a.bias[o] = bias;
    if (a.valid) a.valid[o] = vld ? 1 : 0;
  }
}


__global__ void __launch_bounds__(kRouteThreads) route_kernel(const RouteArgs a) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int rpc = a.rows_per_cta;
  const int64_t nblk = a.nblk;
  float* xs_all = reinterpret_cast<float*>(smem_raw);
  uint8_t* fl_all = reinterpret_cast<uint8_t*>(xs_all + rpc * nblk);
  __shared__ int any_cand[8];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wpr = 8 / rpc;  // warps per row
  const int rr = warp / wpr, wr = warp % wpr;
  const int64_t n = static_cast<int64_t>(blockIdx.x) * rpc + rr;
  const bool row_ok = n < a.N;
  float* xs = xs_all + rr * nblk;
  uint8_t* fl = fl_all + rr * nblk;

  int64_t seq = 0, p = 0, c_hi = 0;
  if (row_ok) {
    seq = route_row_seq(a, n);
    if (!a.from_scores) {
      p = a.q_pos ? a.q_pos[n] : static_cast<int64_t>(a.seq_lens[seq]) - a.rows_per_seq + n % a.rows_per_seq;
      // remote blocks: c <= p/BS - L, holding a token (c*BS < seq_len)
      c_hi = p >= 0 ? p / a.BS - a.L + 1 : 0;
      if (c_hi < 0) c_hi = 0;
      if (c_hi > nblk) c_hi = nblk;
      if (a.seq_lens) {
        const int64_t nb = (static_cast<int64_t>(a.seq_lens[seq]) + a.BS - 1) / a.BS;
        if (c_hi > nb) c_hi = nb;
      }
    }
  }
  if (warp < 8 && wr == 0 && lane == 0) any_cand[rr] = 0;

  // ---- phase 1: scores (z), SCORE_NEG outside [0, c_hi) ----
  if (row_ok) {
    if (a.from_scores) {
      for (int64_t c = wr * 32 + lane; c < nblk; c += wpr * 32) xs[c] = a.scores_in[n * a.s_sc + c];
    } else {
      for (int64_t c = c_hi + wr * 32 + lane; c < nblk; c += wpr * 32) xs[c] = kScoreNeg;
      if (a.d == 128) route_dots<32>(a, n, seq, c_hi, xs, wr, wpr, lane);
      else route_dots<16>(a, n, seq, c_hi, xs, wr, wpr, lane);
    }
  }
  __syncthreads();
  // ---- phase 2: candidacy flags, x = cand ? z*idx_scale : -1e4 ----
  if (row_ok) {
    int found = 0;
    for (int64_t c = wr * 32 + lane; c < nblk; c += wpr * 32) {
      const float z = xs[c];
      if (a.scores_out) a.scores_out[n * nblk + c] = z;
      const bool remote = z > kScoreNeg * 0.5f;  // NaN -> not remote
      const bool cm = remote && (a.cand == nullptr || a.cand[n * a.s_cand + c] != 0);
      fl[c] = static_cast<uint8_t>((remote ? 2 : 0) | (cm ? 1 : 0));
      found |= cm;
    }
    found = __any_sync(0xffffffffu, found);
    if (lane == 0 && found) atomicOr(&any_cand[rr], 1);
  }
  __syncthreads();
  if (row_ok) {
    const bool fallback = any_cand[rr] == 0;
    for (int64_t c = wr * 32 + lane; c < nblk; c += wpr * 32) {
      uint8_t f = fl[c];
      if (fallback) f = (f & 2) ? 3 : 0;  // rows with an empty domain use all remote blocks
      fl[c] = f;
      float x = (f & 1) ? xs[c] * a.idx_scale : kEntmaxNeg;
      if (!isfinite(x)) x = kEntmaxNeg;
      xs[c] = x;
    }
  }
  __syncthreads();
  if (!row_ok || wr != 0) return;

  // ---- phase 3: top-M by repeated warp arg-max (ties: lower index first) ----
  const int M = static_cast<int>(a.M);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int64_t c = lane; c < nblk; c += 32)
    if (better(xs[c], static_cast<int>(c), bv, bi)) { bv = xs[c]; bi = static_cast<int>(c); }
  float sel_v = 0.f;
  int sel_i = -1;
  for (int j = 0; j < M; ++j) {
    float wv = bv;
    int wi = bi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, wi, o);
      if (better(ov, oi, wv, wi)) { wv = ov; wi = oi; }
    }
    if (lane == j) { sel_v = wv; sel_i = wi; }
    if (wi != 0x7fffffff && (wi & 31) == lane) {
      xs[wi] = -INFINITY;  // removed
      bv = -INFINITY;
      bi = 0x7fffffff;
      for (int64_t c = lane; c < nblk; c += 32)
        if (better(xs[c], static_cast<int>(c), bv, bi)) { bv = xs[c]; bi = static_cast<int>(c); }
    }
    __syncwarp();
  }

  const bool sel_cand = lane < M && sel_i >= 0 && (fl[sel_i] & 1);
  route_epilogue(a, n, lane, sel_v, sel_i, sel_cand);
}

// ============================================================================
// a2 + a4 for wide rows (decode shapes: few rows, hundreds to thousands of
// candidate blocks): two kernels.
//
// route_score_kernel  streaming scores: one CTA per (row, 128-block chunk),
//   clamped scores z (SCORE_NEG outside the row's remote range, with no loads
//   there) written to a [N, nblk] array.
// select_wide_kernel  one CTA per row.  x = cand ? z * idx_scale : -1e4 is
//   packed with its block index and candidacy into a 64-bit key (x descending,
//   then block ascending); each of the 8 warps extracts the top-M keys of its
//   slice by repeated warp arg-max, warp 0 merges the 8 lists and runs the
//   entmax / top-K / bias epilogue.  A candidate mask with no candidate in the
//   row falls back to all remote blocks (CTA-wide OR).
// ============================================================================
constexpr int kWideMaxBlocks = 24576;  // shared-memory key array bound (192 KiB)

__device__ __forceinline__ uint32_t ordered_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float from_ordered(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}
__device__ __forceinline__ unsigned long long pack_key(float x, int64_t c, bool cand) {
  const uint32_t lo = (static_cast<uint32_t>(0x7fffffff - static_cast<int32_t>(c)) << 1) | (cand ? 1u : 0u);
  return (static_cast<unsigned long long>(ordered_bits(x)) << 32) | lo;
}
// Warp-wide maximum of 64-bit keys: the high words by one warp reduction,
// then the low words of the lanes holding that high word.
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
  const uint32_t hi = static_cast<uint32_t>(v >> 32), lo = static_cast<uint32_t>(v);
  const uint32_t mh = __reduce_max_sync(0xffffffffu, hi);
  const uint32_t ml = __reduce_max_sync(0xffffffffu, hi == mh ? lo : 0u);
  return (static_cast<unsigned long long>(mh) << 32) | ml;
}

// Top-M keys of k[0..n) (shared memory, unique non-zero keys) by one warp;
// written in descending order to out[0..M) (0 where fewer than M keys).
// Extracted keys are zeroed in k.
__device__ void warp_topm_smem(unsigned long long* k, int n, int M, unsigned long long* out, int lane) {
  unsigned long long best = 0ull;
  for (int i = lane; i < n; i += 32) best = k[i] > best ? k[i] : best;
  for (int m = 0; m < M; ++m) {
    const unsigned long long w = warp_max_u64(best);
    if (lane == 0) out[m] = w;
    if (w != 0ull && best == w) {  // unique keys: exactly one owner lane
      best = 0ull;
      for (int i = lane; i < n; i += 32) {
        unsigned long long v = k[i];
        if (v == w) { k[i] = 0ull; v = 0ull; }
        best = v > best ? v : best;
      }
    }
    __syncwarp();
  }
}

// One CTA per (row, 128-block chunk): the chunk's block-table slice (one
// coalesced load), then its k_bar rows in a single round (16 independent
// 16-byte loads per lane, 8 warps).  Register-capped for 3 CTAs per SM.
constexpr int kChunkBlocks = 128;

// Chunks of kChunkBlocks blocks per CTA: the row position and the block-table
// slice are loaded once for all of them (two dependent round trips), then
// the k_bar loads of one chunk after the other.
constexpr int kScoreReps = 2;
__global__ void __launch_bounds__(kRouteThreads, 3) route_score_kernel(const RouteArgs a, float* zout,
                                                                       int64_t row0) {
  pdl_launch_dependents();  // lets the selection kernel launch early
  constexpr int kSpan = kChunkBlocks * kScoreReps;
  __shared__ int32_t bts[kSpan];
  const int64_t n = row0 + blockIdx.y;  // rows go in launches of at most 65535 (grid.y)
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kSpan;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t seq = route_row_seq(a, n);
  const int64_t p = a.q_pos ? a.q_pos[n]
                            : static_cast<int64_t>(a.seq_lens[seq]) - a.rows_per_seq + n % a.rows_per_seq;
  int64_t c_hi = p >= 0 ? p / a.BS - a.L + 1 : 0;
  if (c_hi < 0) c_hi = 0;
  if (c_hi > a.nblk) c_hi = a.nblk;
  if (a.seq_lens) {
    const int64_t nb = (static_cast<int64_t>(a.seq_lens[seq]) + a.BS - 1) / a.BS;
    if (c_hi > nb) c_hi = nb;
  }
  const int64_t hi = min(lo + kSpan, a.nblk);
  const int64_t dhi = max(lo, min(hi, c_hi));  // blocks [lo, dhi) are remote
  float* zrow = zout + n * a.nblk;
  for (int64_t c = dhi + tid; c < hi; c += kRouteThreads) zrow[c] = kScoreNeg;
  if (dhi == lo) return;  // CTA-uniform: nothing remote in this span
  if (a.block_table)
    for (int64_t i = tid; i < dhi - lo; i += kRouteThreads) bts[i] = a.block_table[seq * a.s_bt + lo + i];
  __syncthreads();
  const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(a.d));
  float qv[4];
  load4(a.q, n * a.s_q + 4 * lane, a.q_dtype, qv);
  for (int rep = 0; rep < kScoreReps; ++rep) {
    const int64_t c0 = lo + static_cast<int64_t>(rep) * kChunkBlocks + warp * 16;
    if (c0 >= dhi) break;  // warp-uniform
    float4 f[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int64_t c = c0 + i;
      f[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < dhi) {
        const int64_t off = a.block_table ? static_cast<int64_t>(bts[c - lo]) * a.s_kbar_c
                                          : seq * a.s_kbar_b + c * a.s_kbar_c;
        f[i] = __ldg(reinterpret_cast<const float4*>(a.kbar + off + 4 * lane));
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float part[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = f[8 * h + i];
        part[i] = qv[0] * v.x + qv[1] * v.y + qv[2] * v.z + qv[3] * v.w;
      }
      const float sdot = transpose_reduce8<32>(part, lane);
      const int my = 4 * ((lane & 16) != 0) + 2 * ((lane & 8) != 0) + ((lane & 4) != 0);
      const int64_t c = c0 + 8 * h + my;
      if ((lane & 3) == 0 && c < dhi) {
        float z = fminf(fmaxf(sdot * inv_sqrt_d, -kActClamp), kActClamp);
        if (sdot != sdot) z = sdot;  // NaN stays NaN (then "not remote")
        zrow[c] = z;
      }
    }
  }
}

// Top-M of unique non-zero keys held in registers, NPL per lane, by one warp:
// each lane sorts its keys descending (compare-swap network), then every
// round takes the warp maximum of the lanes' heads and the owning lane shifts
// its list.  Lane m returns the m-th key (0 past the last key).
template <int NPL>
__device__ __forceinline__ unsigned long long warp_topm_regs(unsigned long long (&v)[NPL], int M, int lane) {
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
#pragma unroll
    for (int j = 0; j + 1 < NPL - i; ++j) {
      const unsigned long long x = v[j], y = v[j + 1];
      v[j] = x > y ? x : y;
      v[j + 1] = x > y ? y : x;
    }
  }
  unsigned long long mine = 0ull;
  for (int m = 0; m < M; ++m) {
    const unsigned long long w = warp_max_u64(v[0]);
    if (lane == m) mine = w;
    if (w != 0ull && v[0] == w) {  // unique keys: exactly one owner
#pragma unroll
      for (int j = 0; j + 1 < NPL; ++j) v[j] = v[j + 1];
      v[NPL - 1] = 0ull;
    }
  }
  return mine;
}

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v), m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), m);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}
__device__ __forceinline__ unsigned long long max_u64(unsigned long long a, unsigned long long b) { return a > b ? a : b; }
__device__ __forceinline__ unsigned long long min_u64(unsigned long long a, unsigned long long b) { return a > b ? b : a; }

// Descending bitonic sort of 64 keys held two per lane (element i = 32 *
// slot + lane: e0 = slot 0, e1 = slot 1).
__device__ __forceinline__ void bitonic64_desc(unsigned long long& e0, unsigned long long& e1, int lane) {
#pragma unroll
  for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j == 32) {  // partners in one lane (only in the final merge: descending)
        const unsigned long long a = e0, b = e1;
        e0 = max_u64(a, b);
        e1 = min_u64(a, b);
      } else {
        const unsigned long long p0 = shfl_xor_u64(e0, j), p1 = shfl_xor_u64(e1, j);
        const bool first = (lane & j) == 0;
        const bool d0 = (lane & k) == 0, d1 = ((32 + lane) & k) == 0;  // descending blocks
        e0 = (first == d0) ? max_u64(e0, p0) : min_u64(e0, p0);
        e1 = (first == d1) ? max_u64(e1, p1) : min_u64(e1, p1);
      }
    }
  }
}

// Descending bitonic sort of 32 keys, one per lane.
__device__ __forceinline__ unsigned long long bitonic32_desc(unsigned long long e, int lane) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long p = shfl_xor_u64(e, j);
      const bool take_max = ((lane & j) == 0) == ((lane & k) == 0);
      e = take_max ? max_u64(e, p) : min_u64(e, p);
    }
  }
  return e;
}

// Second half of the threshold top-M: the keys >= t0 (t0 a lower bound of
// the M-th largest key) go to the warp's 64-entry scratch and one bitonic
// sort orders them: 32 keys, one per lane, when at most 32 survive, else 64
// keys, two per lane.  More than 64 such keys: the round-based
// warp_topm_regs.  Lane m returns the m-th key.
template <int NPL>
__device__ __forceinline__ unsigned long long topm_above(unsigned long long (&v)[NPL], unsigned long long t0, int M,
                                                         int lane, unsigned long long* scratch) {
  // survivors: nonzero keys >= t0; exclusive prefix of the lanes' counts
  int cnt = 0;
#pragma unroll
  for (int k = 0; k < NPL; ++k) cnt += (v[k] != 0ull && v[k] >= t0) ? 1 : 0;
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  if (total > 64) return warp_topm_regs<NPL>(v, M, lane);  // warp-uniform
  int pos = incl - cnt;
#pragma unroll
  for (int k = 0; k < NPL; ++k)
    if (v[k] != 0ull && v[k] >= t0) scratch[pos++] = v[k];
  if (total <= 32) {  // warp-uniform: one key per lane
    __syncwarp();
    unsigned long long e = lane < total ? scratch[lane] : 0ull;
    __syncwarp();
    e = bitonic32_desc(e, lane);
    return lane < M ? e : 0ull;
  }
  for (int i = total + lane; i < 64; i += 32) scratch[i] = 0ull;
  __syncwarp();
  unsigned long long e0 = scratch[lane], e1 = scratch[lane + 32];
  __syncwarp();
  bitonic64_desc(e0, e1, lane);
  return lane < M ? e0 : 0ull;
}

__device__ __forceinline__ unsigned long long shfl_u64(unsigned long long v, int src) {
  const uint32_t lo = __shfl_sync(0xffffffffu, static_cast<uint32_t>(v), src);
  const uint32_t hi = __shfl_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), src);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

// Top-M (M <= 32) of unique keys held in registers, NPL per lane, by one warp,
// with the same result as warp_topm_regs.  The M-th largest of the 32 lane
// maxima (bitonic sort across the lanes) is a lower bound of the M-th largest
// key, since at least M keys reach it; the keys at or above it (normally a
// few more than M for keys in no particular order) are sorted by topm_above.
template <int NPL>
__device__ __forceinline__ unsigned long long warp_topm_filtered(unsigned long long (&v)[NPL], int M, int lane,
                                                               unsigned long long* scratch) {
  unsigned long long lm = 0ull;
#pragma unroll
  for (int k = 0; k < NPL; ++k) lm = max_u64(lm, v[k]);
  // lane i <- the i-th largest lane maximum
  const unsigned long long srt = bitonic32_desc(lm, lane);
  return topm_above<NPL>(v, shfl_u64(srt, M - 1), M, lane, scratch);
}

// As warp_topm_filtered for keys sorted descending within each lane (pieces
// of sorted lists): the threshold is the M-th largest of every lane's first
// two keys (a 64-key bitonic sort), which keeps few keys even when the lanes'
// maxima are few or all near the top.
template <int NPL>
__device__ __forceinline__ unsigned long long warp_topm_sorted(unsigned long long (&v)[NPL], int M, int lane,
                                                             unsigned long long* scratch) {
  static_assert(NPL >= 2, "two keys per lane sample the threshold");
  unsigned long long e0 = v[0], e1 = v[1];
  bitonic64_desc(e0, e1, lane);
  return topm_above<NPL>(v, shfl_u64(e0, M - 1), M, lane, scratch);
}

// Top-M of the 8 per-warp lists (M keys each, sorted descending, kMaxTopM
// apart) by warp 0; lane m returns the m-th key.  Lane l holds ranks
// l / 8 + 4k of list l % 8 (descending within the lane), so the sampled
// threshold is drawn from the first eight ranks of every list.
__device__ unsigned long long merge8_topm(const unsigned long long* flat, int M, int lane,
                                          unsigned long long* scratch) {
  unsigned long long v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = (lane >> 3) + 4 * k;
    v[k] = r < M ? flat[(lane & 7) * kMaxTopM + r] : 0ull;
  }
  return warp_topm_sorted<8>(v, M, lane, scratch);
}
__device__ __forceinline__ void unpack_key(unsigned long long k, float& x, int& blk, bool& cand) {
  x = from_ordered(static_cast<uint32_t>(k >> 32));
  const uint32_t lo32 = static_cast<uint32_t>(k);
  blk = 0x7fffffff - static_cast<int>(lo32 >> 1);
  cand = (lo32 & 1u) != 0;
}

// Top-M of `total` unique keys in shared memory (consumed) by the whole CTA:
// one warp for short lists, else a per-warp top-M of each eighth and a merge
// of the 8 lists.  Called by all threads; lane m of warp 0 gets key m.
__device__ unsigned long long block_topm(unsigned long long* mk, int64_t total, int M,
                                         unsigned long long (*lists)[kMaxTopM],
                                         unsigned long long (*scratch)[64], int warp, int lane) {
  unsigned long long mine = 0ull;
  if (total <= 256) {  // CTA-uniform
    if (warp == 0) {
      warp_topm_smem(mk, static_cast<int>(total), M, lists[0], lane);
      __syncwarp();
      mine = lane < M ? lists[0][lane] : 0ull;
    }
    return mine;
  }
  const int64_t per = (total + 7) / 8;
  const int64_t wlo = warp * per;
  const int64_t rem = total - wlo;
  const int64_t wn = rem < 0 ? 0 : (rem < per ? rem : per);
  warp_topm_smem(mk + wlo, static_cast<int>(wn), M, lists[warp], lane);
  __syncthreads();
  if (warp == 0) mine = merge8_topm(&lists[0][0], M, lane, scratch[0]);
  return mine;
}

// Top-M of up to 32 key lists held one per lane (v, sorted descending,
// 0-padded) by one warp: M rounds of a warp arg-max over the list heads, the
// owner lane shifts its list.  Lane m returns the m-th key.
__device__ __forceinline__ unsigned long long warp_merge_heads(unsigned long long (&v)[16], int M, int lane) {
  unsigned long long mine = 0ull;
#pragma unroll 1
  for (int m = 0; m < M; ++m) {
    const unsigned long long w = warp_max_u64(v[0]);
    if (lane == m) mine = w;
    if (w != 0ull && v[0] == w) {  // unique keys: one owner lane
#pragma unroll
      for (int k = 0; k + 1 < 16; ++k) v[k] = v[k + 1];
      v[15] = 0ull;
    }
  }
  return mine;
}

// Top-M (M <= 16) of nlists (<= 256) key lists, each sorted descending (M
// keys, 0-padded), list l at src + l * stride (global memory), by the whole
// CTA: lane j of warp w loads list w * per + j into registers and the warp
// merges its lists (warp_merge_heads), then warp 0 merges the 8 warps'
// lists.  Two short loops: the merge runs once per row, from a cold
// instruction cache.  Called by all threads; lane m of warp 0 gets key m.
constexpr int64_t kSortedListsMax = 8 * 32;
template <bool kShared = false>  // lists in shared memory instead of global
__device__ unsigned long long block_merge_lists(const unsigned long long* src, int64_t stride, int64_t nlists,
                                                int M, unsigned long long (*lists)[kMaxTopM], int warp, int lane) {
  const int64_t per = (nlists + 7) / 8;
  const int64_t l = static_cast<int64_t>(warp) * per + lane;
  const bool has = lane < per && l < nlists;
  unsigned long long v[16];
#pragma unroll
  for (int k = 0; k < 16; ++k)
    v[k] = (has && k < M) ? (kShared ? src[l * stride + k] : __ldcg(src + l * stride + k)) : 0ull;
  const unsigned long long top = warp_merge_heads(v, M, lane);
  if (lane < M) lists[warp][lane] = top;
  __syncthreads();
  if (warp != 0) return 0ull;
#pragma unroll
  for (int k = 0; k < 16; ++k) v[k] = (lane < 8 && k < M) ? lists[lane][k] : 0ull;
  return warp_merge_heads(v, M, lane);
}

__global__ void __launch_bounds__(kRouteThreads) select_wide_kernel(const RouteArgs a, const float* zin,
                                                                    int64_t s_z) {
  pdl_launch_dependents();  // lets an overlapping attend start on its window
  pdl_wait();               // the scores of the kernel ahead
  extern __shared__ __align__(16) unsigned long long wk[];  // [nblk] keys
  __shared__ unsigned long long lists[kRouteThreads / 32][kMaxTopM];
  __shared__ unsigned long long topm_scratch[kRouteThreads / 32][64];
  const int64_t n = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t nblk = a.nblk;
  const int M = static_cast<int>(a.M);
  const float* z = zin + n * s_z;
  // the row's scores (and candidate flags), eight per thread in flight at once
  constexpr int kBatch = 8 * kRouteThreads;
  int any = 1;
  if (a.cand) {
    int f = 0;
    for (int64_t c0 = 0; c0 < nblk; c0 += kBatch) {
      float zc[8];
      uint8_t cf[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int64_t c = c0 + tid + k * kRouteThreads;
        zc[k] = c < nblk ? z[c] : kScoreNeg;
        cf[k] = c < nblk ? a.cand[n * a.s_cand + c] : 0;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) f |= (zc[k] > kScoreNeg * 0.5f) && cf[k] != 0;
    }
    any = __syncthreads_or(f);
  }
  for (int64_t c0 = 0; c0 < nblk; c0 += kBatch) {
    float zc[8];
    uint8_t cf[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t c = c0 + tid + k * kRouteThreads;
      zc[k] = c < nblk ? z[c] : kScoreNeg;
      cf[k] = (a.cand && c < nblk) ? a.cand[n * a.s_cand + c] : 1;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t c = c0 + tid + k * kRouteThreads;
      if (c >= nblk) break;
      if (a.scores_out) a.scores_out[n * nblk + c] = zc[k];
      const bool remote = zc[k] > kScoreNeg * 0.5f;
      const bool cm = remote && (a.cand == nullptr || !any || cf[k] != 0);
      float x = cm ? zc[k] * a.idx_scale : kEntmaxNeg;
      if (!isfinite(x)) x = kEntmaxNeg;
      wk[c] = pack_key(x, c, cm);
    }
  }
  __syncthreads();
  const int64_t per = (nblk + 7) / 8;
  const int64_t wlo = warp * per;
  const int64_t rem = nblk - wlo;
  const int64_t wn = rem < 0 ? 0 : (rem < per ? rem : per);
  if (per <= 512) {  // the warp's slice fits 16 registers per lane
    unsigned long long v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int64_t i = lane + 32 * k;
      v[k] = i < wn ? wk[wlo + i] : 0ull;
    }
    const unsigned long long top = warp_topm_filtered<16>(v, M, lane, topm_scratch[warp]);
    if (lane < M) lists[warp][lane] = top;
  } else {
    warp_topm_smem(wk + wlo, static_cast<int>(wn), M, lists[warp], lane);
  }
  __syncthreads();
  if (warp != 0) return;
  unsigned long long mine;
  if (M <= 16) {  // the 8 warps' sorted lists: a short head-merge loop
    unsigned long long v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = (lane < 8 && k < M) ? lists[lane][k] : 0ull;
    mine = warp_merge_heads(v, M, lane);
  } else {
    mine = merge8_topm(&lists[0][0], M, lane, topm_scratch[0]);
  }
  float sel_v = 0.f;
  int sel_i = -1;
  bool sel_c = false;
  if (lane < M) unpack_key(mine, sel_v, sel_i, sel_c);
  route_epilogue<true>(a, n, lane, sel_v, sel_i, sel_c);  // once per CTA
}

// ============================================================================
// Split-KV router: rows whose blocks are spread over shards (GPUs), or are too
// many for one CTA (16384 blocks of a 1M-token row).  Packed keys are the
// interface between the stages (and between processes):
//   bits 63..32 ordered bits of x, bits 31..1 0x7fffffff - global block id,
//   bit 0 candidate; larger = ranks first; 0 = no key.
// route_chunk_keys_kernel  one CTA per (row, 128 owned blocks): scores like
//   route_score_kernel (global candidacy: block id = block_offset + local),
//   packs keys in shared memory, warp 0 keeps the chunk's top-M.
// keys_merge_kernel  one CTA per row over nlists lists of M keys: per-warp
//   top-M, 8-list merge; then either the merged M keys or the entmax / top-K
//   / bias epilogue (plus the shard-owned copy of topi32).
// The top-M of a union of disjoint sets is contained in the union of the
// sets' top-Ms, so both stages are exact.
// With ShardFinish.on the row's last CTA of route_chunk_keys_kernel also does
// the second stage: alone (one shard), or after pushing its keys to every
// peer and a bounded wait for theirs (the lists sit in this rank's region).
// ============================================================================
struct ShardFinish {
  int on;
  int64_t own_lo, own_hi;
  int32_t* topi32_own;
};

__device__ __forceinline__ void finish_row(const RouteArgs& a, const ShardFinish& fin, int64_t n, int lane,
                                           unsigned long long key) {
  float sel_v = 0.f;
  int sel_i = -1;
  bool sel_c = false;
  if (lane < a.M) unpack_key(key, sel_v, sel_i, sel_c);
  route_epilogue<true>(a, n, lane, sel_v, sel_i, sel_c);
  if (fin.topi32_own && lane < a.K) {
    const bool own = sel_c && sel_i >= fin.own_lo && sel_i < fin.own_hi;
    fin.topi32_own[n * a.K + lane] = own ? sel_i : -1;
  }
}

__global__ void __launch_bounds__(kRouteThreads) route_chunk_keys_kernel(const RouteArgs a, int64_t blk_off,
                                                                         int64_t nblk_local,
                                                                         unsigned long long* chunk_out,
                                                                         unsigned int* counters,
                                                                         unsigned long long* keys_out,
                                                                         const srswa_peer push,
                                                                         const ShardFinish fin) {
  pdl_launch_dependents();  // lets an overlapping attend start on its window
  // [max(nch, world) * M]: the chunk lists (last CTA of a row), then the ranks' lists
  extern __shared__ __align__(16) unsigned long long mk[];
  __shared__ int32_t bts[kChunkBlocks];
  __shared__ float zs[kChunkBlocks];
  __shared__ unsigned long long keys[kChunkBlocks];
  __shared__ unsigned long long lists[kRouteThreads / 32][kMaxTopM];
  __shared__ unsigned long long rowk[kMaxTopM];
  __shared__ unsigned long long topm_scratch[kRouteThreads / 32][64];
  __shared__ unsigned int ticket;
  const int64_t n = blockIdx.y;
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * kChunkBlocks;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t seq = route_row_seq(a, n);
  const int64_t p = a.q_pos ? a.q_pos[n]
                            : static_cast<int64_t>(a.seq_lens[seq]) - a.rows_per_seq + n % a.rows_per_seq;
  int64_t c_hi = p >= 0 ? p / a.BS - a.L + 1 : 0;  // global: remote blocks are [0, c_hi)
  if (c_hi < 0) c_hi = 0;
  if (c_hi > a.nblk) c_hi = a.nblk;
  if (a.seq_lens) {
    const int64_t nb = (static_cast<int64_t>(a.seq_lens[seq]) + a.BS - 1) / a.BS;
    if (c_hi > nb) c_hi = nb;
  }
  const int64_t hi = min(lo + kChunkBlocks, nblk_local);
  const int64_t dhi = max(lo, min(hi, c_hi - blk_off));  // local blocks [lo, dhi) are remote
  for (int64_t c = lo + tid; c < lo + kChunkBlocks; c += kRouteThreads) zs[c - lo] = kScoreNeg;
  if (a.block_table && tid < dhi - lo) bts[tid] = a.block_table[seq * a.s_bt + blk_off + lo + tid];
  __syncthreads();
  const int64_t c0 = lo + warp * 16;
  if (c0 < dhi) {  // warp-uniform
    const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(a.d));
    float qv[4];
    load4(a.q, n * a.s_q + 4 * lane, a.q_dtype, qv);
    float4 f[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int64_t c = c0 + i;
      f[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < dhi) {
        const int64_t off = a.block_table ? static_cast<int64_t>(bts[c - lo]) * a.s_kbar_c
                                          : seq * a.s_kbar_b + c * a.s_kbar_c;
        f[i] = __ldg(reinterpret_cast<const float4*>(a.kbar + off + 4 * lane));
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float part[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = f[8 * h + i];
        part[i] = qv[0] * v.x + qv[1] * v.y + qv[2] * v.z + qv[3] * v.w;
      }
      const float sdot = transpose_reduce8<32>(part, lane);
      const int my = 4 * ((lane & 16) != 0) + 2 * ((lane & 8) != 0) + ((lane & 4) != 0);
      const int64_t c = c0 + 8 * h + my;
      if ((lane & 3) == 0 && c < dhi) {
        float z = fminf(fmaxf(sdot * inv_sqrt_d, -kActClamp), kActClamp);
        if (sdot != sdot) z = sdot;
        zs[c - lo] = z;
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < kChunkBlocks; i += kRouteThreads) {
    const int64_t c = lo + i;
    unsigned long long key = 0ull;
    if (c < hi) {
      const float zc = zs[i];
      const bool cm = zc > kScoreNeg * 0.5f;  // no candidate mask in this form
      float x = cm ? zc * a.idx_scale : kEntmaxNeg;
      if (!isfinite(x)) x = kEntmaxNeg;
      key = pack_key(x, blk_off + c, cm);
    }
    keys[i] = key;
  }
  __syncthreads();
  const int M = static_cast<int>(a.M);
  const int64_t nch = gridDim.x;
  if (warp == 0) {  // the chunk's top-M (4 keys per lane, threshold filter)
    unsigned long long v[kChunkBlocks / 32];
#pragma unroll
    for (int k = 0; k < kChunkBlocks / 32; ++k) v[k] = keys[lane + 32 * k];
    const unsigned long long top = warp_topm_filtered<kChunkBlocks / 32>(v, M, lane, topm_scratch[0]);
    if (lane < M) {
      if (nch == 1) rowk[lane] = top;  // the chunk is the whole shard row
      else chunk_out[(n * nch + blockIdx.x) * M + lane] = top;
    }
  }
  if (nch > 1) {
    // the last CTA of the row to finish merges the row's chunk lists
    __threadfence();
    __syncthreads();
    if (tid == 0) ticket = atomicAdd(counters + n, 1u);
    __syncthreads();
    if (ticket != static_cast<unsigned int>(nch - 1)) return;
    __threadfence();
    const int64_t total = nch * M;
    const unsigned long long* src = chunk_out + n * total;
    unsigned long long mine;
    if (nch <= kSortedListsMax && M <= 16) {  // CTA-uniform
      mine = block_merge_lists(src, M, nch, M, lists, warp, lane);
    } else {
      for (int64_t i = tid; i < total; i += kRouteThreads) mk[i] = __ldcg(src + i);
      __syncthreads();
      mine = block_topm(mk, total, M, lists, topm_scratch, warp, lane);
    }
    if (warp == 0 && lane < M) rowk[lane] = mine;
    if (tid == 0) counters[n] = 0u;
  }
  __syncthreads();
  // rowk: this rank's top-M keys of the row
  if (push.regions && push.ll) {  // LL exchange (with the finish stage only)
    // this rank's keys as LL words to every region, then every rank's from
    // this rank's region, each word polled until it carries the epoch
    const uint32_t ep = ll_epoch(push);
    if (tid < M) {
      const unsigned long long key = rowk[tid];
      ll_put(push, 2 * (n * M + tid), ep, static_cast<uint32_t>(key));
      ll_put(push, 2 * (n * M + tid) + 1, ep, static_cast<uint32_t>(key >> 32));
    }
    const int world = static_cast<int>(push.world);
    bool ok = true;
    for (int i = tid; i < world * M; i += kRouteThreads) {
      const int r = i / M, j = i - r * M;
      const uint32_t lo = ll_get(push, r, 2 * (n * M + j), ep, ok);
      const uint32_t hi = ll_get(push, r, 2 * (n * M + j) + 1, ep, ok);
      mk[i] = (static_cast<unsigned long long>(hi) << 32) | lo;
    }
    __syncthreads();
    if (tid == 0) ll_consumer_done(push, gridDim.y);
    const unsigned long long merged =
        M <= 16 ? block_merge_lists<true>(mk, M, world, M, lists, warp, lane)
                : block_topm(mk, static_cast<int64_t>(world) * M, M, lists, topm_scratch, warp, lane);
    if (warp == 0) finish_row(a, fin, n, lane, merged);
    return;
  }
  if (push.regions && tid < M) peer_put8(push, (n * M + tid) * 8, rowk[tid]);  // to every peer
  if (!fin.on) {
    if (keys_out && tid < M) keys_out[n * M + tid] = rowk[tid];
    if (push.regions) {
      __syncthreads();
      if (tid == 0) peer_unit_done(push, gridDim.y);  // one unit per row
    }
    return;
  }
  if (!push.regions) {  // one shard: its list is the row's
    if (warp == 0) finish_row(a, fin, n, lane, lane < M ? rowk[lane] : 0ull);
    return;
  }
  // every rank's list of the row, from this rank's region (bounded wait)
  __syncthreads();
  if (tid == 0) {
    peer_unit_done(push, gridDim.y);
    peer_wait_all(push, gridDim.y);
  }
  __syncthreads();
  const int world = static_cast<int>(push.world);
  const unsigned long long* base =
      reinterpret_cast<const unsigned long long*>(static_cast<const char*>(push.own_region) + kPeerHeader) + n * M;
  const int64_t s_list = push.slot_bytes / 8;  // slot r = rank r's keys
  unsigned long long merged;
  if (M <= 16) {  // CTA-uniform
    merged = block_merge_lists(base, s_list, world, M, lists, warp, lane);
  } else {
    for (int l = warp; l < world; l += kRouteThreads / 32)
      if (lane < M) mk[l * M + lane] = __ldcg(base + l * s_list + lane);
    __syncthreads();
    merged = block_topm(mk, static_cast<int64_t>(world) * M, M, lists, topm_scratch, warp, lane);
  }
  if (warp == 0) finish_row(a, fin, n, lane, merged);
}

constexpr int64_t kMergeMaxKeys = 24576;  // nlists * M per row (192 KiB of shared memory)
constexpr int64_t kShardSelectMaxRowsPeer = 128;  // rows of srswa_route_shard_select with an exchange

__global__ void __launch_bounds__(kRouteThreads) keys_merge_kernel(const RouteArgs a, const unsigned long long* keys,
                                                                   int64_t nlists, int64_t s_list, int64_t s_row,
                                                                   unsigned long long* keys_out, int64_t own_lo,
                                                                   int64_t own_hi, int32_t* topi32_own,
                                                                   const srswa_peer wait) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) unsigned long long mk[];
  __shared__ unsigned long long lists[kRouteThreads / 32][kMaxTopM];
  __shared__ unsigned long long topm_scratch[kRouteThreads / 32][64];
  const int64_t n = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (wait.regions) {  // the lists are the peers' pushes into this rank's region
    if (tid == 0) peer_wait_all(wait, gridDim.x);
    __syncthreads();
  }
  const int M = static_cast<int>(a.M);
  const int64_t total = nlists * M;
  unsigned long long mine;
  if (nlists <= kSortedListsMax && M <= 16) {  // CTA-uniform
    mine = block_merge_lists(keys + n * s_row, s_list, nlists, M, lists, warp, lane);
  } else {
    for (int64_t l = warp; l < nlists; l += kRouteThreads / 32)
      if (lane < M) mk[l * M + lane] = __ldcg(keys + l * s_list + n * s_row + lane);
    __syncthreads();
    mine = block_topm(mk, total, M, lists, topm_scratch, warp, lane);
  }
  if (warp != 0) return;
  if (keys_out) {
    if (lane < M) keys_out[n * M + lane] = mine;
    return;
  }
  float sel_v = 0.f;
  int sel_i = -1;
  bool sel_c = false;
  if (lane < M) unpack_key(mine, sel_v, sel_i, sel_c);
  route_epilogue<true>(a, n, lane, sel_v, sel_i, sel_c);  // once per CTA
  if (topi32_own && lane < a.K) {
    const bool own = sel_c && sel_i >= own_lo && sel_i < own_hi;
    topi32_own[n * a.K + lane] = own ? sel_i : -1;
  }
}

// ============================================================================
// a3: token block-max scores, 64 queries x 1 key block per CTA, fp32 FMA
// ============================================================================
constexpr int kBmQ = 64;

struct BlockMaxArgs {
  const void* q;
  int q_dtype;
  int64_t sqb, sqc;
  const void* k;
  int k_dtype;
  int64_t skb, sks;
  const int64_t* pos;
  const int64_t* seg;
  int64_t B, C, Sk, D, BS, nblk, LW;
  int mode;
  float* out;
};

__global__ void __launch_bounds__(256) block_max_kernel(const BlockMaxArgs a) {
  extern __shared__ __align__(16) float bm_smem[];
  const int64_t D = a.D;
  const int64_t DP = D + 1;  // padded rows: conflict-free column reads
  float* qs = bm_smem;                  // [64][DP]
  float* ks = bm_smem + kBmQ * DP;      // [BS][DP]
  __shared__ int64_t lo_s[kBmQ], hi_s[kBmQ];
  const int64_t b = blockIdx.z, blk = blockIdx.y, q0 = static_cast<int64_t>(blockIdx.x) * kBmQ;
  const int tid = threadIdx.x;
  const int64_t j0 = blk * a.BS;
  const float fill = a.mode == 0 ? -INFINITY : kScoreNeg;
  // per-query valid key range [lo, hi) inside this block
  if (tid < kBmQ) {
    const int64_t c = q0 + tid;
    int64_t lo = j0, hi = j0;
    if (c < a.C) {
      const int64_t pc = a.pos[b * a.C + c];
      int64_t ls = pc - a.LW + 1;
      if (a.mode == 0 && ls < 0) ls = 0;
      const int64_t sg = a.seg ? a.seg[b * a.C + c] : 0;
      lo = max(j0, sg);
      hi = min(min(j0 + a.BS, a.Sk), ls);
    }
    lo_s[tid] = lo;
    hi_s[tid] = hi;
  }
  __syncthreads();
  int any = 0;
  for (int i = 0; i < kBmQ; ++i) any |= lo_s[i] < hi_s[i];
  if (!any) {
    if (tid < kBmQ && q0 + tid < a.C) a.out[(b * a.C + q0 + tid) * a.nblk + blk] = fill;
    return;
  }
  for (int64_t e = tid; e < kBmQ * D; e += 256) {
    const int64_t r = e / D, dd = e % D;
    const int64_t c = q0 + r;
    qs[r * DP + dd] = c < a.C ? load_elem(a.q, b * a.sqb + c * a.sqc + dd, a.q_dtype) : 0.f;
  }
  for (int64_t e = tid; e < a.BS * D; e += 256) {
    const int64_t r = e / D, dd = e % D;
    const int64_t j = j0 + r;
    ks[r * DP + dd] = j < a.Sk ? load_elem(a.k, b * a.skb + j * a.sks + dd, a.k_dtype) : 0.f;
  }
  __syncthreads();
  // thread -> (query ty*4..+4, keys tx + 16*m)
  const int tx = tid & 15, ty = tid >> 4;
  float best[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  for (int64_t kk0 = 0; kk0 < a.BS; kk0 += 64) {
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int64_t dd = 0; dd < D; ++dd) {
      float qa[4], kb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qa[i] = qs[(ty * 4 + i) * DP + dd];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t kr = kk0 + tx + 16 * j;
        kb[j] = kr < a.BS ? ks[kr * DP + dd] : 0.f;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(qa[i], kb[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t jj = j0 + kk0 + tx + 16 * j;
        if (kk0 + tx + 16 * j < a.BS && jj >= lo_s[r] && jj < hi_s[r]) best[i] = fmaxf(best[i], acc[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) best[i] = fmaxf(best[i], __shfl_xor_sync(0xffffffffu, best[i], o));
  }
  if (tx == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      const int64_t c = q0 + r;
      if (c >= a.C) continue;
      float v;
      if (lo_s[r] >= hi_s[r]) v = fill;
      else v = a.mode == 1 ? fminf(fmaxf(best[i], -kActClamp), kActClamp) : best[i];
      a.out[(b * a.C + c) * a.nblk + blk] = v;
    }
  }
}

// ============================================================================
// a5: selection packing (dedup; invalid ids -> -1)
// ============================================================================
__global__ void pack_selection_kernel(const void* sel, int is64, int64_t rows, int64_t S, int64_t nblk,
                                      int32_t* out) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  for (int64_t s = 0; s < S; ++s) {
    const int64_t v = load_index(sel, r * S + s, is64);
    bool keep = v >= 0 && v < nblk;
    for (int64_t t = 0; t < s && keep; ++t) keep = load_index(sel, r * S + t, is64) != v;
    out[r * S + s] = keep ? static_cast<int32_t>(v) : -1;
  }
}

// ============================================================================
// a2 + a4 for prefill rows (many rows of one sequence, up to 1024 blocks):
// route_tile_kernel, one CTA per 32 consecutive rows of one sequence.
//   scores  k_bar is staged in 64-block chunks in shared memory (rows padded
//           to 132 floats: the float4 reads of 8 consecutive lanes hit
//           distinct bank quads); thread = 4 rows x 2 blocks (lane, lane+32),
//           fp32 FMAs over d; z = clamp(dot / sqrt(d)) for blocks below the
//           row's remote bound, SCORE_NEG elsewhere (same values as
//           route_kernel up to summation order);
//   select  warp w takes rows 4w..4w+3 one after another: 64-bit keys (x
//           descending, then block ascending), warp top-M by warp maxima,
//           the exact entmax / top-K / bias epilogue.
// ============================================================================
constexpr int kRtRows = 32;
constexpr int kRtChunk = 64;
constexpr int kRtLd = 132;
constexpr int64_t kRtMaxBlocks = 1024;  // [32][1024] fp32 scores + staging: 192 KB of shared memory

static size_t route_tile_smem(int64_t nblk, bool paged) {
  const size_t ab = static_cast<size_t>(kRtRows + kRtChunk) * kRtLd * 4;   // q tile + k_bar chunk
  const size_t keys = static_cast<size_t>(8) * nblk * 8;                   // per-warp keys (aliases ab)
  return (ab > keys ? ab : keys) + static_cast<size_t>(kRtRows) * nblk * 4 +  // + scores
         (paged ? static_cast<size_t>(nblk) * 4 : 0);                        // + block table
}

// Selection of route_tile_kernel for the 4 rows of one warp (NPL keys per
// lane: blocks lane + 32 i, i < NPL, NPL * 32 >= nblk).
template <int NPL>
__device__ __forceinline__ void route_tile_select(const RouteArgs& a, const float* zs, int64_t n0, int r0, int lane,
                                                  unsigned long long* scratch) {
  const int64_t nblk = a.nblk;
  const int M = static_cast<int>(a.M);
  for (int rr = 0; rr < 4; ++rr) {
    const int r = r0 + rr;
    const int64_t n = n0 + r;
    if (n >= a.N) break;  // warp-uniform
    const float* z = zs + r * nblk;
    int found = 1;
    if (a.cand) {
      int f = 0;
      for (int64_t c = lane; c < nblk; c += 32) f |= (z[c] > kScoreNeg * 0.5f) && a.cand[n * a.s_cand + c] != 0;
      found = __any_sync(0xffffffffu, f);
    }
    unsigned long long v[NPL];
#pragma unroll
    for (int k = 0; k < NPL; ++k) {
      const int64_t c = lane + 32 * k;
      v[k] = 0ull;
      if (c < nblk) {
        const float zc = z[c];
        if (a.scores_out) a.scores_out[n * nblk + c] = zc;
        const bool remote = zc > kScoreNeg * 0.5f;  // NaN -> not remote
        const bool cm = remote && (a.cand == nullptr || !found || a.cand[n * a.s_cand + c] != 0);
        float x = cm ? zc * a.idx_scale : kEntmaxNeg;
        if (!isfinite(x)) x = kEntmaxNeg;
        v[k] = pack_key(x, c, cm);
      }
    }
    const unsigned long long mine = warp_topm_filtered<NPL>(v, M, lane, scratch);
    float sel_v = 0.f;
    int sel_i = -1;
    bool sel_c = false;
    if (lane < M) unpack_key(mine, sel_v, sel_i, sel_c);
    route_epilogue(a, n, lane, sel_v, sel_i, sel_c);
    __syncwarp();
  }
}

// NPLMAX: keys per lane of the widest selection compiled in (16: up to 512
// blocks; 32: up to 1024, a separate instantiation since its registers would
// halve the CTAs per SM of the narrower cases).
template <int NPLMAX>
__global__ void __launch_bounds__(kRouteThreads) route_tile_kernel(const RouteArgs a) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) float rt_smem[];
  const int64_t nblk = a.nblk;
  float* qs = rt_smem;                       // [32][132]
  float* kb = qs + kRtRows * kRtLd;          // [64][132]
  const size_t ab = static_cast<size_t>(kRtRows + kRtChunk) * kRtLd;
  const size_t kw = static_cast<size_t>(8) * nblk * 2;
  float* zs = rt_smem + (ab > kw ? ab : kw);  // [32][nblk]
  int32_t* bts = reinterpret_cast<int32_t*>(zs + kRtRows * nblk);  // [nblk] block table (paged k_bar)
  __shared__ int64_t chi[kRtRows];
  __shared__ int64_t cmax_s;
  __shared__ unsigned long long topm_scratch[kRouteThreads / 32][64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kRtRows;
  const int64_t seq = n0 / a.rows_per_seq;  // all 32 rows share it (rows_per_seq % 32 == 0)
  if (tid < kRtRows) {
    const int64_t n = n0 + tid;
    int64_t c_hi = 0;
    if (n < a.N) {
      const int64_t p = a.q_pos ? a.q_pos[n]
                                : static_cast<int64_t>(a.seq_lens[seq]) - a.rows_per_seq + n % a.rows_per_seq;
      c_hi = p >= 0 ? p / a.BS - a.L + 1 : 0;
      if (c_hi < 0) c_hi = 0;
      if (c_hi > nblk) c_hi = nblk;
      if (a.seq_lens) {
        const int64_t nb = (static_cast<int64_t>(a.seq_lens[seq]) + a.BS - 1) / a.BS;
        if (c_hi > nb) c_hi = nb;
      }
    }
    chi[tid] = c_hi;
    int64_t m = c_hi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int64_t y = __shfl_xor_sync(0xffffffffu, m, o);
      m = y > m ? y : m;
    }
    if (tid == 0) cmax_s = m;
  }
  // q tile (fp32): 32 rows x 128 = 1024 float4
  for (int i = tid; i < kRtRows * 32; i += kRouteThreads) {
    const int r = i >> 5, u = i & 31;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (n0 + r < a.N) load4(a.q, (n0 + r) * a.s_q + 4 * u, a.q_dtype, v);
    *reinterpret_cast<float4*>(qs + r * kRtLd + 4 * u) = make_float4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();
  const int64_t cmax = cmax_s;
  // paged k_bar: the sequence's block-table entries of the remote range,
  // staged once (the chunk loads then take one dependent round trip, not two)
  if (a.block_table) {
    for (int64_t c = tid; c < cmax; c += kRouteThreads) bts[c] = a.block_table[seq * a.s_bt + c];
    __syncthreads();
  }
  const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(a.d));
  const int r0 = warp * 4;
  // k_bar chunks: this thread's 8 float4 of the next chunk are loaded into
  // registers while the current chunk's FMAs run
  float4 pf[kRtChunk * 32 / kRouteThreads];
  auto load_chunk = [&](int64_t cb) {
#pragma unroll
    for (int k8 = 0; k8 < kRtChunk * 32 / kRouteThreads; ++k8) {
      const int i = tid + k8 * kRouteThreads, j = i >> 5, u = i & 31;
      const int64_t c = cb + j;
      // k_bar row of block c: contiguous per sequence, or a page of the cache
      // (the block table is read for remote blocks only: c < cmax <= nblk)
      pf[k8] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < cmax) {
        const int64_t kb_off = a.block_table ? static_cast<int64_t>(bts[c]) * a.s_kbar_c
                                             : seq * a.s_kbar_b + c * a.s_kbar_c;
        pf[k8] = __ldg(reinterpret_cast<const float4*>(a.kbar + kb_off + 4 * u));
      }
    }
  };
  if (cmax > 0) load_chunk(0);
  for (int64_t c0 = 0; c0 < nblk; c0 += kRtChunk) {
    if (c0 >= cmax) {  // no row has remote blocks here: sentinel scores only
      for (int i = tid; i < kRtRows * kRtChunk; i += kRouteThreads) {
        const int r = i / kRtChunk;
        const int64_t c = c0 + i % kRtChunk;
        if (c < nblk) zs[r * nblk + c] = kScoreNeg;
      }
      continue;
    }
#pragma unroll
    for (int k8 = 0; k8 < kRtChunk * 32 / kRouteThreads; ++k8) {
      const int i = tid + k8 * kRouteThreads, j = i >> 5, u = i & 31;
      *reinterpret_cast<float4*>(kb + j * kRtLd + 4 * u) = pf[k8];
    }
    __syncthreads();
    if (c0 + kRtChunk < cmax) load_chunk(c0 + kRtChunk);
    float acc[4][2];
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) acc[rr][0] = acc[rr][1] = 0.f;
#pragma unroll 4
    for (int d4 = 0; d4 < 32; ++d4) {
      const float4 k0v = *reinterpret_cast<const float4*>(kb + lane * kRtLd + 4 * d4);
      const float4 k1v = *reinterpret_cast<const float4*>(kb + (lane + 32) * kRtLd + 4 * d4);
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const float4 qv = *reinterpret_cast<const float4*>(qs + (r0 + rr) * kRtLd + 4 * d4);
        acc[rr][0] = fmaf(qv.x, k0v.x, acc[rr][0]);
        acc[rr][0] = fmaf(qv.y, k0v.y, acc[rr][0]);
        acc[rr][0] = fmaf(qv.z, k0v.z, acc[rr][0]);
        acc[rr][0] = fmaf(qv.w, k0v.w, acc[rr][0]);
        acc[rr][1] = fmaf(qv.x, k1v.x, acc[rr][1]);
        acc[rr][1] = fmaf(qv.y, k1v.y, acc[rr][1]);
        acc[rr][1] = fmaf(qv.z, k1v.z, acc[rr][1]);
        acc[rr][1] = fmaf(qv.w, k1v.w, acc[rr][1]);
      }
    }
#pragma unroll
    for (int rr = 0; rr < 4; ++rr) {
      const int r = r0 + rr;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int64_t c = c0 + lane + 32 * h;
        if (c >= nblk) continue;
        const float sdot = acc[rr][h];
        float z = fminf(fmaxf(sdot * inv_sqrt_d, -kActClamp), kActClamp);
        if (sdot != sdot) z = sdot;
        zs[r * nblk + c] = c < chi[r] ? z : kScoreNeg;
      }
    }
    __syncthreads();  // k_bar chunk reuse
  }
  __syncthreads();
  // ---- selection: warp w, rows 4w .. 4w+3; lane holds blocks lane + 32 i ----
  if (nblk <= 128) route_tile_select<4>(a, zs, n0, r0, lane, topm_scratch[warp]);
  else if (nblk <= 256) route_tile_select<8>(a, zs, n0, r0, lane, topm_scratch[warp]);
  else if (NPLMAX == 16 || nblk <= 512) route_tile_select<16>(a, zs, n0, r0, lane, topm_scratch[warp]);
  else route_tile_select<NPLMAX>(a, zs, n0, r0, lane, topm_scratch[warp]);
}

// Rows of one sequence (at least 32), or of several whose row counts are
// multiples of 32 (a tile never spans two sequences); k_bar contiguous or
// paged.
static bool use_tile(const RouteArgs& a) {
  return !a.from_scores && a.row_seq == nullptr && a.d == 128 && a.nblk <= kRtMaxBlocks &&
         ((a.rows_per_seq == a.N && a.N >= kRtRows) || (a.rows_per_seq % kRtRows == 0 && a.N % kRtRows == 0));
}

// ----------------------------------------------------------------------------
// route_tile_long_kernel: prefill rows of one sequence with more than 1024
// blocks (long contexts).  As route_tile_kernel, 32 rows per CTA share each
// staged 64-block k_bar chunk; the blocks go in 512-block spans: each span's
// scores sit in shared memory, each row's top-M of the span (warp top-M) is
// merged into the row's running top-M (a 64-key bitonic sort of the two
// sorted lists) and the entmax / top-K / bias epilogue runs once at the end.
// The top-M of a union is the top-M of the spans' top-Ms, so the selection
// equals the one-pass kernels'.  Spans past every row's remote range are
// skipped: their blocks rank below the first span's (sentinel x, larger
// index).  A candidate mask keeps a second running list over every remote
// block, taken for a row none of whose remote blocks is a candidate (the
// reference's fallback).  No scores output in this form.
// ----------------------------------------------------------------------------
constexpr int kRlSpan = 512;
constexpr int kRlChunk = 128;  // k_bar blocks staged at a time

static size_t route_tile_long_smem(int64_t nblk, bool paged) {
  return static_cast<size_t>(kRtRows + kRlChunk) * kRtLd * 4 + static_cast<size_t>(kRtRows) * kRlSpan * 4 +
         (paged ? static_cast<size_t>(nblk) * 4 : 0);
}
// paged long rows: the staged block table bounds the block count (48 KB)
constexpr int64_t kRlMaxPagedBlocks = 12288;

__global__ void __launch_bounds__(kRouteThreads) route_tile_long_kernel(const RouteArgs a) {
  pdl_launch_dependents();
  extern __shared__ __align__(16) float rt_smem[];
  const int64_t nblk = a.nblk;
  float* qs = rt_smem;                     // [32][132]
  float* kb = qs + kRtRows * kRtLd;        // [128][132]
  float* zs = kb + kRlChunk * kRtLd;       // [32][512]: one span's scores
  int32_t* bts = reinterpret_cast<int32_t*>(zs + kRtRows * kRlSpan);  // [nblk] block table (paged k_bar)
  __shared__ int64_t chi[kRtRows];
  __shared__ int64_t cmax_s;
  __shared__ unsigned long long topm_scratch[kRouteThreads / 32][64];
  __shared__ unsigned long long best[kRtRows][kMaxTopM];  // running top-M per row, descending
  __shared__ unsigned long long best_all[kRtRows][kMaxTopM];  // the same over every remote block (masks)
  __shared__ int found_s[kRtRows];                            // a candidate among the row's remote blocks
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = static_cast<int>(a.M);
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kRtRows;
  const int64_t seq = n0 / a.rows_per_seq;  // all 32 rows share it
  if (tid < kRtRows) {
    const int64_t n = n0 + tid;
    int64_t c_hi = 0;
    if (n < a.N) {
      const int64_t p = a.q_pos ? a.q_pos[n]
                                : static_cast<int64_t>(a.seq_lens[seq]) - a.rows_per_seq + n % a.rows_per_seq;
      c_hi = p >= 0 ? p / a.BS - a.L + 1 : 0;
      if (c_hi < 0) c_hi = 0;
      if (c_hi > nblk) c_hi = nblk;
      if (a.seq_lens) {
        const int64_t nb = (static_cast<int64_t>(a.seq_lens[seq]) + a.BS - 1) / a.BS;
        if (c_hi > nb) c_hi = nb;
      }
    }
    chi[tid] = c_hi;
    int64_t m = c_hi;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const int64_t y = __shfl_xor_sync(0xffffffffu, m, o);
      m = y > m ? y : m;
    }
    if (tid == 0) cmax_s = m;
  }
  for (int i = tid; i < kRtRows * kMaxTopM; i += kRouteThreads) {
    best[i / kMaxTopM][i % kMaxTopM] = 0ull;
    best_all[i / kMaxTopM][i % kMaxTopM] = 0ull;
  }
  if (tid < kRtRows) found_s[tid] = 0;
  for (int i = tid; i < kRtRows * 32; i += kRouteThreads) {
    const int r = i >> 5, u = i & 31;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (n0 + r < a.N) load4(a.q, (n0 + r) * a.s_q + 4 * u, a.q_dtype, v);
    *reinterpret_cast<float4*>(qs + r * kRtLd + 4 * u) = make_float4(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();
  const int64_t cmax = cmax_s;
  // paged k_bar: the sequence's block-table entries of the remote range,
  // staged once (the chunk loads then take one dependent round trip, not two)
  if (a.block_table) {
    for (int64_t c = tid; c < cmax; c += kRouteThreads) bts[c] = a.block_table[seq * a.s_bt + c];
    __syncthreads();
  }
  const float inv_sqrt_d = 1.0f / sqrtf(static_cast<float>(a.d));
  const int r0 = warp * 4;                 // selection: rows 4w .. 4w + 3
  const int rg = (warp & 3) * 8, bh = (warp >> 2) * 64;  // scores: rows rg .. rg + 7, blocks bh + lane (+32)
  float4 pf[kRlChunk * 32 / kRouteThreads];
  auto load_chunk = [&](int64_t cb) {
#pragma unroll
    for (int k8 = 0; k8 < kRlChunk * 32 / kRouteThreads; ++k8) {
      const int i = tid + k8 * kRouteThreads, j = i >> 5, u = i & 31;
      const int64_t c = cb + j;
      pf[k8] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c < cmax) {
        const int64_t kb_off = a.block_table ? static_cast<int64_t>(bts[c]) * a.s_kbar_c
                                             : seq * a.s_kbar_b + c * a.s_kbar_c;
        pf[k8] = __ldg(reinterpret_cast<const float4*>(a.kbar + kb_off + 4 * u));
      }
    }
  };
  // spans [s0, s0 + 512): at least the first (fillers of rows with fewer
  // than M remote blocks), then those holding remote blocks of some row
  const int64_t s_end = cmax > kRlSpan ? cmax : kRlSpan;
  if (cmax > 0) load_chunk(0);
  for (int64_t s0 = 0; s0 < s_end && s0 < nblk; s0 += kRlSpan) {
    const int64_t s1 = min(s0 + kRlSpan, nblk);
    for (int64_t c0 = s0; c0 < s1; c0 += kRlChunk) {
      if (c0 >= cmax) {  // no row has remote blocks here: sentinel scores only
        for (int i = tid; i < kRtRows * kRlChunk; i += kRouteThreads) {
          const int r = i / kRlChunk;
          const int64_t c = c0 + i % kRlChunk;
          if (c < s1) zs[r * kRlSpan + (c - s0)] = kScoreNeg;
        }
        continue;
      }
#pragma unroll
      for (int k8 = 0; k8 < kRlChunk * 32 / kRouteThreads; ++k8) {
        const int i = tid + k8 * kRouteThreads, j = i >> 5, u = i & 31;
        *reinterpret_cast<float4*>(kb + j * kRtLd + 4 * u) = pf[k8];
      }
      __syncthreads();
      if (c0 + kRlChunk < cmax) load_chunk(c0 + kRlChunk);
      // thread: 8 rows x 2 blocks (two k_bar reads per 8 broadcast q reads)
      float acc[8][2];
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) acc[rr][0] = acc[rr][1] = 0.f;
#pragma unroll 2
      for (int d4 = 0; d4 < 32; ++d4) {
        const float4 k0v = *reinterpret_cast<const float4*>(kb + (bh + lane) * kRtLd + 4 * d4);
        const float4 k1v = *reinterpret_cast<const float4*>(kb + (bh + lane + 32) * kRtLd + 4 * d4);
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const float4 qv = *reinterpret_cast<const float4*>(qs + (rg + rr) * kRtLd + 4 * d4);
          acc[rr][0] = fmaf(qv.x, k0v.x, acc[rr][0]);
          acc[rr][0] = fmaf(qv.y, k0v.y, acc[rr][0]);
          acc[rr][0] = fmaf(qv.z, k0v.z, acc[rr][0]);
          acc[rr][0] = fmaf(qv.w, k0v.w, acc[rr][0]);
          acc[rr][1] = fmaf(qv.x, k1v.x, acc[rr][1]);
          acc[rr][1] = fmaf(qv.y, k1v.y, acc[rr][1]);
          acc[rr][1] = fmaf(qv.z, k1v.z, acc[rr][1]);
          acc[rr][1] = fmaf(qv.w, k1v.w, acc[rr][1]);
        }
      }
#pragma unroll
      for (int rr = 0; rr < 8; ++rr) {
        const int r = rg + rr;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int64_t c = c0 + bh + lane + 32 * h;
          if (c >= s1) continue;
          const float sdot = acc[rr][h];
          float z = fminf(fmaxf(sdot * inv_sqrt_d, -kActClamp), kActClamp);
          if (sdot != sdot) z = sdot;
          zs[r * kRlSpan + (c - s0)] = c < chi[r] ? z : kScoreNeg;
        }
      }
      __syncthreads();  // k_bar chunk reuse
    }
    __syncthreads();
    // this span's top-M of each of the warp's rows, merged into the running
    // list; with a candidate mask also the list of every remote block (the
    // fallback of a row whose candidate set turns out empty)
    for (int rr = 0; rr < 4; ++rr) {
      const int r = r0 + rr;
      const int64_t n = n0 + r;
      if (n >= a.N) break;  // warp-uniform
      for (int pass = 0; pass < (a.cand ? 2 : 1); ++pass) {
        const bool masked = a.cand && pass == 0;
        unsigned long long v[kRlSpan / 32];
        int f = 0;
#pragma unroll
        for (int k = 0; k < kRlSpan / 32; ++k) {
          const int64_t c = s0 + lane + 32 * k;
          v[k] = 0ull;
          if (c < s1) {
            const float zc = zs[r * kRlSpan + (c - s0)];
            const bool remote = zc > kScoreNeg * 0.5f;  // NaN -> not remote
            const bool cm = remote && (!masked || a.cand[n * a.s_cand + c] != 0);
            f |= masked && cm;
            float x = cm ? zc * a.idx_scale : kEntmaxNeg;
            if (!isfinite(x)) x = kEntmaxNeg;
            v[k] = pack_key(x, c, cm);
          }
        }
        if (masked && __any_sync(0xffffffffu, f) && lane == 0) found_s[r] = 1;
        unsigned long long (*lst)[kMaxTopM] = pass == 0 ? best : best_all;
        const unsigned long long top = warp_topm_filtered<kRlSpan / 32>(v, M, lane, topm_scratch[warp]);
        unsigned long long e0 = lane < M ? lst[r][lane] : 0ull;
        unsigned long long e1 = lane < M ? top : 0ull;
        bitonic64_desc(e0, e1, lane);
        __syncwarp();
        if (lane < M) lst[r][lane] = e0;
        __syncwarp();
      }
    }
    __syncthreads();  // zs reuse
  }
  for (int rr = 0; rr < 4; ++rr) {
    const int r = r0 + rr;
    const int64_t n = n0 + r;
    if (n >= a.N) break;  // warp-uniform
    float sel_v = 0.f;
    int sel_i = -1;
    bool sel_c = false;
    const bool fallback = a.cand && !found_s[r];  // no candidate among the remote blocks
    if (lane < M) unpack_key(fallback ? best_all[r][lane] : best[r][lane], sel_v, sel_i, sel_c);
    route_epilogue(a, n, lane, sel_v, sel_i, sel_c);
    __syncwarp();
  }
}

static int route_tile_long_launch(const RouteArgs& a, cudaStream_t st) {
  const size_t smem = route_tile_long_smem(a.nblk, a.block_table != nullptr);
  cudaError_t e = cudaFuncSetAttribute(route_tile_long_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return static_cast<int>(e);
  const int64_t grid = (a.N + kRtRows - 1) / kRtRows;
  if (grid >= (1ll << 31)) return SRSWA_ETOOLARGE;
  route_tile_long_kernel<<<static_cast<unsigned>(grid), kRouteThreads, smem, st>>>(a);
  return srswa_last_launch_status();
}

template <int NPLMAX>
static int route_tile_launch_npl(const RouteArgs& a, cudaStream_t st) {
  const size_t smem = route_tile_smem(a.nblk, a.block_table != nullptr);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(route_tile_kernel<NPLMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  const int64_t grid = (a.N + kRtRows - 1) / kRtRows;
  if (grid >= (1ll << 31)) return SRSWA_ETOOLARGE;
  route_tile_kernel<NPLMAX><<<static_cast<unsigned>(grid), kRouteThreads, smem, st>>>(a);
  return srswa_last_launch_status();
}

// Long rows of one sequence (> 1024 blocks), no scores output.
static bool use_tile_long(const RouteArgs& a) {
  return !a.from_scores && a.row_seq == nullptr && a.d == 128 && a.nblk > kRtMaxBlocks && a.scores_out == nullptr && (a.block_table == nullptr || a.nblk <= kRlMaxPagedBlocks) &&
         ((a.rows_per_seq == a.N && a.N >= kRtRows) || (a.rows_per_seq % kRtRows == 0 && a.N % kRtRows == 0));
}

static int route_tile_launch(const RouteArgs& a, cudaStream_t st) {
  return a.nblk <= 512 ? route_tile_launch_npl<16>(a, st) : route_tile_launch_npl<kRtMaxBlocks / 32>(a, st);
}

static bool use_wide(const RouteArgs& a) { return a.nblk >= 512 && a.nblk <= kWideMaxBlocks; }

static size_t chunk_workspace(int64_t N, int64_t nblk) {
  return (static_cast<size_t>(N * nblk) * 4 + 255) & ~static_cast<size_t>(255);
}

// Rows per CTA of route_kernel (several short rows share a CTA).
static int route_rows_per_cta(int64_t nblk) {
  int rpc = 1;
  while (rpc < 8 && nblk * rpc * 2 <= 2048) rpc *= 2;
  return rpc;
}

// Decode-shaped rows go to the chunked score pass + one-CTA-per-row select
// when they have many blocks, or when they are too few for route_kernel to
// give every SM a CTA (e.g. 32 decode rows of 256 blocks would be 8 CTAs of 4
// rows: 146 us against 25 us for the two chunked kernels).  A function of
// (N, nblk, d) only, so that srswa_route_workspace_size agrees with it.
constexpr int64_t kFewRowCtas = 148;
static bool use_chunked(const RouteArgs& a) {
  if (a.from_scores || a.d != 128 || a.nblk > kWideMaxBlocks) return false;
  if (use_wide(a)) return true;
  const int rpc = route_rows_per_cta(a.nblk);
  return (a.N + rpc - 1) / rpc < kFewRowCtas;
}

static int select_wide_launch(RouteArgs a, const float* z, int64_t s_z, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(a.nblk) * 8;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(select_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  if (a.N >= (1ll << 31)) return SRSWA_ETOOLARGE;
  // may start while the score kernel runs (it waits for the scores itself)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.N), 1, 1);
  cfg.blockDim = dim3(kRouteThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, select_wide_kernel, a, z, s_z);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

static int route_chunk_launch(RouteArgs a, void* ws, size_t ws_bytes, cudaStream_t st) {
  // scores go to the caller's scores output when requested, else to workspace
  float* z = a.scores_out;
  if (!z) {
    if (!ws || ws_bytes < chunk_workspace(a.N, a.nblk)) return SRSWA_EWORKSPACE;
    z = static_cast<float*>(ws);
  }
  const int64_t nch = (a.nblk + kChunkBlocks * kScoreReps - 1) / (kChunkBlocks * kScoreReps);
  // grid.y holds at most 65535 rows: longer row sets (prefill of >= 64k
  // tokens) take several launches, each complete before the next starts
  constexpr int64_t kMaxGridY = 65535;
  for (int64_t r0 = 0; r0 < a.N; r0 += kMaxGridY) {
    const int64_t nr = a.N - r0 < kMaxGridY ? a.N - r0 : kMaxGridY;
    route_score_kernel<<<dim3(static_cast<unsigned>(nch), static_cast<unsigned>(nr)), kRouteThreads, 0, st>>>(
        a, z, r0);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  a.scores_out = nullptr;  // already written
  return select_wide_launch(a, z, a.nblk, st);
}

// The rows of sequence b as a call of their own (one sequence, its rows
// first): pointers advanced past the earlier sequences' rows.
static RouteArgs route_seq_args(const RouteArgs& a, int64_t b) {
  RouteArgs s = a;
  const int64_t r0 = b * a.rows_per_seq;
  s.N = a.rows_per_seq;  // callers: N a multiple of rows_per_seq
  s.rows_per_seq = s.N;
  const int64_t esz = a.q_dtype == SRSWA_F32 ? 4 : 2;
  s.q = static_cast<const char*>(a.q) + r0 * a.s_q * esz;
  if (a.q_pos) s.q_pos = a.q_pos + r0;
  if (a.seq_lens) s.seq_lens = a.seq_lens + b;
  if (a.block_table) s.block_table = a.block_table + b * a.s_bt;
  else s.kbar = a.kbar + b * a.s_kbar_b;
  if (a.cand) s.cand = a.cand + r0 * a.s_cand;
  if (a.topi64) s.topi64 = a.topi64 + r0 * a.K;
  if (a.topi32) s.topi32 = a.topi32 + r0 * a.K;
  if (a.bias) s.bias = a.bias + r0 * a.K;
  if (a.valid) s.valid = a.valid + r0 * a.K;
  if (a.scores_out) s.scores_out = a.scores_out + r0 * a.nblk;
  return s;
}

static int route_launch(RouteArgs a, cudaStream_t st, void* ws = nullptr, size_t ws_bytes = 0) {
  if (a.N == 0) return 0;
  // prefill rows: many rows of one sequence sharing a contiguous k_bar
  if (use_tile(a)) return route_tile_launch(a, st);
  if (use_tile_long(a)) return route_tile_long_launch(a, st);
  // several sequences whose row count is not a multiple of the 32-row tile
  // (a tile would span two of them): the tiled routers once per sequence
  constexpr int64_t kMaxSeqLaunches = 64;
  if (!a.from_scores && a.row_seq == nullptr && a.rows_per_seq < a.N && a.rows_per_seq >= 4 * kRtRows &&
      a.N % a.rows_per_seq == 0 && a.N / a.rows_per_seq <= kMaxSeqLaunches) {
    const RouteArgs s0 = route_seq_args(a, 0);
    if (use_tile(s0) || use_tile_long(s0)) {
      for (int64_t b = 0; b < a.N / a.rows_per_seq; ++b) {
        const RouteArgs sb = route_seq_args(a, b);
        const int rc = use_tile(sb) ? route_tile_launch(sb, st) : route_tile_long_launch(sb, st);
        if (rc) return rc;
      }
      return 0;
    }
  }
  // decode-shaped rows with many candidate blocks -> chunked score + merge
  if (use_chunked(a)) return route_chunk_launch(a, ws, ws_bytes, st);
  if (a.from_scores && use_wide(a)) return select_wide_launch(a, a.scores_in, a.s_sc, st);
  const int rpc = route_rows_per_cta(a.nblk);
  a.rows_per_cta = rpc;
  const size_t smem = static_cast<size_t>(rpc) * a.nblk * (sizeof(float) + 1);
  if (smem > 227 * 1024) return SRSWA_ETOOLARGE;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  const int64_t grid = (a.N + rpc - 1) / rpc;
  if (grid >= (1ll << 31)) return SRSWA_ETOOLARGE;
  route_kernel<<<static_cast<unsigned>(grid), kRouteThreads, smem, st>>>(a);
  return srswa_last_launch_status();
}

static int fill_route_params(RouteArgs& a, const srswa_route_params& p, int64_t nblk) {
  if (p.block_size <= 0 || p.local_blocks < 0 || p.sigma == 0.f) return SRSWA_EINVAL;
  int64_t M = p.topm > 0 ? (p.topm < nblk ? p.topm : nblk) : nblk;
  if (M < 1) M = 1;
  if (M > kMaxTopM) return SRSWA_EUNSUPPORTED;
  int64_t K = p.topk < M ? p.topk : M;
  if (K < 1) K = 1;
  a.BS = p.block_size;
  a.L = p.local_blocks;
  a.M = M;
  a.K = K;
  a.idx_scale = p.idx_scale;
  a.floor_ = p.prior_floor;
  a.inv_sigma = static_cast<float>(1.0 / static_cast<double>(p.sigma));
  return 0;
}

}  // namespace srswa

using namespace srswa;

extern "C" int srswa_kbar_contig(const void* idx_k, int dtype, int64_t sb, int64_t st, int64_t B,
                                 int64_t S, int64_t d, int64_t block_size, const float* head_cls,
                                 float* kbar, uint8_t* chunk_valid, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(idx_k && head_cls && kbar && B >= 0 && S >= 0, SRSWA_EINVAL);
  const int64_t align = dtype == SRSWA_F32 ? 4 : 8;  // 16-byte vector loads
  SRSWA_CHECK_ARG(d > 0 && d <= 128 && d % align == 0, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG(block_size > 0 && block_size <= kMaxBlockSize, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG((sb % align) == 0 && (st % align) == 0 && (reinterpret_cast<uintptr_t>(idx_k) & 15) == 0,
                  SRSWA_EALIGN);
  const int64_t nblk = (S + block_size - 1) / block_size;
  if (B * nblk == 0) return 0;
  KbarArgs a = {};
  a.keys = idx_k; a.dtype = dtype; a.d = d; a.bs = block_size; a.hc = head_cls; a.out = kbar;
  a.chunk_valid = chunk_valid; a.sb = sb; a.st = st; a.S = S; a.nblk = nblk; a.B = B; a.paged = 0;
  return kbar_launch(a, B * nblk, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_kbar_paged(const void* idx_cache, int dtype, int64_t s_page, int64_t s_tok,
                                int64_t d, int64_t block_size, const int32_t* block_table, int64_t s_bt,
                                int64_t W, const int32_t* seq_lens, int64_t R, int64_t tail_pages,
                                const float* head_cls, float* kbar_cache, int64_t s_kbar,
                                srswa_stream_t stream) {
  SRSWA_CHECK_ARG(idx_cache && block_table && seq_lens && head_cls && kbar_cache, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(R >= 0 && W > 0, SRSWA_EINVAL);
  const int64_t align = dtype == SRSWA_F32 ? 4 : 8;  // 16-byte vector loads
  SRSWA_CHECK_ARG(d > 0 && d <= 128 && d % align == 0, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG(block_size > 0 && block_size <= kMaxBlockSize, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG((s_page % align) == 0 && (s_tok % align) == 0 &&
                      (reinterpret_cast<uintptr_t>(idx_cache) & 15) == 0,
                  SRSWA_EALIGN);
  const int64_t per = tail_pages > 0 ? tail_pages : W;
  if (R * per == 0) return 0;
  KbarArgs a = {};
  a.keys = idx_cache; a.dtype = dtype; a.d = d; a.bs = block_size; a.hc = head_cls; a.out = kbar_cache;
  a.st = s_tok; a.block_table = block_table; a.seq_lens = seq_lens; a.s_page = s_page; a.s_bt = s_bt;
  a.W = W; a.R = R; a.tail = tail_pages; a.s_kbar = s_kbar; a.paged = 1;
  return kbar_launch(a, R * per, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_kbar_pages(const void* idx_cache, int dtype, int64_t s_page, int64_t s_tok, int64_t d,
                                int64_t block_size, const int64_t* pages, const int32_t* tok, int64_t n,
                                const float* head_cls, float* kbar_cache, int64_t s_kbar, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(idx_cache && head_cls && kbar_cache && n >= 0 && (n == 0 || (pages && tok)), SRSWA_EINVAL);
  const int64_t align = dtype == SRSWA_F32 ? 4 : 8;  // 16-byte vector loads
  SRSWA_CHECK_ARG(d > 0 && d <= 128 && d % align == 0, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG(block_size > 0 && block_size <= kMaxBlockSize, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG((s_page % align) == 0 && (s_tok % align) == 0 &&
                      (reinterpret_cast<uintptr_t>(idx_cache) & 15) == 0,
                  SRSWA_EALIGN);
  if (n == 0) return 0;
  KbarArgs a = {};
  a.keys = idx_cache; a.dtype = dtype; a.d = d; a.bs = block_size; a.hc = head_cls; a.out = kbar_cache;
  a.st = s_tok; a.s_page = s_page; a.s_kbar = s_kbar; a.paged = 2;
  a.plan_pages = pages; a.plan_tok = tok; a.plan_n = n;
  return kbar_launch(a, n, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_route(const void* idx_q, int q_dtype, int64_t s_q, int64_t N, int64_t d,
                           const float* kbar, int64_t s_kbar_b, int64_t s_kbar_c, int64_t nblk,
                           const int32_t* block_table, int64_t s_bt, const int32_t* seq_lens,
                           int64_t rows_per_seq, const int32_t* row_seq, const int64_t* q_pos,
                           const uint8_t* cand, int64_t s_cand, srswa_route_params params, int64_t* topi64,
                           int32_t* topi32, float* bias, uint8_t* valid, float* scores,
                           void* workspace, size_t workspace_bytes, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(idx_q && kbar && N >= 0 && nblk > 0 && rows_per_seq > 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(q_pos || seq_lens, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(!row_seq || q_pos, SRSWA_EINVAL);  // varlen rows carry their positions
  SRSWA_CHECK_ARG(d == 128 || d == 64, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG((reinterpret_cast<uintptr_t>(kbar) & 15) == 0 && (s_kbar_b % 4) == 0 &&
                      (s_kbar_c % 4) == 0 && (s_q % 4) == 0,
                  SRSWA_EALIGN);
  RouteArgs a = {};
  int rc = fill_route_params(a, params, nblk);
  if (rc) return rc;
  a.from_scores = 0; a.q = idx_q; a.q_dtype = q_dtype; a.s_q = s_q; a.d = d; a.kbar = kbar;
  a.s_kbar_b = s_kbar_b; a.s_kbar_c = s_kbar_c; a.block_table = block_table; a.s_bt = s_bt;
  a.seq_lens = seq_lens; a.rows_per_seq = rows_per_seq; a.row_seq = row_seq; a.q_pos = q_pos; a.cand = cand;
  a.s_cand = s_cand; a.N = N; a.nblk = nblk; a.topi64 = topi64; a.topi32 = topi32; a.bias = bias;
  a.valid = valid; a.scores_out = scores;
  return route_launch(a, reinterpret_cast<cudaStream_t>(stream), workspace, workspace_bytes);
}

extern "C" size_t srswa_route_workspace_size(int64_t N, int64_t nblk, int64_t d, srswa_route_params params,
                                             int has_cand) {
  RouteArgs a = {};
  if (N < 0 || nblk <= 0 || fill_route_params(a, params, nblk)) return 0;
  a.d = d;
  a.nblk = nblk;
  a.N = N;
  (void)has_cand;
  if (!use_chunked(a)) return 0;
  return chunk_workspace(N, nblk);
}

extern "C" int srswa_route_select(const float* scores, int64_t s_sc, int64_t N, int64_t nblk,
                                  const uint8_t* cand, int64_t s_cand, srswa_route_params params,
                                  int64_t* topi64, int32_t* topi32, float* bias, uint8_t* valid,
                                  srswa_stream_t stream) {
  SRSWA_CHECK_ARG(scores && N >= 0 && nblk > 0, SRSWA_EINVAL);
  RouteArgs a = {};
  int rc = fill_route_params(a, params, nblk);
  if (rc) return rc;
  a.from_scores = 1; a.scores_in = scores; a.s_sc = s_sc; a.cand = cand; a.s_cand = s_cand;
  a.N = N; a.nblk = nblk; a.rows_per_seq = 1; a.topi64 = topi64; a.topi32 = topi32; a.bias = bias;
  a.valid = valid;
  return route_launch(a, reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- split-KV --
static int64_t shard_topm_bound(const srswa_route_params& p) {
  const int64_t M = p.topm > 0 ? p.topm : kMaxTopM;
  return M < kMaxTopM ? (M < 1 ? 1 : M) : kMaxTopM;
}

static int keys_merge_launch(const RouteArgs& a, const unsigned long long* keys, int64_t nlists, int64_t s_list,
                             int64_t s_row, unsigned long long* keys_out, int64_t own_lo, int64_t own_hi,
                             int32_t* topi32_own, const srswa_peer& wait, cudaStream_t st) {
  if (nlists * a.M > kMergeMaxKeys) return SRSWA_ETOOLARGE;
  if (a.N >= (1ll << 31)) return SRSWA_ETOOLARGE;
  const size_t smem = static_cast<size_t>(nlists * a.M) * 8;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(keys_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  keys_merge_kernel<<<static_cast<unsigned>(a.N), kRouteThreads, smem, st>>>(a, keys, nlists, s_list, s_row, keys_out,
                                                                             own_lo, own_hi, topi32_own, wait);
  return srswa_last_launch_status();
}

extern "C" size_t srswa_route_shard_workspace_size(int64_t N, int64_t nblk_local, srswa_route_params params) {
  if (N <= 0 || nblk_local <= 0) return 0;
  const int64_t nch = (nblk_local + kChunkBlocks - 1) / kChunkBlocks;
  if (nch == 1) return 0;
  const size_t cnt_bytes = (static_cast<size_t>(N) * 4 + 255) & ~static_cast<size_t>(255);
  return cnt_bytes + ((static_cast<size_t>(N * nch * shard_topm_bound(params)) * 8 + 255) & ~static_cast<size_t>(255));
}

// Stage 1 (and with fin.on the stage-2 merge and epilogue) of the split-KV
// router for this shard's blocks; checks shared by the two entry points.
static int shard_launch(const void* idx_q, int q_dtype, int64_t s_q, int64_t N, int64_t d, const float* kbar,
                        int64_t s_kbar_b, int64_t s_kbar_c, int64_t nblk_local, int64_t block_offset,
                        int64_t nblk_total, const int32_t* block_table, int64_t s_bt, const int32_t* seq_lens,
                        int64_t rows_per_seq, const int64_t* q_pos, const srswa_route_params& params,
                        RouteArgs& a, uint64_t* keys_out, void* workspace, size_t workspace_bytes,
                        const srswa_peer* push, const ShardFinish& fin, cudaStream_t st) {
  SRSWA_CHECK_ARG(idx_q && kbar && N >= 0 && rows_per_seq > 0, SRSWA_EINVAL);
  srswa_peer pp = {};
  if (push) {
    SRSWA_CHECK_ARG(push->regions && push->own_region && push->counter && push->tickets && push->world >= 1 &&
                        push->world <= 32 && push->rank >= 0 && push->rank < push->world,
                    SRSWA_EINVAL);
    pp = *push;
  }
  SRSWA_CHECK_ARG(nblk_local > 0 && block_offset >= 0 && block_offset + nblk_local <= nblk_total, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(q_pos || seq_lens, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(d == 128, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG((reinterpret_cast<uintptr_t>(kbar) & 15) == 0 && (s_kbar_b % 4) == 0 && (s_kbar_c % 4) == 0 &&
                      (s_q % 4) == 0,
                  SRSWA_EALIGN);
  int rc = fill_route_params(a, params, nblk_total);
  if (rc) return rc;
  a.from_scores = 0; a.q = idx_q; a.q_dtype = q_dtype; a.s_q = s_q; a.d = d; a.kbar = kbar;
  a.s_kbar_b = s_kbar_b; a.s_kbar_c = s_kbar_c; a.block_table = block_table; a.s_bt = s_bt;
  a.seq_lens = seq_lens; a.rows_per_seq = rows_per_seq; a.q_pos = q_pos; a.N = N; a.nblk = nblk_total;
  if (N == 0) return 0;
  SRSWA_CHECK_ARG(N < 65536, SRSWA_ETOOLARGE);
  const int64_t nch = (nblk_local + kChunkBlocks - 1) / kChunkBlocks;
  unsigned long long* out = reinterpret_cast<unsigned long long*>(keys_out);
  SRSWA_CHECK_ARG(!push || N * a.M * (push->ll ? 16 : 8) <= push->slot_bytes, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(!push || !push->ll || fin.on, SRSWA_EUNSUPPORTED);  // LL: keys are merged in the same launch
  // the ranks' lists of a row are merged in the same shared array as its chunk lists
  const int64_t lists = fin.on && push ? (nch > push->world ? nch : push->world) : (nch > 1 ? nch : 0);
  SRSWA_CHECK_ARG(lists * a.M <= kMergeMaxKeys, SRSWA_ETOOLARGE);
  const size_t smem = static_cast<size_t>(lists * a.M) * 8;
  if (smem > 40 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(route_chunk_keys_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  unsigned int* counters = nullptr;
  unsigned long long* ck = nullptr;
  if (nch > 1) {
    const size_t cnt_bytes = (static_cast<size_t>(N) * 4 + 255) & ~static_cast<size_t>(255);
    const size_t need = cnt_bytes + static_cast<size_t>(N * nch * a.M) * 8;
    SRSWA_CHECK_ARG(workspace && workspace_bytes >= need, SRSWA_EWORKSPACE);
    counters = static_cast<unsigned int*>(workspace);
    ck = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) + cnt_bytes);
    SRSWA_CUDA_TRY(cudaMemsetAsync(counters, 0, static_cast<size_t>(N) * 4, st));
  }
  route_chunk_keys_kernel<<<dim3(static_cast<unsigned>(nch), static_cast<unsigned>(N)), kRouteThreads, smem, st>>>(
      a, block_offset, nblk_local, ck, counters, out, pp, fin);
  return srswa_last_launch_status();
}

extern "C" int srswa_route_shard_keys(const void* idx_q, int q_dtype, int64_t s_q, int64_t N, int64_t d,
                                      const float* kbar, int64_t s_kbar_b, int64_t s_kbar_c, int64_t nblk_local,
                                      int64_t block_offset, int64_t nblk_total, const int32_t* block_table,
                                      int64_t s_bt, const int32_t* seq_lens, int64_t rows_per_seq,
                                      const int64_t* q_pos, srswa_route_params params, uint64_t* keys_out,
                                      void* workspace, size_t workspace_bytes, const srswa_peer* push,
                                      srswa_stream_t stream) {
  SRSWA_CHECK_ARG(keys_out, SRSWA_EINVAL);
  RouteArgs a = {};
  const ShardFinish fin = {};
  return shard_launch(idx_q, q_dtype, s_q, N, d, kbar, s_kbar_b, s_kbar_c, nblk_local, block_offset, nblk_total,
                      block_table, s_bt, seq_lens, rows_per_seq, q_pos, params, a, keys_out, workspace,
                      workspace_bytes, push, fin, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_route_shard_select(const void* idx_q, int q_dtype, int64_t s_q, int64_t N, int64_t d,
                                        const float* kbar, int64_t s_kbar_b, int64_t s_kbar_c, int64_t nblk_local,
                                        int64_t block_offset, int64_t nblk_total, const int32_t* block_table,
                                        int64_t s_bt, const int32_t* seq_lens, int64_t rows_per_seq,
                                        const int64_t* q_pos, srswa_route_params params, int64_t* topi64,
                                        int32_t* topi32, float* bias, uint8_t* valid, int64_t own_lo,
                                        int64_t own_hi, int32_t* topi32_own, void* workspace,
                                        size_t workspace_bytes, const srswa_peer* exchange,
                                        srswa_stream_t stream) {
  // the row's last CTA waits for the peers: every such CTA must be resident
  // while the other CTAs of the grid still run
  SRSWA_CHECK_ARG(!exchange || N <= kShardSelectMaxRowsPeer, SRSWA_ETOOLARGE);
  RouteArgs a = {};
  a.topi64 = topi64; a.topi32 = topi32; a.bias = bias; a.valid = valid;
  ShardFinish fin = {};
  fin.on = 1; fin.own_lo = own_lo; fin.own_hi = own_hi; fin.topi32_own = topi32_own;
  return shard_launch(idx_q, q_dtype, s_q, N, d, kbar, s_kbar_b, s_kbar_c, nblk_local, block_offset, nblk_total,
                      block_table, s_bt, seq_lens, rows_per_seq, q_pos, params, a, nullptr, workspace,
                      workspace_bytes, exchange, fin, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_route_merge_keys(const uint64_t* keys, int64_t nlists, int64_t s_list, int64_t s_row, int64_t N,
                                      int64_t nblk_total, srswa_route_params params, int64_t* topi64,
                                      int32_t* topi32, float* bias, uint8_t* valid, int64_t own_lo, int64_t own_hi,
                                      int32_t* topi32_own, const srswa_peer* wait, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(keys && nlists > 0 && N >= 0 && nblk_total > 0, SRSWA_EINVAL);
  srswa_peer pw = {};
  if (wait) {
    SRSWA_CHECK_ARG(wait->regions && wait->own_region && wait->counter && wait->tickets && wait->world >= 1 &&
                        wait->world <= 32,
                    SRSWA_EINVAL);
    SRSWA_CHECK_ARG(!wait->ll, SRSWA_EUNSUPPORTED);
    pw = *wait;
  }
  RouteArgs a = {};
  int rc = fill_route_params(a, params, nblk_total);
  if (rc) return rc;
  SRSWA_CHECK_ARG(s_list >= 0 && s_row >= a.M, SRSWA_EINVAL);
  a.N = N; a.nblk = nblk_total; a.topi64 = topi64; a.topi32 = topi32; a.bias = bias; a.valid = valid;
  if (N == 0) return 0;
  return keys_merge_launch(a, reinterpret_cast<const unsigned long long*>(keys), nlists, s_list, s_row, nullptr,
                           own_lo, own_hi, topi32_own, pw, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_block_max_score(const void* q, int q_dtype, int64_t sqb, int64_t sqc, const void* k,
                                     int k_dtype, int64_t skb, int64_t sks, const int64_t* pos,
                                     const int64_t* seg, int64_t B, int64_t C, int64_t Sk, int64_t D,
                                     int64_t block_size, int64_t nblk, int64_t local_window, int mode,
                                     float* out, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(q && k && pos && out && B >= 0 && C >= 0 && Sk >= 0 && nblk >= 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(mode == 0 || mode == 1, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(D > 0 && D <= 256, SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG(block_size > 0 && block_size <= 128, SRSWA_EUNSUPPORTED);
  if (B * C * nblk == 0) return 0;
  SRSWA_CHECK_ARG(nblk < 65536 && B < 65536, SRSWA_ETOOLARGE);
  BlockMaxArgs a = {};
  a.q = q; a.q_dtype = q_dtype; a.sqb = sqb; a.sqc = sqc; a.k = k; a.k_dtype = k_dtype; a.skb = skb;
  a.sks = sks; a.pos = pos; a.seg = seg; a.B = B; a.C = C; a.Sk = Sk; a.D = D; a.BS = block_size;
  a.nblk = nblk; a.LW = local_window > 0 ? local_window : block_size; a.mode = mode; a.out = out;
  const size_t smem = static_cast<size_t>(kBmQ + block_size) * (D + 1) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(block_max_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  dim3 grid(static_cast<unsigned>((C + kBmQ - 1) / kBmQ), static_cast<unsigned>(nblk), static_cast<unsigned>(B));
  block_max_kernel<<<grid, 256, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return srswa_last_launch_status();
}

extern "C" int srswa_pack_selection(const void* sel, int is64, int64_t rows, int64_t S, int64_t nblk,
                                    int32_t* out, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(rows >= 0 && S >= 0, SRSWA_EINVAL);
  if (rows * S == 0) return 0;
  SRSWA_CHECK_ARG(sel && out, SRSWA_EINVAL);
  pack_selection_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(sel, is64, rows, S, nblk, out);
  return srswa_last_launch_status();
}
