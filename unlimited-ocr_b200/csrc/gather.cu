// Fused gather-attention forward / backward entry points (a6, a7).
//
// Forward: query-major streaming over (selected remote blocks U local window)
// with the row-streaming kernel of attend.cu.
//
// Backward (deterministic, no atomics on floating-point data):
//   1. delta[b,t,h] = sum_d o*dO                            (bwd_delta_kernel)
//   2. dQ and per-head d_bias partials, query-major          (bwd_dq_kernel)
//   3. d_bias = sum over heads of the partials, fixed order  (bwd_dbias_reduce_kernel)
//   4. bitmap[b,hi,blk,t] = query t selected block blk      (bwd_bitmap_kernel;
//      integer atomicOr, order-independent)
//   5. dK/dV key-block-major: each CTA owns one (b, kv head, block) and walks
//      the local-window queries and the bitmap's queries in increasing t
//                                                            (bwd_dkdv_kernel)
// Math: P = exp(s - lse), dP = dO V^T, dS = P (dP - delta), dQ = scale dS K,
// dK = scale dS^T Q, dV = P^T dO, d_bias[t,slot] = sum_{h, remote keys of slot} dS
// (hf-model-code/sparse_gather_triton.py:125-279, 324-353;
//  sparse_gather_e2e_triton.py:124-275, 324-352).

#include "attend.cuh"
#include "common.cuh"

namespace srswa {

struct BwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;
  const int32_t* sel;
  const float* bias;
  const int32_t* seg;
  void* dq;
  void* dk;
  void* dv;
  float* d_bias;
  float* delta;     // [B,T,HQ]
  float* dbias_part;  // [B,T,HQ,S]
  uint32_t* bitmap;   // [B,HI,nblk,T32]
  int dtype;
  int64_t B, T, HQ, Hkv, HI, D, S, BS, LW, nblk, T32;
  float scale;
  int64_t sqb, sqt, sqh, skb, skt, skh, svb, svt, svh, sob, sot, soh;
};

__device__ __forceinline__ int64_t seg_of(const BwdArgs& a, int64_t b, int64_t t) {
  return a.seg ? static_cast<int64_t>(a.seg[b * a.T + t]) : 0;
}

// ---- 1. delta -------------------------------------------------------------
__global__ void bwd_delta_kernel(const BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (item >= a.B * a.T * a.HQ) return;
  const int64_t h = item % a.HQ, bt = item / a.HQ, t = bt % a.T, b = bt / a.T;
  float acc = 0.f;
  for (int64_t d = lane; d < a.D; d += 32) {
    const float ov = load_elem(a.o, b * a.sob + t * a.sot + h * a.soh + d, a.dtype);
    const float gv = load_elem(a.dout, b * a.sob + t * a.sot + h * a.soh + d, a.dtype);
    acc = fmaf(ov, gv, acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) a.delta[item] = acc;
}

// ---- 2. dQ + d_bias partials, one (b,t,h) row per CTA --------------------
struct BwdSlot {
  int64_t key0;
  float bias;
  int slot;
  int remote;
};

template <int D, int KVT>
__global__ void __launch_bounds__(kAttendThreads) bwd_dq_kernel(const BwdArgs a) {
  constexpr int LPK = D / 8;
  constexpr int KPI = 32 / LPK;
  constexpr int KPC = KPI * 8;
  __shared__ BwdSlot slots[kAttendMaxSlots];
  __shared__ int n_slots;
  __shared__ float db_w[kAttendWarps][kAttendMaxSlots];
  __shared__ __align__(16) float dq_w[kAttendWarps][D];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t row = blockIdx.x;  // b*T + t
  const int h = blockIdx.y;
  const int64_t b = row / a.T, t = row % a.T;
  const int hk = static_cast<int>(h / (a.HQ / a.Hkv));
  const int hi = static_cast<int>((static_cast<int64_t>(hk) * a.HI) / a.Hkv);
  const int64_t BS = a.BS, sg = seg_of(a, b, t);
  int64_t ls = t - a.LW + 1;
  if (ls < sg) ls = sg;
  if (ls < 0) ls = 0;

  for (int i = tid; i < kAttendWarps * kAttendMaxSlots; i += kAttendThreads) (&db_w[0][0])[i] = 0.f;
  if (tid == 0) {
    int n = 0;
    const int32_t* srow = a.sel + ((b * a.HI + hi) * a.T + t) * a.S;
    for (int64_t s = 0; s < a.S && n < kAttendMaxSlots; ++s) {
      const int64_t blk = srow[s];
      if (blk < 0 || blk >= a.nblk) continue;
      const int64_t lo = blk * BS > sg ? blk * BS : sg;
      const int64_t hi_ = (blk + 1) * BS < ls ? (blk + 1) * BS : ls;
      if (lo >= hi_ || lo > t) continue;
      bool dup = false;
      for (int j = 0; j < n; ++j) dup |= (slots[j].key0 == blk * BS);
      if (dup) continue;
      slots[n].key0 = blk * BS;
      slots[n].bias = a.bias ? a.bias[(b * a.T + t) * a.S + s] : 0.f;
      slots[n].slot = static_cast<int>(s);
      slots[n].remote = 1;
      ++n;
    }
    for (int64_t blk = ls / BS; blk <= t / BS && n < kAttendMaxSlots; ++blk) {
      slots[n].key0 = blk * BS;
      slots[n].bias = 0.f;
      slots[n].slot = -1;
      slots[n].remote = 0;
      ++n;
    }
    n_slots = n;
  }
  __syncthreads();

  const int g = lane / LPK, u = lane % LPK;
  float qv[8], gv[8];
  load8(a.q, b * a.sqb + t * a.sqt + h * a.sqh + u * 8, a.dtype, qv);
  load8(a.dout, b * a.sob + t * a.sot + h * a.soh + u * 8, a.dtype, gv);
  const float lse = a.lse[row * a.HQ + h];
  const float dlt = a.delta[row * a.HQ + h];
  const float sc = a.scale;
  const int count_lane = (u & (LPK / 8 - 1)) == 0;
  const int my_idx = 4 * ((u & (LPK / 2)) != 0) + 2 * ((u & (LPK / 4)) != 0) + ((u & (LPK / 8)) != 0);
  float dq[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) dq[e] = 0.f;

  const int cpb = static_cast<int>(BS / KPC);
  const int nch = n_slots * cpb;
  for (int ch = warp; ch < nch; ch += kAttendWarps) {
    const BwdSlot si = slots[ch / cpb];
    const int sub = ch % cpb;
    const int64_t k0 = si.key0 + static_cast<int64_t>(sub) * KPC;
    int64_t lo, hi_;
    if (si.remote) { lo = k0 > sg ? k0 : sg; hi_ = min(min(k0 + KPC, t + 1), ls); }
    else { lo = k0 > ls ? k0 : ls; hi_ = min(k0 + KPC, t + 1); }
    if (lo >= hi_ || lse == -INFINITY) continue;
    uint4 kr[8], vr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t pos = k0 + i * KPI + g;
      if (pos >= lo && pos < hi_) {
        kr[i] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned short*>(a.k) +
                                                     b * a.skb + pos * a.skt + hk * a.skh + u * 8));
        vr[i] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned short*>(a.v) +
                                                     b * a.svb + pos * a.svt + hk * a.svh + u * 8));
      } else {
        kr[i] = make_uint4(0, 0, 0, 0);
        vr[i] = make_uint4(0, 0, 0, 0);
      }
    }
    float ps[8], pd[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float fk[8], fv[8];
      unpack8<KVT>(kr[i], fk);
      unpack8<KVT>(vr[i], fv);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) { s1 = fmaf(qv[e], fk[e], s1); s2 = fmaf(gv[e], fv[e], s2); }
      ps[i] = s1;
      pd[i] = s2;
    }
    const float s = transpose_reduce8<LPK>(ps, u);
    const float dp = transpose_reduce8<LPK>(pd, u);
    const int64_t my_pos = k0 + my_idx * KPI + g;
    const bool ok = my_pos >= lo && my_pos < hi_;
    const float pr = ok ? expf(s * sc + si.bias - lse) : 0.f;
    const float ds = pr * (dp - dlt);
    if (si.remote) {
      const float tot = warp_sum(count_lane ? ds : 0.f);
      if (lane == 0) db_w[warp][ch / cpb] += tot;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float di = __shfl_sync(0xffffffffu, ds, g * LPK + transpose_owner<LPK>(i));
      float fk[8];
      unpack8<KVT>(kr[i], fk);
#pragma unroll
      for (int e = 0; e < 8; ++e) dq[e] = fmaf(di, fk[e], dq[e]);
    }
  }
#pragma unroll
  for (int msk = LPK; msk < 32; msk <<= 1) {
#pragma unroll
    for (int e = 0; e < 8; ++e) dq[e] += __shfl_xor_sync(0xffffffffu, dq[e], msk);
  }
  if (lane < LPK) {
#pragma unroll
    for (int e = 0; e < 8; ++e) dq_w[warp][u * 8 + e] = dq[e];
  }
  __syncthreads();
  for (int d = tid; d < D; d += kAttendThreads) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAttendWarps; ++w) acc += dq_w[w][d];
    store_elem(a.dq, b * a.sqb + t * a.sqt + h * a.sqh + d, a.dtype, acc * sc);
  }
  if (a.dbias_part) {
    float* part = a.dbias_part + (row * a.HQ + h) * a.S;
    for (int64_t s = tid; s < a.S; s += kAttendThreads) part[s] = 0.f;
    __syncthreads();
    if (tid == 0) {
      for (int i = 0; i < n_slots; ++i) {
        if (!slots[i].remote) continue;
        float acc = 0.f;
        for (int w = 0; w < kAttendWarps; ++w) acc += db_w[w][i];
        part[slots[i].slot] = acc;
      }
    }
  }
}

// ---- 3. d_bias reduce over heads ----------------------------------------
__global__ void bwd_dbias_reduce_kernel(const BwdArgs a) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= a.B * a.T * a.S) return;
  const int64_t row = i / a.S, s = i % a.S;
  float acc = 0.f;
  for (int64_t h = 0; h < a.HQ; ++h) acc += a.dbias_part[(row * a.HQ + h) * a.S + s];
  a.d_bias[i] = acc;
}

// ---- 4. selection bitmap --------------------------------------------------
__global__ void bwd_bitmap_kernel(const BwdArgs a) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (b,hi,t)
  if (i >= a.B * a.HI * a.T) return;
  const int64_t t = i % a.T, bh = i / a.T, b = bh / a.HI;
  const int64_t sg = seg_of(a, b, t);
  int64_t ls = t - a.LW + 1;
  if (ls < sg) ls = sg;
  if (ls < 0) ls = 0;
  const int32_t* srow = a.sel + i * a.S;
  for (int64_t s = 0; s < a.S; ++s) {
    const int64_t blk = srow[s];
    if (blk < 0 || blk >= a.nblk) continue;
    const int64_t lo = blk * a.BS > sg ? blk * a.BS : sg;
    const int64_t hi_ = (blk + 1) * a.BS < ls ? (blk + 1) * a.BS : ls;
    if (lo >= hi_ || lo > t) continue;
    atomicOr(a.bitmap + (bh * a.nblk + blk) * a.T32 + t / 32, 1u << (t % 32));
  }
}

// ---- 5. dK/dV, one (b, kv head, key block) per CTA -----------------------
// thread -> key j = tid / 4 of the block, features [(tid%4)*D/4, +D/4)
template <int D>
__global__ void __launch_bounds__(256) bwd_dkdv_kernel(const BwdArgs a) {
  constexpr int FPT = D / 4;
  const int tid = threadIdx.x;
  const int64_t c = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int64_t BS = a.BS;
  const int jj = tid >> 2, f0 = (tid & 3) * FPT;
  const int64_t j = c * BS + jj;
  const bool key_ok = jj < BS && j < a.T;
  const int hi = static_cast<int>((hk * a.HI) / a.Hkv);
  const int64_t G = a.HQ / a.Hkv;
  float kf[FPT], vf[FPT], dk[FPT], dv[FPT];
#pragma unroll
  for (int e = 0; e < FPT; ++e) {
    kf[e] = key_ok ? load_elem(a.k, b * a.skb + j * a.skt + hk * a.skh + f0 + e, a.dtype) : 0.f;
    vf[e] = key_ok ? load_elem(a.v, b * a.svb + j * a.svt + hk * a.svh + f0 + e, a.dtype) : 0.f;
    dk[e] = 0.f;
    dv[e] = 0.f;
  }
  const uint32_t* bits = a.bitmap + ((b * a.HI + hi) * a.nblk + c) * a.T32;
  const int64_t loc_lo = c * BS, loc_hi = min(a.T, (c + 1) * BS - 1 + a.LW);  // [lo, hi)

  auto visit = [&](int64_t t) {
    const int64_t sg = seg_of(a, b, t);
    int64_t ls = t - a.LW + 1;
    if (ls < sg) ls = sg;
    if (ls < 0) ls = 0;
    const bool sel = (bits[t / 32] >> (t % 32)) & 1u;
    float bias = 0.f;
    if (sel && a.bias) {
      const int32_t* srow = a.sel + ((b * a.HI + hi) * a.T + t) * a.S;
      for (int64_t s = 0; s < a.S; ++s)
        if (srow[s] == c) { bias = a.bias[(b * a.T + t) * a.S + s]; break; }
    }
    const bool is_local = key_ok && j >= ls && j <= t;
    const bool is_remote = key_ok && sel && j >= sg && j < ls && j <= t;
    for (int64_t gq = 0; gq < G; ++gq) {
      const int64_t h = hk * G + gq;
      const float lse = a.lse[(b * a.T + t) * a.HQ + h];
      const float dlt = a.delta[(b * a.T + t) * a.HQ + h];
      float qf[FPT], gf[FPT];
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int e = 0; e < FPT; ++e) {
        qf[e] = load_elem(a.q, b * a.sqb + t * a.sqt + h * a.sqh + f0 + e, a.dtype);
        gf[e] = load_elem(a.dout, b * a.sob + t * a.sot + h * a.soh + f0 + e, a.dtype);
        s1 = fmaf(qf[e], kf[e], s1);
        s2 = fmaf(gf[e], vf[e], s2);
      }
      s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
      s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
      s2 += __shfl_xor_sync(0xffffffffu, s2, 2);
      float p = 0.f;
      if ((is_local || is_remote) && lse != -INFINITY)
        p = expf(s1 * a.scale + (is_remote ? bias : 0.f) - lse);
      const float ds = p * (s2 - dlt) * a.scale;
#pragma unroll
      for (int e = 0; e < FPT; ++e) {
        dv[e] = fmaf(p, gf[e], dv[e]);
        dk[e] = fmaf(ds, qf[e], dk[e]);
      }
    }
  };
  for (int64_t t = loc_lo; t < loc_hi; ++t) visit(t);
  // remote queries beyond the local range, increasing t
  for (int64_t w = loc_hi / 32; w < a.T32; ++w) {
    uint32_t word = bits[w];
    if (w * 32 < loc_hi) word &= ~((loc_hi - w * 32 >= 32) ? 0xffffffffu : ((1u << (loc_hi - w * 32)) - 1u));
    while (word) {
      const int bit = __ffs(word) - 1;
      word &= word - 1;
      visit(w * 32 + bit);
    }
  }
  if (key_ok) {
#pragma unroll
    for (int e = 0; e < FPT; ++e) {
      store_elem(a.dk, b * a.skb + j * a.skt + hk * a.skh + f0 + e, a.dtype, dk[e]);
      store_elem(a.dv, b * a.svb + j * a.svt + hk * a.svh + f0 + e, a.dtype, dv[e]);
    }
  }
}

static size_t align_up(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct BwdLayout {
  size_t delta, part, bitmap, total;
};
static BwdLayout bwd_layout(const srswa_gather_desc* g, bool with_bias) {
  BwdLayout L;
  const int64_t nblk = (g->T + g->block_size - 1) / g->block_size;
  const int64_t T32 = (g->T + 31) / 32;
  L.delta = 0;
  size_t off = align_up(static_cast<size_t>(g->B * g->T * g->HQ) * sizeof(float));
  L.part = off;
  if (with_bias) off += align_up(static_cast<size_t>(g->B * g->T * g->HQ * g->S) * sizeof(float));
  L.bitmap = off;
  off += align_up(static_cast<size_t>(g->B * g->HI * nblk * T32) * sizeof(uint32_t));
  L.total = off;
  return L;
}

static int check_gather_desc(const srswa_gather_desc* g) {
  if (!g) return SRSWA_EINVAL;
  if (g->B < 0 || g->T < 0 || g->HQ <= 0 || g->Hkv <= 0 || g->HI <= 0 || g->S < 0) return SRSWA_EINVAL;
  if (g->HQ % g->Hkv || g->HQ % g->HI || g->Hkv % g->HI) return SRSWA_EINVAL;
  if (g->block_size <= 0) return SRSWA_EINVAL;
  if (!(g->D == 64 || g->D == 128)) return SRSWA_EUNSUPPORTED;
  if (!(g->dtype == SRSWA_BF16 || g->dtype == SRSWA_F16)) return SRSWA_EUNSUPPORTED;
  if (g->block_size > 64 || (g->block_size % ((32 / (g->D / 8)) * 8))) return SRSWA_EUNSUPPORTED;
  if (((g->sqb | g->sqt | g->sqh | g->skb | g->skt | g->skh | g->svb | g->svt | g->svh) & 7) != 0)
    return SRSWA_EALIGN;
  return 0;
}

}  // namespace srswa

using namespace srswa;

namespace srswa {
TcLayout tc_layout(const srswa_gather_desc* g, int64_t qoff);
bool tc_eligible(const srswa_gather_desc* g);
bool tc_paged_eligible(const srswa_gather_desc* g, int64_t qoff);
int tc_gather_fwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v, const int32_t* sel,
                  const float* bias, const int32_t* seg, void* o, int64_t sob, int64_t sot, int64_t soh, float* lse,
                  void* workspace, size_t workspace_bytes, int* status, cudaStream_t st,
                  const TcPagedKV* pk = nullptr);
size_t tc_bwd_workspace(const srswa_gather_desc* g, bool with_bias);
int tc_gather_bwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v, const void* o,
                  int64_t sob, int64_t sot, int64_t soh, const void* dout, const float* lse, const int32_t* sel,
                  const float* bias, const int32_t* seg, void* dq, void* dk, void* dv, float* d_bias,
                  void* workspace, size_t workspace_bytes, int* status, cudaStream_t st);

// The first kStatusBytes of every gather workspace hold the call's status
// word (int32): cleared at the start of the call, set by a tensor-core kernel
// whose bounded wait expired.  The rest of the workspace follows.
constexpr size_t kStatusBytes = 256;

// Clears the status word at the workspace head and returns it (null when the
// caller gave no workspace); advances the workspace past it.
static int take_status(void** workspace, size_t* bytes, int** status, cudaStream_t st) {
  *status = nullptr;
  if (*workspace == nullptr || *bytes < kStatusBytes) {
    *workspace = nullptr;
    *bytes = 0;
    return 0;
  }
  *status = static_cast<int*>(*workspace);
  SRSWA_CUDA_TRY(cudaMemsetAsync(*status, 0, sizeof(int), st));
  *workspace = static_cast<char*>(*workspace) + kStatusBytes;
  *bytes -= kStatusBytes;
  return 0;
}

// The tensor-core backward takes bf16 / head dim 128 / 64-token blocks with
// 8-element-aligned strides (o and do included); other shapes use the
// CUDA-core kernels below.
static bool tc_bwd_path(const srswa_gather_desc* g, int64_t sob, int64_t sot, int64_t soh) {
  return tc_eligible(g) && ((sob | sot | soh) & 7) == 0;
}
// The tensor-core workspace also fits the CUDA-core kernels, which take over
// when the driver refuses a tensor map.
static size_t bwd_need(const srswa_gather_desc* g, int64_t sob, int64_t sot, int64_t soh, bool with_bias) {
  const size_t cc = bwd_layout(g, with_bias).total;
  if (!tc_bwd_path(g, sob, sot, soh)) return cc;
  const size_t tc = tc_bwd_workspace(g, with_bias);
  return tc > cc ? tc : cc;
}
}  // namespace srswa

extern "C" size_t srswa_gather_fwd_workspace_size(const srswa_gather_desc* g) {
  if (check_gather_desc(g)) return 0;
  return kStatusBytes + (tc_eligible(g) ? tc_layout(g, 0).total : 0);
}

extern "C" size_t srswa_gather_fwd_paged_workspace_size(const srswa_gather_desc* g, int64_t qoff) {
  if (check_gather_desc(g) || !tc_paged_eligible(g, qoff)) return 0;
  return kStatusBytes + tc_layout(g, qoff).total;
}

extern "C" int srswa_gather_fwd_paged(const srswa_gather_desc* g, const void* q, const void* k_cache,
                                      const void* v_cache, int64_t num_pages, const int32_t* pages, int64_t qoff,
                                      const int32_t* sel, const float* bias, void* o, int64_t sob, int64_t sot,
                                      int64_t soh, float* lse, void* workspace, size_t workspace_bytes,
                                      srswa_stream_t stream) {
  int rc = check_gather_desc(g);
  if (rc) return rc;
  SRSWA_CHECK_ARG(q && k_cache && v_cache && pages && o && num_pages > 0 && (g->S == 0 || sel), SRSWA_EINVAL);
  SRSWA_CHECK_ARG(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) |
                    reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(o)) & 15) == 0, SRSWA_EALIGN);
  // tensor cores only: bf16, D = 128, 64-token pages, one sequence
  SRSWA_CHECK_ARG(tc_paged_eligible(g, qoff) && ((sob | sot | soh) & 7) == 0, SRSWA_EUNSUPPORTED);
  if (g->T == 0) return 0;
  SRSWA_CHECK_ARG(workspace && workspace_bytes >= kStatusBytes + tc_layout(g, qoff).total, SRSWA_EWORKSPACE);
  int* status = nullptr;
  rc = take_status(&workspace, &workspace_bytes, &status, reinterpret_cast<cudaStream_t>(stream));
  if (rc) return rc;
  TcPagedKV pk = {num_pages, pages, 0, qoff};
  rc = tc_gather_fwd(g, q, k_cache, v_cache, sel, bias, nullptr, o, sob, sot, soh, lse, workspace, workspace_bytes,
                     status, reinterpret_cast<cudaStream_t>(stream), &pk);
  return rc == kTcNoTensorMap ? SRSWA_EUNSUPPORTED : rc;
}

extern "C" int srswa_gather_fwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v,
                                const int32_t* sel, const float* bias, const int32_t* seg, void* o,
                                int o_dtype, int64_t sob, int64_t sot, int64_t soh, float* lse,
                                void* workspace, size_t workspace_bytes, srswa_stream_t stream) {
  int rc = check_gather_desc(g);
  if (rc) return rc;
  SRSWA_CHECK_ARG(q && k && v && o && (g->S == 0 || sel), SRSWA_EINVAL);
  SRSWA_CHECK_ARG(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                    reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15) == 0, SRSWA_EALIGN);
  if (g->B * g->T == 0) return 0;
  int* status = nullptr;
  rc = take_status(&workspace, &workspace_bytes, &status, reinterpret_cast<cudaStream_t>(stream));
  if (rc) return rc;
  // tensor-core path (bf16, D = 128, 64-token blocks); CUDA-core rows otherwise
  if (tc_eligible(g) && o_dtype == SRSWA_BF16 && ((sob | sot | soh) & 7) == 0) {
    rc = tc_gather_fwd(g, q, k, v, sel, bias, seg, o, sob, sot, soh, lse, workspace, workspace_bytes, status,
                       reinterpret_cast<cudaStream_t>(stream));
    if (rc != kTcNoTensorMap) return rc;
  }
  const int64_t nblk = (g->T + g->block_size - 1) / g->block_size;
  AttendArgs a = {};
  a.q = q; a.k = k; a.v = v; a.q_dtype = g->dtype; a.out_dtype = o_dtype;
  a.N = g->B * g->T; a.rps = g->T; a.H = g->HQ; a.Hkv = g->Hkv;
  a.seg = seg; a.pos_mode = 2;
  a.block_table = nullptr; a.W = nblk;
  a.s_seq = g->skb; a.s_blk = g->block_size * g->skt; a.s_pos = g->skt; a.s_head = g->skh;
  // v shares k's layout in this kernel
  SRSWA_CHECK_ARG(g->svb == g->skb && g->svt == g->skt && g->svh == g->skh, SRSWA_EUNSUPPORTED);
  a.sel = sel; a.idx_is64 = 0; a.K = g->S; a.s_sel_seq = g->HI * g->T * g->S; a.s_sel_t = g->S;
  a.s_sel_h = g->T * g->S; a.HI = g->HI; a.valid = nullptr;
  a.bias = bias; a.s_b_seq = g->T * g->S; a.s_b_t = g->S; a.s_b_h = 0;
  a.BS = g->block_size; a.LW = g->local_window > 0 ? g->local_window : g->block_size;
  a.q_scale_log2 = g->scale * kLog2e;
  a.s_q_seq = g->sqb; a.s_q_t = g->sqt; a.s_qh = g->sqh;
  a.out = o; a.s_o_seq = sob; a.s_o_t = sot; a.s_oh = soh;
  a.lse_out = lse; a.s_l_seq = g->T * g->HQ; a.s_l_t = g->HQ;
  a.nsplit = 1; a.skip_local = 0;
  return attend_rows_launch(a, g->D, g->dtype, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t srswa_gather_bwd_workspace_size(const srswa_gather_desc* g) {
  if (check_gather_desc(g)) return 0;
  return kStatusBytes + bwd_need(g, 8, 8, 8, true);
}

extern "C" int srswa_gather_bwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v,
                                const void* o, int64_t sob, int64_t sot, int64_t soh, const void* dout,
                                const float* lse, const int32_t* sel, const float* bias,
                                const int32_t* seg, void* dq, void* dk, void* dv, float* d_bias,
                                void* workspace, size_t workspace_bytes, srswa_stream_t stream) {
  int rc = check_gather_desc(g);
  if (rc) return rc;
  SRSWA_CHECK_ARG(q && k && v && o && dout && lse && dq && dk && dv && (g->S == 0 || sel), SRSWA_EINVAL);
  SRSWA_CHECK_ARG(!bias || d_bias, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(((sob | sot | soh) & 7) == 0, SRSWA_EALIGN);
  SRSWA_CHECK_ARG(((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
                    reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(dq) |
                    reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15) == 0,
                  SRSWA_EALIGN);
  if (g->B * g->T == 0) return 0;
  int* status = nullptr;
  rc = take_status(&workspace, &workspace_bytes, &status, reinterpret_cast<cudaStream_t>(stream));
  if (rc) return rc;
  if (tc_bwd_path(g, sob, sot, soh)) {
    SRSWA_CHECK_ARG(g->B * g->T < (1ll << 31) && g->HQ < 65536 && g->B * g->HI * g->T * g->S < (1ll << 31),
                    SRSWA_ETOOLARGE);
    rc = tc_gather_bwd(g, q, k, v, o, sob, sot, soh, dout, lse, sel, bias, seg, dq, dk, dv, d_bias, workspace,
                       workspace_bytes, status, reinterpret_cast<cudaStream_t>(stream));
    if (rc != kTcNoTensorMap) return rc;
  }
  const BwdLayout L = bwd_layout(g, bias != nullptr);
  SRSWA_CHECK_ARG(workspace && workspace_bytes >= L.total, SRSWA_EWORKSPACE);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  BwdArgs a = {};
  a.q = q; a.k = k; a.v = v; a.o = o; a.dout = dout; a.lse = lse; a.sel = sel; a.bias = bias;
  a.seg = seg; a.dq = dq; a.dk = dk; a.dv = dv; a.d_bias = d_bias;
  char* ws = static_cast<char*>(workspace);
  a.delta = reinterpret_cast<float*>(ws + L.delta);
  a.dbias_part = bias ? reinterpret_cast<float*>(ws + L.part) : nullptr;
  a.bitmap = reinterpret_cast<uint32_t*>(ws + L.bitmap);
  a.dtype = g->dtype; a.B = g->B; a.T = g->T; a.HQ = g->HQ; a.Hkv = g->Hkv; a.HI = g->HI; a.D = g->D;
  a.S = g->S; a.BS = g->block_size; a.LW = g->local_window > 0 ? g->local_window : g->block_size;
  a.nblk = (g->T + g->block_size - 1) / g->block_size; a.T32 = (g->T + 31) / 32; a.scale = g->scale;
  a.sqb = g->sqb; a.sqt = g->sqt; a.sqh = g->sqh; a.skb = g->skb; a.skt = g->skt; a.skh = g->skh;
  a.svb = g->svb; a.svt = g->svt; a.svh = g->svh; a.sob = sob; a.sot = sot; a.soh = soh;
  SRSWA_CHECK_ARG(g->B * g->T < (1ll << 31) && g->HQ < 65536, SRSWA_ETOOLARGE);

  const int64_t nrows_h = g->B * g->T * g->HQ;
  bwd_delta_kernel<<<static_cast<unsigned>((nrows_h + 7) / 8), 256, 0, st>>>(a);
  SRSWA_CUDA_TRY(cudaGetLastError());
  dim3 gq(static_cast<unsigned>(g->B * g->T), static_cast<unsigned>(g->HQ));
  if (g->D == 128) {
    if (g->dtype == SRSWA_BF16) bwd_dq_kernel<128, SRSWA_BF16><<<gq, kAttendThreads, 0, st>>>(a);
    else bwd_dq_kernel<128, SRSWA_F16><<<gq, kAttendThreads, 0, st>>>(a);
  } else {
    if (g->dtype == SRSWA_BF16) bwd_dq_kernel<64, SRSWA_BF16><<<gq, kAttendThreads, 0, st>>>(a);
    else bwd_dq_kernel<64, SRSWA_F16><<<gq, kAttendThreads, 0, st>>>(a);
  }
  SRSWA_CUDA_TRY(cudaGetLastError());
  if (bias) {
    const int64_t n = g->B * g->T * g->S;
    bwd_dbias_reduce_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(a);
    SRSWA_CUDA_TRY(cudaGetLastError());
  }
  SRSWA_CUDA_TRY(cudaMemsetAsync(a.bitmap, 0, static_cast<size_t>(g->B * g->HI * a.nblk * a.T32) * 4, st));
  const int64_t nb = g->B * g->HI * g->T;
  bwd_bitmap_kernel<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, st>>>(a);
  SRSWA_CUDA_TRY(cudaGetLastError());
  dim3 gk(static_cast<unsigned>(a.nblk), static_cast<unsigned>(g->Hkv), static_cast<unsigned>(g->B));
  if (g->D == 128) bwd_dkdv_kernel<128><<<gk, 256, 0, st>>>(a);
  else bwd_dkdv_kernel<64><<<gk, 256, 0, st>>>(a);
  return srswa_last_launch_status();
}

// ---------------------------------------------------------------------------
// Backward without any allocation by anyone: the scratch the backward needs
// (delta, per-head d_bias partials, selection bitmap; on the tensor-core path
// also the remote dQ / dK / dV partials and pair lists) lives in a file-scope
// device array instead of a caller workspace.  For callers that cannot call
// cudaMalloc or an allocator at all: code embedded in a runtime that reserves
// all device memory up front and forbids allocation afterwards, plugin or FFI
// hosts that hand a kernel only its input/output buffers, and host code with
// no device allocator of its own.
//
// The array is kNoAllocScratchBytes (32 MiB) on every device that loads this
// library, held until process exit.  Problems whose backward scratch exceeds
// it are rejected with SRSWA_ETOOLARGE.  In host code the array's name is a
// host-side stand-in, so its device address is looked up once per device
// (cudaGetSymbolAddress, with that device current) on the first call made on
// that device; make that first call outside any stream capture.  All calls
// share the one array, so calls whose GPU work overlaps (different streams,
// or graph replays running concurrently) race on it and must be serialised by
// the caller.  The backward clears the parts that must start at zero (bitmaps,
// d_bias partials) on every call; the rest is fully overwritten.
// ---------------------------------------------------------------------------
#include <mutex>

namespace srswa {
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(32) << 20;
static __device__ __align__(256) unsigned char g_bwd_scratch[kNoAllocScratchBytes];
constexpr int kMaxDevices = 64;
static void* g_bwd_scratch_dev[kMaxDevices] = {};
static std::mutex g_bwd_scratch_mu;

static int bwd_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return SRSWA_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_bwd_scratch_mu);
  if (g_bwd_scratch_dev[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    g_bwd_scratch_dev[dev] = p;
  }
  *out = g_bwd_scratch_dev[dev];
  return 0;
}
}  // namespace srswa

extern "C" size_t srswa_gather_bwd_noalloc_max_scratch(void) { return srswa::kNoAllocScratchBytes; }

extern "C" int srswa_gather_bwd_noalloc(const srswa_gather_desc* g, const void* q, const void* k,
                                        const void* v, const void* o, int64_t sob, int64_t sot, int64_t soh,
                                        const void* dout, const float* lse, const int32_t* sel,
                                        const float* bias, const int32_t* seg, void* dq, void* dk, void* dv,
                                        float* d_bias, srswa_stream_t stream) {
  int rc = check_gather_desc(g);
  if (rc) return rc;
  const size_t need = srswa::kStatusBytes + srswa::bwd_need(g, sob, sot, soh, bias != nullptr);
  if (need > srswa::kNoAllocScratchBytes) return SRSWA_ETOOLARGE;
  void* scratch = nullptr;
  rc = srswa::bwd_scratch_address(&scratch);
  if (rc) return rc;
  return srswa_gather_bwd(g, q, k, v, o, sob, sot, soh, dout, lse, sel, bias, seg, dq, dk, dv, d_bias,
                          scratch, srswa::kNoAllocScratchBytes, stream);
}

extern "C" int srswa_gather_bwd_noalloc_status(int* out, srswa_stream_t stream) {
  if (!out) return SRSWA_EINVAL;
  void* scratch = nullptr;
  const int rc = srswa::bwd_scratch_address(&scratch);
  if (rc) return rc;
  return srswa_workspace_status(scratch, out, stream);
}

extern "C" int srswa_workspace_status(const void* workspace, int* out, srswa_stream_t stream) {
  if (!workspace || !out) return SRSWA_EINVAL;
  int v = 0;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  SRSWA_CUDA_TRY(cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st));
  SRSWA_CUDA_TRY(cudaStreamSynchronize(st));
  *out = v;
  return 0;
}
