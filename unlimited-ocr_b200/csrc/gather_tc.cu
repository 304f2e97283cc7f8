// Gather-attention forward on the 5th-generation tensor cores (tcgen05 / TMEM).
//
// Same semantics as the query-major forward (K1/K5 of the reference:
// hf-model-code/sparse_gather_triton.py:35-122, sparse_gather_e2e_triton.py:36-121),
// split in two passes so that every MMA has M = 128 real rows:
//
//  1. remote pass (remote_fwd_kernel): the selection is inverted into per
//     (batch, index head, block) lists of (query, slot) pairs; a work item is
//     one block and up to 128 of its pairs for one query head.  The pairs' q
//     rows are gathered into shared memory, S = Q_g K_blk^T (M=128, N=64,
//     K=128) goes to TMEM, the per-row softmax (slot bias, keys below the
//     query's window start) runs on the 128 rows, O = P V_blk (N=128) goes to
//     TMEM and the normalised partial (o bf16, lse fp32 log2) is written to a
//     [B, T, S, HQ, D] workspace.
//  2. band pass (band_fwd_kernel): one CTA per (batch, head, 128-query tile)
//     walks the ~LW/64 + 2 key blocks of the local window with an online
//     softmax (lazy rescaling of O in TMEM when the running max grows by more
//     than 2^8), then merges each row with its remote partials (log-sum-exp
//     weights) and writes o and lse.
//
// Shared-memory operand layout: see tc.cuh (128-byte swizzle, K-major Q/K/P,
// MN-major V).  Every mbarrier is waited on by thread 0 only, with a bounded
// spin; the result is broadcast through __syncthreads so an expired wait takes
// a CTA-uniform exit path that drains the tensor pipe and frees TMEM.

#include "attend.cuh"
#include "common.cuh"
#include "tc.cuh"

namespace srswa {

constexpr int kTcThreads = 128;
constexpr int kTileM = 128;
constexpr int kBlk = 64;        // key block (BS)
constexpr int kD = 128;         // head dim
constexpr uint32_t kTmemCols = 256;
constexpr float kRescaleLog2 = 8.0f;  // lazy O rescale threshold (factor 256)

// smem layout of the band kernel (bytes, 1024-aligned pieces)
constexpr uint32_t kQBytes = kTileM * 128 * 2;  // two 64-col halves of [128 x 128 B]
constexpr uint32_t kKVHalf = kBlk * 128;        // [64 rows x 128 B]
constexpr uint32_t kKVBytes = 2 * kKVHalf;      // one 64 x 128 operand
constexpr uint32_t kPBytes = kTileM * 128;      // [128 x 64 keys] bf16 (fits a K operand's 16 KB)
// P of a block is written over that block's K operand, dead once S is in TMEM
constexpr uint32_t kBandSmem = kQBytes + 2 * 2 * kKVBytes + 1024;  // + alignment slack -> 2 CTAs/SM
constexpr uint32_t kRemoteSmem = kQBytes + 2 * kKVBytes + 1024;     // -> 3 CTAs/SM
constexpr uint32_t kRemoteTmemCols = 128;  // S (cols 0-63) is dead before O (cols 0-127) is written

struct TcArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t sqb, sqt, sqh, skb, skt, skh, svb, svt, svh;
  __nv_bfloat16* o;
  int64_t sob, sot, soh;
  float* lse;                 // [B, T, HQ] natural log
  const int32_t* sel;         // [B, HI, T, S] packed
  const float* bias;          // [B, T, S] or null
  const int32_t* seg;         // [B, T] or null
  __nv_bfloat16* part_o;      // [B, T, S, HQ, D]
  float* part_lse;            // [B, T, S, HQ] log2 domain
  const int32_t* pairs;       // packed t * S + s, grouped by (b, hi, block)
  const int4* tiles;          // (b*HI + hi, block, first pair, count)
  const int32_t* ntiles;      // device count of tiles
  int64_t B, T, HQ, Hkv, HI, S, LW, nblk;
  float scale_log2;
};

__device__ __forceinline__ int64_t seg_start(const TcArgs& a, int64_t b, int64_t t) {
  return a.seg ? static_cast<int64_t>(a.seg[b * a.T + t]) : 0;
}
__device__ __forceinline__ int64_t win_start(const TcArgs& a, int64_t b, int64_t t) {
  int64_t ls = t - a.LW + 1;
  const int64_t sg = seg_start(a, b, t);
  if (ls < sg) ls = sg;
  return ls < 0 ? 0 : ls;
}
// remote key range of block blk for query t: [lo, hi) (empty if lo >= hi)
__device__ __forceinline__ void remote_range(const TcArgs& a, int64_t b, int64_t t, int64_t blk, int64_t& lo,
                                             int64_t& hi) {
  const int64_t sg = seg_start(a, b, t);
  const int64_t ls = win_start(a, b, t);
  lo = blk * kBlk > sg ? blk * kBlk : sg;
  hi = min(min((blk + 1) * kBlk, ls), t + 1);
}

// 16-byte chunk loads of a [rows x 128] bf16 operand into the two swizzled
// halves at sbase; row r of the operand comes from src(r) (null -> zeros).
template <int ROWS, typename RowPtr>
__device__ __forceinline__ void load_operand(uint32_t sbase, uint32_t half_bytes, RowPtr src, int tid,
                                             const void* any_valid) {
#pragma unroll
  for (int i = 0; i < ROWS * 16 / kTcThreads; ++i) {
    const int id = tid + i * kTcThreads;
    const int r = id >> 4, c = id & 15;
    const __nv_bfloat16* g = src(r);
    const uint32_t dst = sbase + (c >> 3) * half_bytes + sw128_off(r, c & 7);
    cp_async16_zfill(dst, g ? static_cast<const void*>(g + c * 8) : any_valid, g != nullptr);
  }
}

// 32 fp32 -> 32 bf16 stored as four 16-byte chunks of a swizzled P row
__device__ __forceinline__ void store_p_row(uint32_t pbase, int r, int chunk0, const float* p) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 h = __floats2bfloat162_rn(p[8 * c + 2 * e], p[8 * c + 2 * e + 1]);
      w[e] = *reinterpret_cast<uint32_t*>(&h);
    }
    const uint32_t dst = pbase + sw128_off(r, chunk0 + c);
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
  }
}

// S = Q K^T : M=128, N=64, K=128 (8 k-steps of 16)
__device__ __forceinline__ void issue_qk(uint32_t tmem_s, uint32_t q_s, uint32_t k_s) {
  constexpr uint32_t id = idesc_bf16(128, 64, 0);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint32_t off = (ks & 3) * 32u;  // 16-element step inside the 128-byte row
    const uint64_t ad = sw128_desc(q_s + (ks >> 2) * kQBytes / 2 + off, 16, 1024);
    const uint64_t bd = sw128_desc(k_s + (ks >> 2) * kKVHalf + off, 16, 1024);
    mma_bf16_ss(tmem_s, ad, bd, id, ks > 0 ? 1u : 0u);
  }
}
// O (+)= P V : M=128, N=128, K=64 (4 k-steps of 16 keys); V MN-major (halves LBO apart)
__device__ __forceinline__ void issue_pv(uint32_t tmem_o, uint32_t p_s, uint32_t v_s, bool accumulate) {
  constexpr uint32_t id = idesc_bf16(128, 128, 1);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint64_t ad = sw128_desc(p_s + ks * 32u, 16, 1024);
    const uint64_t bd = sw128_desc(v_s + ks * 2048u, kKVHalf, 1024);
    mma_bf16_ss(tmem_o, ad, bd, id, (accumulate || ks > 0) ? 1u : 0u);
  }
}

// ============================================================================
// band pass
// ============================================================================
__global__ void __launch_bounds__(kTcThreads) band_fwd_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t bar_s, bar_o;
  __shared__ uint32_t tmem_base;
  __shared__ int ok_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t G = a.HQ / a.Hkv;
  const int64_t hk = h / G;
  const int64_t t0 = tile * kTileM;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t q_s = sbase;
  const uint32_t kv_s = q_s + kQBytes;  // stage st: K at kv_s + st*2*kKVBytes, V after it

  if (warp == 0) {
    tmem_alloc(&tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    fence_mbar_init();
    ok_s = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tm_s = tmem, tm_o = tmem + 128;

  // this thread's row
  const int64_t t = t0 + tid;
  const bool row_ok = t < a.T;
  const int64_t ls = row_ok ? win_start(a, b, t) : 0;

  // key blocks of the tile's window
  const int64_t tlast = min(a.T, t0 + kTileM) - 1;
  int64_t key_lo = t0 - a.LW + 1;
  if (key_lo < 0) key_lo = 0;
  const int64_t blo = key_lo / kBlk, bhi = tlast / kBlk;

  auto q_row = [&](int r) -> const __nv_bfloat16* {
    const int64_t tt = t0 + r;
    return tt < a.T ? a.q + b * a.sqb + tt * a.sqt + h * a.sqh : nullptr;
  };
  auto kv_rows = [&](int64_t blk, const __nv_bfloat16* base, int64_t sb, int64_t st, int64_t sh) {
    return [=](int r) -> const __nv_bfloat16* {
      const int64_t kk = blk * kBlk + r;
      return kk < a.T ? base + b * sb + kk * st + hk * sh : nullptr;
    };
  };
  load_operand<kTileM>(q_s, kQBytes / 2, q_row, tid, a.q);
  load_operand<kBlk>(kv_s, kKVHalf, kv_rows(blo, a.k, a.skb, a.skt, a.skh), tid, a.k);
  load_operand<kBlk>(kv_s + kKVBytes, kKVHalf, kv_rows(blo, a.v, a.svb, a.svt, a.svh), tid, a.v);
  cp_async_commit();

  float m_ref = -INFINITY, l = 0.f;
  bool aborted = false;
  for (int64_t j = blo; j <= bhi; ++j) {
    const int jj = static_cast<int>(j - blo);
    const int st = jj & 1;
    // block j's operands have landed (its group; the prefetch group may pend)
    cp_async_wait<0>();
    fence_async_smem();
    __syncthreads();
    const uint32_t k_cur = kv_s + st * 2 * kKVBytes;
    if (tid == 0) {
      // S_j queues behind P.V_{j-1}; its completion implies P.V_{j-1} done
      tc_fence_after();
      issue_qk(tm_s, q_s, k_cur);
      mma_commit(&bar_s);
      ok_s = mbar_wait(&bar_s, jj & 1, 102) ? 1 : 0;
    }
    __syncthreads();
    if (!ok_s) { aborted = true; break; }
    // the other stage (block j-1, its P.V done) is free: prefetch block j+1
    if (j + 1 <= bhi) {
      const uint32_t nx = kv_s + (st ^ 1) * 2 * kKVBytes;
      load_operand<kBlk>(nx, kKVHalf, kv_rows(j + 1, a.k, a.skb, a.skt, a.skh), tid, a.k);
      load_operand<kBlk>(nx + kKVBytes, kKVHalf, kv_rows(j + 1, a.v, a.svb, a.svt, a.svh), tid, a.v);
    }
    cp_async_commit();
    tc_fence_after();
    // ---- softmax of this row over the block's 64 keys ----
    float s[64];
    {
      float s0[32], s1[32];
      tmem_ld32(tm_s + lane_off, s0);
      tmem_ld32(tm_s + lane_off + 32, s1);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) { s[i] = s0[i]; s[32 + i] = s1[i]; }
    }
    const int64_t k0 = j * kBlk;
    float mloc = -INFINITY;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int64_t key = k0 + i;
      const bool valid = row_ok && key >= ls && key <= t;
      s[i] = valid ? s[i] * a.scale_log2 : -INFINITY;
      mloc = fmaxf(mloc, s[i]);
    }
    const bool need = mloc > m_ref + kRescaleLog2;  // also true on the first valid block
    const float alpha = need ? (m_ref == -INFINITY ? 0.f : exp2f(m_ref - mloc)) : 1.f;
    if (need) {
      l *= alpha;
      m_ref = mloc;
    }
    if (__any_sync(0xffffffffu, need && jj > 0)) {  // rescale O rows of this warp in TMEM
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tm_o + lane_off + 32 * c, ov);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
        tmem_st32(tm_o + lane_off + 32 * c, ov);
      }
      tmem_wait_st();
    }
    float lsum = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float p = (s[i] == -INFINITY) ? 0.f : exp2f(s[i] - m_ref);
      s[i] = p;
      lsum += p;
    }
    l += lsum;
    store_p_row(k_cur, tid, 0, s);  // P over the dead K operand of this stage
    store_p_row(k_cur, tid, 4, s + 32);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      issue_pv(tm_o, k_cur, k_cur + kKVBytes, jj > 0);
      mma_commit(&bar_o);
    }
  }
  const int nblocks = static_cast<int>(bhi - blo + 1);
  // drain: the last P.V (or, after an abort, whatever was committed)
  if (tid == 0) ok_s = mbar_wait(&bar_o, (nblocks - 1) & 1, 103) ? 1 : 0;
  __syncthreads();
  cp_async_wait<0>();
  if (!aborted && ok_s) {
    tc_fence_after();
    // ---- epilogue: merge with remote partials, write o and lse ----
    const int64_t hi = (hk * a.HI) / a.Hkv;
    float M = (l > 0.f) ? m_ref + log2f(l) : -INFINITY;
    float lse_s[64];
    int64_t slot_base = 0;
    int nslot = 0;
    if (row_ok && a.part_o) {
      const int32_t* srow = a.sel + ((b * a.HI + hi) * a.T + t) * a.S;
      slot_base = ((b * a.T + t) * a.S) * a.HQ + h;
      for (int64_t s2 = 0; s2 < a.S && s2 < 64; ++s2) {
        lse_s[s2] = -INFINITY;
        const int64_t blk = srow[s2];
        if (blk < 0 || blk >= a.nblk) continue;
        int64_t lo, hi2;
        remote_range(a, b, t, blk, lo, hi2);
        if (lo >= hi2) continue;
        bool dup = false;
        for (int64_t u = 0; u < s2; ++u) dup |= srow[u] == blk;
        if (dup) continue;
        lse_s[s2] = a.part_lse[slot_base + s2 * a.HQ];
        M = fmaxf(M, lse_s[s2]);
      }
      nslot = static_cast<int>(a.S < 64 ? a.S : 64);
    }
    const float Mu = (M == -INFINITY) ? 0.f : M;
    const float wb = (l > 0.f) ? exp2f(m_ref - Mu) : 0.f;
    float den = l * wb;
    for (int s2 = 0; s2 < nslot; ++s2)
      if (lse_s[s2] != -INFINITY) den += exp2f(lse_s[s2] - Mu);
    const float inv = den > 0.f ? 1.f / den : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float ov[32];
      tmem_ld32(tm_o + lane_off + 32 * c, ov);
      tmem_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] *= wb;
        for (int s2 = 0; s2 < nslot; ++s2) {
          if (lse_s[s2] == -INFINITY) continue;
          const float w = exp2f(lse_s[s2] - Mu);
          const uint4* src = reinterpret_cast<const uint4*>(a.part_o + (slot_base + s2 * a.HQ) * kD + 32 * c);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 u = src[q4];
            ov[8 * q4 + 0] = fmaf(w, bf16_lo(u.x), ov[8 * q4 + 0]);
            ov[8 * q4 + 1] = fmaf(w, bf16_hi(u.x), ov[8 * q4 + 1]);
            ov[8 * q4 + 2] = fmaf(w, bf16_lo(u.y), ov[8 * q4 + 2]);
            ov[8 * q4 + 3] = fmaf(w, bf16_hi(u.y), ov[8 * q4 + 3]);
            ov[8 * q4 + 4] = fmaf(w, bf16_lo(u.z), ov[8 * q4 + 4]);
            ov[8 * q4 + 5] = fmaf(w, bf16_hi(u.z), ov[8 * q4 + 5]);
            ov[8 * q4 + 6] = fmaf(w, bf16_lo(u.w), ov[8 * q4 + 6]);
            ov[8 * q4 + 7] = fmaf(w, bf16_hi(u.w), ov[8 * q4 + 7]);
          }
        }
        __nv_bfloat16* dst = a.o + b * a.sob + t * a.sot + h * a.soh + 32 * c;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float tmp[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tmp[e] = ov[8 * q4 + e] * inv;
          store8(dst, 8 * q4, SRSWA_BF16, tmp);
        }
      }
    }
    if (row_ok && a.lse) a.lse[(b * a.T + t) * a.HQ + h] = den > 0.f ? (Mu + log2f(den)) * kLn2 : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// ============================================================================
// remote pass: inverted selection lists
// ============================================================================
// count[b*HI+hi][blk] += 1 for every usable (t, slot) selection
__global__ void pairs_count_kernel(const TcArgs a, int32_t* count) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (b, hi, t)
  if (i >= a.B * a.HI * a.T) return;
  const int64_t t = i % a.T, bh = i / a.T, b = bh / a.HI;
  const int32_t* srow = a.sel + i * a.S;
  for (int64_t s = 0; s < a.S; ++s) {
    const int64_t blk = srow[s];
    if (blk < 0 || blk >= a.nblk) continue;
    int64_t lo, hi;
    remote_range(a, b, t, blk, lo, hi);
    if (lo >= hi) continue;
    bool dup = false;
    for (int64_t u = 0; u < s; ++u) dup |= srow[u] == blk;
    if (dup) continue;
    atomicAdd(count + bh * a.nblk + blk, 1);
  }
}

// single-CTA exclusive scans: pair offsets and tile offsets per (b*HI+hi, blk);
// writes the tile descriptors and the tile count
__global__ void pairs_scan_kernel(const TcArgs a, const int32_t* count, int32_t* offs, int32_t* cursor,
                                  int4* tiles, int32_t* ntiles) {
  __shared__ int32_t sh_p[1024], sh_t[1024];
  const int64_t n = a.B * a.HI * a.nblk;
  int32_t base_p = 0, base_t = 0;
  for (int64_t c0 = 0; c0 < n; c0 += 1024) {
    const int64_t i = c0 + threadIdx.x;
    const int32_t cnt = i < n ? count[i] : 0;
    sh_p[threadIdx.x] = cnt;
    sh_t[threadIdx.x] = (cnt + kTileM - 1) / kTileM;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {  // inclusive Hillis-Steele scan
      const int32_t vp = threadIdx.x >= static_cast<unsigned>(o) ? sh_p[threadIdx.x - o] : 0;
      const int32_t vt = threadIdx.x >= static_cast<unsigned>(o) ? sh_t[threadIdx.x - o] : 0;
      __syncthreads();
      sh_p[threadIdx.x] += vp;
      sh_t[threadIdx.x] += vt;
      __syncthreads();
    }
    if (i < n) {
      const int32_t op = base_p + sh_p[threadIdx.x] - cnt;
      const int32_t nt = (cnt + kTileM - 1) / kTileM;
      const int32_t ot = base_t + sh_t[threadIdx.x] - nt;
      offs[i] = op;
      cursor[i] = op;
      for (int32_t k = 0; k < nt; ++k) {
        const int32_t first = op + k * kTileM;
        tiles[ot + k] = make_int4(static_cast<int>(i / a.nblk), static_cast<int>(i % a.nblk), first,
                                  min(kTileM, cnt - k * kTileM));
      }
    }
    __syncthreads();
    base_p += sh_p[1023];
    base_t += sh_t[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) *ntiles = base_t;
}

__global__ void pairs_fill_kernel(const TcArgs a, int32_t* cursor, int32_t* pairs) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= a.B * a.HI * a.T) return;
  const int64_t t = i % a.T, bh = i / a.T, b = bh / a.HI;
  const int32_t* srow = a.sel + i * a.S;
  for (int64_t s = 0; s < a.S; ++s) {
    const int64_t blk = srow[s];
    if (blk < 0 || blk >= a.nblk) continue;
    int64_t lo, hi;
    remote_range(a, b, t, blk, lo, hi);
    if (lo >= hi) continue;
    bool dup = false;
    for (int64_t u = 0; u < s; ++u) dup |= srow[u] == blk;
    if (dup) continue;
    const int32_t pos = atomicAdd(cursor + bh * a.nblk + blk, 1);
    pairs[pos] = static_cast<int32_t>(t * a.S + s);
  }
}

// One work item = (tile, query head of the tile's index head).  Persistent:
// grid-stride over items; the item count comes from device memory.
__global__ void __launch_bounds__(kTcThreads) remote_fwd_kernel(const TcArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int ok_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t q_s = sbase;
  const uint32_t k_s = q_s + kQBytes;
  const uint32_t v_s = k_s + kKVBytes;
  const uint32_t p_s = k_s;  // P over K (dead once S is in TMEM)
  if (warp == 0) {
    tmem_alloc(&tmem_base, kRemoteTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    ok_s = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tm_s = tmem, tm_o = tmem;  // O overwrites S after the softmax read it
  const int64_t hpi = a.HQ / a.HI;  // query heads per index head
  const int64_t nitems = static_cast<int64_t>(*a.ntiles) * hpi;
  uint32_t phase = 0;
  for (int64_t item = blockIdx.x; item < nitems; item += gridDim.x) {
    const int4 td = a.tiles[item / hpi];
    const int64_t bh = td.x, blk = td.y, first = td.z, cnt = td.w;
    const int64_t b = bh / a.HI, hi = bh % a.HI;
    const int64_t h = hi * hpi + item % hpi;
    const int64_t hk = h / (a.HQ / a.Hkv);
    // this thread's pair
    int64_t t = -1, slot = 0;
    if (tid < cnt) {
      const int32_t pk = a.pairs[first + tid];
      t = pk / a.S;
      slot = pk % a.S;
    }
    auto q_row = [&](int r) -> const __nv_bfloat16* {
      if (r >= cnt) return nullptr;
      const int32_t pk = a.pairs[first + r];
      return a.q + b * a.sqb + static_cast<int64_t>(pk / a.S) * a.sqt + h * a.sqh;
    };
    auto k_row = [&](int r) -> const __nv_bfloat16* {
      const int64_t kk = blk * kBlk + r;
      return kk < a.T ? a.k + b * a.skb + kk * a.skt + hk * a.skh : nullptr;
    };
    auto v_row = [&](int r) -> const __nv_bfloat16* {
      const int64_t kk = blk * kBlk + r;
      return kk < a.T ? a.v + b * a.svb + kk * a.svt + hk * a.svh : nullptr;
    };
    load_operand<kTileM>(q_s, kQBytes / 2, q_row, tid, a.q);
    load_operand<kBlk>(k_s, kKVHalf, k_row, tid, a.k);
    load_operand<kBlk>(v_s, kKVHalf, v_row, tid, a.v);
    cp_async_commit();
    cp_async_wait<0>();
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      issue_qk(tm_s, q_s, k_s);
      mma_commit(&bar);
      ok_s = mbar_wait(&bar, phase, 201) ? 1 : 0;
    }
    phase ^= 1;
    __syncthreads();
    if (!ok_s) break;
    tc_fence_after();
    float s[64];
    {
      float s0[32], s1[32];
      tmem_ld32(tm_s + lane_off, s0);
      tmem_ld32(tm_s + lane_off + 32, s1);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) { s[i] = s0[i]; s[32 + i] = s1[i]; }
    }
    float m = -INFINITY;
    int64_t lo = 0, hi2 = 0;
    float bias2 = 0.f;
    if (t >= 0) {
      remote_range(a, b, t, blk, lo, hi2);
      if (a.bias) bias2 = a.bias[(b * a.T + t) * a.S + slot] * kLog2e;
    }
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int64_t key = blk * kBlk + i;
      const bool valid = t >= 0 && key >= lo && key < hi2;
      s[i] = valid ? s[i] * a.scale_log2 + bias2 : -INFINITY;
      m = fmaxf(m, s[i]);
    }
    float lsum = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float p = (s[i] == -INFINITY) ? 0.f : exp2f(s[i] - m);
      s[i] = p;
      lsum += p;
    }
    store_p_row(p_s, tid, 0, s);
    store_p_row(p_s, tid, 4, s + 32);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      issue_pv(tm_o, p_s, v_s, false);
      mma_commit(&bar);
      ok_s = mbar_wait(&bar, phase, 202) ? 1 : 0;
    }
    phase ^= 1;
    __syncthreads();
    if (!ok_s) break;
    tc_fence_after();
    const int64_t prow = ((b * a.T + (t < 0 ? 0 : t)) * a.S + slot) * a.HQ + h;
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float ov[32];
      tmem_ld32(tm_o + lane_off + 32 * c, ov);
      tmem_wait_ld();
      if (t >= 0) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float tmp[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) tmp[e] = ov[8 * q4 + e] * inv;
          store8(a.part_o + prow * kD + 32 * c, 8 * q4, SRSWA_BF16, tmp);
        }
      }
    }
    if (t >= 0) a.part_lse[prow] = lsum > 0.f ? m + log2f(lsum) : -INFINITY;
    tc_fence_before();
    __syncthreads();  // smem and TMEM reuse by the next item
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kRemoteTmemCols);
}

// ============================================================================
// backward (deterministic: every gradient element has one writer; remote and
// band contributions meet through fixed-order partial sums)
// ============================================================================
struct TcBwdArgs {
  TcArgs f;
  const __nv_bfloat16* dout;  // strides sob/sot/soh of TcArgs
  const float* lse;           // [B, T, HQ] natural log
  float* delta;               // [B, T, HQ]
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  __nv_bfloat16* dq_part;     // [B, T, S, HQ, D] (scaled)
  float* dbias_part;          // [B, T, S, HQ]
  float* dkv_part;            // [B, HQ, nblk, 2, 64, 128] (dK scaled, dV)
  const int32_t* count;       // [B*HI*nblk]
  const int32_t* offs;        // [B*HI*nblk]
  float* d_bias;              // [B, T, S]
  float scale;
};

constexpr uint32_t kTile128 = 128 * 128 * 2;  // [128 rows x 128 bf16] = two 16 KB halves

// D = A^T B with A, B both stored rows = K (MN-major): M = 128 (A's 128
// features, halves a_lbo apart), N = 64 (B's 64 columns), K = 128 rows.
__device__ __forceinline__ void issue_tn(uint32_t tmem_d, uint32_t a_s, uint32_t a_lbo, uint32_t b_s,
                                         bool accumulate) {
  constexpr uint32_t id = idesc_bf16(128, 64, 1, 1);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint64_t ad = sw128_desc(a_s + ks * 2048u, a_lbo, 1024);
    const uint64_t bd = sw128_desc(b_s + ks * 2048u, 8192, 1024);
    mma_bf16_ss(tmem_d, ad, bd, id, (accumulate || ks > 0) ? 1u : 0u);
  }
}
// D = A B^T, A and B K-major [128 rows x 128]: M = N = K = 128
__device__ __forceinline__ void issue_nt128(uint32_t tmem_d, uint32_t a_s, uint32_t b_s) {
  constexpr uint32_t id = idesc_bf16(128, 128, 0);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint32_t off = (ks >> 2) * (kTile128 / 2) + (ks & 3) * 32u;
    mma_bf16_ss(tmem_d, sw128_desc(a_s + off, 16, 1024), sw128_desc(b_s + off, 16, 1024), id, ks > 0 ? 1u : 0u);
  }
}
// D (+)= A B, A K-major [128 x 128 (K)], B MN-major [128 (K) rows x 128 (N)]
__device__ __forceinline__ void issue_nn128(uint32_t tmem_d, uint32_t a_s, uint32_t b_s, bool accumulate) {
  constexpr uint32_t id = idesc_bf16(128, 128, 1);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint32_t aoff = (ks >> 2) * (kTile128 / 2) + (ks & 3) * 32u;
    mma_bf16_ss(tmem_d, sw128_desc(a_s + aoff, 16, 1024), sw128_desc(b_s + ks * 2048u, kTile128 / 2, 1024), id,
                (accumulate || ks > 0) ? 1u : 0u);
  }
}

__device__ __forceinline__ void store_row128(uint32_t base, int r, const float* v) {
  store_p_row(base, r, 0, v);
  store_p_row(base, r, 4, v + 32);
  store_p_row(base + kTile128 / 2, r, 0, v + 64);
  store_p_row(base + kTile128 / 2, r, 4, v + 96);
}

__global__ void tc_delta_kernel(const TcBwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const TcArgs& f = a.f;
  if (item >= f.B * f.T * f.HQ) return;
  const int64_t h = item % f.HQ, bt = item / f.HQ, t = bt % f.T, b = bt / f.T;
  const int64_t off = b * f.sob + t * f.sot + h * f.soh + lane * 4;
  const uint2 uo = *reinterpret_cast<const uint2*>(f.o + off);
  const uint2 ug = *reinterpret_cast<const uint2*>(a.dout + off);
  float acc = bf16_lo(uo.x) * bf16_lo(ug.x) + bf16_hi(uo.x) * bf16_hi(ug.x) + bf16_lo(uo.y) * bf16_lo(ug.y) +
              bf16_hi(uo.y) * bf16_hi(ug.y);
  acc = warp_sum(acc);
  if (lane == 0) a.delta[item] = acc;
}

// ---- backward pair lists, ordered by query inside each (b, hi, block) list,
// so that the remote dK / dV accumulation order is fixed from call to call.
// A query selects a block at most once (later duplicate slots are dropped),
// so one bit per (list, query) is the whole list.
__global__ void bwd_pairs_bitmap_kernel(const TcArgs a, uint32_t* bitmap, int64_t T32) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // (b, hi, t)
  if (i >= a.B * a.HI * a.T) return;
  const int64_t t = i % a.T, bh = i / a.T, b = bh / a.HI;
  const int32_t* srow = a.sel + i * a.S;
  for (int64_t s = 0; s < a.S; ++s) {
    const int64_t blk = srow[s];
    if (blk < 0 || blk >= a.nblk) continue;
    int64_t lo, hi;
    remote_range(a, b, t, blk, lo, hi);
    if (lo >= hi) continue;
    atomicOr(bitmap + (bh * a.nblk + blk) * T32 + (t >> 5), 1u << (t & 31));
  }
}

// one warp per list: its length
__global__ void bwd_pairs_count_kernel(const TcArgs a, const uint32_t* bitmap, int64_t T32, int32_t* count) {
  const int lane = threadIdx.x & 31;
  const int64_t seg = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (seg >= a.B * a.HI * a.nblk) return;
  const uint32_t* w = bitmap + seg * T32;
  int n = 0;
  for (int64_t i = lane; i < T32; i += 32) n += __popc(w[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  if (lane == 0) count[seg] = n;
}

// one warp per list: emit (t * S + first slot holding the block) in t order
__global__ void bwd_pairs_fill_kernel(const TcArgs a, const uint32_t* bitmap, int64_t T32, const int32_t* offs,
                                      int32_t* pairs) {
  const int lane = threadIdx.x & 31;
  const int64_t seg = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (seg >= a.B * a.HI * a.nblk) return;
  const int64_t blk = seg % a.nblk, bh = seg / a.nblk;
  const uint32_t* w = bitmap + seg * T32;
  int64_t pos = offs[seg];
  for (int64_t w0 = 0; w0 < T32; w0 += 32) {
    uint32_t word = (w0 + lane < T32) ? w[w0 + lane] : 0u;
    const int n = __popc(word);
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int64_t p = pos + incl - n;
    while (word) {
      const int bit = __ffs(word) - 1;
      word &= word - 1;
      const int64_t t = (w0 + lane) * 32 + bit;
      const int32_t* srow = a.sel + (bh * a.T + t) * a.S;
      int64_t s = 0;
      while (s < a.S && srow[s] != blk) ++s;
      pairs[p++] = static_cast<int32_t>(t * a.S + s);
    }
    pos += __shfl_sync(0xffffffffu, incl, 31);
  }
}

// ---- remote pairs: one item = (batch, index head, block, query head) ------
constexpr uint32_t kRBSmem = 2 * kKVBytes + 2 * kTile128 + 2 * kPBytes + 1024;

__global__ void __launch_bounds__(kTcThreads) bwd_remote_kernel(const TcBwdArgs a) {
  const TcArgs& f = a.f;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int ok_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t k_s = sbase, v_s = k_s + kKVBytes;
  const uint32_t q_s = v_s + kKVBytes, do_s = q_s + kTile128;
  const uint32_t p_s = do_s + kTile128, ds_s = p_s + kPBytes;
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    ok_s = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tm_s = tmem, tm_dp = tmem + 64, tm_dq = tmem, tm_dvt = tmem + 128, tm_dkt = tmem + 192;
  const int64_t hpi = f.HQ / f.HI, G = f.HQ / f.Hkv;
  const int64_t nitems = f.B * f.HI * f.nblk * hpi;
  uint32_t phase = 0;
  bool failed = false;
  for (int64_t item = blockIdx.x; item < nitems && !failed; item += gridDim.x) {
    const int64_t bhc = item / hpi;
    const int64_t cnt = a.count[bhc];
    if (cnt == 0) continue;
    const int64_t first = a.offs[bhc];
    const int64_t bh = bhc / f.nblk, blk = bhc % f.nblk, b = bh / f.HI, hi = bh % f.HI;
    const int64_t h = hi * hpi + item % hpi, hk = h / G;
    auto k_row = [&](int r) -> const __nv_bfloat16* {
      const int64_t kk = blk * kBlk + r;
      return kk < f.T ? f.k + b * f.skb + kk * f.skt + hk * f.skh : nullptr;
    };
    auto v_row = [&](int r) -> const __nv_bfloat16* {
      const int64_t kk = blk * kBlk + r;
      return kk < f.T ? f.v + b * f.svb + kk * f.svt + hk * f.svh : nullptr;
    };
    load_operand<kBlk>(k_s, kKVHalf, k_row, tid, f.k);
    load_operand<kBlk>(v_s, kKVHalf, v_row, tid, f.v);
    const int64_t ntile = (cnt + kTileM - 1) / kTileM;
    for (int64_t tl = 0; tl < ntile; ++tl) {
      const int64_t base = first + tl * kTileM, n_here = (cnt - tl * kTileM) < kTileM ? (cnt - tl * kTileM) : int64_t(kTileM);
      int64_t t = -1, slot = 0;
      if (tid < n_here) {
        const int32_t pk = f.pairs[base + tid];
        t = pk / f.S;
        slot = pk % f.S;
      }
      auto q_row = [&](int r) -> const __nv_bfloat16* {
        if (r >= n_here) return nullptr;
        const int64_t tt = f.pairs[base + r] / f.S;
        return f.q + b * f.sqb + tt * f.sqt + h * f.sqh;
      };
      auto g_row = [&](int r) -> const __nv_bfloat16* {
        if (r >= n_here) return nullptr;
        const int64_t tt = f.pairs[base + r] / f.S;
        return a.dout + b * f.sob + tt * f.sot + h * f.soh;
      };
      load_operand<kTileM>(q_s, kTile128 / 2, q_row, tid, f.q);
      load_operand<kTileM>(do_s, kTile128 / 2, g_row, tid, a.dout);
      cp_async_commit();
      cp_async_wait<0>();
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        issue_qk(tm_s, q_s, k_s);
        issue_qk(tm_dp, do_s, v_s);
        mma_commit(&bar);
        ok_s = mbar_wait(&bar, phase, 301) ? 1 : 0;
      }
      phase ^= 1;
      __syncthreads();
      if (!ok_s) { failed = true; break; }
      tc_fence_after();
      float sv[64], dp[64];
      {
        float x0[32], x1[32];
        tmem_ld32(tm_s + lane_off, x0);
        tmem_ld32(tm_s + lane_off + 32, x1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { sv[i] = x0[i]; sv[32 + i] = x1[i]; }
        tmem_ld32(tm_dp + lane_off, x0);
        tmem_ld32(tm_dp + lane_off + 32, x1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { dp[i] = x0[i]; dp[32 + i] = x1[i]; }
      }
      float lse2 = 0.f, dlt = 0.f, bias2 = 0.f;
      int64_t lo = 0, hi2 = 0;
      if (t >= 0) {
        lse2 = a.lse[(b * f.T + t) * f.HQ + h] * kLog2e;
        dlt = a.delta[(b * f.T + t) * f.HQ + h];
        if (f.bias) bias2 = f.bias[(b * f.T + t) * f.S + slot] * kLog2e;
        remote_range(f, b, t, blk, lo, hi2);
      }
      float dsum = 0.f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const int64_t key = blk * kBlk + i;
        const bool valid = t >= 0 && key >= lo && key < hi2 && lse2 != -INFINITY;
        const float p = valid ? exp2f(sv[i] * f.scale_log2 + bias2 - lse2) : 0.f;
        const float ds = p * (dp[i] - dlt);
        sv[i] = p;
        dp[i] = ds;
        dsum += ds;
      }
      if (t >= 0 && a.dbias_part) a.dbias_part[((b * f.T + t) * f.S + slot) * f.HQ + h] = dsum;
      store_p_row(p_s, tid, 0, sv);
      store_p_row(p_s, tid, 4, sv + 32);
      store_p_row(ds_s, tid, 0, dp);
      store_p_row(ds_s, tid, 4, dp + 32);
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        issue_pv(tm_dq, ds_s, k_s, false);                 // dQ_g = dS K
        issue_tn(tm_dvt, do_s, kTile128 / 2, p_s, tl > 0);  // dV^T += dO_g^T P
        issue_tn(tm_dkt, q_s, kTile128 / 2, ds_s, tl > 0);  // dK^T += Q_g^T dS
        mma_commit(&bar);
        ok_s = mbar_wait(&bar, phase, 302) ? 1 : 0;
      }
      phase ^= 1;
      __syncthreads();
      if (!ok_s) { failed = true; break; }
      tc_fence_after();
      const int64_t prow = ((b * f.T + (t < 0 ? 0 : t)) * f.S + slot) * f.HQ + h;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[32];
        tmem_ld32(tm_dq + lane_off + 32 * c, ov);
        tmem_wait_ld();
        if (t >= 0) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            float tmp[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) tmp[e] = ov[8 * q4 + e] * a.scale;
            store8(a.dq_part + prow * kD + 32 * c, 8 * q4, SRSWA_BF16, tmp);
          }
        }
      }
      tc_fence_before();
      __syncthreads();
    }
    if (failed) break;
    // this block's remote dK / dV for query head h: thread = feature d
    tc_fence_after();
    float* dst = a.dkv_part + ((b * f.HQ + h) * f.nblk + blk) * (2 * 64 * 128);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float kv[32], vv[32];
      tmem_ld32(tm_dkt + lane_off + 32 * half, kv);
      tmem_ld32(tm_dvt + lane_off + 32 * half, vv);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        dst[(32 * half + i) * 128 + tid] = kv[i] * a.scale;
        dst[8192 + (32 * half + i) * 128 + tid] = vv[i];
      }
    }
    tc_fence_before();
    __syncthreads();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---- band dK / dV: one CTA per (batch, kv head, 128-key tile) -------------
constexpr uint32_t kBDSmem = 6 * kTile128 + 1024;

__global__ void __launch_bounds__(kTcThreads) bwd_band_dkdv_kernel(const TcBwdArgs a) {
  const TcArgs& f = a.f;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int ok_s;
  __shared__ float lse2_s[128], dl_s[128];
  __shared__ int64_t ls_s[128];
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t tile = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int64_t k0 = tile * 128, G = f.HQ / f.Hkv;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t kt_s = sbase, vt_s = kt_s + kTile128, qt_s = vt_s + kTile128, dot_s = qt_s + kTile128;
  const uint32_t pt_s = dot_s + kTile128, dst_s = pt_s + kTile128;
  if (warp == 0) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    ok_s = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tm_st = tmem, tm_dpt = tmem + 128, tm_dk = tmem + 256, tm_dv = tmem + 384;
  auto kt_row = [&](int r) -> const __nv_bfloat16* {
    const int64_t kk = k0 + r;
    return kk < f.T ? f.k + b * f.skb + kk * f.skt + hk * f.skh : nullptr;
  };
  auto vt_row = [&](int r) -> const __nv_bfloat16* {
    const int64_t kk = k0 + r;
    return kk < f.T ? f.v + b * f.svb + kk * f.svt + hk * f.svh : nullptr;
  };
  load_operand<kTileM>(kt_s, kTile128 / 2, kt_row, tid, f.k);
  load_operand<kTileM>(vt_s, kTile128 / 2, vt_row, tid, f.v);
  const int64_t key = k0 + tid;
  const int64_t q_hi = min(f.T, k0 + 127 + f.LW);  // exclusive end of queries seeing this tile locally
  const int64_t nqt = (q_hi - k0 + 127) / 128;
  uint32_t phase = 0;
  bool failed = false, any = false;
  for (int64_t gq = 0; gq < G && !failed; ++gq) {
    const int64_t h = hk * G + gq;
    for (int64_t qt = 0; qt < nqt; ++qt) {
      const int64_t q0 = k0 + qt * 128;
      auto q_row = [&](int r) -> const __nv_bfloat16* {
        const int64_t tt = q0 + r;
        return tt < f.T ? f.q + b * f.sqb + tt * f.sqt + h * f.sqh : nullptr;
      };
      auto g_row = [&](int r) -> const __nv_bfloat16* {
        const int64_t tt = q0 + r;
        return tt < f.T ? a.dout + b * f.sob + tt * f.sot + h * f.soh : nullptr;
      };
      load_operand<kTileM>(qt_s, kTile128 / 2, q_row, tid, f.q);
      load_operand<kTileM>(dot_s, kTile128 / 2, g_row, tid, a.dout);
      cp_async_commit();
      {
        const int64_t tq = q0 + tid;
        const bool ok = tq < f.T;
        lse2_s[tid] = ok ? a.lse[(b * f.T + tq) * f.HQ + h] * kLog2e : INFINITY;
        dl_s[tid] = ok ? a.delta[(b * f.T + tq) * f.HQ + h] : 0.f;
        ls_s[tid] = ok ? win_start(f, b, tq) : (int64_t(1) << 62);
      }
      cp_async_wait<0>();
      fence_async_smem();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        issue_nt128(tm_st, kt_s, qt_s);   // S^T = K Q^T
        issue_nt128(tm_dpt, vt_s, dot_s); // dP^T = V dO^T
        mma_commit(&bar);
        ok_s = mbar_wait(&bar, phase, 311) ? 1 : 0;
      }
      phase ^= 1;
      __syncthreads();
      if (!ok_s) { failed = true; break; }
      tc_fence_after();
      // row = key; columns = the tile's 128 queries, 32 at a time
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float sv[32], dp[32];
        tmem_ld32(tm_st + lane_off + 32 * c, sv);
        tmem_ld32(tm_dpt + lane_off + 32 * c, dp);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int qi = 32 * c + i;
          const int64_t tq = q0 + qi;
          const bool local = key < f.T && key <= tq && key >= ls_s[qi];
          const float p = local ? exp2f(sv[i] * f.scale_log2 - lse2_s[qi]) : 0.f;
          sv[i] = p;
          dp[i] = p * (dp[i] - dl_s[qi]);
        }
        const uint32_t half = (c >> 1) * (kTile128 / 2);
        store_p_row(pt_s + half, tid, (c & 1) * 4, sv);
        store_p_row(dst_s + half, tid, (c & 1) * 4, dp);
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
        issue_nn128(tm_dv, pt_s, dot_s, any);   // dV += P^T dO
        issue_nn128(tm_dk, dst_s, qt_s, any);   // dK += dS^T Q
        mma_commit(&bar);
        ok_s = mbar_wait(&bar, phase, 312) ? 1 : 0;
      }
      phase ^= 1;
      any = true;
      __syncthreads();
      if (!ok_s) { failed = true; break; }
    }
  }
  if (!failed) {
    tc_fence_after();
    const int64_t blk = key / kBlk, hi = (hk * f.HI) / f.Hkv;
    const int64_t bhc = (b * f.HI + hi) * f.nblk + blk;
    const bool has_remote = key < f.T && a.count && a.count[bhc] > 0;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float kv[32], vv[32];
      if (any) {
        tmem_ld32(tm_dk + lane_off + 32 * c, kv);
        tmem_ld32(tm_dv + lane_off + 32 * c, vv);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) kv[i] = vv[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) kv[i] *= a.scale;
      if (has_remote) {
        for (int64_t gq = 0; gq < G; ++gq) {
          const float* src = a.dkv_part + ((b * f.HQ + hk * G + gq) * f.nblk + blk) * (2 * 64 * 128) +
                             (key % kBlk) * 128 + 32 * c;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            kv[i] += src[i];
            vv[i] += src[8192 + i];
          }
        }
      }
      if (key < f.T) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          store8(a.dk + b * f.skb + key * f.skt + hk * f.skh + 32 * c, 8 * q4, SRSWA_BF16, kv + 8 * q4);
          store8(a.dv + b * f.svb + key * f.svt + hk * f.svh + 32 * c, 8 * q4, SRSWA_BF16, vv + 8 * q4);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---- band dQ (+ remote dQ partials): one CTA per (batch, head, 128 queries)
constexpr uint32_t kBQSmem = 2 * kTile128 + 2 * 2 * kKVBytes + 1024;

__global__ void __launch_bounds__(kTcThreads) bwd_band_dq_kernel(const TcBwdArgs a) {
  const TcArgs& f = a.f;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t bar_s, bar_o;
  __shared__ uint32_t tmem_base;
  __shared__ int ok_s;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t hk = h / (f.HQ / f.Hkv);
  const int64_t t0 = tile * kTileM;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t q_s = sbase, do_s = q_s + kTile128, kv_s = do_s + kTile128;
  if (warp == 0) {
    tmem_alloc(&tmem_base, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    fence_mbar_init();
    ok_s = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const uint32_t tm_s = tmem, tm_dp = tmem + 64, tm_dq = tmem + 128;
  const int64_t t = t0 + tid;
  const bool row_ok = t < f.T;
  const int64_t ls = row_ok ? win_start(f, b, t) : 0;
  const float lse2 = row_ok ? a.lse[(b * f.T + t) * f.HQ + h] * kLog2e : INFINITY;
  const float dlt = row_ok ? a.delta[(b * f.T + t) * f.HQ + h] : 0.f;
  const int64_t tlast = min(f.T, t0 + kTileM) - 1;
  int64_t key_lo = t0 - f.LW + 1;
  if (key_lo < 0) key_lo = 0;
  const int64_t blo = key_lo / kBlk, bhi = tlast / kBlk;
  auto q_row = [&](int r) -> const __nv_bfloat16* {
    const int64_t tt = t0 + r;
    return tt < f.T ? f.q + b * f.sqb + tt * f.sqt + h * f.sqh : nullptr;
  };
  auto g_row = [&](int r) -> const __nv_bfloat16* {
    const int64_t tt = t0 + r;
    return tt < f.T ? a.dout + b * f.sob + tt * f.sot + h * f.soh : nullptr;
  };
  auto kv_rows = [&](int64_t blk, const __nv_bfloat16* base, int64_t sb, int64_t st, int64_t sh) {
    return [=](int r) -> const __nv_bfloat16* {
      const int64_t kk = blk * kBlk + r;
      return kk < f.T ? base + b * sb + kk * st + hk * sh : nullptr;
    };
  };
  load_operand<kTileM>(q_s, kTile128 / 2, q_row, tid, f.q);
  load_operand<kTileM>(do_s, kTile128 / 2, g_row, tid, a.dout);
  load_operand<kBlk>(kv_s, kKVHalf, kv_rows(blo, f.k, f.skb, f.skt, f.skh), tid, f.k);
  load_operand<kBlk>(kv_s + kKVBytes, kKVHalf, kv_rows(blo, f.v, f.svb, f.svt, f.svh), tid, f.v);
  cp_async_commit();
  bool aborted = false;
  for (int64_t j = blo; j <= bhi; ++j) {
    const int jj = static_cast<int>(j - blo);
    const int st = jj & 1;
    cp_async_wait<0>();
    fence_async_smem();
    __syncthreads();
    const uint32_t k_cur = kv_s + st * 2 * kKVBytes, v_cur = k_cur + kKVBytes;
    if (tid == 0) {
      tc_fence_after();
      issue_qk(tm_s, q_s, k_cur);
      issue_qk(tm_dp, do_s, v_cur);
      mma_commit(&bar_s);
      ok_s = mbar_wait(&bar_s, jj & 1, 321) ? 1 : 0;
    }
    __syncthreads();
    if (!ok_s) { aborted = true; break; }
    if (j + 1 <= bhi) {
      const uint32_t nx = kv_s + (st ^ 1) * 2 * kKVBytes;
      load_operand<kBlk>(nx, kKVHalf, kv_rows(j + 1, f.k, f.skb, f.skt, f.skh), tid, f.k);
      load_operand<kBlk>(nx + kKVBytes, kKVHalf, kv_rows(j + 1, f.v, f.svb, f.svt, f.svh), tid, f.v);
    }
    cp_async_commit();
    tc_fence_after();
    float sv[64], dp[64];
    {
      float x0[32], x1[32];
      tmem_ld32(tm_s + lane_off, x0);
      tmem_ld32(tm_s + lane_off + 32, x1);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) { sv[i] = x0[i]; sv[32 + i] = x1[i]; }
      tmem_ld32(tm_dp + lane_off, x0);
      tmem_ld32(tm_dp + lane_off + 32, x1);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) { dp[i] = x0[i]; dp[32 + i] = x1[i]; }
    }
    const int64_t k0 = j * kBlk;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int64_t kk = k0 + i;
      const bool valid = row_ok && kk >= ls && kk <= t;
      const float p = valid ? exp2f(sv[i] * f.scale_log2 - lse2) : 0.f;
      dp[i] = p * (dp[i] - dlt);
    }
    store_p_row(v_cur, tid, 0, dp);  // dS over the dead V operand of this stage
    store_p_row(v_cur, tid, 4, dp + 32);
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      issue_pv(tm_dq, v_cur, k_cur, jj > 0);  // dQ += dS K (K MN-major)
      mma_commit(&bar_o);
    }
  }
  const int nblocks = static_cast<int>(bhi - blo + 1);
  if (tid == 0) ok_s = mbar_wait(&bar_o, (nblocks - 1) & 1, 322) ? 1 : 0;
  __syncthreads();
  cp_async_wait<0>();
  if (!aborted && ok_s) {
    tc_fence_after();
    const int64_t hi = (hk * f.HI) / f.Hkv;
    int64_t slot_rows[64];
    int nsl = 0;
    if (row_ok && f.S > 0) {
      const int32_t* srow = f.sel + ((b * f.HI + hi) * f.T + t) * f.S;
      for (int64_t s2 = 0; s2 < f.S && s2 < 64; ++s2) {
        const int64_t blk = srow[s2];
        if (blk < 0 || blk >= f.nblk) continue;
        int64_t lo, hi2;
        remote_range(f, b, t, blk, lo, hi2);
        if (lo >= hi2) continue;
        bool dup = false;
        for (int64_t u = 0; u < s2; ++u) dup |= srow[u] == blk;
        if (dup) continue;
        slot_rows[nsl++] = ((b * f.T + t) * f.S + s2) * f.HQ + h;
      }
    }
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float ov[32];
      tmem_ld32(tm_dq + lane_off + 32 * c, ov);
      tmem_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int i = 0; i < 32; ++i) ov[i] *= a.scale;
        for (int u = 0; u < nsl; ++u) {
          const uint4* src = reinterpret_cast<const uint4*>(a.dq_part + slot_rows[u] * kD + 32 * c);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint4 w = src[q4];
            ov[8 * q4 + 0] += bf16_lo(w.x); ov[8 * q4 + 1] += bf16_hi(w.x);
            ov[8 * q4 + 2] += bf16_lo(w.y); ov[8 * q4 + 3] += bf16_hi(w.y);
            ov[8 * q4 + 4] += bf16_lo(w.z); ov[8 * q4 + 5] += bf16_hi(w.z);
            ov[8 * q4 + 6] += bf16_lo(w.w); ov[8 * q4 + 7] += bf16_hi(w.w);
          }
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          store8(a.dq + b * f.sqb + t * f.sqt + h * f.sqh + 32 * c, 8 * q4, SRSWA_BF16, ov + 8 * q4);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// d_bias[b,t,s] = sum over query heads of the per-head partials (fixed order)
__global__ void tc_dbias_reduce_kernel(const TcBwdArgs a) {
  const TcArgs& f = a.f;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= f.B * f.T * f.S) return;
  float acc = 0.f;
  for (int64_t h = 0; h < f.HQ; ++h) acc += a.dbias_part[i * f.HQ + h];
  a.d_bias[i] = acc;
}

// ---------------------------------------------------------------------------
struct TcLayout {
  size_t part_o, part_lse, count, offs, cursor, tiles, ntiles, pairs, total;
  int64_t max_tiles;
};

static size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

TcLayout tc_layout(const srswa_gather_desc* g) {
  TcLayout L;
  const int64_t nblk = (g->T + kBlk - 1) / kBlk;
  const int64_t nbh = g->B * g->HI * nblk;
  const int64_t npairs = g->B * g->HI * g->T * g->S;
  L.max_tiles = npairs / kTileM + nbh + 1;
  size_t off = 0;
  L.part_o = off;
  off += al256(static_cast<size_t>(g->B * g->T * g->S * g->HQ * kD) * 2);
  L.part_lse = off;
  off += al256(static_cast<size_t>(g->B * g->T * g->S * g->HQ) * 4);
  L.count = off;
  off += al256(static_cast<size_t>(nbh) * 4);
  L.offs = off;
  off += al256(static_cast<size_t>(nbh) * 4);
  L.cursor = off;
  off += al256(static_cast<size_t>(nbh) * 4);
  L.tiles = off;
  off += al256(static_cast<size_t>(L.max_tiles) * 16);
  L.ntiles = off;
  off += 256;
  L.pairs = off;
  off += al256(static_cast<size_t>(npairs) * 4);
  L.total = off;
  return L;
}

bool tc_eligible(const srswa_gather_desc* g) {
  return g->D == kD && g->block_size == kBlk && g->dtype == SRSWA_BF16 && g->S <= 64 && g->T > 0 &&
         ((g->sqb | g->sqt | g->sqh | g->skb | g->skt | g->skh | g->svb | g->svt | g->svh) & 7) == 0;
}

int tc_gather_fwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v, const int32_t* sel,
                  const float* bias, const int32_t* seg, void* o, int64_t sob, int64_t sot, int64_t soh, float* lse,
                  void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const TcLayout L = tc_layout(g);
  if (!workspace || workspace_bytes < L.total) return SRSWA_EWORKSPACE;
  char* ws = static_cast<char*>(workspace);
  TcArgs a = {};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.sqb = g->sqb; a.sqt = g->sqt; a.sqh = g->sqh; a.skb = g->skb; a.skt = g->skt; a.skh = g->skh;
  a.svb = g->svb; a.svt = g->svt; a.svh = g->svh;
  a.o = static_cast<__nv_bfloat16*>(o); a.sob = sob; a.sot = sot; a.soh = soh; a.lse = lse;
  a.sel = sel; a.bias = bias; a.seg = seg;
  a.part_o = reinterpret_cast<__nv_bfloat16*>(ws + L.part_o);
  a.part_lse = reinterpret_cast<float*>(ws + L.part_lse);
  a.pairs = reinterpret_cast<int32_t*>(ws + L.pairs);
  a.tiles = reinterpret_cast<int4*>(ws + L.tiles);
  a.ntiles = reinterpret_cast<int32_t*>(ws + L.ntiles);
  a.B = g->B; a.T = g->T; a.HQ = g->HQ; a.Hkv = g->Hkv; a.HI = g->HI; a.S = g->S;
  a.LW = g->local_window > 0 ? g->local_window : kBlk;
  a.nblk = (g->T + kBlk - 1) / kBlk;
  a.scale_log2 = g->scale * kLog2e;
  int32_t* count = reinterpret_cast<int32_t*>(ws + L.count);
  int32_t* offs = reinterpret_cast<int32_t*>(ws + L.offs);
  int32_t* cursor = reinterpret_cast<int32_t*>(ws + L.cursor);

  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(band_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBandSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaFuncSetAttribute(remote_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRemoteSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done = true;
  }
  if (g->S > 0) {
    const int64_t nbh = a.B * a.HI * a.nblk;
    SRSWA_CUDA_TRY(cudaMemsetAsync(count, 0, static_cast<size_t>(nbh) * 4, st));
    const int64_t rows = a.B * a.HI * a.T;
    pairs_count_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, st>>>(a, count);
    SRSWA_CUDA_TRY(cudaGetLastError());
    pairs_scan_kernel<<<1, 1024, 0, st>>>(a, count, offs, cursor, const_cast<int4*>(a.tiles),
                                          const_cast<int32_t*>(a.ntiles));
    SRSWA_CUDA_TRY(cudaGetLastError());
    pairs_fill_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, st>>>(a, cursor,
                                                                               const_cast<int32_t*>(a.pairs));
    SRSWA_CUDA_TRY(cudaGetLastError());
    remote_fwd_kernel<<<148 * 3, kTcThreads, kRemoteSmem, st>>>(a);
    SRSWA_CUDA_TRY(cudaGetLastError());
  } else {
    a.part_o = nullptr;
  }
  dim3 grid(static_cast<unsigned>((g->T + kTileM - 1) / kTileM), static_cast<unsigned>(g->HQ),
            static_cast<unsigned>(g->B));
  band_fwd_kernel<<<grid, kTcThreads, kBandSmem, st>>>(a);
  return srswa_last_launch_status();
}


// ---------------------------------------------------------------------------
struct TcBwdLayout {
  size_t delta, dq_part, dbias_part, dkv_part, bitmap, count, offs, cursor, tiles, ntiles, pairs, total;
  int64_t max_tiles, T32;
};

TcBwdLayout tc_bwd_layout(const srswa_gather_desc* g, bool with_bias) {
  TcBwdLayout L;
  const int64_t nblk = (g->T + kBlk - 1) / kBlk;
  const int64_t nbh = g->B * g->HI * nblk;
  const int64_t npairs = g->B * g->HI * g->T * g->S;
  L.max_tiles = npairs / kTileM + nbh + 1;
  L.T32 = (g->T + 31) / 32;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += al256(bytes);
    return at;
  };
  L.delta = take(static_cast<size_t>(g->B * g->T * g->HQ) * 4);
  const bool remote = g->S > 0;
  L.dq_part = take(remote ? static_cast<size_t>(g->B * g->T * g->S * g->HQ * kD) * 2 : 0);
  L.dbias_part = take(remote && with_bias ? static_cast<size_t>(g->B * g->T * g->S * g->HQ) * 4 : 0);
  L.dkv_part = take(remote ? static_cast<size_t>(g->B * g->HQ * nblk) * 2 * kBlk * kD * 4 : 0);
  L.bitmap = take(remote ? static_cast<size_t>(nbh * L.T32) * 4 : 0);
  L.count = take(static_cast<size_t>(nbh) * 4);
  L.offs = take(static_cast<size_t>(nbh) * 4);
  L.cursor = take(static_cast<size_t>(nbh) * 4);
  L.tiles = take(remote ? static_cast<size_t>(L.max_tiles) * 16 : 0);
  L.ntiles = take(4);
  L.pairs = take(static_cast<size_t>(npairs) * 4);
  L.total = off;
  return L;
}

size_t tc_bwd_workspace(const srswa_gather_desc* g, bool with_bias) { return tc_bwd_layout(g, with_bias).total; }

int tc_gather_bwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v, const void* o,
                  int64_t sob, int64_t sot, int64_t soh, const void* dout, const float* lse, const int32_t* sel,
                  const float* bias, const int32_t* seg, void* dq, void* dk, void* dv, float* d_bias,
                  void* workspace, size_t workspace_bytes, cudaStream_t st) {
  const TcBwdLayout L = tc_bwd_layout(g, bias != nullptr);
  if (!workspace || workspace_bytes < L.total) return SRSWA_EWORKSPACE;
  char* ws = static_cast<char*>(workspace);
  TcBwdArgs a = {};
  TcArgs& f = a.f;
  f.q = static_cast<const __nv_bfloat16*>(q);
  f.k = static_cast<const __nv_bfloat16*>(k);
  f.v = static_cast<const __nv_bfloat16*>(v);
  f.sqb = g->sqb; f.sqt = g->sqt; f.sqh = g->sqh; f.skb = g->skb; f.skt = g->skt; f.skh = g->skh;
  f.svb = g->svb; f.svt = g->svt; f.svh = g->svh;
  f.o = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(o));
  f.sob = sob; f.sot = sot; f.soh = soh;
  f.sel = sel; f.bias = bias; f.seg = seg;
  f.pairs = reinterpret_cast<int32_t*>(ws + L.pairs);
  f.tiles = reinterpret_cast<int4*>(ws + L.tiles);
  f.ntiles = reinterpret_cast<int32_t*>(ws + L.ntiles);
  f.B = g->B; f.T = g->T; f.HQ = g->HQ; f.Hkv = g->Hkv; f.HI = g->HI; f.S = g->S;
  f.LW = g->local_window > 0 ? g->local_window : kBlk;
  f.nblk = (g->T + kBlk - 1) / kBlk;
  f.scale_log2 = g->scale * kLog2e;
  a.dout = static_cast<const __nv_bfloat16*>(dout);
  a.lse = lse;
  a.delta = reinterpret_cast<float*>(ws + L.delta);
  a.dq = static_cast<__nv_bfloat16*>(dq);
  a.dk = static_cast<__nv_bfloat16*>(dk);
  a.dv = static_cast<__nv_bfloat16*>(dv);
  a.d_bias = d_bias;
  a.scale = g->scale;
  const bool remote = g->S > 0;
  a.dq_part = remote ? reinterpret_cast<__nv_bfloat16*>(ws + L.dq_part) : nullptr;
  a.dbias_part = remote && bias ? reinterpret_cast<float*>(ws + L.dbias_part) : nullptr;
  a.dkv_part = remote ? reinterpret_cast<float*>(ws + L.dkv_part) : nullptr;
  int32_t* count = reinterpret_cast<int32_t*>(ws + L.count);
  int32_t* offs = reinterpret_cast<int32_t*>(ws + L.offs);
  a.count = remote ? count : nullptr;
  a.offs = offs;

  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(bwd_remote_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRBSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaFuncSetAttribute(bwd_band_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBDSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    e = cudaFuncSetAttribute(bwd_band_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBQSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_done = true;
  }
  const int64_t nrows_h = g->B * g->T * g->HQ;
  tc_delta_kernel<<<static_cast<unsigned>((nrows_h + 7) / 8), 256, 0, st>>>(a);
  SRSWA_CUDA_TRY(cudaGetLastError());
  if (remote) {
    const int64_t nbh = f.B * f.HI * f.nblk;
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(ws + L.bitmap);
    SRSWA_CUDA_TRY(cudaMemsetAsync(bitmap, 0, static_cast<size_t>(nbh * L.T32) * 4, st));
    const int64_t rows = f.B * f.HI * f.T;
    bwd_pairs_bitmap_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, st>>>(f, bitmap, L.T32);
    SRSWA_CUDA_TRY(cudaGetLastError());
    bwd_pairs_count_kernel<<<static_cast<unsigned>((nbh + 7) / 8), 256, 0, st>>>(f, bitmap, L.T32, count);
    SRSWA_CUDA_TRY(cudaGetLastError());
    pairs_scan_kernel<<<1, 1024, 0, st>>>(f, count, offs, reinterpret_cast<int32_t*>(ws + L.cursor),
                                          const_cast<int4*>(f.tiles), const_cast<int32_t*>(f.ntiles));
    SRSWA_CUDA_TRY(cudaGetLastError());
    bwd_pairs_fill_kernel<<<static_cast<unsigned>((nbh + 7) / 8), 256, 0, st>>>(f, bitmap, L.T32, offs,
                                                                              const_cast<int32_t*>(f.pairs));
    SRSWA_CUDA_TRY(cudaGetLastError());
    if (a.dbias_part)
      SRSWA_CUDA_TRY(cudaMemsetAsync(a.dbias_part, 0, static_cast<size_t>(g->B * g->T * g->S * g->HQ) * 4, st));
    bwd_remote_kernel<<<148, kTcThreads, kRBSmem, st>>>(a);
    SRSWA_CUDA_TRY(cudaGetLastError());
  }
  const unsigned ntile = static_cast<unsigned>((g->T + kTileM - 1) / kTileM);
  bwd_band_dkdv_kernel<<<dim3(ntile, static_cast<unsigned>(g->Hkv), static_cast<unsigned>(g->B)), kTcThreads,
                         kBDSmem, st>>>(a);
  SRSWA_CUDA_TRY(cudaGetLastError());
  bwd_band_dq_kernel<<<dim3(ntile, static_cast<unsigned>(g->HQ), static_cast<unsigned>(g->B)), kTcThreads,
                       kBQSmem, st>>>(a);
  SRSWA_CUDA_TRY(cudaGetLastError());
  if (bias) {
    if (remote) {
      const int64_t n = g->B * g->T * g->S;
      tc_dbias_reduce_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(a);
    }
  }
  return srswa_last_launch_status();
}
}  // namespace srswa

extern "C" int srswa_device_status(int* out) {
  if (!out) return SRSWA_EINVAL;
  return srswa::tc_read_clear_error(out);
}
