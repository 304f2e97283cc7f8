// Gather attention (forward and backward) on the 5th-generation tensor cores
// (tcgen05 / TMEM), fed by TMA and cp.async gathers.
//
// Same semantics as the query-major kernels (K1/K5 of the reference:
// hf-model-code/sparse_gather_triton.py:35-122, sparse_gather_e2e_triton.py:36-121,
// and their backward), split in two passes so that every MMA has M = 128
// real rows:
//
//  1. remote pass (remote_ws_kernel): the selection is inverted into per
//     (batch, index head, block) lists of (query, slot) pairs; a work item is
//     one selected block of one query head with all of its pairs, in tiles of
//     128 rows gathered into shared memory.  S = Q_g K_blk^T (M=128, N=64,
//     K=128) goes to TMEM, the per-row softmax (slot bias, keys below the
//     query's window start) runs on the 128 rows, O = P V_blk (N=128) goes to
//     TMEM and the normalised partial (o bf16, lse fp32 log2) is written to a
//     [B, T, S, HQ, D] workspace.
//  2. band pass (fwd_ws_kernel): per (batch, head, 128-query tile) the ~LW/64
//     + 2 key blocks of the local window go through an online softmax (lazy
//     rescaling of O in TMEM when the running max grows by more than 2^8) and
//     the window result (o, lse) is written.
//  3. merge_partials_kernel folds each row's remote partials into the window
//     result with log-sum-exp weights.
//
// The backward mirrors it: bwd_remote_ws_kernel (dK/dV/dq partials per
// selected block), bwd_band_dq_ws_kernel and bwd_band_dkdv_ws_kernel (the
// window), then bandwidth-bound merges of the dq and dK/dV partials.
//
// All kernels are warp-specialised and persistent: producer warps (TMA or
// cp.async), one MMA-issuing thread, and softmax / compute warpgroups, tied
// by mbarriers.  Every wait is bounded; an expired wait sets an abort flag,
// the MMA warp drains the tensor pipe with a final commit and TMEM is freed.
// Shared-memory operand layout: see tc.cuh (128-byte swizzle, K-major Q/K/P,
// MN-major V).

#include <mutex>

#include <cuda.h>  // CUtensorMap (the encoder is looked up at run time; libcuda is not linked)

#include "attend.cuh"
#include "common.cuh"
#include "tc.cuh"

namespace srswa {

constexpr int kTileM = 128;
constexpr int kBlk = 64;        // key block (BS)
constexpr int kD = 128;         // head dim
constexpr float kRescaleLog2 = 8.0f;  // lazy O rescale threshold (factor 256)

// smem layout of the band kernel (bytes, 1024-aligned pieces)
constexpr uint32_t kQBytes = kTileM * 128 * 2;  // two 64-col halves of [128 x 128 B]
constexpr uint32_t kKVHalf = kBlk * 128;        // [64 rows x 128 B]
constexpr uint32_t kKVBytes = 2 * kKVHalf;      // one 64 x 128 operand
constexpr uint32_t kPBytes = kTileM * 128;      // [128 x 64 keys] bf16 (fits a K operand's 16 KB)
// P of a block is written over that block's K operand, dead once S is in TMEM

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
  // forward remote pass: every (b*HI + hi, block) list owns whole 128-row
  // tiles of partial rows; a selection's partial row is prow[b, hi, t, s]
  __nv_bfloat16* part_o;      // [prow_cap, HQ/HI, D] bf16, normalised
  float* part_lse;            // [prow_cap, HQ/HI] log2 domain
  int32_t* prow;              // [B, HI, T, S] partial row, -1 if none
  int32_t* pair_t;            // per partial row: query t
  int64_t* pair_q;            // per partial row: b * sqb + t * sqt (the query head's offset is added per unit)
  float* pair_bias;           // per partial row: slot bias * log2 e (0 without bias)
  const int4* work;           // nonempty lists: (b*HI + hi) * nblk + block, first tile, pair count, 0
  const int32_t* totals;      // {tiles, nonempty lists}
  int* status;                // the call's status word: 0, or the code of the first expired wait
  int64_t prow_cap;           // partial rows (each holds the HQ/HI heads of an index head)
  // backward lists
  const int32_t* pairs;       // packed t * S + s, grouped by (b, hi, block)
  const int4* tiles;          // (b*HI + hi, block, first pair, count)
  const int32_t* ntiles;      // device count of tiles
  const int32_t* count;       // pairs per (b*HI + hi, block)
  const int32_t* offs;        // first pair of each (b*HI + hi, block)
  int64_t B, T, HQ, Hkv, HI, S, LW, nblk;
  float scale_log2;
  // paged K / V (forward only): key block j of batch element b is the whole
  // page kv_pages[b * s_pages + j] of the caches (the tensor maps then span
  // [pages, 64 slots, Hkv, D]); query row t sits at position t + qoff (a
  // cached prefix of qoff tokens precedes the rows).  Null / 0: contiguous
  // [B, T, H, D] keys at the rows' own positions.
  const int32_t* kv_pages;
  int64_t s_pages, qoff;
  int64_t tail_blk, tail_slots;  // paged (B = 1): the last block and its used slots (0: full)
};

// position of query row t
__device__ __forceinline__ int64_t qpos(const TcArgs& a, int64_t t) { return t + a.qoff; }

// TMA coordinates (row, batch) of key block blk of batch element b; kPaged:
// the forward kernels' paged instantiation (a.kv_pages set)
template <bool kPaged>
__device__ __forceinline__ void kv_coord(const TcArgs& a, int64_t b, int64_t blk, int& row0, int& bb) {
  if constexpr (kPaged) {
    row0 = 0;
    bb = a.kv_pages[b * a.s_pages + blk];
  } else {
    row0 = static_cast<int>(blk * kBlk);
    bb = static_cast<int>(b);
  }
}

__device__ __forceinline__ int64_t seg_start(const TcArgs& a, int64_t b, int64_t t) {
  return a.seg ? static_cast<int64_t>(a.seg[b * a.T + t]) : 0;
}
__device__ __forceinline__ int64_t win_start(const TcArgs& a, int64_t b, int64_t t) {
  int64_t ls = qpos(a, t) - a.LW + 1;
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
  hi = min(min((blk + 1) * kBlk, ls), qpos(a, t) + 1);
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

// O (+)= P V with P (bf16, [128 x 64 keys]) in TMEM: A from TMEM, 8 columns
// per 16-key step; V MN-major in shared memory as in issue_pv
__device__ __forceinline__ void issue_pv_tmem(uint32_t tmem_o, uint32_t tmem_p, uint32_t v_s, bool accumulate) {
  constexpr uint32_t id = idesc_bf16(128, 128, 1);
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    const uint64_t bd = sw128_desc(v_s + ks * 2048u, kKVHalf, 1024);
    mma_bf16_ts(tmem_o, tmem_p + ks * 8u, bd, id, (accumulate || ks > 0) ? 1u : 0u);
  }
}
// 64 fp32 -> 32 packed bf16 pairs (lower key in the low half) into a row's
// 32 TMEM columns (warp-collective)
__device__ __forceinline__ void store_p_tmem(uint32_t taddr, const float (&p)[64]) {
  uint32_t w[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(p[2 * i], p[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  tmem_st32u(taddr, w);
}

// ============================================================================
// remote pass: inverted selection lists
// ============================================================================
// Usable selection (t, slot) of row srow: a valid block with remote keys for
// the query and not a repeat of an earlier slot (else -1).
__device__ __forceinline__ int64_t usable_block(const TcArgs& a, const int32_t* srow, int64_t b, int64_t t,
                                                int64_t s) {
  const int64_t blk = srow[s];
  if (blk < 0 || blk >= a.nblk) return -1;
  int64_t lo, hi;
  remote_range(a, b, t, blk, lo, hi);
  if (lo >= hi) return -1;
  for (int64_t u = 0; u < s; ++u)
    if (srow[u] == blk) return -1;
  return blk;
}

// count[b*HI+hi][blk] += 1 for every usable (t, slot) selection.  A CTA
// takes 256 queries of one (b, hi) (thread = query) and counts into a
// shared-memory histogram over the blocks first, so the global counters see
// one atomic per nonzero bin and CTA.
constexpr int kListRows = 256;
__global__ void __launch_bounds__(kListRows) pairs_count_kernel(const TcArgs a, int32_t* count) {
  extern __shared__ int32_t hist[];  // [nblk]
  const int64_t bh = blockIdx.y, b = bh / a.HI;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kListRows + threadIdx.x;
  for (int64_t i = threadIdx.x; i < a.nblk; i += kListRows) hist[i] = 0;
  __syncthreads();
  if (t < a.T) {
    const int32_t* srow = a.sel + (bh * a.T + t) * a.S;
    for (int64_t s = 0; s < a.S; ++s) {
      const int64_t blk = usable_block(a, srow, b, t, s);
      if (blk >= 0) atomicAdd(&hist[blk], 1);
    }
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < a.nblk; i += kListRows)
    if (hist[i]) atomicAdd(count + bh * a.nblk + i, hist[i]);
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

// Forward lists: single-CTA scans over the (b*HI + hi, block) lists.  Every
// list gets whole 128-row tiles of partial rows: its first tile (exclusive
// scan of ceil(count / 128)) sets its fill cursor to tile * 128, and the
// nonempty lists are compacted into work[] = (list, first tile, count, 0).
// totals = {tiles, nonempty lists}.
__global__ void fwd_lists_scan_kernel(const TcArgs a, const int32_t* count, int32_t* cursor, int4* work,
                                      int32_t* totals) {
  __shared__ int32_t sh_t[1024], sh_w[1024];
  const int64_t n = a.B * a.HI * a.nblk;
  int32_t base_t = 0, base_w = 0;
  for (int64_t c0 = 0; c0 < n; c0 += 1024) {
    const int64_t i = c0 + threadIdx.x;
    const int32_t cnt = i < n ? count[i] : 0;
    const int32_t nt = (cnt + kTileM - 1) / kTileM;
    sh_t[threadIdx.x] = nt;
    sh_w[threadIdx.x] = cnt > 0 ? 1 : 0;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {  // inclusive Hillis-Steele scans
      const int32_t vt = threadIdx.x >= static_cast<unsigned>(o) ? sh_t[threadIdx.x - o] : 0;
      const int32_t vw = threadIdx.x >= static_cast<unsigned>(o) ? sh_w[threadIdx.x - o] : 0;
      __syncthreads();
      sh_t[threadIdx.x] += vt;
      sh_w[threadIdx.x] += vw;
      __syncthreads();
    }
    if (i < n) {
      const int32_t ot = base_t + sh_t[threadIdx.x] - nt;
      cursor[i] = ot * kTileM;
      if (cnt > 0) work[base_w + sh_w[threadIdx.x] - 1] = make_int4(static_cast<int>(i), ot, cnt, 0);
    }
    __syncthreads();
    base_t += sh_t[1023];
    base_w += sh_w[1023];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    totals[0] = base_t;
    totals[1] = base_w;
  }
}

// Forward lists: each usable (t, slot) selection takes the next partial row
// of its list and records the row's query, q offset and bias; prow maps
// every selection to its row (-1: unused, repeated or without remote keys).
// A CTA takes 256 queries of one (b, hi): it counts its selections per block
// in shared memory, reserves each block's rows with one global atomic, then
// hands out the rows from shared-memory counters.
__global__ void __launch_bounds__(kListRows) pairs_fill_kernel(const TcArgs a, int32_t* cursor) {
  extern __shared__ int32_t hist[];  // [2 * nblk]: counts, then reserved bases
  int32_t* base = hist + a.nblk;
  const int64_t bh = blockIdx.y, b = bh / a.HI;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kListRows + threadIdx.x;
  for (int64_t i = threadIdx.x; i < a.nblk; i += kListRows) hist[i] = 0;
  __syncthreads();
  const int32_t* srow = a.sel + (bh * a.T + t) * a.S;
  if (t < a.T)
    for (int64_t s = 0; s < a.S; ++s) {
      const int64_t blk = usable_block(a, srow, b, t, s);
      if (blk >= 0) atomicAdd(&hist[blk], 1);
    }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < a.nblk; i += kListRows) {
    base[i] = hist[i] ? atomicAdd(cursor + bh * a.nblk + i, hist[i]) : 0;
    hist[i] = 0;
  }
  __syncthreads();
  if (t >= a.T) return;
  int32_t* prow = a.prow + (bh * a.T + t) * a.S;
  for (int64_t s = 0; s < a.S; ++s) {
    const int64_t blk = usable_block(a, srow, b, t, s);
    int32_t row = -1;
    if (blk >= 0) {
      row = base[blk] + atomicAdd(&hist[blk], 1);
      a.pair_t[row] = static_cast<int32_t>(t);
      a.pair_q[row] = b * a.sqb + t * a.sqt;
      a.pair_bias[row] = a.bias ? a.bias[(b * a.T + t) * a.S + s] * kLog2e : 0.f;
    }
    prow[s] = row;
  }
}

// ============================================================================
// Warp-specialised band forward (the local window of every query).
//
// A CTA is persistent over work items (b, h, 128-query tile) and runs two
// items at a time, one per slot.
//   warps 0-3 / 4-7  softmax warpgroup of slot 0 / 1 (thread = query row): S
//                    from TMEM, causal / window mask, online softmax with lazy
//                    O rescale, P (bf16) over the dead K operand, and the
//                    item's epilogue (o, lse) from O in TMEM;
//   warp 8           producer: TMA loads of the slot's Q tile and of each key
//                    block's K and V into the slot's 2-stage ring;
//   warp 9           MMA issuer (one thread) and TMEM owner: S = Q K^T and
//                    O += P V of the two slots in ping-pong order, so one
//                    slot's MMAs run while the other slot's softmax does.
// Every wait is bounded and also gives up once another role has set the CTA's
// abort flag, so a stuck role releases the others; the CTA then drains the
// tensor pipe and frees TMEM.
// ============================================================================
constexpr int kWsThreads = 320;
constexpr int kWsProducer = 8, kWsMma = 9;
constexpr uint32_t kWsStage = 2 * kKVBytes;                              // K then V
constexpr uint32_t kWsSmem = 2 * kQBytes + 2 * 2 * kWsStage + 1024;      // 193 KB -> 1 CTA/SM
constexpr uint32_t kWsTmemCols = 512;  // per slot: S 0-63, P (bf16) 64-95, O 128-255

// Bounded wait of one role: suspended try_waits until the phase completes,
// the CTA's abort flag is set (another role gave up) or the wall-clock bound
// expires (error recorded, abort flag set).  The first test is inline; the
// rest is one shared out-of-line function, which keeps the roles' loops small
// in the instruction cache.
__device__ __noinline__ bool ws_wait_slow(uint32_t a, uint32_t parity, volatile int* abort_flag, int code) {
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait(a, parity)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > kWaitLimitNs) break;
  }
  atomicCAS(const_cast<int*>(abort_flag), 0, code);
  return false;
}
__device__ __forceinline__ bool ws_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  return ws_wait_slow(a, parity, abort_flag, code);
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// arrive once every cp.async this thread issued so far has landed
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 2^x on the MUFU unit (ex2.approx, flush-to-zero; 2^-inf = +0)
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Max of one row's raw scores of a 64-key block; keys outside [lo, hi)
// (relative to the block) are set to -inf first unless `full` (warp-uniform)
// says every key is valid.  Four independent max chains.
__device__ __forceinline__ float block_row_max(float (&sv)[64], int lo, int hi, bool full) {
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  if (full) {
#pragma unroll
    for (int i = 0; i < 64; ++i) m[i & 3] = fmaxf(m[i & 3], sv[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      sv[i] = (i >= lo && i < hi) ? sv[i] : -INFINITY;
      m[i & 3] = fmaxf(m[i & 3], sv[i]);
    }
  }
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}
// In place p = 2^(s * c + off) (c > 0; masked keys hold -inf and give 0);
// returns the row sum (four independent chains)
__device__ __forceinline__ float block_row_exp(float (&sv)[64], float c, float off) {
  float l[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    sv[i] = fast_exp2(fmaf(sv[i], c, off));
    l[i & 3] += sv[i];
  }
  return (l[0] + l[1]) + (l[2] + l[3]);
}
__device__ __forceinline__ int clamp_key(int64_t v) { return static_cast<int>(v < 0 ? 0 : (v > kBlk ? kBlk : v)); }

// A band work item: (b, h, 128-query tile) and its window's key blocks.
struct WsItem {
  int64_t b, h, hk;
  int64_t blo, bhi;  // key blocks, inclusive
  int64_t t0;        // first query row
};

__device__ __forceinline__ int64_t ws_num_items(const TcArgs& a) {
  return a.B * a.HQ * ((a.T + kTileM - 1) / kTileM);
}

__device__ __forceinline__ WsItem ws_item(const TcArgs& a, int64_t item) {
  WsItem w;
  const int64_t nt = (a.T + kTileM - 1) / kTileM;
  const int64_t tile = item % nt, bh = item / nt;
  w.b = bh / a.HQ;
  w.h = bh % a.HQ;
  w.t0 = tile * kTileM;
  const int64_t tlast = min(a.T, w.t0 + kTileM) - 1;
  int64_t key_lo = qpos(a, w.t0) - a.LW + 1;
  if (key_lo < 0) key_lo = 0;
  w.blo = key_lo / kBlk;
  w.bhi = qpos(a, tlast) / kBlk;
  w.hk = w.h / (a.HQ / a.Hkv);
  return w;
}

// The step sequence of one slot: its items (blockIdx.x + (2m + slot) *
// gridDim.x) and, inside each, the key blocks blo..bhi.  Every role walks the
// same sequence.
struct WsCursor {
  int64_t item, nitems, m, j, n;
  WsItem w;
  bool done;
  __device__ __forceinline__ void start(const TcArgs& a, int slot, int64_t ni) {
    nitems = ni;
    item = blockIdx.x + static_cast<int64_t>(slot) * gridDim.x;
    m = 0;
    n = 0;
    done = item >= nitems;
    if (!done) {
      w = ws_item(a, item);
      j = w.blo;
    }
  }
  __device__ __forceinline__ bool first() const { return j == w.blo; }
  __device__ __forceinline__ bool last() const { return j == w.bhi; }
  __device__ __forceinline__ void advance(const TcArgs& a) {
    ++n;
    if (j < w.bhi) {
      ++j;
      return;
    }
    ++m;
    item += 2 * static_cast<int64_t>(gridDim.x);
    done = item >= nitems;
    if (!done) {
      w = ws_item(a, item);
      j = w.blo;
    }
  }
};

// 16 fp32 * scale -> 16 bf16 stored as one 32-byte word (dst 32-byte aligned)
__device__ __forceinline__ void st_global_bf16x16(__nv_bfloat16* dst, const float* v, float scale) {
  uint32_t w[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e] * scale, v[2 * e + 1] * scale);
    w[e] = *reinterpret_cast<uint32_t*>(&h);
  }
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// 32 fp32 * scale -> 32 bf16 at dst (16-byte aligned): two 32-byte stores
// where dst is 32-byte aligned, else four 16-byte ones.  A thread writes one
// row, so each store of a warp touches 32 rows: wide stores halve the count.
__device__ __forceinline__ void store_row32(__nv_bfloat16* dst, const float* v, float scale) {
  if ((reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
    st_global_bf16x16(dst, v, scale);
    st_global_bf16x16(dst + 16, v + 16, scale);
    return;
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * q + 2 * e] * scale, v[8 * q + 2 * e + 1] * scale);
      w[e] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(dst + 8 * q) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Band epilogue of one row in the warp-specialised kernel: the window-only
// result, o = O / l (bf16) and lse (ln); merge_partials_kernel folds the
// remote partials in afterwards.  Called by whole warps (tcgen05.ld is
// warp-collective).
__device__ __forceinline__ void band_row_store(const TcArgs& a, int64_t b, int64_t h, int64_t t, bool row_ok,
                                               float m_ref, float l, uint32_t tm_o_row) {
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float ov[32];
    tmem_ld32(tm_o_row + 32 * c, ov);
    tmem_wait_ld();
    if (row_ok) store_row32(a.o + b * a.sob + t * a.sot + h * a.soh + 32 * c, ov, inv);
  }
  if (row_ok && a.lse) a.lse[(b * a.T + t) * a.HQ + h] = l > 0.f ? (m_ref + log2f(l)) * kLn2 : -INFINITY;
}

// Log-sum-exp merge of the window result (o, lse, as written by the band
// pass) with the remote partials.  One CTA per (b, t) and up to 16 heads
// (blockIdx.y), thread = (head, 8 features): a selection's partials of all
// heads of its index head are one contiguous run of rows, so every load is a
// coalesced 16-byte word.  prow (-1: no partial, i.e. unused, repeated or
// without remote keys) is read by all threads of the index head; slots go in
// groups of eight with an online rescale.  Heads without a partial keep the
// window result.  Memory-bound.
constexpr int kMgHeads = 16;  // heads per CTA
__global__ void __launch_bounds__(kMgHeads * 16) merge_partials_kernel(const TcArgs a) {
  const int64_t bt = blockIdx.x;
  const int64_t h = static_cast<int64_t>(blockIdx.y) * kMgHeads + (threadIdx.x >> 4);
  const int f8 = threadIdx.x & 15;
  if (h >= a.HQ) return;
  const int64_t t = bt % a.T, b = bt / a.T;
  const int64_t hpi = a.HQ / a.HI, hi = h / hpi, hl = h - hi * hpi;
  const int32_t* pr = a.prow + ((b * a.HI + hi) * a.T + t) * a.S;
  float* lse_p = a.lse + bt * a.HQ + h;
  uint4* op = reinterpret_cast<uint4*>(a.o + b * a.sob + t * a.sot + h * a.soh) + f8;
  const float lb = *lse_p * kLog2e;
  const uint4 ob = *op;
  const int ns = static_cast<int>(a.S);
  float M = lb, den = lb == -INFINITY ? 0.f : 1.f;  // weights relative to M
  float acc[8];
  {
    const uint32_t wv[4] = {ob.x, ob.y, ob.z, ob.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[2 * e] = lb == -INFINITY ? 0.f : bf16_lo(wv[e]);
      acc[2 * e + 1] = lb == -INFINITY ? 0.f : bf16_hi(wv[e]);
    }
  }
  bool any = false;
  for (int g0 = 0; g0 < ns; g0 += 8) {
    int32_t rk[8];
    float lk[8];
    uint4 uk[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) rk[k] = g0 + k < ns ? __ldg(pr + g0 + k) : -1;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t row = static_cast<int64_t>(rk[k]) * hpi + hl;
      lk[k] = rk[k] >= 0 ? __ldcs(a.part_lse + row) : -INFINITY;
      uk[k] = rk[k] >= 0 ? __ldcs(reinterpret_cast<const uint4*>(a.part_o + row * kD) + f8) : make_uint4(0, 0, 0, 0);
    }
    float gm = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) gm = fmaxf(gm, lk[k]);
    if (gm == -INFINITY) continue;
    any = true;
    if (gm > M) {  // rescale what is accumulated so far
      const float c = M == -INFINITY ? 0.f : exp2f(M - gm);
      den *= c;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] *= c;
      M = gm;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (lk[k] == -INFINITY) continue;
      const float w = exp2f(lk[k] - M);
      den += w;
      const uint32_t wv[4] = {uk[k].x, uk[k].y, uk[k].z, uk[k].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] = fmaf(w, bf16_lo(wv[e]), acc[2 * e]);
        acc[2 * e + 1] = fmaf(w, bf16_hi(wv[e]), acc[2 * e + 1]);
      }
    }
  }
  if (!any) return;  // no remote partial: the window result stands
  const float inv = den > 0.f ? 1.f / den : 0.f;
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 hv = __floats2bfloat162_rn(acc[2 * e] * inv, acc[2 * e + 1] * inv);
    w[e] = *reinterpret_cast<uint32_t*>(&hv);
  }
  *op = make_uint4(w[0], w[1], w[2], w[3]);
  if (f8 == 0) *lse_p = den > 0.f ? (M + log2f(den)) * kLn2 : -INFINITY;
}

template <bool kPaged>
__global__ void __launch_bounds__(kWsThreads, 1)
    fwd_ws_kernel(const TcArgs a, const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmk_tail,
                  const __grid_constant__ CUtensorMap tmv_tail) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t q_full[2], q_empty[2], kv_full[2][2], kv_empty[2][2], s_full[2], p_full[2], o_full[2];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  auto q_s = [&](int s) { return sbase + static_cast<uint32_t>(s) * kQBytes; };
  auto kv_s = [&](int s, int st) { return sbase + 2 * kQBytes + static_cast<uint32_t>(s * 2 + st) * kWsStage; };
  if (warp == kWsMma) {
    tmem_alloc(&tmem_base, kWsTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], kTileM);
      mbar_init(&o_full[s], 1);
      for (int st = 0; st < 2; ++st) {
        mbar_init(&kv_full[s][st], 1);
        mbar_init(&kv_empty[s][st], 1);
      }
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  volatile int* abort_p = &abort_flag;
  const int64_t nitems = ws_num_items(a);

  if (warp == kWsProducer) {
    // ---------------------------------------------------------------- producer
    WsCursor c[2];
    c[0].start(a, 0, nitems);
    c[1].start(a, 1, nitems);
    bool ok = true;
    while (ok && !(c[0].done && c[1].done)) {
      for (int s = 0; s < 2 && ok; ++s) {
        WsCursor& cs = c[s];
        if (cs.done) continue;
        const WsItem& w = cs.w;
        if (cs.first()) {
          if (cs.m > 0 &&
              !__all_sync(0xffffffffu, ws_wait(&q_empty[s], static_cast<uint32_t>((cs.m - 1) & 1), abort_p, 401))) {
            ok = false;
            break;
          }
          if (lane == 0) {
            mbar_arrive_expect_tx(&q_full[s], kQBytes);
            tma_load_4d(q_s(s), &tmq, 0, static_cast<int>(w.t0), static_cast<int>(w.h), static_cast<int>(w.b),
                        &q_full[s]);
            tma_load_4d(q_s(s) + kQBytes / 2, &tmq, 64, static_cast<int>(w.t0), static_cast<int>(w.h),
                        static_cast<int>(w.b), &q_full[s]);
          }
        }
        const int st = static_cast<int>(cs.n & 1);
        if (cs.n >= 2 && !__all_sync(0xffffffffu, ws_wait(&kv_empty[s][st],
                                                          static_cast<uint32_t>(((cs.n >> 1) - 1) & 1), abort_p,
                                                          402))) {
          ok = false;
          break;
        }
        if (lane == 0) {  // K and V of the block: four 64 x 64 boxes (rows past T read as zeros)
          const int hh = static_cast<int>(w.hk);
          int row0, bb;
          kv_coord<kPaged>(a, w.b, cs.j, row0, bb);
          // paged: the sequence's partial last page goes through maps whose
          // slot extent ends at the last token, so its unused slots read as
          // zeros like rows past T of a contiguous tensor
          const bool tail = kPaged && a.tail_slots > 0 && cs.j == a.tail_blk;
          const CUtensorMap* mk = &tmk;
          const CUtensorMap* mv = &tmv;
          if constexpr (kPaged) {
            if (tail) {
              mk = &tmk_tail;
              mv = &tmv_tail;
            }
          }
          const uint32_t dst = kv_s(s, st);
          mbar_arrive_expect_tx(&kv_full[s][st], kWsStage);
          tma_load_4d(dst, mk, 0, row0, hh, bb, &kv_full[s][st]);
          tma_load_4d(dst + kKVHalf, mk, 64, row0, hh, bb, &kv_full[s][st]);
          tma_load_4d(dst + kKVBytes, mv, 0, row0, hh, bb, &kv_full[s][st]);
          tma_load_4d(dst + kKVBytes + kKVHalf, mv, 64, row0, hh, bb, &kv_full[s][st]);
        }
        __syncwarp();
        cs.advance(a);
      }
    }
  } else if (warp == kWsMma) {
    // --------------------------------------------------------------------- MMA
    if (lane == 0) {
      WsCursor c[2];
      c[0].start(a, 0, nitems);
      c[1].start(a, 1, nitems);
      bool pend[2] = {false, false}, pfirst[2] = {false, false}, plast[2] = {false, false};
      int64_t pn[2] = {0, 0};
      bool ok = true;
      auto issue_s = [&](int s) -> bool {
        WsCursor& cs = c[s];
        const int st = static_cast<int>(cs.n & 1);
        if (!ws_wait(&kv_full[s][st], static_cast<uint32_t>((cs.n >> 1) & 1), abort_p, 403)) return false;
        if (cs.first() && !ws_wait(&q_full[s], static_cast<uint32_t>(cs.m & 1), abort_p, 404)) return false;
        tc_fence_after();
        issue_qk(tmem + s * 256, q_s(s), kv_s(s, st));
        mma_commit(&s_full[s]);
        if (cs.last()) mma_commit(&q_empty[s]);
        pend[s] = true;
        pfirst[s] = cs.first();
        plast[s] = cs.last();
        pn[s] = cs.n;
        cs.advance(a);
        return true;
      };
      auto issue_pv_step = [&](int s) -> bool {
        if (!ws_wait(&p_full[s], static_cast<uint32_t>(pn[s] & 1), abort_p, 405)) return false;
        const int st = static_cast<int>(pn[s] & 1);
        tc_fence_after();
        issue_pv_tmem(tmem + s * 256 + 128, tmem + s * 256 + 64, kv_s(s, st) + kKVBytes, !pfirst[s]);
        mma_commit(&kv_empty[s][st]);
        if (plast[s]) mma_commit(&o_full[s]);
        pend[s] = false;
        return true;
      };
      for (int s = 0; s < 2 && ok; ++s)
        if (!c[s].done) ok = issue_s(s);
      while (ok && (pend[0] || pend[1])) {
        for (int s = 0; s < 2 && ok; ++s) {
          if (pend[s]) ok = issue_pv_step(s);
          if (ok && !c[s].done) ok = issue_s(s);
        }
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------------- softmax
    const int s = warp >> 2;
    const int r = tid & (kTileM - 1);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tm_s = tmem + s * 256 + lane_off, tm_o = tmem + s * 256 + 128 + lane_off;
    WsCursor cs;
    cs.start(a, s, nitems);
    float m_ref = -INFINITY, l = 0.f;
    int64_t t = -1, ls = 0;
    bool row_ok = false;
    while (!cs.done) {
      const WsItem& w = cs.w;
      const bool first = cs.first(), last = cs.last();
      if (first) {
        m_ref = -INFINITY;
        l = 0.f;
        t = w.t0 + r;
        row_ok = t < a.T;
        ls = row_ok ? win_start(a, w.b, t) : 0;
      }
      // warp-uniform outcome: the TMEM accesses below are warp-collective
      if (!__all_sync(0xffffffffu, ws_wait(&s_full[s], static_cast<uint32_t>(cs.n & 1), abort_p, 406))) break;
      tc_fence_after();
      float sv[64];
      {
        float s0[32], s1[32];
        tmem_ld32(tm_s, s0);
        tmem_ld32(tm_s + 32, s1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { sv[i] = s0[i]; sv[32 + i] = s1[i]; }
      }
      const int64_t k0 = cs.j * kBlk;
      int klo = 0, khi = 0;  // this row's valid keys of the block, relative
      if (row_ok) {
        klo = clamp_key(ls - k0);
        khi = clamp_key(qpos(a, t) + 1 - k0);
      }
      const bool full = __all_sync(0xffffffffu, klo == 0 && khi == kBlk);
      const float mraw = block_row_max(sv, klo, khi, full);
      const float mloc = mraw == -INFINITY ? -INFINITY : mraw * a.scale_log2;
      const bool need = mloc > m_ref + kRescaleLog2;
      const float alpha = need ? (m_ref == -INFINITY ? 0.f : exp2f(m_ref - mloc)) : 1.f;
      if (need) {
        l *= alpha;
        m_ref = mloc;
      }
      if (__any_sync(0xffffffffu, need && !first)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float ov[32];
          tmem_ld32(tm_o + 32 * c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= alpha;
          tmem_st32(tm_o + 32 * c, ov);
        }
        tmem_wait_st();
      }
      l += block_row_exp(sv, a.scale_log2, m_ref == -INFINITY ? 0.f : -m_ref);
      // P (bf16) into the slot's P columns of TMEM: the previous step's O += P V
      // has read them (S of this step was committed after it)
      store_p_tmem(tmem + s * 256 + 64 + lane_off, sv);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[s]);
      if (last) {
        if (!__all_sync(0xffffffffu, ws_wait(&o_full[s], static_cast<uint32_t>(cs.m & 1), abort_p, 407))) break;
        tc_fence_after();
        band_row_store(a, w.b, w.h, t, row_ok, m_ref, l, tm_o);
        tc_fence_before();
      }
      cs.advance(a);
    }
  }
  // ------------------------------------------------------------------- exit
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) report_status(a.status, abort_p);
  if (warp == kWsMma) {
    if (*abort_p) {  // MMAs may still be in flight: wait for all of them
      if (lane == 0) {
        mma_commit(&drain_bar);
        mbar_wait(&drain_bar, 0, 408, abort_p);
      }
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, kWsTmemCols);
  }
}

// ============================================================================
// Warp-specialised remote pass.  A unit is one 128-row tile of one
// (b*HI + hi, block) pair list for one query head of the index head.  The
// global unit sequence is ordered by list, head and tile, and each CTA takes
// one contiguous, equal share of it: every CTA gets the same number of tiles,
// and consecutive units mostly share their block, whose K and V are loaded
// once per run (a run = the units of one list and head; two TMA stages).
// Roles (thread = row inside the warpgroups):
//   warps 0-3 / 4-7  row warpgroup 0 / 1, the CTA's even / odd units: S from
//                    TMEM, masked to the row's remote keys, exp2 with the slot
//                    bias, P (bf16) into the warpgroup's P columns of TMEM
//                    (O += P V reads A from TMEM); then O from TMEM scaled by
//                    1/l, bf16, staged over the unit's dead Q tile in the
//                    128-byte-swizzled layout and sent to the unit's partial
//                    rows by two TMA stores (one thread); lse (log2) per row.
//                    Both warpgroups run the same code (one instruction
//                    stream in the caches) and each has its own S and O
//                    buffers in TMEM;
//   warps 8-11       producers, 32 rows each: the rows' query and bias into
//                    shared memory, the q rows gathered (cp.async) into a
//                    4-deep Q ring; warp 8 also loads K and V (TMA) at each
//                    run start;
//   warp 12          MMA issuer (one thread) and TMEM owner: S = Q K^T and
//                    O = P V, issuing whichever is ready first (S of unit n+1
//                    may go before O of unit n).
// Every wait is bounded and gives up once another role set the abort flag.
// ============================================================================
constexpr int kRwThreads = 416;
constexpr int kRwProd = 8, kRwMma = 12;  // first warp of each role
constexpr int kRwQ = 4;                  // Q ring depth (Q, then P, then the staged O of a unit)
constexpr uint32_t kRwSmem = kRwQ * kQBytes + 2 * kWsStage + 1024;  // 193 KB

// Walks a CTA's units in order (every role keeps its own copy); 32-bit
// arithmetic (unit, tile and list counts are below 2^31, checked on the host).
struct RwUnit {
  int32_t u, uend, k, nw, toff, cnt, ntile, hl, j, hpi, grp, nblk, HI;
  int32_t b, h, hk, blk;
  int4 next;  // work[k + 1], loaded ahead
  bool done, run_start;
  __device__ __forceinline__ void take(const TcArgs& a, int4 w) {
    toff = w.y;
    cnt = w.z;
    ntile = (cnt + kTileM - 1) / kTileM;
    const int32_t bh = w.x / nblk;
    blk = w.x - bh * nblk;
    b = bh / HI;
    h = (bh - b * HI) * hpi + hl;
    hk = h / grp;
    next = k + 1 < nw ? a.work[k + 1] : make_int4(0, 0, 0, 0);
  }
  __device__ __forceinline__ void start(const TcArgs& a, int64_t u0, int64_t u1, int32_t k0, int32_t nwork) {
    hpi = static_cast<int32_t>(a.HQ / a.HI);
    grp = static_cast<int32_t>(a.HQ / a.Hkv);
    nblk = static_cast<int32_t>(a.nblk);
    HI = static_cast<int32_t>(a.HI);
    u = static_cast<int32_t>(u0);
    uend = static_cast<int32_t>(u1);
    nw = nwork;
    run_start = true;
    done = u >= uend;
    if (done) return;
    k = k0;
    const int4 w = a.work[k];
    const int32_t nt = (w.z + kTileM - 1) / kTileM;
    const int32_t v = u - hpi * w.y;
    hl = v / nt;
    j = v - hl * nt;
    take(a, w);
  }
  __device__ __forceinline__ bool last_of_run() const { return j == ntile - 1 || u + 1 == uend; }
  __device__ __forceinline__ int64_t row0() const { return static_cast<int64_t>(toff + j) * kTileM; }
  __device__ __forceinline__ int rows() const {
    const int r = cnt - j * kTileM;
    return r < kTileM ? r : kTileM;
  }
  __device__ __forceinline__ void advance(const TcArgs& a) {
    ++u;
    run_start = false;
    if (u >= uend) {
      done = true;
      return;
    }
    if (++j < ntile) return;
    j = 0;
    run_start = true;
    if (++hl < hpi) {
      ++h;
      hk = h / grp;
      return;
    }
    hl = 0;
    ++k;
    take(a, next);
  }
};

// 8 fp32 * inv -> 8 bf16 as one 16-byte shared-memory store
__device__ __forceinline__ void store_o_chunk(uint32_t addr, const float* v, float inv) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e] * inv, v[2 * e + 1] * inv);
    w[e] = *reinterpret_cast<uint32_t*>(&h);
  }
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
               : "memory");
}

template <bool kPaged>
__global__ void __launch_bounds__(kRwThreads, 1)
    remote_ws_kernel(const TcArgs a, const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                     const __grid_constant__ CUtensorMap tmp) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t kv_full[2], kv_empty[2], q_full[kRwQ], q_empty[kRwQ], info_full[kRwQ], info_empty[kRwQ];
  __shared__ uint64_t stg_full[kRwQ], s_full[2], s_empty[2], p_full[2], o_full[2], o_empty[2], drain_bar;
  __shared__ int32_t r_t[kRwQ][kTileM];
  __shared__ float r_bias[kRwQ][kTileM];
  __shared__ int64_t sh_u0, sh_u1;
  __shared__ int32_t sh_k0, sh_nw;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  auto q_buf = [&](int qi) { return sbase + static_cast<uint32_t>(qi) * kQBytes; };
  auto kv_buf = [&](int st) { return sbase + kRwQ * kQBytes + static_cast<uint32_t>(st) * kWsStage; };
  const int64_t hpi = a.HQ / a.HI;
  if (warp == kRwMma) {
    tmem_alloc(&tmem_base, kWsTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kTileM);
      mbar_init(&p_full[i], kTileM);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], kTileM);
    }
    for (int i = 0; i < kRwQ; ++i) {
      mbar_init(&q_full[i], kTileM);  // one cp.async arrival per producer lane
      mbar_init(&q_empty[i], 1);      // the unit's stores have read the staged O
      mbar_init(&info_full[i], kTileM);
      mbar_init(&info_empty[i], kTileM);
      mbar_init(&stg_full[i], kTileM);
    }
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
    // this CTA's share [u0, u1) of the unit sequence
    const int32_t nw = a.totals[1];
    const int64_t U = static_cast<int64_t>(a.totals[0]) * hpi;
    const int64_t G = (U + gridDim.x - 1) / gridDim.x;
    int64_t u0 = static_cast<int64_t>(blockIdx.x) * G;
    if (u0 > U) u0 = U;
    sh_u0 = u0;
    sh_u1 = u0 + G < U ? u0 + G : U;
    sh_nw = nw;
    sh_k0 = 0;
  }
  __syncthreads();
  {  // the last list starting at or before u0 (lists are in tile order)
    const int64_t u0 = sh_u0;
    const int32_t nw = sh_nw, per = (nw + kRwThreads - 1) / kRwThreads;
    const int32_t i0 = tid * per, i1 = i0 + per < nw ? i0 + per : nw;
    int32_t best = -1;
    for (int32_t i = i0; i < i1; ++i)
      if (hpi * static_cast<int64_t>(__ldg(&a.work[i].y)) <= u0) best = i;
    if (best >= 0) atomicMax(&sh_k0, best);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  volatile int* abort_p = &abort_flag;
  const int64_t u0 = sh_u0, u1 = sh_u1;
  const int32_t k0 = sh_k0, nw = sh_nw;

  if (warp >= kRwProd && warp < kRwMma) {
    // -------------------------------------------------------------- producers
    const int pw = warp - kRwProd;  // rows 32 pw .. 32 pw + 31
    const int r = 32 * pw + lane;
    RwUnit cs;
    cs.start(a, u0, u1, k0, nw);
    int32_t pt = -1;
    int64_t pq = 0;
    float pbz = 0.f;
    auto fetch = [&]() {  // this lane's row of the unit (loaded one unit ahead)
      const int64_t row = cs.row0() + r;
      pt = -1;
      if (r < cs.rows()) {
        pt = a.pair_t[row];
        pq = a.pair_q[row];
        pbz = a.pair_bias[row];
      }
    };
    if (!cs.done) fetch();
    int qi = 0;
    uint32_t qph = 0;
    int64_t n = 0, run = 0;
    bool ok = true;
    while (ok && !cs.done) {
      if (cs.run_start) {
        if (pw == 0) {
          const int st = static_cast<int>(run & 1);
          if (run >= 2 && !__all_sync(0xffffffffu, ws_wait(&kv_empty[st], static_cast<uint32_t>(((run >> 1) - 1) & 1),
                                                           abort_p, 421))) {
            ok = false;
            break;
          }
          if (lane == 0) {  // K and V of the block: four 64 x 64 boxes
            int row0, bb;
            kv_coord<kPaged>(a, cs.b, cs.blk, row0, bb);
            const uint32_t dst = kv_buf(st);
            mbar_arrive_expect_tx(&kv_full[st], kWsStage);
            tma_load_4d(dst, &tmk, 0, row0, cs.hk, bb, &kv_full[st]);
            tma_load_4d(dst + kKVHalf, &tmk, 64, row0, cs.hk, bb, &kv_full[st]);
            tma_load_4d(dst + kKVBytes, &tmv, 0, row0, cs.hk, bb, &kv_full[st]);
            tma_load_4d(dst + kKVBytes + kKVHalf, &tmv, 64, row0, cs.hk, bb, &kv_full[st]);
          }
          __syncwarp();
        }
        ++run;
      }
      if (n >= kRwQ && !__all_sync(0xffffffffu, ws_wait(&q_empty[qi], qph ^ 1u, abort_p, 422) &&
                                                    ws_wait(&info_empty[qi], qph ^ 1u, abort_p, 423))) {
        ok = false;
        break;
      }
      r_t[qi][r] = pt;
      r_bias[qi][r] = pbz;
      mbar_arrive(&info_full[qi]);  // release: the row info above
      const unsigned long long src =
          pt >= 0 ? reinterpret_cast<unsigned long long>(a.q + pq + cs.h * a.sqh) : 0ull;
      const int cc = lane & 15;
      const uint32_t dst0 = q_buf(qi) + (cc >> 3) * (kQBytes / 2);
#pragma unroll 1
      for (int i = 0; i < 16; ++i) {
        const int rr = 2 * i + (lane >> 4);
        const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(__shfl_sync(0xffffffffu, src, rr));
        cp_async16_zfill(dst0 + sw128_off(32 * pw + rr, cc & 7), g ? static_cast<const void*>(g + cc * 8) : a.q,
                         g != nullptr);
      }
      cp_async_mbar_arrive(&q_full[qi]);
      cs.advance(a);
      if (!cs.done) fetch();  // the next unit's rows in flight while this one's copies land
      ++n;
      if (++qi == kRwQ) {
        qi = 0;
        qph ^= 1u;
      }
    }
    cp_async_wait_all();
  } else if (warp == kRwMma) {
    // --------------------------------------------------------------------- MMA
    if (lane == 0) {
      RwUnit cq;
      cq.start(a, u0, u1, k0, nw);
      int64_t nq = 0, np = 0, run = -1;  // units with S / O issued; KV run of the last S
      int qi = 0;
      uint32_t qph = 0;
      // per unit between its S and O (byte n & 1): KV stage << 2 | last of run << 3
      uint32_t pv_info = 0;
      uint64_t idle_since = 0;  // start of the current idle stretch (0: busy)
      bool ok = true;
      while (ok && (!cq.done || np < nq)) {
        bool did = false;
        if (!cq.done && nq < np + 2) {
          const int sb = static_cast<int>(nq & 1);
          const int64_t rn = cq.run_start ? run + 1 : run;
          const int st = static_cast<int>(rn & 1);
          if ((!cq.run_start || mbar_ready(&kv_full[st], static_cast<uint32_t>((rn >> 1) & 1))) &&
              mbar_ready(&q_full[qi], qph) &&
              (nq < 2 || mbar_ready(&s_empty[sb], static_cast<uint32_t>(((nq >> 1) - 1) & 1)))) {
            tc_fence_after();
            issue_qk(tmem + sb * 64, q_buf(qi), kv_buf(st));
            mma_commit(&s_full[sb]);
            run = rn;
            const uint32_t inf = static_cast<uint32_t>(st) << 2 |
                                 (cq.last_of_run() ? 8u : 0u);
            pv_info = (pv_info & ~(0xffu << (8 * sb))) | inf << (8 * sb);
            cq.advance(a);
            ++nq;
            if (++qi == kRwQ) {
              qi = 0;
              qph ^= 1u;
            }
            did = true;
          }
        }
        if (np < nq) {
          const int sb = static_cast<int>(np & 1);
          if (mbar_ready(&p_full[sb], static_cast<uint32_t>((np >> 1) & 1)) &&
              (np < 2 || mbar_ready(&o_empty[sb], static_cast<uint32_t>(((np >> 1) - 1) & 1)))) {
            const uint32_t inf = (pv_info >> (8 * sb)) & 0xffu;
            const int pst = static_cast<int>((inf >> 2) & 1u);
            tc_fence_after();
            issue_pv_tmem(tmem + 128 + sb * 128, tmem + 384 + sb * 32, kv_buf(pst) + kKVBytes, false);
            mma_commit(&o_full[sb]);
            if (inf & 8u) mma_commit(&kv_empty[pst]);
            ++np;
            did = true;
          }
        }
        if (did) {
          idle_since = 0;
        } else {  // nothing ready: back off so the other warps of this SM sub-partition can issue
          const uint64_t now = global_ns();
          if (idle_since == 0) {
            idle_since = now;
          } else if (now - idle_since > kWaitLimitNs) {
            atomicCAS(const_cast<int*>(abort_p), 0, 424);
            ok = false;
          } else if (*abort_p) {
            ok = false;
          }
          __nanosleep(40);
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------- row warpgroups 0 / 1
    const int wg = warp >> 2;
    const int r = tid & (kTileM - 1);
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tm_s = tmem + wg * 64 + lane_off, tm_o = tmem + 128 + wg * 128 + lane_off;
    const bool elected = r == 0;
    RwUnit cs;
    cs.start(a, u0, u1, k0, nw);
    if (wg == 1 && !cs.done) cs.advance(a);
    int qi = wg;            // Q ring slot of unit n = 2 m + wg
    uint32_t qph = 0;
    uint32_t m = 0;         // this warpgroup's unit count
    while (!cs.done) {
      const uint32_t ph = m & 1;
      if (!__all_sync(0xffffffffu, ws_wait(&info_full[qi], qph, abort_p, 427))) break;
      const int64_t t = r_t[qi][r];
      const float bias2 = r_bias[qi][r];
      mbar_arrive(&info_empty[qi]);
      const bool row_ok = t >= 0;
      int64_t rlo = 0, rhi = 0;
      if (row_ok) remote_range(a, cs.b, t, cs.blk, rlo, rhi);
      if (!__all_sync(0xffffffffu, ws_wait(&s_full[wg], ph, abort_p, 428))) break;
      tc_fence_after();
      float sv[64];
      {
        float s0[32], s1[32];
        tmem_ld32(tm_s, s0);
        tmem_ld32(tm_s + 32, s1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[i] = s0[i];
          sv[32 + i] = s1[i];
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[wg]);
      const int64_t k0b = static_cast<int64_t>(cs.blk) * kBlk;
      const int klo = row_ok ? clamp_key(rlo - k0b) : 0, khi = row_ok ? clamp_key(rhi - k0b) : 0;
      const bool full = __all_sync(0xffffffffu, klo == 0 && khi == kBlk);
      const float mraw = block_row_max(sv, klo, khi, full);
      const float mx = mraw == -INFINITY ? -INFINITY : fmaf(mraw, a.scale_log2, bias2);
      const float l = block_row_exp(sv, a.scale_log2, bias2 - (mx == -INFINITY ? 0.f : mx));
      // P (bf16) into this warpgroup's P columns of TMEM (its previous unit's
      // O += P V has read them: S of this unit was committed after it)
      store_p_tmem(tmem + 384 + wg * 32 + lane_off, sv);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[wg]);
      const uint32_t tile = q_buf(qi);  // Q of this unit is dead once S is in TMEM: staging for O
      if (!__all_sync(0xffffffffu, ws_wait(&o_full[wg], ph, abort_p, 429))) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        float o0[32], o1[32];
        tmem_ld32(tm_o + 64 * hf, o0);
        tmem_ld32(tm_o + 64 * hf + 32, o1);
        tmem_wait_ld();
        const uint32_t dst = tile + hf * (kQBytes / 2);
#pragma unroll
        for (int c = 0; c < 4; ++c) store_o_chunk(dst + sw128_off(r, c), o0 + 8 * c, inv);
#pragma unroll
        for (int c = 0; c < 4; ++c) store_o_chunk(dst + sw128_off(r, 4 + c), o1 + 8 * c, inv);
      }
      tc_fence_before();
      mbar_arrive(&o_empty[wg]);
      fence_async_smem();
      mbar_arrive(&stg_full[qi]);
      const int64_t row0 = cs.row0();
      if (r < cs.rows()) a.part_lse[(row0 + r) * hpi + cs.hl] = l > 0.f ? mx + log2f(l) : -INFINITY;
      if (elected) {
        if (ws_wait(&stg_full[qi], qph, abort_p, 432)) {
          tma_store_3d(&tmp, tile, 0, cs.hl, static_cast<int>(row0));
          tma_store_3d(&tmp, tile + kQBytes / 2, 64, cs.hl, static_cast<int>(row0));
          bulk_commit();
          bulk_wait_read<0>();
        }
        mbar_arrive(&q_empty[qi]);  // the tile may be refilled
      }
      __syncwarp();
      cs.advance(a);
      if (!cs.done) cs.advance(a);  // the other warpgroup's unit
      ++m;
      qi += 2;
      if (qi >= kRwQ) {
        qi -= kRwQ;
        qph ^= 1u;
      }
    }
    if (elected) bulk_wait<0>();
  }
  // ------------------------------------------------------------------- exit
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) report_status(a.status, abort_p);
  if (warp == kRwMma) {
    if (*abort_p) {  // MMAs may still be in flight: wait for all of them
      if (lane == 0) {
        mma_commit(&drain_bar);
        mbar_wait(&drain_bar, 0, 430, abort_p);
      }
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, kWsTmemCols);
  }
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

// one CTA per list: emit (t * S + first slot holding the block) in t order.
// Warp w owns a contiguous eighth of the list's words; the warps' counts are
// scanned in shared memory, then each warp emits its pairs in order.
__device__ __forceinline__ int32_t first_slot(const int32_t* srow, int64_t S, int64_t blk) {
  int32_t found = static_cast<int32_t>(S);
  if ((S & 3) == 0 && (reinterpret_cast<uintptr_t>(srow) & 15) == 0) {
    const int4* v = reinterpret_cast<const int4*>(srow);
    for (int64_t q = S / 4 - 1; q >= 0; --q) {  // backwards: the first match wins
      const int4 x = v[q];
      const int32_t b4 = static_cast<int32_t>(4 * q);
      found = x.w == blk ? b4 + 3 : found;
      found = x.z == blk ? b4 + 2 : found;
      found = x.y == blk ? b4 + 1 : found;
      found = x.x == blk ? b4 : found;
    }
  } else {
    for (int64_t q = S - 1; q >= 0; --q) found = srow[q] == blk ? static_cast<int32_t>(q) : found;
  }
  return found;
}

__global__ void __launch_bounds__(256) bwd_pairs_fill_kernel(const TcArgs a, const uint32_t* bitmap, int64_t T32,
                                                             const int32_t* offs, int32_t* pairs) {
  __shared__ int32_t wcount[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t seg = blockIdx.x;
  if (seg >= a.B * a.HI * a.nblk) return;  // CTA-uniform
  const int64_t blk = seg % a.nblk, bh = seg / a.nblk;
  const uint32_t* w = bitmap + seg * T32;
  const int64_t per = (T32 + 7) / 8;
  const int64_t wlo = warp * per, whi = min(T32, wlo + per);
  int n = 0;
  for (int64_t i = wlo + lane; i < whi; i += 32) n += __popc(w[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  if (lane == 0) wcount[warp] = n;
  __syncthreads();
  int64_t pos = offs[seg];
  for (int u = 0; u < warp; ++u) pos += wcount[u];
  for (int64_t w0 = wlo; w0 < whi; w0 += 32) {
    uint32_t word = (w0 + lane < whi) ? w[w0 + lane] : 0u;
    const int nb = __popc(word);
    int incl = nb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int64_t p = pos + incl - nb;
    while (word) {
      const int bit = __ffs(word) - 1;
      word &= word - 1;
      const int64_t t = (w0 + lane) * 32 + bit;
      pairs[p++] = static_cast<int32_t>(t * a.S + first_slot(a.sel + (bh * a.T + t) * a.S, a.S, blk));
    }
    pos += __shfl_sync(0xffffffffu, incl, 31);
  }
}

// ---- remote pairs, warp-specialised -------------------------------------
// Same work items as bwd_remote_kernel: one item = one selected block of one
// query head with all of its (query, slot) pairs, in tiles of 128.
//   warps 0-7  compute: warps w and w + 4 share TMEM lane quarter w (pair
//              rows 32w ..) and split the columns (keys 0-31 / 32-63 of S and
//              dP, features 0-63 / 64-127 of dQ): P and dS = P (dP - delta),
//              the row's d_bias partial (the high half hands its sum to the
//              low half through shared memory and an mbarrier), P and dS
//              (bf16) to shared memory, the row's dQ
//              partial, and at the end of an item this block's dK / dV
//              (thread = feature);
//   warps 8-11 producers (one per SM sub-partition; a warp's cp.async issue
//              rate bounds the gather): cp.async gathers of the tile's q and
//              dO rows into a double-buffered tile (warp 8 + i rows 32i ..
//              32i + 31), the rows' (query, slot) and softmax metadata into
//              shared memory, and (warp 8) the item's K and V by TMA;
//   warp 12    MMA issuer: S = Q K^T, dP = dO V^T; dQ = dS K; dV^T += dO^T P,
//              dK^T += Q^T dS accumulated over the item's tiles in TMEM.
//              dQ first, then the next tile's S / dP (same item) ahead of
//              this tile's dV / dK when its rows have landed.
// All waits bounded; abort protocol as in fwd_ws_kernel.
constexpr int kRbThreads = 416;
constexpr int kRbCompute = 256;  // compute threads (8 warps)
constexpr int kRbProd = 8;       // first of 4 gather warps (one per SM sub-partition)
constexpr int kRbMma = 12;
constexpr uint32_t kRbQD = 2 * kTile128;                        // q tile + dO tile
constexpr uint32_t kRbSmem = 2 * kRbQD + 2 * kKVBytes + 2 * kPBytes + 1024;  // 193 KB

struct RbCursor {  // the remote work items of the backward (same order for every role)
  int64_t item, nitems, m, j, n, ntile, pbase, cnt, b, h, hk, blk;
  bool done;
  __device__ __forceinline__ void seek(const TcBwdArgs& a) {
    const TcArgs& f = a.f;
    const int64_t hpi = f.HQ / f.HI;
    while (item < nitems) {
      const int64_t bhc = item / hpi;
      const int32_t c = a.count[bhc];
      if (c > 0) {
        cnt = c;
        pbase = a.offs[bhc];
        ntile = (c + kTileM - 1) / kTileM;
        const int64_t bh = bhc / f.nblk;
        blk = bhc % f.nblk;
        b = bh / f.HI;
        h = (bh % f.HI) * hpi + item % hpi;
        hk = h / (f.HQ / f.Hkv);
        j = 0;
        done = false;
        return;
      }
      item += gridDim.x;
    }
    done = true;
  }
  __device__ __forceinline__ void start(const TcBwdArgs& a) {
    nitems = a.f.B * a.f.HI * a.f.nblk * (a.f.HQ / a.f.HI);
    item = blockIdx.x;
    m = 0;
    n = 0;
    seek(a);
  }
  __device__ __forceinline__ bool first() const { return j == 0; }
  __device__ __forceinline__ bool last() const { return j == ntile - 1; }
  __device__ __forceinline__ int64_t tile_first() const { return pbase + j * kTileM; }
  __device__ __forceinline__ int64_t tile_rows() const {
    const int64_t r = cnt - j * kTileM;
    return r < kTileM ? r : kTileM;
  }
  __device__ __forceinline__ void advance(const TcBwdArgs& a) {
    ++n;
    if (j + 1 < ntile) {
      ++j;
      return;
    }
    ++m;
    item += gridDim.x;
    seek(a);
  }
};

__global__ void __launch_bounds__(kRbThreads, 1)
    bwd_remote_ws_kernel(const TcBwdArgs a, const __grid_constant__ CUtensorMap tmk,
                         const __grid_constant__ CUtensorMap tmv) {
  const TcArgs& f = a.f;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t kv_full, kv_empty, q_full[2], q_empty[2], info_full[2], info_empty[2];
  __shared__ uint64_t s_full, p_full, pds_empty, o_full, dq_empty, dkv_full, dkv_empty, drain_bar;
  __shared__ const __nv_bfloat16* qrows[kTileM];
  __shared__ const __nv_bfloat16* grows[kTileM];
  __shared__ int32_t r_t[2][kTileM], r_slot[2][kTileM];
  // per-row softmax metadata, fetched by the producers one tile ahead:
  // exponent offset (bias - lse, log2), delta, and the row's remote key range
  // inside the block (lo | hi << 8; empty for an absent row or lse = -inf)
  __shared__ float r_off[2][kTileM], r_dlt[2][kTileM];
  __shared__ int32_t r_kr[2][kTileM];
  __shared__ float dsum_hi[2][kTileM];  // d_bias partial of the keys 32-63 half, by tile parity
  __shared__ uint64_t dsum_full[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  auto qd_buf = [&](int bq) { return sbase + static_cast<uint32_t>(bq) * kRbQD; };  // q tile, dO tile after it
  const uint32_t k_s = sbase + 2 * kRbQD, v_s = k_s + kKVBytes;
  const uint32_t p_s = v_s + kKVBytes, ds_s = p_s + kPBytes;
  if (warp == kRbMma) {
    tmem_alloc(&tmem_base, kWsTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&kv_full, 1);
    mbar_init(&kv_empty, 1);
    for (int bq = 0; bq < 2; ++bq) {
      mbar_init(&q_full[bq], 128);
      mbar_init(&q_empty[bq], 1);
      mbar_init(&info_full[bq], 128);
      mbar_init(&info_empty[bq], kRbCompute);
    }
    mbar_init(&s_full, 1);
    mbar_init(&p_full, kRbCompute);
    mbar_init(&pds_empty, 1);
    mbar_init(&o_full, 1);
    mbar_init(&dq_empty, kRbCompute);
    mbar_init(&dkv_full, 1);
    mbar_init(&dkv_empty, kRbCompute);
    mbar_init(&dsum_full[0], kRbCompute / 2);
    mbar_init(&dsum_full[1], kRbCompute / 2);
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t tm_s = tmem, tm_dp = tmem + 64, tm_dq = tmem + 128, tm_dvt = tmem + 256, tm_dkt = tmem + 320;
  volatile int* abort_p = &abort_flag;

  if (warp >= kRbProd && warp < kRbProd + 4) {
    // ---------------------------------------------------------- producers
    // gathers are bound by the issue rate of each warp's cp.async, so four
    // warps (one per SM sub-partition) share a tile: rows 32 * quarter + lane
    const int quarter = warp - kRbProd;
    const int r = 32 * quarter + lane;
    RbCursor cs;
    cs.start(a);
    int32_t ppk = -1;
    auto fetch = [&]() {
      const int64_t fp = cs.tile_first(), nh = cs.tile_rows();
      ppk = r < nh ? a.f.pairs[fp + r] : -1;
    };
    if (!cs.done) fetch();
    bool ok = true;
    while (ok && !cs.done) {
      if (cs.first() && quarter == 0) {
        if (cs.m > 0 && !__all_sync(0xffffffffu, ws_wait(&kv_empty, static_cast<uint32_t>((cs.m - 1) & 1), abort_p, 441))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const int row0 = static_cast<int>(cs.blk * kBlk), hh = static_cast<int>(cs.hk), bb = static_cast<int>(cs.b);
          mbar_arrive_expect_tx(&kv_full, 2 * kKVBytes);
          tma_load_4d(k_s, &tmk, 0, row0, hh, bb, &kv_full);
          tma_load_4d(k_s + kKVHalf, &tmk, 64, row0, hh, bb, &kv_full);
          tma_load_4d(v_s, &tmv, 0, row0, hh, bb, &kv_full);
          tma_load_4d(v_s + kKVHalf, &tmv, 64, row0, hh, bb, &kv_full);
        }
        __syncwarp();
      }
      const int bq = static_cast<int>(cs.n & 1);
      if (cs.n >= 2) {
        const uint32_t par = static_cast<uint32_t>(((cs.n >> 1) - 1) & 1);
        if (!__all_sync(0xffffffffu, ws_wait(&q_empty[bq], par, abort_p, 442) &&
                                         ws_wait(&info_empty[bq], par, abort_p, 443))) {
          ok = false;
          break;
        }
      }
      const int32_t tt = ppk >= 0 ? ppk / static_cast<int32_t>(f.S) : -1;
      const int32_t sl = ppk >= 0 ? ppk - tt * static_cast<int32_t>(f.S) : 0;
      qrows[r] = ppk >= 0 ? f.q + cs.b * f.sqb + static_cast<int64_t>(tt) * f.sqt + cs.h * f.sqh : nullptr;
      grows[r] = ppk >= 0 ? a.dout + cs.b * f.sob + static_cast<int64_t>(tt) * f.sot + cs.h * f.soh : nullptr;
      r_t[bq][r] = tt;
      r_slot[bq][r] = sl;
      // issued now, consumed after the gathers below are in flight
      const int64_t bt = cs.b * f.T + (ppk >= 0 ? tt : 0);
      const float m_lse = ppk >= 0 ? a.lse[bt * f.HQ + cs.h] : -INFINITY;
      const float m_dlt = ppk >= 0 ? a.delta[bt * f.HQ + cs.h] : 0.f;
      const float m_bias = ppk >= 0 && f.bias ? f.bias[bt * f.S + sl] : 0.f;
      const int32_t m_seg = ppk >= 0 && f.seg ? f.seg[bt] : 0;
      __syncwarp();
      const int cc = lane & 15;
      const uint32_t qdst = qd_buf(bq) + (cc >> 3) * (kTile128 / 2);
      const uint32_t gdst = qdst + kTile128;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int rr = 32 * quarter + (lane >> 4) + 2 * i;
        const __nv_bfloat16* gq = qrows[rr];
        const __nv_bfloat16* gg = grows[rr];
        cp_async16_zfill(qdst + sw128_off(rr, cc & 7), gq ? static_cast<const void*>(gq + cc * 8) : f.q, gq != nullptr);
        cp_async16_zfill(gdst + sw128_off(rr, cc & 7), gg ? static_cast<const void*>(gg + cc * 8) : f.q, gg != nullptr);
      }
      cp_async_mbar_arrive(&q_full[bq]);
      int32_t kr = 0;
      if (tt >= 0 && m_lse != -INFINITY) {
        const int64_t sg = m_seg;
        int64_t ls = tt - f.LW + 1;
        if (ls < sg) ls = sg;
        if (ls < 0) ls = 0;
        const int64_t k0 = cs.blk * kBlk;
        const int64_t lo = (k0 > sg ? k0 : sg) - k0;
        const int64_t hi = min(min(k0 + kBlk, ls), static_cast<int64_t>(tt) + 1) - k0;
        kr = clamp_key(lo) | (clamp_key(hi) << 8);
      }
      r_off[bq][r] = (m_bias - m_lse) * kLog2e;
      r_dlt[bq][r] = m_dlt;
      r_kr[bq][r] = kr;
      mbar_arrive(&info_full[bq]);
      __syncwarp();
      cs.advance(a);
      if (!cs.done) fetch();
    }
    cp_async_wait_all();
  } else if (warp == kRbMma) {
    // -------------------------------------------------------------------- MMA
    if (lane == 0) {
      RbCursor cs;
      cs.start(a);
      bool ok = !cs.done;
      // S / dP of the cursor's current tile
      auto issue_sdp = [&]() -> bool {
        const int bq = static_cast<int>(cs.n & 1);
        if (cs.first() && !ws_wait(&kv_full, static_cast<uint32_t>(cs.m & 1), abort_p, 444)) return false;
        if (!ws_wait(&q_full[bq], static_cast<uint32_t>((cs.n >> 1) & 1), abort_p, 445)) return false;
        tc_fence_after();
        issue_qk(tm_s, qd_buf(bq), k_s);
        issue_qk(tm_dp, qd_buf(bq) + kTile128, v_s);
        mma_commit(&s_full);
        return true;
      };
      // operands of the cursor's tile already landed (no wait)
      auto sdp_ready = [&]() -> bool {
        const int bq = static_cast<int>(cs.n & 1);
        if (cs.first() && !mbar_ready(&kv_full, static_cast<uint32_t>(cs.m & 1))) return false;
        return mbar_ready(&q_full[bq], static_cast<uint32_t>((cs.n >> 1) & 1));
      };
      // Issuing a tcgen05.mma blocks while the tensor pipe is busy, so the
      // issue order is the execution order: dQ of this tile first (the
      // compute warps wait for it), then the next tile's S / dP if its rows
      // are already in shared memory, else this tile's dV / dK first (which
      // frees its Q / dO buffer for the next gather).
      if (ok) ok = issue_sdp();
      while (ok && !cs.done) {
        const int64_t n = cs.n, m = cs.m;
        const int bq = static_cast<int>(n & 1);
        const bool first = cs.first(), last = cs.last();
        if (!ws_wait(&p_full, static_cast<uint32_t>(n & 1), abort_p, 446)) break;
        if (n > 0 && !ws_wait(&dq_empty, static_cast<uint32_t>((n - 1) & 1), abort_p, 447)) break;
        tc_fence_after();
        issue_pv(tm_dq, ds_s, k_s, false);  // dQ = dS K
        mma_commit(&o_full);
        cs.advance(a);  // cs now names the next tile
        const bool early = !cs.done && cs.m == m && sdp_ready();
        if (early && !(ok = issue_sdp())) break;
        if (first && m > 0 && !ws_wait(&dkv_empty, static_cast<uint32_t>((m - 1) & 1), abort_p, 448)) break;
        tc_fence_after();
        issue_tn(tm_dvt, qd_buf(bq) + kTile128, kTile128 / 2, p_s, !first);  // dV^T += dO^T P
        issue_tn(tm_dkt, qd_buf(bq), kTile128 / 2, ds_s, !first);            // dK^T += Q^T dS
        mma_commit(&pds_empty);
        mma_commit(&q_empty[bq]);
        if (last) {
          mma_commit(&dkv_full);
          mma_commit(&kv_empty);
        }
        if (!cs.done && !early && !(ok = issue_sdp())) break;
      }
    }
    __syncwarp();
  } else if (warp < 8) {
    // ---------------------------------------------------------------- compute
    const int q4 = warp & 3, ch = warp >> 2;  // lane quarter, column half
    const int r = 32 * q4 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    RbCursor cs;
    cs.start(a);
    while (!cs.done) {
      const int64_t n = cs.n;
      const int bq = static_cast<int>(n & 1);
      if (!__all_sync(0xffffffffu, ws_wait(&info_full[bq], static_cast<uint32_t>((n >> 1) & 1), abort_p, 449))) break;
      const int64_t t = r_t[bq][r], slot = r_slot[bq][r];
      const float off = r_off[bq][r], dlt = r_dlt[bq][r];
      const int32_t kr = r_kr[bq][r];
      mbar_arrive(&info_empty[bq]);
      const bool row_ok = t >= 0;
      const int klo = max((kr & 0xff) - 32 * ch, 0), khi = max((kr >> 8) - 32 * ch, 0);
      if (!__all_sync(0xffffffffu, ws_wait(&s_full, static_cast<uint32_t>(n & 1), abort_p, 450))) break;
      tc_fence_after();
      float sv[32], dp[32];
      tmem_ld32(tm_s + lane_off + 32 * ch, sv);
      tmem_ld32(tm_dp + lane_off + 32 * ch, dp);
      tmem_wait_ld();
      float ds4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const bool valid = i >= klo && i < khi;
        const float pv = valid ? fast_exp2(fmaf(sv[i], f.scale_log2, off)) : 0.f;
        const float ds = pv * (dp[i] - dlt);
        sv[i] = pv;
        dp[i] = ds;
        ds4[i & 3] += ds;
      }
      const float dsum = (ds4[0] + ds4[1]) + (ds4[2] + ds4[3]);
      // P and dS of the previous tile are read by its dV / dK MMAs: wait for them
      if (n > 0 && !__all_sync(0xffffffffu, ws_wait(&pds_empty, static_cast<uint32_t>((n - 1) & 1), abort_p, 451)))
        break;
      store_p_row(p_s, r, 4 * ch, sv);
      store_p_row(ds_s, r, 4 * ch, dp);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full);
      if (ch == 1) {
        dsum_hi[bq][r] = dsum;
        mbar_arrive(&dsum_full[bq]);  // release: the sum above
      } else {
        if (!__all_sync(0xffffffffu, ws_wait(&dsum_full[bq], static_cast<uint32_t>((n >> 1) & 1), abort_p, 455))) break;
        if (row_ok && a.dbias_part)
          a.dbias_part[((cs.b * f.T + t) * f.S + slot) * f.HQ + cs.h] = dsum + dsum_hi[bq][r];
      }
      if (!__all_sync(0xffffffffu, ws_wait(&o_full, static_cast<uint32_t>(n & 1), abort_p, 452))) break;
      tc_fence_after();
      const int64_t prow = ((cs.b * f.T + (row_ok ? t : 0)) * f.S + slot) * f.HQ + cs.h;
      {
        float ov0[32], ov1[32];
        tmem_ld32(tm_dq + lane_off + 64 * ch, ov0);
        tmem_ld32(tm_dq + lane_off + 64 * ch + 32, ov1);
        tmem_wait_ld();
        if (row_ok) {  // this half row (128 bytes, 32-byte aligned) as four 32-byte stores
          __nv_bfloat16* dst = a.dq_part + prow * kD + 64 * ch;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            st_global_bf16x16(dst + 16 * q, ov0 + 16 * q, a.scale);
            st_global_bf16x16(dst + 32 + 16 * q, ov1 + 16 * q, a.scale);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&dq_empty);
      if (cs.last()) {  // this block's remote dK / dV for the item's head: thread = feature, keys of half ch
        if (!__all_sync(0xffffffffu, ws_wait(&dkv_full, static_cast<uint32_t>(cs.m & 1), abort_p, 453))) break;
        tc_fence_after();
        float* dst = a.dkv_part + ((cs.b * f.HQ + cs.h) * f.nblk + cs.blk) * (2 * 64 * 128);
        float kv[32], vv[32];
        tmem_ld32(tm_dkt + lane_off + 32 * ch, kv);
        tmem_ld32(tm_dvt + lane_off + 32 * ch, vv);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          dst[(32 * ch + i) * 128 + r] = kv[i] * a.scale;
          dst[8192 + (32 * ch + i) * 128 + r] = vv[i];
        }
        tc_fence_before();
        mbar_arrive(&dkv_empty);
      }
      cs.advance(a);
    }
  }
  // ------------------------------------------------------------------- exit
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) report_status(a.f.status, abort_p);
  if (warp == kRbMma) {
    if (*abort_p) {
      if (lane == 0) {
        mma_commit(&drain_bar);
        mbar_wait(&drain_bar, 0, 454, abort_p);
      }
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, kWsTmemCols);
  }
}

// ---- band dQ, warp-specialised: one work item = (b, h, 128-query tile) -----
//   warps 0-3  compute (thread = query row): P = 2^(s c - lse), dS = P (dP -
//              delta) over the window keys, dS (bf16) over the stage's dead V;
//              after the item's last block, dQ (window part) from TMEM;
//   warp 4     producer: TMA of the tile's q and dO (per item) and of each
//              window block's K and V into a 3-stage ring;
//   warp 5     MMA issuer: S = Q K^T and dP = dO V^T into one of two TMEM
//              buffers (the next block's run while the compute warps work
//              on this one), dQ += dS K.
// The remote dQ partials are added by dq_merge_kernel.
constexpr int kBqThreads = 192;
constexpr int kBqStages = 3;
constexpr uint32_t kBqSmem = 2 * kTile128 + kBqStages * 2 * kKVBytes + 1024;  // 161 KB

__global__ void __launch_bounds__(kBqThreads, 1)
    bwd_band_dq_ws_kernel(const TcBwdArgs a, const __grid_constant__ CUtensorMap tmq,
                          const __grid_constant__ CUtensorMap tmdo, const __grid_constant__ CUtensorMap tmk,
                          const __grid_constant__ CUtensorMap tmv) {
  const TcArgs& f = a.f;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // p_full per S / dP buffer: the MMA issues the next block's S / dP before it
  // waits for this block's dS, so one barrier could be completed twice ahead
  __shared__ uint64_t q_full, q_empty, kv_full[kBqStages], kv_empty[kBqStages], s_full[2], p_full[2], o_full, dq_empty;
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t q_s = sbase, do_s = sbase + kTile128;
  auto k_s = [&](int st) { return sbase + 2 * kTile128 + static_cast<uint32_t>(st) * 2 * kKVBytes; };
  if (warp == 5) {
    tmem_alloc(&tmem_base, kWsTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int st = 0; st < kBqStages; ++st) {
      mbar_init(&kv_full[st], 1);
      mbar_init(&kv_empty[st], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], kTileM);
    mbar_init(&p_full[1], kTileM);
    mbar_init(&o_full, 1);
    mbar_init(&dq_empty, kTileM);
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t tm_dq = tmem + 256;
  volatile int* abort_p = &abort_flag;
  const int64_t nitems = f.B * f.HQ * ((f.T + kTileM - 1) / kTileM);
  // the CTA's items are blockIdx.x + k * gridDim.x, blocks blo..bhi of each
  struct Cur {
    int64_t item, m, n, j;
    WsItem w;
    bool done;
  };
  auto cur_start = [&](Cur& c) {
    c.item = blockIdx.x;
    c.m = 0;
    c.n = 0;
    c.done = c.item >= nitems;
    if (!c.done) {
      c.w = ws_item(f, c.item);
      c.j = c.w.blo;
    }
  };
  auto cur_advance = [&](Cur& c) {
    ++c.n;
    if (c.j < c.w.bhi) {
      ++c.j;
      return;
    }
    ++c.m;
    c.item += gridDim.x;
    c.done = c.item >= nitems;
    if (!c.done) {
      c.w = ws_item(f, c.item);
      c.j = c.w.blo;
    }
  };

  if (warp == 4) {
    // -------------------------------------------------------------- producer
    Cur c;
    cur_start(c);
    bool ok = true;
    while (ok && !c.done) {
      if (c.j == c.w.blo) {
        if (c.m > 0 && !__all_sync(0xffffffffu, ws_wait(&q_empty, static_cast<uint32_t>((c.m - 1) & 1), abort_p, 461))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const int t0 = static_cast<int>(c.w.t0), hh = static_cast<int>(c.w.h), bb = static_cast<int>(c.w.b);
          mbar_arrive_expect_tx(&q_full, 2 * kTile128);
          tma_load_4d(q_s, &tmq, 0, t0, hh, bb, &q_full);
          tma_load_4d(q_s + kTile128 / 2, &tmq, 64, t0, hh, bb, &q_full);
          tma_load_4d(do_s, &tmdo, 0, t0, hh, bb, &q_full);
          tma_load_4d(do_s + kTile128 / 2, &tmdo, 64, t0, hh, bb, &q_full);
        }
        __syncwarp();
      }
      const int st = static_cast<int>(c.n % kBqStages);
      if (c.n >= kBqStages &&
          !__all_sync(0xffffffffu, ws_wait(&kv_empty[st], static_cast<uint32_t>((c.n / kBqStages - 1) & 1), abort_p, 462))) {
        ok = false;
        break;
      }
      if (lane == 0) {
        const int row0 = static_cast<int>(c.j * kBlk), hh = static_cast<int>(c.w.hk), bb = static_cast<int>(c.w.b);
        const uint32_t dst = k_s(st);
        mbar_arrive_expect_tx(&kv_full[st], 2 * kKVBytes);
        tma_load_4d(dst, &tmk, 0, row0, hh, bb, &kv_full[st]);
        tma_load_4d(dst + kKVHalf, &tmk, 64, row0, hh, bb, &kv_full[st]);
        tma_load_4d(dst + kKVBytes, &tmv, 0, row0, hh, bb, &kv_full[st]);
        tma_load_4d(dst + kKVBytes + kKVHalf, &tmv, 64, row0, hh, bb, &kv_full[st]);
      }
      __syncwarp();
      cur_advance(c);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------- MMA
    if (lane == 0) {
      Cur c;
      cur_start(c);
      auto issue_sdp = [&](const Cur& x) -> bool {
        const int st = static_cast<int>(x.n % kBqStages), sb = static_cast<int>(x.n & 1);
        if (x.j == x.w.blo && !ws_wait(&q_full, static_cast<uint32_t>(x.m & 1), abort_p, 463)) return false;
        if (!ws_wait(&kv_full[st], static_cast<uint32_t>((x.n / kBqStages) & 1), abort_p, 464)) return false;
        tc_fence_after();
        issue_qk(tmem + 64 * sb, q_s, k_s(st));
        issue_qk(tmem + 128 + 64 * sb, do_s, k_s(st) + kKVBytes);
        mma_commit(&s_full[sb]);
        if (x.j == x.w.bhi) mma_commit(&q_empty);  // the item's q / dO are read by S / dP only
        return true;
      };
      bool ok = !c.done && issue_sdp(c);
      while (ok && !c.done) {
        Cur nx = c;
        cur_advance(nx);
        if (!nx.done && !(ok = issue_sdp(nx))) break;  // next block's S / dP overlap this block's dS
        if (!ws_wait(&p_full[c.n & 1], static_cast<uint32_t>((c.n >> 1) & 1), abort_p, 465)) break;
        const bool first = c.j == c.w.blo, last = c.j == c.w.bhi;
        if (first && c.m > 0 && !ws_wait(&dq_empty, static_cast<uint32_t>((c.m - 1) & 1), abort_p, 466)) break;
        const int st = static_cast<int>(c.n % kBqStages);
        tc_fence_after();
        issue_pv(tm_dq, k_s(st) + kKVBytes, k_s(st), !first);  // dQ += dS K, dS over the dead V
        mma_commit(&kv_empty[st]);
        if (last) mma_commit(&o_full);
        c = nx;
      }
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- compute
    const int r = tid;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    Cur c;
    cur_start(c);
    int64_t t = 0, ls = 0;
    bool row_ok = false;
    float lse2 = 0.f, dlt = 0.f;
    while (!c.done) {
      const bool first = c.j == c.w.blo, last = c.j == c.w.bhi;
      if (first) {
        t = c.w.t0 + r;
        row_ok = t < f.T;
        ls = row_ok ? win_start(f, c.w.b, t) : 0;
        lse2 = row_ok ? a.lse[(c.w.b * f.T + t) * f.HQ + c.w.h] * kLog2e : 0.f;
        dlt = row_ok ? a.delta[(c.w.b * f.T + t) * f.HQ + c.w.h] : 0.f;
      }
      const int sb = static_cast<int>(c.n & 1);
      if (!__all_sync(0xffffffffu, ws_wait(&s_full[sb], static_cast<uint32_t>((c.n >> 1) & 1), abort_p, 467))) break;
      tc_fence_after();
      float sv[64], dp[64];
      {
        float x0[32], x1[32];
        tmem_ld32(tmem + 64 * sb + lane_off, x0);
        tmem_ld32(tmem + 64 * sb + lane_off + 32, x1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { sv[i] = x0[i]; sv[32 + i] = x1[i]; }
        tmem_ld32(tmem + 128 + 64 * sb + lane_off, x0);
        tmem_ld32(tmem + 128 + 64 * sb + lane_off + 32, x1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { dp[i] = x0[i]; dp[32 + i] = x1[i]; }
      }
      const int64_t k0 = c.j * kBlk;
      const int klo = row_ok ? clamp_key(ls - k0) : 0, khi = row_ok ? clamp_key(t + 1 - k0) : 0;
      const bool okl = lse2 != -INFINITY;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const bool valid = okl && i >= klo && i < khi;
        const float pv = valid ? fast_exp2(fmaf(sv[i], f.scale_log2, -lse2)) : 0.f;
        dp[i] = pv * (dp[i] - dlt);
      }
      const uint32_t ds_s = k_s(static_cast<int>(c.n % kBqStages)) + kKVBytes;  // over the dead V
      store_p_row(ds_s, r, 0, dp);
      store_p_row(ds_s, r, 4, dp + 32);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
      if (last) {
        if (!__all_sync(0xffffffffu, ws_wait(&o_full, static_cast<uint32_t>(c.m & 1), abort_p, 468))) break;
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float ov[32];
          tmem_ld32(tm_dq + lane_off + 32 * cc, ov);
          tmem_wait_ld();
          if (row_ok) store_row32(a.dq + c.w.b * f.sqb + t * f.sqt + c.w.h * f.sqh + 32 * cc, ov, a.scale);
        }
        tc_fence_before();
        mbar_arrive(&dq_empty);
      }
      cur_advance(c);
    }
  }
  // ------------------------------------------------------------------- exit
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) report_status(a.f.status, abort_p);
  if (warp == 5) {
    if (*abort_p) {
      if (lane == 0) {
        mma_commit(&drain_bar);
        mbar_wait(&drain_bar, 0, 469, abort_p);
      }
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, kWsTmemCols);
  }
}

// dq[b,t,h] += sum of the row's remote dQ partials (usable first-occurrence
// slots, as in the pair lists); one warp per (b, t, h), lane = 4 features.
// Slot validity is recomputed from the selection row with warp shuffles; all
// partial loads of the row are issued together.
// Adds the remote dQ partials ([B, T, S, HQ, D] bf16) to the band dQ.  One
// CTA per (b, t) and up to 16 heads (blockIdx.y), thread = (head, 8
// features); each warp first finds the usable slots of its two heads' index
// heads (lane = slot: a valid block with remote keys for the query and not a
// repeat of an earlier slot).  A slot's partials of all heads are contiguous,
// so every load is a coalesced 16-byte word.  Memory-bound.
constexpr int kDqHeads = 16;
__global__ void __launch_bounds__(kDqHeads * 16) dq_merge_kernel(const TcBwdArgs a) {
  const TcArgs& f = a.f;
  const int lane = threadIdx.x & 31, f8 = threadIdx.x & 15;
  const int64_t bt = blockIdx.x, t = bt % f.T, b = bt / f.T;
  const int64_t h = static_cast<int64_t>(blockIdx.y) * kDqHeads + (threadIdx.x >> 4);
  const int64_t hpi = f.HQ / f.HI;
  const int ns = static_cast<int>(f.S < 64 ? f.S : 64);
  // usable-slot masks of one index head (warp-collective)
  auto slot_masks = [&](int64_t hi, uint32_t& m0, uint32_t& m1) {
    const int32_t* srow = f.sel + ((b * f.HI + hi) * f.T + t) * f.S;
    const int32_t blk0 = lane < ns ? srow[lane] : -1, blk1 = lane + 32 < ns ? srow[lane + 32] : -1;
    auto usable = [&](int32_t blk) {
      if (blk < 0 || blk >= f.nblk) return false;
      int64_t lo, hi2;
      remote_range(f, b, t, blk, lo, hi2);
      return lo < hi2;
    };
    bool ok0 = usable(blk0), ok1 = usable(blk1);
    for (int u = 0; u < 32; ++u) {  // drop repeats of an earlier slot
      const int32_t o0 = __shfl_sync(0xffffffffu, blk0, u);
      if (u < lane && o0 == blk0) ok0 = false;
      if (o0 == blk1) ok1 = false;
      const int32_t o1 = __shfl_sync(0xffffffffu, blk1, u);
      if (u < lane && o1 == blk1) ok1 = false;
    }
    m0 = __ballot_sync(0xffffffffu, ok0);
    m1 = __ballot_sync(0xffffffffu, ok1);
  };
  // the warp's two heads (a head past HQ borrows the last one's index head)
  const int64_t h_lo = static_cast<int64_t>(blockIdx.y) * kDqHeads + ((threadIdx.x & ~31u) >> 4);
  const int64_t hi_lo = (h_lo < f.HQ ? h_lo : f.HQ - 1) / hpi;
  const int64_t hi_hi = (h_lo + 1 < f.HQ ? h_lo + 1 : f.HQ - 1) / hpi;
  uint32_t m0, m1;
  slot_masks(hi_lo, m0, m1);
  if (hi_hi != hi_lo) {
    uint32_t n0, n1;
    slot_masks(hi_hi, n0, n1);
    if (lane >= 16) {
      m0 = n0;
      m1 = n1;
    }
  }
  if (h >= f.HQ || (m0 | m1) == 0) return;
  uint4* dqp = reinterpret_cast<uint4*>(a.dq + b * f.sqb + t * f.sqt + h * f.sqh) + f8;
  const uint4 d0 = *dqp;
  float acc[8];
  {
    const uint32_t wv[4] = {d0.x, d0.y, d0.z, d0.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[2 * e] = bf16_lo(wv[e]);
      acc[2 * e + 1] = bf16_hi(wv[e]);
    }
  }
  const uint4* part = reinterpret_cast<const uint4*>(a.dq_part + (bt * f.S * f.HQ + h) * kD) + f8;
  for (int g0 = 0; g0 < ns; g0 += 8) {
    uint4 u8[8];
#pragma unroll
    for (int k8 = 0; k8 < 8; ++k8) {
      const int s2 = g0 + k8;
      const bool use = s2 < ns && (((s2 < 32 ? m0 : m1) >> (s2 & 31)) & 1u);
      u8[k8] = use ? __ldcs(part + static_cast<int64_t>(s2) * f.HQ * (kD / 8)) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int k8 = 0; k8 < 8; ++k8) {
      const uint32_t wv[4] = {u8[k8].x, u8[k8].y, u8[k8].z, u8[k8].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] += bf16_lo(wv[e]);
        acc[2 * e + 1] += bf16_hi(wv[e]);
      }
    }
  }
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 hv = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t*>(&hv);
  }
  *dqp = make_uint4(w[0], w[1], w[2], w[3]);
}

// ---- band dK / dV, warp-specialised: one work item = (b, kv head, 128-key
// tile); steps = (query head of the group) x (64-query chunk of the window)
//   warps 0-3  compute (thread = key row): P^T = 2^(s c - lse_q), dS^T =
//              P^T (dP^T - delta_q) over the pairs with ls_q <= key <= q,
//              P^T / dS^T (bf16 pairs) written back into the first 32
//              columns of the step's S^T / dP^T buffer in TMEM; after the
//              item's last step, dK (scaled) and dV from TMEM;
//   warp 4     producer: TMA of the item's K / V tile and of each chunk's q /
//              dO rows (4 stages), plus the chunk's per-query lse, delta and
//              window bounds in shared memory and a whole-chunk-valid flag;
//   warp 5     MMA issuer: S^T = K Q^T and dP^T = V dO^T into one of two TMEM
//              buffers (the next step's run while the compute warps work;
//              a buffer is reused once the MMAs that read its P^T / dS^T are
//              complete), dV += P^T dO and dK += dS^T Q accumulated over the
//              item, A read from TMEM.
// The remote dK / dV partials are added by dkv_merge_kernel.
constexpr int kBkThreads = 192;
constexpr uint32_t kQc = 64 * 128 * 2;                                       // 64 rows x 128 bf16
constexpr int kBkStages = 4;                                                 // q / dO chunk ring
constexpr uint32_t kBkSmem = 2 * kTile128 + kBkStages * 2 * kQc + 1024;      // 193 KB

__global__ void __launch_bounds__(kBkThreads, 1)
    bwd_band_dkdv_ws_kernel(const TcBwdArgs a, const __grid_constant__ CUtensorMap tmq64,
                            const __grid_constant__ CUtensorMap tmdo64, const __grid_constant__ CUtensorMap tmk,
                            const __grid_constant__ CUtensorMap tmv) {
  const TcArgs& f = a.f;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t kv_full, kv_empty, qd_full[kBkStages], qd_empty[kBkStages], s_full[2], p_full[2], pds_empty[2];
  __shared__ uint64_t dkv_full, dkv_empty, drain_bar;
  __shared__ __align__(16) int32_t v_lo[kBkStages][64], v_hi[kBkStages][64];
  __shared__ __align__(16) float v_lse[kBkStages][64], v_dl[kBkStages][64];
  __shared__ int v_full[kBkStages];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t k_s = sbase, v_s = sbase + kTile128;
  auto qd_s = [&](int st) { return sbase + 2 * kTile128 + static_cast<uint32_t>(st) * 2 * kQc; };  // q, then dO
  if (warp == 5) {
    tmem_alloc(&tmem_base, kWsTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&kv_full, 1);
    mbar_init(&kv_empty, 1);
    for (int i = 0; i < kBkStages; ++i) {
      mbar_init(&qd_full[i], 32);
      mbar_init(&qd_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], kTileM);
      mbar_init(&pds_empty[i], 1);
    }
    mbar_init(&dkv_full, 1);
    mbar_init(&dkv_empty, kTileM);
    mbar_init(&drain_bar, 1);
    fence_mbar_init();
    abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const uint32_t tm_dk = tmem + 256, tm_dv = tmem + 384;
  volatile int* abort_p = &abort_flag;
  const int64_t G = f.HQ / f.Hkv;
  const int64_t ntk = (f.T + kTileM - 1) / kTileM;
  const int64_t nitems = f.B * f.Hkv * ntk;
  struct Cur {
    int64_t item, m, n, b, hk, k0, g, c, nch;
    bool done;
  };
  auto load_item = [&](Cur& x) {
    x.done = x.item >= nitems;
    if (x.done) return;
    const int64_t tile = x.item % ntk, bh = x.item / ntk;
    x.b = bh / f.Hkv;
    x.hk = bh % f.Hkv;
    x.k0 = tile * kTileM;
    const int64_t q_end = min(f.T, x.k0 + kTileM - 1 + f.LW);
    x.nch = (q_end - x.k0 + 63) / 64;
    x.g = 0;
    x.c = 0;
  };
  auto cur_start = [&](Cur& x) {
    x.item = blockIdx.x;
    x.m = 0;
    x.n = 0;
    load_item(x);
  };
  auto is_first = [&](const Cur& x) { return x.g == 0 && x.c == 0; };
  auto is_last = [&](const Cur& x) { return x.g == G - 1 && x.c == x.nch - 1; };
  auto cur_advance = [&](Cur& x) {
    ++x.n;
    if (++x.c < x.nch) return;
    x.c = 0;
    if (++x.g < G) return;
    ++x.m;
    x.item += gridDim.x;
    load_item(x);
  };

  if (warp == 4) {
    // -------------------------------------------------------------- producer
    Cur c;
    cur_start(c);
    bool ok = true;
    while (ok && !c.done) {
      const int bb = static_cast<int>(c.b);
      if (is_first(c)) {
        if (c.m > 0 && !__all_sync(0xffffffffu, ws_wait(&kv_empty, static_cast<uint32_t>((c.m - 1) & 1), abort_p, 481))) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const int k0 = static_cast<int>(c.k0), hh = static_cast<int>(c.hk);
          mbar_arrive_expect_tx(&kv_full, 2 * kTile128);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
            for (int rb = 0; rb < 2; ++rb) {
              const uint32_t off = hf * (kTile128 / 2) + rb * kKVHalf;
              tma_load_4d(k_s + off, &tmk, 64 * hf, k0 + 64 * rb, hh, bb, &kv_full);
              tma_load_4d(v_s + off, &tmv, 64 * hf, k0 + 64 * rb, hh, bb, &kv_full);
            }
          }
        }
        __syncwarp();
      }
      const int st = static_cast<int>(c.n % kBkStages);
      if (c.n >= kBkStages &&
          !__all_sync(0xffffffffu, ws_wait(&qd_empty[st], static_cast<uint32_t>(((c.n / kBkStages) - 1) & 1), abort_p,
                                           482))) {
        ok = false;
        break;
      }
      const int64_t h = c.hk * G + c.g, q0 = c.k0 + 64 * c.c;
      bool all_ok = true;
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int i = lane + 32 * k2;
        const int64_t q = q0 + i;
        int32_t lo = 0x7fffffff, hi = -1;
        float l2 = 0.f, dl = 0.f;
        if (q < f.T) {
          lo = static_cast<int32_t>(win_start(f, c.b, q));
          hi = static_cast<int32_t>(q);
          l2 = a.lse[(c.b * f.T + q) * f.HQ + h] * kLog2e;
          dl = a.delta[(c.b * f.T + q) * f.HQ + h];
        }
        v_lo[st][i] = lo;
        v_hi[st][i] = hi;
        v_lse[st][i] = l2;
        v_dl[st][i] = dl;
        all_ok = all_ok && q < f.T && lo <= c.k0 && hi >= c.k0 + kTileM - 1 && c.k0 + kTileM <= f.T &&
                 l2 != -INFINITY;
      }
      const bool full = __all_sync(0xffffffffu, all_ok);
      if (lane == 0) v_full[st] = full ? 1 : 0;
      __syncwarp();
      if (lane == 0) {
        const int hh = static_cast<int>(h), qq = static_cast<int>(q0);
        mbar_arrive_expect_tx(&qd_full[st], 2 * kQc);
        tma_load_4d(qd_s(st), &tmq64, 0, qq, hh, bb, &qd_full[st]);
        tma_load_4d(qd_s(st) + kKVHalf, &tmq64, 64, qq, hh, bb, &qd_full[st]);
        tma_load_4d(qd_s(st) + kQc, &tmdo64, 0, qq, hh, bb, &qd_full[st]);
        tma_load_4d(qd_s(st) + kQc + kKVHalf, &tmdo64, 64, qq, hh, bb, &qd_full[st]);
      } else {
        mbar_arrive(&qd_full[st]);  // release: this lane's vectors above
      }
      cur_advance(c);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------- MMA
    if (lane == 0) {
      Cur c;
      cur_start(c);
      auto issue_sdp = [&](const Cur& x) -> bool {
        const int sb = static_cast<int>(x.n & 1), qs = static_cast<int>(x.n % kBkStages);
        if (is_first(x) && !ws_wait(&kv_full, static_cast<uint32_t>(x.m & 1), abort_p, 483)) return false;
        if (!ws_wait(&qd_full[qs], static_cast<uint32_t>((x.n / kBkStages) & 1), abort_p, 484)) return false;
        // the buffer's P^T / dS^T of step n - 2 have been read by their MMAs
        if (x.n >= 2 && !ws_wait(&pds_empty[sb], static_cast<uint32_t>(((x.n >> 1) - 1) & 1), abort_p, 489))
          return false;
        tc_fence_after();
        issue_qk(tmem + 64 * sb, k_s, qd_s(qs));               // S^T = K Q^T
        issue_qk(tmem + 128 + 64 * sb, v_s, qd_s(qs) + kQc);   // dP^T = V dO^T
        mma_commit(&s_full[sb]);
        if (is_last(x)) mma_commit(&kv_empty);  // K / V are read by S^T / dP^T only
        return true;
      };
      bool ok = !c.done && issue_sdp(c);
      while (ok && !c.done) {
        Cur nx = c;
        cur_advance(nx);
        if (!nx.done && !(ok = issue_sdp(nx))) break;
        const int sb = static_cast<int>(c.n & 1), qs = static_cast<int>(c.n % kBkStages);
        if (!ws_wait(&p_full[sb], static_cast<uint32_t>((c.n >> 1) & 1), abort_p, 485)) break;
        const bool first = is_first(c), last = is_last(c);
        if (first && c.m > 0 && !ws_wait(&dkv_empty, static_cast<uint32_t>((c.m - 1) & 1), abort_p, 486)) break;
        tc_fence_after();
        issue_pv_tmem(tm_dv, tmem + 64 * sb, qd_s(qs) + kQc, !first);        // dV += P^T dO
        issue_pv_tmem(tm_dk, tmem + 128 + 64 * sb, qd_s(qs), !first);        // dK += dS^T Q
        mma_commit(&pds_empty[sb]);
        mma_commit(&qd_empty[qs]);
        if (last) mma_commit(&dkv_full);
        c = nx;
      }
    }
    __syncwarp();
  } else {
    // --------------------------------------------------------------- compute
    const int r = tid;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    Cur c;
    cur_start(c);
    while (!c.done) {
      const int sb = static_cast<int>(c.n & 1), st = static_cast<int>(c.n % kBkStages);
      const int64_t key = c.k0 + r;
      const bool key_ok = key < f.T;
      if (!__all_sync(0xffffffffu, ws_wait(&qd_full[st], static_cast<uint32_t>((c.n / kBkStages) & 1), abort_p, 487) &&
                                       ws_wait(&s_full[sb], static_cast<uint32_t>((c.n >> 1) & 1), abort_p, 488)))
        break;
      tc_fence_after();
      float sv[64], dp[64];
      {
        float x0[32], x1[32];
        tmem_ld32(tmem + 64 * sb + lane_off, x0);
        tmem_ld32(tmem + 64 * sb + lane_off + 32, x1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { sv[i] = x0[i]; sv[32 + i] = x1[i]; }
        tmem_ld32(tmem + 128 + 64 * sb + lane_off, x0);
        tmem_ld32(tmem + 128 + 64 * sb + lane_off + 32, x1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) { dp[i] = x0[i]; dp[32 + i] = x1[i]; }
      }
      const int32_t k32 = static_cast<int32_t>(key);
      if (v_full[st]) {  // every (key, query) pair of the step is local
#pragma unroll
        for (int i4 = 0; i4 < 16; ++i4) {
          const float4 l4 = *reinterpret_cast<const float4*>(&v_lse[st][4 * i4]);
          const float4 d4 = *reinterpret_cast<const float4*>(&v_dl[st][4 * i4]);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 4 * i4 + e;
            const float pv = fast_exp2(fmaf(sv[i], f.scale_log2, -lv[e]));
            sv[i] = pv;
            dp[i] = pv * (dp[i] - dv4[e]);
          }
        }
      } else {
#pragma unroll
        for (int i4 = 0; i4 < 16; ++i4) {
          const float4 l4 = *reinterpret_cast<const float4*>(&v_lse[st][4 * i4]);
          const float4 d4 = *reinterpret_cast<const float4*>(&v_dl[st][4 * i4]);
          const int4 lo4 = *reinterpret_cast<const int4*>(&v_lo[st][4 * i4]);
          const int4 hi4 = *reinterpret_cast<const int4*>(&v_hi[st][4 * i4]);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dv4[4] = {d4.x, d4.y, d4.z, d4.w};
          const int32_t lo[4] = {lo4.x, lo4.y, lo4.z, lo4.w}, hi[4] = {hi4.x, hi4.y, hi4.z, hi4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 4 * i4 + e;
            const bool valid = key_ok && k32 >= lo[e] && k32 <= hi[e] && lv[e] != -INFINITY;
            const float pv = valid ? fast_exp2(fmaf(sv[i], f.scale_log2, -lv[e])) : 0.f;
            sv[i] = pv;
            dp[i] = pv * (dp[i] - dv4[e]);
          }
        }
      }
      // P^T and dS^T over the first 32 columns of the buffers just read
      store_p_tmem(tmem + 64 * sb + lane_off, sv);
      store_p_tmem(tmem + 128 + 64 * sb + lane_off, dp);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
      if (is_last(c)) {
        if (!__all_sync(0xffffffffu, ws_wait(&dkv_full, static_cast<uint32_t>(c.m & 1), abort_p, 490))) break;
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          float kv[32], vv[32];
          tmem_ld32(tm_dk + lane_off + 32 * cc, kv);
          tmem_ld32(tm_dv + lane_off + 32 * cc, vv);
          tmem_wait_ld();
          if (key_ok) {
            store_row32(a.dk + c.b * f.skb + key * f.skt + c.hk * f.skh + 32 * cc, kv, a.scale);
            store_row32(a.dv + c.b * f.svb + key * f.svt + c.hk * f.svh + 32 * cc, vv, 1.f);
          }
        }
        tc_fence_before();
        mbar_arrive(&dkv_empty);
      }
      cur_advance(c);
    }
  }
  // ------------------------------------------------------------------- exit
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) report_status(a.f.status, abort_p);
  if (warp == 5) {
    if (*abort_p) {
      if (lane == 0) {
        mma_commit(&drain_bar);
        mbar_wait(&drain_bar, 0, 491, abort_p);
      }
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem, kWsTmemCols);
  }
}

// dk / dv += the remote partials of the key's block over the kv group's query
// heads (blocks some query selected); thread = (b, key, kv head, 8 features),
// 16 consecutive threads cover one 256-byte row.
__global__ void __launch_bounds__(256) dkv_merge_kernel(const TcBwdArgs a) {
  const TcArgs& f = a.f;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (idx >= f.B * f.T * f.Hkv * 16) return;
  const int64_t ch = idx & 15, rest = idx >> 4;
  const int64_t hk = rest % f.Hkv, bt = rest / f.Hkv, key = bt % f.T, b = bt / f.T;
  const int64_t blk = key / kBlk, G = f.HQ / f.Hkv, hi = (hk * f.HI) / f.Hkv;
  if (a.count[(b * f.HI + hi) * f.nblk + blk] == 0) return;
  __nv_bfloat16* dkp = a.dk + b * f.skb + key * f.skt + hk * f.skh + ch * 8;
  __nv_bfloat16* dvp = a.dv + b * f.svb + key * f.svt + hk * f.svh + ch * 8;
  float kacc[8], vacc[8];
  load8(dkp, 0, SRSWA_BF16, kacc);
  load8(dvp, 0, SRSWA_BF16, vacc);
  for (int64_t g = 0; g < G; ++g) {
    const float* src =
        a.dkv_part + ((b * f.HQ + hk * G + g) * f.nblk + blk) * (2 * 64 * 128) + (key % kBlk) * 128 + ch * 8;
    const float4 k0 = __ldcs(reinterpret_cast<const float4*>(src));
    const float4 k1 = __ldcs(reinterpret_cast<const float4*>(src + 4));
    const float4 v0 = __ldcs(reinterpret_cast<const float4*>(src + 8192));
    const float4 v1 = __ldcs(reinterpret_cast<const float4*>(src + 8196));
    kacc[0] += k0.x; kacc[1] += k0.y; kacc[2] += k0.z; kacc[3] += k0.w;
    kacc[4] += k1.x; kacc[5] += k1.y; kacc[6] += k1.z; kacc[7] += k1.w;
    vacc[0] += v0.x; vacc[1] += v0.y; vacc[2] += v0.z; vacc[3] += v0.w;
    vacc[4] += v1.x; vacc[5] += v1.y; vacc[6] += v1.z; vacc[7] += v1.w;
  }
  store8(dkp, 0, SRSWA_BF16, kacc);
  store8(dvp, 0, SRSWA_BF16, vacc);
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

static size_t al256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

TcLayout tc_layout(const srswa_gather_desc* g, int64_t qoff) {
  TcLayout L;
  const int64_t nblk = (g->T + qoff + kBlk - 1) / kBlk;
  const int64_t nbh = g->B * g->HI * nblk;
  const int64_t nsel = g->B * g->HI * g->T * g->S;
  const int64_t hpi = g->HI > 0 ? g->HQ / g->HI : 1;
  // every nonempty list rounds its pairs up to whole tiles
  L.max_tiles = nsel / kTileM + nbh + 1;
  const size_t cap = static_cast<size_t>(L.max_tiles) * kTileM;
  size_t off = 0;
  L.part_o = off;
  off += al256(static_cast<size_t>(hpi) * cap * kD * 2);
  L.part_lse = off;
  off += al256(static_cast<size_t>(hpi) * cap * 4);
  L.count = off;
  off += al256(static_cast<size_t>(nbh) * 4);
  L.cursor = off;
  off += al256(static_cast<size_t>(nbh) * 4);
  L.work = off;
  off += al256(static_cast<size_t>(nbh) * 16);
  L.totals = off;
  off += 256;
  L.pair_t = off;
  off += al256(cap * 4);
  L.pair_q = off;
  off += al256(cap * 8);
  L.pair_bias = off;
  off += al256(cap * 4);
  L.prow = off;
  off += al256(static_cast<size_t>(nsel) * 4);
  L.lse = off;  // the window lse when the caller asks for none (the merge reads it)
  off += al256(static_cast<size_t>(g->B * g->T * g->HQ) * 4);
  L.total = off;
  return L;
}

// cuTensorMapEncodeTiled, looked up through the runtime (no libcuda link)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn tmap_encoder() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}
// Tensor map of a [B, T, H, 128] bf16 tensor with element strides (sb, st, sh):
// dims (D, T, H, B), box of 64 features x box_rows rows, 128-byte swizzle,
// out-of-range rows read as zeros.  False when the driver refuses it.
static bool make_tmap(CUtensorMap* m, const void* base, int64_t B, int64_t T, int64_t H, int64_t sb, int64_t st,
                      int64_t sh, uint32_t box_rows) {
  EncodeTiledFn enc = tmap_encoder();
  if (!enc) return false;
  auto stride_of = [](int64_t extent, int64_t s_el) -> cuuint64_t {
    // the coordinate of a size-1 dimension is always 0: any legal stride will do
    return extent == 1 ? static_cast<cuuint64_t>(256) : static_cast<cuuint64_t>(s_el) * 2;
  };
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {stride_of(T, st), stride_of(H, sh), stride_of(B, sb)};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of the partial rows [cap, hpi, 128] bf16: box of 64 features x
// one head x 128 rows, 128-byte swizzle (the stores of the remote pass).
static bool make_tmap_rows(CUtensorMap* m, void* base, int64_t cap, int64_t hpi) {
  EncodeTiledFn enc = tmap_encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(hpi), static_cast<cuuint64_t>(cap)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD) * 2, static_cast<cuuint64_t>(hpi) * kD * 2};
  cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kTileM)};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The list kernels keep two counters per key block in shared memory (up to
// 227 KB), and their grid has one row per (b, index head).
constexpr int64_t kMaxListBlocks = 227 * 1024 / 8;

bool tc_eligible(const srswa_gather_desc* g) {
  return g->D == kD && g->block_size == kBlk && g->dtype == SRSWA_BF16 && g->S <= 64 && g->T > 0 && g->scale > 0.f &&
         (g->T + kBlk - 1) / kBlk <= kMaxListBlocks && g->B * g->HI <= 65535 &&
         ((g->sqb | g->sqt | g->sqh | g->skb | g->skt | g->skh | g->svb | g->svt | g->svh) & 7) == 0;
}

// The paged forward: one sequence whose rows follow a prefix of qoff tokens.
bool tc_paged_eligible(const srswa_gather_desc* g, int64_t qoff) {
  return tc_eligible(g) && g->B == 1 && qoff >= 0 && (g->T + qoff + kBlk - 1) / kBlk <= kMaxListBlocks &&
         g->T + qoff < (1ll << 31);
}

// Launch properties per device: the SM count, and whether the kernels'
// shared-memory limits have been raised there (a per-context setting).  The
// only process-wide state of the tensor-core path; filled under a mutex on
// the first call made on each device.
struct TcDeviceProps {
  int num_sms = 0;
  bool fwd_ready = false, bwd_ready = false;
};
constexpr int kTcMaxDevices = 64;
static TcDeviceProps g_tc_props[kTcMaxDevices];
static std::mutex g_tc_props_mu;

static int tc_device_props(bool bwd, int* num_sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kTcMaxDevices) return SRSWA_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_tc_props_mu);
  TcDeviceProps& p = g_tc_props[dev];
  if (p.num_sms == 0) {
    e = cudaDeviceGetAttribute(&p.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  if (!bwd && !p.fwd_ready) {
    e = cudaFuncSetAttribute(remote_ws_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRwSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(remote_ws_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRwSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fwd_ws_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWsSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fwd_ws_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kWsSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    p.fwd_ready = true;
  }
  if (bwd && !p.bwd_ready) {
    e = cudaFuncSetAttribute(bwd_remote_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRbSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(bwd_band_dq_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBqSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(bwd_band_dkdv_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBkSmem);
    if (e != cudaSuccess) return static_cast<int>(e);
    p.bwd_ready = true;
  }
  *num_sms = p.num_sms;
  return 0;
}

int tc_gather_fwd(const srswa_gather_desc* g, const void* q, const void* k, const void* v, const int32_t* sel,
                  const float* bias, const int32_t* seg, void* o, int64_t sob, int64_t sot, int64_t soh, float* lse,
                  void* workspace, size_t workspace_bytes, int* status, cudaStream_t st, const TcPagedKV* pk) {
  const int64_t qoff = pk ? pk->qoff : 0;
  const TcLayout L = tc_layout(g, qoff);
  if (!workspace || workspace_bytes < L.total) return SRSWA_EWORKSPACE;
  char* ws = static_cast<char*>(workspace);
  TcArgs a = {};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.sqb = g->sqb; a.sqt = g->sqt; a.sqh = g->sqh; a.skb = g->skb; a.skt = g->skt; a.skh = g->skh;
  a.svb = g->svb; a.svt = g->svt; a.svh = g->svh;
  a.o = static_cast<__nv_bfloat16*>(o); a.sob = sob; a.sot = sot; a.soh = soh;
  a.lse = lse ? lse : reinterpret_cast<float*>(ws + L.lse);
  a.sel = sel; a.bias = bias; a.seg = seg;
  const int64_t hpi = g->HQ / g->HI;
  a.part_o = reinterpret_cast<__nv_bfloat16*>(ws + L.part_o);
  a.part_lse = reinterpret_cast<float*>(ws + L.part_lse);
  a.prow = reinterpret_cast<int32_t*>(ws + L.prow);
  a.pair_t = reinterpret_cast<int32_t*>(ws + L.pair_t);
  a.pair_q = reinterpret_cast<int64_t*>(ws + L.pair_q);
  a.pair_bias = reinterpret_cast<float*>(ws + L.pair_bias);
  a.work = reinterpret_cast<int4*>(ws + L.work);
  a.totals = reinterpret_cast<int32_t*>(ws + L.totals);
  a.status = status;
  a.prow_cap = L.max_tiles * kTileM;
  a.B = g->B; a.T = g->T; a.HQ = g->HQ; a.Hkv = g->Hkv; a.HI = g->HI; a.S = g->S;
  a.LW = g->local_window > 0 ? g->local_window : kBlk;
  a.nblk = (g->T + qoff + kBlk - 1) / kBlk;
  a.scale_log2 = g->scale * kLog2e;
  if (pk) {
    a.kv_pages = pk->pages;
    a.s_pages = pk->s_pages;
    a.qoff = qoff;
    a.tail_blk = (qoff + g->T - 1) / kBlk;
    a.tail_slots = (qoff + g->T) % kBlk;
  }
  int32_t* count = reinterpret_cast<int32_t*>(ws + L.count);
  int32_t* cursor = reinterpret_cast<int32_t*>(ws + L.cursor);
  // partial rows and selections are indexed with 32-bit integers
  if (a.prow_cap >= (1ll << 31) || L.max_tiles * hpi >= (1ll << 31) || g->B * g->HI * g->T * g->S >= (1ll << 31))
    return SRSWA_ETOOLARGE;

  int num_sms = 0;
  if (const int prc = tc_device_props(false, &num_sms)) return prc;
  // the tensor maps of q, k, v and the partial rows; when the driver refuses
  // one, the caller runs the CUDA-core kernels instead (nothing launched yet)
  alignas(64) CUtensorMap tmq, tmk, tmv, tmp, tmk_tail, tmv_tail;
  // paged caches: [pages, 64 slots, Hkv, D]; the tail maps end the slot
  // extent at the sequence's last token (its partial last page)
  const int64_t kv_b = pk ? pk->num_pages : g->B, kv_t = pk ? kBlk : g->T;
  if (!(make_tmap(&tmq, q, g->B, g->T, g->HQ, g->sqb, g->sqt, g->sqh, kTileM) &&
        make_tmap(&tmk, k, kv_b, kv_t, g->Hkv, g->skb, g->skt, g->skh, kBlk) &&
        make_tmap(&tmv, v, kv_b, kv_t, g->Hkv, g->svb, g->svt, g->svh, kBlk) &&
        make_tmap_rows(&tmp, a.part_o, a.prow_cap, hpi)))
    return kTcNoTensorMap;
  tmk_tail = tmk;
  tmv_tail = tmv;
  if (pk && a.tail_slots > 0 &&
      !(make_tmap(&tmk_tail, k, kv_b, a.tail_slots, g->Hkv, g->skb, g->skt, g->skh, kBlk) &&
        make_tmap(&tmv_tail, v, kv_b, a.tail_slots, g->Hkv, g->svb, g->svt, g->svh, kBlk)))
    return kTcNoTensorMap;
  if (g->S > 0) {
    const int64_t nbh = a.B * a.HI * a.nblk;
    SRSWA_CUDA_TRY(cudaMemsetAsync(count, 0, static_cast<size_t>(nbh) * 4, st));
    const dim3 lgrid(static_cast<unsigned>((a.T + kListRows - 1) / kListRows), static_cast<unsigned>(nbh / a.nblk));
    if (a.nblk * 8 > 48 * 1024) {  // above the default dynamic shared-memory limit
      SRSWA_CUDA_TRY(cudaFuncSetAttribute(pairs_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(a.nblk * 4)));
      SRSWA_CUDA_TRY(cudaFuncSetAttribute(pairs_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(a.nblk * 8)));
    }
    pairs_count_kernel<<<lgrid, kListRows, static_cast<size_t>(a.nblk) * 4, st>>>(a, count);
    SRSWA_CUDA_TRY(cudaGetLastError());
    fwd_lists_scan_kernel<<<1, 1024, 0, st>>>(a, count, cursor, const_cast<int4*>(a.work),
                                              const_cast<int32_t*>(a.totals));
    SRSWA_CUDA_TRY(cudaGetLastError());
    pairs_fill_kernel<<<lgrid, kListRows, static_cast<size_t>(a.nblk) * 8, st>>>(a, cursor);
    SRSWA_CUDA_TRY(cudaGetLastError());
    if (pk)
      remote_ws_kernel<true><<<num_sms, kRwThreads, kRwSmem, st>>>(a, tmk, tmv, tmp);
    else
      remote_ws_kernel<false><<<num_sms, kRwThreads, kRwSmem, st>>>(a, tmk, tmv, tmp);
    SRSWA_CUDA_TRY(cudaGetLastError());
  } else {
    a.part_o = nullptr;
  }
  const int64_t band_items = g->B * g->HQ * ((g->T + kTileM - 1) / kTileM);
  const unsigned band_grid = static_cast<unsigned>(band_items < num_sms ? band_items : num_sms);
  if (pk)
    fwd_ws_kernel<true><<<band_grid, kWsThreads, kWsSmem, st>>>(a, tmq, tmk, tmv, tmk_tail, tmv_tail);
  else
    fwd_ws_kernel<false><<<band_grid, kWsThreads, kWsSmem, st>>>(a, tmq, tmk, tmv, tmk_tail, tmv_tail);
  if (a.part_o) {
    SRSWA_CUDA_TRY(cudaGetLastError());
    const int64_t hpc = g->HQ < kMgHeads ? g->HQ : kMgHeads;
    const dim3 grid(static_cast<unsigned>(g->B * g->T), static_cast<unsigned>((g->HQ + kMgHeads - 1) / kMgHeads));
    merge_partials_kernel<<<grid, static_cast<unsigned>(hpc * 16), 0, st>>>(a);
  }
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
                  void* workspace, size_t workspace_bytes, int* status, cudaStream_t st) {
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
  f.status = status;
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

  int num_sms = 0;
  if (const int prc = tc_device_props(true, &num_sms)) return prc;
  // tensor maps of k, v, q and dO; when the driver refuses one, the caller
  // runs the CUDA-core kernels instead (nothing has been launched yet)
  alignas(64) CUtensorMap tmk, tmv, tmq, tmdo, tmq64, tmdo64;
  if (!(make_tmap(&tmk, k, g->B, g->T, g->Hkv, g->skb, g->skt, g->skh, kBlk) &&
        make_tmap(&tmv, v, g->B, g->T, g->Hkv, g->svb, g->svt, g->svh, kBlk) &&
        make_tmap(&tmq, q, g->B, g->T, g->HQ, g->sqb, g->sqt, g->sqh, kTileM) &&
        make_tmap(&tmdo, dout, g->B, g->T, g->HQ, sob, sot, soh, kTileM) &&
        make_tmap(&tmq64, q, g->B, g->T, g->HQ, g->sqb, g->sqt, g->sqh, 64) &&
        make_tmap(&tmdo64, dout, g->B, g->T, g->HQ, sob, sot, soh, 64)))
    return kTcNoTensorMap;
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
    bwd_pairs_fill_kernel<<<static_cast<unsigned>(nbh), 256, 0, st>>>(f, bitmap, L.T32, offs,
                                                                              const_cast<int32_t*>(f.pairs));
    SRSWA_CUDA_TRY(cudaGetLastError());
    if (a.dbias_part)
      SRSWA_CUDA_TRY(cudaMemsetAsync(a.dbias_part, 0, static_cast<size_t>(g->B * g->T * g->S * g->HQ) * 4, st));
    bwd_remote_ws_kernel<<<num_sms, kRbThreads, kRbSmem, st>>>(a, tmk, tmv);
    SRSWA_CUDA_TRY(cudaGetLastError());
  }
  const unsigned ntile = static_cast<unsigned>((g->T + kTileM - 1) / kTileM);
  {
    const int64_t items = g->B * g->Hkv * static_cast<int64_t>(ntile);
    const unsigned grid_k = static_cast<unsigned>(items < num_sms ? items : num_sms);
    bwd_band_dkdv_ws_kernel<<<grid_k, kBkThreads, kBkSmem, st>>>(a, tmq64, tmdo64, tmk, tmv);
    SRSWA_CUDA_TRY(cudaGetLastError());
    if (remote) {
      const int64_t n16 = g->B * g->T * g->Hkv * 16;
      dkv_merge_kernel<<<static_cast<unsigned>((n16 + 255) / 256), 256, 0, st>>>(a);
      SRSWA_CUDA_TRY(cudaGetLastError());
    }
  }
  {
    const int64_t items = g->B * g->HQ * static_cast<int64_t>(ntile);
    const unsigned grid_q = static_cast<unsigned>(items < num_sms ? items : num_sms);
    bwd_band_dq_ws_kernel<<<grid_q, kBqThreads, kBqSmem, st>>>(a, tmq, tmdo, tmk, tmv);
    SRSWA_CUDA_TRY(cudaGetLastError());
    if (remote) {
      const int64_t hpc = g->HQ < kDqHeads ? g->HQ : kDqHeads;
      const dim3 grid(static_cast<unsigned>(g->B * g->T), static_cast<unsigned>((g->HQ + kDqHeads - 1) / kDqHeads));
      dq_merge_kernel<<<grid, static_cast<unsigned>((hpc * 16 + 31) / 32 * 32), 0, st>>>(a);
      SRSWA_CUDA_TRY(cudaGetLastError());
    }
  }
  if (bias) {
    if (remote) {
      const int64_t n = g->B * g->T * g->S;
      tc_dbias_reduce_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(a);
    }
  }
  return srswa_last_launch_status();
}
}  // namespace srswa
