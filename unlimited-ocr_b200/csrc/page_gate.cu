// PageGate: page-aware remote candidates of the SR-SWA router.
//
// Token ids -> per-token page ids (image pages, query pages) -> per-query
// "same-page image block" candidate masks for the prefill router, and the
// decode-side allow mask of one new token per request.  Integer work, bound
// by HBM (the [B, Lq, nblk] mask write) or by launch latency.
//
// Reference: hf-model-code/_sparse_base_impl.py:2392-2402 (image block allow),
// :2404-2497 (_build_page_aware_ids), :2609-2627 (flat image mask),
// :2629-2648 (_build_page_aware_image_block_mask), :2697-2730
// (_build_kl_candidate_mask); hf-model-code/modeling_unlimitedocr.py:482-528
// (_uocr_dash_decode_allow).
//
// Row scans (page ids, decode state) run in two launches over 2048-token
// chunks: page_count_kernel reduces each chunk (markers, image tokens, last
// image token, markers up to it), page_scan_kernel combines the counts of the
// chunks before its own and scans its chunk, so every SM works on one row.
// Candidate masks test each key block against the query's page through a
// 16-byte block descriptor {min page, max page, 64-bit page set}: image page
// ids only rise along a row and a 64-token block spans at most 64 of them, so
// the set is exact; a block whose pages span more (only possible with page
// ids a caller built otherwise) is flagged and scanned token by token.
#include "common.cuh"

namespace srswa {

constexpr int kPgThreads = 256;
constexpr int kPgPer = 8;                         // consecutive tokens per thread
constexpr int kPgChunk = kPgThreads * kPgPer;     // tokens per CTA
constexpr uint8_t kCodeImg = 1, kCodeMark = 2;

struct PgRow {
  const int64_t* ids;
  int64_t s_row, n_ids, n_tok;  // ids columns available, tokens scanned (pad: -1)
  int64_t img_id, page_id, per_page;
};

// Chunk of one row: token codes into shared memory with coalesced loads.
__device__ __forceinline__ void load_codes(const PgRow& r, int64_t b, int64_t c0, uint8_t* codes) {
  const int64_t lim = min(r.n_ids, r.n_tok);
  const int64_t* row = r.ids + b * r.s_row;
#pragma unroll
  for (int k = 0; k < kPgPer; ++k) {
    const int i = k * kPgThreads + threadIdx.x;
    const int64_t j = c0 + i;
    const int64_t t = j < lim ? __ldg(row + j) : -1;
    codes[i] = static_cast<uint8_t>((t == r.img_id ? kCodeImg : 0) | (t == r.page_id ? kCodeMark : 0));
  }
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5;
  __syncthreads();  // red reused across calls
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  T x = red[0];
#pragma unroll
  for (int i = 1; i < kPgThreads / 32; ++i) x = op(x, red[i]);
  return x;
}
struct OpAdd { template <typename T> __device__ T operator()(T a, T b) const { return a + b; } };
struct OpMax { template <typename T> __device__ T operator()(T a, T b) const { return a > b ? a : b; } };

// Per chunk {markers, image tokens, chunk-local index of the last image token
// (-1: none), markers at or before it}.
__global__ void __launch_bounds__(kPgThreads) page_count_kernel(const PgRow r, int64_t nchunk, int4* stats) {
  __shared__ uint8_t codes[kPgChunk];
  __shared__ int red[kPgThreads / 32];
  const int64_t b = blockIdx.y, c0 = static_cast<int64_t>(blockIdx.x) * kPgChunk;
  load_codes(r, b, c0, codes);
  __syncthreads();
  const int base = threadIdx.x * kPgPer;
  int nm = 0, ni = 0, last = -1;
#pragma unroll
  for (int k = 0; k < kPgPer; ++k) {
    const uint8_t c = codes[base + k];
    nm += (c & kCodeMark) ? 1 : 0;
    if (c & kCodeImg) {
      ++ni;
      last = base + k;
    }
  }
  nm = block_reduce(nm, OpAdd(), red);
  ni = block_reduce(ni, OpAdd(), red);
  last = block_reduce(last, OpMax(), red);
  int upto = 0;
#pragma unroll
  for (int k = 0; k < kPgPer; ++k) upto += (base + k <= last && (codes[base + k] & kCodeMark)) ? 1 : 0;
  upto = block_reduce(upto, OpAdd(), red);
  if (threadIdx.x == 0) stats[b * nchunk + blockIdx.x] = make_int4(nm, ni, last, upto);
}

struct PgOut {
  // mode 0: page-aware ids
  uint8_t* itm;
  int64_t* ipi;
  int64_t* qpi;
  int32_t* flags;  // [0]: an image token seen, [1]: a query page >= 0 seen
  int scope;       // page_scope_prefill
  // mode 1: decode-allow prefill state
  int64_t *bmin, *bmax, *pp, *mcum;
  int64_t bs, nblk;
  // modes 2 / 3: page2d RoPE coordinates
  int64_t* mpos;      // [B, s_mpos]: position of the k-th <PAGE> marker of the row (k >= 1)
  int64_t s_mpos;
  int64_t *tok, *page;  // [B, n_tok]
  int64_t* pf;        // [B, pf_cap]: prefill tokens of each page
  int64_t pf_cap;
  int64_t span;       // > 0: page prefill spans mapped onto `span` token steps
  int32_t* rflags;    // [0] image token seen, [1] marker seen, [2] rows without prompt pages, [3] page count
};

// Prefill tokens of page p of a row with pp prompt pages (pp >= 1): the BOS
// prefix before the first marker (p = 0), the run from marker p to the next
// one (or to the last image token) for p <= pp, none above.
__device__ __forceinline__ int64_t prefill_count(const int64_t* mp, int64_t p, int64_t pp, int64_t last_img) {
  if (p > pp) return 0;
  if (p == 0) return mp[1];
  return (p < pp ? mp[p + 1] : last_img + 1) - mp[p];
}

// Exclusive block scan of two counts packed in one 64-bit word (low: markers,
// high: image tokens; each < 2^32 per chunk).
__device__ __forceinline__ uint64_t block_excl_scan(uint64_t v, uint64_t* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) red[w] = x;
  __syncthreads();
  uint64_t off = 0;
  for (int i = 0; i < w; ++i) off += red[i];
  return off + x - v;
}

// Scan one chunk of a row with the counts of every chunk before it.
//   MODE 0: itm / ipi / qpi of _build_page_aware_ids (marker mode per row).
//   MODE 1: per-block [min, max] image page, pp and the marker count of
//           _uocr_dash_decode_allow's prefill (image page: cum > 0 ? cum - 1 :
//           (run - 1) / per_page per token).
template <int MODE>
__global__ void __launch_bounds__(kPgThreads) page_scan_kernel(const PgRow r, int64_t nchunk, const int4* stats,
                                                             const PgOut o) {
  __shared__ uint8_t codes[kPgChunk];
  // MODE 0: image pages (buf[0]) and query pages (buf[1]) of the chunk's
  // tokens; MODE 1: min / max image page per block of the chunk (as int)
  __shared__ __align__(16) int64_t buf[2][kPgChunk];
  __shared__ int64_t red64[kPgThreads / 32];
  __shared__ uint64_t redu[kPgThreads / 32];
  int* bmn = reinterpret_cast<int*>(buf[0]);
  int* bmx = bmn + kPgChunk;
  const int64_t b = blockIdx.y, chunk = blockIdx.x, c0 = chunk * kPgChunk;
  const int4* st = stats + b * nchunk;
  load_codes(r, b, c0, codes);
  // ---- row-level combination of the chunk counts
  int64_t mb = 0, ib = 0, mall = 0, lastc = -1;
  for (int64_t c = threadIdx.x; c < nchunk; c += kPgThreads) {
    const int4 s = __ldg(st + c);
    mall += s.x;
    if (c < chunk) {
      mb += s.x;
      ib += s.y;
    }
    if (s.z >= 0) lastc = c;
  }
  mb = block_reduce(mb, OpAdd(), red64);
  ib = block_reduce(ib, OpAdd(), red64);
  mall = block_reduce(mall, OpAdd(), red64);
  lastc = block_reduce(lastc, OpMax(), red64);
  int64_t pp = 0, last_img = -1;
  if (lastc >= 0) {
    int64_t m = 0;
    for (int64_t c = threadIdx.x; c < lastc; c += kPgThreads) m += __ldg(st + c).x;
    m = block_reduce(m, OpAdd(), red64);
    const int4 s = __ldg(st + lastc);
    pp = m + s.w;
    last_img = lastc * kPgChunk + s.z;
  }
  const bool marker = pp > 0;
  // ---- chunk scan
  const int base = threadIdx.x * kPgPer;
  uint64_t cnt = 0;
  uint8_t cd[kPgPer];
#pragma unroll
  for (int k = 0; k < kPgPer; ++k) {
    cd[k] = codes[base + k];
    cnt += ((cd[k] & kCodeMark) ? 1ull : 0ull) + ((cd[k] & kCodeImg) ? (1ull << 32) : 0ull);
  }
  const uint64_t ex = block_excl_scan(cnt, redu);
  int64_t cum = mb + static_cast<int64_t>(ex & 0xffffffffu);
  int64_t run = ib + static_cast<int64_t>(ex >> 32);
  if (MODE == 1) {
    for (int i = threadIdx.x; i < kPgChunk; i += kPgThreads) {
      bmn[i] = 0x7fffffff;
      bmx[i] = -1;
    }
    __syncthreads();
  }
  bool any_q = false;
#pragma unroll
  for (int k = 0; k < kPgPer; ++k) {
    const int64_t j = c0 + base + k;
    const bool img = cd[k] & kCodeImg;
    cum += (cd[k] & kCodeMark) ? 1 : 0;
    run += img ? 1 : 0;
    if (MODE == 0) {
      const int64_t ip = img ? (marker ? cum - 1 : (run - 1) / r.per_page) : -1;
      const int64_t raw = cum - 1;
      int64_t q = j <= last_img ? (o.scope ? raw : -1) : raw - (marker ? pp : 0);
      q = q < 0 ? -1 : q;
      any_q |= (q >= 0 && j < r.n_tok);
      buf[0][base + k] = ip;
      buf[1][base + k] = q;
    } else if (MODE == 1) {
      if (img) {
        const int64_t pg = cum > 0 ? cum - 1 : (run - 1) / r.per_page;
        const int blk = static_cast<int>((base + k) / o.bs);
        atomicMin(&bmn[blk], static_cast<int>(pg));
        atomicMax(&bmx[blk], static_cast<int>(pg));
      }
    } else if (MODE == 2) {
      if ((cd[k] & kCodeMark) && j < r.n_tok) o.mpos[b * o.s_mpos + cum] = j;
    } else if (pp > 0) {  // MODE 3 (rows without prompt pages make the call return None)
      const int64_t* mp = o.mpos + b * o.s_mpos;
      const bool pre = j <= last_img;
      const int64_t pg = pre ? cum : cum - pp;
      int64_t rs = cum >= 1 ? mp[cum] : 0;  // the run of a page starts at its marker
      if (!pre && rs <= last_img) rs = last_img + 1;
      const int64_t pf = prefill_count(mp, pg, pp, last_img);
      int64_t t = pre ? j - rs : pf + (j - rs);
      if (o.span > 0 && pg > 0) {
        const float sp = static_cast<float>(o.span);
        const float v = pre ? rintf(static_cast<float>(t) * sp / static_cast<float>(pf > 1 ? pf : 1))
                            : sp + static_cast<float>(t - pf);
        t = static_cast<int64_t>(v);
      }
      buf[0][base + k] = t;
      buf[1][base + k] = pg;
    } else {
      buf[0][base + k] = 0;
      buf[1][base + k] = 0;
    }
  }
  __syncthreads();
  const int64_t nvalid = min(static_cast<int64_t>(kPgChunk), r.n_tok - c0);
  if (MODE == 0) {
    const int64_t rowo = b * r.n_tok + c0;
    for (int i = threadIdx.x; i < nvalid; i += kPgThreads) {
      o.itm[rowo + i] = codes[i] & kCodeImg;
      o.ipi[rowo + i] = buf[0][i];
      o.qpi[rowo + i] = buf[1][i];
    }
    const int any_img = __syncthreads_or(ib + static_cast<int64_t>(ex >> 32) < run);
    const int anyq = __syncthreads_or(any_q);
    if (threadIdx.x == 0) {
      if (any_img) atomicOr(&o.flags[0], 1);
      if (anyq) atomicOr(&o.flags[1], 1);
    }
  } else if (MODE == 2) {
    if (chunk == 0 && threadIdx.x == 0) {
      if (lastc >= 0) atomicOr(&o.rflags[0], 1);
      if (mall > 0) atomicOr(&o.rflags[1], 1);
      if (pp == 0) atomicAdd(&o.rflags[2], 1);
      const int64_t top = (pp > mall - pp ? pp : mall - pp) + 1;
      atomicMax(&o.rflags[3], static_cast<int>(top));
    }
  } else if (MODE == 3) {
    const int64_t rowo = b * r.n_tok + c0;
    for (int i = threadIdx.x; i < nvalid; i += kPgThreads) {
      o.tok[rowo + i] = buf[0][i];
      o.page[rowo + i] = buf[1][i];
    }
    // this chunk's share of the per-page prefill counts (the last chunk also
    // covers the rest of the capacity)
    const int64_t p1 = chunk == nchunk - 1 ? o.pf_cap : min(o.pf_cap, c0 + kPgChunk);
    const int64_t* mp = o.mpos + b * o.s_mpos;
    for (int64_t pg = c0 + threadIdx.x; pg < p1; pg += kPgThreads)
      o.pf[b * o.pf_cap + pg] = pp > 0 ? prefill_count(mp, pg, pp, last_img) : 0;
  } else {
    const int nb = static_cast<int>((nvalid + o.bs - 1) / o.bs);
    const int64_t blk0 = c0 / o.bs;
    for (int i = threadIdx.x; i < nb; i += kPgThreads) {
      const int mx = bmx[i];
      o.bmax[b * o.nblk + blk0 + i] = mx;
      o.bmin[b * o.nblk + blk0 + i] = mx >= 0 ? bmn[i] : -1;
    }
    if (chunk == 0 && threadIdx.x == 0) {
      o.pp[b] = pp;
      o.mcum[b] = mall;
    }
  }
}

// ---------------------------------------------------------------------------
// Block descriptors {min page (-1: no image token), max page, page set lo,
// page set hi}; the set holds bit (p - min) for every page p of the block when
// max - min < 64, else it is empty (a wide block, scanned by the mask kernel).
// Flat mode (image-token mask given instead of page ids): {0, 0, 1, 0} for a
// block with an image token, {-1, -1, 0, 0} else.  One warp per block.
__global__ void __launch_bounds__(256) page_block_desc_kernel(const int64_t* ipi, const uint8_t* itm, int64_t s_row,
                                                              int64_t n_tok, int64_t bs, int64_t nblk, int64_t B,
                                                              int4* desc) {
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= B * nblk) return;
  const int64_t b = wid / nblk, c = wid - b * nblk;
  const int64_t j0 = c * bs, j1 = min(j0 + bs, n_tok);
  if (itm) {
    bool any = false;
    for (int64_t j = j0 + lane; j < j1; j += 32) any |= itm[b * s_row + j] != 0;
    any = __any_sync(0xffffffffu, any);
    if (lane == 0) desc[wid] = any ? make_int4(0, 0, 1, 0) : make_int4(-1, -1, 0, 0);
    return;
  }
  int64_t mn = INT64_MAX, mx = -1;
  for (int64_t j = j0 + lane; j < j1; j += 32) {
    const int64_t p = __ldg(ipi + b * s_row + j);
    if (p >= 0) {
      mn = min(mn, p);
      mx = max(mx, p);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (mx < 0) {
    if (lane == 0) desc[wid] = make_int4(-1, -1, 0, 0);
    return;
  }
  uint64_t bits = 0;
  if (mx - mn < 64) {
    for (int64_t j = j0 + lane; j < j1; j += 32) {
      const int64_t p = __ldg(ipi + b * s_row + j);
      if (p >= 0) bits |= 1ull << (p - mn);
    }
    uint32_t lo = __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(bits));
    uint32_t hi = __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(bits >> 32));
    bits = (static_cast<uint64_t>(hi) << 32) | lo;
  }
  if (lane == 0)
    desc[wid] = make_int4(static_cast<int>(mn), static_cast<int>(min(mx, static_cast<int64_t>(INT32_MAX))),
                          static_cast<int>(static_cast<uint32_t>(bits)), static_cast<int>(static_cast<uint32_t>(bits >> 32)));
}

struct PgCand {
  const int4* desc;
  const int64_t* ipi;  // for wide blocks
  int64_t s_ipi, n_tok, bs, B, nblk;
  const int64_t* qpi;
  int64_t s_qpi, n_q;
  const int64_t* pos;
  int64_t s_pos, cq;
  int flat, fallback;
  uint8_t* out;        // [B, cq, nblk]
};

__device__ __forceinline__ bool block_has_page(const PgCand& a, int64_t b, int64_t c, int4 d, int64_t qp) {
  if (d.x < 0 || qp < d.x || qp > d.y) return false;
  const uint64_t bits = (static_cast<uint64_t>(static_cast<uint32_t>(d.w)) << 32) | static_cast<uint32_t>(d.z);
  if (bits) return qp - d.x < 64 && ((bits >> (qp - d.x)) & 1ull);
  // wide block: token scan
  const int64_t j1 = min((c + 1) * a.bs, a.n_tok);
  for (int64_t j = c * a.bs; j < j1; ++j)
    if (__ldg(a.ipi + b * a.s_ipi + j) == qp) return true;
  return false;
}

// One warp per 16 consecutive query rows of one batch row, 4 consecutive
// blocks per lane per 128-block step.  A step's mask word is computed once
// per run of rows with the same query page (consecutive queries nearly
// always share it) and stored for every row of the run, so the kernel is
// bound by the mask write rather than the descriptor reads.  Rows with a
// query page < 0 have no candidate; rows without one get every block when
// `fallback` (the reference's per-query fallback), else stay zero.
constexpr int kCandWarps = 8;
constexpr int kCandRows = 16;
__device__ __forceinline__ uint32_t cand_word(const PgCand& a, int64_t b, const int4* dr, int64_t c0, int64_t qp) {
  uint32_t word = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int64_t c = c0 + e;
    if (c < a.nblk) {
      const int4 d = __ldg(dr + c);
      const bool y = a.flat ? d.x >= 0 : block_has_page(a, b, c, d, qp);
      word |= static_cast<uint32_t>(y) << (8 * e);
    }
  }
  return word;
}
__global__ void __launch_bounds__(kCandWarps * 32) page_cand_kernel(const PgCand a) {
  const int lane = threadIdx.x & 31;
  const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * kCandWarps + (threadIdx.x >> 5)) * kCandRows;
  const int64_t b = blockIdx.y;
  if (row0 >= a.cq) return;  // warp-uniform
  const int nr = static_cast<int>(min(static_cast<int64_t>(kCandRows), a.cq - row0));
  int64_t my_qp = 0;  // lane r < nr: query page of row row0 + r
  if (!a.flat && lane < nr) {
    int64_t p = __ldg(a.pos + b * a.s_pos + row0 + lane);
    p = p < 0 ? 0 : (p > a.n_q - 1 ? a.n_q - 1 : p);
    my_qp = __ldg(a.qpi + b * a.s_qpi + p);
  }
  // runs of consecutive rows with the same page: bit r set where a run starts
  const int64_t up = __shfl_up_sync(0xffffffffu, my_qp, 1);
  const unsigned starts = __ballot_sync(0xffffffffu, lane < nr && (lane == 0 || up != my_qp));
  const unsigned rows_mask = nr >= 32 ? 0xffffffffu : ((1u << nr) - 1u);
  const bool w32 = (a.nblk & 3) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 3) == 0;
  const int4* dr = a.desc + b * a.nblk;
  uint8_t* const out0 = a.out + (b * a.cq + row0) * a.nblk;
  unsigned anyrows = 0;  // bit r: row r has a candidate among this lane's blocks
  for (int64_t base = 0; base < a.nblk; base += 128) {
    const int64_t c0 = base + 4 * lane;
    unsigned todo = starts;
    while (todo) {  // warp-uniform: one mask word per run, stored to each of its rows
      const int rs = __ffs(todo) - 1;
      todo &= todo - 1;
      const int re = todo ? __ffs(todo) - 1 : nr;
      const int64_t qp = a.flat ? 0 : static_cast<int64_t>(__shfl_sync(0xffffffffu, my_qp, rs));
      const uint32_t word = (a.flat || qp >= 0) ? cand_word(a, b, dr, c0, qp) : 0u;
      if (word) anyrows |= rows_mask & ((re >= 32 ? 0xffffffffu : ((1u << re) - 1u)) & ~((1u << rs) - 1u));
      if (c0 < a.nblk) {
        uint8_t* p = out0 + static_cast<int64_t>(rs) * a.nblk + c0;
        if (w32) {
          for (int r = rs; r < re; ++r, p += a.nblk) *reinterpret_cast<uint32_t*>(p) = word;
        } else {
          for (int r = rs; r < re; ++r, p += a.nblk) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (c0 + e < a.nblk) p[e] = static_cast<uint8_t>(word >> (8 * e));
          }
        }
      }
    }
  }
  if (!a.fallback) return;  // rows without a candidate stay zero
  const unsigned any = __reduce_or_sync(0xffffffffu, anyrows);
  for (int r = 0; r < nr; ++r) {
    if ((any >> r) & 1u) continue;
    uint8_t* row = out0 + static_cast<int64_t>(r) * a.nblk;
    for (int64_t c = lane; c < a.nblk; c += 32) row[c] = 1;
  }
}

// Decode allow of one new token per request: advances the marker count, then
// allow[c] = (c < nblk_state and block c holds image pages [bmin, bmax] around
// the query page) or the row is open (no page / no such block).  One CTA per
// request.
__global__ void __launch_bounds__(256) decode_allow_kernel(const int64_t* last_ids, int64_t s_ids, int64_t page_id,
                                                           const int64_t* bmin, const int64_t* bmax, int64_t s_state,
                                                           int64_t nblk_state, const int64_t* pp, int64_t* mcum,
                                                           int64_t nblk, uint8_t* allow) {
  __shared__ int64_t qps;
  const int64_t b = blockIdx.x;
  if (threadIdx.x == 0) {
    const int64_t m = mcum[b] + (__ldg(last_ids + b * s_ids) == page_id ? 1 : 0);
    const int64_t q = m - 1 - pp[b];
    qps = q >= 0 ? q : -1;
    mcum[b] = m;
  }
  __syncthreads();
  const int64_t qp = qps;
  const int64_t n0 = min(nblk, nblk_state);
  const int64_t* mn = bmin + b * s_state;
  const int64_t* mx = bmax + b * s_state;
  int any = 0;
  if (qp >= 0)
    for (int64_t c = threadIdx.x; c < n0; c += blockDim.x) {
      const int64_t lo = __ldg(mn + c);
      any |= (lo >= 0 && lo <= qp && __ldg(mx + c) >= qp);
    }
  any = __syncthreads_or(any);
  const bool open = qp < 0 || !any;
  uint8_t* out = allow + b * nblk;
  for (int64_t c = threadIdx.x; c < nblk; c += blockDim.x) {
    bool y = open;
    if (!y && c < n0) {
      const int64_t lo = __ldg(mn + c);
      y = lo >= 0 && lo <= qp && __ldg(mx + c) >= qp;
    }
    out[c] = y;
  }
}

}  // namespace srswa

using namespace srswa;

static size_t al16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

extern "C" size_t srswa_page_scan_workspace_size(int64_t B, int64_t n_tok) {
  if (B <= 0 || n_tok <= 0) return 0;
  return static_cast<size_t>(B) * static_cast<size_t>(cdiv<int64_t>(n_tok, kPgChunk)) * sizeof(int4);
}

static int page_scan_launch(const PgRow& r, int64_t B, int mode, const PgOut& o, void* ws, size_t ws_bytes,
                            cudaStream_t s) {
  const int64_t nchunk = cdiv<int64_t>(r.n_tok, kPgChunk);
  SRSWA_CHECK_ARG(nchunk <= INT32_MAX && B <= 65535, SRSWA_ETOOLARGE);
  SRSWA_CHECK_ARG(ws && ws_bytes >= srswa_page_scan_workspace_size(B, r.n_tok), SRSWA_EWORKSPACE);
  SRSWA_CHECK_ARG((reinterpret_cast<uintptr_t>(ws) & 15) == 0, SRSWA_EALIGN);
  int4* stats = static_cast<int4*>(ws);
  const dim3 grid(static_cast<unsigned>(nchunk), static_cast<unsigned>(B));
  page_count_kernel<<<grid, kPgThreads, 0, s>>>(r, nchunk, stats);
  if (mode == 0) {
    page_scan_kernel<0><<<grid, kPgThreads, 0, s>>>(r, nchunk, stats, o);
  } else if (mode == 1) {
    page_scan_kernel<1><<<grid, kPgThreads, 0, s>>>(r, nchunk, stats, o);
  } else {  // RoPE coordinates: marker positions first, then the tokens
    page_scan_kernel<2><<<grid, kPgThreads, 0, s>>>(r, nchunk, stats, o);
    page_scan_kernel<3><<<grid, kPgThreads, 0, s>>>(r, nchunk, stats, o);
  }
  return srswa_last_launch_status();
}

extern "C" int srswa_page_ids(const int64_t* ids, int64_t s_row, int64_t B, int64_t n_ids, int64_t key_length,
                              int64_t img_id, int64_t page_id, int64_t per_page, int page_scope_prefill,
                              uint8_t* itm, int64_t* ipi, int64_t* qpi, int32_t* flags, void* workspace,
                              size_t workspace_bytes, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(ids && itm && ipi && qpi && flags && B >= 0 && n_ids >= 0 && key_length >= 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(s_row >= n_ids || B <= 1, SRSWA_EINVAL);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SRSWA_CUDA_TRY(cudaMemsetAsync(flags, 0, 2 * sizeof(int32_t), s));
  if (B * key_length == 0) return 0;
  PgRow r = {ids, s_row, n_ids, key_length, img_id, page_id, per_page < 1 ? 1 : per_page};
  PgOut o = {};
  o.itm = itm; o.ipi = ipi; o.qpi = qpi; o.flags = flags; o.scope = page_scope_prefill ? 1 : 0;
  return page_scan_launch(r, B, 0, o, workspace, workspace_bytes, s);
}

extern "C" int srswa_decode_allow_state(const int64_t* ids, int64_t s_row, int64_t B, int64_t L, int64_t img_id,
                                        int64_t page_id, int64_t per_page, int64_t block_size, int64_t* bmin,
                                        int64_t* bmax, int64_t* pp, int64_t* mcum, void* workspace,
                                        size_t workspace_bytes, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(ids && bmin && bmax && pp && mcum && B >= 0 && L > 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(s_row >= L || B <= 1, SRSWA_EINVAL);
  // per-block reductions stay inside one chunk: the block size must divide it
  SRSWA_CHECK_ARG(block_size > 0 && block_size <= kPgChunk && kPgChunk % block_size == 0, SRSWA_EUNSUPPORTED);
  if (B == 0) return 0;
  PgRow r = {ids, s_row, L, L, img_id, page_id, per_page < 1 ? 1 : per_page};
  PgOut o = {};
  o.bmin = bmin; o.bmax = bmax; o.pp = pp; o.mcum = mcum; o.bs = block_size; o.nblk = cdiv<int64_t>(L, block_size);
  return page_scan_launch(r, B, 1, o, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_page_block_desc(const int64_t* ipi, const uint8_t* itm, int64_t s_row, int64_t B,
                                     int64_t n_tok, int64_t block_size, int64_t nblk, int32_t* desc,
                                     srswa_stream_t stream) {
  SRSWA_CHECK_ARG((ipi != nullptr) != (itm != nullptr) && desc && B >= 0 && n_tok >= 0 && nblk >= 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(block_size > 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG((reinterpret_cast<uintptr_t>(desc) & 15) == 0, SRSWA_EALIGN);
  const int64_t warps = B * nblk;
  if (warps == 0) return 0;
  SRSWA_CHECK_ARG(cdiv<int64_t>(warps, 8) <= INT32_MAX, SRSWA_ETOOLARGE);
  page_block_desc_kernel<<<static_cast<unsigned>(cdiv<int64_t>(warps, 8)), 256, 0,
                           reinterpret_cast<cudaStream_t>(stream)>>>(ipi, itm, s_row, n_tok, block_size, nblk, B,
                                                                     reinterpret_cast<int4*>(desc));
  return srswa_last_launch_status();
}

extern "C" int srswa_page_cand_mask(const int32_t* desc, const int64_t* ipi, int64_t s_ipi, int64_t n_tok,
                                    int64_t block_size, int64_t B, int64_t nblk, const int64_t* qpi, int64_t s_qpi,
                                    int64_t n_q, const int64_t* pos, int64_t s_pos, int64_t cq, int flat,
                                    int fallback, uint8_t* cand, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(desc && cand && B >= 0 && nblk >= 0 && cq >= 0 && block_size > 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(flat || (ipi && qpi && pos && n_q > 0), SRSWA_EINVAL);
  SRSWA_CHECK_ARG((reinterpret_cast<uintptr_t>(desc) & 15) == 0, SRSWA_EALIGN);
  if (B * cq * nblk == 0) return 0;
  SRSWA_CHECK_ARG(B <= 65535 && cdiv<int64_t>(cq, kCandWarps * kCandRows) <= INT32_MAX, SRSWA_ETOOLARGE);
  PgCand a = {};
  a.desc = reinterpret_cast<const int4*>(desc); a.ipi = ipi; a.s_ipi = s_ipi; a.n_tok = n_tok; a.bs = block_size;
  a.B = B; a.nblk = nblk; a.qpi = qpi; a.s_qpi = s_qpi; a.n_q = n_q; a.pos = pos; a.s_pos = s_pos; a.cq = cq;
  a.flat = flat ? 1 : 0; a.fallback = fallback ? 1 : 0; a.out = cand;
  const dim3 grid(static_cast<unsigned>(cdiv<int64_t>(cq, kCandWarps * kCandRows)), static_cast<unsigned>(B));
  page_cand_kernel<<<grid, kCandWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return srswa_last_launch_status();
}

extern "C" int srswa_decode_allow(const int64_t* last_ids, int64_t s_ids, int64_t B, int64_t page_id,
                                  const int64_t* bmin, const int64_t* bmax, int64_t s_state, int64_t nblk_state,
                                  const int64_t* pp, int64_t* mcum, int64_t nblk, uint8_t* allow,
                                  srswa_stream_t stream) {
  SRSWA_CHECK_ARG(last_ids && bmin && bmax && pp && mcum && allow && B >= 0 && nblk >= 0 && nblk_state >= 0,
                  SRSWA_EINVAL);
  SRSWA_CHECK_ARG(s_state >= nblk_state || B <= 1, SRSWA_EINVAL);
  if (B == 0) return 0;
  SRSWA_CHECK_ARG(B <= INT32_MAX, SRSWA_ETOOLARGE);
  decode_allow_kernel<<<static_cast<unsigned>(B), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      last_ids, s_ids, page_id, bmin, bmax, s_state, nblk_state, pp, mcum, nblk, allow);
  return srswa_last_launch_status();
}

namespace srswa {

// ------------------------------------------------------------ scan window --
// Remote page span of each decode row (K14): one warp per row scans the
// row's allow mask with 16-byte loads and reduces the first / last allowed
// live remote block.  Mask columns at or past min(W, WQ) are never read.
__global__ void __launch_bounds__(256) win_bounds_kernel(const uint8_t* __restrict__ allow, int64_t s_allow,
                                                         int64_t WQ, const int32_t* __restrict__ seq_lens,
                                                         int64_t nd, int64_t W, int64_t bs, int64_t L, int64_t dql,
                                                         int64_t tile, int32_t* lo_out, int32_t* hi_out,
                                                         int8_t* fit_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= nd) return;
  const int64_t seq = seq_lens[row / dql];
  const int64_t q_pos = seq - dql + row % dql;
  const int64_t q_blk = q_pos / bs;  // truncating, as the reference's integer division
  // allowed live remote blocks: off <= q_blk - L and off * bs < seq
  int64_t lim = q_blk - L + 1;
  const int64_t live = (seq + bs - 1) / bs;
  if (lim > live) lim = live;
  const int64_t width = W < WQ ? W : WQ;
  if (lim > width) lim = width;
  int64_t lo = W, hi = -1;
  const uint8_t* a = allow + row * s_allow;
  if (lim > 0) {
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(a) | static_cast<uintptr_t>(s_allow)) & 15) == 0;
    const int64_t nvec = vec_ok ? lim / 16 : 0;
    for (int64_t v = lane; v < nvec; v += 32) {
      const uint4 u = *reinterpret_cast<const uint4*>(a + v * 16);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if ((w[e >> 2] >> ((e & 3) * 8)) & 0xffu) {
          const int64_t off = v * 16 + e;
          lo = off < lo ? off : lo;
          hi = off > hi ? off : hi;
        }
      }
    }
    for (int64_t off = nvec * 16 + lane; off < lim; off += 32) {
      if (a[off]) {
        lo = off < lo ? off : lo;
        hi = off > hi ? off : hi;
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t l2 = __shfl_xor_sync(0xffffffffu, lo, o);
    const int64_t h2 = __shfl_xor_sync(0xffffffffu, hi, o);
    lo = l2 < lo ? l2 : lo;
    hi = h2 > hi ? h2 : hi;
  }
  if (lane == 0) {
    const bool any_r = hi >= 0;
    const int64_t nb = (seq + bs - 1) / bs;
    const int64_t nb1 = nb > 1 ? nb : 1;
    const int64_t w_seq = W < nb1 ? W : nb1;
    const bool no_remote = seq <= 0 || (q_blk - L) < 0;
    const int64_t lo_v = any_r ? lo : 0;
    const int64_t hi_v = any_r ? hi + 1 : (no_remote ? 0 : w_seq);
    lo_out[row] = static_cast<int32_t>(lo_v);
    hi_out[row] = static_cast<int32_t>(hi_v);
    fit_out[row] = (hi_v - lo_v) <= tile ? 1 : 0;
  }
}

}  // namespace srswa

extern "C" int srswa_win_bounds_decode(const uint8_t* allow, int64_t s_allow, int64_t WQ, const int32_t* seq_lens,
                                       int64_t nd, int64_t W, int64_t block_size, int64_t local_blocks,
                                       int64_t decode_query_len, int64_t tile, int32_t* lo, int32_t* hi,
                                       int8_t* fit, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(nd >= 0 && W > 0 && WQ >= 0 && block_size > 0 && local_blocks >= 0 && decode_query_len > 0,
                  SRSWA_EINVAL);
  if (nd == 0) return 0;
  SRSWA_CHECK_ARG(allow && seq_lens && lo && hi && fit, SRSWA_EINVAL);
  SRSWA_CHECK_ARG((nd + 7) / 8 < (1ll << 31), SRSWA_ETOOLARGE);
  srswa::win_bounds_kernel<<<static_cast<unsigned>((nd + 7) / 8), 256, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(
      allow, s_allow, WQ, seq_lens, nd, W, block_size, local_blocks, decode_query_len, tile, lo, hi, fit);
  return srswa_last_launch_status();
}

namespace srswa {

// ---------------------------------------------------------------------------
// page2d RoPE: the two-axis rotary of the indexer and main branch
// (hf-model-code/_sparse_base_impl.py:1984-2058).  Pair i < n_tok turns by
// tok * inv_tok[i], pair n_tok + i by (page mod page_mod) * inv_page[i]; the
// table is [angles, angles] over dim = 2 * (n_tok + page_pairs) features.
struct Rope2D {
  const int64_t* tok;
  const int64_t* page;
  int64_t s_pos;  // row stride of tok / page ([B, S])
  const float* inv_tok;
  const float* inv_page;
  int n_tok, half, page_mod;
};

__device__ __forceinline__ float rope_angle(const Rope2D& r, int64_t t, int64_t p, int pair) {
  if (pair < r.n_tok) return static_cast<float>(t) * __ldg(r.inv_tok + pair);
  if (r.page_mod > 0) {
    p %= r.page_mod;
    if (p < 0) p += r.page_mod;
  }
  return static_cast<float>(p) * __ldg(r.inv_page + pair - r.n_tok);
}

// cos / sin tables [B, S, 2 * half] (fp32 or bf16), one thread per (row, pair)
__global__ void __launch_bounds__(256) rope2d_table_kernel(const Rope2D r, int64_t B, int64_t S, void* cos_out,
                                                           void* sin_out, int dtype) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= B * S * r.half) return;
  const int pair = static_cast<int>(i % r.half);
  const int64_t row = i / r.half, b = row / S, s = row - b * S;
  float sn, cs;
  sincosf(rope_angle(r, __ldg(r.tok + b * r.s_pos + s), __ldg(r.page + b * r.s_pos + s), pair), &sn, &cs);
  const int64_t o = row * 2 * r.half + pair;
  store_elem(cos_out, o, dtype, cs);
  store_elem(cos_out, o + r.half, dtype, cs);
  store_elem(sin_out, o, dtype, sn);
  store_elem(sin_out, o + r.half, dtype, sn);
}

// In place x <- x * cos + rotate_half(x) * sin over the first D features of
// x [B, S, H, D] (strides s_b, s_s, s_h; D contiguous), feature f using pair
// f mod half; cos / sin are rounded to table_dtype first (the reference casts
// its tables to the activation dtype).  One thread per (b, s) and 8 pairs
// (f, f + D/2): the angles of a token are shared by its heads, so they are
// computed once (once per pair when D covers the table) and every head is
// rotated with them; 16-byte loads and stores where the rows allow.
template <typename T>
__device__ __forceinline__ void rope_load8(const T* p, bool vec, float* v) {
  if constexpr (sizeof(T) == 2) {
    if (vec) {
      const uint4 u = *reinterpret_cast<const uint4*>(p);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) { v[2 * e] = bf16_lo(w[e]); v[2 * e + 1] = bf16_hi(w[e]); }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = static_cast<float>(p[e]);
}
template <typename T>
__device__ __forceinline__ void rope_store8(T* p, bool vec, const float* v) {
  if constexpr (sizeof(T) == 2) {
    if (vec) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
        w[e] = *reinterpret_cast<uint32_t*>(&h);
      }
      *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) p[e] = static_cast<T>(v[e]);
}
template <typename T>
__global__ void __launch_bounds__(256) rope2d_apply_kernel(const Rope2D r, T* x, int64_t B, int64_t S, int64_t H,
                                                           int D, int64_t s_b, int64_t s_s, int64_t s_h,
                                                           int table_bf16) {
  const int g8 = D / 16;  // groups of 8 pairs per row
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= B * S * g8) return;
  const int g = static_cast<int>(i % g8);
  const int64_t bs_ = i / g8, s = bs_ % S, b = bs_ / S;
  const int64_t t = __ldg(r.tok + b * r.s_pos + s), p = __ldg(r.page + b * r.s_pos + s);
  const int hd = D / 2;
  const bool same = hd == r.half;  // both halves of a pair use the same angle
  float c1[8], s1[8], c2[8], s2[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const int f = 8 * g + e;
    sincosf(rope_angle(r, t, p, f % r.half), &s1[e], &c1[e]);
    if (same) {
      c2[e] = c1[e];
      s2[e] = s1[e];
    } else {
      sincosf(rope_angle(r, t, p, (f + hd) % r.half), &s2[e], &c2[e]);
    }
    if (table_bf16) {
      c1[e] = __bfloat162float(__float2bfloat16_rn(c1[e]));
      s1[e] = __bfloat162float(__float2bfloat16_rn(s1[e]));
      c2[e] = __bfloat162float(__float2bfloat16_rn(c2[e]));
      s2[e] = __bfloat162float(__float2bfloat16_rn(s2[e]));
    }
  }
  T* base = x + b * s_b + s * s_s;
  const bool vec = ((reinterpret_cast<uintptr_t>(base) | static_cast<uintptr_t>(s_h * sizeof(T)) |
                     static_cast<uintptr_t>(hd * sizeof(T))) & 15) == 0;
  for (int64_t h = 0; h < H; ++h) {
    T* row = base + h * s_h;
    float lo[8], hi[8];
    rope_load8(row + 8 * g, vec, lo);
    rope_load8(row + hd + 8 * g, vec, hi);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float a = lo[e], bb = hi[e];
      lo[e] = a * c1[e] - bb * s1[e];
      hi[e] = bb * c2[e] + a * s2[e];
    }
    rope_store8(row + 8 * g, vec, lo);
    rope_store8(row + hd + 8 * g, vec, hi);
  }
}

// Decode update of the (tok, page) coordinates of one new token per row
// (_main_rope_coords, _sparse_base_impl.py:1482-1489).
__global__ void rope2d_decode_kernel(const int64_t* new_ids, int64_t s_ids, int64_t B, int64_t page_id,
                                     int64_t* page, int64_t* tok, const int64_t* pf, int64_t s_pf, int64_t n_pg) {
  const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const bool is_pg = __ldg(new_ids + b * s_ids) == page_id;
  int64_t pg = page[b];
  if (is_pg) pg = pg + 1 < n_pg - 1 ? pg + 1 : n_pg - 1;
  page[b] = pg;
  tok[b] = is_pg ? __ldg(pf + b * s_pf + (pg > 0 ? pg : 0)) : tok[b] + 1;
}

}  // namespace srswa (page2d RoPE)

extern "C" size_t srswa_rope2d_pos_workspace_size(int64_t B, int64_t n_tok) {
  if (B <= 0 || n_tok <= 0) return 0;
  return al16(srswa_page_scan_workspace_size(B, n_tok)) + static_cast<size_t>(B) * (n_tok + 2) * sizeof(int64_t);
}

extern "C" int srswa_rope2d_pos(const int64_t* ids, int64_t s_row, int64_t B, int64_t n_ids, int64_t key_length,
                                int64_t img_id, int64_t page_id, int64_t span, int64_t* tok, int64_t* page,
                                int64_t* pf_cnt, int64_t pf_cap, int32_t* flags, void* workspace,
                                size_t workspace_bytes, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(ids && tok && page && pf_cnt && flags && B >= 0 && n_ids >= 0 && key_length >= 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(s_row >= n_ids || B <= 1, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(pf_cap >= key_length + 1, SRSWA_EINVAL);  // pages <= markers <= tokens
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SRSWA_CHECK_ARG(workspace_bytes >= srswa_rope2d_pos_workspace_size(B, key_length), SRSWA_EWORKSPACE);
  SRSWA_CUDA_TRY(cudaMemsetAsync(flags, 0, 4 * sizeof(int32_t), s));
  if (B * key_length == 0) return 0;
  PgRow r = {ids, s_row, n_ids, key_length, img_id, page_id, 1};
  PgOut o = {};
  const size_t stats_bytes = al16(srswa_page_scan_workspace_size(B, key_length));
  o.mpos = reinterpret_cast<int64_t*>(static_cast<unsigned char*>(workspace) + stats_bytes);
  o.s_mpos = key_length + 2;
  o.tok = tok; o.page = page; o.pf = pf_cnt; o.pf_cap = pf_cap; o.span = span; o.rflags = flags;
  return page_scan_launch(r, B, 2, o, workspace, stats_bytes, s);
}

static int rope2d_check(const Rope2D& r) {
  SRSWA_CHECK_ARG(r.tok && r.page && r.inv_tok && r.n_tok >= 0 && r.half > r.n_tok, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(r.half == r.n_tok || r.inv_page, SRSWA_EINVAL);
  return 0;
}

extern "C" int srswa_rope2d_table(const int64_t* tok, const int64_t* page, int64_t s_pos, int64_t B, int64_t S,
                                  const float* inv_tok, int64_t n_tok, const float* inv_page, int64_t page_pairs,
                                  int64_t page_mod, void* cos_out, void* sin_out, int dtype, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(cos_out && sin_out && B >= 0 && S >= 0 && n_tok >= 0 && page_pairs >= 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(dtype == SRSWA_F32 || dtype == SRSWA_BF16 || dtype == SRSWA_F16, SRSWA_EUNSUPPORTED);
  Rope2D r = {tok, page, s_pos, inv_tok, inv_page, static_cast<int>(n_tok), static_cast<int>(n_tok + page_pairs),
              static_cast<int>(page_mod)};
  if (int rc = rope2d_check(r)) return rc;
  const int64_t n = B * S * r.half;
  if (n == 0) return 0;
  SRSWA_CHECK_ARG(cdiv<int64_t>(n, 256) <= INT32_MAX, SRSWA_ETOOLARGE);
  rope2d_table_kernel<<<static_cast<unsigned>(cdiv<int64_t>(n, 256)), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      r, B, S, cos_out, sin_out, dtype);
  return srswa_last_launch_status();
}

extern "C" int srswa_rope2d_apply(void* x, int dtype, int64_t B, int64_t S, int64_t H, int64_t D, int64_t s_b,
                                  int64_t s_s, int64_t s_h, const int64_t* tok, const int64_t* page, int64_t s_pos,
                                  const float* inv_tok, int64_t n_tok, const float* inv_page, int64_t page_pairs,
                                  int64_t page_mod, int table_dtype, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(x && B >= 0 && S >= 0 && H >= 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(D > 0 && D % 16 == 0 && D <= 2 * (n_tok + page_pairs), SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG(dtype == SRSWA_F32 || dtype == SRSWA_BF16, SRSWA_EUNSUPPORTED);
  Rope2D r = {tok, page, s_pos, inv_tok, inv_page, static_cast<int>(n_tok), static_cast<int>(n_tok + page_pairs),
              static_cast<int>(page_mod)};
  if (int rc = rope2d_check(r)) return rc;
  const int64_t n = B * S * (D / 16);  // threads: (token, 8 pairs); heads looped inside
  if (n == 0 || H == 0) return 0;
  SRSWA_CHECK_ARG(cdiv<int64_t>(n, 256) <= INT32_MAX, SRSWA_ETOOLARGE);
  const unsigned grid = static_cast<unsigned>(cdiv<int64_t>(n, 256));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int tb = table_dtype == SRSWA_BF16 ? 1 : 0;
  if (dtype == SRSWA_BF16)
    rope2d_apply_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(r, static_cast<__nv_bfloat16*>(x), B, S, H,
                                                            static_cast<int>(D), s_b, s_s, s_h, tb);
  else
    rope2d_apply_kernel<float><<<grid, 256, 0, s>>>(r, static_cast<float*>(x), B, S, H, static_cast<int>(D), s_b,
                                                    s_s, s_h, tb);
  return srswa_last_launch_status();
}

extern "C" int srswa_rope2d_decode(const int64_t* new_ids, int64_t s_ids, int64_t B, int64_t page_id,
                                   int64_t* page, int64_t* tok, const int64_t* pf_cnt, int64_t s_pf, int64_t n_pg,
                                   srswa_stream_t stream) {
  SRSWA_CHECK_ARG(new_ids && page && tok && pf_cnt && B >= 0 && n_pg >= 1 && s_pf >= n_pg, SRSWA_EINVAL);
  if (B == 0) return 0;
  rope2d_decode_kernel<<<static_cast<unsigned>(cdiv<int64_t>(B, 128)), 128, 0,
                         reinterpret_cast<cudaStream_t>(stream)>>>(new_ids, s_ids, B, page_id, page, tok, pf_cnt,
                                                                   s_pf, n_pg);
  return srswa_last_launch_status();
}
