// Row-streaming sparse attend: one query row x one head per CTA (or per
// cluster of CTAs), keys = selected remote blocks U local window.
//
// Used by
//   * the paged decode attend, semantics of dash_sparse_attn_decode / K9+K10
//     (whl:sglang/srt/layers/attention/unlimited_dash_ops/attend_triton.py:307-518,
//     600-715; common.py:43-89) and _decode_attend
//     (hf-model-code/modeling_deepseekv2.py:455-481);
//   * the query-major gather-attention forward, semantics of K1/K5
//     (hf-model-code/sparse_gather_triton.py:35-122; sparse_gather_e2e_triton.py:36-121).
//
// For a query at position p with segment start sg (0 when unpacked):
//   ls = max(p - LW + 1, sg)
//   remote keys: keys j of selected blocks with sg <= j < ls and j <= p,
//                logit scale*q.k + bias(slot)
//   local keys:  ls <= j <= p, logit scale*q.k
// One softmax over the (disjoint) union; empty rows give o = 0, lse = -inf.
// Unused slots (id < 0, >= W, or valid == 0) are skipped wherever they sit; a
// repeated block id counts once.
//
// Design (memory-bound per row):
//   * grid.x = rows * nsplit, grid.y = heads; the nsplit CTAs of one
//     (row, head) form a thread-block cluster and merge (m, l, o) through
//     distributed shared memory: no global scratch, no second launch;
//   * each warp streams chunks of KPC keys: lanes form groups of LPK = D/8,
//     each lane loads 16 B (8 elements) of a key row, so a warp instruction
//     covers 32/LPK whole rows (fully coalesced 128-bit loads);
//   * q.k partials are combined by a transposed butterfly (7-8 shuffles per 8
//     keys); online softmax in the log2 domain; P.V accumulates 8 features per
//     lane in fp32.

#include <cmath>
#include <cooperative_groups.h>

#include "common.cuh"
#include "attend.cuh"
#include "peer.cuh"

namespace cg = cooperative_groups;

namespace srswa {

struct SlotInfo {
  int64_t page_off;  // element offset of the block (without pos / head)
  int64_t key0;      // absolute position of the block's first key
  float bias2;       // bias * log2(e) (0 for local)
  int remote;        // 1 remote, 0 local
};

__device__ __forceinline__ void attend_row_position(const AttendArgs& a, int64_t row, int64_t& seq,
                                                    int64_t& t, int64_t& p, int64_t& sg) {
  if (a.pos_mode == 3) {  // varlen rows: the request holding this row (binary search)
    int64_t lo = 0, hi = a.nreq;
    while (hi - lo > 1) {
      const int64_t mid = (lo + hi) >> 1;
      if (a.cu_rows[mid] <= row) lo = mid;
      else hi = mid;
    }
    seq = lo;
    t = row;
    p = static_cast<int64_t>(a.prefix_lens[lo]) + row - a.cu_rows[lo];
    sg = 0;
    return;
  }
  seq = row / a.rps;
  t = row % a.rps;
  if (a.pos_mode == 0) p = a.q_pos[row];
  else if (a.pos_mode == 1) p = static_cast<int64_t>(a.seq_lens[seq]) - a.rps + t;
  else p = t;
  sg = a.seg ? static_cast<int64_t>(a.seg[row]) : 0;
}

__device__ __forceinline__ int64_t block_offset(const AttendArgs& a, int64_t seq, int64_t blk) {
  if (a.block_table) return static_cast<int64_t>(a.block_table[seq * a.s_bt + blk]) * a.s_page;
  return seq * a.s_seq + blk * a.s_blk;
}

// MINB = CTAs per SM the register allocation must allow: 4 (128 registers)
// for the bandwidth-bound loads; 5 (96 registers, a few spills) for light
// loads, where a whole 2-way split then fits in one wave.
// One output value: to a.out; with a.push also to every region of the
// exchange: as LL word i (ll), or at the same offset (fp32 out inside this
// rank's own slot, flag protocol).
__device__ __forceinline__ void put_out(const AttendArgs& a, int64_t i, float v, uint32_t ep) {
  if (!a.push.regions) {
    store_elem(a.out, i, a.out_dtype, v);
    return;
  }
  if (a.push.ll) {
    static_cast<float*>(a.out)[i] = v;
    ll_put(a.push, i, ep, __float_as_uint(v));
    return;
  }
  const int64_t off = reinterpret_cast<const char*>(static_cast<const float*>(a.out) + i) -
                      static_cast<const char*>(a.push.own_region);
  for (int d = 0; d < static_cast<int>(a.push.world); ++d)
    *reinterpret_cast<float*>(static_cast<char*>(a.push.regions[d]) + off) = v;
}
// o_elems: N * H * D, the LL word of lse element 0
__device__ __forceinline__ void put_lse(const AttendArgs& a, int64_t i, float v, uint32_t ep, int64_t o_elems) {
  if (!a.push.regions) {
    a.lse_out[i] = v;
    return;
  }
  if (a.push.ll) {
    a.lse_out[i] = v;
    ll_put(a.push, o_elems + i, ep, __float_as_uint(v));
    return;
  }
  const int64_t off = reinterpret_cast<const char*>(a.lse_out + i) - static_cast<const char*>(a.push.own_region);
  for (int d = 0; d < static_cast<int>(a.push.world); ++d)
    *reinterpret_cast<float*>(static_cast<char*>(a.push.regions[d]) + off) = v;
}
// after a storing CTA's puts: it is one producer unit of the exchange
__device__ __forceinline__ void push_done(const AttendArgs& a) {
  if (!a.push.regions || a.push.ll) return;  // LL words need no flag
  __syncthreads();
  if (threadIdx.x == 0) peer_unit_done(a.push, static_cast<unsigned>(a.N * a.H));
}

// LL exchange + merge of one (row, head), by its storing CTA after its own
// puts: every rank's partial o (LL words e_o .. e_o + D - 1) and lse (word
// e_l) from this rank's region, merged by log-sum-exp in the same order and
// arithmetic as lse_merge_kernel into final_out[fo .. fo + D - 1]; then the
// CTA is one consumer unit of the exchange.
template <int D>
__device__ void merge_exchange(const AttendArgs& a, int64_t e_o, int64_t e_l, int64_t fo, int64_t fl,
                               uint32_t ep) {
  __shared__ float lse_s[32];
  const int tid = threadIdx.x;
  const int C = static_cast<int>(a.push.world);
  bool ok = true;
  if (tid < C) lse_s[tid] = __uint_as_float(ll_get(a.push, tid, e_l, ep, ok));
  __syncthreads();
  float M = -INFINITY;
  for (int c = 0; c < C; ++c) M = fmaxf(M, lse_s[c]);
  const float Mu = (M == -INFINITY) ? 0.f : M;
  float den = 0.f;
  for (int c = 0; c < C; ++c) den += (lse_s[c] == -INFINITY) ? 0.f : expf(lse_s[c] - Mu);
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int d = tid; d < D; d += kAttendThreads) {
    float acc = 0.f;
    for (int c = 0; c < C; ++c) {
      const float ov = __uint_as_float(ll_get(a.push, c, e_o + d, ep, ok));
      if (lse_s[c] != -INFINITY) acc += expf(lse_s[c] - Mu) * ov;
    }
    store_elem(a.final_out, fo + d, a.final_dtype, acc * inv);
  }
  if (tid == 0 && a.final_lse) a.final_lse[fl] = den > 0.f ? Mu + logf(den) : -INFINITY;
  __syncthreads();
  if (tid == 0) ll_consumer_done(a.push, static_cast<unsigned>(a.N * a.H));
}

template <int D, int KVT, int MINB>
__global__ void __launch_bounds__(kAttendThreads, MINB) attend_rows_kernel(const AttendArgs a) {
  constexpr int LPK = D / 8;     // lanes per key row
  constexpr int KPI = 32 / LPK;  // key rows per warp load instruction
  constexpr int KPC = KPI * 8;   // keys per chunk (8 loads per lane)

  __shared__ SlotInfo slots[kAttendMaxSlots];
  __shared__ int n_win, n_slots;
  __shared__ float w_m[kAttendWarps], w_l[kAttendWarps];
  __shared__ __align__(16) float w_o[kAttendWarps][D];
  __shared__ float c_m, c_l;
  __shared__ __align__(16) float c_o[D];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // without overlap nothing is read before the kernel ahead on the stream
  // has completed; with it only the selection waits (srswa_decode_desc.overlap)
  if (!a.overlap) pdl_wait();
  pdl_launch_dependents();
  const int nsplit = a.nsplit;
  // heads_inner: grid (heads x splits, rows), so that the CTAs of one row's
  // heads are launched together and read the same key rows (whole 2560-byte
  // rows of a page between them); else grid (rows x splits, heads)
  const int64_t row = a.row0 + (a.heads_inner ? static_cast<int64_t>(blockIdx.y) : blockIdx.x / nsplit);
  const int split = blockIdx.x % nsplit;
  const int h = a.heads_inner ? static_cast<int>(blockIdx.x / nsplit) : static_cast<int>(blockIdx.y);
  const int hk = static_cast<int>(h / (a.H / a.Hkv));
  const int hi = static_cast<int>((static_cast<int64_t>(hk) * a.HI) / a.Hkv);
  int64_t seq, t, p, sg;
  attend_row_position(a, row, seq, t, p, sg);
  const int64_t BS = a.BS;
  int64_t ls = p - a.LW + 1;
  if (ls < sg) ls = sg;
  if (ls < 0) ls = 0;
  const bool live = p >= 0 && p >= sg;

  // ---- window slots first: they do not depend on the selection ----
  if (warp == 0) {
    int n = 0;
    if (live && !a.skip_local) {
      const int64_t b_lo = ls / BS, b_hi = min(p / BS, a.W - 1);
      for (int64_t b0 = b_lo; b0 <= b_hi; b0 += 32) {
        const int64_t blk = b0 + lane;
        const bool ok = blk <= b_hi;
        const int64_t off = ok ? block_offset(a, seq, blk) : 0;
        const unsigned msk = __ballot_sync(0xffffffffu, ok);
        const int pos = n + lane;
        if (ok && pos < kAttendMaxSlots) {
          slots[pos].page_off = off;
          slots[pos].key0 = blk * BS;
          slots[pos].bias2 = 0.f;
          slots[pos].remote = 0;
        }
        n += __popc(msk);
        if (n > kAttendMaxSlots) n = kAttendMaxSlots;
      }
    }
    if (lane == 0) n_win = n;
  }
  __syncthreads();

  // ---- this lane's slice of q (pre-scaled into the log2 domain) ----
  const int g = lane / LPK, u = lane % LPK;
  float2 qv2[4];  // features (2w, 2w + 1): operands of the paired fp32 FMAs
  {
    float qv[8];
    load8(a.q, seq * a.s_q_seq + t * a.s_q_t + static_cast<int64_t>(h) * a.s_qh + u * 8, a.q_dtype, qv);
#pragma unroll
    for (int w = 0; w < 4; ++w) qv2[w] = make_float2(qv[2 * w] * a.q_scale_log2, qv[2 * w + 1] * a.q_scale_log2);
  }

  const int cpb = static_cast<int>(BS / KPC);  // chunks per block

  float m = -INFINITY, lsum = 0.f;
  float2 o2[4];  // this lane's 8 output features, paired
#pragma unroll
  for (int w = 0; w < 4; ++w) o2[w] = make_float2(0.f, 0.f);
  // after transpose_reduce8 each key's score sits in LPK/8 lanes; count it once
  const int count_lane = (u & (LPK / 8 - 1)) == 0;
  const int my_idx = 4 * ((u & (LPK / 2)) != 0) + 2 * ((u & (LPK / 4)) != 0) + ((u & (LPK / 8)) != 0);

  // chunks of slots [s_lo, s_hi): this split's share, one warp per chunk
  auto stream_slots = [&](int s_lo, int s_hi) {
    const int nch = (s_hi - s_lo) * cpb;
    const int c_begin = static_cast<int>((static_cast<int64_t>(nch) * split) / nsplit);
    const int c_end = static_cast<int>((static_cast<int64_t>(nch) * (split + 1)) / nsplit);
    for (int ch = c_begin + warp; ch < c_end; ch += kAttendWarps) {
      const SlotInfo si = slots[s_lo + ch / cpb];
      const int sub = ch % cpb;
      const int64_t k0 = si.key0 + static_cast<int64_t>(sub) * KPC;
      int64_t lo, hi_;  // valid absolute key range [lo, hi_)
      if (si.remote) {
        lo = k0 > sg ? k0 : sg;
        hi_ = min(min(k0 + KPC, p + 1), ls);
      } else {
        lo = k0 > ls ? k0 : ls;
        hi_ = min(k0 + KPC, p + 1);
      }
      if (lo >= hi_) continue;  // warp-uniform

      const int64_t base = si.page_off + static_cast<int64_t>(hk) * a.s_head +
                           static_cast<int64_t>(sub) * KPC * a.s_pos + u * 8;
      uint4 kr[8], vr[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int j = i * KPI + g;
        const int64_t pos = k0 + j;
        if (pos >= lo && pos < hi_) {
          const int64_t off = base + j * a.s_pos;
          kr[i] = load_kv8<KVT>(a.k, off);
          vr[i] = load_kv8<KVT>(a.v, off);
        } else {
          kr[i] = make_uint4(0, 0, 0, 0);
          vr[i] = make_uint4(0, 0, 0, 0);
        }
      }
      // q.k over this lane's 8 features: paired FMAs (fma.rn.f32x2) into
      // even / odd partial sums
      float part[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 acc = make_float2(0.f, 0.f);
        acc = __ffma2_rn(qv2[0], kv_pair<KVT, 0>(kr[i]), acc);
        acc = __ffma2_rn(qv2[1], kv_pair<KVT, 1>(kr[i]), acc);
        acc = __ffma2_rn(qv2[2], kv_pair<KVT, 2>(kr[i]), acc);
        acc = __ffma2_rn(qv2[3], kv_pair<KVT, 3>(kr[i]), acc);
        part[i] = acc.x + acc.y;
      }
      const float dot = transpose_reduce8<LPK>(part, u);
      const int64_t my_pos = k0 + my_idx * KPI + g;
      const float s2 = (my_pos >= lo && my_pos < hi_) ? dot + si.bias2 : -INFINITY;
      const float cmax = warp_max(s2);
      const float m_new = fmaxf(m, cmax);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);
      const float pr = exp2f(s2 - m_use);
      lsum = lsum * alpha + (count_lane ? pr : 0.f);
      const float2 alpha2 = make_float2(alpha, alpha);
#pragma unroll
      for (int w = 0; w < 4; ++w) o2[w] = __fmul2_rn(o2[w], alpha2);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float pi = __shfl_sync(0xffffffffu, pr, g * LPK + transpose_owner<LPK>(i));
        const float2 p2 = make_float2(pi, pi);
        o2[0] = __ffma2_rn(p2, kv_pair<KVT, 0>(vr[i]), o2[0]);
        o2[1] = __ffma2_rn(p2, kv_pair<KVT, 1>(vr[i]), o2[1]);
        o2[2] = __ffma2_rn(p2, kv_pair<KVT, 2>(vr[i]), o2[2]);
        o2[3] = __ffma2_rn(p2, kv_pair<KVT, 3>(vr[i]), o2[3]);
      }
      m = m_new;
    }
  };

  const int nw = n_win;
  stream_slots(0, nw);
  if (a.overlap) pdl_wait();  // the selection comes from the kernel ahead

  // ---- remote slots: the selections (deduped, useful only), after the
  //      window.  Built by warp 0 with one lane per slot: the index,
  //      block-table and bias loads of all slots are issued together. ----
  if (warp == 0) {
    int n = nw;
    if (live) {
      const int64_t ibase = seq * a.s_sel_seq + t * a.s_sel_t + hi * a.s_sel_h;
      const int64_t bbase = seq * a.s_b_seq + t * a.s_b_t + hi * a.s_b_h;
      for (int64_t s0 = 0; s0 < a.K; s0 += 32) {
        const int64_t s = s0 + lane;
        int64_t blk = -1;
        bool ok = false;
        if (s < a.K) {
          blk = load_index(a.sel, ibase + s, a.idx_is64);
          ok = blk >= 0 && blk < a.W && (a.valid == nullptr || a.valid[ibase + s] != 0);
          if (ok) {  // a remote key must satisfy sg <= j < ls and j <= p
            const int64_t lo = blk * BS > sg ? blk * BS : sg;
            const int64_t hi_ = (blk + 1) * BS < ls ? (blk + 1) * BS : ls;
            ok = lo < hi_ && lo <= p;
          }
        }
        // drop repeats of an earlier usable slot (this batch, then earlier
        // batches; window slots cover other keys of a block and stay)
        for (int j = 0; j < 32; ++j) {
          const int64_t ob = __shfl_sync(0xffffffffu, blk, j);
          const bool ook = __shfl_sync(0xffffffffu, ok, j);
          if (j < lane && ook && ob == blk) ok = false;
        }
        for (int j = nw; j < n; ++j)
          if (ok && slots[j].key0 == blk * BS) ok = false;
        int64_t off = 0;
        float b2 = 0.f;
        if (ok) {
          off = block_offset(a, seq, blk);
          b2 = a.bias ? a.bias[bbase + s] * kLog2e : 0.f;
        }
        const unsigned msk = __ballot_sync(0xffffffffu, ok);
        if (ok) {
          const int pos = n + __popc(msk & ((1u << lane) - 1u));
          if (pos < kAttendMaxSlots) {
            slots[pos].page_off = off;
            slots[pos].key0 = blk * BS;
            slots[pos].bias2 = b2;
            slots[pos].remote = 1;
          }
        }
        n += __popc(msk);
        if (n > kAttendMaxSlots) n = kAttendMaxSlots;
        __syncwarp();
      }
    }
    if (lane == 0) n_slots = n;
  }
  __syncthreads();
  stream_slots(nw, n_slots);

  float o[8];
#pragma unroll
  for (int w = 0; w < 4; ++w) { o[2 * w] = o2[w].x; o[2 * w + 1] = o2[w].y; }

  // ---- warp combine: sum l over lanes, o over key groups ----
  lsum = warp_sum(lsum);
#pragma unroll
  for (int msk = LPK; msk < 32; msk <<= 1) {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], msk);
  }
  if (lane == 0) { w_m[warp] = m; w_l[warp] = lsum; }
  if (lane < LPK) {
#pragma unroll
    for (int e = 0; e < 8; ++e) w_o[warp][u * 8 + e] = o[e];
  }
  __syncthreads();

  // ---- CTA combine ----
  float M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kAttendWarps; ++w) M = fmaxf(M, w_m[w]);
  const float Mu = (M == -INFINITY) ? 0.f : M;
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < kAttendWarps; ++w) L += w_l[w] * exp2f(w_m[w] - Mu);
  for (int d = tid; d < D; d += kAttendThreads) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kAttendWarps; ++w) acc += w_o[w][d] * exp2f(w_m[w] - Mu);
    c_o[d] = acc;
  }
  if (tid == 0) { c_m = M; c_l = L; }

  const int64_t obase = seq * a.s_o_seq + t * a.s_o_t + static_cast<int64_t>(h) * a.s_oh;
  const int64_t lbase = seq * a.s_l_seq + t * a.s_l_t + h;
  if (nsplit == 1) {
    __syncthreads();
    const float inv = c_l > 0.f ? 1.f / c_l : 0.f;
    const uint32_t ep = a.push.regions && a.push.ll ? ll_epoch(a.push) : 0u;
    for (int d = tid; d < D; d += kAttendThreads) put_out(a, obase + d, c_o[d] * inv, ep);
    if (tid == 0 && a.lse_out)
      put_lse(a, lbase, c_l > 0.f ? (c_m + log2f(c_l)) * kLn2 : -INFINITY, ep, a.N * a.H * D);
    push_done(a);
    if (a.final_out) {
      __syncthreads();  // this CTA's puts precede its gets (its own slot included)
      merge_exchange<D>(a, obase, a.N * a.H * D + lbase, obase, lbase, ep);
    }
    return;
  }

  // ---- cluster combine through distributed shared memory ----
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (cluster.block_rank() == 0) {
    const uint32_t ep = a.push.regions && a.push.ll ? ll_epoch(a.push) : 0u;
    float Mg = -INFINITY;
    for (int s = 0; s < nsplit; ++s) Mg = fmaxf(Mg, *cluster.map_shared_rank(&c_m, s));
    const float Mgu = (Mg == -INFINITY) ? 0.f : Mg;
    float Lg = 0.f;
    for (int s = 0; s < nsplit; ++s)
      Lg += *cluster.map_shared_rank(&c_l, s) * exp2f(*cluster.map_shared_rank(&c_m, s) - Mgu);
    const float inv = Lg > 0.f ? 1.f / Lg : 0.f;
    for (int d = tid; d < D; d += kAttendThreads) {
      float acc = 0.f;
      for (int s = 0; s < nsplit; ++s)
        acc += cluster.map_shared_rank(c_o, s)[d] * exp2f(*cluster.map_shared_rank(&c_m, s) - Mgu);
      put_out(a, obase + d, acc * inv, ep);
    }
    if (tid == 0 && a.lse_out) put_lse(a, lbase, Lg > 0.f ? (Mg + log2f(Lg)) * kLn2 : -INFINITY, ep, a.N * a.H * D);
    push_done(a);  // CTA-uniform: the cluster's first CTA stores
    if (a.final_out) {
      __syncthreads();
      merge_exchange<D>(a, obase, a.N * a.H * D + lbase, obase, lbase, ep);
    }
  }
  cluster.sync();
}

template <int D, int KVT, int MINB = 4>
static int launch_attend(const AttendArgs& a, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = a.heads_inner ? dim3(static_cast<unsigned>(a.H * a.nsplit), static_cast<unsigned>(a.N), 1)
                              : dim3(static_cast<unsigned>(a.N * a.nsplit), static_cast<unsigned>(a.H), 1);
  cfg.blockDim = dim3(kAttendThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.nsplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // may start while the kernel ahead on the stream runs: the kernel waits
  // for it (pdl_wait) before reading what it writes
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attend_rows_kernel<D, KVT, MINB>, a);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// Split count of the (row, head) items when the caller leaves it open: the
// items run in waves of (SMs x resident CTAs), each split adds a cluster
// merge.  Modelled time = waves x (keys per CTA + merge cost), keys per item
// = window + selected blocks.  A CTA streams at a fixed rate whatever the
// load (a wave that is nearly empty still costs a full CTA time), and a
// cluster merge costs about as much as streaming 175 keys: fitted to the cfg3
// decode at 16 to 256 requests per GPU with fixed split counts (best: 2 at
// 160 items, 1 from 320 items up).  Smallest modelled time wins, by at least
// 3 % over a smaller split.
// Resident CTAs of the attend kernel per SM and the SM count (cached per device).
// Resident CTAs of a kernel instantiation on the current device (cached per
// device and instantiation).
template <typename K>
static double kernel_slots(K kern, int idx) {
  static int sms[64] = {0}, per_sm[64][12] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (sms[dev] == 0) {
    int v = 0;
    sms[dev] = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0 ? v : 148;
  }
  if (per_sm[dev][idx] == 0) {
    int nb = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kAttendThreads, 0);
    per_sm[dev][idx] = e == cudaSuccess && nb > 0 ? nb : 4;
  }
  return static_cast<double>(sms[dev]) * per_sm[dev][idx];
}

static double attend_slots(int64_t D, int kv_dtype) {
  if (D == 128) {
    switch (kv_dtype) {
      case SRSWA_BF16: return kernel_slots(attend_rows_kernel<128, SRSWA_BF16, 4>, 0);
      case SRSWA_F16: return kernel_slots(attend_rows_kernel<128, SRSWA_F16, 4>, 1);
      case SRSWA_F8E4M3: return kernel_slots(attend_rows_kernel<128, SRSWA_F8E4M3, 4>, 5);
      default: return kernel_slots(attend_rows_kernel<128, SRSWA_F8E5M2, 4>, 6);
    }
  }
  switch (kv_dtype) {
    case SRSWA_BF16: return kernel_slots(attend_rows_kernel<64, SRSWA_BF16, 4>, 2);
    case SRSWA_F16: return kernel_slots(attend_rows_kernel<64, SRSWA_F16, 4>, 3);
    case SRSWA_F8E4M3: return kernel_slots(attend_rows_kernel<64, SRSWA_F8E4M3, 4>, 7);
    default: return kernel_slots(attend_rows_kernel<64, SRSWA_F8E5M2, 4>, 8);
  }
}

// The light-load instantiation (5 CTAs per SM), bf16, head dim 128.
static double attend_slots_light() { return kernel_slots(attend_rows_kernel<128, SRSWA_BF16, 5>, 4); }

static int auto_nsplit(const AttendArgs& a, int64_t D, int kv_dtype) {
  const double slots = attend_slots(D, kv_dtype);
  const double items = static_cast<double>(a.N) * a.H;
  const double keys = static_cast<double>(a.LW) + static_cast<double>(a.K) * a.BS;
  int best = 1;
  double best_t = 0.0;
  for (int n = 1; n <= 8; n *= 2) {
    const double waves = std::ceil(items * n / slots);
    const double t = waves * (keys / n + (n > 1 ? 175.0 : 0.0));
    if (n == 1 || t < best_t * 0.97) {
      best = n;
      best_t = t;
    }
  }
  return best;
}

template <int D, int KVT>
static int launch_attend_rows(AttendArgs a, cudaStream_t st);

// With unsplit items the last wave of CTAs can run nearly empty (cfg3: 2560
// (row, head) items on 592 resident CTAs = 4.32 waves, the fifth a third
// full).  When the caller leaves the split open and the model picks 1, the
// rows that fill whole waves run unsplit and the remaining rows run first,
// split over clusters so that they cover the GPU for a fraction of a CTA's
// time: e.g. 20 tail rows x 10 heads x 2 CTAs, then 236 rows in 4 full
// waves.  Same results (the split merges in a cluster as any split does).
template <int D, int KVT>
static int launch_attend_rows(AttendArgs a, cudaStream_t st) {
  if (a.nsplit == 1 && a.split_tail) {
    const double slots = attend_slots(D, KVT);
    const int64_t items = a.N * a.H;
    const int64_t full = static_cast<int64_t>(items / slots);
    const int64_t r1 = static_cast<int64_t>((static_cast<double>(full) * slots) / static_cast<double>(a.H));
    const int64_t tail_rows = a.N - r1;
    const int64_t nt = tail_rows > 0 ? static_cast<int64_t>(slots / static_cast<double>(tail_rows * a.H)) : 0;
    if (full >= 1 && r1 > 0 && tail_rows > 0 && nt >= 2) {
      AttendArgs t = a;
      t.row0 = a.row0 + r1;
      t.N = tail_rows;
      t.nsplit = static_cast<int>(nt > 8 ? 8 : nt);
      int rc = launch_attend<D, KVT>(t, st);
      if (rc) return rc;
      a.N = r1;
    }
  }
  return launch_attend<D, KVT>(a, st);
}

int attend_rows_launch(AttendArgs a, int64_t D, int kv_dtype, cudaStream_t st) {
  if (a.N == 0) return 0;
  if (!(D == 64 || D == 128)) return SRSWA_EUNSUPPORTED;
  if (!(kv_dtype == SRSWA_BF16 || kv_dtype == SRSWA_F16 || kv_is_fp8(kv_dtype))) return SRSWA_EUNSUPPORTED;
  const int kpc = (32 / (static_cast<int>(D) / 8)) * 8;
  if (a.BS % kpc != 0) return SRSWA_EUNSUPPORTED;
  if (a.K + a.LW / a.BS + 2 > kAttendMaxSlots) return SRSWA_ETOOLARGE;
  if (a.H >= 65536) return SRSWA_ETOOLARGE;
  int nsplit = a.nsplit;
  // a push counts its producer units over one launch: no second launch
  a.split_tail = (nsplit <= 0 && !a.push.regions) ? 1 : 0;
  if (nsplit <= 0) nsplit = auto_nsplit(a, D, kv_dtype);
  if (nsplit < 1 || nsplit > 8) return SRSWA_EUNSUPPORTED;
  if (a.N * 8 >= (1ll << 31)) return SRSWA_ETOOLARGE;
  a.nsplit = nsplit;
  a.heads_inner = (a.N <= 65535 && a.H * 8 <= 65535) ? 1 : 0;
  // the merge inside the attend waits for the peers' CTAs of the same (row,
  // head): the whole grid must be resident at once
  if (a.final_out && static_cast<double>(a.N) * a.H * nsplit > attend_slots(D, kv_dtype)) return SRSWA_ETOOLARGE;
  if (D == 128) {
    if (kv_dtype == SRSWA_BF16) {
      // A light load that one wave holds unsplit but not 2-way split (e.g.
      // 32 requests x 10 heads per GPU): with 5 CTAs per SM the 2-way split
      // fits in one wave, halving each CTA's keys.
      const double items = static_cast<double>(a.N) * a.H;
      if (a.split_tail && nsplit == 1 && items <= attend_slots(D, kv_dtype) &&
          2.0 * items > attend_slots(D, kv_dtype) && 2.0 * items <= attend_slots_light()) {
        a.nsplit = 2;
        a.split_tail = 0;
        return launch_attend<128, SRSWA_BF16, 5>(a, st);
      }
      return launch_attend_rows<128, SRSWA_BF16>(a, st);
    }
    if (kv_dtype == SRSWA_F16) return launch_attend_rows<128, SRSWA_F16>(a, st);
    if (kv_dtype == SRSWA_F8E4M3) return launch_attend_rows<128, SRSWA_F8E4M3>(a, st);
    return launch_attend_rows<128, SRSWA_F8E5M2>(a, st);
  }
  if (kv_dtype == SRSWA_BF16) return launch_attend_rows<64, SRSWA_BF16>(a, st);
  if (kv_dtype == SRSWA_F16) return launch_attend_rows<64, SRSWA_F16>(a, st);
  if (kv_dtype == SRSWA_F8E4M3) return launch_attend_rows<64, SRSWA_F8E4M3>(a, st);
  return launch_attend_rows<64, SRSWA_F8E5M2>(a, st);
}

__global__ void lse_merge_kernel(const float* __restrict__ o_parts, const float* __restrict__ lse_parts,
                                 int64_t C, int64_t NH, int64_t D, int64_t s_o, int64_t s_l, void* out,
                                 int out_dtype, float* lse_out, const srswa_peer wait) {
  const int64_t nh = blockIdx.x;
  pdl_wait();  // launched to overlap the kernel ahead: its writes are visible from here
  if (wait.regions && wait.ll) {  // the parts are LL words in this rank's region: part c = source rank c
    __shared__ float lse_s[32];
    const uint32_t ep = ll_epoch(wait);
    bool ok = true;
    if (threadIdx.x < C) lse_s[threadIdx.x] = __uint_as_float(ll_get(wait, threadIdx.x, NH * D + nh, ep, ok));
    __syncthreads();
    float M = -INFINITY;
    for (int64_t c = 0; c < C; ++c) M = fmaxf(M, lse_s[c]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float den = 0.f;
    for (int64_t c = 0; c < C; ++c) den += (lse_s[c] == -INFINITY) ? 0.f : expf(lse_s[c] - Mu);
    const float inv = den > 0.f ? 1.f / den : 0.f;
    for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
      float acc = 0.f;
      for (int64_t c = 0; c < C; ++c) {
        const float ov = __uint_as_float(ll_get(wait, static_cast<int>(c), nh * D + d, ep, ok));
        if (lse_s[c] != -INFINITY) acc += expf(lse_s[c] - Mu) * ov;
      }
      store_elem(out, nh * D + d, out_dtype, acc * inv);
    }
    if (threadIdx.x == 0 && lse_out) lse_out[nh] = den > 0.f ? Mu + logf(den) : -INFINITY;
    __syncthreads();
    if (threadIdx.x == 0) ll_consumer_done(wait, gridDim.x);
    return;
  }
  if (wait.regions) {  // the parts are the peers' pushes into this rank's region
    if (threadIdx.x == 0) peer_wait_all(wait, gridDim.x);
    __syncthreads();
  }
  float M = -INFINITY;
  for (int64_t c = 0; c < C; ++c) M = fmaxf(M, lse_parts[c * s_l + nh]);
  const float Mu = (M == -INFINITY) ? 0.f : M;
  float den = 0.f;
  for (int64_t c = 0; c < C; ++c) {
    const float l = lse_parts[c * s_l + nh];
    den += (l == -INFINITY) ? 0.f : expf(l - Mu);
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int64_t c = 0; c < C; ++c) {
      const float l = lse_parts[c * s_l + nh];
      if (l != -INFINITY) acc += expf(l - Mu) * o_parts[c * s_o + nh * D + d];
    }
    store_elem(out, nh * D + d, out_dtype, acc * inv);
  }
  if (threadIdx.x == 0 && lse_out) lse_out[nh] = den > 0.f ? Mu + logf(den) : -INFINITY;
}

}  // namespace srswa

using namespace srswa;

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

static int decode_attend(const srswa_decode_desc* dd, const void* q, const void* k_cache, const void* v_cache,
                         const int32_t* block_table, const int32_t* seq_lens, const int64_t* q_pos,
                         const void* topk_idx, const float* bias, const uint8_t* valid, void* out, float* lse_out,
                         const srswa_peer* push, srswa_stream_t stream, void* final_out = nullptr,
                         int final_dtype = 0, float* final_lse = nullptr);

extern "C" int srswa_decode_attend(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                                   const void* v_cache, const int32_t* block_table,
                                   const int32_t* seq_lens, const int64_t* q_pos,
                                   const void* topk_idx, const float* bias, const uint8_t* valid,
                                   void* out, float* lse_out, srswa_stream_t stream) {
  return decode_attend(dd, q, k_cache, v_cache, block_table, seq_lens, q_pos, topk_idx, bias, valid, out, lse_out,
                       nullptr, stream);
}

extern "C" int srswa_decode_attend_push(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                                        const void* v_cache, const int32_t* block_table,
                                        const int32_t* seq_lens, const int64_t* q_pos,
                                        const void* topk_idx, const float* bias, const uint8_t* valid,
                                        float* out, float* lse_out, const srswa_peer* push,
                                        srswa_stream_t stream) {
  SRSWA_CHECK_ARG(push && push->regions && push->own_region && push->counter && push->tickets &&
                      push->world >= 1 && push->world <= 32 && push->rank >= 0 && push->rank < push->world,
                  SRSWA_EINVAL);
  SRSWA_CHECK_ARG(dd && out && lse_out && dd->out_dtype == SRSWA_F32, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(dd->s_on == dd->H * dd->D && dd->s_oh == dd->D, SRSWA_EINVAL);  // contiguous [N, H, D]
  const int64_t ob = dd->N * dd->H * dd->D * 4, lb = dd->N * dd->H * 4;
  if (push->ll) {  // LL words of the packed o then lse, 8 bytes per element
    SRSWA_CHECK_ARG((ob + lb) * 2 <= push->slot_bytes, SRSWA_EINVAL);
  } else {  // o and lse must lie in this rank's own slot, contiguous [N, H, D] and [N, H]
    const char* slot = static_cast<const char*>(push->own_region) + kPeerHeader + push->rank * push->slot_bytes;
    const char* o0 = reinterpret_cast<const char*>(out);
    const char* l0 = reinterpret_cast<const char*>(lse_out);
    SRSWA_CHECK_ARG(o0 >= slot && o0 + ob <= slot + push->slot_bytes && l0 >= slot &&
                        l0 + lb <= slot + push->slot_bytes,
                    SRSWA_EINVAL);
  }
  return decode_attend(dd, q, k_cache, v_cache, block_table, seq_lens, q_pos, topk_idx, bias, valid, out, lse_out,
                       push, stream);
}

extern "C" int srswa_decode_attend_exchange(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                                            const void* v_cache, const int32_t* block_table,
                                            const int32_t* seq_lens, const int64_t* q_pos,
                                            const void* topk_idx, const float* bias, const uint8_t* valid,
                                            float* out, float* lse_out, const srswa_peer* exchange,
                                            void* final_out, int final_dtype, float* final_lse,
                                            srswa_stream_t stream) {
  SRSWA_CHECK_ARG(exchange && exchange->ll && final_out, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(final_dtype == SRSWA_F32 || final_dtype == SRSWA_BF16 || final_dtype == SRSWA_F16,
                  SRSWA_EUNSUPPORTED);
  SRSWA_CHECK_ARG(aligned16(final_out), SRSWA_EALIGN);
  SRSWA_CHECK_ARG(exchange->regions && exchange->own_region && exchange->counter && exchange->tickets &&
                      exchange->world >= 1 && exchange->world <= 32 && exchange->rank >= 0 &&
                      exchange->rank < exchange->world,
                  SRSWA_EINVAL);
  SRSWA_CHECK_ARG(dd && out && lse_out && dd->out_dtype == SRSWA_F32, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(dd->s_on == dd->H * dd->D && dd->s_oh == dd->D, SRSWA_EINVAL);
  SRSWA_CHECK_ARG((dd->N * dd->H * (dd->D + 1)) * 8 <= exchange->slot_bytes, SRSWA_EINVAL);
  return decode_attend(dd, q, k_cache, v_cache, block_table, seq_lens, q_pos, topk_idx, bias, valid, out, lse_out,
                       exchange, stream, final_out, final_dtype, final_lse);
}

static int decode_attend(const srswa_decode_desc* dd, const void* q, const void* k_cache, const void* v_cache,
                         const int32_t* block_table, const int32_t* seq_lens, const int64_t* q_pos,
                         const void* topk_idx, const float* bias, const uint8_t* valid, void* out, float* lse_out,
                         const srswa_peer* push, srswa_stream_t stream, void* final_out, int final_dtype,
                         float* final_lse) {
  SRSWA_CHECK_ARG(dd && q && k_cache && v_cache && out, SRSWA_EINVAL);
  const srswa_decode_desc& d = *dd;
  SRSWA_CHECK_ARG(d.N >= 0 && d.H > 0 && d.Hkv > 0 && d.H % d.Hkv == 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(d.K >= 0 && (d.K == 0 || topk_idx), SRSWA_EINVAL);
  SRSWA_CHECK_ARG(q_pos || seq_lens, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(d.rows_per_req > 0 && d.block_size > 0 && d.local_blocks >= 0 && d.W > 0, SRSWA_EINVAL);
  // every row's request must exist: rows n / rows_per_req < R
  SRSWA_CHECK_ARG(d.R > 0 && (d.N + d.rows_per_req - 1) / d.rows_per_req <= d.R, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(aligned16(q) && aligned16(k_cache) && aligned16(v_cache), SRSWA_EALIGN);
  SRSWA_CHECK_ARG(((d.s_page | d.s_pos | d.s_head) & 7) == 0, SRSWA_EALIGN);
  SRSWA_CHECK_ARG(((d.s_qn | d.s_qh) & (d.q_dtype == SRSWA_F32 ? 3 : 7)) == 0, SRSWA_EALIGN);
  AttendArgs a = {};
  a.q = q; a.k = k_cache; a.v = v_cache; a.q_dtype = d.q_dtype; a.out_dtype = d.out_dtype;
  a.N = d.N; a.rps = d.rows_per_req; a.H = d.H; a.Hkv = d.Hkv;
  a.seq_lens = seq_lens; a.q_pos = q_pos; a.seg = nullptr;
  a.pos_mode = q_pos ? 0 : 1;
  a.block_table = block_table; a.s_bt = d.W; a.W = d.W;
  a.s_page = d.s_page; a.s_seq = d.s_req; a.s_blk = d.s_page;
  a.s_pos = d.s_pos; a.s_head = d.s_head;
  a.sel = topk_idx; a.idx_is64 = d.idx_is64; a.K = d.K; a.valid = valid;
  a.s_sel_seq = d.rows_per_req * d.s_ti_n; a.s_sel_t = d.s_ti_n; a.s_sel_h = d.s_ti_h; a.HI = d.Hkv;
  a.bias = bias; a.s_b_seq = d.rows_per_req * d.s_b_n; a.s_b_t = d.s_b_n; a.s_b_h = d.s_b_h;
  a.BS = d.block_size; a.LW = d.local_blocks * d.block_size;
  a.q_scale_log2 = d.sm_scale * kLog2e;
  a.s_q_seq = d.rows_per_req * d.s_qn; a.s_q_t = d.s_qn; a.s_qh = d.s_qh;
  a.out = out; a.s_o_seq = d.rows_per_req * d.s_on; a.s_o_t = d.s_on; a.s_oh = d.s_oh;
  a.lse_out = lse_out; a.s_l_seq = d.rows_per_req * d.H; a.s_l_t = d.H;
  a.nsplit = d.nsplit; a.skip_local = d.skip_local ? 1 : 0; a.overlap = d.overlap ? 1 : 0;
  if (push) a.push = *push;
  a.final_out = final_out; a.final_dtype = final_dtype; a.final_lse = final_lse;
  return attend_rows_launch(a, d.D, d.kv_dtype, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_prefill_attend(const srswa_decode_desc* dd, const void* q, const void* k_cache,
                                    const void* v_cache, const int32_t* block_table, const int32_t* cu_seqlens_q,
                                    const int32_t* prefix_lens, const void* topk_idx, const float* bias,
                                    void* out, float* lse_out, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(dd && q && k_cache && v_cache && out && block_table && cu_seqlens_q && prefix_lens,
                  SRSWA_EINVAL);
  const srswa_decode_desc& d = *dd;
  SRSWA_CHECK_ARG(d.N >= 0 && d.H > 0 && d.Hkv > 0 && d.H % d.Hkv == 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(d.K >= 0 && (d.K == 0 || topk_idx), SRSWA_EINVAL);
  SRSWA_CHECK_ARG(d.R > 0 && d.block_size > 0 && d.local_blocks >= 0 && d.W > 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(aligned16(q) && aligned16(k_cache) && aligned16(v_cache), SRSWA_EALIGN);
  SRSWA_CHECK_ARG(((d.s_page | d.s_pos | d.s_head) & 7) == 0, SRSWA_EALIGN);
  SRSWA_CHECK_ARG(((d.s_qn | d.s_qh) & (d.q_dtype == SRSWA_F32 ? 3 : 7)) == 0, SRSWA_EALIGN);
  AttendArgs a = {};
  a.q = q; a.k = k_cache; a.v = v_cache; a.q_dtype = d.q_dtype; a.out_dtype = d.out_dtype;
  a.N = d.N; a.rps = 1; a.H = d.H; a.Hkv = d.Hkv;
  a.seq_lens = nullptr; a.q_pos = nullptr; a.seg = nullptr;
  a.pos_mode = 3; a.cu_rows = cu_seqlens_q; a.prefix_lens = prefix_lens; a.nreq = d.R;
  a.block_table = block_table; a.s_bt = d.W; a.W = d.W;
  a.s_page = d.s_page; a.s_seq = 0; a.s_blk = d.s_page;
  a.s_pos = d.s_pos; a.s_head = d.s_head;
  a.sel = topk_idx; a.idx_is64 = d.idx_is64; a.K = d.K; a.valid = nullptr;
  a.s_sel_seq = 0; a.s_sel_t = d.s_ti_n; a.s_sel_h = d.s_ti_h; a.HI = d.Hkv;
  a.bias = bias; a.s_b_seq = 0; a.s_b_t = d.s_b_n; a.s_b_h = d.s_b_h;
  a.BS = d.block_size; a.LW = d.local_blocks * d.block_size;
  a.q_scale_log2 = d.sm_scale * kLog2e;
  a.s_q_seq = 0; a.s_q_t = d.s_qn; a.s_qh = d.s_qh;
  a.out = out; a.s_o_seq = 0; a.s_o_t = d.s_on; a.s_oh = d.s_oh;
  a.lse_out = lse_out; a.s_l_seq = 0; a.s_l_t = d.H;
  a.nsplit = d.nsplit; a.skip_local = d.skip_local ? 1 : 0; a.overlap = d.overlap ? 1 : 0;
  return attend_rows_launch(a, d.D, d.kv_dtype, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int srswa_lse_merge(const float* o_parts, const float* lse_parts, int64_t C, int64_t N,
                               int64_t H, int64_t D, int64_t s_o_part, int64_t s_l_part, void* out,
                               int out_dtype, float* lse_out, const srswa_peer* wait, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(out && C > 0 && N >= 0 && H > 0 && D > 0, SRSWA_EINVAL);
  SRSWA_CHECK_ARG((o_parts && lse_parts) || (wait && wait->ll), SRSWA_EINVAL);
  srswa_peer pw = {};
  if (wait) {
    SRSWA_CHECK_ARG(wait->regions && wait->own_region && wait->counter && wait->tickets && wait->world >= 1 &&
                        wait->world <= 32,
                    SRSWA_EINVAL);
    // LL: the parts are read from the region (o_parts / lse_parts unused), one per rank
    SRSWA_CHECK_ARG(!wait->ll || (C == wait->world && (N * H * D + N * H) * 8 <= wait->slot_bytes), SRSWA_EINVAL);
    pw = *wait;
  }
  if (s_o_part == 0) s_o_part = N * H * D;
  if (s_l_part == 0) s_l_part = N * H;
  SRSWA_CHECK_ARG(s_o_part >= N * H * D && s_l_part >= N * H, SRSWA_EINVAL);
  if (N == 0) return 0;
  SRSWA_CHECK_ARG(N * H < (1ll << 31), SRSWA_ETOOLARGE);
  // may launch while the kernel ahead (the attend making the parts) runs:
  // the kernel waits for it before reading anything
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(N * H), 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, lse_merge_kernel, o_parts, lse_parts, C, N * H, D, s_o_part,
                                           s_l_part, out, out_dtype, lse_out, pw);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
