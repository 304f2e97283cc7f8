// Internal interface of the row-streaming sparse attend (attend.cu).
#pragma once

#include <cuda_fp8.h>

#include "common.cuh"

namespace srswa {

constexpr int kAttendWarps = 4;
constexpr int kAttendThreads = kAttendWarps * 32;
constexpr int kAttendMaxSlots = 64;  // remote slots + window blocks per row

// Row n is (seq = n / rps, t = n % rps).  Its query position p is q_pos[n]
// (pos_mode 0), seq_lens[seq] - rps + t (pos_mode 1) or t (pos_mode 2).
// pos_mode 3 (varlen prefill): seq is the request r with cu_rows[r] <= n <
// cu_rows[r + 1], t = n (per-row strides, request strides 0) and
// p = prefix_lens[r] + n - cu_rows[r].
// A key block blk of sequence seq starts at element
//   block_table[seq * s_bt + blk] * s_page      (paged), or
//   seq * s_seq + blk * s_blk                   (contiguous),
// and key position i inside it / kv head h add i * s_pos + h * s_head.
// Workspace layout of the tensor-core gather forward (byte offsets); one
// definition shared by gather.cu (sizing) and gather_tc.cu (use).
// Internal status of the tensor-core entry points: the driver refused a
// tensor map (TMA descriptor) for these operands; the caller takes the
// CUDA-core kernels instead.  Never returned through the C ABI.
constexpr int kTcNoTensorMap = -1000;

struct TcLayout {
  size_t part_o, part_lse, count, cursor, work, totals, pair_t, pair_q, pair_bias, prow, lse, total;
  int64_t max_tiles;  // tiles of partial rows (128 each) per query head of an index head
};

// Paged K / V for the tensor-core forward (one sequence, B = 1): the caches
// are [num_pages, 64, Hkv, D] (strides in the gather descriptor's k / v
// fields), key block j is page pages[j], and query row t sits at position
// qoff + t.
struct TcPagedKV {
  int64_t num_pages;
  const int32_t* pages;
  int64_t s_pages;
  int64_t qoff;
};

struct AttendArgs {
  const void* q;
  const void* k;
  const void* v;
  int q_dtype, out_dtype;
  int64_t N, rps, H, Hkv;
  const int32_t* seq_lens;
  const int64_t* q_pos;
  const int32_t* seg;  // per row segment start (NULL = 0)
  int pos_mode;
  const int32_t* cu_rows;      // pos_mode 3: [nreq + 1] first row of each request
  const int32_t* prefix_lens;  // pos_mode 3: [nreq] cached tokens before the request's first row
  int64_t nreq;
  const int32_t* block_table;
  int64_t s_bt, W;
  int64_t s_page, s_seq, s_blk, s_pos, s_head;
  const void* sel;  // selection ids, offset seq*s_sel_seq + t*s_sel_t + hi*s_sel_h + slot
  int idx_is64;
  int64_t K, s_sel_seq, s_sel_t, s_sel_h, HI;
  const uint8_t* valid;  // same offsets as sel (NULL = every id >= 0 is used)
  const float* bias;     // offset seq*s_b_seq + t*s_b_t + hi*s_b_h + slot (NULL = 0)
  int64_t s_b_seq, s_b_t, s_b_h;
  int64_t BS, LW;
  float q_scale_log2;
  int64_t s_q_seq, s_q_t, s_qh;
  void* out;
  int64_t s_o_seq, s_o_t, s_oh;
  float* lse_out;  // natural log, offset seq*s_l_seq + t*s_l_t + h
  int64_t s_l_seq, s_l_t;
  int nsplit;      // CTAs per (row, head); 0 = choose
  int skip_local;  // 1: attend remote selections only
  int64_t row0;    // first row of this launch (rows row0 .. row0 + N - 1)
  int split_tail;  // the split was left open: a nearly empty last wave may be split
  int heads_inner; // grid (heads x splits, rows) instead of (rows x splits, heads)
  int overlap;     // window keys before pdl_wait (srswa_decode_desc.overlap)
  srswa_peer push; // regions != NULL: out / lse_out lie in this rank's own slot
                   // and every (row, head) result goes to that slot of every
                   // region; the storing CTAs are the exchange's producer units
  void* final_out; // LL push only: each storing CTA also waits for every rank's
                   // partial of its (row, head) and writes the log-sum-exp
                   // merge here ([N, H, D] contiguous, final_dtype)
  int final_dtype;
  float* final_lse;  // [N, H] natural log (optional)
};

template <int KVT>
__device__ __forceinline__ void unpack8(const uint4& r, float* f) {
  if (KVT == SRSWA_BF16) {
    f[0] = bf16_lo(r.x); f[1] = bf16_hi(r.x); f[2] = bf16_lo(r.y); f[3] = bf16_hi(r.y);
    f[4] = bf16_lo(r.z); f[5] = bf16_hi(r.z); f[6] = bf16_lo(r.w); f[7] = bf16_hi(r.w);
  } else {
    const __half2* hh = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __half22float2(hh[e]);
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
  }
}

// Two consecutive 16-bit elements (one 32-bit word) -> fp32 pair.
template <int KVT>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if (KVT == SRSWA_BF16) return make_float2(bf16_lo(w), bf16_hi(w));
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

constexpr bool kv_is_fp8(int kvt) { return kvt == SRSWA_F8E4M3 || kvt == SRSWA_F8E5M2; }

// 8 consecutive K / V elements at element offset off: one 16-byte load for
// 16-bit caches, one 8-byte load (in .x / .y) for fp8 caches.
template <int KVT>
__device__ __forceinline__ uint4 load_kv8(const void* p, int64_t off) {
  if constexpr (kv_is_fp8(KVT)) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(p) + off));
    return make_uint4(v.x, v.y, 0u, 0u);
  } else {
    return __ldg(reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(p) + off));
  }
}

// Elements (2w, 2w + 1) of 8 loaded by load_kv8, as fp32 (fp8 -> fp16 by the
// hardware conversion, exact, then fp32: the reference casts fp8 caches to
// the query dtype, which is exact too).
template <int KVT, int W>
__device__ __forceinline__ float2 kv_pair(const uint4& r) {
  if constexpr (kv_is_fp8(KVT)) {
    const uint32_t word = W < 2 ? r.x : r.y;
    const __nv_fp8x2_storage_t h = static_cast<__nv_fp8x2_storage_t>((W & 1) ? (word >> 16) : (word & 0xffffu));
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(h, KVT == SRSWA_F8E4M3 ? __NV_E4M3 : __NV_E5M2);
    return __half22float2(__half2(hr));
  } else {
    return unpack2<KVT>(W == 0 ? r.x : W == 1 ? r.y : W == 2 ? r.z : r.w);
  }
}

int attend_rows_launch(AttendArgs a, int64_t D, int kv_dtype, cudaStream_t st);

}  // namespace srswa
