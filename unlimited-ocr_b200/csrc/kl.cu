// DSA gather-KL distillation (training stage "sparse", one index head):
// per query row, KL(teacher || student) over the keys of the row's selected
// key blocks, and its gradients to the index q / k.
//
// Reference: select_and_kl_loss's gather branch and _kl_chunk_core
// (hf-model-code/_sparse_base_impl.py:3397-3450, 2071-2137).  A row's keys
// are the selected blocks' keys (a repeated block counts once) with
// seg <= j <= pos and j < max(pos - LW + 1, 0); the student logits are
// idx_q . idx_k[j], the teacher's per main head h are
// (q_main[h] . k_main[j, h / group]) * scaling, both rounded to bf16 first
// when the inputs are bf16 (the reference's bf16 matmul outputs); P_idx is a
// softmax over the row's keys, P the mean over heads of per-head softmaxes;
// kl = sum_j p_j (log max(p_j, 1e-12) - log p_idx_j).
//
// kl_row_kernel: one CTA per query row; a group of 8 lanes computes one dot
// product (each lane a contiguous 1/8 of the features), logits and
// probabilities live in shared memory (S * BS keys).  Its backward instance
// also writes the logit gradients ds_j = g (P p_idx_j - p_j) of the row
// (P = sum of p over the row's keys) and dQ = sum_j ds_j idx_k[j].
// kl_dk_kernel: one CTA per (batch, key block): dK of the block's keys, the
// sum over the rows that selected the block in row order (no atomics: the
// gradient is deterministic), walking the block's list of (row, slot) pairs
// built by the kl_pairs_* kernels.
// Memory-bound on gathered rows (the keys of a row are read by that row only).
#include "common.cuh"

namespace srswa {

constexpr int kKlThreads = 256;
constexpr int kKlMaxKeys = 2048;  // S * block_size per row
constexpr int kKlMaxDim = 128;

struct KlArgs {
  const void* iq;
  const void* ik;
  const void* qm;
  const void* km;
  int iq_dtype, ik_dtype, qm_dtype, km_dtype;
  int64_t s_iq_b, s_iq_c, s_ik_b, s_ik_s, s_qm_b, s_qm_c, s_qm_h, s_km_b, s_km_s, s_km_h;
  const int32_t* sel;
  const int64_t* pos;
  const int64_t* seg;
  int64_t B, C, Sk, H, Hkv, D, d, S, BS, LW;
  float scaling;
  int logits_bf16;
  float* kl;
  uint8_t* valid;
  const float* g;
  float* ds;   // [B, C, S * BS] logit gradients (backward)
  float* tp_out;       // forward: averaged teacher probabilities [B, C, S * BS] (optional)
  const float* tp_in;  // backward: those probabilities instead of recomputing the teacher
  float* dq;   // [B, C, d]
  float* dk;   // [B, Sk, d]
};

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// dot of an 8-lane group: this lane's nd features of q (registers) with the
// same features of the row at p (element offset off), reduced over the group
// (loops run to the compile-time bound with a predicate so that qv stays in
// registers: nd <= kKlMaxDim / 8 = 16)
__device__ __forceinline__ float group_dot(const float* qv, int nd, const void* p, int64_t off, int dtype) {
  float acc = 0.f;
  if (nd % 8 == 0 && dtype != SRSWA_F32) {
#pragma unroll
    for (int e = 0; e < kKlMaxDim / 8; e += 8) {
      if (e < nd) {
        float v[8];
        load8(p, off + e, dtype, v);
#pragma unroll
        for (int u = 0; u < 8; ++u) acc = fmaf(qv[e + u], v[u], acc);
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < kKlMaxDim / 8; ++e)
      if (e < nd) acc = fmaf(qv[e], load_elem(p, off + e, dtype), acc);
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  acc += __shfl_xor_sync(0xffffffffu, acc, 4);
  return acc;
}

__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < kKlThreads / 32; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
  return r;
}

template <bool BWD>
__global__ void __launch_bounds__(kKlThreads) kl_row_kernel(const KlArgs a) {
  __shared__ float sv[kKlMaxKeys], pa[kKlMaxKeys], tv[kKlMaxKeys];
  __shared__ int32_t s_lo[64], s_hi[64];
  __shared__ float red[kKlThreads / 32];
  __shared__ float dq_part[kKlThreads / 8][kKlMaxDim];
  const int64_t row = blockIdx.x;
  const int64_t b = row / a.C, c = row % a.C;
  const int tid = threadIdx.x;
  const int BS = static_cast<int>(a.BS), S = static_cast<int>(a.S), NK = S * BS;
  const int64_t pos = a.pos[row];
  const int64_t sg = a.seg ? a.seg[row] : 0;
  const int64_t ls = max(pos - (a.LW - 1), static_cast<int64_t>(0));
  // each slot's kept key range [lo, hi) (relative to its block); a repeat of
  // an earlier slot's block keeps nothing
  if (tid < S) {
    const int32_t blk = a.sel[row * a.S + tid];
    int lo = 0, hi = 0;
    bool dup = false;
    for (int u = 0; u < tid; ++u) dup |= a.sel[row * a.S + u] == blk;
    if (blk >= 0 && !dup) {
      const int64_t j0 = static_cast<int64_t>(blk) * a.BS;
      int64_t l = max(j0, sg), h = min(min(j0 + a.BS, a.Sk), min(pos + 1, ls));
      if (h > l) {
        lo = static_cast<int>(l - j0);
        hi = static_cast<int>(h - j0);
      }
    }
    s_lo[tid] = lo;
    s_hi[tid] = hi;
  }
  __syncthreads();
  const int grp = tid >> 3, u = tid & 7;
  const int nd = static_cast<int>(a.d) / 8, nD = static_cast<int>(a.D) / 8;
  auto kept = [&](int k) { const int s = k / BS, i = k - s * BS; return i >= s_lo[s] && i < s_hi[s]; };
  auto key_pos = [&](int k) {
    const int s = k / BS;
    return static_cast<int64_t>(a.sel[row * a.S + s]) * a.BS + (k - s * BS);
  };
  // ---- student logits ----
  float qv[kKlMaxDim / 8];
#pragma unroll
  for (int e = 0; e < kKlMaxDim / 8; ++e)
    qv[e] = e < nd ? load_elem(a.iq, b * a.s_iq_b + c * a.s_iq_c + u * nd + e, a.iq_dtype) : 0.f;
  float mx = -INFINITY;
  for (int k0 = 0; k0 < NK; k0 += kKlThreads / 8) {
    const int k = k0 + grp;
    const bool on = k < NK && kept(k);
    float dot = 0.f;
    if (__any_sync(0xffffffffu, on)) {  // groups of a warp share the shuffles
      const int64_t j = on ? key_pos(k) : 0;
      dot = group_dot(qv, nd, a.ik, b * a.s_ik_b + j * a.s_ik_s + u * nd, a.ik_dtype);
    }
    if (on && u == 0) {
      const float z = a.logits_bf16 ? round_bf16(dot) : dot;
      sv[k] = z;
      mx = fmaxf(mx, z);
    }
  }
  const float m_s = block_reduce(mx, red, true);
  float sum = 0.f;
  for (int k = tid; k < NK; k += kKlThreads) {
    pa[k] = 0.f;
    if (kept(k)) sum += expf(sv[k] - m_s);
  }
  const float l_s = block_reduce(sum, red, false);
  const bool any = m_s != -INFINITY;
  const float lse_s = any ? m_s + logf(l_s) : 0.f;
  // ---- teacher: per main head softmax over the same keys, averaged ----
  // (pa holds the sum over heads; with a saved teacher the backward reads
  // pa / H directly)
  const int64_t grp_h = a.H / a.Hkv;
  const bool saved = BWD && a.tp_in != nullptr;
  if (saved) {
    for (int k = tid; k < NK; k += kKlThreads) pa[k] = a.tp_in[row * NK + k];
    __syncthreads();
  }
  for (int64_t h = 0; h < (saved ? 0 : a.H); ++h) {
#pragma unroll
    for (int e = 0; e < kKlMaxDim / 8; ++e)
      qv[e] = e < nD ? load_elem(a.qm, b * a.s_qm_b + c * a.s_qm_c + h * a.s_qm_h + u * nD + e, a.qm_dtype) : 0.f;
    float mh = -INFINITY;
    for (int k0 = 0; k0 < NK; k0 += kKlThreads / 8) {
      const int k = k0 + grp;
      const bool on = k < NK && kept(k);
      float dot = 0.f;
      if (__any_sync(0xffffffffu, on)) {
        const int64_t j = on ? key_pos(k) : 0;
        dot = group_dot(qv, nD, a.km, b * a.s_km_b + j * a.s_km_s + (h / grp_h) * a.s_km_h + u * nD, a.km_dtype);
      }
      if (on && u == 0) {
        const float t = (a.logits_bf16 ? round_bf16(dot) : dot) * a.scaling;
        tv[k] = t;
        mh = fmaxf(mh, t);
      }
    }
    const float m_h = block_reduce(mh, red, true);
    float sh = 0.f;
    for (int k = tid; k < NK; k += kKlThreads)
      if (kept(k)) sh += expf(tv[k] - m_h);
    const float l_h = block_reduce(sh, red, false);
    const float inv = any ? 1.f / l_h : 0.f;
    for (int k = tid; k < NK; k += kKlThreads)
      if (kept(k)) pa[k] += expf(tv[k] - m_h) * inv;
    __syncthreads();
  }
  const float invH = 1.f / static_cast<float>(a.H);
  // averaged teacher probability of slot k: a rounded product (never fused
  // into a neighbouring add), so the saved and the recomputed value are the
  // same float and every use rounds alike
  auto pt = [&](int k) { return saved ? pa[k] : __fmul_rn(pa[k], invH); };
  if (!BWD && a.tp_out) {
    for (int k = tid; k < NK; k += kKlThreads) a.tp_out[row * NK + k] = kept(k) ? pt(k) : 0.f;
  }
  if (!BWD) {
    float acc = 0.f;
    for (int k = tid; k < NK; k += kKlThreads)
      if (kept(k)) {
        const float p = pt(k);
        acc += p * (logf(fmaxf(p, 1e-12f)) - (sv[k] - lse_s));
      }
    const float kl = block_reduce(acc, red, false);
    if (tid == 0) {
      a.kl[row] = any ? kl : 0.f;
      a.valid[row] = any ? 1 : 0;
    }
    return;
  }
  // ---- backward: logit gradients of the row, then dQ ----
  float ps = 0.f;
  for (int k = tid; k < NK; k += kKlThreads)
    if (kept(k)) ps += pt(k);
  const float P = block_reduce(ps, red, false);
  const float gr = a.g[row];
  for (int k = tid; k < NK; k += kKlThreads) {
    float dsk = 0.f;
    if (kept(k)) dsk = gr * (P * expf(sv[k] - lse_s) - pt(k));
    tv[k] = dsk;
    a.ds[row * NK + k] = dsk;
  }
  __syncthreads();
  float dacc[kKlMaxDim / 8];
#pragma unroll
  for (int e = 0; e < kKlMaxDim / 8; ++e) dacc[e] = 0.f;
  for (int k = grp; k < NK; k += kKlThreads / 8) {
    if (!kept(k)) continue;
    const float w = tv[k];
    const int64_t off = b * a.s_ik_b + key_pos(k) * a.s_ik_s + u * nd;
#pragma unroll
    for (int e = 0; e < kKlMaxDim / 8; ++e)
      if (e < nd) dacc[e] = fmaf(w, load_elem(a.ik, off + e, a.ik_dtype), dacc[e]);
  }
#pragma unroll
  for (int e = 0; e < kKlMaxDim / 8; ++e)
    if (e < nd) dq_part[grp][u * nd + e] = dacc[e];
  __syncthreads();
  for (int e = tid; e < a.d; e += kKlThreads) {
    float v = 0.f;
    for (int q = 0; q < kKlThreads / 8; ++q) v += dq_part[q][e];  // fixed order
    a.dq[row * a.d + e] = v;
  }
}

// dK of key block bk of batch b: the sum over the rows that selected the
// block (ascending row order) of ds[row, slot, i] * idx_q[row].
// ---- dK through per-block pair lists (row order, deterministic) ----
// kl_pairs_bitmap_kernel: bit (b, block, row) set when the row selects the
//   block (atomicOr: the bitmap does not depend on the order of the ORs);
// kl_pairs_count_kernel: one warp per list, its length;
// kl_pairs_scan_kernel: one CTA, exclusive offsets of the lists;
// kl_pairs_fill_kernel: one CTA per list, (row * S + first slot holding the
//   block) in row order;
// kl_dk_kernel: one CTA per (batch, key block) over its list, 16 pairs at a
//   time staged in shared memory; the sum runs in row order, as before.
constexpr int kKlPairGroup = 16;

__global__ void kl_pairs_bitmap_kernel(const KlArgs a, int64_t nbk, int64_t C32, uint32_t* bitmap) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // b * C + c
  if (row >= a.B * a.C) return;
  const int64_t b = row / a.C, c = row % a.C;
  const int32_t* sr = a.sel + row * a.S;
  for (int64_t s = 0; s < a.S; ++s) {
    const int32_t blk = sr[s];
    if (blk < 0 || blk >= nbk) continue;
    atomicOr(bitmap + (b * nbk + blk) * C32 + (c >> 5), 1u << (c & 31));
  }
}

__global__ void kl_pairs_count_kernel(int64_t nlists, int64_t C32, const uint32_t* bitmap, int32_t* count) {
  const int lane = threadIdx.x & 31;
  const int64_t l = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (l >= nlists) return;
  const uint32_t* w = bitmap + l * C32;
  int n = 0;
  for (int64_t i = lane; i < C32; i += 32) n += __popc(w[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  if (lane == 0) count[l] = n;
}

// exclusive scan of count[0, n) into offs (one CTA of 1024 threads: each
// thread a contiguous range, a CTA scan of the range sums)
__global__ void __launch_bounds__(1024) kl_pairs_scan_kernel(const int32_t* count, int64_t n, int32_t* offs) {
  __shared__ int32_t part[1024];
  const int tid = threadIdx.x;
  const int64_t per = (n + 1023) / 1024;
  const int64_t lo = tid * per, hi = min(n, lo + per);
  int32_t sum = 0;
  for (int64_t i = lo; i < hi; ++i) sum += count[i];
  part[tid] = sum;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    const int32_t v = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  int32_t run = part[tid] - sum;
  for (int64_t i = lo; i < hi; ++i) {
    offs[i] = run;
    run += count[i];
  }
}

__global__ void __launch_bounds__(256) kl_pairs_fill_kernel(const KlArgs a, int64_t nbk, int64_t C32,
                                                            const uint32_t* bitmap, const int32_t* offs,
                                                            int32_t* pairs) {
  __shared__ int32_t wcount[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t l = blockIdx.x;  // b * nbk + block
  const int64_t b = l / nbk, blk = l % nbk;
  const uint32_t* w = bitmap + l * C32;
  const int64_t per = (C32 + 7) / 8;
  const int64_t wlo = warp * per, whi = min(C32, wlo + per);
  int n = 0;
  for (int64_t i = wlo + lane; i < whi; i += 32) n += __popc(w[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
  if (lane == 0) wcount[warp] = n;
  __syncthreads();
  int64_t pos = offs[l];
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
      const int64_t c = (w0 + lane) * 32 + bit;
      const int32_t* sr = a.sel + (b * a.C + c) * a.S;
      int32_t slot = 0;
      for (int32_t s = static_cast<int32_t>(a.S) - 1; s >= 0; --s) slot = sr[s] == blk ? s : slot;  // first
      pairs[p++] = static_cast<int32_t>((c << 6) | slot);  // S <= 64
    }
    pos += __shfl_sync(0xffffffffu, incl, 31);
  }
}

template <bool kFast>  // kFast: d == 128 and BS == 64
__global__ void __launch_bounds__(kKlThreads) kl_dk_kernel(const KlArgs a, int64_t nbk, const int32_t* offs,
                                                          const int32_t* count, const int32_t* pairs) {
  __shared__ __align__(16) float s_ds[kKlPairGroup][64];
  __shared__ float s_iq[kKlPairGroup][kKlMaxDim];
  const int64_t bk = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x;
  const int BS = static_cast<int>(a.BS), d = static_cast<int>(a.d);
  const int NK = static_cast<int>(a.S) * BS;
  const int nel = BS * d;
  // element r of this thread: key ki[r], feature fe[r] of the block's
  // [BS, d] dK; kFast: feature tid % 128 and keys 32 (tid / 128) + r, so one
  // index-query value per pair and four 16-byte loads of its logit
  // gradients feed the 32 FMAs.  Registers only (r loops unrolled).
  float acc[32];
  int ki[32], fe[32];
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    acc[r] = 0.f;
    if (kFast) {
      ki[r] = (tid >> 7) * 32 + r;
      fe[r] = tid & 127;
    } else {
      const int el = tid + r * kKlThreads;
      ki[r] = el < nel ? el / d : -1;
      fe[r] = el < nel ? el - (el / d) * d : 0;
    }
  }
  const int64_t l = b * nbk + bk;
  const int32_t* lp = pairs + offs[l];
  const int np = count[l];
  for (int g0 = 0; g0 < np; g0 += kKlPairGroup) {
    const int ng = min(kKlPairGroup, np - g0);
    // stage the group's logit-gradient slices and index-query rows
    for (int e = tid; e < ng * BS; e += kKlThreads) {
      const int f = e / BS, i = e - f * BS;
      const int32_t pr = lp[g0 + f];
      const int64_t c = pr >> 6, slot = pr & 63;
      s_ds[f][i] = a.ds[(b * a.C + c) * NK + slot * BS + i];
    }
    for (int e = tid; e < ng * d; e += kKlThreads) {
      const int f = e / d, k = e - f * d;
      const int64_t c = lp[g0 + f] >> 6;
      s_iq[f][k] = load_elem(a.iq, b * a.s_iq_b + c * a.s_iq_c + k, a.iq_dtype);
    }
    __syncthreads();
    for (int f = 0; f < ng; ++f) {
      if (kFast) {
        const float q = s_iq[f][tid & 127];
        const float4* dsv = reinterpret_cast<const float4*>(&s_ds[f][(tid >> 7) * 32]);
#pragma unroll
        for (int r4 = 0; r4 < 8; ++r4) {
          const float4 v = dsv[r4];
          acc[4 * r4] = fmaf(v.x, q, acc[4 * r4]);
          acc[4 * r4 + 1] = fmaf(v.y, q, acc[4 * r4 + 1]);
          acc[4 * r4 + 2] = fmaf(v.z, q, acc[4 * r4 + 2]);
          acc[4 * r4 + 3] = fmaf(v.w, q, acc[4 * r4 + 3]);
        }
      } else {
#pragma unroll
        for (int r = 0; r < 32; ++r)
          if (ki[r] >= 0) acc[r] = fmaf(s_ds[f][ki[r]], s_iq[f][fe[r]], acc[r]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    if (ki[r] < 0) continue;
    const int64_t j = bk * a.BS + ki[r];
    if (j < a.Sk) a.dk[(b * a.Sk + j) * a.d + fe[r]] = acc[r];
  }
}

static int kl_args(const srswa_kl_desc* g, KlArgs& a) {
  if (!g) return SRSWA_EINVAL;
  if (g->B < 0 || g->C < 0 || g->Sk < 0 || g->H <= 0 || g->Hkv <= 0 || g->H % g->Hkv || g->S < 0 ||
      g->block_size <= 0 || g->local_window <= 0)
    return SRSWA_EINVAL;
  if (g->d % 8 || g->D % 8 || g->d > kKlMaxDim || g->D > kKlMaxDim || g->block_size > 64 || g->S > 64 ||
      g->S * g->block_size > kKlMaxKeys)
    return SRSWA_EUNSUPPORTED;
  a = {};
  a.iq_dtype = g->iq_dtype; a.ik_dtype = g->ik_dtype; a.qm_dtype = g->qm_dtype; a.km_dtype = g->km_dtype;
  a.s_iq_b = g->s_iq_b; a.s_iq_c = g->s_iq_c; a.s_ik_b = g->s_ik_b; a.s_ik_s = g->s_ik_s;
  a.s_qm_b = g->s_qm_b; a.s_qm_c = g->s_qm_c; a.s_qm_h = g->s_qm_h;
  a.s_km_b = g->s_km_b; a.s_km_s = g->s_km_s; a.s_km_h = g->s_km_h;
  a.B = g->B; a.C = g->C; a.Sk = g->Sk; a.H = g->H; a.Hkv = g->Hkv; a.D = g->D; a.d = g->d; a.S = g->S;
  a.BS = g->block_size; a.LW = g->local_window; a.scaling = g->scaling; a.logits_bf16 = g->logits_bf16;
  return 0;
}

}  // namespace srswa

using namespace srswa;

extern "C" int srswa_gather_kl_fwd_save(const srswa_kl_desc* g, const void* idx_q, const void* idx_k,
                                        const void* q_main, const void* k_main, const int32_t* sel,
                                        const int64_t* pos, const int64_t* seg, float* kl, uint8_t* valid,
                                        float* teacher, srswa_stream_t stream);

extern "C" int srswa_gather_kl_fwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                                   const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                                   float* kl, uint8_t* valid, srswa_stream_t stream) {
  return srswa_gather_kl_fwd_save(g, idx_q, idx_k, q_main, k_main, sel, pos, seg, kl, valid, nullptr, stream);
}

extern "C" int srswa_gather_kl_fwd_save(const srswa_kl_desc* g, const void* idx_q, const void* idx_k,
                                        const void* q_main, const void* k_main, const int32_t* sel,
                                        const int64_t* pos, const int64_t* seg, float* kl, uint8_t* valid,
                                        float* teacher, srswa_stream_t stream) {
  KlArgs a;
  int rc = kl_args(g, a);
  if (rc) return rc;
  if (g->B * g->C == 0) return 0;
  SRSWA_CHECK_ARG(idx_q && idx_k && q_main && k_main && pos && kl && valid && (g->S == 0 || sel), SRSWA_EINVAL);
  SRSWA_CHECK_ARG(g->B * g->C < (1ll << 31), SRSWA_ETOOLARGE);
  a.iq = idx_q; a.ik = idx_k; a.qm = q_main; a.km = k_main; a.sel = sel; a.pos = pos; a.seg = seg;
  a.kl = kl; a.valid = valid; a.tp_out = teacher;
  kl_row_kernel<false><<<static_cast<unsigned>(g->B * g->C), kKlThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return srswa_last_launch_status();
}

// backward workspace: logit gradients [B, C, S * BS] fp32, then the dK pair
// lists: bitmap [B, nbk, ceil(C / 32)], count and offsets [B, nbk], pairs
// [B, C, S] (each part 256-byte aligned)
struct KlBwdLayout {
  size_t ds, bitmap, count, offs, pairs, total;
  int64_t nbk, C32;
};
static size_t kl_align(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
static KlBwdLayout kl_bwd_layout(const srswa_kl_desc* g) {
  KlBwdLayout L = {};
  L.nbk = g->Sk > 0 ? (g->Sk + g->block_size - 1) / g->block_size : 0;
  L.C32 = (g->C + 31) / 32;
  size_t off = 0;
  L.ds = off; off += kl_align(static_cast<size_t>(g->B * g->C * g->S * g->block_size) * sizeof(float));
  L.bitmap = off; off += kl_align(static_cast<size_t>(g->B * L.nbk * L.C32) * 4);
  L.count = off; off += kl_align(static_cast<size_t>(g->B * L.nbk) * 4);
  L.offs = off; off += kl_align(static_cast<size_t>(g->B * L.nbk) * 4);
  L.pairs = off; off += kl_align(static_cast<size_t>(g->B * g->C * g->S) * 4);
  L.total = off;
  return L;
}

extern "C" size_t srswa_gather_kl_bwd_workspace_size(const srswa_kl_desc* g) {
  if (!g || g->B < 0 || g->C < 0 || g->S < 0 || g->block_size <= 0 || g->Sk < 0) return 0;
  return kl_bwd_layout(g).total;
}

static int kl_bwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                  const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                  const float* teacher, const float* grad, float* d_idx_q, float* d_idx_k, void* workspace,
                  size_t workspace_bytes, srswa_stream_t stream);

extern "C" int srswa_gather_kl_bwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                                   const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                                   const float* grad, float* d_idx_q, float* d_idx_k, void* workspace,
                                   size_t workspace_bytes, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(q_main && k_main, SRSWA_EINVAL);
  return kl_bwd(g, idx_q, idx_k, q_main, k_main, sel, pos, seg, nullptr, grad, d_idx_q, d_idx_k, workspace,
                workspace_bytes, stream);
}

extern "C" int srswa_gather_kl_bwd_saved(const srswa_kl_desc* g, const void* idx_q, const void* idx_k,
                                         const int32_t* sel, const int64_t* pos, const int64_t* seg,
                                         const float* teacher, const float* grad, float* d_idx_q, float* d_idx_k,
                                         void* workspace, size_t workspace_bytes, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(teacher, SRSWA_EINVAL);
  return kl_bwd(g, idx_q, idx_k, nullptr, nullptr, sel, pos, seg, teacher, grad, d_idx_q, d_idx_k, workspace,
                workspace_bytes, stream);
}

static int kl_bwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                  const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                  const float* teacher, const float* grad, float* d_idx_q, float* d_idx_k, void* workspace,
                  size_t workspace_bytes, srswa_stream_t stream) {
  KlArgs a;
  int rc = kl_args(g, a);
  if (rc) return rc;
  SRSWA_CHECK_ARG(idx_q && idx_k && pos && grad && d_idx_q && d_idx_k && (g->S == 0 || sel), SRSWA_EINVAL);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (g->B * g->Sk > 0 && (g->B * g->C == 0 || g->S == 0))  // no row selects anything: dK is zero
    SRSWA_CUDA_TRY(cudaMemsetAsync(d_idx_k, 0, static_cast<size_t>(g->B * g->Sk * g->d) * 4, st));
  if (g->B * g->C == 0) return 0;
  SRSWA_CHECK_ARG(workspace && workspace_bytes >= srswa_gather_kl_bwd_workspace_size(g), SRSWA_EWORKSPACE);
  SRSWA_CHECK_ARG(g->B * g->C < (1ll << 31) && g->B < 65536, SRSWA_ETOOLARGE);
  a.iq = idx_q; a.ik = idx_k; a.qm = q_main; a.km = k_main; a.sel = sel; a.pos = pos; a.seg = seg;
  const KlBwdLayout L = kl_bwd_layout(g);
  char* ws = static_cast<char*>(workspace);
  a.g = grad; a.ds = reinterpret_cast<float*>(ws + L.ds); a.dq = d_idx_q; a.dk = d_idx_k; a.tp_in = teacher;
  kl_row_kernel<true><<<static_cast<unsigned>(g->B * g->C), kKlThreads, 0, st>>>(a);
  SRSWA_CUDA_TRY(cudaGetLastError());
  if (g->S > 0 && g->Sk > 0) {
    const int64_t nlists = g->B * L.nbk;
    SRSWA_CHECK_ARG(L.nbk < 65536 && g->B * g->C * g->S < (1ll << 31), SRSWA_ETOOLARGE);
    uint32_t* bitmap = reinterpret_cast<uint32_t*>(ws + L.bitmap);
    int32_t* count = reinterpret_cast<int32_t*>(ws + L.count);
    int32_t* offs = reinterpret_cast<int32_t*>(ws + L.offs);
    int32_t* pairs = reinterpret_cast<int32_t*>(ws + L.pairs);
    SRSWA_CUDA_TRY(cudaMemsetAsync(bitmap, 0, static_cast<size_t>(nlists * L.C32) * 4, st));
    kl_pairs_bitmap_kernel<<<static_cast<unsigned>((g->B * g->C + 255) / 256), 256, 0, st>>>(a, L.nbk, L.C32,
                                                                                            bitmap);
    kl_pairs_count_kernel<<<static_cast<unsigned>((nlists + 7) / 8), 256, 0, st>>>(nlists, L.C32, bitmap, count);
    kl_pairs_scan_kernel<<<1, 1024, 0, st>>>(count, nlists, offs);
    kl_pairs_fill_kernel<<<static_cast<unsigned>(nlists), 256, 0, st>>>(a, L.nbk, L.C32, bitmap, offs, pairs);
    const dim3 grid(static_cast<unsigned>(L.nbk), static_cast<unsigned>(g->B));
    if (g->d == 128 && g->block_size == 64)
      kl_dk_kernel<true><<<grid, kKlThreads, 0, st>>>(a, L.nbk, offs, count, pairs);
    else
      kl_dk_kernel<false><<<grid, kKlThreads, 0, st>>>(a, L.nbk, offs, count, pairs);
  }
  return srswa_last_launch_status();
}
