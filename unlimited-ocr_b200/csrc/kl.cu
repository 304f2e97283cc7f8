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
// gradient is deterministic).
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
  float* dq;   // [B, C, d]
  float* dk;   // [B, Sk, d]
};

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// dot of an 8-lane group: this lane's nd features of q (registers) with the
// same features of the row at p (element offset off), reduced over the group
__device__ __forceinline__ float group_dot(const float* qv, int nd, const void* p, int64_t off, int dtype) {
  float acc = 0.f;
  if (nd % 8 == 0 && dtype != SRSWA_F32) {
    for (int e = 0; e < nd; e += 8) {
      float v[8];
      load8(p, off + e, dtype, v);
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = fmaf(qv[e + u], v[u], acc);
    }
  } else {
    for (int e = 0; e < nd; ++e) acc = fmaf(qv[e], load_elem(p, off + e, dtype), acc);
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
  for (int e = 0; e < nd; ++e) qv[e] = load_elem(a.iq, b * a.s_iq_b + c * a.s_iq_c + u * nd + e, a.iq_dtype);
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
  const int64_t grp_h = a.H / a.Hkv;
  for (int64_t h = 0; h < a.H; ++h) {
    for (int e = 0; e < nD; ++e)
      qv[e] = load_elem(a.qm, b * a.s_qm_b + c * a.s_qm_c + h * a.s_qm_h + u * nD + e, a.qm_dtype);
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
  if (!BWD) {
    float acc = 0.f;
    for (int k = tid; k < NK; k += kKlThreads)
      if (kept(k)) {
        const float p = pa[k] * invH;
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
    if (kept(k)) ps += pa[k] * invH;
  const float P = block_reduce(ps, red, false);
  const float gr = a.g[row];
  for (int k = tid; k < NK; k += kKlThreads) {
    float dsk = 0.f;
    if (kept(k)) dsk = gr * (P * expf(sv[k] - lse_s) - pa[k] * invH);
    tv[k] = dsk;
    a.ds[row * NK + k] = dsk;
  }
  __syncthreads();
  float dacc[kKlMaxDim / 8];
  for (int e = 0; e < nd; ++e) dacc[e] = 0.f;
  for (int k = grp; k < NK; k += kKlThreads / 8) {
    if (!kept(k)) continue;
    const float w = tv[k];
    const int64_t off = b * a.s_ik_b + key_pos(k) * a.s_ik_s + u * nd;
    for (int e = 0; e < nd; ++e) dacc[e] = fmaf(w, load_elem(a.ik, off + e, a.ik_dtype), dacc[e]);
  }
  for (int e = 0; e < nd; ++e) dq_part[grp][u * nd + e] = dacc[e];
  __syncthreads();
  for (int e = tid; e < a.d; e += kKlThreads) {
    float v = 0.f;
    for (int q = 0; q < kKlThreads / 8; ++q) v += dq_part[q][e];  // fixed order
    a.dq[row * a.d + e] = v;
  }
}

// dK of key block bk of batch b: the sum over the rows that selected the
// block (ascending row order) of ds[row, slot, i] * idx_q[row].
__global__ void __launch_bounds__(kKlThreads) kl_dk_kernel(const KlArgs a) {
  __shared__ int32_t rows[kKlThreads], slots[kKlThreads];
  __shared__ int n_found;
  const int64_t bk = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x;
  const int BS = static_cast<int>(a.BS), d = static_cast<int>(a.d);
  const int NK = static_cast<int>(a.S) * BS;
  const int nel = BS * d;
  const int per = (nel + kKlThreads - 1) / kKlThreads;  // <= 32 (BS <= 64, d <= 128)
  float acc[32];
  for (int r = 0; r < 32; ++r) acc[r] = 0.f;
  for (int64_t c0 = 0; c0 < a.C; c0 += kKlThreads) {
    if (tid == 0) n_found = 0;
    __syncthreads();
    const int64_t c = c0 + tid;
    int hit = -1;
    if (c < a.C) {
      const int32_t* sr = a.sel + (b * a.C + c) * a.S;
      for (int s = 0; s < a.S; ++s)
        if (sr[s] == bk) {
          hit = s;  // the first slot: a repeat keeps no keys (ds = 0)
          break;
        }
    }
    // compact the hits in row order (warp ballots, then warps in order)
    const unsigned m = __ballot_sync(0xffffffffu, hit >= 0);
    __shared__ int warp_cnt[kKlThreads / 32];
    if ((tid & 31) == 0) warp_cnt[tid >> 5] = __popc(m);
    __syncthreads();
    int base = 0;
    for (int w = 0; w < (tid >> 5); ++w) base += warp_cnt[w];
    if (hit >= 0) {
      const int at = base + __popc(m & ((1u << (tid & 31)) - 1u));
      rows[at] = static_cast<int32_t>(c);
      slots[at] = hit;
    }
    if (tid == kKlThreads - 1) {
      int t = 0;
      for (int w = 0; w < kKlThreads / 32; ++w) t += warp_cnt[w];
      n_found = t;
    }
    __syncthreads();
    const int nf = n_found;
    for (int f = 0; f < nf; ++f) {
      const int64_t rr = b * a.C + rows[f];
      const float* dsr = a.ds + rr * NK + static_cast<int64_t>(slots[f]) * BS;
      for (int r = 0; r < per; ++r) {
        const int el = tid + r * kKlThreads;
        if (el < nel) {
          const int i = el / d, e = el - i * d;
          acc[r] = fmaf(dsr[i], load_elem(a.iq, b * a.s_iq_b + rows[f] * a.s_iq_c + e, a.iq_dtype), acc[r]);
        }
      }
    }
    __syncthreads();
  }
  for (int r = 0; r < per; ++r) {
    const int el = tid + r * kKlThreads;
    if (el < nel) {
      const int i = el / d, e = el - i * d;
      const int64_t j = bk * a.BS + i;
      if (j < a.Sk) a.dk[(b * a.Sk + j) * a.d + e] = acc[r];
    }
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

extern "C" int srswa_gather_kl_fwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                                   const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                                   float* kl, uint8_t* valid, srswa_stream_t stream) {
  KlArgs a;
  int rc = kl_args(g, a);
  if (rc) return rc;
  if (g->B * g->C == 0) return 0;
  SRSWA_CHECK_ARG(idx_q && idx_k && q_main && k_main && pos && kl && valid && (g->S == 0 || sel), SRSWA_EINVAL);
  SRSWA_CHECK_ARG(g->B * g->C < (1ll << 31), SRSWA_ETOOLARGE);
  a.iq = idx_q; a.ik = idx_k; a.qm = q_main; a.km = k_main; a.sel = sel; a.pos = pos; a.seg = seg;
  a.kl = kl; a.valid = valid;
  kl_row_kernel<false><<<static_cast<unsigned>(g->B * g->C), kKlThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return srswa_last_launch_status();
}

extern "C" size_t srswa_gather_kl_bwd_workspace_size(const srswa_kl_desc* g) {
  if (!g || g->B < 0 || g->C < 0 || g->S < 0 || g->block_size <= 0) return 0;
  return static_cast<size_t>(g->B * g->C * g->S * g->block_size) * sizeof(float);
}

extern "C" int srswa_gather_kl_bwd(const srswa_kl_desc* g, const void* idx_q, const void* idx_k, const void* q_main,
                                   const void* k_main, const int32_t* sel, const int64_t* pos, const int64_t* seg,
                                   const float* grad, float* d_idx_q, float* d_idx_k, void* workspace,
                                   size_t workspace_bytes, srswa_stream_t stream) {
  KlArgs a;
  int rc = kl_args(g, a);
  if (rc) return rc;
  SRSWA_CHECK_ARG(idx_q && idx_k && q_main && k_main && pos && grad && d_idx_q && d_idx_k && (g->S == 0 || sel),
                  SRSWA_EINVAL);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (g->B * g->Sk > 0 && (g->B * g->C == 0 || g->S == 0))  // no row selects anything: dK is zero
    SRSWA_CUDA_TRY(cudaMemsetAsync(d_idx_k, 0, static_cast<size_t>(g->B * g->Sk * g->d) * 4, st));
  if (g->B * g->C == 0) return 0;
  SRSWA_CHECK_ARG(workspace && workspace_bytes >= srswa_gather_kl_bwd_workspace_size(g), SRSWA_EWORKSPACE);
  SRSWA_CHECK_ARG(g->B * g->C < (1ll << 31) && g->B < 65536, SRSWA_ETOOLARGE);
  a.iq = idx_q; a.ik = idx_k; a.qm = q_main; a.km = k_main; a.sel = sel; a.pos = pos; a.seg = seg;
  a.g = grad; a.ds = static_cast<float*>(workspace); a.dq = d_idx_q; a.dk = d_idx_k;
  kl_row_kernel<true><<<static_cast<unsigned>(g->B * g->C), kKlThreads, 0, st>>>(a);
  SRSWA_CUDA_TRY(cudaGetLastError());
  if (g->S > 0 && g->Sk > 0) {
    const int64_t nbk = (g->Sk + g->block_size - 1) / g->block_size;
    kl_dk_kernel<<<dim3(static_cast<unsigned>(nbk), static_cast<unsigned>(g->B)), kKlThreads, 0, st>>>(a);
  }
  return srswa_last_launch_status();
}
