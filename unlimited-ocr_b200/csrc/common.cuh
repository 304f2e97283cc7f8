// Shared device/host helpers for the SR-SWA sm_100a library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "srswa.h"

namespace srswa {

// Finite sentinels of the reference path (hf-model-code/dash_attention.py:740-754,
// modeling_deepseekv2.py:65).
constexpr float kScoreNeg = -1.0e9f;
constexpr float kMaskNeg = -1.0e9f;
constexpr float kEntmaxNeg = -1.0e4f;
constexpr float kActClamp = 1.0e4f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// programmatic dependent launch (sm_90+).  A kernel launched with the
// attribute cudaLaunchAttributeProgrammaticStreamSerialization may start once
// every CTA of the kernel before it on the stream has called
// pdl_launch_dependents (or exited); pdl_wait then blocks until that kernel
// has completed and its writes are visible.  Both are no-ops for a kernel
// launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// element loads (fp32 / bf16 / fp16 selected by a runtime dtype code)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dtype) {
  if (dtype == SRSWA_F32) return __ldg(reinterpret_cast<const float*>(p) + i);
  if (dtype == SRSWA_BF16) {
    unsigned short u = __ldg(reinterpret_cast<const unsigned short*>(p) + i);
    return __uint_as_float(static_cast<uint32_t>(u) << 16);
  }
  return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
}

// 8 consecutive elements starting at element i (16 B aligned for 16-bit types,
// 32 B for fp32) -> fp32.
__device__ __forceinline__ void load8(const void* p, int64_t i, int dtype, float* o) {
  if (dtype == SRSWA_BF16) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned short*>(p) + i));
    o[0] = bf16_lo(u.x); o[1] = bf16_hi(u.x); o[2] = bf16_lo(u.y); o[3] = bf16_hi(u.y);
    o[4] = bf16_lo(u.z); o[5] = bf16_hi(u.z); o[6] = bf16_lo(u.w); o[7] = bf16_hi(u.w);
  } else if (dtype == SRSWA_F32) {
    const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    float4 a = __ldg(f), b = __ldg(f + 1);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p) + i));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __half22float2(h[j]);
      o[2 * j] = f.x; o[2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void store_elem(void* p, int64_t i, int dtype, float v) {
  if (dtype == SRSWA_F32) reinterpret_cast<float*>(p)[i] = v;
  else if (dtype == SRSWA_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
}

__device__ __forceinline__ void store8(void* p, int64_t i, int dtype, const float* v) {
  if (dtype == SRSWA_F32) {
    float4* f = reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i);
    f[0] = make_float4(v[0], v[1], v[2], v[3]);
    f[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else if (dtype == SRSWA_BF16) {
    uint4 u;
    __nv_bfloat162 t[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
    u = *reinterpret_cast<uint4*>(t);
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p) + i) = u;
  } else {
    __half2 t[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) t[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(p) + i) = *reinterpret_cast<uint4*>(t);
  }
}

__device__ __forceinline__ int64_t load_index(const void* p, int64_t i, int is64) {
  return is64 ? __ldg(reinterpret_cast<const long long*>(p) + i)
              : static_cast<int64_t>(__ldg(reinterpret_cast<const int*>(p) + i));
}

// ---------------------------------------------------------------------------
// warp reductions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Transposed butterfly reduction of 8 per-lane partial sums over groups of
// LPK consecutive lanes (LPK in {8, 16, 32}).  On return lane l holds the full
// sum of value index i = 4*b(LPK/2) + 2*b(LPK/4) + b(LPK/8), where b(m) is
// ((l & m) != 0); with LPK > 8 the remaining levels are plain sums, so lanes
// differing only in the low bits hold the same total.  Uses 7 shuffles for
// LPK = 8 (4+2+1) plus one per extra level, instead of 8*log2(LPK).
template <int LPK>
__device__ __forceinline__ float transpose_reduce8(float (&v)[8], int lane) {
  constexpr int m1 = LPK / 2, m2 = LPK / 4, m3 = LPK / 8;
  float a[4];
  {
    const bool up = (lane & m1) != 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float send = up ? v[j] : v[j + 4];
      float keep = up ? v[j + 4] : v[j];
      a[j] = keep + __shfl_xor_sync(0xffffffffu, send, m1);
    }
  }
  float b[2];
  {
    const bool up = (lane & m2) != 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float send = up ? a[j] : a[j + 2];
      float keep = up ? a[j + 2] : a[j];
      b[j] = keep + __shfl_xor_sync(0xffffffffu, send, m2);
    }
  }
  float c;
  {
    const bool up = (lane & m3) != 0;
    float send = up ? b[0] : b[1];
    float keep = up ? b[1] : b[0];
    c = keep + __shfl_xor_sync(0xffffffffu, send, m3);
  }
#pragma unroll
  for (int m = LPK / 16; m > 0; m >>= 1) c += __shfl_xor_sync(0xffffffffu, c, m);
  return c;
}

// lane (within an LPK-group) that holds value index i after transpose_reduce8
template <int LPK>
__device__ __forceinline__ int transpose_owner(int i) {
  return ((i >> 2) & 1) * (LPK / 2) + ((i >> 1) & 1) * (LPK / 4) + (i & 1) * (LPK / 8);
}

template <typename T>
__host__ __device__ __forceinline__ T cdiv(T a, T b) { return (a + b - 1) / b; }

}  // namespace srswa

// Host-side status helpers
#define SRSWA_CHECK_ARG(cond, code) \
  do {                              \
    if (!(cond)) return (code);     \
  } while (0)

#define SRSWA_CUDA_TRY(expr)                        \
  do {                                              \
    cudaError_t _e = (expr);                        \
    if (_e != cudaSuccess) return static_cast<int>(_e); \
  } while (0)

static inline int srswa_last_launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
