// Peer-memory all-gather over NVLink for the split-KV decode (cfg5): every
// rank writes its payload with plain 16-byte stores straight into its slot of
// every peer's exchange region (CUDA IPC mappings), then releases a
// per-source flag there at system scope; a rank's consumers run after a
// bounded wait on the flags of its own region.  This replaces a library
// all-gather per exchange (two per layer of a decode step) with one push and
// one wait launch, both capturable in a CUDA graph: the epoch each exchange
// waits for lives in device memory and advances on the device.
//
// Region layout (one per rank, all ranks the same size):
//   [0, 8 * world)            flags: uint64 epoch last published by source r
//   [256, 256 + world * slot) data:  slot r = the payload of source rank r
//
// Ordering argument for reusing one region across exchanges: a rank pushes
// exchange e+1 only after its own wait for exchange e returned, and that wait
// needs every peer's push of e, which each peer issues only after its
// consumers of e-1 (stream order).  Two regions used alternately (router keys,
// then attention partials) therefore never overwrite data a peer still reads.
//
// No TMA, no multicast, no library kernel touches peer memory: peer bytes are
// moved only by the plain stores of peer_push_kernel.
#include <cstring>

#include "common.cuh"

namespace srswa {

constexpr int kPeerThreads = 256;
constexpr int64_t kPeerHeader = 256;  // flag bytes reserved at the head of a region (world <= 32)
// bound of a wait (wall clock, %globaltimer ns)
constexpr uint64_t kPeerWaitNs = 2000000000ull;

__device__ __forceinline__ uint64_t peer_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// CTA d copies the payload into slot `rank` of peer d's region (d == rank:
// the local region), then publishes epoch = *counter + 1 in that region's
// flag `rank`.  nbytes is a multiple of 16 and all addresses 16-byte aligned.
__global__ void __launch_bounds__(kPeerThreads) peer_push_kernel(const uint4* __restrict__ src, int64_t n16,
                                                                 char* const* __restrict__ regions, int64_t slot,
                                                                 int rank, const uint64_t* __restrict__ counter) {
  const int d = blockIdx.x;
  char* region = regions[d];
  uint4* dst = reinterpret_cast<uint4*>(region + kPeerHeader + static_cast<int64_t>(rank) * slot);
  for (int64_t i = threadIdx.x; i < n16; i += kPeerThreads) dst[i] = __ldg(src + i);
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t epoch = *counter + 1;
    __threadfence_system();  // the payload stores above (all threads, via the barrier) before the flag
    uint64_t* flag = reinterpret_cast<uint64_t*>(region) + rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(epoch) : "memory");
  }
}

// One warp: lane r waits until source r has published epoch *counter + 1 in
// this rank's region (acquire, system scope), bounded in wall-clock time; on
// expiry it records `code` in *status.  Then the counter advances.
__global__ void peer_wait_kernel(const char* region, int world, uint64_t* counter, int* status, int code) {
  const int r = threadIdx.x;
  const uint64_t epoch = *counter + 1;
  bool ok = true;
  if (r < world) {
    const uint64_t* flag = reinterpret_cast<const uint64_t*>(region) + r;
    const uint64_t t0 = peer_now();
    for (;;) {
      uint64_t v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
      if (v >= epoch) break;
      if (peer_now() - t0 > kPeerWaitNs) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  const bool all_ok = __all_sync(0xffffffffu, ok);
  if (r == 0) {
    if (!all_ok && status) atomicCAS(status, 0, code);
    *counter = epoch;  // advance even on expiry: the next exchange does not wait for a stale epoch
  }
}

}  // namespace srswa

using namespace srswa;

extern "C" int srswa_peer_region_size(int64_t world, int64_t slot_bytes, size_t* out) {
  if (!out || world < 1 || world > 32 || slot_bytes < 0 || (slot_bytes & 15)) return SRSWA_EINVAL;
  *out = static_cast<size_t>(kPeerHeader + world * slot_bytes);
  return 0;
}

extern "C" int srswa_peer_region_alloc(size_t bytes, void** out) {
  if (!out || bytes == 0) return SRSWA_EINVAL;
  void* p = nullptr;
  SRSWA_CUDA_TRY(cudaMalloc(&p, bytes));  // a whole allocation: its IPC handle maps exactly this region
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return static_cast<int>(e);
  }
  *out = p;
  return 0;
}

extern "C" int srswa_peer_region_free(void* p) {
  if (!p) return SRSWA_EINVAL;
  SRSWA_CUDA_TRY(cudaFree(p));
  return 0;
}

extern "C" int srswa_peer_ipc_handle(const void* region, void* handle64) {
  if (!region || !handle64) return SRSWA_EINVAL;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  SRSWA_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(region)));
  memcpy(handle64, &h, sizeof(h));
  return 0;
}

extern "C" int srswa_peer_ipc_open(const void* handle64, void** out) {
  if (!handle64 || !out) return SRSWA_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  SRSWA_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *out = p;
  return 0;
}

extern "C" int srswa_peer_ipc_close(void* mapped) {
  if (!mapped) return SRSWA_EINVAL;
  SRSWA_CUDA_TRY(cudaIpcCloseMemHandle(mapped));
  return 0;
}

extern "C" int srswa_peer_allgather(const void* src, int64_t nbytes, void* const* regions, const void* own_region,
                                    int64_t slot_bytes, int64_t rank, int64_t world, uint64_t* counter,
                                    int* status, srswa_stream_t stream) {
  SRSWA_CHECK_ARG(src && regions && own_region && counter && world >= 1 && world <= 32 && rank >= 0 &&
                      rank < world && nbytes >= 0 && nbytes <= slot_bytes,
                  SRSWA_EINVAL);
  SRSWA_CHECK_ARG(((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(own_region) |
                    static_cast<uintptr_t>(nbytes) | static_cast<uintptr_t>(slot_bytes)) & 15) == 0,
                  SRSWA_EALIGN);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  peer_push_kernel<<<static_cast<unsigned>(world), kPeerThreads, 0, st>>>(
      static_cast<const uint4*>(src), nbytes / 16, reinterpret_cast<char* const*>(regions), slot_bytes,
      static_cast<int>(rank), counter);
  SRSWA_CUDA_TRY(cudaGetLastError());
  peer_wait_kernel<<<1, 32, 0, st>>>(static_cast<const char*>(own_region), static_cast<int>(world), counter, status,
                                     501);
  return srswa_last_launch_status();
}
