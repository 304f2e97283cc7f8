// Peer-memory all-gather over NVLink for the split-KV decode (cfg5): every
// rank writes its payload with plain 16-byte stores straight into its slot of
// every peer's exchange region (CUDA IPC mappings), then releases a
// per-source flag there at system scope; a rank's consumers run after a
// bounded wait on the flags of its own region.  This replaces a library
// all-gather per exchange (two per layer of a decode step): the router's
// shard kernel pushes its keys itself, the key merge and the log-sum-exp
// merge wait themselves, and the attention partials take one push launch.
// All of it is capturable in a CUDA graph: the epoch each exchange waits for
// lives in device memory and advances on the device.
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

#include "peer.cuh"

namespace srswa {

constexpr int kPeerThreads = 256;

// CTA d copies the payload into slot `rank` of region d (d == rank: the
// local region); the last CTA to finish publishes the flags.  nbytes is a
// multiple of 16 and all addresses 16-byte aligned.
__global__ void __launch_bounds__(kPeerThreads) peer_push_kernel(const uint4* __restrict__ src, int64_t n16,
                                                                 const srswa_peer p) {
  uint4* dst = reinterpret_cast<uint4*>(peer_slot(p, blockIdx.x));
  for (int64_t i = threadIdx.x; i < n16; i += kPeerThreads) dst[i] = __ldg(src + i);
  __syncthreads();
  if (threadIdx.x == 0) peer_unit_done(p, gridDim.x);
}

// One thread: wait for every source's flag, then advance the counter.
__global__ void peer_wait_kernel(const srswa_peer p) {
  if (threadIdx.x == 0) peer_wait_all(p, 1u);
}

}  // namespace srswa

using namespace srswa;

static int check_peer(const srswa_peer* p) {
  if (!p || !p->regions || !p->own_region || !p->counter || !p->tickets) return SRSWA_EINVAL;
  if (p->ll) return SRSWA_EUNSUPPORTED;  // the generic push / wait move flagged payloads
  if (p->world < 1 || p->world > 32 || p->rank < 0 || p->rank >= p->world || p->slot_bytes < 0) return SRSWA_EINVAL;
  if (((reinterpret_cast<uintptr_t>(p->own_region) | static_cast<uintptr_t>(p->slot_bytes)) & 15) != 0)
    return SRSWA_EALIGN;
  return 0;
}

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

extern "C" int srswa_peer_push(const void* src, int64_t nbytes, const srswa_peer* peer, srswa_stream_t stream) {
  int rc = check_peer(peer);
  if (rc) return rc;
  SRSWA_CHECK_ARG(src && nbytes >= 0 && nbytes <= peer->slot_bytes, SRSWA_EINVAL);
  SRSWA_CHECK_ARG(((reinterpret_cast<uintptr_t>(src) | static_cast<uintptr_t>(nbytes)) & 15) == 0, SRSWA_EALIGN);
  peer_push_kernel<<<static_cast<unsigned>(peer->world), kPeerThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), nbytes / 16, *peer);
  return srswa_last_launch_status();
}

extern "C" int srswa_peer_allgather(const void* src, int64_t nbytes, const srswa_peer* peer, srswa_stream_t stream) {
  int rc = srswa_peer_push(src, nbytes, peer, stream);
  if (rc) return rc;
  peer_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*peer);
  return srswa_last_launch_status();
}
