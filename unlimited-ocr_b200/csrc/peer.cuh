// Device side of the peer-memory exchange (srswa_peer, include/srswa.h):
// producers put their payload into slot `rank` of every region with plain
// stores and the last producer unit releases the flags; consumers acquire
// every source's flag (bounded wait) and the last consumer CTA advances the
// region's counter.  Used inside the router / merge kernels and by the
// stand-alone push / wait kernels.
#pragma once

#include "common.cuh"

namespace srswa {

constexpr int64_t kPeerHeader = 256;             // flag bytes at the head of a region (world <= 32)
constexpr uint64_t kPeerWaitNs = 2000000000ull;  // bound of a wait (wall clock, %globaltimer ns)
constexpr int kPeerExpired = 501;                // status code of an expired wait

__device__ __forceinline__ uint64_t peer_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ char* peer_slot(const srswa_peer& p, int d) {
  return static_cast<char*>(p.regions[d]) + kPeerHeader + p.rank * p.slot_bytes;
}

// 8 payload bytes at byte offset off of this rank's slot, in every region
__device__ __forceinline__ void peer_put8(const srswa_peer& p, int64_t off, unsigned long long v) {
  for (int d = 0; d < static_cast<int>(p.world); ++d)
    *reinterpret_cast<unsigned long long*>(peer_slot(p, d) + off) = v;
}

// Thread 0 of a producer unit, after the unit's stores (and a barrier among
// the unit's threads): the last of nunits units releases flag `rank` in
// every region with epoch *counter + 1.
__device__ __forceinline__ void peer_unit_done(const srswa_peer& p, unsigned nunits) {
  __threadfence_system();
  const unsigned t = atomicAdd(p.tickets, 1u);
  if (t != nunits - 1) return;
  __threadfence_system();
  const uint64_t epoch = *p.counter + 1;
  for (int d = 0; d < static_cast<int>(p.world); ++d) {
    uint64_t* flag = static_cast<uint64_t*>(p.regions[d]) + p.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(epoch) : "memory");
  }
  *p.tickets = 0u;
}

// Thread 0 of each consumer CTA: acquire every source's flag at epoch
// *counter + 1 (bounded; on expiry status = 501 and false), then the last of
// nunits consumer CTAs advances the counter.  Callers follow it with a
// barrier before reading the slots.
__device__ __forceinline__ bool peer_wait_all(const srswa_peer& p, unsigned nunits) {
  const uint64_t epoch = *p.counter + 1;
  bool ok = true;
  const uint64_t* flags = static_cast<const uint64_t*>(p.own_region);
  for (int r = 0; r < static_cast<int>(p.world) && ok; ++r) {
    const uint64_t t0 = peer_now();
    for (;;) {
      uint64_t v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flags + r) : "memory");
      if (v >= epoch) break;
      if (peer_now() - t0 > kPeerWaitNs) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
  }
  if (!ok && p.status) atomicCAS(reinterpret_cast<int*>(p.status), 0, kPeerExpired);
  const unsigned t = atomicAdd(p.tickets + 1, 1u);
  if (t == nunits - 1) {
    *p.counter = epoch;
    p.tickets[1] = 0u;
  }
  return ok;
}

}  // namespace srswa
