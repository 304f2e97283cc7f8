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

// ---- LL protocol (srswa_peer.ll = 1) ----
// A 32-bit payload word travels with the exchange's epoch in one aligned
// 8-byte store (single-copy atomic), so a consumer that reads the epoch has
// the payload too: no fence, no flag, no producer ticket.
__device__ __forceinline__ uint32_t ll_epoch(const srswa_peer& p) {
  return static_cast<uint32_t>(*p.counter + 1);
}

// word k of this rank's slot, in every region
__device__ __forceinline__ void ll_put(const srswa_peer& p, int64_t k, uint32_t epoch, uint32_t v) {
  const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | v;
  for (int d = 0; d < static_cast<int>(p.world); ++d) {
    unsigned long long* a = reinterpret_cast<unsigned long long*>(peer_slot(p, d)) + k;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(w) : "memory");
  }
}

// word k of source rank r's slot in this rank's region, once it carries
// `epoch` (bounded wait; on expiry ok = false, status 501, returns 0)
__device__ __forceinline__ uint32_t ll_get(const srswa_peer& p, int r, int64_t k, uint32_t epoch, bool& ok) {
  const unsigned long long* a = reinterpret_cast<const unsigned long long*>(
                                    static_cast<const char*>(p.own_region) + kPeerHeader + r * p.slot_bytes) + k;
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
  if (static_cast<uint32_t>(w >> 32) == epoch) return static_cast<uint32_t>(w);
  if (!ok) return 0u;  // this thread already gave up on a peer: no second wait
  const uint64_t t0 = peer_now();
  for (;;) {
    __nanosleep(20);
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(a) : "memory");
    if (static_cast<uint32_t>(w >> 32) == epoch) return static_cast<uint32_t>(w);
    if (peer_now() - t0 > kPeerWaitNs) {
      if (ok && p.status) atomicCAS(reinterpret_cast<int*>(p.status), 0, kPeerExpired);
      ok = false;
      return 0u;
    }
  }
}

// one consumer unit has read everything it needs: the last of nunits
// advances the counter (the next exchange's epoch)
__device__ __forceinline__ void ll_consumer_done(const srswa_peer& p, unsigned nunits) {
  const unsigned t = atomicAdd(p.tickets + 1, 1u);
  if (t == nunits - 1) {
    *p.counter = *p.counter + 1;
    p.tickets[1] = 0u;
  }
}

}  // namespace srswa
