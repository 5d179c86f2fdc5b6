// Device side of the fused tensor-parallel collectives (see tp.cu): flagged-word transfers.
//
// Every value crosses NVLink as one 8-byte word, the 32-bit payload in the low half and the
// step's flag (a counter that every rank advances in lockstep) in the high half, written with a
// single 8-byte store. An aligned 8-byte store is seen whole or not at all, so the reader polls
// the word itself: when the flag matches, the payload is this step's. No fence, no counter and
// no second round trip: the transfer costs one NVLink one-way latency.
#pragma once
#include "common.cuh"
#include "api.h"

namespace hk {

constexpr unsigned long long kTpWaitNs = 1000000000ull;  // default bound of a peer wait: 1 s, then HK_ERR_PEER_TIMEOUT

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void ll_store(unsigned long long* p, uint32_t v, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v), "r"(flag) : "memory");
}

__device__ __forceinline__ uint2 ll_load(const unsigned long long* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// Re-polls `w` (already loaded once) until its flag matches; gives up at `deadline` and clears
// `ok` (later waits of the same thread then return at once with what they hold).
__device__ __forceinline__ void ll_settle(uint2& w, const unsigned long long* p, uint32_t flag,
                                         unsigned long long deadline, bool& ok) {
  while (w.y != flag && ok) {
    if (global_ns() > deadline) {
      ok = false;
      break;
    }
    w = ll_load(p);
  }
}

}  // namespace hk
