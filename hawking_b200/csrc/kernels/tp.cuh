// Device side of the fused tensor-parallel collectives (see tp.cu).
#pragma once
#include "common.cuh"
#include "api.h"

namespace hk {

// Producer side, called by every thread of a CTA after its stores to the peers' receive regions:
// one system-scope release, then one arrival on every rank's counter.
__device__ __forceinline__ void tp_signal(const TpSite& t) {
  __threadfence_system();  // every thread orders its own peer stores before the arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int p = 0; p < t.n; ++p) atomicAdd_system(t.counters[p], 1ull);
  }
}

}  // namespace hk
