// Named host ranges for timeline profilers: NVTX push/pop (header-only NVTX v3 from the CUDA
// toolkit; without an attached tool each call is a cheap no-op). Compiled to no-ops when the
// NVTX headers are absent.
//
// Parity: crates/hawking-core/src/metal/physical_signpost.c (os_signpost begin/end intervals),
// crates/hawking-core/src/metal/mod.rs:177-231 (PhysicalTraceGuard).
#pragma once
#include <string>

namespace hk {

bool trace_available();
void trace_push(const std::string& name);
void trace_pop();

}  // namespace hk
