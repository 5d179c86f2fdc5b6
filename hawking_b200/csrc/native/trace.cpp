#include "trace.h"

#if defined(__has_include)
#if __has_include(<nvtx3/nvToolsExt.h>)
#include <nvtx3/nvToolsExt.h>
#define HK_HAVE_NVTX 1
#endif
#endif

namespace hk {

#ifdef HK_HAVE_NVTX
bool trace_available() { return true; }
void trace_push(const std::string& name) { nvtxRangePushA(name.c_str()); }
void trace_pop() { nvtxRangePop(); }
#else
bool trace_available() { return false; }
void trace_push(const std::string&) {}
void trace_pop() {}
#endif

}  // namespace hk
