// spatten_prog_attn_noalloc: the progressive attention op for callers that
// cannot allocate device memory.
//
// spatten_prog_attn needs a workspace for its importance partial sums, which
// the caller normally allocates. Some callers cannot call cudaMalloc at all:
// hosts that fix their device-memory budget at start-up and forbid any
// allocation afterwards (serving processes with a pre-planned memory map,
// real-time loops where an allocation's latency or failure is not
// acceptable), and plugins that may only use the memory their host
// application hands them. This entry point takes the workspace from a fixed
// array in device memory that is part of the library instead.
//
// Limits and sharing:
//  * The array holds kNoAllocBytes (16 MiB). A request whose workspace
//    (spatten_prog_attn_workspace_size) exceeds that is rejected with
//    SPATTEN_ERR_INVALID before anything runs.
//  * The array is reserved on a device when the library's device code is
//    loaded there -- at the first use of any of its kernels on that device
//    under CUDA's default lazy module loading (which can be the first call of
//    this entry point), at context creation with eager loading -- and it is
//    held until the process exits.
//  * All calls on a device share the one array and it keeps the last call's
//    contents. The kernels write every partial sum they later read, so
//    nothing has to start at zero. Calls that can overlap on the GPU (on
//    different streams without ordering between them) race on the array;
//    order them on one stream or with events.
//  * Every call looks up the array's device address (cudaGetSymbolAddress)
//    on the current device, so a call after cudaDeviceReset finds the array
//    of the new context. The first call on a device may load the module
//    there (lazy loading): make that first call before any stream capture.
#include <cstdio>

#include "../../include/spatten_b200.h"
#include "kernels.h"

constexpr size_t kNoAllocBytes = size_t(16) << 20;

// The workspace. In host code this name is a host-side stand-in, not a device
// address: only the address from cudaGetSymbolAddress may be passed to a kernel.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {

// Device address of the array on the current device. Looked up on every call
// rather than cached: a cached address would outlive the context it belongs
// to after cudaDeviceReset.
int scratch_address(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return spatten::set_last_error(SPATTEN_ERR_CUDA, "prog_attn_noalloc: cudaGetSymbolAddress failed");
  *out = p;
  return SPATTEN_OK;
}

}  // namespace

extern "C" size_t spatten_prog_attn_noalloc_capacity(void) { return kNoAllocBytes; }

extern "C" int spatten_prog_attn_noalloc(const spatten_prog_attn_args* a, void* stream) {
  const size_t need = spatten_prog_attn_workspace_size(a);
  if (need > kNoAllocBytes) {
    char msg[160];
    snprintf(msg, sizeof(msg),
             "prog_attn_noalloc: workspace of %zu bytes exceeds the fixed %zu-byte array", need,
             kNoAllocBytes);
    return spatten::set_last_error(SPATTEN_ERR_INVALID, msg);
  }
  void* ws = nullptr;
  if (need > 0) {
    if (int e = scratch_address(&ws)) return e;
  }
  return spatten_prog_attn(a, ws, need > 0 ? kNoAllocBytes : 0, stream);
}
