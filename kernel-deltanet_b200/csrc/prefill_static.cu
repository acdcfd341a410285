// prefill_static.cu -- kdn_chunked_prefill_static: the exact fp32 prefill run over a
// fixed scratch array compiled into the library, for callers that cannot allocate.
//
// Some callers may not allocate device memory at the point where they run a
// prefill: a serving engine that has handed nearly all device memory to its own
// state/KV pool up front (a cudaMalloc there fails or fragments that pool), or a
// latency-bound step loop that cannot take the implicit device synchronisation of
// cudaFree.  This entry point takes no workspace argument; the scratch of the
// CUDA-core path lives in g_prefill_scratch below, KDN_STATIC_SCRATCH_BYTES per
// device, reserved when the CUDA runtime loads this module on that device.
//
// Set-up: the first call on each device looks the array's device address up
// (cudaGetSymbolAddress, with that device current) and keeps it together with the
// ID of the device's current CUDA context; a later call on the device looks the
// address up again only if that context has changed (a device reset releases the
// context and the module, and the array may come back elsewhere).  Nothing here
// calls cudaMalloc, cudaFree or any allocating library routine.  Make the first
// call on a device before any stream capture begins.
//
// Nothing in the scratch has to start at zero: the lift kernel writes every row of
// the lifted features (zeros for padded rows) and the chunk kernel writes every
// matrix and gate the chain kernel reads, so no clearing pass is needed.
//
// All calls on one device share the one array: two calls whose kernels overlap
// (different streams without ordering between them, or several host threads)
// race on it.  Order them on one stream, or use kdn_chunked_prefill with a
// workspace per stream.
#include <cuda.h>
#include <mutex>

#include "kdn_internal.h"

namespace kdn {
namespace {

static __device__ __align__(256) unsigned char g_prefill_scratch[KDN_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};  // ID of the context the address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// ID of the calling thread's current context (0 if the driver cannot tell)
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {  // under g_scratch_mu
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    looked_up = true;
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS)
    return id;
  return 0;
}

}  // namespace

cudaError_t static_prefill_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  void* p = nullptr;
  if (!g_scratch_ptr[dev]) {
    // the first lookup also makes the device's primary context current
    if ((e = cudaGetSymbolAddress(&p, g_prefill_scratch)) != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = current_context_id();
  } else {
    const unsigned long long ctx = current_context_id();
    if (ctx != g_scratch_ctx[dev]) {
      if ((e = cudaGetSymbolAddress(&p, g_prefill_scratch)) != cudaSuccess) return e;
      g_scratch_ptr[dev] = p;
      g_scratch_ctx[dev] = ctx;
    }
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace kdn
