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
// (cudaGetSymbolAddress, with that device current) and caches it; nothing here
// calls cudaMalloc, cudaFree or any allocating library routine.  Make that first
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
#include <mutex>

#include "kdn_internal.h"

namespace kdn {
namespace {

static __device__ __align__(256) unsigned char g_prefill_scratch[KDN_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

cudaError_t static_prefill_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_prefill_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace kdn
