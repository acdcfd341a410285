// lift.cu -- standalone feature-lift kernel (kdn_fwht_lift).
//
// One warp per 64-d vector, grid-stride over vectors.  HBM traffic per vector:
// 64 input elements + D output elements; the butterfly and the cosines stay in
// registers.
#include "kdn_internal.h"
#include "lift.cuh"

namespace kdn {

__global__ void __launch_bounds__(256) lift_kernel(const void* __restrict__ x, int x_dtype, void* __restrict__ out,
                                                   int out_dtype, int64_t n, ProjParams P) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int D = 64 * P.M;
  for (int64_t r = warp; r < n; r += nwarps) {
    const float2 xv = ld2_as_f32(x, x_dtype, r * kDk + 2 * lane);
    float c[kMaxBlocks][2];
    lift_warp(xv.x, xv.y, P, lane, c);
#pragma unroll
    for (int m = 0; m < kMaxBlocks; ++m)
      if (m < P.M) st2_from_f32(out, out_dtype, r * D + 64 * m + 2 * lane, c[m][0], c[m][1]);
  }
}

cudaError_t launch_lift(const void* x, int x_dtype, void* out, int out_dtype, int64_t n, const ProjParams& P,
                        cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const int threads = 256;
  int64_t blocks = (n + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  lift_kernel<<<dim3(unsigned(blocks)), threads, 0, stream>>>(x, x_dtype, out, out_dtype, n, P);
  return cudaGetLastError();
}

}  // namespace kdn
