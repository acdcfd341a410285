// gemv.cu -- y = x W^T for decode-size batches (a handful of rows), bf16 operands, fp32 accumulation.
//
// In a decode step every projection of the hybrid LM (q|k|v|beta, the anchors' q|k|v, the output
// projections, SwiGLU, the LM head) multiplies a few token rows by a large weight: the weight bytes
// are the whole cost, so each weight row is streamed exactly once, in 16-byte loads that bypass L1.
// A CTA owns R consecutive weight rows (output columns) and splits K over its four warps; a warp
// takes 256-element steps of K (8 elements a lane, two steps in flight) and dots them with every row
// of x (a few KiB, served from L1/L2).  The R x MR partial sums of a warp are reduced across lanes by
// a halving butterfly (each exchange sends half of the remaining values, 2 V - 2 shuffles for V
// values instead of 5 V), then across the four warps in shared memory.
#include <cuda_bf16.h>

#include "kdn_internal.h"

namespace kdn {
namespace {

constexpr int kWarps = 4;  // K is split over the CTA's warps
constexpr int kMaxM = 16;  // x rows handled by one launch

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

// weight rows are read once: keep them out of L1
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// acc[r][m] += <w row r, x row m> over the 8 elements at k0
template <int MR, int R>
__device__ __forceinline__ void dot_step(const uint4 (&u)[R], const __nv_bfloat16* __restrict__ x, int K, int k0,
                                         int M, float (&acc)[R][MR]) {
  float wf[R][8];
#pragma unroll
  for (int r = 0; r < R; ++r) bf16x8_to_f32(u[r], wf[r]);
#pragma unroll
  for (int m = 0; m < MR; ++m) {
    if (m < M) {
      float xf[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(x + int64_t(m) * K + k0), xf);
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[r][m] = fmaf(wf[r][j], xf[j], acc[r][m]);
    }
  }
}

template <int MR, int R>
__global__ void __launch_bounds__(32 * kWarps) gemv_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ w, void* __restrict__ y,
                                                           int y_bf16, int M, int N, int K, int64_t ldo) {
  constexpr int V = R * MR;  // partial sums per lane; a power of two >= 32
  static_assert(V >= 32 && (V & (V - 1)) == 0, "butterfly needs a power-of-two count >= 32");
  __shared__ float red[kWarps][V];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n0 = int64_t(blockIdx.x) * R;
  const int nsteps = (K + 255) / 256;
  float acc[R][MR];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;

  for (int s = warp; s < nsteps; s += 2 * kWarps) {  // steps s and s + kWarps, loads of both first
    const int k0 = 256 * s + 8 * lane, k1 = k0 + 256 * kWarps;
    const bool v0 = k0 < K, v1 = k1 < K;
    uint4 u0[R], u1[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const bool row = n0 + r < N;
      u0[r] = (v0 && row) ? ld_stream(w + (n0 + r) * K + k0) : make_uint4(0u, 0u, 0u, 0u);
      u1[r] = (v1 && row) ? ld_stream(w + (n0 + r) * K + k1) : make_uint4(0u, 0u, 0u, 0u);
    }
    if (v0) dot_step<MR, R>(u0, x, K, k0, M, acc);
    if (v1) dot_step<MR, R>(u1, x, K, k1, M, acc);
  }

  // halving butterfly: after the exchange at offset o a lane keeps the half of its values selected by
  // its lane bit o; at the end lane l holds the full sums of flat indices [l V/32, (l + 1) V/32)
  float v[V];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MR; ++m) v[r * MR + m] = acc[r][m];
#pragma unroll
  for (int o = 16, cnt = V; o > 0; o >>= 1, cnt >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < cnt / 2; ++i) {
      const float send = upper ? v[i] : v[i + cnt / 2];
      const float keep = upper ? v[i + cnt / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
#pragma unroll
  for (int i = 0; i < V / 32; ++i) red[warp][lane * (V / 32) + i] = v[i];
  __syncthreads();
  for (int j = threadIdx.x; j < V; j += 32 * kWarps) {
    const int r = j / MR, m = j % MR;
    if (m < M && n0 + r < N) {
      float s = 0.f;
#pragma unroll
      for (int q = 0; q < kWarps; ++q) s += red[q][j];
      const int64_t i = int64_t(m) * ldo + n0 + r;
      if (y_bf16) static_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(s);
      else static_cast<float*>(y)[i] = s;
    }
  }
}

template <int MR, int R>
void launch_bucket(const __nv_bfloat16* x, const __nv_bfloat16* w, void* y, bool y_bf16, int M, int N, int K,
                   int64_t ldo, cudaStream_t stream) {
  const int64_t grid = (int64_t(N) + R - 1) / R;
  gemv_kernel<MR, R><<<unsigned(grid), 32 * kWarps, 0, stream>>>(x, w, y, y_bf16 ? 1 : 0, M, N, K, ldo);
}

}  // namespace

int gemv_max_rows() { return kMaxM; }

cudaError_t launch_gemv(const void* x, const void* w, void* y, bool y_bf16, int64_t M, int N, int K, int64_t ldo,
                        cudaStream_t stream) {
  const size_t es = y_bf16 ? 2 : 4;
  for (int64_t m0 = 0; m0 < M; m0 += kMaxM) {
    const int m = int(M - m0 < kMaxM ? M - m0 : kMaxM);
    const __nv_bfloat16* xm = static_cast<const __nv_bfloat16*>(x) + m0 * K;
    const __nv_bfloat16* wb = static_cast<const __nv_bfloat16*>(w);
    void* ym = static_cast<char*>(y) + m0 * ldo * es;
    if (m <= 4) launch_bucket<4, 8>(xm, wb, ym, y_bf16, m, N, K, ldo, stream);
    else if (m <= 8) launch_bucket<8, 8>(xm, wb, ym, y_bf16, m, N, K, ldo, stream);
    else launch_bucket<16, 4>(xm, wb, ym, y_bf16, m, N, K, ldo, stream);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace kdn
