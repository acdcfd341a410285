// gemv.cu -- y = x W^T for decode-size batches (up to 16 token rows), bf16 operands, fp32 accumulation.
//
// In a decode step every projection of the hybrid LM (q|k|v|beta, the anchors' q|k|v, the output
// projections, SwiGLU, the LM head) multiplies a few token rows by a large weight: the weight bytes
// are the whole cost (HBM-bound, about 2 bytes per multiply-add per token row).  At 8 token rows an
// fp32 FMA dot product needs 4 FMAs per weight byte -- as much ALU time as the SMs have at full HBM
// bandwidth -- so the products run on the tensor cores instead, as m16n8k16 MMAs with the weight rows
// as M and the tokens as N, and the SM's issue slots stay free for the loads.
//
// A CTA owns 16 weight rows and splits K over its 8 warps (32-element blocks, warp w taking blocks
// w, w + 8, ...; eight blocks' loads in flight before their MMAs).  Lane (g, t) (g = lane / 4,
// t = lane % 4) loads the 16 bytes at k0 + 8t of weight rows g and g + 8 and of token row g: the
// MMA fragment slots {2t, 2t+1, 2t+8, 2t+9} of lane t take elements 0-3 of the chunk in the first
// MMA and 4-7 in the second, for A and B alike, so the 32 elements of a block are each multiplied
// once, every load is a contiguous 16 bytes and no shuffle is needed.  The eight warps' 16 x 8 (x 2
// for 9-16 tokens) partial products are summed in shared memory and stored.
#include <cuda_bf16.h>

#include "kdn_internal.h"

namespace kdn {
namespace {

constexpr int kWarps = 8;   // K is split over the CTA's warps
constexpr int kRowsCta = 16;
constexpr int kMaxM = 16;   // token rows per launch (two groups of 8)
constexpr int kUnroll = 8;  // 32-element blocks in flight per warp

__device__ __forceinline__ uint4 ld_stream(const void* p) {  // weight bytes are read once: no L1 allocation
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_x(const void* p) {  // token rows are re-read by every CTA
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// d += A(16 x 16, bf16) B(16 x 8, bf16), fp32 accumulators
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int G>  // token groups of 8
__global__ void __launch_bounds__(32 * kWarps) gemv_kernel(const __nv_bfloat16* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ w, void* __restrict__ y,
                                                           int y_bf16, int M, int N, int K, int64_t ldo) {
  __shared__ float red[kWarps][G][kRowsCta * 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t n0 = int64_t(blockIdx.x) * kRowsCta;
  const bool r0_ok = n0 + g < N, r1_ok = n0 + g + 8 < N;
  const __nv_bfloat16* w0 = w + (n0 + g) * K + 8 * t;
  const __nv_bfloat16* w1 = w0 + int64_t(8) * K;
  bool x_ok[G];
  const __nv_bfloat16* xr[G];
#pragma unroll
  for (int q = 0; q < G; ++q) {
    x_ok[q] = 8 * q + g < M;
    xr[q] = x + int64_t(8 * q + g) * K + 8 * t;
  }
  float acc[G][4];
#pragma unroll
  for (int q = 0; q < G; ++q)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[q][i] = 0.f;

  const int nkb = K / 32;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int kb0 = warp; kb0 < nkb; kb0 += kWarps * kUnroll) {
    uint4 a[kUnroll][2], b[kUnroll][G];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int kb = kb0 + kWarps * u;
      const bool in = kb < nkb;
      const int64_t off = int64_t(kb) * 32;
      a[u][0] = (in && r0_ok) ? ld_stream(w0 + off) : zero;
      a[u][1] = (in && r1_ok) ? ld_stream(w1 + off) : zero;
#pragma unroll
      for (int q = 0; q < G; ++q) b[u][q] = (in && x_ok[q]) ? ld_x(xr[q] + off) : zero;
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
#pragma unroll
      for (int q = 0; q < G; ++q) {
        // elements 0-3 of each chunk: slots 2t, 2t+1 (.x) and 2t+8, 2t+9 (.y); elements 4-7 likewise
        mma_bf16(acc[q], a[u][0].x, a[u][1].x, a[u][0].y, a[u][1].y, b[u][q].x, b[u][q].y);
        mma_bf16(acc[q], a[u][0].z, a[u][1].z, a[u][0].w, a[u][1].w, b[u][q].z, b[u][q].w);
      }
    }
  }
  // D fragment: (row g, tokens 2t, 2t+1) and (row g + 8, tokens 2t, 2t+1); stored token-major
#pragma unroll
  for (int q = 0; q < G; ++q) {
    red[warp][q][(2 * t) * kRowsCta + g] = acc[q][0];
    red[warp][q][(2 * t + 1) * kRowsCta + g] = acc[q][1];
    red[warp][q][(2 * t) * kRowsCta + g + 8] = acc[q][2];
    red[warp][q][(2 * t + 1) * kRowsCta + g + 8] = acc[q][3];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < G * kRowsCta * 8; j += 32 * kWarps) {
    const int q = j / (kRowsCta * 8), e = j % (kRowsCta * 8);
    const int m = 8 * q + e / kRowsCta, r = e % kRowsCta;
    if (m < M && n0 + r < N) {
      float s = 0.f;
#pragma unroll
      for (int v = 0; v < kWarps; ++v) s += red[v][q][e];
      const int64_t i = int64_t(m) * ldo + n0 + r;
      if (y_bf16) static_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(s);
      else static_cast<float*>(y)[i] = s;
    }
  }
}

}  // namespace

int gemv_max_rows() { return kMaxM; }

cudaError_t launch_gemv(const void* x, const void* w, void* y, bool y_bf16, int64_t M, int N, int K, int64_t ldo,
                        cudaStream_t stream) {
  const size_t es = y_bf16 ? 2 : 4;
  const int64_t grid = (int64_t(N) + kRowsCta - 1) / kRowsCta;
  for (int64_t m0 = 0; m0 < M; m0 += kMaxM) {
    const int m = int(M - m0 < kMaxM ? M - m0 : kMaxM);
    const __nv_bfloat16* xm = static_cast<const __nv_bfloat16*>(x) + m0 * K;
    const __nv_bfloat16* wb = static_cast<const __nv_bfloat16*>(w);
    void* ym = static_cast<char*>(y) + m0 * ldo * es;
    if (m <= 8)
      gemv_kernel<1><<<unsigned(grid), 32 * kWarps, 0, stream>>>(xm, wb, ym, y_bf16 ? 1 : 0, m, N, K, ldo);
    else
      gemv_kernel<2><<<unsigned(grid), 32 * kWarps, 0, stream>>>(xm, wb, ym, y_bf16 ? 1 : 0, m, N, K, ldo);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace kdn
