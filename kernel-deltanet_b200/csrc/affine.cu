// affine.cu -- the affine semigroup of block state maps, exact fp32 on CUDA cores.
//
// The delta-rule state map of a block of tokens is affine in the entering state:
//     S_out = S_in A + B,      S [dv, D],  A [D, D],  B [dv, D]
// and blocks compose as (kernels/blelloch_scan.py:42-56, core/associative_algebra.py:45-60)
//     (A1, B1) o (A2, B2) = (A1 A2, B1 A2 + B2).
//
// Both entry points reduce to one batched product with a shared right operand:
//     out1 = L1 R            (m1 rows, no addend)
//     out2 = L2 R + add2     (m2 rows, add2 may be null)
// compose:          L1 = A1, L2 = B1, R = A2, add2 = B2     (one launch)
// prefix states:    m1 = 0,  L2 = S_c, R = A_c, add2 = B_c  (one launch per block)
//
// The product is tiny next to a prefill (a 512 x 512 x 576 compose is 0.3 GFLOP per
// head), and fp32 parity (1e-4) rules out a single bf16/tf32 tensor-core pass, so
// it runs as a register-tiled SIMT GEMM: 64 x 64 output tile per CTA, K in steps of 16
// staged through shared memory, a 4 x 4 register tile per thread.
#include "kdn_internal.h"

namespace kdn {
namespace {

constexpr int kTile = 64;
constexpr int kKStep = 16;
constexpr int kThreads = 256;

struct AffineGemm {
  const float* L1;  // [batch, m1, K]
  const float* L2;  // [batch, m2, K]
  const float* R;   // [batch, K, N]
  const float* add2;  // [batch, m2, N] or null
  float* out1;      // [batch, m1, N]
  float* out2;      // [batch, m2, N]
  int m1, m2, K, N;
};

__global__ void __launch_bounds__(kThreads) affine_gemm_kernel(AffineGemm g) {
  __shared__ __align__(16) float Ls[kKStep][kTile + 4];
  __shared__ __align__(16) float Rs[kKStep][kTile];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t b = blockIdx.z;
  const int n0 = blockIdx.x * kTile;
  const int m0 = blockIdx.y * kTile;
  const int M = g.m1 + g.m2;

  // the L row this thread stages: row m0 + tid/4, k offset (tid%4)*4 within the step
  const int lrow = m0 + (tid >> 2);
  const float* lsrc = nullptr;
  if (lrow < g.m1)
    lsrc = g.L1 + (b * g.m1 + lrow) * int64_t(g.K);
  else if (lrow < M)
    lsrc = g.L2 + (b * g.m2 + (lrow - g.m1)) * int64_t(g.K);
  const int lk = (tid & 3) * 4;
  // the R element group this thread stages: k row tid/16, columns (tid%16)*4
  const int rk = tid >> 4, rc = n0 + (tid & 15) * 4;
  const float* rsrc = g.R + b * int64_t(g.K) * g.N;

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < g.K; k0 += kKStep) {
    float4 lv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (lsrc) lv = *reinterpret_cast<const float4*>(lsrc + k0 + lk);
    float4 rv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rc < g.N) rv = *reinterpret_cast<const float4*>(rsrc + int64_t(k0 + rk) * g.N + rc);
    __syncthreads();  // the previous step's reads are done
    Ls[lk + 0][tid >> 2] = lv.x;
    Ls[lk + 1][tid >> 2] = lv.y;
    Ls[lk + 2][tid >> 2] = lv.z;
    Ls[lk + 3][tid >> 2] = lv.w;
    *reinterpret_cast<float4*>(&Rs[rk][(tid & 15) * 4]) = rv;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kKStep; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&Ls[kk][ty * 4]);
      const float4 r = *reinterpret_cast<const float4*>(&Rs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float rv4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], rv4[j], acc[i][j]);
    }
  }

  const int col = n0 + tx * 4;
  if (col >= g.N) return;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = m0 + ty * 4 + i;
    if (row >= M) break;
    float4 o = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    float* dst;
    if (row < g.m1) {
      dst = g.out1 + (b * g.m1 + row) * int64_t(g.N) + col;
    } else {
      const int64_t off = (b * g.m2 + (row - g.m1)) * int64_t(g.N) + col;
      if (g.add2) {
        const float4 a = *reinterpret_cast<const float4*>(g.add2 + off);
        o.x += a.x;
        o.y += a.y;
        o.z += a.z;
        o.w += a.w;
      }
      dst = g.out2 + off;
    }
    *reinterpret_cast<float4*>(dst) = o;
  }
}

// A [batch, D, D] = I (rows of a zero-length block's map)
__global__ void affine_identity_kernel(float* A, int64_t batch, int D) {
  const int64_t total = batch * D * int64_t(D);
  for (int64_t e = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; e < total; e += int64_t(gridDim.x) * blockDim.x) {
    const int64_t rc = e % (int64_t(D) * D);
    A[e] = (rc / D == rc % D) ? 1.f : 0.f;
  }
}

cudaError_t launch_gemm(const AffineGemm& g, int64_t batch, cudaStream_t stream) {
  const int M = g.m1 + g.m2;
  dim3 grid(unsigned((g.N + kTile - 1) / kTile), unsigned((M + kTile - 1) / kTile), unsigned(batch));
  affine_gemm_kernel<<<grid, kThreads, 0, stream>>>(g);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_affine_compose(const float* A1, const float* B1, const float* A2, const float* B2, float* A_out,
                                  float* B_out, int64_t batch, int D, int dv, cudaStream_t stream) {
  AffineGemm g;
  g.L1 = A1;
  g.L2 = B1;
  g.R = A2;
  g.add2 = B2;
  g.out1 = A_out;
  g.out2 = B_out;
  g.m1 = A_out ? D : 0;
  g.m2 = B_out ? dv : 0;
  g.K = D;
  g.N = D;
  if (g.m1 + g.m2 == 0) return cudaSuccess;
  return launch_gemm(g, batch, stream);
}

cudaError_t launch_affine_identity(float* A, int64_t batch, int D, cudaStream_t stream) {
  const int64_t total = batch * D * int64_t(D);
  int64_t blocks = (total + kThreads - 1) / kThreads;
  if (blocks > 148 * 8) blocks = 148 * 8;
  affine_identity_kernel<<<unsigned(blocks), kThreads, 0, stream>>>(A, batch, D);
  return cudaGetLastError();
}

cudaError_t launch_affine_prefix_states(const float* A, const float* B, const float* S0, float* states,
                                        float* final_state, int64_t n_c, int64_t batch, int D, int dv,
                                        cudaStream_t stream) {
  const size_t state_elems = size_t(batch) * dv * D;
  cudaError_t e = cudaSuccess;
  if (!S0)
    e = cudaMemsetAsync(states, 0, state_elems * sizeof(float), stream);
  else if (S0 != states)
    e = cudaMemcpyAsync(states, S0, state_elems * sizeof(float), cudaMemcpyDeviceToDevice, stream);
  if (e != cudaSuccess) return e;
  for (int64_t c = 0; c < n_c; ++c) {
    const bool last = c + 1 == n_c;
    if (last && !final_state) break;
    AffineGemm g;
    g.L1 = nullptr;
    g.out1 = nullptr;
    g.m1 = 0;
    g.L2 = states + c * state_elems;
    g.R = A + c * size_t(batch) * D * D;
    g.add2 = B + c * state_elems;
    g.out2 = last ? final_state : states + (c + 1) * state_elems;
    g.m2 = dv;
    g.K = D;
    g.N = D;
    if ((e = launch_gemm(g, batch, stream)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace kdn
