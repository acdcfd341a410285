// tc_chunk.cuh -- pieces shared by the tensor-core chunk kernels (prefill_tc.cu,
// prefill_split.cu): problem constants, kernel arguments, fp16/bf16 packing, and the
// loads of one chunk's k, q, v rows into swizzled shared-memory tiles.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kdn_common.cuh"
#include "lift.cuh"
#include "tc_prims.cuh"

namespace kdn {
namespace tcc {

constexpr int kC = 64;       // chunk
constexpr int kDV = 64;      // value dim
constexpr int kD = 512;      // lifted dim
constexpr int kSlices = 4;   // 128-feature slices

struct TcArgs {
  const void* q;
  const void* k;
  const void* v;
  int in_dtype;
  const void* beta;
  const void* decay;
  int gate_dtype;
  const float* S0;
  void* y;
  int y_dtype;
  float* S_out;
  int64_t T;
  int NC;
  // varlen batches (fused path): scan n reads token rows [var_off[n], var_off[n] + var_len[n]) of
  // q, k, v, y, beta, decay (rows counted in tokens); null = the uniform [N, T] layout
  const int64_t* var_off = nullptr;
  const int64_t* var_len = nullptr;
  int64_t var_rows = 0;  // rows in the varlen tensors (bounds of var_off + var_len)
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// two floats -> packed fp16 pair (a in the low half); values already inside the fp16 range
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
// same, saturating to the largest finite fp16 instead of overflowing to inf
__device__ __forceinline__ uint32_t pack_f16_sat(float a, float b) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// index of element (i, j) of a 64x64 fp32 matrix whose float4 slots are swizzled
// by row, so that row-wise and column-wise vector accesses are conflict-free
__device__ __forceinline__ int sx(int i, int j) { return i * 64 + ((((j >> 2) ^ i) & 15) << 2) + (j & 3); }

// k and q rows of chunk c -> the K-major swizzled input tile (bf16 inputs); 512 threads
__device__ __forceinline__ void prefetch_kq(const TcArgs& a, int64_t n, int c, uint32_t xin, int tid) {
  const int r = tid >> 2, qq = tid & 3;  // row r of [k;q], 16-element quarter qq
  const int64_t t = int64_t(c) * kC + (r & 63);
  const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(r < 64 ? a.k : a.q);
  const bool in = t < a.T;
  const __nv_bfloat16* src = base + (in ? (n * a.T + t) * 64 + 16 * qq : 0);
#pragma unroll
  for (int i = 0; i < 2; ++i)
    tc::cp_async16(xin + tc::sw128_offset(r, 16 * qq + 8 * i), src + (in ? 8 * i : 0), in ? 16 : 0);
}

// fp32 inputs: load and round to bf16 into the input tile
__device__ __forceinline__ void load_kq_f32(const TcArgs& a, int64_t n, int c, uint8_t* xin, int tid) {
  const int r = tid >> 2, qq = tid & 3;
  const int64_t t = int64_t(c) * kC + (r & 63);
  const float* src = reinterpret_cast<const float*>(r < 64 ? a.k : a.q) + (n * a.T + t) * 64 + 16 * qq;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    uint4 pk = make_uint4(0, 0, 0, 0);
    if (t < a.T) {
      const float4 x0 = reinterpret_cast<const float4*>(src)[2 * i];
      const float4 x1 = reinterpret_cast<const float4*>(src)[2 * i + 1];
      pk = make_uint4(pack_bf16(x0.x, x0.y), pack_bf16(x0.z, x0.w), pack_bf16(x1.x, x1.y), pack_bf16(x1.z, x1.w));
    }
    *reinterpret_cast<uint4*>(xin + tc::sw128_offset(r, 16 * qq + 8 * i)) = pk;
  }
}

// v rows of chunk c -> row-major bf16 tile (bf16 inputs); 512 threads, one 16-byte piece each
__device__ __forceinline__ void prefetch_v(const TcArgs& a, int64_t n, int c, uint32_t vb, int tid) {
  const int row = tid >> 3, cc = tid & 7;
  const int64_t t = int64_t(c) * kC + row;
  const bool in = t < a.T;
  const char* src = reinterpret_cast<const char*>(a.v) + (in ? ((n * a.T + t) * 64) * 2 + 16 * cc : 0);
  tc::cp_async16(vb + row * 128 + 16 * cc, src, in ? 16 : 0);
}

// Omega = H D3 H D2 H D1 / 8 as the bf16 B operand of the lift product: feature
// f = 64 blk + i, input index d; slice s (128 features) at 16 KiB s, K-major.
// One warp shuffle butterfly per (blk, d) on a unit input vector.
__device__ __forceinline__ void build_omega(uint8_t* om_base, const ProjParams& P, int warp, int lane, int nwarps) {
  for (int job = warp; job < 8 * 64; job += nwarps) {
    const int blk = job >> 6, d = job & 63;
    const float x0 = (d == 2 * lane) ? 1.f : 0.f, x1 = (d == 2 * lane + 1) ? 1.f : 0.f;
    float u0, u1;
    structured_block(x0, x1, P.sign_bits[blk], lane, u0, u1);
    const int f0 = 64 * blk + 2 * lane, s = f0 >> 7, fl = f0 & 127;
    uint8_t* om = om_base + s * 16384;
    *reinterpret_cast<__nv_bfloat16*>(om + tc::sw128_offset(fl, d)) = __float2bfloat16_rn(u0);
    *reinterpret_cast<__nv_bfloat16*>(om + tc::sw128_offset(fl + 1, d)) = __float2bfloat16_rn(u1);
  }
}

}  // namespace tcc
}  // namespace kdn
