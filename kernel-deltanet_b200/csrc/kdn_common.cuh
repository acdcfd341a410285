// kdn_common.cuh -- shared device helpers for libkdn (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kdn.h"

namespace kdn {

constexpr int kDk = 64;        // head dim of q/k (the FWHT order); fixed by the butterfly layout
constexpr int kMaxBlocks = 8;  // D = M * 64 with M <= 8

// Projection constants passed to kernels by value (kernel parameter space).
struct ProjParams {
  uint64_t sign_bits[kMaxBlocks][3];
  const float* phase;  // [D]
  float tau_inv;
  float amp;
  int M;  // number of 64-wide blocks, D = 64 * M
};

inline ProjParams make_proj_params(const kdn_projection& p) {
  ProjParams q;
  for (int m = 0; m < kMaxBlocks; ++m)
    for (int s = 0; s < 3; ++s) q.sign_bits[m][s] = p.sign_bits[m][s];
  q.phase = p.phase;
  q.tau_inv = p.tau_inv;
  q.amp = p.amp;
  q.M = p.D / kDk;
  return q;
}

// ---------------------------------------------------------------- dtype I/O
__device__ __forceinline__ float ld_as_f32(const void* p, int dtype, int64_t i) {
  return dtype == KDN_DTYPE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                                 : reinterpret_cast<const float*>(p)[i];
}

// Element i of a gate array (bf16 or fp32) as raw bits: the bf16 bits in the low half, else the fp32
// bits.  The two loads are predicated into one register, so nothing consumes the value at the load
// and the issuing warp does not wait for it until the bits are converted.
__device__ __forceinline__ uint32_t ld_gate_bits(const void* p, bool bf16, int64_t i) {
  uint32_t r;
  const char* b = reinterpret_cast<const char*>(p);
  asm volatile(
      "{\n\t.reg .pred q;\n\tsetp.ne.u32 q, %1, 0;\n\t@q ld.global.u16 %0, [%2];\n\t@!q ld.global.b32 %0, [%3];\n\t}"
      : "=r"(r)
      : "r"(uint32_t(bf16)), "l"(b + 2 * i), "l"(b + 4 * i));
  return r;
}

__device__ __forceinline__ void st_from_f32(void* p, int dtype, int64_t i, float x) {
  if (dtype == KDN_DTYPE_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else
    reinterpret_cast<float*>(p)[i] = x;
}

// two consecutive elements starting at an even index
__device__ __forceinline__ float2 ld2_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == KDN_DTYPE_BF16) {
    __nv_bfloat162 h = reinterpret_cast<const __nv_bfloat162*>(p)[i >> 1];
    return __bfloat1622float2(h);
  }
  return reinterpret_cast<const float2*>(p)[i >> 1];
}

__device__ __forceinline__ void st2_from_f32(void* p, int dtype, int64_t i, float a, float b) {
  if (dtype == KDN_DTYPE_BF16)
    reinterpret_cast<__nv_bfloat162*>(p)[i >> 1] = __floats2bfloat162_rn(a, b);
  else
    reinterpret_cast<float2*>(p)[i >> 1] = make_float2(a, b);
}

// ---------------------------------------------------------------- warp FWHT
// A 64-point vector lives in one warp: lane l holds elements 2l (v0) and 2l+1 (v1).
// fwht64 computes H v with H the +-1 Sylvester matrix (H_ij = (-1)^popc(i&j)),
// in place: level h=1 pairs the two registers of a lane, levels h=2..32 pair
// lane l with lane l^(h/2) through shuffles.
__device__ __forceinline__ void fwht64(float& v0, float& v1, int lane) {
  float a = v0 + v1, b = v0 - v1;
  v0 = a;
  v1 = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float p0 = __shfl_xor_sync(0xffffffffu, v0, o);
    const float p1 = __shfl_xor_sync(0xffffffffu, v1, o);
    const bool hi = (lane & o) != 0;
    v0 = hi ? (p0 - v0) : (v0 + p0);
    v1 = hi ? (p1 - v1) : (v1 + p1);
  }
}

__device__ __forceinline__ void apply_signs(float& v0, float& v1, uint64_t bits, int lane) {
  const uint64_t two = bits >> (2 * lane);
  if (two & 1ull) v0 = -v0;
  if (two & 2ull) v1 = -v1;
}

// u = H diag(d3) H diag(d2) H diag(d1) x / 8 for block m (kernels/fwht.py:103-110),
// x given as the lane's two elements.
__device__ __forceinline__ void structured_block(float x0, float x1, const uint64_t (&bits)[3], int lane,
                                                 float& u0, float& u1) {
  float v0 = x0, v1 = x1;
  apply_signs(v0, v1, bits[0], lane);
  fwht64(v0, v1, lane);
  apply_signs(v0, v1, bits[1], lane);
  fwht64(v0, v1, lane);
  apply_signs(v0, v1, bits[2], lane);
  fwht64(v0, v1, lane);
  u0 = v0 * 0.125f;
  u1 = v1 * 0.125f;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Kernels whose bounds checks skip an access record a nonzero code in an error
// word of their translation unit (first code wins); kdn_device_error() reads
// and clears all of them.
__device__ __forceinline__ void record_device_error(int* word, int code) { atomicCAS(word, 0, code); }

// device error codes
constexpr int kErrSlotOutOfRange = 1;
constexpr int kErrTcWaitTimeout = 2;     // fused tensor-core prefill: a bounded wait gave up
constexpr int kErrSplitWaitTimeout = 3;  // two-phase prefill: a bounded wait gave up
constexpr int kErrDecodeWaitTimeout = 4; // decode: a bounded wait gave up
constexpr int kErrProjWaitTimeout = 5;   // tensor-parallel projection: a bounded wait gave up
constexpr int kErrLiftWaitTimeout = 6;   // tensor-core lift: a bounded wait gave up
constexpr int kErrAttnWaitTimeout = 7;   // anchor attention: a bounded wait gave up

}  // namespace kdn
