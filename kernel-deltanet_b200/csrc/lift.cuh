// lift.cuh -- warp-level structured-FWHT feature lift (device function).
//
// phi(x) = u / (||u|| + 1e-8),  u_f = amp * cos(tau_inv * (Omega x)_f + phase_f),
// Omega block m = H diag(d3) H diag(d2) H diag(d1) / 8   (kernels/fwht.py:96-130).
//
// The 64-d input is held by one warp (lane l: elements 2l, 2l+1); block m of
// the output is produced in the same layout (lane l: features 64m+2l, 64m+2l+1),
// so the butterfly never leaves registers.
#pragma once

#include "kdn_common.cuh"

namespace kdn {

// Lifts one vector; c[m][0..1] receive the normalised features 64m+2l, 64m+2l+1.
__device__ __forceinline__ void lift_warp(float x0, float x1, const ProjParams& P, int lane,
                                          float (&c)[kMaxBlocks][2]) {
  float ss = 0.f;
#pragma unroll
  for (int m = 0; m < kMaxBlocks; ++m) {
    c[m][0] = 0.f;
    c[m][1] = 0.f;
    if (m < P.M) {
      float u0, u1;
      structured_block(x0, x1, P.sign_bits[m], lane, u0, u1);
      const int f = 64 * m + 2 * lane;
      const float2 ph = *reinterpret_cast<const float2*>(P.phase + f);
      c[m][0] = P.amp * cosf(fmaf(u0, P.tau_inv, ph.x));
      c[m][1] = P.amp * cosf(fmaf(u1, P.tau_inv, ph.y));
      ss = fmaf(c[m][0], c[m][0], fmaf(c[m][1], c[m][1], ss));
    }
  }
  ss = warp_sum(ss);
  const float scale = 1.0f / (sqrtf(ss) + 1e-8f);
#pragma unroll
  for (int m = 0; m < kMaxBlocks; ++m) {
    c[m][0] *= scale;
    c[m][1] *= scale;
  }
}

}  // namespace kdn
