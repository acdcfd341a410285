// lift.cu -- standalone feature-lift kernel (kdn_fwht_lift).
//
// phi(x) = c / (||c|| + 1e-8), c = amp cos(tau^-1 H D3 H D2 H D1 x / 8 + b) per 64-wide block
// (kernels/fwht.py:113-130).  The traffic is 64 input elements + D output elements per vector, so
// the kernel should be HBM bound; what stands in the way is instruction issue: 24 64-point
// transforms and D cosines per vector.
//
// Main kernel (lift_pair_kernel): a vector lives in a lane pair, 32 elements per lane (element
// 32 hb + r in register r of half hb).  Five of a transform's six butterfly levels run inside
// the registers and only the last crosses the pair (one shuffle per element), against five
// shuffle levels when a vector is spread over a whole warp.  A warp lifts 16 vectors at a time.
// The norm needs all D features, so each lane stages its unnormalised cosines in shared memory (fp32,
// or fp16 when the output is bf16; the sum of squares is taken in fp32 before that rounding).  Once
// the pair's sum of squares is known, the warp reads the 16 rows back, scales them and writes them
// with coalesced 16-byte stores (16 contiguous output rows per warp).  The next group's
// inputs are loaded before the current group is computed.  Cosines: the argument is reduced by the
// nearest multiple of 2 pi (Cody and Waite's method, 2 pi split in two floats), then __cosf.
//
// Fallback (lift_kernel): one warp per vector, for inputs or outputs that are not 16-byte aligned.
#include <cuda_fp16.h>

#include <type_traits>

#include "kdn_internal.h"
#include "lift.cuh"

namespace kdn {
namespace {

constexpr int kGroupVecs = 16;                              // vectors per warp and group
constexpr int kStageElems = kGroupVecs * 64 * kMaxBlocks;   // one warp's staging: 16 rows of up to 512 features
constexpr int kStageBudget = 192 * 1024;                    // shared memory for the staging of all warps

// Staging element: fp16 for bf16 outputs (its rounding, 2^-12, is well inside the output's 2^-9), fp32 for
// fp32 outputs.  The half-size staging doubles the warps an SM holds (12 instead of 6).
template <typename TO>
struct LiftStage {
  using S = typename std::conditional<sizeof(TO) == 2, __half, float>::type;
  static constexpr int kWarps = kStageBudget / (kStageElems * int(sizeof(S)));
};
constexpr int kMaxLiftWarps = 12;

// cos(z): z - k 2 pi with k = rint(z / 2 pi), the product subtracted in two parts (2 pi = C1 + C2,
// C1 the float nearest 2 pi, C2 the float nearest the remainder), then the hardware cosine on
// [-pi, pi].
__device__ __forceinline__ float cos_reduced(float z) {
  constexpr float kInv2Pi = 0.159154937f;
  constexpr float kC1 = 6.28318548f;      // float(2 pi)
  constexpr float kC2 = -1.74845553e-7f;  // float(2 pi - kC1)
  const float k = rintf(z * kInv2Pi);
  float r = fmaf(-k, kC1, z);
  r = fmaf(-k, kC2, r);
  return __cosf(r);
}

// element r of this lane's half: flip its sign where bit r of w is set
__device__ __forceinline__ void apply_sign_word(float (&v)[32], uint32_t w) {
#pragma unroll
  for (int r = 0; r < 32; ++r) v[r] = __int_as_float(__float_as_int(v[r]) ^ ((w << (31 - r)) & 0x80000000u));
}

// H v over the 64 elements of a lane pair: levels 1..16 in registers, level 32 across the pair
__device__ __forceinline__ void fwht_pair(float (&v)[32], float lane_sign) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1)
#pragma unroll
    for (int r = 0; r < 32; ++r)
      if ((r & h) == 0) {
        const float a = v[r], b = v[r + h];
        v[r] = a + b;
        v[r + h] = a - b;
      }
#pragma unroll
  for (int r = 0; r < 32; ++r) {
    const float p = __shfl_xor_sync(0xffffffffu, v[r], 1);
    v[r] = fmaf(lane_sign, v[r], p);  // low half: v + p; high half: p - v
  }
}

template <typename T>
__device__ __forceinline__ void load_half(const T* p, float (&x)[32]) {  // 32 elements, 16-byte loads
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = reinterpret_cast<const uint4*>(p)[c];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        x[8 * c + 2 * i] = t.x;
        x[8 * c + 2 * i + 1] = t.y;
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 t = reinterpret_cast<const float4*>(p)[c];
      x[4 * c] = t.x;
      x[4 * c + 1] = t.y;
      x[4 * c + 2] = t.z;
      x[4 * c + 3] = t.w;
    }
  }
}

// 16-byte chunk c of staged row g, XOR-swizzled so that the 8 lanes of a quarter warp, which write
// the same chunk of 8 different (row, half) pairs, land on 8 different bank groups.  fp32 rows: 128
// chunks of 4 features, lane half hb writes chunks 8 hb .. 8 hb + 7 of each 16; fp16 rows: 64 chunks of
// 8 features, half hb writes chunks 4 hb .. 4 hb + 3 of each 8.
__device__ __forceinline__ int stage_chunk(int g, int c) { return c ^ ((2 * g + ((c >> 3) & 1)) & 7); }
__device__ __forceinline__ int stage_chunk_h(int g, int c) { return c ^ (g & 3); }

template <typename TI, typename TO>
__global__ void __launch_bounds__(32 * LiftStage<TO>::kWarps, 1)
    lift_pair_kernel(const TI* __restrict__ x, TO* __restrict__ out, int64_t n, ProjParams P) {
  using S = typename LiftStage<TO>::S;
  constexpr int kLiftWarps = LiftStage<TO>::kWarps;
  constexpr bool kHalfStage = sizeof(S) == 2;
  extern __shared__ float4 lift_smem[];
  __shared__ float s_phase[64 * kMaxBlocks];
  __shared__ uint32_t s_signs[kMaxBlocks][3][2];
  __shared__ float s_scale[kMaxLiftWarps][kGroupVecs];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int M = P.M, D = 64 * M;
  for (int i = threadIdx.x; i < D; i += blockDim.x) s_phase[i] = P.phase[i];
  if (threadIdx.x < kMaxBlocks * 3 * 2) {
    const int m = threadIdx.x / 6, s = (threadIdx.x / 2) % 3, h = threadIdx.x & 1;
    s_signs[m][s][h] = uint32_t(P.sign_bits[m][s] >> (32 * h));
  }
  __syncthreads();
  S* stage = reinterpret_cast<S*>(lift_smem) + warp * kStageElems;
  const int g = lane >> 1, hb = lane & 1;
  const float lane_sign = hb ? -1.f : 1.f;
  const float t8 = 0.125f * P.tau_inv;  // the butterfly's 1/8 folded into tau^-1 (a power of two: exact)
  const int64_t groups = (n + kGroupVecs - 1) / kGroupVecs;
  const int64_t stride = int64_t(gridDim.x) * kLiftWarps;
  int64_t grp = int64_t(blockIdx.x) * kLiftWarps + warp;
  float xn[32];
  auto load_group = [&](int64_t gi) {
    const int64_t vec = gi * kGroupVecs + g;
    if (gi < groups && vec < n) {
      load_half(x + vec * kDk + 32 * hb, xn);
    } else {
#pragma unroll
      for (int r = 0; r < 32; ++r) xn[r] = 0.f;
    }
  };
  load_group(grp);
  for (; grp < groups; grp += stride) {
    float xv[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) xv[r] = xn[r];
    load_group(grp + stride);  // in flight while this group is computed
    float ss = 0.f;
#pragma unroll 1
    for (int m = 0; m < M; ++m) {
      float v[32];
#pragma unroll
      for (int r = 0; r < 32; ++r) v[r] = xv[r];
      apply_sign_word(v, s_signs[m][0][hb]);
      fwht_pair(v, lane_sign);
      apply_sign_word(v, s_signs[m][1][hb]);
      fwht_pair(v, lane_sign);
      apply_sign_word(v, s_signs[m][2][hb]);
      fwht_pair(v, lane_sign);
      const float4* ph = reinterpret_cast<const float4*>(s_phase + 64 * m + 32 * hb);
      float4* srow = reinterpret_cast<float4*>(stage + g * (64 * kMaxBlocks));
      if constexpr (kHalfStage) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 b0 = ph[2 * k], b1 = ph[2 * k + 1];
          const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          float c[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            c[e] = cos_reduced(fmaf(v[8 * k + e], t8, bb[e]));
            ss = fmaf(c[e], c[e], ss);
          }
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __half2 h2 = __floats2half2_rn(c[2 * e], c[2 * e + 1]);
            w[e] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          reinterpret_cast<uint4*>(srow)[stage_chunk_h(g, 8 * m + 4 * hb + k)] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 b = ph[k];
          float4 c;
          c.x = cos_reduced(fmaf(v[4 * k], t8, b.x));
          c.y = cos_reduced(fmaf(v[4 * k + 1], t8, b.y));
          c.z = cos_reduced(fmaf(v[4 * k + 2], t8, b.z));
          c.w = cos_reduced(fmaf(v[4 * k + 3], t8, b.w));
          ss = fmaf(c.x, c.x, fmaf(c.y, c.y, fmaf(c.z, c.z, fmaf(c.w, c.w, ss))));
          srow[stage_chunk(g, 16 * m + 8 * hb + k)] = c;
        }
      }
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    // phi = amp cos / (amp ||cos|| + 1e-8)
    if (hb == 0) s_scale[warp][g] = P.amp / fmaf(P.amp, sqrtf(ss), 1e-8f);
    __syncwarp();
    // write back: 16 contiguous rows of D outputs, 16 bytes per lane and store
    constexpr int kOut = 16 / sizeof(TO);  // outputs per store
    const int per_row = D / kOut;
    const int64_t row0 = grp * kGroupVecs;
    for (int L = lane; L < kGroupVecs * per_row; L += 32) {
      const int go = L / per_row, q = L - go * per_row;
      if (row0 + go >= n) break;  // rows are in order: the rest of this warp's rows are past n as well
      const float sc = s_scale[warp][go];
      const float4* srow = reinterpret_cast<const float4*>(stage + go * (64 * kMaxBlocks));
      TO* dst = out + (row0 + go) * D + int64_t(q) * kOut;
      if constexpr (sizeof(TO) == 2) {  // fp16 staging: one chunk holds the store's 8 features
        const uint4 u = reinterpret_cast<const uint4*>(srow)[stage_chunk_h(go, q)];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
          const __nv_bfloat162 b2 = __floats2bfloat162_rn(f.x * sc, f.y * sc);
          o[e] = *reinterpret_cast<const uint32_t*>(&b2);
        }
        *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
      } else {
        const float4 a = srow[stage_chunk(go, q)];
        *reinterpret_cast<float4*>(dst) = make_float4(a.x * sc, a.y * sc, a.z * sc, a.w * sc);
      }
    }
    __syncwarp();  // the staging and the scales are rewritten by the next group
  }
}

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

template <typename TI, typename TO>
cudaError_t launch_pair(const void* x, void* out, int64_t n, const ProjParams& P, cudaStream_t stream) {
  constexpr int kLiftWarps = LiftStage<TO>::kWarps;
  constexpr size_t kLiftSmem = size_t(kLiftWarps) * kStageElems * sizeof(typename LiftStage<TO>::S);
  static_assert(kLiftWarps <= kMaxLiftWarps, "lift warps exceed the scale table");
  static bool configured = false;  // the attribute is per function; setting it twice is harmless
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(lift_pair_kernel<TI, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               int(kLiftSmem));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t groups = (n + kGroupVecs - 1) / kGroupVecs;
  int64_t blocks = (groups + kLiftWarps - 1) / kLiftWarps;
  if (blocks > sms) blocks = sms;  // persistent: one CTA per SM
  lift_pair_kernel<TI, TO><<<dim3(unsigned(blocks)), 32 * kLiftWarps, kLiftSmem, stream>>>(
      static_cast<const TI*>(x), static_cast<TO*>(out), n, P);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_lift(const void* x, int x_dtype, void* out, int out_dtype, int64_t n, const ProjParams& P,
                        cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const bool a16 = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  if (a16 && P.M >= 1 && P.M <= kMaxBlocks) {
    const bool ib = x_dtype == KDN_DTYPE_BF16, ob = out_dtype == KDN_DTYPE_BF16;
    if (ib && ob) return launch_pair<__nv_bfloat16, __nv_bfloat16>(x, out, n, P, stream);
    if (ib) return launch_pair<__nv_bfloat16, float>(x, out, n, P, stream);
    if (ob) return launch_pair<float, __nv_bfloat16>(x, out, n, P, stream);
    return launch_pair<float, float>(x, out, n, P, stream);
  }
  const int threads = 256;
  int64_t blocks = (n + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  lift_kernel<<<dim3(unsigned(blocks)), threads, 0, stream>>>(x, x_dtype, out, out_dtype, n, P);
  return cudaGetLastError();
}

}  // namespace kdn
