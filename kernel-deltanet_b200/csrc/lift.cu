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
// Tensor-core kernels (bf16 inputs, D = 512, Omega exact in bf16): the three transforms of a block are one
// dense product x Omega^T.  Omega = H D3 H D2 H D1 / 8 has entries that are integers / 8; when those are
// exact in bf16 (checked on the host per sign pattern) a bf16 x bf16 product with fp32 accumulation is
// exact up to the accumulation order.  A persistent CTA per SM builds Omega once (64 KiB, the B operand),
// then per tile of 128 vectors one thread issues 16 tcgen05 MMAs into 512 TMEM columns (lanes = vectors,
// columns = features).
//  - lift_tc_bf16_kernel (bf16 outputs): the features are two halves of 256 columns with their own
//    products, handed back to the issuer half by half, so the next tile's products overlap this tile's
//    epilogue.  Sixteen epilogue warps take the cosines and sums of squares (pass 1, cosines staged as
//    fp16), then scale whole rows and write them as 512-byte stores (pass 2).
//  - lift_tc_kernel (fp32 outputs): eight epilogue warps (two per TMEM lane quarter, one column half each)
//    write the cosines back in place in TMEM with the sums of squares, then scale each row and write it
//    through a per-warp staging buffer as coalesced 16-byte stores; the next tile's inputs load during
//    the epilogue.
// KDN_LIFT_PATH=pair forces the CUDA-core kernel.
//
// Fallback (lift_kernel): one warp per vector, for inputs or outputs that are not 16-byte aligned.
#include <cuda_fp16.h>

#include <type_traits>

#include <stdlib.h>
#include <string.h>

#include <atomic>

#include "kdn_internal.h"
#include "lift.cuh"
#include "tc_chunk.cuh"

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

// Raise Kernel's dynamic shared-memory limit to `bytes` on device `dev`.  The attribute is held per
// function and device, so it is set once for each device a kernel runs on (one table per kernel; devices
// past the table: on every call).
template <auto Kernel>
cudaError_t allow_smem(int bytes, int dev) {
  constexpr int kDevs = 64;
  static std::atomic<bool> done[kDevs] = {};  // host threads may launch on several devices at once
  if (dev >= 0 && dev < kDevs && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && dev >= 0 && dev < kDevs) done[dev].store(true, std::memory_order_release);
  return e;
}

// ---------------------------------------------------------------- tensor-core lift
__device__ int g_lift_error;

namespace tcl {
constexpr int kTile = 128;                      // vectors per tile (MMA M)
constexpr int kEpiWarps = 8;                    // 2 per TMEM lane quarter, one column half each
constexpr int kIssuerWarp = kEpiWarps;          // warp 8 issues the MMAs
constexpr int kThreads = 32 * (kEpiWarps + 1);
constexpr uint32_t kWaitLimit = 1u << 24;
// shared memory, bytes from a 1024-aligned base
constexpr uint32_t OFF_OMG = 0;       // 64 KiB Omega (bf16, K-major SW128), slice s (features 128 s..) at 16 KiB s
constexpr uint32_t OFF_X = 65536;     // 16 KiB input tile (bf16, K-major SW128, 128 rows x 64)
constexpr uint32_t OFF_STG = 81920;   // fp32 outputs: 8 x 4 KiB write-back staging (32 rows x 128 B), one per
                                      // epilogue warp; bf16 outputs: 128 KiB of fp16 cosines (128 rows x 1 KiB,
                                      // row r's 16-byte chunk c at c ^ (r & 7))
constexpr uint32_t OFF_PH = 212992;   // 2 KiB phase b[512]
constexpr uint32_t OFF_SS = 215040;   // 1 KiB sums of squares [column half][row]
constexpr uint32_t OFF_BAR = 216064;  // 2 mbarriers + TMEM address
constexpr uint32_t kSmem = OFF_BAR + 64 + 1024;  // + alignment slack
}  // namespace tcl

__global__ void __launch_bounds__(tcl::kThreads, 1) lift_tc_kernel(const __nv_bfloat16* __restrict__ x,
                                                                   float* __restrict__ out, int64_t n, ProjParams P) {
  using namespace tcl;
  extern __shared__ uint8_t lift_tc_raw[];
  uint8_t* sm;
  {
    const uint32_t a = tc::smem_u32(lift_tc_raw);
    sm = lift_tc_raw + ((1024u - (a & 1023u)) & 1023u);
  }
  const uint32_t sbase = tc::smem_u32(sm);
  float* ph = reinterpret_cast<float*>(sm + OFF_PH);
  float* ssx = reinterpret_cast<float*>(sm + OFF_SS);
  uint64_t* bar_lift = reinterpret_cast<uint64_t*>(sm + OFF_BAR);       // a tile's products are done
  uint64_t* bar_ready = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 8);  // TMEM read out, next tile loaded
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tiles = (n + kTile - 1) / kTile;
  bool ok = true;

  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(bar_lift, 1);
    tc::mbar_init(bar_ready, kEpiWarps);
    tc::fence_mbar_init();
  }
  tcc::build_omega(sm + OFF_OMG, P, warp, lane, kThreads / 32);
  for (int i = tid; i < 64 * kMaxBlocks; i += kThreads) ph[i] = P.phase[i];
  // the 128 x 64 input tile of tile t, swizzled for the A operand (epilogue threads; rows past n read as 0)
  auto load_tile = [&](int64_t t) {
    const int64_t row0 = t * kTile;
    for (int j = tid; j < kTile * 8; j += 32 * kEpiWarps) {
      const int r = j >> 3, c = j & 7;
      const bool in = row0 + r < n;
      tc::cp_async16(sbase + OFF_X + tc::sw128_offset(r, 8 * c), x + (in ? (row0 + r) * kDk + 8 * c : 0),
                     in ? 16 : 0);
    }
    tc::cp_async_commit();
  };
  if (warp < kEpiWarps && int64_t(blockIdx.x) < tiles) load_tile(blockIdx.x);
  if (warp < kEpiWarps) tc::cp_async_wait_all();
  tc::fence_proxy_async_smem();  // Omega (generic stores) and the first tile, for the tensor core
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  if (warp == kIssuerWarp) {
    if (lane == 0) {
      const uint32_t id = tc::idesc_bf16_f32(128, 128, false, false);
      uint32_t pr = 0;
      int64_t i = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
        if (i > 0) {  // the epilogue has read TMEM out and loaded this tile
          ok &= tc::mbar_wait_bounded(bar_ready, pr, kWaitLimit);
          pr ^= 1;
          tc::fence_after_sync();
        }
#pragma unroll
        for (int s = 0; s < 4; ++s)
#pragma unroll
          for (int k0 = 0; k0 < 64; k0 += 16)
            tc::mma_ss(tmem + 128 * s, tc::smem_desc_sw128(sbase + OFF_X + 2 * k0, 16, 1024),
                       tc::smem_desc_sw128(sbase + OFF_OMG + s * 16384 + 2 * k0, 16, 1024), id, k0 > 0);
        tc::mma_commit(bar_lift);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3, ch = warp >> 2;  // TMEM lane quarter, column half
    const uint32_t lane_off = uint32_t(32 * q) << 16;
    const int row = 32 * q + lane;           // this thread's row of the tile
    uint8_t* stg = sm + OFF_STG + warp * 4096;
    uint32_t pl = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      ok &= tc::mbar_wait_bounded(bar_lift, pl, kWaitLimit);
      pl ^= 1;
      tc::fence_after_sync();
      const int64_t next = t + gridDim.x;
      if (next < tiles) load_tile(next);  // the products of this tile have read the input tile
      // fp32 outputs. Pass 1: cos(tau^-1 z + b) in place in TMEM, sum of squares over this half's 256 features
      float ss = 0.f;
#pragma unroll 1
      for (int cc = 0; cc < 8; ++cc) {
        const uint32_t col = 256 * ch + 32 * cc;
        float z[32];
        tc::tmem_ld32(tmem + lane_off + col, z);
        tc::tmem_ld_wait();
        const float4* b4 = reinterpret_cast<const float4*>(ph + col);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 b = b4[j >> 2];
          z[j] = cos_reduced(fmaf(z[j], P.tau_inv, b.x));
          z[j + 1] = cos_reduced(fmaf(z[j + 1], P.tau_inv, b.y));
          z[j + 2] = cos_reduced(fmaf(z[j + 2], P.tau_inv, b.z));
          z[j + 3] = cos_reduced(fmaf(z[j + 3], P.tau_inv, b.w));
          ss = fmaf(z[j], z[j], fmaf(z[j + 1], z[j + 1], fmaf(z[j + 2], z[j + 2], fmaf(z[j + 3], z[j + 3], ss))));
        }
        tc::tmem_st32(tmem + lane_off + col, z);
      }
      tc::tmem_st_wait();
      ssx[128 * ch + row] = ss;
      tc::named_bar_sync(1, 32 * kEpiWarps);
      // phi = amp cos / (amp ||cos|| + 1e-8)
      const float scale = P.amp / fmaf(P.amp, sqrtf(ssx[row] + ssx[128 + row]), 1e-8f);
      // pass 2: 128 output bytes (32 fp32 columns) of each row at a time, scaled and transposed through the
      // staging (row r's 16-byte chunk c at c ^ (r & 7)) into whole-row 128-byte stores
      const int64_t grow0 = t * kTile + 32 * q;  // output row of lane 0 of this warp
#pragma unroll 1
      for (int blk = 0; blk < 8; ++blk) {
        const uint32_t col = 256 * ch + 32 * blk;
        float a[32];
        tc::tmem_ld32(tmem + lane_off + col, a);
        tc::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<float4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) =
              make_float4(a[4 * c] * scale, a[4 * c + 1] * scale, a[4 * c + 2] * scale, a[4 * c + 3] * scale);
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int jj = lane + 32 * k, r = jj >> 3, c = jj & 7;
          const uint4 u = *reinterpret_cast<const uint4*>(stg + r * 128 + ((c ^ (r & 7)) << 4));
          if (grow0 + r < n)
            *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(out + (grow0 + r) * 512 + col) + 16 * c) = u;
        }
        __syncwarp();  // the staging is rewritten by the next block
      }
      if (next < tiles) {  // TMEM read out and the next tile in shared memory: hand both to the issuer
        tc::cp_async_wait_all();
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_ready);
      }
    }
  }
  if (!ok) record_device_error(&g_lift_error, kErrLiftWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

// Tensor-core lift for bf16 outputs.  The 512 features of a tile are two halves of 256 TMEM columns,
// produced by separate groups of products: the issuer gives half hh of the next tile its products as
// soon as the epilogue has read half hh of this tile, so the tensor core never waits for a whole
// epilogue and the epilogue never waits for the tensor core.  Sixteen epilogue warps (four per TMEM
// lane quarter; warp w takes columns 64 (w >> 2) .. +63 of each half) take the cosines (plain __cosf:
// its error, about 2e-6 for the arguments here, is far inside the bf16 output's 2^-9) and the
// per-row sums of squares, staging the cosines as fp16 (2^-12 rounding); then each warp scales eight
// whole rows and writes each as two coalesced 512-byte stores.
namespace tcl2 {
constexpr int kTile = 128;
constexpr int kEpiWarps = 16;
constexpr int kIssuerWarp = kEpiWarps;  // warp 16 issues the MMAs
constexpr int kThreads = 32 * (kEpiWarps + 1);
constexpr uint32_t kWaitLimit = 1u << 24;
constexpr uint32_t OFF_OMG = 0;       // 64 KiB Omega (bf16, K-major SW128), slice s at 16 KiB s
constexpr uint32_t OFF_X = 65536;     // 16 KiB input tile (bf16, K-major SW128, 128 rows x 64)
constexpr uint32_t OFF_STG = 81920;   // 128 KiB fp16 cosines: row r at 1 KiB r, its 16-byte chunk c at c ^ (r & 7)
constexpr uint32_t OFF_PH = 212992;   // 2 KiB phase b[512]
constexpr uint32_t OFF_SS = 215040;   // 2 KiB partial sums of squares [column quarter][row]
constexpr uint32_t OFF_BAR = 217088;  // 5 mbarriers + TMEM address
constexpr uint32_t kSmem = OFF_BAR + 64 + 1024;  // + alignment slack
}  // namespace tcl2

__global__ void __launch_bounds__(tcl2::kThreads, 1) lift_tc_bf16_kernel(const __nv_bfloat16* __restrict__ x,
                                                                         __nv_bfloat16* __restrict__ out,
                                                                         int64_t n, ProjParams P) {
  using namespace tcl2;
  extern __shared__ uint8_t lift_tc2_raw[];
  uint8_t* sm;
  {
    const uint32_t a = tc::smem_u32(lift_tc2_raw);
    sm = lift_tc2_raw + ((1024u - (a & 1023u)) & 1023u);
  }
  const uint32_t sbase = tc::smem_u32(sm);
  float* ph = reinterpret_cast<float*>(sm + OFF_PH);
  float* ssx = reinterpret_cast<float*>(sm + OFF_SS);
  uint64_t* bar_half = reinterpret_cast<uint64_t*>(sm + OFF_BAR);       // [2] products of half hh done
  uint64_t* bar_free = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 16);  // [2] half hh read out (16 warps)
  uint64_t* bar_in = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 32);    // next input tile loaded (16 warps)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 40);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t tiles = (n + kTile - 1) / kTile;
  bool ok = true;

  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int hh = 0; hh < 2; ++hh) {
      tc::mbar_init(&bar_half[hh], 1);
      tc::mbar_init(&bar_free[hh], kEpiWarps);
    }
    tc::mbar_init(bar_in, kEpiWarps);
    tc::fence_mbar_init();
  }
  tcc::build_omega(sm + OFF_OMG, P, warp, lane, kThreads / 32);
  for (int i = tid; i < 64 * kMaxBlocks; i += kThreads) ph[i] = P.phase[i];
  // the 128 x 64 input tile of tile t, swizzled for the A operand (epilogue threads; rows past n read as 0)
  auto load_tile = [&](int64_t t) {
    const int64_t row0 = t * kTile;
    for (int j = tid; j < kTile * 8; j += 32 * kEpiWarps) {
      const int r = j >> 3, c = j & 7;
      const bool in = row0 + r < n;
      tc::cp_async16(sbase + OFF_X + tc::sw128_offset(r, 8 * c), x + (in ? (row0 + r) * kDk + 8 * c : 0),
                     in ? 16 : 0);
    }
    tc::cp_async_commit();
  };
  if (warp < kEpiWarps && int64_t(blockIdx.x) < tiles) load_tile(blockIdx.x);
  if (warp < kEpiWarps) tc::cp_async_wait_all();
  tc::fence_proxy_async_smem();  // Omega (generic stores) and the first tile, for the tensor core
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  if (warp == kIssuerWarp) {
    if (lane == 0) {
      const uint32_t id = tc::idesc_bf16_f32(128, 128, false, false);
      uint32_t pf = 0, pin = 0;  // pf: bits per half
      int64_t i = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
        if (i > 0) {  // this tile's inputs are in shared memory
          ok &= tc::mbar_wait_bounded(bar_in, pin, kWaitLimit);
          pin ^= 1;
        }
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if (i > 0) {  // the epilogue has read half hh of the previous tile
            ok &= tc::mbar_wait_bounded(&bar_free[hh], (pf >> hh) & 1u, kWaitLimit);
            pf ^= 1u << hh;
          }
          tc::fence_after_sync();
#pragma unroll
          for (int s = 2 * hh; s < 2 * hh + 2; ++s)
#pragma unroll
            for (int k0 = 0; k0 < 64; k0 += 16)
              tc::mma_ss(tmem + 128 * s, tc::smem_desc_sw128(sbase + OFF_X + 2 * k0, 16, 1024),
                         tc::smem_desc_sw128(sbase + OFF_OMG + s * 16384 + 2 * k0, 16, 1024), id, k0 > 0);
          tc::mma_commit(&bar_half[hh]);
        }
      }
    }
    __syncwarp();
  } else if (warp < kEpiWarps) {
    const int q = warp & 3, cq = warp >> 2;  // TMEM lane quarter, column quarter of each half
    const uint32_t lane_off = uint32_t(32 * q) << 16;
    const int row = 32 * q + lane;           // this thread's row of the tile in pass 1
    uint8_t* cs = sm + OFF_STG;
    uint32_t ph_half = 0;  // bits per half
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int64_t next = t + gridDim.x;
      // pass 1: cos(tau^-1 z + b) of this thread's row over 2 x 64 features, the sum of their squares,
      // the cosines staged as fp16; each half of TMEM goes back to the issuer once read
      float ss = 0.f;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        ok &= tc::mbar_wait_bounded(&bar_half[hh], (ph_half >> hh) & 1u, kWaitLimit);
        ph_half ^= 1u << hh;
        tc::fence_after_sync();
        if (hh == 1 && next < tiles) load_tile(next);  // every product of this tile has read the input tile
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const uint32_t col = 256 * hh + 64 * cq + 32 * cc;
          float z[32];
          tc::tmem_ld32(tmem + lane_off + col, z);
          tc::tmem_ld_wait();
          const float4* b4 = reinterpret_cast<const float4*>(ph + col);
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 b = b4[j >> 2];
            z[j] = __cosf(fmaf(z[j], P.tau_inv, b.x));
            z[j + 1] = __cosf(fmaf(z[j + 1], P.tau_inv, b.y));
            z[j + 2] = __cosf(fmaf(z[j + 2], P.tau_inv, b.z));
            z[j + 3] = __cosf(fmaf(z[j + 3], P.tau_inv, b.w));
            ss = fmaf(z[j], z[j], fmaf(z[j + 1], z[j + 1], fmaf(z[j + 2], z[j + 2], fmaf(z[j + 3], z[j + 3], ss))));
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // chunk col / 8 + k of this thread's row
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __half2 h2 = __floats2half2_rn(z[8 * k + 2 * e], z[8 * k + 2 * e + 1]);
              w[e] = *reinterpret_cast<const uint32_t*>(&h2);
            }
            const int c = int(col >> 3) + k;
            *reinterpret_cast<uint4*>(cs + row * 1024 + ((c ^ (row & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bar_free[hh]);
      }
      ssx[128 * cq + row] = ss;
      if (next < tiles) {  // the next tile's inputs are in place: its products may start
        tc::cp_async_wait_all();
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_in);
      }
      tc::named_bar_sync(1, 32 * kEpiWarps);  // every row's cosines and partial sums are in shared memory
      // pass 2: rows 8 warp .. 8 warp + 7, each as two 512-byte stores; phi = amp cos / (amp ||cos|| + 1e-8).
      // Lane k forms row 8 warp + k's scale (the norm and the quotient by the hardware reciprocal square
      // root and reciprocal: about 1e-7 relative, far inside bf16's 2^-9) and passes it to the warp.
      float sc_own;
      {
        const int r = 8 * warp + (lane & 7);
        const float ssr = ssx[r] + ssx[128 + r] + ssx[256 + r] + ssx[384 + r];
        sc_own = __fdividef(P.amp, fmaf(P.amp, ssr * rsqrtf(ssr), 1e-8f));
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = 8 * warp + k;  // r & 7 == k: the swizzle below folds to constants
        const float sc = __shfl_sync(0xffffffffu, sc_own, k);
        const int64_t grow = t * kTile + r;
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          const int c = 32 * hb + lane;
          const uint4 u = *reinterpret_cast<const uint4*>(cs + r * 1024 + ((c ^ (r & 7)) << 4));
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(f.x * sc, f.y * sc);
            o[e] = *reinterpret_cast<const uint32_t*>(&b2);
          }
          if (grow < n) *reinterpret_cast<uint4*>(out + grow * 512 + 8 * c) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      tc::named_bar_sync(1, 32 * kEpiWarps);  // the staging and the partial sums take the next tile
    }
  }
  if (!ok) record_device_error(&g_lift_error, kErrLiftWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

cudaError_t launch_tc(const void* x, void* out, int64_t n, const ProjParams& P, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = allow_smem<lift_tc_kernel>(int(tcl::kSmem), dev)) != cudaSuccess) return e;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = (n + tcl::kTile - 1) / tcl::kTile;
  const int64_t blocks = tiles < sms ? tiles : sms;  // persistent: one CTA per SM
  lift_tc_kernel<<<dim3(unsigned(blocks)), tcl::kThreads, tcl::kSmem, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<float*>(out), n, P);
  return cudaGetLastError();
}

cudaError_t launch_tc_bf16(const void* x, void* out, int64_t n, const ProjParams& P, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = allow_smem<lift_tc_bf16_kernel>(int(tcl2::kSmem), dev)) != cudaSuccess) return e;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = (n + tcl2::kTile - 1) / tcl2::kTile;
  const int64_t blocks = tiles < sms ? tiles : sms;  // persistent: one CTA per SM
  lift_tc_bf16_kernel<<<dim3(unsigned(blocks)), tcl2::kThreads, tcl2::kSmem, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(out), n, P);
  return cudaGetLastError();
}

template <typename TI, typename TO>
cudaError_t launch_pair(const void* x, void* out, int64_t n, const ProjParams& P, cudaStream_t stream) {
  constexpr int kLiftWarps = LiftStage<TO>::kWarps;
  constexpr size_t kLiftSmem = size_t(kLiftWarps) * kStageElems * sizeof(typename LiftStage<TO>::S);
  static_assert(kLiftWarps <= kMaxLiftWarps, "lift warps exceed the scale table");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = allow_smem<lift_pair_kernel<TI, TO>>(int(kLiftSmem), dev)) != cudaSuccess) return e;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t groups = (n + kGroupVecs - 1) / kGroupVecs;
  int64_t blocks = (groups + kLiftWarps - 1) / kLiftWarps;
  if (blocks > sms) blocks = sms;  // persistent: one CTA per SM
  lift_pair_kernel<TI, TO><<<dim3(unsigned(blocks)), 32 * kLiftWarps, kLiftSmem, stream>>>(
      static_cast<const TI*>(x), static_cast<TO*>(out), n, P);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_lift(const void* x, int x_dtype, void* out, int out_dtype, int64_t n, const ProjParams& P,
                        bool omega_bf16_exact, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const bool a16 = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const char* path = getenv("KDN_LIFT_PATH");
  const bool force_pair = path && strcmp(path, "pair") == 0;
  if (a16 && omega_bf16_exact && P.M == kMaxBlocks && x_dtype == KDN_DTYPE_BF16 && !force_pair)
    return out_dtype == KDN_DTYPE_BF16 ? launch_tc_bf16(x, out, n, P, stream) : launch_tc(x, out, n, P, stream);
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

cudaError_t lift_read_error(cudaStream_t stream, int* code) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_lift_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  if (h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_lift_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  }
  *code = h;
  return cudaSuccess;
}

}  // namespace kdn
