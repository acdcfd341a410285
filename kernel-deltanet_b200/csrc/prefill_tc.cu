// prefill_tc.cu -- fused tensor-core chunked prefill (KDN_MODE_BF16), sm_100a.
//
// One 4-CTA cluster per sequence.  CTA m of the cluster owns features
// [128m, 128m+128) of D = 512 -- i.e. Omega blocks 2m, 2m+1 -- and the matching
// 128 columns of the state S [d_v=64, D].  Per chunk of C = 64 tokens:
//
//   1  k,q rows of the chunk -> shared memory (bf16, K-major, 128B swizzle)
//   2  tcgen05: Z = [k;q] Omega_m^T  (M=128 tokens, N=128 features, K=64)   [TMEM]
//      Omega_m is built once per CTA from the sign bits by the warp butterfly.
//   3  u = cos(tau_inv z + b) -> feature tile F = [U_k; U_q] (un-normalised), kept
//      as a bf16 pair F = F_hi + F_lo, and per-token partial sums of squares
//   4  tcgen05: [G;P]_m = F_hi U_k,hi^T + F_lo U_k,hi^T + F_hi U_k,lo^T,
//               [X;Yq]_m = F_hi S_m^T + F_lo S_m^T                          [TMEM]
//      (the lo terms keep outputs of near-orthogonal tokens accurate)
//   5  DSMEM reduce-scatter of G, P, X, Yq and of the sums of squares
//   6  owner CTA sums its 16-row blocks, applies the feature norms
//      (phi = u / (||u|| + 1e-8) becomes a row/column scaling), all-gathers G and X
//   7  every CTA: A = beta_i exp(g_i - g_j) G_ij (j<i), T = (I + A)^-1 (blocked),
//      R = beta (v - exp(g) X), E = T R; CTA m writes output rows [16m, 16m+16):
//      y_i = exp(g_{i-1}) Yq_i + sum_{j<i} exp(g_{i-1} - g_j) P_ij e_j
//      E'' = exp(g_{C-1} - g_j) s_kj E_j split into bf16 hi + lo
//   8  tcgen05: S_m^T = exp(g_{C-1}) S_m^T + U_k^T E''_hi + U_k^T E''_lo       [TMEM, fp32]
//   9  S_m^T -> bf16 operand tile for the next chunk's step 4
//
// The algebra is the same as the CUDA-core path (prefill_simt.cu) and the
// reference chunk step kernels/fused_kernel_deltanet.py:95-149; only the
// products run on tcgen05 with bf16 operands and fp32 accumulation.  The state
// stays fp32 in tensor memory for the whole sequence.
#include <math.h>

#include "kdn_internal.h"
#include "lift.cuh"
#include "tc_prims.cuh"

namespace kdn {
namespace {

__device__ int g_tc_error;

constexpr int kG = 4;          // CTAs per sequence (cluster size)
constexpr int kC = 64;         // chunk
constexpr int kDV = 64;        // value dim
constexpr int kThr = 256;      // threads per CTA
constexpr uint32_t kWaitLimit = 1u << 24;

// shared-memory map (bytes from a 1024-aligned base)
constexpr uint32_t OFF_OMG = 0;        // Omega slice, B operand: 128 features x 64 (16 KiB)
constexpr uint32_t OFF_XIN = 16384;    // [k;q] inputs, A operand: 128 x 64 (16 KiB); then F_lo K-block 0
                                       // (steps 3-4); then T (64x64 f32, step 7)
constexpr uint32_t OFF_F = 32768;      // features [U_k;U_q]: 2 K-blocks x 128 rows x 128 B (32 KiB)
constexpr uint32_t OFF_SB = 65536;     // S_m bf16, B operand: 128 features x 64 dv (16 KiB); reused as E (64x64 f32)
constexpr uint32_t OFF_EB = 81920;     // F_lo K-block 1 (steps 3-4); then E'' hi, lo: 2 x 64 x 64 (16 KiB)
constexpr uint32_t OFF_RS = 98304;     // reduce-scatter inbox: [4 src][4 mat][16][64] f32 (64 KiB)
constexpr uint32_t OFF_AG = 163840;    // all-gather inbox: [4 src][G,X][16][64] f32 (32 KiB)
constexpr uint32_t OFF_SS = 196608;    // sums of squares inbox: [4 src][128] f32 (2 KiB)
constexpr uint32_t OFF_MYP = 198656;   // owned rows of P~ (16 x 64 f32, 4 KiB)
constexpr uint32_t OFF_MYY = 202752;   // owned rows of Yq~ (4 KiB)
constexpr uint32_t OFF_MT = 206848;    // block-inverse scratch 16 x 48 f32 (3 KiB)
constexpr uint32_t OFF_SSP = 209920;   // per-half partial sums of squares [2][128] (1 KiB)
constexpr uint32_t OFF_SC = 210944;    // token scales s[128] (512 B)
constexpr uint32_t OFF_GL = 211456;    // g[64] cumulative log decay (256 B)
constexpr uint32_t OFF_BT = 211712;    // beta[64] (256 B)
constexpr uint32_t OFF_BAR = 211968;   // mbarrier (8 B) + TMEM address (4 B)
constexpr uint32_t kSmemBytes = 212032 + 1024;  // + alignment slack

// TMEM columns
constexpr uint32_t COL_S = 0;     // S_m^T: lanes = features, 64 cols = dv (fp32 master)
constexpr uint32_t COL_Z = 64;    // lift result: lanes = tokens, 128 cols = features
constexpr uint32_t COL_GP = 192;  // [G;P]: lanes = [k;q] tokens, 64 cols = k tokens
constexpr uint32_t COL_XY = 256;  // [X;Yq]: lanes = [k;q] tokens, 64 cols = dv

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
};

__device__ __forceinline__ float cos_reduced(float x) {
  // Cody-Waite reduction to [-pi, pi] (two-constant split of 2*pi), then the
  // hardware cosine, accurate there to ~2^-21 absolute.
  const float k = rintf(x * 0.15915494309189535f);
  float r = fmaf(-k, 6.28318548202514648f, x);
  r = fmaf(-k, -1.7484556e-07f, r);
  return __cosf(r);
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __cluster_dims__(kG, 1, 1) __launch_bounds__(kThr, 1)
    prefill_tc_kernel(TcArgs a, ProjParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm;
  {
    const uint32_t s = tc::smem_u32(smem_raw);
    sm = smem_raw + ((1024u - (s & 1023u)) & 1023u);
  }
  const uint32_t sbase = tc::smem_u32(sm);
  float* Ts = reinterpret_cast<float*>(sm + OFF_XIN);  // [64][64]
  float* Es = reinterpret_cast<float*>(sm + OFF_SB);   // [64][64]
  float* RS = reinterpret_cast<float*>(sm + OFF_RS);
  float* AG = reinterpret_cast<float*>(sm + OFF_AG);
  float* SS = reinterpret_cast<float*>(sm + OFF_SS);
  float* myP = reinterpret_cast<float*>(sm + OFF_MYP);
  float* myY = reinterpret_cast<float*>(sm + OFF_MYY);
  float* Mt = reinterpret_cast<float*>(sm + OFF_MT);
  float* ssp = reinterpret_cast<float*>(sm + OFF_SSP);
  float* sc = reinterpret_cast<float*>(sm + OFF_SC);
  float* gl = reinterpret_cast<float*>(sm + OFF_GL);
  float* bt = reinterpret_cast<float*>(sm + OFF_BT);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t m = tc::cluster_ctarank();
  const int64_t n = blockIdx.y;
  const int quarter = warp & 3, half = warp >> 2;
  const int trow = quarter * 32 + lane;  // TMEM lane owned by this thread
  const uint32_t lane_off = uint32_t(quarter * 32) << 16;
  const float amp = P.amp;
  bool ok = true;
  uint32_t phase = 0;

  // ---------------------------------------------------------------- setup
  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(mbar, 1);
    tc::fence_mbar_init();
  }
  // Omega slice: feature row fl (block 2m + fl/64, row fl%64), column d = input index.
  for (int job = warp; job < 128; job += kThr / 32) {
    const int bl = job >> 6, d = job & 63;
    const int blk = 2 * int(m) + bl;
    const float x0 = (d == 2 * lane) ? 1.f : 0.f, x1 = (d == 2 * lane + 1) ? 1.f : 0.f;
    float u0, u1;
    structured_block(x0, x1, P.sign_bits[blk], lane, u0, u1);
    const int f0 = 64 * bl + 2 * lane;
    *reinterpret_cast<__nv_bfloat16*>(sm + OFF_OMG + tc::sw128_offset(f0, d)) = __float2bfloat16_rn(u0);
    *reinterpret_cast<__nv_bfloat16*>(sm + OFF_OMG + tc::sw128_offset(f0 + 1, d)) = __float2bfloat16_rn(u1);
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  // state: S_m^T master (fp32, TMEM) and its bf16 operand copy
  {
    float v[32];
    const int f = 128 * int(m) + trow;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int dv = 32 * half + j;
      v[j] = a.S0 ? a.S0[(n * kDV + dv) * 512 + f] : 0.f;
    }
    tc::tmem_st32(tmem + lane_off + COL_S + 32 * half, v);
    tc::tmem_st_wait();
#pragma unroll
    for (int c4 = 0; c4 < 4; ++c4) {
      uint4 pk;
      pk.x = pack_bf16(v[8 * c4 + 0], v[8 * c4 + 1]);
      pk.y = pack_bf16(v[8 * c4 + 2], v[8 * c4 + 3]);
      pk.z = pack_bf16(v[8 * c4 + 4], v[8 * c4 + 5]);
      pk.w = pack_bf16(v[8 * c4 + 6], v[8 * c4 + 7]);
      *reinterpret_cast<uint4*>(sm + OFF_SB + tc::sw128_offset(trow, 32 * half + 8 * c4)) = pk;
    }
  }
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  tc::cluster_sync();  // all CTAs of the cluster are running before any DSMEM access
  tc::fence_after_sync();

  const uint32_t id_lift = tc::idesc_bf16_f32(128, 128, false, false);
  const uint32_t id_gp = tc::idesc_bf16_f32(128, 64, false, false);
  const uint32_t id_xy = tc::idesc_bf16_f32(128, 64, false, true);
  const uint32_t id_ds = tc::idesc_bf16_f32(128, 64, true, true);

  for (int c = 0; c < a.NC; ++c) {
    const int64_t t0 = int64_t(c) * kC;
    // ------------------------------------------------ 1. inputs and gates
    {
      const int r = tid >> 1, hh = tid & 1;  // row r of [k;q], 32-element half hh
      const int64_t t = t0 + (r & 63);
      const void* src = r < 64 ? a.k : a.q;
      uint4 pk[4];
      if (t < a.T) {
        if (a.in_dtype == KDN_DTYPE_BF16) {
          const uint4* s4 = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src) +
                                                           (n * a.T + t) * 64 + 32 * hh);
#pragma unroll
          for (int i = 0; i < 4; ++i) pk[i] = s4[i];
        } else {
          const float4* s4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) +
                                                             (n * a.T + t) * 64 + 32 * hh);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 x0 = s4[2 * i], x1 = s4[2 * i + 1];
            pk[i] = make_uint4(pack_bf16(x0.x, x0.y), pack_bf16(x0.z, x0.w), pack_bf16(x1.x, x1.y),
                               pack_bf16(x1.z, x1.w));
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) pk[i] = make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(sm + OFF_XIN + tc::sw128_offset(r, 32 * hh + 8 * i)) = pk[i];
      if (warp == 0) {  // beta and the inclusive scan of log clamp(decay, 1e-5, 1)
        float lg[2], bb[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int64_t tt = t0 + 2 * lane + e;
          float b = 0.f, dec = 1.f;
          if (tt < a.T) {
            b = ld_as_f32(a.beta, a.gate_dtype, n * a.T + tt);
            if (a.decay) dec = ld_as_f32(a.decay, a.gate_dtype, n * a.T + tt);
          }
          bb[e] = b;
          lg[e] = logf(fminf(fmaxf(dec, 1e-5f), 1.0f));
        }
        float s = lg[0] + lg[1];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, s, o);
          if (lane >= o) s += y;
        }
        const float excl = s - (lg[0] + lg[1]);
        gl[2 * lane] = excl + lg[0];
        gl[2 * lane + 1] = s;
        bt[2 * lane] = bb[0];
        bt[2 * lane + 1] = bb[1];
      }
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ------------------------------------------------ 2. lift product
    if (tid == 0) {
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) {
        const uint64_t ad = tc::smem_desc_sw128(sbase + OFF_XIN + 2 * k0, 16, 1024);
        const uint64_t bd = tc::smem_desc_sw128(sbase + OFF_OMG + 2 * k0, 16, 1024);
        tc::mma_bf16_ss(tmem + COL_Z, ad, bd, id_lift, k0 > 0);
      }
      tc::mma_commit(mbar);
    }
    __syncwarp();
    ok &= tc::mbar_wait_bounded(mbar, phase, kWaitLimit);
    phase ^= 1;
    tc::fence_after_sync();

    // ------------------------------------------------ 3. features
    {
      float ss = 0.f;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        float z[32];
        tc::tmem_ld32(tmem + lane_off + COL_Z + 64 * half + 32 * part, z);
        tc::tmem_ld_wait();
        const int fl0 = 64 * half + 32 * part;       // local feature of z[0]
        const float* ph = P.phase + 128 * m + fl0;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          float u[8], lo[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            u[j] = cos_reduced(fmaf(z[8 * c4 + j], P.tau_inv, __ldg(ph + 8 * c4 + j)));
            ss = fmaf(u[j], u[j], ss);
            lo[j] = u[j] - __bfloat162float(__float2bfloat16_rn(u[j]));
          }
          const uint32_t off = tc::sw128_offset(trow, 32 * part + 8 * c4);
          *reinterpret_cast<uint4*>(sm + OFF_F + half * 16384 + off) =
              make_uint4(pack_bf16(u[0], u[1]), pack_bf16(u[2], u[3]), pack_bf16(u[4], u[5]), pack_bf16(u[6], u[7]));
          *reinterpret_cast<uint4*>(sm + (half ? OFF_EB : OFF_XIN) + off) = make_uint4(
              pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]), pack_bf16(lo[4], lo[5]), pack_bf16(lo[6], lo[7]));
        }
      }
      ssp[half * 128 + trow] = ss;
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ------------------------------------------------ 4. Gram and state products
    if (tid == 0) {
#pragma unroll
      for (int k0 = 0; k0 < 128; k0 += 16) {
        const uint64_t fd = tc::smem_desc_sw128(sbase + OFF_F + (k0 >> 6) * 16384 + 2 * (k0 & 63), 16, 1024);
        const uint64_t ld = tc::smem_desc_sw128(sbase + ((k0 >> 6) ? OFF_EB : OFF_XIN) + 2 * (k0 & 63), 16, 1024);
        const uint64_t sd = tc::smem_desc_sw128(sbase + OFF_SB + 128 * k0, 16384, 1024);
        tc::mma_bf16_ss(tmem + COL_GP, fd, fd, id_gp, k0 > 0);
        tc::mma_bf16_ss(tmem + COL_GP, ld, fd, id_gp, true);
        tc::mma_bf16_ss(tmem + COL_GP, fd, ld, id_gp, true);
        tc::mma_bf16_ss(tmem + COL_XY, fd, sd, id_xy, k0 > 0);
        tc::mma_bf16_ss(tmem + COL_XY, ld, sd, id_xy, true);
      }
      tc::mma_commit(mbar);
    }
    __syncwarp();
    ok &= tc::mbar_wait_bounded(mbar, phase, kWaitLimit);
    phase ^= 1;
    tc::fence_after_sync();

    // ------------------------------------------------ 5. reduce-scatter to the row owners
    {
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        float v[32];
        tc::tmem_ld32(tmem + lane_off + (which ? COL_XY : COL_GP) + 32 * half, v);
        tc::tmem_ld_wait();
        const int mat = 2 * which + (trow >= 64 ? 1 : 0);  // 0 G, 1 P, 2 X, 3 Yq
        const int i = trow & 63;
        const uint32_t owner = uint32_t(i >> 4);
        const uint32_t laddr = sbase + OFF_RS + 4u * uint32_t((((m * 4 + mat) * 16 + (i & 15)) * 64) + 32 * half);
        const uint32_t raddr = tc::mapa(laddr, owner);
#pragma unroll
        for (int j = 0; j < 8; ++j) tc::st_cluster_v4(raddr + 16 * j, v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
      if (tid < 128) {
        const float ss = ssp[tid] + ssp[128 + tid];
        const uint32_t laddr = sbase + OFF_SS + 4u * (m * 128 + tid);
#pragma unroll
        for (uint32_t o = 0; o < kG; ++o) tc::st_cluster_f32(tc::mapa(laddr, o), ss);
      }
    }
    tc::fence_before_sync();
    tc::cluster_sync();
    tc::fence_after_sync();

    // ------------------------------------------------ 6. owner reduction, norms, all-gather
    if (tid < 128) {
      const float ss = SS[tid] + SS[128 + tid] + SS[256 + tid] + SS[384 + tid];
      sc[tid] = amp / (amp * sqrtf(ss) + 1e-8f);  // phi = s * u
    }
    __syncthreads();
    {
      // 4 matrices x 16 rows x 64 cols = 4096 values, 16 per thread (4 float4)
#pragma unroll
      for (int rep = 0; rep < 4; ++rep) {
        const int e4 = tid + kThr * rep;  // float4 index in [0, 1024)
        const int mat = e4 >> 8, lr = (e4 >> 4) & 15, c0 = (e4 & 15) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < kG; ++s) {
          const float4 x = *reinterpret_cast<const float4*>(RS + (((s * 4 + mat) * 16 + lr) * 64) + c0);
          acc.x += x.x;
          acc.y += x.y;
          acc.z += x.z;
          acc.w += x.w;
        }
        const int i = 16 * int(m) + lr;  // row within the 64-row matrix
        float rs;
        float cs[4] = {1.f, 1.f, 1.f, 1.f};
        if (mat == 0) {
          rs = sc[i];
#pragma unroll
          for (int q = 0; q < 4; ++q) cs[q] = sc[c0 + q];
        } else if (mat == 1) {
          rs = sc[64 + i];
#pragma unroll
          for (int q = 0; q < 4; ++q) cs[q] = sc[c0 + q];
        } else if (mat == 2) {
          rs = sc[i];
        } else {
          rs = sc[64 + i];
        }
        acc.x *= rs * cs[0];
        acc.y *= rs * cs[1];
        acc.z *= rs * cs[2];
        acc.w *= rs * cs[3];
        if (mat == 1) {
          *reinterpret_cast<float4*>(myP + lr * 64 + c0) = acc;
        } else if (mat == 3) {
          *reinterpret_cast<float4*>(myY + lr * 64 + c0) = acc;
        } else {
          const int slot_mat = mat == 0 ? 0 : 1;
          const uint32_t laddr = sbase + OFF_AG + 4u * uint32_t(((m * 2 + slot_mat) * 16 + lr) * 64 + c0);
#pragma unroll
          for (uint32_t o = 0; o < kG; ++o) tc::st_cluster_v4(tc::mapa(laddr, o), acc.x, acc.y, acc.z, acc.w);
        }
      }
    }
    tc::fence_before_sync();
    tc::cluster_sync();
    tc::fence_after_sync();

    // ------------------------------------------------ 7. small chunk algebra (CUDA cores)
    auto AGG = [&](int i) -> float* { return AG + ((i >> 4) * 2 + 0) * 1024 + (i & 15) * 64; };
    auto AGX = [&](int i) -> float* { return AG + ((i >> 4) * 2 + 1) * 1024 + (i & 15) * 64; };
    // A in place of G~, R in place of X~, T zero-initialised
    for (int e = tid; e < 64 * 64; e += kThr) {
      const int i = e >> 6, j = e & 63;
      float* g = AGG(i) + j;
      *g = (j < i) ? bt[i] * __expf(gl[i] - gl[j]) * (*g) : 0.f;
      float vv = 0.f;
      const int64_t t = t0 + i;
      if (t < a.T) vv = ld_as_f32(a.v, a.in_dtype, (n * a.T + t) * kDV + j);
      float* x = AGX(i) + j;
      *x = bt[i] * (vv - __expf(gl[i]) * (*x));
      Ts[e] = 0.f;
    }
    __syncthreads();
    // diagonal 16x16 blocks of T = (I + A)^-1, one warp per block, one lane per column
    if (warp < 4 && lane < 16) {
      const int I = warp, j = lane;
      float tcol[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float s = (r == j) ? 1.f : 0.f;
        const float* arow = AGG(16 * I + r) + 16 * I;
#pragma unroll
        for (int kk = 0; kk < r; ++kk) s = fmaf(-arow[kk], tcol[kk], s);
        tcol[r] = (r >= j) ? s : 0.f;
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) Ts[(16 * I + r) * 64 + 16 * I + j] = tcol[r];
    }
    __syncthreads();
    // off-diagonal block rows: T_IJ = -T_II sum_{K=J}^{I-1} A_IK T_KJ
    for (int I = 1; I < 4; ++I) {
      const int W = 16 * I;
      for (int e = tid; e < 16 * W; e += kThr) {
        const int r = e / W, j = e % W;
        const float* arow = AGG(W + r);
        float s = 0.f;
        for (int kk = j; kk < W; ++kk) s = fmaf(arow[kk], Ts[kk * 64 + j], s);
        Mt[r * 48 + j] = s;
      }
      __syncthreads();
      for (int e = tid; e < 16 * W; e += kThr) {
        const int r = e / W, j = e % W;
        float s = 0.f;
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) s = fmaf(Ts[(W + r) * 64 + W + kk], Mt[kk * 48 + j], s);
        Ts[(W + r) * 64 + j] = -s;
      }
      __syncthreads();
    }
    // E = T R  (thread: column v, rows ig, ig+4, ...)
    {
      const int v = tid & 63, ig = tid >> 6;
#pragma unroll 4
      for (int rr = 0; rr < 16; ++rr) {
        const int i = ig + 4 * rr;
        float s = 0.f;
        for (int j = 0; j <= i; ++j) s = fmaf(Ts[i * 64 + j], AGX(j)[v], s);
        Es[i * 64 + v] = s;
      }
    }
    // Aq rows owned by this CTA (in place of P~): P~_ij exp(g_{i-1} - g_j), j < i
    for (int e = tid; e < 16 * 64; e += kThr) {
      const int lr = e >> 6, j = e & 63, i = 16 * int(m) + lr;
      const float gp = i > 0 ? gl[i - 1] : 0.f;
      myP[e] = (j < i) ? myP[e] * __expf(gp - gl[j]) : 0.f;
    }
    __syncthreads();
    // outputs y for rows [16m, 16m+16)
    {
      const int v = tid & 63, rg = tid >> 6;
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const int lr = rg + 4 * rr, i = 16 * int(m) + lr;
        const float gp = i > 0 ? __expf(gl[i - 1]) : 1.f;
        float s = gp * myY[lr * 64 + v];
        for (int j = 0; j < i; ++j) s = fmaf(myP[lr * 64 + j], Es[j * 64 + v], s);
        const int64_t t = t0 + i;
        if (t < a.T) st_from_f32(a.y, a.y_dtype, (n * a.T + t) * kDV + v, s);
      }
    }
    // E'' = exp(g_{C-1} - g_j) s_kj E_j, bf16 hi + lo, MN-major (token rows, dv contiguous)
    for (int e = tid; e < 64 * 8; e += kThr) {
      const int j = e >> 3, c8 = (e & 7) * 8;
      const float w = __expf(gl[63] - gl[j]) * sc[j];
      float hi[8], lo[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float x = w * Es[j * 64 + c8 + q];
        hi[q] = __bfloat162float(__float2bfloat16_rn(x));
        lo[q] = x - hi[q];
      }
      const uint32_t off = tc::sw128_offset(j, c8);
      *reinterpret_cast<uint4*>(sm + OFF_EB + off) =
          make_uint4(pack_bf16(hi[0], hi[1]), pack_bf16(hi[2], hi[3]), pack_bf16(hi[4], hi[5]), pack_bf16(hi[6], hi[7]));
      *reinterpret_cast<uint4*>(sm + OFF_EB + 8192 + off) =
          make_uint4(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]), pack_bf16(lo[4], lo[5]), pack_bf16(lo[6], lo[7]));
    }
    // decay of the carried state
    {
      const float gC = __expf(gl[63]);
      if (gC != 1.0f) {
        float v[32];
        tc::tmem_ld32(tmem + lane_off + COL_S + 32 * half, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] *= gC;
        tc::tmem_st32(tmem + lane_off + COL_S + 32 * half, v);
        tc::tmem_st_wait();
      }
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ------------------------------------------------ 8. state update
    if (tid == 0) {
#pragma unroll
      for (int part = 0; part < 2; ++part) {
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16) {
          const uint64_t ad = tc::smem_desc_sw128(sbase + OFF_F + 128 * k0, 16384, 1024);
          const uint64_t bd = tc::smem_desc_sw128(sbase + OFF_EB + 8192 * part + 128 * k0, 8192, 1024);
          tc::mma_bf16_ss(tmem + COL_S, ad, bd, id_ds, true);
        }
      }
      tc::mma_commit(mbar);
    }
    __syncwarp();
    ok &= tc::mbar_wait_bounded(mbar, phase, kWaitLimit);
    phase ^= 1;
    tc::fence_after_sync();

    // ------------------------------------------------ 9. bf16 operand copy of the state
    {
      float v[32];
      tc::tmem_ld32(tmem + lane_off + COL_S + 32 * half, v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint4 pk = make_uint4(pack_bf16(v[8 * c4], v[8 * c4 + 1]), pack_bf16(v[8 * c4 + 2], v[8 * c4 + 3]),
                              pack_bf16(v[8 * c4 + 4], v[8 * c4 + 5]), pack_bf16(v[8 * c4 + 6], v[8 * c4 + 7]));
        *reinterpret_cast<uint4*>(sm + OFF_SB + tc::sw128_offset(trow, 32 * half + 8 * c4)) = pk;
      }
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }

  // ---------------------------------------------------------------- output state
  {
    float v[32];
    tc::tmem_ld32(tmem + lane_off + COL_S + 32 * half, v);
    tc::tmem_ld_wait();
    const int f = 128 * int(m) + trow;
#pragma unroll
    for (int j = 0; j < 32; ++j) a.S_out[(n * kDV + 32 * half + j) * 512 + f] = v[j];
  }
  if (!ok && lane == 0) record_device_error(&g_tc_error, 2);
  tc::fence_before_sync();
  tc::cluster_sync();  // no CTA leaves while a peer may still address its shared memory
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

}  // namespace

bool tc_prefill_supported(int D, int dv, int C, const ProjParams& P) {
  if (D != 512 || dv != kDV || C != kC) return false;
  // the Omega entries (integers / 8) must be exact in bf16 for the lift product
  for (int m = 0; m < 8; ++m) {
    for (int d = 0; d < 64; ++d) {
      double col[64];
      for (int i = 0; i < 64; ++i) col[i] = (i == d) ? ((P.sign_bits[m][0] >> i) & 1 ? -1.0 : 1.0) : 0.0;
      for (int s = 0; s < 3; ++s) {
        if (s > 0)
          for (int i = 0; i < 64; ++i)
            if ((P.sign_bits[m][s] >> i) & 1) col[i] = -col[i];
        for (int h = 1; h < 64; h <<= 1)
          for (int i = 0; i < 64; ++i)
            if (!(i & h)) {
              const double x = col[i], y = col[i + h];
              col[i] = x + y;
              col[i + h] = x - y;
            }
      }
      for (int i = 0; i < 64; ++i) {
        const float v = float(col[i] / 8.0);
        if (float(__float2bfloat16_rn(v)) != v) return false;
      }
    }
  }
  return true;
}

cudaError_t launch_tc_prefill(const PrefillProblem& p, const ProjParams& P, cudaStream_t stream) {
  TcArgs a;
  a.q = p.q;
  a.k = p.k;
  a.v = p.v;
  a.in_dtype = p.in_dtype;
  a.beta = p.beta;
  a.decay = p.decay;
  a.gate_dtype = p.gate_dtype;
  a.S0 = p.S0;
  a.y = p.y;
  a.y_dtype = p.y_dtype;
  a.S_out = p.S_out;
  a.T = p.T;
  a.NC = int((p.T + kC - 1) / kC);
  cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
  if (e != cudaSuccess) return e;
  prefill_tc_kernel<<<dim3(kG, unsigned(p.N)), kThr, kSmemBytes, stream>>>(a, P);
  return cudaGetLastError();
}

cudaError_t tc_read_error(cudaStream_t stream, int* code) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  if (h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  }
  *code = h;
  return cudaSuccess;
}

}  // namespace kdn
