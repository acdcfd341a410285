// prefill_tc.cu -- fused tensor-core chunked prefill (KDN_MODE_BF16), sm_100a.
//
// One 4-CTA cluster per sequence.  CTA m of the cluster owns features
// [128m, 128m+128) of D = 512 -- Omega blocks 2m, 2m+1 -- and the matching 128
// columns of the state S [d_v=64, D].  Per chunk of C = 64 tokens:
//
//   1  gates (beta, cumulative log decay); k,q rows were prefetched by cp.async
//      into a K-major 128B-swizzled bf16 tile during the previous chunk
//   2  tcgen05 (bf16): Z = [k;q] Omega_m^T (M=128 tokens, N=128 features, K=64)  [TMEM]
//      Omega_m is built once per CTA from the sign bits by the warp butterfly
//      and is exact in bf16 (integers / 8).
//   3  u = cos(tau_inv z + b) -> fp16 feature tile F = [U_k; U_q] (un-normalised)
//      and per-token partial sums of squares
//   4  tcgen05 (fp16): [G;P]_m = F U_k^T, [X;Yq]_m = F S_m^T                   [TMEM]
//   5  DSMEM reduce-scatter of the G, P, X, Yq partials and the sums of squares
//   6  the owner CTA of each 16-row block sums it, applies the feature norms
//      (phi = u / (||u|| + 1e-8) becomes a row/column scaling) and all-gathers G, X
//   7  every CTA (CUDA cores): A_ij = beta_i exp(g_i - g_j) G_ij (j<i),
//      R = beta (v - exp(g) X), E = (I + A)^-1 R by blocked forward substitution;
//      CTA m writes output rows [16m, 16m+16):
//      y_i = exp(g_{i-1}) Yq_i + sum_{j<i} exp(g_{i-1} - g_j) P_ij e_j;
//      E'' = exp(g_{C-1} - g_j) s_kj e_j (fp16)
//   8  tcgen05 (fp16): S_m^T = exp(g_{C-1}) S_m^T + U_k^T E''                   [TMEM, fp32]
//   9  S_m^T -> fp16 operand tile for the next chunk's step 4
//
// The algebra is the one of the CUDA-core path (prefill_simt.cu), itself the
// reference chunk step kernels/fused_kernel_deltanet.py:95-149 rearranged.
// Products run on tcgen05 with fp32 accumulation; the features, the state
// operand copy and E'' are fp16 (10-bit mantissa, |values| well inside range);
// the state itself stays fp32 in tensor memory for the whole sequence.
#include <cuda_fp16.h>
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
constexpr uint32_t OFF_OMG = 0;        // 16 KiB Omega slice (bf16, K-major; B of the lift)
constexpr uint32_t OFF_XIN = 16384;    // 16 KiB [k;q] chunk inputs (bf16, K-major; A of the lift)
constexpr uint32_t OFF_F = 32768;      // 32 KiB features [U_k;U_q] (fp16), 2 K-blocks x 128 rows x 128 B
constexpr uint32_t OFF_SB = 65536;     // 16 KiB S_m operand (fp16, MN-major); in step 7: E (64x64 f32)
constexpr uint32_t OFF_EB = 81920;     // 8 KiB  E'' (fp16, MN-major)
constexpr uint32_t OFF_VB = 90112;     // 16 KiB v rows of the chunk (input dtype, row-major)
constexpr uint32_t OFF_RS = 106496;    // 64 KiB reduce-scatter inbox [4 src][G,P,X,Yq][16][64] f32
constexpr uint32_t OFF_AG = 172032;    // 32 KiB all-gather inbox [4 src][G,X][16][64] f32
constexpr uint32_t OFF_SS = 204800;    // 2 KiB  sums-of-squares inbox [4 src][128] f32
constexpr uint32_t OFF_MYP = 206848;   // 4 KiB  owned rows of P~, then of Aq
constexpr uint32_t OFF_MYY = 210944;   // 4 KiB  owned rows of Yq~
constexpr uint32_t OFF_TD = 215040;    // 4 KiB  diagonal 16x16 blocks of (I + A)^-1
constexpr uint32_t OFF_US = 219136;    // 4 KiB  forward-substitution scratch [16][64]
constexpr uint32_t OFF_PH = 223232;    // 512 B  phase of this CTA's 128 features
constexpr uint32_t OFF_GL = 223744;    // 256 B  g_i (cumulative log decay)
constexpr uint32_t OFF_BT = 224000;    // 256 B  beta_i
constexpr uint32_t OFF_EG = 224256;    // 256 B  exp(g_i)
constexpr uint32_t OFF_EGP = 224512;   // 256 B  exp(g_{i-1})
constexpr uint32_t OFF_W = 224768;     // 256 B  exp(g_{C-1} - g_i)
constexpr uint32_t OFF_SSP = 225024;   // 1 KiB  partial sums of squares [2][128]
constexpr uint32_t OFF_SC = 226048;    // 512 B  token scales s = amp / (amp ||u|| + 1e-8)
constexpr uint32_t OFF_BAR = 226560;   // mbarrier (8 B) + TMEM address (4 B)
constexpr uint32_t kSmemBytes = 226576 + 1024;  // + alignment slack

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
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  const float lim = 65504.f;  // saturate instead of overflowing to inf
  __half2 h = __floats2half2_rn(fminf(fmaxf(a, -lim), lim), fminf(fmaxf(b, -lim), lim));
  return *reinterpret_cast<uint32_t*>(&h);
}

// k and q rows of chunk c -> the K-major swizzled input tile (bf16 inputs only)
__device__ __forceinline__ void prefetch_kq(const TcArgs& a, int64_t n, int c, uint32_t xin, int tid) {
  const int r = tid >> 1, hh = tid & 1;
  const int64_t t = int64_t(c) * kC + (r & 63);
  const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(r < 64 ? a.k : a.q);
  const bool in = t < a.T;
  const __nv_bfloat16* src = base + (in ? (n * a.T + t) * 64 + 32 * hh : 0);
#pragma unroll
  for (int i = 0; i < 4; ++i) tc::cp_async16(xin + tc::sw128_offset(r, 32 * hh + 8 * i), src + (in ? 8 * i : 0), in ? 16 : 0);
}

// v rows of chunk c -> row-major tile in the input dtype
__device__ __forceinline__ void prefetch_v(const TcArgs& a, int64_t n, int c, uint32_t vb, int tid) {
  const int esz = a.in_dtype == KDN_DTYPE_BF16 ? 2 : 4;
  const int cpr = 64 * esz / 16;  // 16-byte pieces per row
  const char* base = reinterpret_cast<const char*>(a.v);
  for (int e = tid; e < 64 * cpr; e += kThr) {
    const int row = e / cpr, cc = e % cpr;
    const int64_t t = int64_t(c) * kC + row;
    const bool in = t < a.T;
    const char* src = base + (in ? ((n * a.T + t) * 64) * esz + 16 * cc : 0);
    tc::cp_async16(vb + row * 64 * esz + 16 * cc, src, in ? 16 : 0);
  }
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
  float* Es = reinterpret_cast<float*>(sm + OFF_SB);  // [64][64] during step 7
  float* RS = reinterpret_cast<float*>(sm + OFF_RS);
  float* AG = reinterpret_cast<float*>(sm + OFF_AG);
  float* SS = reinterpret_cast<float*>(sm + OFF_SS);
  float* myP = reinterpret_cast<float*>(sm + OFF_MYP);
  float* myY = reinterpret_cast<float*>(sm + OFF_MYY);
  float* TD = reinterpret_cast<float*>(sm + OFF_TD);
  float* US = reinterpret_cast<float*>(sm + OFF_US);
  float* ph = reinterpret_cast<float*>(sm + OFF_PH);
  float* gl = reinterpret_cast<float*>(sm + OFF_GL);
  float* bt = reinterpret_cast<float*>(sm + OFF_BT);
  float* eg = reinterpret_cast<float*>(sm + OFF_EG);
  float* egp = reinterpret_cast<float*>(sm + OFF_EGP);
  float* wdec = reinterpret_cast<float*>(sm + OFF_W);
  float* ssp = reinterpret_cast<float*>(sm + OFF_SSP);
  float* sc = reinterpret_cast<float*>(sm + OFF_SC);
  uint64_t* mbar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 8);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t m = tc::cluster_ctarank();
  const int64_t n = blockIdx.y;
  const int quarter = warp & 3, half = warp >> 2;
  const int trow = quarter * 32 + lane;  // TMEM lane owned by this thread
  const uint32_t lane_off = uint32_t(quarter * 32) << 16;
  const float amp = P.amp;
  const bool kq_async = a.in_dtype == KDN_DTYPE_BF16;
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
  if (tid < 128) ph[tid] = P.phase[128 * m + tid];
  if (kq_async) prefetch_kq(a, n, 0, sbase + OFF_XIN, tid);
  prefetch_v(a, n, 0, sbase + OFF_VB, tid);
  tc::cp_async_commit();
  // gates of the next chunk are carried in registers of warp 0
  float nb[2] = {0.f, 0.f}, nd[2] = {1.f, 1.f};
  if (warp == 0) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int64_t tt = 2 * lane + e;
      if (tt < a.T) {
        nb[e] = ld_as_f32(a.beta, a.gate_dtype, n * a.T + tt);
        if (a.decay) nd[e] = ld_as_f32(a.decay, a.gate_dtype, n * a.T + tt);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  // state: S_m^T master (fp32, TMEM) and its fp16 operand copy
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
      uint4 pk = make_uint4(pack_f16(v[8 * c4], v[8 * c4 + 1]), pack_f16(v[8 * c4 + 2], v[8 * c4 + 3]),
                            pack_f16(v[8 * c4 + 4], v[8 * c4 + 5]), pack_f16(v[8 * c4 + 6], v[8 * c4 + 7]));
      *reinterpret_cast<uint4*>(sm + OFF_SB + tc::sw128_offset(trow, 32 * half + 8 * c4)) = pk;
    }
  }
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  tc::cluster_sync();  // all CTAs of the cluster are running before any DSMEM access
  tc::fence_after_sync();

  const uint32_t id_lift = tc::idesc_bf16_f32(128, 128, false, false);
  const uint32_t id_gp = tc::idesc_f16_f32(128, 64, false, false);
  const uint32_t id_xy = tc::idesc_f16_f32(128, 64, false, true);
  const uint32_t id_ds = tc::idesc_f16_f32(128, 64, true, true);
  auto AGG = [&](int i) -> float* { return AG + ((i >> 4) * 2 + 0) * 1024 + (i & 15) * 64; };
  auto AGX = [&](int i) -> float* { return AG + ((i >> 4) * 2 + 1) * 1024 + (i & 15) * 64; };

  for (int c = 0; c < a.NC; ++c) {
    const int64_t t0 = int64_t(c) * kC;
    const bool has_next = c + 1 < a.NC;
    // ------------------------------------------------ 1. inputs and gates
    tc::cp_async_wait_all();
    if (!kq_async) {  // fp32 inputs: load and round to bf16 here
      const int r = tid >> 1, hh = tid & 1;
      const int64_t t = t0 + (r & 63);
      const float* src = reinterpret_cast<const float*>(r < 64 ? a.k : a.q) + (n * a.T + t) * 64 + 32 * hh;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 pk = make_uint4(0, 0, 0, 0);
        if (t < a.T) {
          const float4 x0 = reinterpret_cast<const float4*>(src)[2 * i];
          const float4 x1 = reinterpret_cast<const float4*>(src)[2 * i + 1];
          pk = make_uint4(pack_bf16(x0.x, x0.y), pack_bf16(x0.z, x0.w), pack_bf16(x1.x, x1.y), pack_bf16(x1.z, x1.w));
        }
        *reinterpret_cast<uint4*>(sm + OFF_XIN + tc::sw128_offset(r, 32 * hh + 8 * i)) = pk;
      }
    }
    if (warp == 0) {  // beta, inclusive scan of log clamp(decay, 1e-5, 1), derived factors
      const float lg0 = logf(fminf(fmaxf(nd[0], 1e-5f), 1.0f)), lg1 = logf(fminf(fmaxf(nd[1], 1e-5f), 1.0f));
      float s = lg0 + lg1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += y;
      }
      const float g0 = s - lg1, g1 = s;
      const float gend = __shfl_sync(0xffffffffu, s, 31);
      const float gprev = __shfl_up_sync(0xffffffffu, g1, 1);
      gl[2 * lane] = g0;
      gl[2 * lane + 1] = g1;
      bt[2 * lane] = nb[0];
      bt[2 * lane + 1] = nb[1];
      eg[2 * lane] = __expf(g0);
      eg[2 * lane + 1] = __expf(g1);
      egp[2 * lane] = lane == 0 ? 1.f : __expf(gprev);
      egp[2 * lane + 1] = __expf(g0);
      wdec[2 * lane] = __expf(gend - g0);
      wdec[2 * lane + 1] = __expf(gend - g1);
      // gates of the next chunk (consumed at its step 1)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t tt = t0 + kC + 2 * lane + e;
        nb[e] = 0.f;
        nd[e] = 1.f;
        if (has_next && tt < a.T) {
          nb[e] = ld_as_f32(a.beta, a.gate_dtype, n * a.T + tt);
          if (a.decay) nd[e] = ld_as_f32(a.decay, a.gate_dtype, n * a.T + tt);
        }
      }
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ------------------------------------------------ 2. lift product (bf16)
    if (tid == 0) {
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) {
        const uint64_t ad = tc::smem_desc_sw128(sbase + OFF_XIN + 2 * k0, 16, 1024);
        const uint64_t bd = tc::smem_desc_sw128(sbase + OFF_OMG + 2 * k0, 16, 1024);
        tc::mma_ss(tmem + COL_Z, ad, bd, id_lift, k0 > 0);
      }
      tc::mma_commit(mbar);
    }
    __syncwarp();
    ok &= tc::mbar_wait_bounded(mbar, phase, kWaitLimit);
    phase ^= 1;
    tc::fence_after_sync();
    // the input tile is free again: prefetch the next chunk's k,q rows into it
    if (has_next && kq_async) prefetch_kq(a, n, c + 1, sbase + OFF_XIN, tid);
    tc::cp_async_commit();

    // ------------------------------------------------ 3. features (fp16)
    {
      float ss = 0.f;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        float z[32];
        tc::tmem_ld32(tmem + lane_off + COL_Z + 64 * half + 32 * part, z);
        tc::tmem_ld_wait();
        const float* phs = ph + 64 * half + 32 * part;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          float u[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            u[j] = cos_reduced(fmaf(z[8 * c4 + j], P.tau_inv, phs[8 * c4 + j]));
            ss = fmaf(u[j], u[j], ss);
          }
          *reinterpret_cast<uint4*>(sm + OFF_F + half * 16384 + tc::sw128_offset(trow, 32 * part + 8 * c4)) =
              make_uint4(pack_f16(u[0], u[1]), pack_f16(u[2], u[3]), pack_f16(u[4], u[5]), pack_f16(u[6], u[7]));
        }
      }
      ssp[half * 128 + trow] = ss;
    }
    tc::fence_proxy_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ------------------------------------------------ 4. Gram and state products (fp16)
    if (tid == 0) {
#pragma unroll
      for (int k0 = 0; k0 < 128; k0 += 16) {
        const uint64_t fd = tc::smem_desc_sw128(sbase + OFF_F + (k0 >> 6) * 16384 + 2 * (k0 & 63), 16, 1024);
        const uint64_t sd = tc::smem_desc_sw128(sbase + OFF_SB + 128 * k0, 16384, 1024);
        tc::mma_ss(tmem + COL_GP, fd, fd, id_gp, k0 > 0);
        tc::mma_ss(tmem + COL_XY, fd, sd, id_xy, k0 > 0);
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
#pragma unroll
    for (int rep = 0; rep < 4; ++rep) {
      const int e4 = tid + kThr * rep;  // float4 index over [4 mat][16 rows][16]
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
      const int i = 16 * int(m) + lr;
      const float rs = (mat == 0 || mat == 2) ? sc[i] : sc[64 + i];
      float cs[4] = {1.f, 1.f, 1.f, 1.f};
      if (mat < 2) {
#pragma unroll
        for (int q = 0; q < 4; ++q) cs[q] = sc[c0 + q];
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
        const uint32_t laddr = sbase + OFF_AG + 4u * uint32_t(((m * 2 + (mat >> 1)) * 16 + lr) * 64 + c0);
#pragma unroll
        for (uint32_t o = 0; o < kG; ++o) tc::st_cluster_v4(tc::mapa(laddr, o), acc.x, acc.y, acc.z, acc.w);
      }
    }
    tc::fence_before_sync();
    tc::cluster_sync();
    tc::fence_after_sync();

    // ------------------------------------------------ 7. small chunk algebra (CUDA cores)
    // A in place of G~, R in place of X~, Aq in place of the owned rows of P~
    {
      const bool vbf = a.in_dtype == KDN_DTYPE_BF16;
      for (int e = tid; e < 64 * 64; e += kThr) {
        const int i = e >> 6, j = e & 63;
        float* g = AGG(i) + j;
        *g = (j < i) ? bt[i] * __expf(gl[i] - gl[j]) * (*g) : 0.f;
        const float vv = vbf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(sm + OFF_VB)[e])
                             : reinterpret_cast<const float*>(sm + OFF_VB)[e];
        float* x = AGX(i) + j;
        *x = bt[i] * (vv - eg[i] * (*x));
      }
      for (int e = tid; e < 16 * 64; e += kThr) {
        const int lr = e >> 6, j = e & 63, i = 16 * int(m) + lr;
        myP[e] = (j < i) ? myP[e] * __expf((i > 0 ? gl[i - 1] : 0.f) - gl[j]) : 0.f;
      }
    }
    __syncthreads();
    if (has_next) prefetch_v(a, n, c + 1, sbase + OFF_VB, tid);  // v tile is free now
    tc::cp_async_commit();
    // diagonal 16x16 blocks of (I + A)^-1: one warp per block, one lane per column
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
      for (int r = 0; r < 16; ++r) TD[(I * 16 + r) * 16 + j] = tcol[r];
    }
    __syncthreads();
    // E = (I + A)^-1 R, block row by block row:
    //   U = R_I - sum_{J<I} A_IJ E_J;  E_I = T_II U
    {
      const int r = tid >> 4, c4 = (tid & 15) * 4;
      for (int I = 0; I < 4; ++I) {
        const float* arow = AGG(16 * I + r);
        float4 acc = *reinterpret_cast<const float4*>(AGX(16 * I + r) + c4);
        float4 acc2 = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int kk = 0; kk < 16 * I; kk += 2) {
          const float a0 = arow[kk], a1 = arow[kk + 1];
          const float4 e0 = *reinterpret_cast<const float4*>(Es + kk * 64 + c4);
          const float4 e1 = *reinterpret_cast<const float4*>(Es + (kk + 1) * 64 + c4);
          acc.x = fmaf(-a0, e0.x, acc.x);
          acc.y = fmaf(-a0, e0.y, acc.y);
          acc.z = fmaf(-a0, e0.z, acc.z);
          acc.w = fmaf(-a0, e0.w, acc.w);
          acc2.x = fmaf(-a1, e1.x, acc2.x);
          acc2.y = fmaf(-a1, e1.y, acc2.y);
          acc2.z = fmaf(-a1, e1.z, acc2.z);
          acc2.w = fmaf(-a1, e1.w, acc2.w);
        }
        acc.x += acc2.x;
        acc.y += acc2.y;
        acc.z += acc2.z;
        acc.w += acc2.w;
        *reinterpret_cast<float4*>(US + r * 64 + c4) = acc;
        __syncthreads();
        float4 e = make_float4(0.f, 0.f, 0.f, 0.f);
        const float* trw = TD + (I * 16 + r) * 16;
        for (int kk = 0; kk <= r; ++kk) {
          const float tv = trw[kk];
          const float4 u = *reinterpret_cast<const float4*>(US + kk * 64 + c4);
          e.x = fmaf(tv, u.x, e.x);
          e.y = fmaf(tv, u.y, e.y);
          e.z = fmaf(tv, u.z, e.z);
          e.w = fmaf(tv, u.w, e.w);
        }
        *reinterpret_cast<float4*>(Es + (16 * I + r) * 64 + c4) = e;
        __syncthreads();
      }
    }
    // outputs y for rows [16m, 16m+16)
    {
      const int r = tid >> 4, c4 = (tid & 15) * 4, i = 16 * int(m) + r;
      float4 y = *reinterpret_cast<const float4*>(myY + r * 64 + c4);
      const float gp = egp[i];
      y.x *= gp;
      y.y *= gp;
      y.z *= gp;
      y.w *= gp;
      const float* prow = myP + r * 64;
      for (int j = 0; j < i; ++j) {
        const float pv = prow[j];
        const float4 e = *reinterpret_cast<const float4*>(Es + j * 64 + c4);
        y.x = fmaf(pv, e.x, y.x);
        y.y = fmaf(pv, e.y, y.y);
        y.z = fmaf(pv, e.z, y.z);
        y.w = fmaf(pv, e.w, y.w);
      }
      const int64_t t = t0 + i;
      if (t < a.T) {
        const int64_t o = (n * a.T + t) * kDV + c4;
        if (a.y_dtype == KDN_DTYPE_BF16)
          *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(a.y) + o) =
              make_uint2(pack_bf16(y.x, y.y), pack_bf16(y.z, y.w));
        else
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + o) = y;
      }
    }
    // E'' = exp(g_{C-1} - g_j) s_kj e_j (fp16, token rows, dv contiguous)
    for (int e = tid; e < 64 * 8; e += kThr) {
      const int j = e >> 3, c8 = (e & 7) * 8;
      const float w = wdec[j] * sc[j];
      const float* er = Es + j * 64 + c8;
      *reinterpret_cast<uint4*>(sm + OFF_EB + tc::sw128_offset(j, c8)) =
          make_uint4(pack_f16(w * er[0], w * er[1]), pack_f16(w * er[2], w * er[3]), pack_f16(w * er[4], w * er[5]),
                     pack_f16(w * er[6], w * er[7]));
    }
    // decay of the carried state
    {
      const float gC = eg[63];
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

    // ------------------------------------------------ 8. state update (fp16 operands, fp32 state)
    if (tid == 0) {
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) {
        const uint64_t ad = tc::smem_desc_sw128(sbase + OFF_F + 128 * k0, 16384, 1024);
        const uint64_t bd = tc::smem_desc_sw128(sbase + OFF_EB + 128 * k0, 8192, 1024);
        tc::mma_ss(tmem + COL_S, ad, bd, id_ds, true);
      }
      tc::mma_commit(mbar);
    }
    __syncwarp();
    ok &= tc::mbar_wait_bounded(mbar, phase, kWaitLimit);
    phase ^= 1;
    tc::fence_after_sync();

    // ------------------------------------------------ 9. fp16 operand copy of the state
    {
      float v[32];
      tc::tmem_ld32(tmem + lane_off + COL_S + 32 * half, v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint4 pk = make_uint4(pack_f16(v[8 * c4], v[8 * c4 + 1]), pack_f16(v[8 * c4 + 2], v[8 * c4 + 3]),
                              pack_f16(v[8 * c4 + 4], v[8 * c4 + 5]), pack_f16(v[8 * c4 + 6], v[8 * c4 + 7]));
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
  tc::cp_async_wait_all();
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
