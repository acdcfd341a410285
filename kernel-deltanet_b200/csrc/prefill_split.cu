// prefill_split.cu -- two-phase tensor-core prefill (KDN_MODE_BF16) for few, long
// sequences, sm_100a.
//
// The fused kernel (prefill_tc.cu) runs one CTA per sequence, so a workload of a
// handful of long sequences (one layer of 16 heads at T = 64k) leaves most of the
// 148 SMs idle.  Here the work of a chunk is split by what depends on the state:
//
//   phase 1, chunk_prep_kernel -- every chunk of every sequence at once
//   (persistent CTAs, one per SM).  With u = cos(tau_inv Omega x + b) the un-normalised
//   features, s = amp / (amp ||u|| + 1e-8) the token scales and the gates of the chunk,
//     G = U_k U_k^T, P = U_q U_k^T                      (tcgen05, fp16 -> fp32)
//     A_ij = beta_i exp(g_i - g_j) s_i s_j G_ij (j<i),  T = (I + A)^-1   (CUDA cores, fp32)
//     W = T diag(beta exp(g) s_k) U_k,  U = T diag(beta) V              (tcgen05)
//     Aq_ij = exp(g_{i-1} - g_j) s_qi s_kj P_ij (j<i)
//   and writes a chunk record: [W; U_q] and U_k (fp16, already in the swizzled
//   shared-memory layouts the state pass feeds to the tensor core), U (fp32),
//   Aq (fp16) and the per-token factors.
//
//   phase 2, state_pass_kernel -- one CTA per sequence, serial over chunks, only the
//   state-dependent products (the fp32 state S^T [D=512 x dv=64] stays in TMEM):
//     [X; Yq] = [W; U_q] S^T          (tcgen05, K = 512, records streamed by bulk copies)
//     E = U - X,  E'' = exp(g_{C-1} - g_j) s_kj e_j
//     S^T = exp(g_{C-1}) S^T + U_k^T E'',  y_i = s_qi exp(g_{i-1}) Yq_i + (Aq E)_i
//
// This is the chunk algebra of prefill_tc.cu (the reference chunk step
// kernels/fused_kernel_deltanet.py:95-149) with (I + A)^-1 applied to the state
// independent parts ahead of time: E = T (beta (v - exp(g) s X')) = U - W S^T.
// Records take 217 KiB per chunk of the workspace; nothing else is allocated.
#include <math.h>

#include "kdn_internal.h"
#include "tc_chunk.cuh"

namespace kdn {
namespace {

using namespace tcc;

__device__ int g_split_error;

constexpr uint32_t kWaitLimit = 1u << 24;

// ------------------------------------------------ chunk record (workspace)
constexpr uint32_t REC_WQ = 0;        // 128 KiB [W; U_q] fp16, K-major SW128: K-block kb (features
                                      //          64kb..64kb+63) at 16 KiB kb, rows 0-63 W, 64-127 U_q
constexpr uint32_t REC_UK = 131072;   // 64 KiB  U_k fp16: slice s at 16 KiB s, half h at 8 KiB h,
                                      //          [64 tokens x 64 features] SW128
constexpr uint32_t REC_U = 196608;    // 16 KiB  U fp32 row-major [64 tokens][64]
constexpr uint32_t REC_AQ = 212992;   // 8 KiB   Aq fp16 K-major SW128 [64 rows x 64]
constexpr uint32_t REC_VEC = 221184;  // 1 KiB   ew[64] = exp(g_{C-1} - g_j) s_kj, yqs[64] = s_qi exp(g_{i-1}),
                                      //          eC = exp(g_{C-1})
constexpr uint32_t REC_BYTES = 222208;

struct SplitArgs {
  TcArgs a;
  int64_t N;
  uint8_t* ws;  // N * NC records, chunk-major: record (c, n) at (c N + n) REC_BYTES
};

__device__ __forceinline__ uint8_t* record(const SplitArgs& sa, int64_t c, int64_t n) {
  return sa.ws + (c * sa.N + n) * int64_t(REC_BYTES);
}

// ================================================================ phase 1
constexpr int kP1Warps = 16;  // compute warps, 4 per TMEM lane quarter
constexpr int kP1Threads = 32 * kP1Warps;
constexpr int kP1Issuer = kP1Warps;
constexpr int kP1Thr = 32 * (kP1Warps + 1);

// TMEM columns (phase 1)
constexpr uint32_t P1_Z = 0;     // lift result, 128 cols
constexpr uint32_t P1_GP = 128;  // [G; P], 64 cols
constexpr uint32_t P1_W0 = 0;    // W features 0..255 (after the chunk matrices are read)
constexpr uint32_t P1_W1 = 256;  // W features 256..383
constexpr uint32_t P1_U = 384;   // U in lanes 64..127
constexpr uint32_t P1_W2 = 0;    // W features 384..511 (second round)

// shared memory (phase 1)
constexpr uint32_t P1_OMG = 0;        // 64 KiB Omega (bf16)
constexpr uint32_t P1_XIN = 65536;    // 16 KiB [k; q] (bf16, K-major)
constexpr uint32_t P1_F = 81920;      // 32 KiB slice features [U_k; U_q] | algebra: A (f32), T (f32)
constexpr uint32_t P1_UK = 114688;    // 64 KiB U_k, all slices (fp16), B operand of W
constexpr uint32_t P1_VB = 180224;    // 8 KiB  V (fp16, MN-major), B operand of U
constexpr uint32_t P1_TOP = 188416;   // 16 KiB [T diag(beta exp(g) s_k); T diag(beta)] (fp16, K-major)
constexpr uint32_t P1_TD = 204800;    // 4 KiB  diagonal 16x16 blocks of T
constexpr uint32_t P1_US = 208896;    // 4 KiB  forward-substitution scratch
constexpr uint32_t P1_PH = 212992;    // 2 KiB  phase b[512]
constexpr uint32_t P1_GL = 215040;    // 5 x 256 B gates: g, beta, exp(g), exp(g_{i-1}), exp(g_{C-1} - g)
constexpr uint32_t P1_SSP = 216320;   // 2 KiB  sums of squares per column quarter
constexpr uint32_t P1_SC = 218368;    // 512 B  token scales
constexpr uint32_t P1_BAR = 218880;   // mbarriers + TMEM address
constexpr uint32_t kP1Smem = P1_BAR + 128 + 1024;

__global__ void __launch_bounds__(kP1Thr, 1) chunk_prep_kernel(SplitArgs sa, ProjParams P) {
  const TcArgs& a = sa.a;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm;
  {
    const uint32_t s = tc::smem_u32(smem_raw);
    sm = smem_raw + ((1024u - (s & 1023u)) & 1023u);
  }
  const uint32_t sbase = tc::smem_u32(sm);
  float* Am = reinterpret_cast<float*>(sm + P1_F);
  float* Es = reinterpret_cast<float*>(sm + P1_F + 16384);
  float* TD = reinterpret_cast<float*>(sm + P1_TD);
  float* US = reinterpret_cast<float*>(sm + P1_US);
  float* ph = reinterpret_cast<float*>(sm + P1_PH);
  float* gl = reinterpret_cast<float*>(sm + P1_GL);
  float* bt = gl + 64;
  float* eg = gl + 128;
  float* egp = gl + 192;
  float* wdec = gl + 256;
  float* ssp = reinterpret_cast<float*>(sm + P1_SSP);
  float* sc = reinterpret_cast<float*>(sm + P1_SC);
  uint64_t* bar_lift = reinterpret_cast<uint64_t*>(sm + P1_BAR);
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(sm + P1_BAR + 8);
  uint64_t* bar_xin = reinterpret_cast<uint64_t*>(sm + P1_BAR + 16);
  uint64_t* bar_zfree = reinterpret_cast<uint64_t*>(sm + P1_BAR + 24);
  uint64_t* bar_fready = reinterpret_cast<uint64_t*>(sm + P1_BAR + 32);
  uint64_t* bar_ops = reinterpret_cast<uint64_t*>(sm + P1_BAR + 40);
  uint64_t* bar_wdone = reinterpret_cast<uint64_t*>(sm + P1_BAR + 48);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + P1_BAR + 56);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, cq = (warp >> 2) & 3;
  const int trow = quarter * 32 + lane;
  const uint32_t lane_off = uint32_t(quarter * 32) << 16;
  const bool bf_in = a.in_dtype == KDN_DTYPE_BF16;
  const bool decayed = a.decay != nullptr;
  const int64_t N = sa.N;
  const int64_t total = N * a.NC;
  bool ok = true;

  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(bar_lift, 1);
    tc::mbar_init(bar_mma, 1);
    tc::mbar_init(bar_xin, kP1Warps);
    tc::mbar_init(bar_zfree, kP1Warps);
    tc::mbar_init(bar_fready, kP1Warps);
    tc::mbar_init(bar_ops, kP1Warps);
    tc::mbar_init(bar_wdone, kP1Warps);
    tc::fence_mbar_init();
  }
  build_omega(sm + P1_OMG, P, warp, lane, kP1Thr / 32);
  for (int i = tid; i < kD; i += kP1Thr) ph[i] = P.phase[i];
  if (warp < kP1Warps && bf_in && blockIdx.x < total)
    prefetch_kq(a, int64_t(blockIdx.x) % N, int(int64_t(blockIdx.x) / N), sbase + P1_XIN, tid);
  tc::cp_async_commit();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  if (warp == kP1Issuer) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      const uint32_t id_lift = tc::idesc_bf16_f32(128, 128, false, false);
      const uint32_t id_gp = tc::idesc_f16_f32(128, 64, false, false);
      const uint32_t id_n256 = tc::idesc_f16_f32(128, 256, false, true);
      const uint32_t id_n128 = tc::idesc_f16_f32(128, 128, false, true);
      const uint32_t id_n64 = tc::idesc_f16_f32(128, 64, false, true);
      uint32_t p_xin = 0, p_zfree = 0, p_fready = 0, p_ops = 0, p_wdone = 0;
      auto lift = [&](int s) {
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16)
          tc::mma_ss(tmem + P1_Z, tc::smem_desc_sw128(sbase + P1_XIN + 2 * k0, 16, 1024),
                     tc::smem_desc_sw128(sbase + P1_OMG + s * 16384 + 2 * k0, 16, 1024), id_lift, k0 > 0);
        tc::mma_commit(bar_lift);
      };
      for (int64_t idx = blockIdx.x; idx < total; idx += gridDim.x) {
        ok &= tc::mbar_wait_bounded(bar_xin, p_xin, kWaitLimit);
        p_xin ^= 1;
        tc::fence_after_sync();
        lift(0);
        for (int s = 0; s < kSlices; ++s) {
          ok &= tc::mbar_wait_bounded(bar_zfree, p_zfree, kWaitLimit);
          p_zfree ^= 1;
          tc::fence_after_sync();
          if (s + 1 < kSlices) lift(s + 1);
          ok &= tc::mbar_wait_bounded(bar_fready, p_fready, kWaitLimit);
          p_fready ^= 1;
          tc::fence_after_sync();
#pragma unroll
          for (int k0 = 0; k0 < 128; k0 += 16) {
            const uint64_t fd = tc::smem_desc_sw128(sbase + P1_F + (k0 >> 6) * 16384 + 2 * (k0 & 63), 16, 1024);
            tc::mma_ss(tmem + P1_GP, fd, fd, id_gp, s > 0 || k0 > 0);
          }
          tc::mma_commit(bar_mma);
        }
        ok &= tc::mbar_wait_bounded(bar_ops, p_ops, kWaitLimit);
        p_ops ^= 1;
        tc::fence_after_sync();
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16) {  // K = the 64 tokens of the chunk
          const uint64_t ad = tc::smem_desc_sw128(sbase + P1_TOP + 2 * k0, 16, 1024);
          tc::mma_ss(tmem + P1_W0, ad, tc::smem_desc_sw128(sbase + P1_UK + 128 * k0, 8192, 1024), id_n256, k0 > 0);
          tc::mma_ss(tmem + P1_W1, ad, tc::smem_desc_sw128(sbase + P1_UK + 32768 + 128 * k0, 8192, 1024), id_n128,
                     k0 > 0);
          tc::mma_ss(tmem + P1_U, ad, tc::smem_desc_sw128(sbase + P1_VB + 128 * k0, 8192, 1024), id_n64, k0 > 0);
        }
        tc::mma_commit(bar_mma);
        ok &= tc::mbar_wait_bounded(bar_wdone, p_wdone, kWaitLimit);
        p_wdone ^= 1;
        tc::fence_after_sync();
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16)
          tc::mma_ss(tmem + P1_W2, tc::smem_desc_sw128(sbase + P1_TOP + 2 * k0, 16, 1024),
                     tc::smem_desc_sw128(sbase + P1_UK + 49152 + 128 * k0, 8192, 1024), id_n128, k0 > 0);
        tc::mma_commit(bar_mma);
      }
    }
    __syncwarp();
  } else {
    // ================================================================ compute warps
    uint32_t ph_lift = 0, ph_mma = 0;
    auto wait_mma = [&]() {
      ok &= tc::mbar_wait_bounded(bar_mma, ph_mma, kWaitLimit);
      ph_mma ^= 1;
      tc::fence_after_sync();
    };
    float nb[2] = {0.f, 0.f}, nd[2] = {1.f, 1.f};  // gates of the coming chunk (warp 0)
    if (warp == 0 && blockIdx.x < total) {
      const int64_t n0 = int64_t(blockIdx.x) % N, t00 = (int64_t(blockIdx.x) / N) * kC;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t tt = t00 + 2 * lane + e;
        if (tt < a.T) {
          nb[e] = ld_as_f32(a.beta, a.gate_dtype, n0 * a.T + tt);
          if (decayed) nd[e] = ld_as_f32(a.decay, a.gate_dtype, n0 * a.T + tt);
        }
      }
    }
    for (int64_t idx = blockIdx.x; idx < total; idx += gridDim.x) {
      const int64_t n = idx % N, c = idx / N, t0 = c * kC;
      const int64_t nidx = idx + gridDim.x;
      const bool has_next = nidx < total;
      const int64_t nn = nidx % N, ncn = nidx / N;
      uint8_t* rec = record(sa, c, n);
      // ---------------------------------------- chunk inputs -> lift of slice 0
      tc::cp_async_wait_all();
      if (!bf_in) load_kq_f32(a, n, int(c), sm + P1_XIN, tid);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_xin);
      float vreg[8];  // v row tid/8, values 8 (tid%8) .. +7 (zero past the end)
      {
        const int row = tid >> 3, cc = tid & 7;
        const int64_t t = t0 + row;
#pragma unroll
        for (int j = 0; j < 8; ++j) vreg[j] = 0.f;
        if (t < a.T) {
          if (bf_in) {
            const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.v) +
                                                           (n * a.T + t) * kDV + 8 * cc);
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(h[j]);
              vreg[2 * j] = f.x;
              vreg[2 * j + 1] = f.y;
            }
          } else {
            const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.v) +
                                                                (n * a.T + t) * kDV + 8 * cc);
            const float4 x0 = src[0], x1 = src[1];
            vreg[0] = x0.x, vreg[1] = x0.y, vreg[2] = x0.z, vreg[3] = x0.w;
            vreg[4] = x1.x, vreg[5] = x1.y, vreg[6] = x1.z, vreg[7] = x1.w;
          }
        }
      }
      if (warp == 0) {  // gates: beta, inclusive scan of log clamp(decay, 1e-5, 1), derived factors
        const float lg0 = decayed ? logf(fminf(fmaxf(nd[0], 1e-5f), 1.0f)) : 0.f;
        const float lg1 = decayed ? logf(fminf(fmaxf(nd[1], 1e-5f), 1.0f)) : 0.f;
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
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int64_t tt = ncn * kC + 2 * lane + e;
          nb[e] = 0.f;
          nd[e] = 1.f;
          if (has_next && tt < a.T) {
            nb[e] = ld_as_f32(a.beta, a.gate_dtype, nn * a.T + tt);
            if (decayed) nd[e] = ld_as_f32(a.decay, a.gate_dtype, nn * a.T + tt);
          }
        }
      }

      // ---------------------------------------- slice loop: features, Gram products
      float ss = 0.f;
#pragma unroll 1
      for (int s = 0; s < kSlices; ++s) {
        ok &= tc::mbar_wait_bounded(bar_lift, ph_lift, kWaitLimit);
        ph_lift ^= 1;
        tc::fence_after_sync();
        float z[32];
        tc::tmem_ld32(tmem + lane_off + P1_Z + 32 * cq, z);
        tc::tmem_ld_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_zfree);
        // u = cos(tau_inv z + b); the hardware cosine's ~1e-6 absolute error is far
        // below the fp16 spacing of the stored features for the |arguments| <= 32 here
        uint32_t fp[16];
        const float4* phs = reinterpret_cast<const float4*>(ph + 128 * s + 32 * cq);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 b4 = phs[j >> 2];
          const float u0 = __cosf(fmaf(z[j], P.tau_inv, b4.x));
          const float u1 = __cosf(fmaf(z[j + 1], P.tau_inv, b4.y));
          const float u2 = __cosf(fmaf(z[j + 2], P.tau_inv, b4.z));
          const float u3 = __cosf(fmaf(z[j + 3], P.tau_inv, b4.w));
          ss = fmaf(u0, u0, fmaf(u1, u1, fmaf(u2, u2, fmaf(u3, u3, ss))));
          fp[j >> 1] = pack_f16(u0, u1);
          fp[(j >> 1) + 1] = pack_f16(u2, u3);
        }
        if (s > 0) wait_mma();  // the previous slice's Gram product is done with F
        {
          const int kb = cq >> 1, e0 = 32 * (cq & 1);
          uint8_t* fb = sm + P1_F + kb * 16384;
          uint8_t* gdst = trow < 64 ? rec + REC_UK + s * 16384 + kb * 8192 : rec + REC_WQ + (2 * s + kb) * 16384;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const uint4 pk = make_uint4(fp[4 * c8], fp[4 * c8 + 1], fp[4 * c8 + 2], fp[4 * c8 + 3]);
            const uint32_t off = tc::sw128_offset(trow, e0 + 8 * c8);
            *reinterpret_cast<uint4*>(fb + off) = pk;
            *reinterpret_cast<uint4*>(gdst + off) = pk;  // U_k rows 0..63 | U_q rows 64..127
            if (trow < 64) *reinterpret_cast<uint4*>(sm + P1_UK + s * 16384 + kb * 8192 + off) = pk;
          }
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_fready);
      }
      ssp[cq * 128 + trow] = ss;
      // every lift of this chunk has completed: the input tile takes the next chunk
      if (has_next && bf_in) prefetch_kq(a, nn, int(ncn), sbase + P1_XIN, tid);
      tc::cp_async_commit();
      wait_mma();  // Gram product of the last slice

      // ---------------------------------------- chunk matrices
      float gp[16];
      tc::tmem_ld16(tmem + lane_off + P1_GP + 16 * cq, gp);
      tc::tmem_ld_wait();
      tc::named_bar_sync(1, kP1Threads);  // sums of squares and gates visible
      if (tid < 128)
        sc[tid] = P.amp / (P.amp * sqrtf(ssp[tid] + ssp[128 + tid] + ssp[256 + tid] + ssp[384 + tid]) + 1e-8f);
      tc::named_bar_sync(1, kP1Threads);
      {
        const int i = trow & 63;
        const float si = sc[trow];
        if (trow < 64) {  // k row: A_ij = beta_i exp(g_i - g_j) s_i s_j G_ij, j < i
          const float bi = bt[i], gi = gl[i];
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            float4 av;
            float* ap = &av.x;
#pragma unroll
            for (int qx = 0; qx < 4; ++qx) {
              const int jj = 4 * j4 + qx, j = 16 * cq + jj;
              const float dec = decayed ? __expf(gi - gl[j]) : 1.f;
              ap[qx] = (j < i) ? bi * dec * gp[jj] * si * sc[j] : 0.f;
            }
            *reinterpret_cast<float4*>(Am + sx(i, 16 * cq + 4 * j4)) = av;
          }
        } else {  // q row: Aq_ij = exp(g_{i-1} - g_j) s_qi s_kj P_ij, j < i (fp16 into the record)
          const float gp_i = i > 0 ? gl[i - 1] : 0.f;
          float aq[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = 16 * cq + jj;
            const float dec = decayed ? __expf(gp_i - gl[j]) : 1.f;
            aq[jj] = (j < i) ? dec * gp[jj] * si * sc[j] : 0.f;
          }
#pragma unroll
          for (int h = 0; h < 2; ++h)
            *reinterpret_cast<uint4*>(rec + REC_AQ + tc::sw128_offset(i, 16 * cq + 8 * h)) = make_uint4(
                pack_f16_sat(aq[8 * h], aq[8 * h + 1]), pack_f16_sat(aq[8 * h + 2], aq[8 * h + 3]),
                pack_f16_sat(aq[8 * h + 4], aq[8 * h + 5]), pack_f16_sat(aq[8 * h + 6], aq[8 * h + 7]));
        }
      }
      {  // per-token factors of the state pass, and V (fp16) as the B operand of U
        float* vec = reinterpret_cast<float*>(rec + REC_VEC);
        if (tid < 64) vec[tid] = wdec[tid] * sc[tid];
        else if (tid < 128) vec[tid] = sc[tid] * egp[tid - 64];
        else if (tid == 128) vec[128] = eg[63];
        const int row = tid >> 3, cc = tid & 7;
        *reinterpret_cast<uint4*>(sm + P1_VB + tc::sw128_offset(row, 8 * cc)) =
            make_uint4(pack_f16_sat(vreg[0], vreg[1]), pack_f16_sat(vreg[2], vreg[3]), pack_f16_sat(vreg[4], vreg[5]),
                       pack_f16_sat(vreg[6], vreg[7]));
      }
      tc::named_bar_sync(1, kP1Threads);
      // diagonal 16x16 blocks of T = (I + A)^-1: one warp per block, one lane per column
      if (warp < 4 && lane < 16) {
        const int I = warp, j = lane;
        float tcol[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          float sacc = (r == j) ? 1.f : 0.f;
#pragma unroll
          for (int kk = 0; kk < r; ++kk) sacc = fmaf(-Am[sx(16 * I + r, 16 * I + kk)], tcol[kk], sacc);
          tcol[r] = (r >= j) ? sacc : 0.f;
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) TD[(I * 16 + r) * 16 + j] = tcol[r];
      }
      tc::named_bar_sync(1, kP1Threads);
      // T by block rows (U = I_I - sum_{J<I} A_IJ T_J ; T_I = T_II U) on warps 0-3:
      // warp w owns rows 4w..4w+3 of the block, lane l columns 2l, 2l+1 (row-major)
      if (warp < 4) {
        const int c2 = 2 * lane;
#pragma unroll
        for (int I = 0; I < 4; ++I) {
          float2 acc[4];
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            const int row = 16 * I + 4 * warp + rr;
            acc[rr] = make_float2(c2 == row ? 1.f : 0.f, c2 + 1 == row ? 1.f : 0.f);
          }
#pragma unroll
          for (int qs = 0; qs < 4 * I; ++qs) {
            float2 e[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) e[u] = *reinterpret_cast<const float2*>(Es + (4 * qs + u) * 64 + c2);
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
              const int row = 16 * I + 4 * warp + rr;
              const float4 a4 = *reinterpret_cast<const float4*>(Am + row * 64 + (((qs ^ row) & 15) << 2));
              acc[rr].x = fmaf(-a4.x, e[0].x, acc[rr].x);
              acc[rr].y = fmaf(-a4.x, e[0].y, acc[rr].y);
              acc[rr].x = fmaf(-a4.y, e[1].x, acc[rr].x);
              acc[rr].y = fmaf(-a4.y, e[1].y, acc[rr].y);
              acc[rr].x = fmaf(-a4.z, e[2].x, acc[rr].x);
              acc[rr].y = fmaf(-a4.z, e[2].y, acc[rr].y);
              acc[rr].x = fmaf(-a4.w, e[3].x, acc[rr].x);
              acc[rr].y = fmaf(-a4.w, e[3].y, acc[rr].y);
            }
          }
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) *reinterpret_cast<float2*>(US + (4 * warp + rr) * 64 + c2) = acc[rr];
          tc::named_bar_sync(2, 128);
          float2 ev[4];
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) ev[rr] = make_float2(0.f, 0.f);
#pragma unroll
          for (int kk = 0; kk < 16; ++kk) {
            const float2 u = *reinterpret_cast<const float2*>(US + kk * 64 + c2);
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
              const float tv = TD[(I * 16 + 4 * warp + rr) * 16 + kk];
              ev[rr].x = fmaf(tv, u.x, ev[rr].x);
              ev[rr].y = fmaf(tv, u.y, ev[rr].y);
            }
          }
#pragma unroll
          for (int rr = 0; rr < 4; ++rr)
            *reinterpret_cast<float2*>(Es + (16 * I + 4 * warp + rr) * 64 + c2) = ev[rr];
          tc::named_bar_sync(2, 128);
        }
      }
      tc::named_bar_sync(1, kP1Threads);
      // A operand [T diag(beta exp(g) s_k); T diag(beta)] (fp16, K-major, 128 x 64)
      {
        const int r = tid >> 2, jq = tid & 3, i = r & 63;
        float w[16];
#pragma unroll
        for (int j4 = 0; j4 < 4; ++j4) {
          const float4 t4 = *reinterpret_cast<const float4*>(Es + i * 64 + 16 * jq + 4 * j4);
          const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
          for (int qx = 0; qx < 4; ++qx) {
            const int j = 16 * jq + 4 * j4 + qx;
            w[4 * j4 + qx] = tv[qx] * (r < 64 ? bt[j] * eg[j] * sc[j] : bt[j]);
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
          *reinterpret_cast<uint4*>(sm + P1_TOP + tc::sw128_offset(r, 16 * jq + 8 * h)) =
              make_uint4(pack_f16_sat(w[8 * h], w[8 * h + 1]), pack_f16_sat(w[8 * h + 2], w[8 * h + 3]),
                         pack_f16_sat(w[8 * h + 4], w[8 * h + 5]), pack_f16_sat(w[8 * h + 6], w[8 * h + 7]));
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      tc::named_bar_sync(1, kP1Threads);  // also: gates and scales of this chunk no longer read
      if (lane == 0) tc::mbar_arrive(bar_ops);
      wait_mma();  // W (features 0..383) and U

      // ---------------------------------------- W, U -> record
      auto drain_w = [&](uint32_t col, int kb) {  // row trow of K-block kb of W (64 columns from col)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float v[32];
          tc::tmem_ld32(tmem + lane_off + col + 32 * hh, v);
          tc::tmem_ld_wait();
#pragma unroll
          for (int m = 0; m < 4; ++m)
            *reinterpret_cast<uint4*>(rec + REC_WQ + kb * 16384 + tc::sw128_offset(trow, 32 * hh + 8 * m)) =
                make_uint4(pack_f16_sat(v[8 * m], v[8 * m + 1]), pack_f16_sat(v[8 * m + 2], v[8 * m + 3]),
                           pack_f16_sat(v[8 * m + 4], v[8 * m + 5]), pack_f16_sat(v[8 * m + 6], v[8 * m + 7]));
        }
      };
      if (trow < 64) {
        drain_w(P1_W0 + 64 * cq, cq);  // K-blocks 0..3
      } else {
        float u[16];
        tc::tmem_ld16(tmem + lane_off + P1_U + 16 * cq, u);
        tc::tmem_ld_wait();
        float4* dst = reinterpret_cast<float4*>(rec + REC_U + ((trow - 64) * 64 + 16 * cq) * 4);
#pragma unroll
        for (int m = 0; m < 4; ++m) dst[m] = make_float4(u[4 * m], u[4 * m + 1], u[4 * m + 2], u[4 * m + 3]);
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_wdone);  // columns 0..127 free for the second round
      if (trow < 64 && cq < 2) drain_w(P1_W1 + 64 * cq, 4 + cq);  // K-blocks 4, 5
      wait_mma();                                                  // W features 384..511
      if (trow < 64 && cq >= 2) drain_w(P1_W2 + 64 * (cq - 2), 4 + cq);  // K-blocks 6, 7
      tc::fence_before_sync();
    }
    tc::cp_async_wait_all();
  }
  if (!ok) record_device_error(&g_split_error, 3);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

// ================================================================ phase 2
constexpr int kP2Warps = 8;  // compute warps: 2 per TMEM lane quarter (column halves)
constexpr int kP2Issuer = kP2Warps;
constexpr int kP2Producer = kP2Warps + 1;
constexpr int kP2Thr = 32 * (kP2Warps + 2);

// TMEM columns (phase 2)
constexpr uint32_t P2_S = 0;     // S^T master, slice s at 64 s (lanes = features), fp32
constexpr uint32_t P2_XY = 256;  // [X; Yq] (lanes = [k; q] tokens, 64 cols = dv)
constexpr uint32_t P2_YE = 320;  // [junk; Aq E]

// shared memory (phase 2)
constexpr uint32_t P2_WQR = 0;       // 2 x 32 KiB ring of [W; U_q] feature slices (K-major)
constexpr uint32_t P2_UKB = 65536;   // 64 KiB U_k of the chunk (A operand of the state update)
constexpr uint32_t P2_SOP = 131072;  // 64 KiB S^T operand (fp16, MN-major), slice s at 16 KiB s
constexpr uint32_t P2_EB = 196608;   // 8 KiB  E'' (fp16, MN-major)
constexpr uint32_t P2_ET = 204800;   // 8 KiB  E (fp16, MN-major)
constexpr uint32_t P2_AQB = 212992;  // 16 KiB [0; Aq] (fp16, K-major); rows 0..63 stay zero
constexpr uint32_t P2_BAR = 229376;
constexpr uint32_t kP2Smem = P2_BAR + 256 + 1024;

__global__ void __launch_bounds__(kP2Thr, 1) state_pass_kernel(SplitArgs sa) {
  const TcArgs& a = sa.a;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm;
  {
    const uint32_t s = tc::smem_u32(smem_raw);
    sm = smem_raw + ((1024u - (s & 1023u)) & 1023u);
  }
  const uint32_t sbase = tc::smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + P2_BAR);
  uint64_t* wq_full = bars;       // [2] ring slot loaded (bytes)
  uint64_t* wq_empty = bars + 2;  // [2] ring slot consumed (MMA commit)
  uint64_t* ukb_full = bars + 4;  // U_k, Aq of the chunk loaded (bytes)
  uint64_t* ukb_empty = bars + 5; // state update of the previous chunk done (MMA commit)
  uint64_t* bar_sop = bars + 6;   // [4] state operand slice s stored (8 warps)
  uint64_t* bar_x = bars + 10;    // [X; Yq] done (MMA commit)
  uint64_t* bar_e = bars + 11;    // E, E'' stored (8 warps)
  uint64_t* bar_s = bars + 12;    // state update and Aq E done (MMA commit)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 14);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n = blockIdx.x;
  const int NC = a.NC;
  bool ok = true;

  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&wq_full[0], 1);
    tc::mbar_init(&wq_full[1], 1);
    tc::mbar_init(&wq_empty[0], 1);
    tc::mbar_init(&wq_empty[1], 1);
    tc::mbar_init(ukb_full, 1);
    tc::mbar_init(ukb_empty, 1);
    for (int s = 0; s < kSlices; ++s) tc::mbar_init(&bar_sop[s], kP2Warps);
    tc::mbar_init(bar_x, 1);
    tc::mbar_init(bar_e, kP2Warps);
    tc::mbar_init(bar_s, 1);
    tc::fence_mbar_init();
  }
  for (int i = tid; i < 8192 / 16; i += kP2Thr) reinterpret_cast<uint4*>(sm + P2_AQB)[i] = make_uint4(0, 0, 0, 0);
  tc::fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  if (warp == kP2Producer) {
    // ================================================================ bulk loads
    if (lane == 0) {
      uint32_t pe[2] = {0, 0}, pu = 0;
      int64_t g = 0;  // ring uses so far
      auto load_slice = [&](const uint8_t* rec, int s) {
        const int b = int(g & 1);
        if (g >= 2) {
          ok &= tc::mbar_wait_bounded(&wq_empty[b], pe[b], kWaitLimit);
          pe[b] ^= 1;
        }
        tc::mbar_arrive_expect_tx(&wq_full[b], 32768);
        for (int o = 0; o < 32768; o += 16384)
          tc::bulk_load(sbase + P2_WQR + b * 32768 + o, rec + REC_WQ + s * 32768 + o, 16384, &wq_full[b]);
        ++g;
      };
      for (int c = 0; c < NC; ++c) {
        const uint8_t* rec = record(sa, c, n);
        load_slice(rec, 0);
        load_slice(rec, 1);
        if (c > 0) {  // the previous chunk's state update has read U_k and Aq
          ok &= tc::mbar_wait_bounded(ukb_empty, pu, kWaitLimit);
          pu ^= 1;
        }
        tc::mbar_arrive_expect_tx(ukb_full, 65536 + 8192);
        for (int o = 0; o < 65536; o += 16384) tc::bulk_load(sbase + P2_UKB + o, rec + REC_UK + o, 16384, ukb_full);
        tc::bulk_load(sbase + P2_AQB + 8192, rec + REC_AQ, 8192, ukb_full);
        load_slice(rec, 2);
        load_slice(rec, 3);
      }
    }
    __syncwarp();
  } else if (warp == kP2Issuer) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      const uint32_t id_x = tc::idesc_f16_f32(128, 64, false, true);
      const uint32_t id_s = tc::idesc_f16_f32(128, 64, true, true);
      uint32_t pf[2] = {0, 0}, psop = 0, pe = 0, pu = 0;
      int64_t g = 0;
      for (int c = 0; c < NC; ++c) {
        for (int s = 0; s < kSlices; ++s, ++g) {
          const int b = int(g & 1);
          ok &= tc::mbar_wait_bounded(&wq_full[b], pf[b], kWaitLimit);
          pf[b] ^= 1;
          ok &= tc::mbar_wait_bounded(&bar_sop[s], psop, kWaitLimit);
          tc::fence_after_sync();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // K = features 128 s + 16 kk
            const uint64_t ad =
                tc::smem_desc_sw128(sbase + P2_WQR + b * 32768 + (kk >> 2) * 16384 + 32 * (kk & 3), 16, 1024);
            const uint64_t bd = tc::smem_desc_sw128(sbase + P2_SOP + s * 16384 + 16 * kk * 128, 8192, 1024);
            tc::mma_ss(tmem + P2_XY, ad, bd, id_x, s > 0 || kk > 0);
          }
          tc::mma_commit(&wq_empty[b]);
        }
        psop ^= 1;
        tc::mma_commit(bar_x);
        ok &= tc::mbar_wait_bounded(bar_e, pe, kWaitLimit);
        pe ^= 1;
        ok &= tc::mbar_wait_bounded(ukb_full, pu, kWaitLimit);
        pu ^= 1;
        tc::fence_after_sync();
#pragma unroll
        for (int s = 0; s < kSlices; ++s)
#pragma unroll
          for (int k0 = 0; k0 < 64; k0 += 16)
            tc::mma_ss(tmem + P2_S + 64 * s, tc::smem_desc_sw128(sbase + P2_UKB + s * 16384 + 128 * k0, 8192, 1024),
                       tc::smem_desc_sw128(sbase + P2_EB + 128 * k0, 8192, 1024), id_s, true);
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16)
          tc::mma_ss(tmem + P2_YE, tc::smem_desc_sw128(sbase + P2_AQB + 2 * k0, 16, 1024),
                     tc::smem_desc_sw128(sbase + P2_ET + 128 * k0, 8192, 1024), id_x, k0 > 0);
        tc::mma_commit(bar_s);
        tc::mma_commit(ukb_empty);
      }
    }
    __syncwarp();
  } else {
    // ================================================================ compute warps
    const int quarter = warp & 3, ch = warp >> 2;  // TMEM lane quarter, column half
    const int trow = quarter * 32 + lane;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const bool decayed = a.decay != nullptr;
#pragma unroll
    for (int s = 0; s < kSlices; ++s) {  // state master from the initial state
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = a.S0 ? a.S0[(n * kDV + 32 * ch + j) * kD + 128 * s + trow] : 0.f;
      tc::tmem_st32(tmem + lane_off + P2_S + 64 * s + 32 * ch, v);
    }
    tc::tmem_st_wait();
    uint32_t px = 0, ps = 0;
    // per-chunk factors, loaded one chunk ahead
    float urow[32], ew = 0.f, yqs = 0.f, eC = 1.f;
    auto load_factors = [&](int c) {
      const uint8_t* rec = record(sa, c, n);
      const float* vec = reinterpret_cast<const float*>(rec + REC_VEC);
      if (trow < 64) {
        const float4* u4 = reinterpret_cast<const float4*>(rec + REC_U + (trow * 64 + 32 * ch) * 4);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float4 x = u4[m];
          urow[4 * m] = x.x, urow[4 * m + 1] = x.y, urow[4 * m + 2] = x.z, urow[4 * m + 3] = x.w;
        }
        ew = vec[trow];
      } else {
        yqs = vec[trow];
      }
      eC = vec[128];
    };
    load_factors(0);
    for (int c = 0; c < NC; ++c) {
      float cu[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) cu[j] = urow[j];
      const float cew = ew, cyqs = yqs, ceC = eC;
      if (c + 1 < NC) load_factors(c + 1);
      // ---------------------------------------- state operand (fp16) and decay, by slice
#pragma unroll
      for (int s = 0; s < kSlices; ++s) {
        float v[32];
        tc::tmem_ld32(tmem + lane_off + P2_S + 64 * s + 32 * ch, v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int m = 0; m < 4; ++m)
          *reinterpret_cast<uint4*>(sm + P2_SOP + s * 16384 + tc::sw128_offset(trow, 32 * ch + 8 * m)) =
              make_uint4(pack_f16_sat(v[8 * m], v[8 * m + 1]), pack_f16_sat(v[8 * m + 2], v[8 * m + 3]),
                         pack_f16_sat(v[8 * m + 4], v[8 * m + 5]), pack_f16_sat(v[8 * m + 6], v[8 * m + 7]));
        if (decayed) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] *= ceC;
          tc::tmem_st32(tmem + lane_off + P2_S + 64 * s + 32 * ch, v);
          tc::tmem_st_wait();
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bar_sop[s]);
      }
      // ---------------------------------------- E = U - X, E'' (k rows)
      ok &= tc::mbar_wait_bounded(bar_x, px, kWaitLimit);
      px ^= 1;
      tc::fence_after_sync();
      if (trow < 64) {
        float x[32];
        tc::tmem_ld32(tmem + lane_off + P2_XY + 32 * ch, x);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = cu[j] - x[j];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const uint32_t off = tc::sw128_offset(trow, 32 * ch + 8 * m);
          *reinterpret_cast<uint4*>(sm + P2_ET + off) =
              make_uint4(pack_f16_sat(x[8 * m], x[8 * m + 1]), pack_f16_sat(x[8 * m + 2], x[8 * m + 3]),
                         pack_f16_sat(x[8 * m + 4], x[8 * m + 5]), pack_f16_sat(x[8 * m + 6], x[8 * m + 7]));
          *reinterpret_cast<uint4*>(sm + P2_EB + off) = make_uint4(
              pack_f16_sat(cew * x[8 * m], cew * x[8 * m + 1]), pack_f16_sat(cew * x[8 * m + 2], cew * x[8 * m + 3]),
              pack_f16_sat(cew * x[8 * m + 4], cew * x[8 * m + 5]),
              pack_f16_sat(cew * x[8 * m + 6], cew * x[8 * m + 7]));
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_e);
      // ---------------------------------------- outputs (q rows)
      ok &= tc::mbar_wait_bounded(bar_s, ps, kWaitLimit);
      ps ^= 1;
      tc::fence_after_sync();
      if (trow >= 64) {
        const int64_t t = int64_t(c) * kC + (trow - 64);
        float yq[32], ye[32];
        tc::tmem_ld32(tmem + lane_off + P2_XY + 32 * ch, yq);
        tc::tmem_ld32(tmem + lane_off + P2_YE + 32 * ch, ye);
        tc::tmem_ld_wait();
        if (t < a.T) {
          const int64_t o = (n * a.T + t) * kDV + 32 * ch;
#pragma unroll
          for (int j = 0; j < 32; ++j) yq[j] = fmaf(cyqs, yq[j], ye[j]);
          if (a.y_dtype == KDN_DTYPE_BF16) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.y) + o);
#pragma unroll
            for (int m = 0; m < 4; ++m)
              dst[m] = make_uint4(pack_bf16(yq[8 * m], yq[8 * m + 1]), pack_bf16(yq[8 * m + 2], yq[8 * m + 3]),
                                  pack_bf16(yq[8 * m + 4], yq[8 * m + 5]), pack_bf16(yq[8 * m + 6], yq[8 * m + 7]));
          } else {
            float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + o);
#pragma unroll
            for (int m = 0; m < 8; ++m) dst[m] = make_float4(yq[4 * m], yq[4 * m + 1], yq[4 * m + 2], yq[4 * m + 3]);
          }
        }
      }
      tc::fence_before_sync();
    }
    // ---------------------------------------- final state
#pragma unroll
    for (int s = 0; s < kSlices; ++s) {
      float v[32];
      tc::tmem_ld32(tmem + lane_off + P2_S + 64 * s + 32 * ch, v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) a.S_out[(n * kDV + 32 * ch + j) * kD + 128 * s + trow] = v[j];
    }
  }
  if (!ok) record_device_error(&g_split_error, 3);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

}  // namespace

size_t split_prefill_workspace(int64_t N, int64_t T) {
  const int64_t NC = (T + kC - 1) / kC;
  return size_t(N) * size_t(NC) * REC_BYTES;
}

cudaError_t launch_split_prefill(const PrefillProblem& p, const ProjParams& P, void* ws, size_t ws_bytes,
                                 cudaStream_t stream) {
  if (ws_bytes < split_prefill_workspace(p.N, p.T)) return cudaErrorInvalidValue;
  SplitArgs sa;
  sa.a.q = p.q;
  sa.a.k = p.k;
  sa.a.v = p.v;
  sa.a.in_dtype = p.in_dtype;
  sa.a.beta = p.beta;
  sa.a.decay = p.decay;
  sa.a.gate_dtype = p.gate_dtype;
  sa.a.S0 = p.S0;
  sa.a.y = p.y;
  sa.a.y_dtype = p.y_dtype;
  sa.a.S_out = p.S_out;
  sa.a.T = p.T;
  sa.a.NC = int((p.T + kC - 1) / kC);
  sa.N = p.N;
  sa.ws = static_cast<uint8_t*>(ws);
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  const int64_t total = p.N * int64_t(sa.a.NC);
  const unsigned grid1 = unsigned(total < sms ? total : sms);
  if ((e = cudaFuncSetAttribute(chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kP1Smem))) !=
      cudaSuccess)
    return e;
  if ((e = cudaFuncSetAttribute(state_pass_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kP2Smem))) !=
      cudaSuccess)
    return e;
  chunk_prep_kernel<<<grid1, kP1Thr, kP1Smem, stream>>>(sa, P);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  state_pass_kernel<<<unsigned(p.N), kP2Thr, kP2Smem, stream>>>(sa);
  return cudaGetLastError();
}

cudaError_t split_read_error(cudaStream_t stream, int* code) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_split_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  if (h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_split_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  }
  *code = h;
  return cudaSuccess;
}

}  // namespace kdn
