// prefill_tc.cu -- fused tensor-core chunked prefill (KDN_MODE_BF16), sm_100a.
//
// One CTA per sequence: 16 compute warps plus one warp that issues every tcgen05 MMA; the whole fp32 state S^T [D=512 x d_v=64]
// lives in tensor memory (4 slices of 128 features = 4 x 64 TMEM columns) for the
// entire sequence.  Per chunk of C = 64 tokens:
//
//   slice loop s = 0..3 (features [128s, 128s+128), Omega blocks 2s, 2s+1):
//     L  tcgen05 (bf16): Z = [k;q] Omega_s^T   (M=128 tokens, N=128 features, K=64)
//        -- the lift of slice s+1 is issued as soon as Z(s) has been read, so it
//           runs under the cosines of slice s
//     F  u = cos(tau_inv z + b) -> fp16 tile F = [U_k,s; U_q,s] (un-normalised),
//        per-token sums of squares; U_k,s is also kept for the state update
//     M  tcgen05 (fp16): [G;P] += F U_k,s^T,  [X;Yq] += F S_s^T          [TMEM]
//   then, on the 64x64 chunk matrices (CUDA cores):
//     feature norms (phi = u / (||u|| + 1e-8) become row/column scalings),
//     A_ij = beta_i exp(g_i - g_j) G_ij (j<i),  R = beta (v - exp(g) X),
//     E = (I + A)^-1 R (16x16 diagonal-block inverses + blocked forward substitution),
//     Aq_ij = exp(g_{i-1} - g_j) P_ij (j<i),  E'' = exp(g_{C-1} - g_j) s_kj e_j (fp16)
//   O  tcgen05 (fp16): [0; Aq] E -> lanes of the q rows;  y_i = exp(g_{i-1}) Yq_i + (Aq E)_i
//   S  tcgen05 (fp16): S_s^T = exp(g_{C-1}) S_s^T + U_k,s^T E''   for s = 0..3 [TMEM, fp32]
//
// The algebra is the one of the CUDA-core path (prefill_simt.cu), itself the
// reference chunk step kernels/fused_kernel_deltanet.py:95-149 rearranged.
// Products accumulate in fp32; the features, the state's operand copy and E''
// are fp16 (10-bit mantissa; cosines are bounded, the other operands saturate);
// the lift product is bf16 x bf16 and exact up to fp32 accumulation (Omega is
// integers / 8, checked on the host).
#include <math.h>

#include "kdn_internal.h"
#include "tc_chunk.cuh"

namespace kdn {
namespace {

using namespace tcc;

__device__ int g_tc_error;

constexpr int kComputeWarps = 16;                 // 4 per TMEM lane quarter
constexpr int kComputeThreads = 32 * kComputeWarps;
constexpr int kIssuerWarp = kComputeWarps;        // one extra warp issues all tcgen05 MMAs
constexpr int kThr = 32 * (kComputeWarps + 1);
constexpr uint32_t kWaitLimit = 1u << 24;

// TMEM columns
constexpr uint32_t COL_S = 0;     // S^T master: slice s at 64 s (lanes = features, cols = dv), fp32
constexpr uint32_t COL_Z = 256;   // lift result: lanes = [k;q] tokens, 128 cols = features
constexpr uint32_t COL_GP = 384;  // [G;P]: lanes = [k;q] tokens, 64 cols = k tokens; later [junk; Aq E]
constexpr uint32_t COL_XY = 448;  // [X;Yq]: lanes = [k;q] tokens, 64 cols = dv

// shared-memory map (bytes from a 1024-aligned base)
constexpr uint32_t OFF_OMG = 0;        // 64 KiB Omega, slice s at 16 KiB s (bf16, K-major 128 x 64)
constexpr uint32_t OFF_XIN = 65536;    // 16 KiB [k;q] inputs (bf16, K-major)
constexpr uint32_t OFF_F = 81920;      // 32 KiB features [U_k;U_q] (fp16, K-major) | algebra: A, R (f32); then
                                       //        the A operand [0; Aq] (fp16, K-major) of the output product
constexpr uint32_t OFF_UK = 114688;    // 64 KiB U_k per slice (fp16), A operand of the state update
constexpr uint32_t OFF_SB = 180224;    // 16 KiB state slice operand (fp16, MN-major)| algebra: E (f32)
constexpr uint32_t OFF_EB = 196608;    // 8 KiB  E'' (fp16, MN-major), B operand of the state update
constexpr uint32_t OFF_VB = 204800;    // 8 KiB  v rows of the chunk (bf16)
constexpr uint32_t OFF_TD = 212992;    // 4 KiB  diagonal 16x16 blocks of (I + A)^-1 | then E (fp16, MN-major,
constexpr uint32_t OFF_US = 217088;    // 4 KiB  forward-substitution scratch        |  8 KiB over TD+US)
constexpr uint32_t OFF_PH = 221184;    // 2 KiB  phase b[512]
constexpr uint32_t OFF_GL = 223232;    // 5 x 256 B: g, beta, exp(g), exp(g_{i-1}), exp(g_{C-1} - g)
constexpr uint32_t OFF_SSP = 224512;   // 2 KiB  sums of squares per column quarter [4][128]
constexpr uint32_t OFF_SC = 226560;    // 512 B  token scales s = amp / (amp ||u|| + 1e-8)
constexpr uint32_t OFF_BAR = 227072;   // 6 mbarriers + TMEM address
constexpr uint32_t kSmemBytes = 227128 + 1024;  // + alignment slack

template <bool kVar>
__global__ void __launch_bounds__(kThr, 1) prefill_tc_kernel(TcArgs a_in, ProjParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm;
  {
    const uint32_t s = tc::smem_u32(smem_raw);
    sm = smem_raw + ((1024u - (s & 1023u)) & 1023u);
  }
  const uint32_t sbase = tc::smem_u32(sm);
  float* Am = reinterpret_cast<float*>(sm + OFF_F);  // algebra phase views
  float* Rm = reinterpret_cast<float*>(sm + OFF_F + 16384);
  float* Es = reinterpret_cast<float*>(sm + OFF_SB);
  float* TD = reinterpret_cast<float*>(sm + OFF_TD);
  float* US = reinterpret_cast<float*>(sm + OFF_US);
  float* ph = reinterpret_cast<float*>(sm + OFF_PH);
  float* gl = reinterpret_cast<float*>(sm + OFF_GL);
  float* bt = gl + 64;
  float* eg = gl + 128;
  float* egp = gl + 192;
  float* wdec = gl + 256;
  float* ssp = reinterpret_cast<float*>(sm + OFF_SSP);
  float* sc = reinterpret_cast<float*>(sm + OFF_SC);
  uint64_t* bar_lift = reinterpret_cast<uint64_t*>(sm + OFF_BAR);       // lift products done
  uint64_t* bar_mma = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 8);    // other products done
  uint64_t* bar_xin = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 16);   // chunk inputs in shared memory
  uint64_t* bar_zfree = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 24); // lift result read by all
  uint64_t* bar_fready = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 32);// feature / state tiles stored
  uint64_t* bar_ops = reinterpret_cast<uint64_t*>(sm + OFF_BAR + 40);   // output / update operands stored
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_BAR + 48);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t ns = blockIdx.x;  // scan index: rows of the initial / final state
  TcArgs a = a_in;
  int64_t n = ns;                 // token-block index of the scan's inputs and outputs
  if (kVar) {                     // varlen batch: rebase the token-side pointers on this scan's rows
    const int64_t base = a_in.var_off[ns], len = a_in.var_len[ns];
    n = 0;
    if (base < 0 || len < 0 || base > a_in.var_rows - len) {  // malformed: no token access, state passes
      a.T = 0;
      if (tid == 0) record_device_error(&g_tc_error, kErrSlotOutOfRange);
    } else {
      const int64_t in_es = a.in_dtype == KDN_DTYPE_BF16 ? 2 : 4, g_es = a.gate_dtype == KDN_DTYPE_BF16 ? 2 : 4;
      const int64_t y_es = a.y_dtype == KDN_DTYPE_BF16 ? 2 : 4;
      a.T = len;
      a.q = static_cast<const char*>(a.q) + base * 64 * in_es;
      a.k = static_cast<const char*>(a.k) + base * 64 * in_es;
      a.v = static_cast<const char*>(a.v) + base * kDV * in_es;
      a.beta = static_cast<const char*>(a.beta) + base * g_es;
      if (a.decay) a.decay = static_cast<const char*>(a.decay) + base * g_es;
      a.y = static_cast<char*>(a.y) + base * kDV * y_es;
    }
    a.NC = int((a.T + kC - 1) / kC);
  }
  const int quarter = warp & 3, cq = (warp >> 2) & 3;  // TMEM lane quarter, column quarter
  const int trow = quarter * 32 + lane;                // TMEM lane owned by this thread
  const uint32_t lane_off = uint32_t(quarter * 32) << 16;
  const bool bf_in = a.in_dtype == KDN_DTYPE_BF16;
  const bool decayed = a.decay != nullptr;
  bool ok = true;

  // ---------------------------------------------------------------- setup
  if (warp == 0) {
    tc::tmem_alloc(tslot, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(bar_lift, 1);
    tc::mbar_init(bar_mma, 1);
    tc::mbar_init(bar_xin, kComputeWarps);
    tc::mbar_init(bar_zfree, kComputeWarps);
    tc::mbar_init(bar_fready, kComputeWarps);
    tc::mbar_init(bar_ops, kComputeWarps);
    tc::fence_mbar_init();
  }
  build_omega(sm + OFF_OMG, P, warp, lane, kThr / 32);
  for (int i = tid; i < kD; i += kThr) ph[i] = P.phase[i];
  if (warp < kComputeWarps && bf_in) {
    prefetch_kq(a, n, 0, sbase + OFF_XIN, tid);
    prefetch_v(a, n, 0, sbase + OFF_VB, tid);
  }
  tc::cp_async_commit();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  if (warp < kComputeWarps) {  // state master S^T (fp32) from the initial state
#pragma unroll
    for (int s = 0; s < kSlices; ++s) {
      float v[16];
      const int f = 128 * s + trow;
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = a.S0 ? a.S0[(ns * kDV + 16 * cq + j) * kD + f] : 0.f;
      tc::tmem_st16(tmem + lane_off + COL_S + 64 * s + 16 * cq, v);
    }
    tc::tmem_st_wait();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (warp == kIssuerWarp) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      const uint32_t id_lift = tc::idesc_bf16_f32(128, 128, false, false);
      const uint32_t id_gp = tc::idesc_f16_f32(128, 64, false, false);
      const uint32_t id_xy = tc::idesc_f16_f32(128, 64, false, true);
      const uint32_t id_ds = tc::idesc_f16_f32(128, 64, true, true);
      uint32_t p_xin = 0, p_zfree = 0, p_fready = 0, p_ops = 0;
      auto lift = [&](int s) {
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16)
          tc::mma_ss(tmem + COL_Z, tc::smem_desc_sw128(sbase + OFF_XIN + 2 * k0, 16, 1024),
                     tc::smem_desc_sw128(sbase + OFF_OMG + s * 16384 + 2 * k0, 16, 1024), id_lift, k0 > 0);
        tc::mma_commit(bar_lift);
      };
      for (int c = 0; c < a.NC; ++c) {
        ok &= tc::mbar_wait_bounded(bar_xin, p_xin, kWaitLimit);
        p_xin ^= 1;
        tc::fence_after_sync();
        lift(0);
        for (int s = 0; s < kSlices; ++s) {
          ok &= tc::mbar_wait_bounded(bar_zfree, p_zfree, kWaitLimit);
          p_zfree ^= 1;
          tc::fence_after_sync();
          if (s + 1 < kSlices) lift(s + 1);  // runs under the cosines of slice s
          ok &= tc::mbar_wait_bounded(bar_fready, p_fready, kWaitLimit);
          p_fready ^= 1;
          tc::fence_after_sync();
#pragma unroll
          for (int k0 = 0; k0 < 128; k0 += 16) {
            const uint64_t fd = tc::smem_desc_sw128(sbase + OFF_F + (k0 >> 6) * 16384 + 2 * (k0 & 63), 16, 1024);
            const uint64_t sd = tc::smem_desc_sw128(sbase + OFF_SB + 128 * k0, 16384, 1024);
            tc::mma_ss(tmem + COL_GP, fd, fd, id_gp, s > 0 || k0 > 0);
            tc::mma_ss(tmem + COL_XY, fd, sd, id_xy, s > 0 || k0 > 0);
          }
          tc::mma_commit(bar_mma);
        }
        ok &= tc::mbar_wait_bounded(bar_ops, p_ops, kWaitLimit);
        p_ops ^= 1;
        tc::fence_after_sync();
#pragma unroll
        for (int k0 = 0; k0 < 64; k0 += 16)  // [0; Aq] E -> lanes of the q rows
          tc::mma_ss(tmem + COL_GP, tc::smem_desc_sw128(sbase + OFF_F + 2 * k0, 16, 1024),
                     tc::smem_desc_sw128(sbase + OFF_TD + 128 * k0, 8192, 1024), id_xy, k0 > 0);
#pragma unroll
        for (int s = 0; s < kSlices; ++s)  // S_s^T += U_k,s^T E''
#pragma unroll
          for (int k0 = 0; k0 < 64; k0 += 16)
            tc::mma_ss(tmem + COL_S + 64 * s,
                       tc::smem_desc_sw128(sbase + OFF_UK + s * 16384 + 128 * k0, 8192, 1024),
                       tc::smem_desc_sw128(sbase + OFF_EB + 128 * k0, 8192, 1024), id_ds, true);
        tc::mma_commit(bar_mma);
      }
    }
    __syncwarp();
  } else {
    // ============================================================ compute warps
    uint32_t ph_lift = 0, ph_mma = 0;
    // gates of the coming chunk (warp 0), as raw bits: converting at the load would make the warp wait
    // for it there, and the next chunk's gates are only used a chunk later
    const bool gate_bf = a.gate_dtype == KDN_DTYPE_BF16;
    uint32_t nb[2] = {0u, 0u}, nd[2] = {0x3f800000u, 0x3f800000u};
    auto load_gates = [&](int64_t t_first) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t tt = t_first + 2 * lane + e;
        nb[e] = 0u;
        nd[e] = 0x3f800000u;  // 1.0f
        if (tt < a.T) {
          nb[e] = ld_gate_bits(a.beta, gate_bf, n * a.T + tt);
          if (decayed) nd[e] = ld_gate_bits(a.decay, gate_bf, n * a.T + tt);
        }
      }
    };
    auto gate_f32 = [&](uint32_t bits) { return __uint_as_float(gate_bf ? bits << 16 : bits); };
    if (warp == 0) load_gates(0);
    for (int c = 0; c < a.NC; ++c) {
      const int64_t t0 = int64_t(c) * kC;
      const bool has_next = c + 1 < a.NC;
      // -------------------------------------------- chunk inputs ready -> lift of slice 0
      tc::cp_async_wait_all();
      if (!bf_in) load_kq_f32(a, n, c, sm + OFF_XIN, tid);
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_xin);
      tc::named_bar_sync(1, kComputeThreads);  // v rows copied by other threads are visible
      if (warp == 0) {  // gates: beta, inclusive scan of log clamp(decay, 1e-5, 1), derived factors
        const float lg0 = decayed ? logf(fminf(fmaxf(gate_f32(nd[0]), 1e-5f), 1.0f)) : 0.f;
        const float lg1 = decayed ? logf(fminf(fmaxf(gate_f32(nd[1]), 1e-5f), 1.0f)) : 0.f;
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
        bt[2 * lane] = gate_f32(nb[0]);
        bt[2 * lane + 1] = gate_f32(nb[1]);
        eg[2 * lane] = __expf(g0);
        eg[2 * lane + 1] = __expf(g1);
        egp[2 * lane] = lane == 0 ? 1.f : __expf(gprev);
        egp[2 * lane + 1] = __expf(g0);
        wdec[2 * lane] = __expf(gend - g0);
        wdec[2 * lane + 1] = __expf(gend - g1);
        if (has_next) load_gates(t0 + kC);
      }

      // -------------------------------------------- slice loop
      float ss = 0.f;
#pragma unroll 1
      for (int s = 0; s < kSlices; ++s) {
        ok &= tc::mbar_wait_bounded(bar_lift, ph_lift, kWaitLimit);
        ph_lift ^= 1;
        tc::fence_after_sync();
        float z[32];
        tc::tmem_ld32(tmem + lane_off + COL_Z + 32 * cq, z);
        tc::tmem_ld_wait();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_zfree);
        // u = cos(tau_inv z + b): the hardware cosine is accurate to ~1e-6 absolute for
        // the |arguments| <= 32 met here, far below the fp16 spacing of the stored result
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
        uint32_t sp[8];
        {
          float v[16];
          tc::tmem_ld16(tmem + lane_off + COL_S + 64 * s + 16 * cq, v);
          tc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 8; ++j) sp[j] = pack_f16_sat(v[2 * j], v[2 * j + 1]);
        }
        if (s > 0) {  // the previous slice's products must be done with F and SB
          ok &= tc::mbar_wait_bounded(bar_mma, ph_mma, kWaitLimit);
          ph_mma ^= 1;
        }
        {
          const int kb = cq >> 1, e0 = 32 * (cq & 1);
          uint8_t* fb = sm + OFF_F + kb * 16384;
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const uint4 pk = make_uint4(fp[4 * c8], fp[4 * c8 + 1], fp[4 * c8 + 2], fp[4 * c8 + 3]);
            const uint32_t off = tc::sw128_offset(trow, e0 + 8 * c8);
            *reinterpret_cast<uint4*>(fb + off) = pk;
            if (trow < 64) *reinterpret_cast<uint4*>(sm + OFF_UK + s * 16384 + kb * 8192 + off) = pk;
          }
#pragma unroll
          for (int c8 = 0; c8 < 2; ++c8)
            *reinterpret_cast<uint4*>(sm + OFF_SB + tc::sw128_offset(trow, 16 * cq + 8 * c8)) =
                make_uint4(sp[4 * c8], sp[4 * c8 + 1], sp[4 * c8 + 2], sp[4 * c8 + 3]);
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(bar_fready);
      }
      ssp[cq * 128 + trow] = ss;
      // all lifts have completed: the input tile is free for the next chunk's k,q rows
      if (has_next && bf_in) prefetch_kq(a, n, c + 1, sbase + OFF_XIN, tid);
      tc::cp_async_commit();
      ok &= tc::mbar_wait_bounded(bar_mma, ph_mma, kWaitLimit);
      ph_mma ^= 1;
      tc::fence_after_sync();

      // -------------------------------------------- chunk matrices
      float gp[16], xy[16], vv[16];
      tc::tmem_ld16(tmem + lane_off + COL_GP + 16 * cq, gp);
      tc::tmem_ld16(tmem + lane_off + COL_XY + 16 * cq, xy);
      tc::tmem_ld_wait();
      if (trow < 64) {
        const int64_t t = t0 + trow;
        if (bf_in) {
          const uint4* vr = reinterpret_cast<const uint4*>(sm + OFF_VB + trow * 128 + 32 * cq);
          const uint4 w0 = vr[0], w1 = vr[1];
          const __nv_bfloat162* h0 = reinterpret_cast<const __nv_bfloat162*>(&w0);
          const __nv_bfloat162* h1 = reinterpret_cast<const __nv_bfloat162*>(&w1);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f0 = __bfloat1622float2(h0[j]), f1 = __bfloat1622float2(h1[j]);
            vv[2 * j] = f0.x;
            vv[2 * j + 1] = f0.y;
            vv[8 + 2 * j] = f1.x;
            vv[8 + 2 * j + 1] = f1.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            vv[j] = t < a.T ? reinterpret_cast<const float*>(a.v)[(n * a.T + t) * kDV + 16 * cq + j] : 0.f;
        }
      }
      tc::named_bar_sync(1, kComputeThreads);  // sums of squares and gates visible; v tile consumed
      if (has_next && bf_in) prefetch_v(a, n, c + 1, sbase + OFF_VB, tid);
      tc::cp_async_commit();
      if (tid < 128)
        sc[tid] = P.amp / (P.amp * sqrtf(ssp[tid] + ssp[128 + tid] + ssp[256 + tid] + ssp[384 + tid]) + 1e-8f);
      tc::named_bar_sync(1, kComputeThreads);
      {  // q-row threads park their row of Aq and of the scaled Yq in the (free) lift columns
        const int i = trow & 63;
        const float si = sc[trow];
        const float bi = bt[i];
        if (trow < 64) {  // k row: A (from G) and R (from X)
          const float gi = gl[i], egi = eg[i];
#pragma unroll
          for (int j4 = 0; j4 < 4; ++j4) {
            const float4 sj = *reinterpret_cast<const float4*>(sc + 16 * cq + 4 * j4);
            const float sjv[4] = {sj.x, sj.y, sj.z, sj.w};
            float4 av, rv;
            float* ap = &av.x;
            float* rp = &rv.x;
#pragma unroll
            for (int qx = 0; qx < 4; ++qx) {
              const int jj = 4 * j4 + qx, j = 16 * cq + jj;
              const float dec = decayed ? __expf(gi - gl[j]) : 1.f;
              ap[qx] = (j < i) ? bi * dec * gp[jj] * si * sjv[qx] : 0.f;
              rp[qx] = bi * (vv[jj] - egi * xy[jj] * si);
            }
            *reinterpret_cast<float4*>(Am + sx(i, 16 * cq + 4 * j4)) = av;
            *reinterpret_cast<float4*>(Rm + sx(i, 16 * cq + 4 * j4)) = rv;
          }
        } else {  // q row
          const float gp_i = i > 0 ? gl[i - 1] : 0.f, yscale = si * egp[i];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int j = 16 * cq + jj;
            const float dec = decayed ? __expf(gp_i - gl[j]) : 1.f;
            gp[jj] = (j < i) ? dec * gp[jj] * si * sc[j] : 0.f;
            xy[jj] *= yscale;
          }
        }
      }
      if (trow >= 64) {
        tc::tmem_st16(tmem + lane_off + COL_Z + 16 * cq, gp);
        tc::tmem_st16(tmem + lane_off + COL_Z + 64 + 16 * cq, xy);
        tc::tmem_st_wait();
      }
      tc::named_bar_sync(1, kComputeThreads);
      // diagonal 16x16 blocks of (I + A)^-1: one warp per block, one lane per column
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
      tc::named_bar_sync(1, kComputeThreads);
      // E = (I + A)^-1 R by block rows (U = R_I - sum_{J<I} A_IJ E_J ; E_I = T_II U), on warps
      // 0-3: warp w owns rows 4w..4w+3 of the block, lane l columns 2l, 2l+1 (E, U row-major)
      if (warp < 4) {
        const int c2 = 2 * lane;
#pragma unroll
        for (int I = 0; I < 4; ++I) {
          float2 acc[4];
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) acc[rr] = *reinterpret_cast<const float2*>(Rm + sx(16 * I + 4 * warp + rr, c2));
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
          for (int kk = 0; kk < 16; ++kk) {  // T_II is lower triangular (zeros above)
            const float2 u = *reinterpret_cast<const float2*>(US + kk * 64 + c2);
#pragma unroll
            for (int rr = 0; rr < 4; ++rr) {
              const float tv = TD[(I * 16 + 4 * warp + rr) * 16 + kk];
              ev[rr].x = fmaf(tv, u.x, ev[rr].x);
              ev[rr].y = fmaf(tv, u.y, ev[rr].y);
            }
          }
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) *reinterpret_cast<float2*>(Es + (16 * I + 4 * warp + rr) * 64 + c2) = ev[rr];
          tc::named_bar_sync(2, 128);
        }
      }
      tc::named_bar_sync(1, kComputeThreads);
      // operands of the output and state products
      {
        const int j = tid >> 3, c8 = (tid & 7) * 8;  // one 8-wide piece of row j of E per thread
        const float4 e0 = *reinterpret_cast<const float4*>(Es + j * 64 + c8);
        const float4 e1 = *reinterpret_cast<const float4*>(Es + j * 64 + c8 + 4);
        const uint32_t off = tc::sw128_offset(j, c8);
        *reinterpret_cast<uint4*>(sm + OFF_TD + off) =  // E (fp16, MN-major) over TD+US
            make_uint4(pack_f16_sat(e0.x, e0.y), pack_f16_sat(e0.z, e0.w), pack_f16_sat(e1.x, e1.y),
                       pack_f16_sat(e1.z, e1.w));
        const float w = wdec[j] * sc[j];
        *reinterpret_cast<uint4*>(sm + OFF_EB + off) =  // E'' = exp(g_{C-1} - g_j) s_kj e_j
            make_uint4(pack_f16_sat(w * e0.x, w * e0.y), pack_f16_sat(w * e0.z, w * e0.w),
                       pack_f16_sat(w * e1.x, w * e1.y), pack_f16_sat(w * e1.z, w * e1.w));
        // A operand [0; Aq] (fp16, K-major, 128 rows x 64) in the (now free) feature tile
        if (trow < 64) {
          if (cq < 2) {
#pragma unroll
            for (int z8 = 0; z8 < 4; ++z8)
              *reinterpret_cast<uint4*>(sm + OFF_F + tc::sw128_offset(trow, 32 * cq + 8 * z8)) = make_uint4(0, 0, 0, 0);
          }
        } else {
          float aq[16];
          tc::tmem_ld16(tmem + lane_off + COL_Z + 16 * cq, aq);
          tc::tmem_ld_wait();
#pragma unroll
          for (int c8b = 0; c8b < 2; ++c8b)
            *reinterpret_cast<uint4*>(sm + OFF_F + tc::sw128_offset(trow, 16 * cq + 8 * c8b)) = make_uint4(
                pack_f16_sat(aq[8 * c8b], aq[8 * c8b + 1]), pack_f16_sat(aq[8 * c8b + 2], aq[8 * c8b + 3]),
                pack_f16_sat(aq[8 * c8b + 4], aq[8 * c8b + 5]), pack_f16_sat(aq[8 * c8b + 6], aq[8 * c8b + 7]));
        }
      }
      if (decayed) {  // decay of the carried state
        const float gC = eg[63];
#pragma unroll
        for (int s = 0; s < kSlices; ++s) {
          float v[16];
          tc::tmem_ld16(tmem + lane_off + COL_S + 64 * s + 16 * cq, v);
          tc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= gC;
          tc::tmem_st16(tmem + lane_off + COL_S + 64 * s + 16 * cq, v);
        }
        tc::tmem_st_wait();
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      tc::named_bar_sync(1, kComputeThreads);  // also: gates of this chunk no longer read
      if (lane == 0) tc::mbar_arrive(bar_ops);
      ok &= tc::mbar_wait_bounded(bar_mma, ph_mma, kWaitLimit);
      ph_mma ^= 1;
      tc::fence_after_sync();
      // outputs: y_i = exp(g_{i-1}) s_qi Yq_i + (Aq E)_i, by the threads of the q rows
      if (trow >= 64) {
        float ye[16], yq[16];
        tc::tmem_ld16(tmem + lane_off + COL_GP + 16 * cq, ye);
        tc::tmem_ld16(tmem + lane_off + COL_Z + 64 + 16 * cq, yq);
        tc::tmem_ld_wait();
        const int i = trow - 64;
        const int64_t t = t0 + i;
        if (t < a.T) {
          const int64_t o = (n * a.T + t) * kDV + 16 * cq;
          float yy[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) yy[j] = yq[j] + ye[j];
          if (a.y_dtype == KDN_DTYPE_BF16) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.y) + o);
            dst[0] = make_uint4(pack_bf16(yy[0], yy[1]), pack_bf16(yy[2], yy[3]), pack_bf16(yy[4], yy[5]),
                                pack_bf16(yy[6], yy[7]));
            dst[1] = make_uint4(pack_bf16(yy[8], yy[9]), pack_bf16(yy[10], yy[11]), pack_bf16(yy[12], yy[13]),
                                pack_bf16(yy[14], yy[15]));
          } else {
            float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.y) + o);
#pragma unroll
            for (int u = 0; u < 4; ++u) dst[u] = make_float4(yy[4 * u], yy[4 * u + 1], yy[4 * u + 2], yy[4 * u + 3]);
          }
        }
      }
      tc::fence_before_sync();
    }
    // ------------------------------------------------------------ output state
#pragma unroll
    for (int s = 0; s < kSlices; ++s) {
      float v[16];
      tc::tmem_ld16(tmem + lane_off + COL_S + 64 * s + 16 * cq, v);
      tc::tmem_ld_wait();
      const int f = 128 * s + trow;
#pragma unroll
      for (int j = 0; j < 16; ++j) a.S_out[(ns * kDV + 16 * cq + j) * kD + f] = v[j];
    }
    tc::cp_async_wait_all();
  }
  if (!ok) record_device_error(&g_tc_error, kErrTcWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 512);
}

}  // namespace

bool tc_prefill_supported(int D, int dv, int C, const ProjParams& P) {
  if (D != kD || dv != kDV || C != kC) return false;
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

cudaError_t launch_tc_prefill(const PrefillProblem& p, const ProjParams& P, cudaStream_t stream, LaunchMarks& marks) {
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
  a.var_off = p.var_off;
  a.var_len = p.var_len;
  a.var_rows = p.var_rows;
  auto kern = a.var_off ? prefill_tc_kernel<true> : prefill_tc_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
  if (e != cudaSuccess) return e;
  marks.begin(stream);
  kern<<<unsigned(p.N), kThr, kSmemBytes, stream>>>(a, P);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  marks.after(stream);
  return cudaSuccess;
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
