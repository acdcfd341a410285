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
//     T' = T diag(beta exp(g) s_k),  U = T diag(beta) V                  (U: tcgen05)
//     Aq_ij = exp(g_{i-1} - g_j) s_qi s_kj P_ij (j<i)
//   and writes a chunk record: U_q, U_k, T' (fp16, already in the swizzled shared-memory
//   layouts the later passes feed to the tensor core), U (fp32), Aq (fp16) and the
//   per-token factors.
//
//   phase 2, state_pass_kernel -- two CTAs per sequence (32 value columns each), serial
//   over chunks, only the state-dependent products (the fp32 state stays in TMEM):
//     Y = U_k S^T (K = 512),  X = T' Y,  E = U - X,  E'' = exp(g_{C-1} - g_j) s_kj e_j
//     S^T = exp(g_{C-1}) S^T + U_k^T E''
//   streaming 72 KiB per chunk (U_k serves both as the A operand of Y and, read as its
//   transpose, of the update); it stores the state entering each chunk and E.
//
//   phase 3, output_pass_kernel -- every chunk at once again:
//     y_i = s_qi exp(g_{i-1}) (U_q S^T)_i + (Aq E)_i
//
// This is the chunk algebra of prefill_tc.cu (the reference chunk step
// kernels/fused_kernel_deltanet.py:95-149) with (I + A)^-1 applied to the state
// independent parts ahead of time: E = T (beta (v - exp(g) s X')) = U - T' (U_k S^T).
// Records take 233 KiB per chunk of the workspace; nothing else is allocated.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "kdn_internal.h"
#include "tc_chunk.cuh"

namespace kdn {
namespace {

using namespace tcc;

__device__ int g_split_error;

constexpr uint32_t kWaitLimit = 1u << 24;

// ------------------------------------------------ chunk record (workspace)
constexpr uint32_t REC_Q = 0;         // 64 KiB  U_q fp16, K-major SW128: K-block kb (features 64kb..64kb+63)
                                      //          at 8 KiB kb, [64 tokens x 128 B]
constexpr uint32_t REC_UK = 65536;    // 64 KiB  U_k fp16: slice s at 16 KiB s, half h at 8 KiB h,
                                      //          [64 tokens x 64 features] SW128
constexpr uint32_t REC_TP = 131072;   // 8 KiB   T' = T diag(beta exp(g) s_k) fp16, K-major SW128 [64 x 64]
constexpr uint32_t REC_U = 139264;    // 16 KiB  U = T diag(beta) V fp32: column half h (value columns
                                      //          32h..32h+31) at 8 KiB h, row-major [64 tokens][32]
constexpr uint32_t REC_AQ = 155648;   // 8 KiB   Aq fp16 K-major SW128 [64 rows x 64]
constexpr uint32_t REC_VEC = 163840;  // 1 KiB   ew[64] = exp(g_{C-1} - g_j) s_kj, yqs[64] = s_qi exp(g_{i-1}),
                                      //          eC = exp(g_{C-1})
// written by the state pass (phase 2), read by the output pass (phase 3):
constexpr uint32_t REC_S0 = 164864;   // 64 KiB  state entering the chunk, S^T fp16, two column halves h at
                                      //          32 KiB h, each MN-major SW64 [512 features x 32]
constexpr uint32_t REC_E = 230400;    // 8 KiB   E fp16, halves at 4 KiB h, MN-major SW64 [64 tokens x 32]
constexpr uint32_t REC_BYTES = 238592;

struct SplitArgs {
  TcArgs a;
  int64_t N;
  uint8_t* ws;       // N * NC records, chunk-major: record (c, n) at (c N + n) REC_BYTES
  uint32_t* abort;   // persistent launch: set by any wait that gives up, so that every other
                     // wait gives up at once (nullptr for the separate launches)
};

__device__ __forceinline__ uint8_t* record(const SplitArgs& sa, int64_t c, int64_t n) {
  return sa.ws + (c * sa.N + n) * int64_t(REC_BYTES);
}

__device__ __forceinline__ bool aborted(const uint32_t* abort) {
  return abort && *reinterpret_cast<const volatile uint32_t*>(abort) != 0u;
}
__device__ __forceinline__ void set_abort(uint32_t* abort) {
  if (abort) atomicExch(abort, 1u);
}

// bounded mbarrier wait of this path; gives up early once another wait has given up
__device__ __forceinline__ bool split_wait(uint64_t* bar, uint32_t parity, uint32_t* abort) {
  uint32_t n = 0;
  while (!tc::mbar_try_wait(bar, parity)) {
    if ((++n & 1023u) == 0 && (n >= kWaitLimit || aborted(abort))) {
      set_abort(abort);
      return false;
    }
  }
  return true;
}

// Phase parities of a group of barriers live in one register, bit i for barrier i: an
// array indexed by a run-time slot would sit in local memory, and beside this path's
// shared-memory carve-out the L1 is too small to keep it (each access became an L2
// round trip of hundreds of cycles on the issuing thread's chain).  These wait for the
// phase whose parity is bit i of `bits`, then flip the bit.
__device__ __forceinline__ bool split_wait_bit(uint64_t* bar, uint32_t& bits, int i, uint32_t* abort) {
  const bool r = split_wait(bar, (bits >> i) & 1u, abort);
  bits ^= 1u << i;
  return r;
}

// ---- hand-over flags between the phases of the persistent launch (global memory)
constexpr uint32_t kFlagSpins = 1u << 24;  // bounded: ~10 s of polling at most
// wait until *flag >= target (acquire at GPU scope)
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t target, uint32_t* abort) {
  for (uint32_t i = 0; i < kFlagSpins; ++i) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= target) return true;
    if ((i & 63u) == 63u && aborted(abort)) return false;
    __nanosleep(64);
  }
  set_abort(abort);
  return false;
}
// completed writes of this thread (generic, and bulk copies already waited for) are ordered
// before *flag = v at GPU scope
__device__ __forceinline__ void publish_store(uint32_t* flag, uint32_t v) {
  tc::fence_proxy_async_global();
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}
// ================================================================ phase 1
// The preparation runs two chunks at once on every CTA: 8 lift warps take the features of chunk
// r + 1 (TMEM -> cosines -> fp16 tiles, MUFU-bound) while 8 algebra warps finish chunk r (scales,
// A, Aq, T = (I + A)^-1, the operand of U and U's copy-out: latency-bound CUDA-core work), so the two
// kinds of work overlap instead of taking turns.  One thread issues every MMA and one copies the
// record out; both poll their barriers and serve whichever side is ready.
constexpr int kP1Warps = 16;                  // compute warps
constexpr int kP1Lift = 8;                    // warps 0..7: lift warps, 2 per TMEM lane quarter
constexpr int kP1Alg = 8;                     // warps 8..15: algebra warps, 2 per TMEM lane quarter
constexpr int kP1AlgThreads = 32 * kP1Alg;
constexpr int kP1Issuer = kP1Warps;           // issues every MMA (lane 0)
constexpr int kP1Publisher = kP1Warps + 1;    // copies the record out and publishes it (lane 0)
constexpr int kP1Thr = 32 * (kP1Warps + 2);
constexpr uint32_t kPollLimit = 1u << 26;     // idle rounds of the issuer / publisher (~64 ns each)

// TMEM columns (phase 1)
constexpr uint32_t P1_Z = 0;     // lift results, 2 x 128 cols (slices s at 128 (s & 1))
constexpr uint32_t P1_GP = 256;  // [G; P] of chunk r at 64 (r & 1), 2 x 64 cols
constexpr uint32_t P1_U = 384;   // U in lanes 64..127, 64 cols

// shared memory (phase 1)
constexpr uint32_t P1_OMG = 0;        // 64 KiB Omega (bf16)
constexpr uint32_t P1_XIN = 65536;    // 16 KiB [k; q] (bf16, K-major)
constexpr uint32_t P1_F = 81920;      // 32 KiB slice features [U_k; U_q] of even slices
constexpr uint32_t P1_AQ = 114688;    // 8 KiB  Aq (fp16, K-major SW128), copied to the record
constexpr uint32_t P1_VEC = 122880;   // 1 KiB  per-token factors of the state pass, copied to the record
constexpr uint32_t P1_F1 = 124928;    // 32 KiB slice features of odd slices (two buffers: a slice's
                                      //        features are written while the previous slice's Gram
                                      //        product and copy-out still read the other buffer)
constexpr uint32_t P1_ES = 157696;    // 17 KiB T = (I + A)^-1 (fp32), rows kEsLd floats apart; between
                                      //        chunks, the next chunk's v rows
constexpr int kEsLd = 68;             // padded row: the row-wise float4 reads of 8 rows hit distinct banks
constexpr uint32_t P1_GL = 175104;    // 3 x 1280 B gates of chunk r at 1280 (r % 3): g, beta, exp(g),
                                      //        exp(g_{i-1}), exp(g_{C-1} - g), 256 B each
constexpr uint32_t P1_VB = 180224;    // 8 KiB  V (fp16, MN-major), B operand of U; then U's value
                                      //        columns 0..31 (fp32 [64][32]), copied to the record
constexpr uint32_t P1_TOP = 188416;   // 16 KiB A (fp32, sx layout) during the inverse; then the A operand
                                      //        [T diag(beta exp(g) s_k); T diag(beta)] (fp16, K-major),
                                      //        whose second half then takes U's value columns 32..63
constexpr uint32_t P1_US = 208896;    // 4 KiB  forward-substitution scratch
constexpr uint32_t P1_PH = 212992;    // 2 KiB  phase b[512]
constexpr uint32_t P1_SSP = 216320;   // 2 KiB  sums of squares per column quarter
constexpr uint32_t P1_SC = 218368;    // 512 B  token scales
constexpr uint32_t P1_BAR = 218880;   // mbarriers
constexpr uint32_t kP1Bars = 256;     // bytes of barriers
constexpr uint32_t P1_FK = 219136;    // 256 B  beta exp(g) s_k per token: the column factors of T'
constexpr uint32_t kP1Smem = P1_FK + 256 + 1024;
static_assert(P1_VEC + 1024 <= P1_F1 && P1_F1 + 32768 <= P1_ES && P1_ES + 64 * kEsLd * 4 <= P1_GL &&
                  P1_GL + 3 * 1280 <= P1_VB &&
                  P1_BAR + kP1Bars <= P1_FK,
              "phase-1 shared-memory regions overlap");

__device__ __forceinline__ uint32_t p1_fbuf(int s) { return (s & 1) ? P1_F1 : P1_F; }  // slice s's features

// Level d of the blocked inverse T = (I + A)^-1 (16x16 blocks, T row-major in Es with rows kEsLd apart,
// A in the float4-swizzled layout of sx()): for the blocks I - J = d,
//   P = sum_{K=J}^{I-1} A_IK T_KJ  (into US),  then  T_IJ = -T_II P.
// gtid = 0..255, the algebra warps' thread index.
template <int D>
__device__ __forceinline__ void t_level(const float* Am, float* Es, float* US, int gtid) {
  constexpr int kIters = 4 - D;  // (4 - D) * 256 block elements over 256 threads
  static_assert(kP1AlgThreads == 256, "one block element per thread and block");
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int e = gtid + 256 * it;
    const int J = e >> 8, I = J + D, r = (e >> 4) & 15, cc = e & 15;
    const int row = 16 * I + r;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < 4 * D; ++q) {
      const int k = 16 * J + 4 * q;
      const float4 a4 = *reinterpret_cast<const float4*>(Am + row * 64 + ((((k >> 2) ^ row) & 15) << 2));
      acc[0] = fmaf(a4.x, Es[k * kEsLd + 16 * J + cc], acc[0]);
      acc[1] = fmaf(a4.y, Es[(k + 1) * kEsLd + 16 * J + cc], acc[1]);
      acc[2] = fmaf(a4.z, Es[(k + 2) * kEsLd + 16 * J + cc], acc[2]);
      acc[3] = fmaf(a4.w, Es[(k + 3) * kEsLd + 16 * J + cc], acc[3]);
    }
    US[e] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
  tc::named_bar_sync(1, kP1AlgThreads);
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int e = gtid + 256 * it;
    const int J = e >> 8, I = J + D, r = (e >> 4) & 15, cc = e & 15;
    const float* trow_ = Es + (16 * I + r) * kEsLd + 16 * I;
    const float* pcol = US + (J << 8) + cc;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 16; k += 4) {
      acc[0] = fmaf(trow_[k], pcol[k << 4], acc[0]);
      acc[1] = fmaf(trow_[k + 1], pcol[(k + 1) << 4], acc[1]);
      acc[2] = fmaf(trow_[k + 2], pcol[(k + 2) << 4], acc[2]);
      acc[3] = fmaf(trow_[k + 3], pcol[(k + 3) << 4], acc[3]);
    }
    Es[(16 * I + r) * kEsLd + 16 * J + cc] = -((acc[0] + acc[1]) + (acc[2] + acc[3]));
  }
  tc::named_bar_sync(1, kP1AlgThreads);
}

// Polling loops of the issuer and the publisher: `poll` counts rounds without progress and gives up
// (setting the abort word) after kPollLimit of them, or at once when another wait has given up.  An
// idle round sleeps briefly, so that the polling thread takes few issue slots from the compute warps
// of its sub-partition.
__device__ __forceinline__ bool poll_on(uint32_t& poll, bool progressed, uint32_t* abort) {
  if (progressed) {
    poll = 0;
    return true;
  }
  __nanosleep(64);
  if ((++poll & 1023u) == 0 && (poll >= kPollLimit || aborted(abort))) {
    set_abort(abort);
    return false;
  }
  return true;
}

// Phase 1 on CTAs cta = 0..ncta-1 (576 threads: 8 lift warps, 8 algebra warps, an MMA issuer and a
// record publisher; `tmem` = 512 allocated columns).  Chunk records idx = cta, cta + ncta, ...  With
// rec_ready, each finished record is published there (1) for the state pass.
__device__ __forceinline__ void prep_role(const SplitArgs& sa, const ProjParams& P, uint8_t* sm, uint32_t tmem,
                                          int64_t cta, int64_t ncta, uint32_t* rec_ready, bool& ok) {
  const TcArgs& a = sa.a;
  const uint32_t sbase = tc::smem_u32(sm);
  float* Am = reinterpret_cast<float*>(sm + P1_TOP);
  float* Es = reinterpret_cast<float*>(sm + P1_ES);
  float* US = reinterpret_cast<float*>(sm + P1_US);
  float* ph = reinterpret_cast<float*>(sm + P1_PH);
  float* gates = reinterpret_cast<float*>(sm + P1_GL);  // chunk r's at 320 (r % 3) floats
  float* ssp = reinterpret_cast<float*>(sm + P1_SSP);
  float* sc = reinterpret_cast<float*>(sm + P1_SC);
  float* fk = reinterpret_cast<float*>(sm + P1_FK);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + P1_BAR);
  uint64_t* bar_lift = bars;         // [2] lift into Z slot s & 1 done (MMA commit)
  uint64_t* bar_zfree = bars + 2;    // [2] Z slot s & 1 read (8 lift warps)
  uint64_t* bar_fready = bars + 4;   // [2] a slice's features written to buffer s & 1 (8 lift warps)
  uint64_t* bar_fdone = bars + 6;    // [2] that slice's Gram product done and its features copied out
                                     //     (MMA commit + publisher)
  uint64_t* bar_gram = bars + 8;     // [2] chunk r's last Gram product into GP buffer r & 1 done
  uint64_t* bar_xin = bars + 10;     // the next chunk's [k; q] tile in place (8 lift warps)
  uint64_t* bar_ssp = bars + 11;     // a chunk's sums of squares written (8 lift warps)
  uint64_t* bar_gpfree = bars + 12;  // a chunk's [G; P] and sums of squares read (8 algebra warps)
  uint64_t* bar_ops = bars + 13;     // the operands of U in place (8 algebra warps)
  uint64_t* bar_mma = bars + 14;     // U done (MMA commit)
  uint64_t* bar_wdone = bars + 15;   // U staged for the copy-out (8 algebra warps)
  uint64_t* bar_stfree = bars + 16;  // the chunk's staged tiles copied out (publisher)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, wh = (warp >> 2) & 1;  // TMEM lane quarter; which of the quarter's 2 warps
  const int trow = quarter * 32 + lane;
  const uint32_t lane_off = uint32_t(quarter * 32) << 16;
  const bool bf_in = a.in_dtype == KDN_DTYPE_BF16;
  const bool decayed = a.decay != nullptr;
  const int64_t N = sa.N;
  const int64_t total = N * a.NC;
  const int64_t nrec = cta < total ? (total - 1 - cta) / ncta + 1 : 0;  // this CTA's chunk records

  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&bar_lift[b], 1);
      tc::mbar_init(&bar_zfree[b], kP1Lift);
      tc::mbar_init(&bar_fready[b], kP1Lift);
      tc::mbar_init(&bar_fdone[b], 2);
      tc::mbar_init(&bar_gram[b], 1);
    }
    tc::mbar_init(bar_xin, kP1Lift);
    tc::mbar_init(bar_ssp, kP1Lift);
    tc::mbar_init(bar_gpfree, kP1Alg);
    tc::mbar_init(bar_ops, kP1Alg);
    tc::mbar_init(bar_mma, 1);
    tc::mbar_init(bar_wdone, kP1Alg);
    tc::mbar_init(bar_stfree, 1);
    tc::fence_mbar_init();
  }
  build_omega(sm + P1_OMG, P, warp, lane, kP1Thr / 32);
  for (int i = tid; i < kD; i += kP1Thr) ph[i] = P.phase[i];
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (warp == kP1Issuer) {
    // ================================================================ MMA issuer
    // Three in-order programs, served as their operands arrive: the lifts (chunk rl, slice sl), the
    // Gram products (rg, sg) and the U products (ru).
    if (lane == 0) {
      const uint32_t id_lift = tc::idesc_bf16_f32(128, 128, false, false);
      const uint32_t id_gp = tc::idesc_f16_f32(128, 64, false, false);
      const uint32_t id_n64 = tc::idesc_f16_f32(128, 64, false, true);
      uint32_t p_xin = 0, p_zfree = 0, p_fready = 0, p_ops = 0;  // p_zfree, p_fready: bits per slot
      int64_t kl = 0, kg = 0, ku = 0;                             // items issued of each program
      const int64_t nl = 4 * nrec;
      uint32_t poll = 0;
      while (ok && (kl < nl || kg < nl || ku < nrec)) {
        bool progressed = false;
        if (ku < nrec && tc::mbar_test_wait(bar_ops, p_ops)) {  // U = T diag(beta) V in lanes 64..127
          p_ops ^= 1;
          tc::fence_after_sync();
#pragma unroll
          for (int k0 = 0; k0 < 64; k0 += 16)
            tc::mma_ss(tmem + P1_U, tc::smem_desc_sw128(sbase + P1_TOP + 2 * k0, 16, 1024),
                       tc::smem_desc_sw128(sbase + P1_VB + 128 * k0, 8192, 1024), id_n64, k0 > 0);
          tc::mma_commit(bar_mma);
          ++ku;
          progressed = true;
        }
        if (kg < nl) {  // [G; P] += F_s F_s^T over the slice's features (rows 0..63 of F are U_k)
          const int sg = int(kg & 3), b = sg & 1;
          if (tc::mbar_test_wait(&bar_fready[b], (p_fready >> b) & 1u)) {
            p_fready ^= 1u << b;
            tc::fence_after_sync();
            const uint32_t gp = tmem + P1_GP + 64 * uint32_t((kg >> 2) & 1);
            const uint32_t fb = sbase + p1_fbuf(sg);
#pragma unroll
            for (int k0 = 0; k0 < 128; k0 += 16) {
              const uint64_t fd = tc::smem_desc_sw128(fb + (k0 >> 6) * 16384 + 2 * (k0 & 63), 16, 1024);
              tc::mma_ss(gp, fd, fd, id_gp, sg > 0 || k0 > 0);
            }
            tc::mma_commit(&bar_fdone[b]);  // the buffer is rewritten once the publisher has copied it out too
            if (sg == 3) tc::mma_commit(&bar_gram[(kg >> 2) & 1]);
            ++kg;
            progressed = true;
          }
        }
        if (kl < nl) {  // Z slot sl & 1 = [k; q] Omega_sl^T
          const int sl = int(kl & 3), b = sl & 1;
          // slices 0, 1 need the chunk's input tile; every use of a slot but its first needs the
          // slot's previous contents read
          bool ready = true;
          if (sl == 0) ready = tc::mbar_test_wait(bar_xin, p_xin);
          if (ready && kl >= 2) ready = tc::mbar_test_wait(&bar_zfree[b], (p_zfree >> b) & 1u);
          if (ready) {
            if (sl == 0) p_xin ^= 1;
            if (kl >= 2) p_zfree ^= 1u << b;
            tc::fence_after_sync();
#pragma unroll
            for (int k0 = 0; k0 < 64; k0 += 16)
              tc::mma_ss(tmem + P1_Z + 128 * b, tc::smem_desc_sw128(sbase + P1_XIN + 2 * k0, 16, 1024),
                         tc::smem_desc_sw128(sbase + P1_OMG + sl * 16384 + 2 * k0, 16, 1024), id_lift, k0 > 0);
            tc::mma_commit(&bar_lift[b]);
            ++kl;
            progressed = true;
          }
        }
        ok &= poll_on(poll, progressed, sa.abort);
      }
    }
    __syncwarp();
  } else if (warp == kP1Publisher) {
    // ================================================================ record copies, publication
    // Two in-order programs: the slices' features (as soon as written) and each chunk's remaining
    // tiles (once staged, and only after the chunk's feature copies were issued).  A slice's buffer is
    // handed back once its copy has read it, which is checked when the next copy is issued (the lift
    // warps rewrite it two slices later), so that this thread seldom waits on a copy.
    if (lane == 0) {
      uint32_t p_fready = 0, p_wdone = 0;  // p_fready: bits per buffer
      int64_t kf = 0, kt = 0;
      int pend = -1;  // buffer of the last feature copy, not yet handed back
      auto hand_back = [&]() {  // every copy issued so far has read its source
        if (pend >= 0) tc::mbar_arrive(&bar_fdone[pend]);
        pend = -1;
      };
      const int64_t nf = 4 * nrec;
      uint32_t poll = 0;
      while (ok && (kf < nf || kt < nrec)) {
        bool progressed = false;
        if (kf < nf) {
          const int s = int(kf & 3), b = s & 1;
          if (tc::mbar_test_wait(&bar_fready[b], (p_fready >> b) & 1u)) {
            p_fready ^= 1u << b;
            const int64_t idx = cta + (kf >> 2) * ncta;
            uint8_t* rec = record(sa, idx / N, idx % N);
            // the slice's features: U_q (rows 64..127) as K-blocks 2s, 2s+1 and U_k (rows 0..63) as slice s
            const uint32_t fb = sbase + p1_fbuf(s);
            for (int kb = 0; kb < 2; ++kb) {
              tc::bulk_store(rec + REC_Q + (2 * s + kb) * 8192, fb + kb * 16384 + 8192, 8192);
              tc::bulk_store(rec + REC_UK + s * 16384 + kb * 8192, fb + kb * 16384, 8192);
            }
            tc::bulk_commit();
            tc::bulk_wait_read_but1();  // the copies before this one have read their buffers
            if (pend >= 0) tc::mbar_arrive(&bar_fdone[pend]);
            pend = b;
            ++kf;
            progressed = true;
          }
        }
        if (kt < nrec && kf >= 4 * (kt + 1) && tc::mbar_test_wait(bar_wdone, p_wdone)) {
          p_wdone ^= 1;
          const int64_t idx = cta + kt * ncta;
          uint8_t* rec = record(sa, idx / N, idx % N);
          // T' (rows 0..63 of the U product's A operand), U (two column halves), Aq and the factors
          tc::bulk_store(rec + REC_TP, sbase + P1_TOP, 8192);
          tc::bulk_store(rec + REC_U, sbase + P1_VB, 8192);
          tc::bulk_store(rec + REC_U + 8192, sbase + P1_TOP + 8192, 8192);
          tc::bulk_store(rec + REC_AQ, sbase + P1_AQ, 8192);
          tc::bulk_store(rec + REC_VEC, sbase + P1_VEC, 1024);
          tc::bulk_commit();
          tc::bulk_wait_read();
          hand_back();
          tc::mbar_arrive(bar_stfree);  // the staging tiles take the next chunk
          if (rec_ready) {              // every byte of the record came through this thread's copies
            tc::bulk_wait_all();
            publish_store(rec_ready + idx, 1u);
          }
          ++kt;
          progressed = true;
        }
        ok &= poll_on(poll, progressed, sa.abort);
      }
      tc::bulk_wait_all();
      hand_back();
    }
    __syncwarp();
  } else if (warp < kP1Lift) {
    // ================================================================ lift warps
    // warp (quarter, wh): rows 32 quarter .. +31 of [k; q], columns 64 wh .. +63 of each slice, as two
    // 32-column groups cc (column quarter 2 wh + cc of the slice)
    uint32_t ph_lift = 0, ph_fd = 0, ph_gpf = 0;  // ph_lift, ph_fd: bits per slot / buffer
    auto load_inputs = [&](int64_t idx) {  // the chunk's [k; q] tile (all 256 lift threads)
      const int64_t n = idx % N, c = idx / N;
      for (int t2 = tid; t2 < 512; t2 += 32 * kP1Lift) {
        if (bf_in) prefetch_kq(a, n, int(c), sbase + P1_XIN, t2);
        else load_kq_f32(a, n, int(c), sm + P1_XIN, t2);
      }
      tc::cp_async_commit();
    };
    auto announce_inputs = [&]() {
      tc::cp_async_wait_all();
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_xin);
    };
    // gates of the coming chunk (warp 0) as raw bits: converting at the load would make the warp wait
    // for it there, and they are only used a chunk later
    const bool gate_bf = a.gate_dtype == KDN_DTYPE_BF16;
    uint32_t nb[2] = {0u, 0u}, nd[2] = {0x3f800000u, 0x3f800000u};
    auto load_gates = [&](int64_t idx) {
      const int64_t n_ = idx % N, c_ = idx / N;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t tt = c_ * kC + 2 * lane + e;
        nb[e] = 0u;
        nd[e] = 0x3f800000u;  // 1.0f
        if (tt < a.T) {
          nb[e] = ld_gate_bits(a.beta, gate_bf, n_ * a.T + tt);
          if (decayed) nd[e] = ld_gate_bits(a.decay, gate_bf, n_ * a.T + tt);
        }
      }
    };
    auto gate_f32 = [&](uint32_t bits) { return __uint_as_float(gate_bf ? bits << 16 : bits); };
    if (nrec > 0) {
      if (warp == 0) load_gates(cta);
      load_inputs(cta);
      announce_inputs();
    }
    for (int64_t r = 0; r < nrec; ++r) {
      const int64_t idx = cta + r * ncta;
      const bool has_next = r + 1 < nrec;
      if (warp == 0) {  // the chunk's gates: beta, inclusive scan of log clamp(decay, 1e-5, 1), derived
        // factors.  Buffer r % 3: the algebra warps are on chunk r - 1 at the latest (the sums of
        // squares of chunk r - 1 were written after they had read chunk r - 2's)
        float* gl = gates + 320 * int(r % 3);
        const float lg0 = decayed ? logf(fminf(fmaxf(gate_f32(nd[0]), 1e-5f), 1.0f)) : 0.f;
        const float lg1 = decayed ? logf(fminf(fmaxf(gate_f32(nd[1]), 1e-5f), 1.0f)) : 0.f;
        float sg = lg0 + lg1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, sg, o);
          if (lane >= o) sg += y;
        }
        const float g0 = sg - lg1, g1 = sg;
        const float gend = __shfl_sync(0xffffffffu, sg, 31);
        const float gprev = __shfl_up_sync(0xffffffffu, g1, 1);
        gl[2 * lane] = g0;
        gl[2 * lane + 1] = g1;
        gl[64 + 2 * lane] = gate_f32(nb[0]);
        gl[64 + 2 * lane + 1] = gate_f32(nb[1]);
        gl[128 + 2 * lane] = __expf(g0);
        gl[128 + 2 * lane + 1] = __expf(g1);
        gl[192 + 2 * lane] = lane == 0 ? 1.f : __expf(gprev);
        gl[192 + 2 * lane + 1] = __expf(g0);
        gl[256 + 2 * lane] = __expf(gend - g0);
        gl[256 + 2 * lane + 1] = __expf(gend - g1);
        if (has_next) load_gates(idx + ncta);
      }
      float ss0 = 0.f, ss1 = 0.f;  // sums of squares of column groups cc = 0, 1
#pragma unroll 1
      for (int s = 0; s < kSlices; ++s) {
        ok &= split_wait_bit(&bar_lift[s & 1], ph_lift, s & 1, sa.abort);
        tc::fence_after_sync();
        if (s == kSlices - 1 && has_next) load_inputs(idx + ncta);  // every lift of the chunk is done
        uint8_t* fb = sm + p1_fbuf(s) + wh * 16384;
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          float z[32];
          tc::tmem_ld32(tmem + lane_off + P1_Z + 128 * (s & 1) + 64 * wh + 32 * cc, z);
          tc::tmem_ld_wait();
          if (cc == 1) {  // the slot is read: the issuer may lift slice s + 2 into it
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&bar_zfree[s & 1]);
          }
          // u = cos(tau_inv z + b); the hardware cosine's ~1e-6 absolute error is far
          // below the fp16 spacing of the stored features for the |arguments| <= 32 here
          uint32_t fp[16];
          const float4* phs = reinterpret_cast<const float4*>(ph + 128 * s + 64 * wh + 32 * cc);
          float acc = cc ? ss1 : ss0;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 b4 = phs[j >> 2];
            const float u0 = __cosf(fmaf(z[j], P.tau_inv, b4.x));
            const float u1 = __cosf(fmaf(z[j + 1], P.tau_inv, b4.y));
            const float u2 = __cosf(fmaf(z[j + 2], P.tau_inv, b4.z));
            const float u3 = __cosf(fmaf(z[j + 3], P.tau_inv, b4.w));
            acc = fmaf(u0, u0, fmaf(u1, u1, fmaf(u2, u2, fmaf(u3, u3, acc))));
            fp[j >> 1] = pack_f16(u0, u1);
            fp[(j >> 1) + 1] = pack_f16(u2, u3);
          }
          if (cc) ss1 = acc;
          else ss0 = acc;
          if (cc == 0 && (s >= 2 || r > 0)) {  // the buffer's previous slice: Gram product and copy-out done
            ok &= split_wait_bit(&bar_fdone[s & 1], ph_fd, s & 1, sa.abort);
            tc::fence_after_sync();
          }
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            const uint4 pk = make_uint4(fp[4 * c8], fp[4 * c8 + 1], fp[4 * c8 + 2], fp[4 * c8 + 3]);
            *reinterpret_cast<uint4*>(fb + tc::sw128_offset(trow, 32 * cc + 8 * c8)) = pk;
          }
        }
        tc::fence_proxy_async_smem();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&bar_fready[s & 1]);
      }
      if (has_next) announce_inputs();  // the next chunk's first lifts may start
      // the sums of squares, once the algebra warps have read the previous chunk's
      if (r > 0) {
        ok &= split_wait(bar_gpfree, ph_gpf, sa.abort);
        ph_gpf ^= 1;
      }
      ssp[(2 * wh) * 128 + trow] = ss0;
      ssp[(2 * wh + 1) * 128 + trow] = ss1;
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_ssp);
    }
  } else if (warp < kP1Warps) {
    // ================================================================ algebra warps
    // warp (quarter, wh): row trow of [k; q], columns 32 wh .. +31 of the 64 x 64 chunk matrices
    const int gtid = tid - 32 * kP1Lift;
    uint32_t ph_ssp = 0, ph_gram = 0, ph_mma = 0, ph_st = 0;  // ph_gram: bits per GP buffer
    // v of chunk idx into the staging area Es (free from one chunk's operand of U to the next chunk's
    // inverse): thread gtid copies row gtid / 4, values 16 (gtid % 4) .. +15 (zeros past the end), and
    // later reads back only what it copied itself
    auto prefetch_v = [&](int64_t idx) {
      const int64_t n_ = idx % N, c_ = idx / N;
      const int row = gtid >> 2, cc = gtid & 3;
      const int64_t t = c_ * kC + row;
      const bool in = t < a.T;
      const int es = bf_in ? 2 : 4;
      const char* src = reinterpret_cast<const char*>(a.v) + (in ? ((n_ * a.T + t) * kDV + 16 * cc) * es : 0);
      const uint32_t dst = sbase + P1_ES + row * 64 * es + 16 * cc * es;
      for (int o = 0; o < 16 * es; o += 16) tc::cp_async16(dst + o, src + (in ? o : 0), in ? 16 : 0);
      tc::cp_async_commit();
    };
    if (nrec > 0) prefetch_v(cta);
    for (int64_t r = 0; r < nrec; ++r) {
      const int64_t idx = cta + r * ncta;
      const bool has_next = r + 1 < nrec;
      const float* gl = gates + 320 * int(r % 3);
      const float* bt = gl + 64;
      const float* eg = gl + 128;
      const float* egp = gl + 192;
      const float* wdec = gl + 256;
      // ---------------------------------------- the chunk's sums of squares and [G; P]
      ok &= split_wait(bar_ssp, ph_ssp, sa.abort);
      ph_ssp ^= 1;
      ok &= split_wait_bit(&bar_gram[r & 1], ph_gram, int(r & 1), sa.abort);
      tc::fence_after_sync();
      float gp[32];
      tc::tmem_ld32(tmem + lane_off + P1_GP + 64 * uint32_t(r & 1) + 32 * wh, gp);
      tc::tmem_ld_wait();
      if (gtid < 128)
        sc[gtid] =
            P.amp / (P.amp * sqrtf(ssp[gtid] + ssp[128 + gtid] + ssp[256 + gtid] + ssp[384 + gtid]) + 1e-8f);
      tc::fence_before_sync();
      tc::named_bar_sync(1, kP1AlgThreads);  // scales and gates visible; sums of squares read
      if (lane == 0) tc::mbar_arrive(bar_gpfree);
      // A and Aq in registers (in place of [G; P]) and this thread's v values, then, once the previous
      // chunk's staged tiles have been copied out, everything into shared memory
      const int i = trow & 63;
      {
        const float si = sc[trow];
        if (trow < 64) {  // k row: A_ij = beta_i exp(g_i - g_j) s_i s_j G_ij, j < i
          const float bi = bt[i], gi = gl[i];
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int j = 32 * wh + jj;
            const float dec = decayed ? __expf(gi - gl[j]) : 1.f;
            gp[jj] = (j < i) ? bi * dec * gp[jj] * si * sc[j] : 0.f;
          }
        } else {  // q row: Aq_ij = exp(g_{i-1} - g_j) s_qi s_kj P_ij, j < i (fp16 into the record)
          const float gp_i = i > 0 ? gl[i - 1] : 0.f;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int j = 32 * wh + jj;
            const float dec = decayed ? __expf(gp_i - gl[j]) : 1.f;
            gp[jj] = (j < i) ? dec * gp[jj] * si * sc[j] : 0.f;
          }
        }
      }
      const int row = gtid >> 2, cc = gtid & 3;
      float vreg[16];
      {
        tc::cp_async_wait_all();  // this thread's v values
        if (bf_in) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 w = *reinterpret_cast<const uint4*>(sm + P1_ES + row * 128 + 32 * cc + 16 * h);
            const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(hp[j]);
              vreg[8 * h + 2 * j] = f.x;
              vreg[8 * h + 2 * j + 1] = f.y;
            }
          }
        } else {
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float4 x = *reinterpret_cast<const float4*>(sm + P1_ES + row * 256 + 64 * cc + 16 * m);
            vreg[4 * m] = x.x, vreg[4 * m + 1] = x.y, vreg[4 * m + 2] = x.z, vreg[4 * m + 3] = x.w;
          }
        }
      }
      if (r > 0) {  // the previous chunk's staged tiles (Aq, factors, V / U, A operand) have been copied out
        ok &= split_wait(bar_stfree, ph_st, sa.abort);
        ph_st ^= 1;
      }
      if (trow < 64) {
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
          *reinterpret_cast<float4*>(Am + sx(i, 32 * wh + 4 * j4)) =
              make_float4(gp[4 * j4], gp[4 * j4 + 1], gp[4 * j4 + 2], gp[4 * j4 + 3]);
      } else {
#pragma unroll
        for (int h = 0; h < 4; ++h)
          *reinterpret_cast<uint4*>(sm + P1_AQ + tc::sw128_offset(i, 32 * wh + 8 * h)) =
              make_uint4(pack_f16_sat(gp[8 * h], gp[8 * h + 1]), pack_f16_sat(gp[8 * h + 2], gp[8 * h + 3]),
                         pack_f16_sat(gp[8 * h + 4], gp[8 * h + 5]), pack_f16_sat(gp[8 * h + 6], gp[8 * h + 7]));
      }
      {  // per-token factors of the state pass, the column factors of T', and V (fp16) as the B operand of U
        float* vec = reinterpret_cast<float*>(sm + P1_VEC);
        if (gtid < 64) vec[gtid] = wdec[gtid] * sc[gtid];
        else if (gtid < 128) vec[gtid] = sc[gtid] * egp[gtid - 64];
        else if (gtid == 128) vec[128] = eg[63];
        else if (gtid >= 192) fk[gtid - 192] = bt[gtid - 192] * eg[gtid - 192] * sc[gtid - 192];
#pragma unroll
        for (int h = 0; h < 2; ++h)
          *reinterpret_cast<uint4*>(sm + P1_VB + tc::sw128_offset(row, 16 * cc + 8 * h)) =
              make_uint4(pack_f16_sat(vreg[8 * h], vreg[8 * h + 1]), pack_f16_sat(vreg[8 * h + 2], vreg[8 * h + 3]),
                         pack_f16_sat(vreg[8 * h + 4], vreg[8 * h + 5]),
                         pack_f16_sat(vreg[8 * h + 6], vreg[8 * h + 7]));
      }
      tc::named_bar_sync(1, kP1AlgThreads);
      // T = (I + A)^-1 (fp32, row-major in Es), with 16x16 blocks T_IJ:
      // (a) diagonal blocks by forward substitution, one thread per column (the first 4 algebra warps,
      //     lanes 0..15), everything above the diagonal zero;
      if (warp < kP1Lift + 4 && lane < 16) {
        const int I = warp - kP1Lift, j = lane;
        float tcol[16];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
          float sacc = (rr == j) ? 1.f : 0.f;
#pragma unroll
          for (int kk = 0; kk < rr; ++kk) sacc = fmaf(-Am[sx(16 * I + rr, 16 * I + kk)], tcol[kk], sacc);
          tcol[rr] = (rr >= j) ? sacc : 0.f;
        }
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) Es[(16 * I + rr) * kEsLd + 16 * I + j] = tcol[rr];
      }
      for (int e = gtid; e < 64 * 64; e += kP1AlgThreads) {  // zeros off the diagonal blocks (lower ones are
        const int rr = e >> 6, cc = e & 63;                  // overwritten below)
        if ((rr >> 4) != (cc >> 4)) Es[rr * kEsLd + cc] = 0.f;
      }
      tc::named_bar_sync(1, kP1AlgThreads);
      // (b) off-diagonal blocks level by level (d = I - J = 1, 2, 3)
      t_level<1>(Am, Es, US, gtid);
      t_level<2>(Am, Es, US, gtid);
      t_level<3>(Am, Es, US, gtid);
      // A operand [T diag(beta exp(g) s_k); T diag(beta)] (fp16, K-major, 128 x 64) over A, which is no
      // longer read
      {
        const int rr = gtid >> 1, jh = gtid & 1, i = rr & 63;
        const float* colf = rr < 64 ? fk : bt;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float w[8];
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const float4 t4 = *reinterpret_cast<const float4*>(Es + i * kEsLd + 32 * jh + 8 * h + 4 * m);
            const float4 f4 = *reinterpret_cast<const float4*>(colf + 32 * jh + 8 * h + 4 * m);
            w[4 * m] = t4.x * f4.x;
            w[4 * m + 1] = t4.y * f4.y;
            w[4 * m + 2] = t4.z * f4.z;
            w[4 * m + 3] = t4.w * f4.w;
          }
          *reinterpret_cast<uint4*>(sm + P1_TOP + tc::sw128_offset(rr, 32 * jh + 8 * h)) =
              make_uint4(pack_f16_sat(w[0], w[1]), pack_f16_sat(w[2], w[3]), pack_f16_sat(w[4], w[5]),
                         pack_f16_sat(w[6], w[7]));
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      tc::named_bar_sync(1, kP1AlgThreads);  // also: gates, scales and Es of this chunk no longer read
      if (lane == 0) tc::mbar_arrive(bar_ops);
      if (has_next) prefetch_v(idx + ncta);
      ok &= split_wait(bar_mma, ph_mma, sa.abort);  // U
      ph_mma ^= 1;
      tc::fence_after_sync();
      // ---------------------------------------- U -> staging tiles (value columns 32 wh .. +31: VB for
      // the first half, the A operand's second half for the other), copied out by the publisher
      if (trow >= 64) {
        float u[32];
        tc::tmem_ld32(tmem + lane_off + P1_U + 32 * wh, u);
        tc::tmem_ld_wait();
        float4* dst = reinterpret_cast<float4*>(sm + (wh ? P1_TOP + 8192 : P1_VB) + (trow - 64) * 128);
#pragma unroll
        for (int m = 0; m < 8; ++m) dst[m] = make_float4(u[4 * m], u[4 * m + 1], u[4 * m + 2], u[4 * m + 3]);
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar_wdone);
    }
    tc::cp_async_wait_all();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

// ================================================================ phase 2
// Two CTAs per sequence, each owning 32 of the 64 value columns: the state's
// columns evolve independently (Y, X, E and the update are column-wise), so the
// halves need no communication; both read the same records (the second read
// mostly hits L2).  Per chunk only U_k (64 KiB, two ring items held until the update
// has read them) and T' (8 KiB) are streamed; the outputs are left to phase 3.
// The chain is serial (state -> Y -> X -> E -> state).  Every role has its own warp so
// that no step waits behind another's work: 8 compute warps move tiles between TMEM
// and shared memory, two threads issue the tensor-core products as soon as a tile's
// warps have arrived (the even and the odd feature slices), one keeps the bulk loads
// ahead, and one copies the entering state and E into the record (and publishes the
// progress) off the chain.
constexpr int kHalf = 32;    // value columns per CTA
constexpr int kP2Warps = 8;  // compute warps: 2 per TMEM lane quarter, 16 columns each
constexpr int kP2Producer = kP2Warps;      // bulk loads (lane 0)
constexpr int kP2Issuer = kP2Warps + 1;    // tensor-core products of the even slices, and X (lane 0)
constexpr int kP2Store = kP2Warps + 2;     // record copies and progress words (lane 0)
constexpr int kP2Issuer2 = kP2Warps + 3;   // tensor-core products of the odd slices (lane 0)
constexpr int kP2Thr = 32 * (kP2Warps + 4);
constexpr int kP2Bars = 25;

// TMEM columns (phase 2)
constexpr uint32_t P2_S = 0;    // S^T master, slice s at 32 s (lanes = features), fp32
constexpr uint32_t P2_Y = 128;  // Y = U_k S^T as 2 partial sums: the even slices' at 128, the odd slices' at 160
constexpr uint32_t P2_X = 256;  // X = T' Y, 32 cols

// shared memory (phase 2)
constexpr int kRing = 4;              // 32 KiB stages; items: U_k slices (0,1), (2,3) of each chunk
constexpr uint32_t P2_RING = 0;       // 128 KiB
constexpr uint32_t P2_TP = 131072;    // 2 x 8 KiB T' (fp16, K-major [64 x 64])
constexpr uint32_t P2_FAC = 147456;   // 2 x 9 KiB per-chunk factors: the CTA's half of U (fp32 [64][32]),
constexpr uint32_t P2_FAC_BYTES = 9216;  //   then ew[64], yqs[64], eC
constexpr uint32_t P2_SOP = 165888;   // 32 KiB S^T operand (fp16, MN-major SW64 [512 x 32]), slice s at 8 KiB s
constexpr uint32_t P2_YB = 198656;    // 4 KiB  Y (fp16, MN-major SW64 [64 x 32])
constexpr uint32_t P2_EB = 202752;    // 4 KiB  E'' (fp16, MN-major SW64)
constexpr uint32_t P2_ET = 206848;    // 2 x 4 KiB E of chunk c at 4 KiB (c & 1) (fp16, MN-major SW64), copied
                                      //        to the record
constexpr uint32_t P2_BAR = 215040;
constexpr uint32_t kP2Smem = P2_BAR + 256 + 1024;
static_assert(8 * kP2Bars <= 256, "phase-2 barriers overflow their slot");

// Phase 2 on CTA cta (sequence cta / 2, value columns 32 (cta % 2)..+31; warps 0..11 work,
// others idle; `tmem` = 512 allocated columns).  With rec_ready it waits for each record
// to be published; with out_prog it publishes, per sequence and column half, how many
// chunks have their entering state and E in the records.
__device__ __forceinline__ void state_role(const SplitArgs& sa, uint8_t* sm, uint32_t tmem, int64_t cta,
                                           const uint32_t* rec_ready, uint32_t* out_prog, bool& ok) {
  const TcArgs& a = sa.a;
  const uint32_t sbase = tc::smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + P2_BAR);
  uint64_t* ring_full = bars;        // [4] stage loaded (bytes) and the state operand of its slice pair
                                     //     written (8 compute warps)
  uint64_t* ring_empty = bars + 4;   // [4] stage consumed (MMA commit)
  uint64_t* tp_full = bars + 8;      // [2] T' loaded (bytes) and the Y operand written (8 compute warps)
  uint64_t* tp_empty = bars + 10;    // [2] T' consumed (MMA commit)
  uint64_t* bar_y = bars + 12;       // Y done (MMA commit)
  uint64_t* bar_x = bars + 13;       // X done (MMA commit)
  uint64_t* bar_s = bars + 14;       // [2] state update of slices 2p, 2p+1 done (MMA commit)
  uint64_t* fac_full = bars + 16;    // [2] factors of the chunk loaded (bytes)
  uint64_t* fac_empty = bars + 18;   // [2] factors copied to registers (8 compute warps)
  uint64_t* bar_e = bars + 20;       // E'' operand and E tile written (8 compute warps)
  uint64_t* bar_stfree = bars + 21;  // [2] the record copy has read slice pair p of the state operand (store warp)
  uint64_t* bar_ed = bars + 23;      // [2] E tile of chunk c in buffer c & 1 written (8 compute warps)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t n = cta >> 1;
  const int half = int(cta & 1);
  const int col0 = kHalf * half;  // first value column of this CTA
  const int NC = a.NC;

  if (tid == 0) {
    for (int b = 0; b < kRing; ++b) {
      tc::mbar_init(&ring_full[b], 1 + kP2Warps);
      tc::mbar_init(&ring_empty[b], 2);  // both issuers' update products of the item
    }
    for (int u = 0; u < 2; ++u) {
      tc::mbar_init(&tp_full[u], 1 + kP2Warps);
      tc::mbar_init(&tp_empty[u], 1);
      tc::mbar_init(&bar_s[u], 2);
      tc::mbar_init(&fac_full[u], 1);
      tc::mbar_init(&fac_empty[u], kP2Warps);
    }
    tc::mbar_init(bar_y, 2);
    tc::mbar_init(bar_x, 1);
    tc::mbar_init(bar_e, kP2Warps);
    tc::mbar_init(&bar_stfree[0], 1);
    tc::mbar_init(&bar_stfree[1], 1);
    tc::mbar_init(&bar_ed[0], kP2Warps);
    tc::mbar_init(&bar_ed[1], kP2Warps);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  auto wait_bar = [&](uint64_t* bar, uint32_t& phase) {
    ok &= split_wait(bar, phase, sa.abort);
    phase ^= 1;
    tc::fence_after_sync();
  };

  if (warp == kP2Producer) {
    // ================================================================ bulk loads
    if (lane == 0) {
      uint32_t pe = 0, pt = 0, pfe = 0;  // phase bits per slot
      int64_t g = 0;  // ring items so far
      for (int c = 0; c < NC; ++c) {
        const uint8_t* rec = record(sa, c, n);
        if (rec_ready) {  // the record has been published by the preparation pass
          ok &= wait_flag(rec_ready + int64_t(c) * sa.N + n, 1u, sa.abort);
          tc::fence_proxy_async_global();
        } else if (c + 2 < NC) {  // every record is in place: the one two chunks ahead into L2 meanwhile
          const uint8_t* ahead = record(sa, c + 2, n);
          tc::bulk_prefetch_l2(ahead + REC_UK, REC_AQ - REC_UK);  // U_k, T', U
          tc::bulk_prefetch_l2(ahead + REC_VEC, 1024);
        }
        for (int p = 0; p < 2; ++p, ++g) {  // U_k slices 2p, 2p+1
          const int b = int(g % kRing);
          if (g >= kRing) {
            ok &= split_wait_bit(&ring_empty[b], pe, b, sa.abort);
          }
          tc::mbar_arrive_expect_tx(&ring_full[b], 32768);
          for (int o = 0; o < 32768; o += 16384)
            tc::bulk_load(sbase + P2_RING + b * 32768 + o, rec + REC_UK + p * 32768 + o, 16384, &ring_full[b]);
        }
        const int u = c & 1;
        if (c >= 2) {
          ok &= split_wait_bit(&tp_empty[u], pt, u, sa.abort);
          ok &= split_wait_bit(&fac_empty[u], pfe, u, sa.abort);
        }
        tc::mbar_arrive_expect_tx(&tp_full[u], 8192);
        tc::bulk_load(sbase + P2_TP + u * 8192, rec + REC_TP, 8192, &tp_full[u]);
        tc::mbar_arrive_expect_tx(&fac_full[u], 8192 + 1024);
        tc::bulk_load(sbase + P2_FAC + u * P2_FAC_BYTES, rec + REC_U + half * 8192, 8192, &fac_full[u]);
        tc::bulk_load(sbase + P2_FAC + u * P2_FAC_BYTES + 8192, rec + REC_VEC, 1024, &fac_full[u]);
      }
    }
    __syncwarp();
  } else if (warp == kP2Issuer || warp == kP2Issuer2) {
    // ================================================================ tensor-core products
    // Two issuing threads: one issue costs the issuing thread about 45 cycles, more than the tensor core
    // needs for these small products, so the even and the odd feature slices are issued by different
    // warps (their accumulators are independent: Y as one partial sum per issuer, the state by slice).
    if (lane == 0) {
      const int sl = warp == kP2Issuer2 ? 1 : 0;  // this thread's slice of each slice pair: 2p + sl
      // Y = U_k S^T and X = T' Y have the chunk's 64 tokens as rows: M = 64 products, whose accumulator
      // rows 16 q .. 16 q + 15 sit in TMEM lanes 32 q .. 32 q + 15
      const uint32_t id_k = tc::idesc_f16_f32(64, kHalf, false, true);  // A K-major, B MN-major
      const uint32_t id_s = tc::idesc_f16_f32(128, kHalf, true, true);   // A MN-major (U_k^T)
      // descriptor bases; the products only add constant offsets
      const uint64_t d_ring = tc::smem_desc_sw128(sbase + P2_RING, 16, 1024);     // U_k as A (K-major)
      const uint64_t d_ringT = tc::smem_desc_sw128(sbase + P2_RING, 8192, 1024);  // U_k^T as A (MN-major)
      const uint64_t d_sop = tc::smem_desc_sw64(sbase + P2_SOP, 8192, 512);
      const uint64_t d_tp = tc::smem_desc_sw128(sbase + P2_TP, 16, 1024);
      const uint64_t d_yb = tc::smem_desc_sw64(sbase + P2_YB, 8192, 512);
      const uint64_t d_eb = tc::smem_desc_sw64(sbase + P2_EB, 8192, 512);
      uint32_t pf = 0, pt = 0, pe = 0;  // pf, pt: phase bits per slot
      for (int c = 0; c < NC; ++c) {
#pragma unroll
        for (int p = 0; p < 2; ++p) {  // Y_s = U_k,s S_s^T for slice s = 2p + sl
          const int b = (2 * c + p) & (kRing - 1);  // item 2c + p: its U_k slices and state operand
          ok &= split_wait_bit(&ring_full[b], pf, b, sa.abort);
          tc::fence_after_sync();
          // item block j = 2 sl + hh: slice 2p + sl, its 64-feature half hh
          const uint64_t da = tc::desc_add(d_ring, uint32_t(b) * 32768 + uint32_t(2 * sl) * 8192);
          const uint64_t db = tc::desc_add(d_sop, uint32_t(p) * 16384 + uint32_t(2 * sl) * 4096);
          const uint32_t dy = tmem + P2_Y + 32 * sl;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc::mma_ss(dy, tc::desc_add(da, hh * 8192 + 32 * kk), tc::desc_add(db, hh * 4096 + 1024 * kk), id_k,
                         p > 0 || hh > 0 || kk > 0);
        }
        tc::mma_commit(bar_y);
        if (sl == 0) {  // X = T' Y
          const int u = c & 1;
          ok &= split_wait_bit(&tp_full[u], pt, u, sa.abort);  // T' and the Y operand
          tc::fence_after_sync();
          const uint64_t dt = tc::desc_add(d_tp, uint32_t(u) * 8192);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // K = the 64 tokens
            tc::mma_ss(tmem + P2_X, tc::desc_add(dt, 32 * kk), tc::desc_add(d_yb, 16 * kk * 64), id_k, kk > 0);
          tc::mma_commit(&tp_empty[u]);
          tc::mma_commit(bar_x);
        }
        // S_s^T += U_k,s^T E'' for s = 2p + sl
        wait_bar(bar_e, pe);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const int b = (2 * c + p) & (kRing - 1);
          const uint64_t a0 = tc::desc_add(d_ringT, uint32_t(b) * 32768 + uint32_t(sl) * 16384);
          const uint32_t dcol = tmem + P2_S + kHalf * (2 * p + sl);
#pragma unroll
          for (int k0 = 0; k0 < 64; k0 += 16)
            tc::mma_ss(dcol, tc::desc_add(a0, 128 * k0), tc::desc_add(d_eb, 64 * k0), id_s, true);
          tc::mma_commit(&ring_empty[b]);
          tc::mma_commit(&bar_s[p]);
        }
      }
    }
    __syncwarp();
  } else if (warp == kP2Store) {
    // ================================================================ record copies, progress
    // Each slice pair of the state operand is copied as soon as it is written and handed back once the
    // copy has read it, well before the next chunk rewrites it (the copies read shared memory at only
    // about 10 bytes per cycle); E is double-buffered, so that its copy never holds up the chain either.
    if (lane == 0) {
      uint32_t pf = 0, ped = 0;  // phase bits per ring slot / E buffer
      for (int c = 0; c < NC; ++c) {
        uint8_t* rec = record(sa, c, n);
        for (int p = 0; p < 2; ++p) {  // slice pair p of the state entering the chunk (its ring item loaded)
          const int b = (2 * c + p) & (kRing - 1);
          ok &= split_wait_bit(&ring_full[b], pf, b, sa.abort);
          tc::bulk_store(rec + REC_S0 + half * 32768 + p * 16384, sbase + P2_SOP + p * 16384, 16384);
          tc::bulk_commit();
          if (p == 1) {
            tc::bulk_wait_read_but1();       // pair 0 (and the previous chunk's E) read
            tc::mbar_arrive(&bar_stfree[0]);
          }
        }
        ok &= split_wait_bit(&bar_ed[c & 1], ped, c & 1, sa.abort);
        tc::bulk_store(rec + REC_E + half * 4096, sbase + P2_ET + 4096 * (c & 1), 4096);
        tc::bulk_commit();
        tc::bulk_wait_read_but1();  // pair 1 read
        tc::mbar_arrive(&bar_stfree[1]);
        if (out_prog) {  // chunks 0..c of this half are in the record
          tc::bulk_wait_all();
          publish_store(out_prog + 2 * n + half, uint32_t(c + 1));
        }
      }
      tc::bulk_wait_all();
    }
    __syncwarp();
  } else if (warp < kP2Warps) {
    // ================================================================ compute warps
    const int quarter = warp & 3, ch = warp >> 2;  // TMEM lane quarter, 16-column half of the CTA's 32
    const int trow = quarter * 32 + lane;          // feature row of the state slices (TMEM lane)
    const int yrow = quarter * 16 + lane;          // token row of the M = 64 products (lanes 0..15)
    const bool ylane = lane < 16;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const int cbase = col0 + 16 * ch;  // first value column of this thread
    const bool decayed = a.decay != nullptr;
#pragma unroll
    for (int s = 0; s < kSlices; ++s) {  // state master from the initial state
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = a.S0 ? a.S0[(n * kDV + cbase + j) * kD + 128 * s + trow] : 0.f;
      tc::tmem_st16(tmem + lane_off + P2_S + kHalf * s + 16 * ch, v);
    }
    tc::tmem_st_wait();
    uint32_t py = 0, px = 0, ps[2] = {0, 0}, pff = 0, pst = 0;  // pff: phase bits per slot
    auto store_tile = [&](uint32_t off, int row, const float* v, float w) {  // 16 values of a row, fp16 SW64
#pragma unroll
      for (int m = 0; m < 2; ++m)
        *reinterpret_cast<uint4*>(sm + off + tc::sw64_offset(row, 16 * ch + 8 * m)) =
            make_uint4(pack_f16_sat(w * v[8 * m], w * v[8 * m + 1]), pack_f16_sat(w * v[8 * m + 2], w * v[8 * m + 3]),
                       pack_f16_sat(w * v[8 * m + 4], w * v[8 * m + 5]),
                       pack_f16_sat(w * v[8 * m + 6], w * v[8 * m + 7]));
    };
    auto signal = [&](uint64_t* bar) {  // this warp's tiles -> tensor core / bulk copies
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(bar);
    };
    for (int c = 0; c < NC; ++c) {
      // ---------------------------------------- the chunk's factors (shared memory -> registers)
      float cu[16], cew = 0.f, ceC;
      {
        const int u = c & 1;
        ok &= split_wait_bit(&fac_full[u], pff, u, sa.abort);
        const float* fac = reinterpret_cast<const float*>(sm + P2_FAC + u * P2_FAC_BYTES);
        if (ylane) {
          const float4* u4 = reinterpret_cast<const float4*>(fac + yrow * 32 + 16 * ch);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float4 x = u4[m];
            cu[4 * m] = x.x, cu[4 * m + 1] = x.y, cu[4 * m + 2] = x.z, cu[4 * m + 3] = x.w;
          }
          cew = fac[2048 + yrow];
        }
        ceC = fac[2048 + 128];
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&fac_empty[u]);
      }
      // ---------------------------------------- per slice pair: state operand (fp16), decay
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        if (c > 0) {
          wait_bar(&bar_s[p], ps[p]);  // the previous chunk's update of slices 2p, 2p+1
          // ... and the record copy of the previous chunk's state operand pair p (E of chunk c - 2, in this
          // chunk's E buffer, was read before that)
          ok &= split_wait_bit(&bar_stfree[p], pst, p, sa.abort);
          tc::fence_after_sync();
        }
        float v0[16], v1[16];  // slices 2p and 2p + 1, loaded together (one wait)
        tc::tmem_ld16(tmem + lane_off + P2_S + kHalf * (2 * p) + 16 * ch, v0);
        tc::tmem_ld16(tmem + lane_off + P2_S + kHalf * (2 * p + 1) + 16 * ch, v1);
        tc::tmem_ld_wait();
        store_tile(P2_SOP + (2 * p) * 8192, trow, v0, 1.f);
        store_tile(P2_SOP + (2 * p + 1) * 8192, trow, v1, 1.f);
        if (decayed) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v0[j] *= ceC;
            v1[j] *= ceC;
          }
          tc::tmem_st16(tmem + lane_off + P2_S + kHalf * (2 * p) + 16 * ch, v0);
          tc::tmem_st16(tmem + lane_off + P2_S + kHalf * (2 * p + 1) + 16 * ch, v1);
          tc::tmem_st_wait();
        }
        signal(&ring_full[(2 * c + p) & (kRing - 1)]);
      }
      // ---------------------------------------- Y (fp16) for X = T' Y
      wait_bar(bar_y, py);
      {  // Y = the sum of the two issuers' partial products
        float y[16], y2[16];
        tc::tmem_ld16(tmem + lane_off + P2_Y + 16 * ch, y);
        tc::tmem_ld16(tmem + lane_off + P2_Y + 32 + 16 * ch, y2);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) y[j] += y2[j];
        if (ylane) store_tile(P2_YB, yrow, y, 1.f);
      }
      signal(&tp_full[c & 1]);
      // ---------------------------------------- E = U - X and E'' for the update
      wait_bar(bar_x, px);
      {
        float x[16];
        tc::tmem_ld16(tmem + lane_off + P2_X + 16 * ch, x);
        tc::tmem_ld_wait();
        if (ylane) {
#pragma unroll
          for (int j = 0; j < 16; ++j) x[j] = cu[j] - x[j];
          store_tile(P2_ET + 4096 * (c & 1), yrow, x, 1.f);
          store_tile(P2_EB, yrow, x, cew);
        }
      }
      tc::fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&bar_ed[c & 1]);
        tc::mbar_arrive(bar_e);
      }
    }
    wait_bar(&bar_s[0], ps[0]);
    wait_bar(&bar_s[1], ps[1]);
    // ---------------------------------------- final state
#pragma unroll
    for (int s = 0; s < kSlices; ++s) {
      float v[16];
      tc::tmem_ld16(tmem + lane_off + P2_S + kHalf * s + 16 * ch, v);
      tc::tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) a.S_out[(n * kDV + cbase + j) * kD + 128 * s + trow] = v[j];
    }
  }
}

// ================================================================ phase 3
// Outputs of every chunk at once: y_i = yqs_i (U_q S^T)_i + (Aq E)_i with the state
// entering the chunk and E from the record.  Persistent CTAs; per chunk 4 ring items
// (feature slice s: U_q K-blocks 2s, 2s+1 and both column halves of the state rows)
// and one small item (Aq, E).  The accumulators are double-buffered in TMEM so the
// epilogue of one chunk overlaps the products of the next.
constexpr int kP3Thr = 128;  // warp 0 issues, warp 1 loads, warps 2 and 3 (the q-row lanes) write y
constexpr int kP3Ring = 4;   // 32 KiB ring stages

// shared memory (phase 3)
constexpr uint32_t P3_RING = 8192;     // 4 x 32 KiB; [U_q kb 2s | U_q kb 2s+1 | S half 0 | S half 1], 8 KiB each
constexpr uint32_t P3_SMALL = 172032;  // 2 x 17 KiB: [Aq 8 KiB | E half 0 | E half 1 | yqs]
constexpr uint32_t P3_SMALL_BYTES = 17408;
constexpr uint32_t P3_BAR = 206848;
constexpr uint32_t kP3Smem = P3_BAR + 256 + 1024;

// Phase 3 on CTAs cta = 0..ncta-1 (warps 0..3 work, others idle; `tmem` >= 256 columns).
// With out_prog it waits until both column halves of the state pass are past each chunk.
__device__ __forceinline__ void output_role(const SplitArgs& sa, uint8_t* sm, uint32_t tmem, int64_t cta,
                                            int64_t ncta, const uint32_t* out_prog, bool& ok) {
  const TcArgs& a = sa.a;
  const uint32_t sbase = tc::smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + P3_BAR);
  uint64_t* ring_full = bars;        // [5]
  uint64_t* ring_empty = bars + 5;   // [5]
  uint64_t* small_full = bars + 10;  // [2]
  uint64_t* small_empty = bars + 12; // [2] small item u read by the MMAs and by the epilogue (2 warps)
  uint64_t* acc_full = bars + 14;    // [2] accumulator buffer u complete (MMA commit)
  uint64_t* acc_free = bars + 16;    // [2] accumulator buffer u read (2 epilogue warps)

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t N = sa.N;
  const int64_t total = N * a.NC;
  if (tid == 0) {
    for (int b = 0; b < kP3Ring; ++b) {
      tc::mbar_init(&ring_full[b], 1);
      tc::mbar_init(&ring_empty[b], 1);
    }
    for (int u = 0; u < 2; ++u) {
      tc::mbar_init(&small_full[u], 1);
      tc::mbar_init(&small_empty[u], 2);
      tc::mbar_init(&acc_full[u], 1);
      tc::mbar_init(&acc_free[u], 2);
    }
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (warp == 1) {
    // ================================================================ bulk loads
    if (lane == 0) {
      uint32_t pe = 0, ps = 0;  // phase bits per slot
      int64_t g = 0, j = 0;
      for (int64_t idx = cta; idx < total; idx += ncta, ++j) {
        const uint8_t* rec = record(sa, idx / N, idx % N);
        if (out_prog) {  // both column halves of the state pass are done with this chunk
          const uint32_t need = uint32_t(idx / N) + 1u;
          ok &= wait_flag(out_prog + 2 * (idx % N), need, sa.abort);
          ok &= wait_flag(out_prog + 2 * (idx % N) + 1, need, sa.abort);
          tc::fence_proxy_async_global();
        }
        for (int s = 0; s < kSlices; ++s, ++g) {
          const int b = int(g % kP3Ring);
          if (g >= kP3Ring) {
            ok &= split_wait_bit(&ring_empty[b], pe, b, sa.abort);
          }
          const uint32_t dst = sbase + P3_RING + b * 32768;
          tc::mbar_arrive_expect_tx(&ring_full[b], 32768);
          for (int h = 0; h < 2; ++h) {
            tc::bulk_load(dst + h * 8192, rec + REC_Q + (2 * s + h) * 8192, 8192, &ring_full[b]);
            tc::bulk_load(dst + 16384 + h * 8192, rec + REC_S0 + h * 32768 + s * 8192, 8192, &ring_full[b]);
          }
        }
        const int u = int(j & 1);
        if (j >= 2) {
          ok &= split_wait_bit(&small_empty[u], ps, u, sa.abort);
        }
        const uint32_t dst = sbase + P3_SMALL + u * P3_SMALL_BYTES;
        tc::mbar_arrive_expect_tx(&small_full[u], 16384 + 256);
        tc::bulk_load(dst, rec + REC_AQ, 8192, &small_full[u]);
        tc::bulk_load(dst + 8192, rec + REC_E, 8192, &small_full[u]);
        tc::bulk_load(dst + 16384, rec + REC_VEC + 256, 256, &small_full[u]);  // yqs
      }
    }
    __syncwarp();
  } else if (warp == 0) {
    // ================================================================ MMA issuer
    if (lane == 0) {
      const uint32_t id = tc::idesc_f16_f32(128, 64, false, true);
      uint32_t pf = 0, psf = 0, pfree = 0;  // phase bits per slot
      int64_t g = 0, j = 0;
      for (int64_t idx = cta; idx < total; idx += ncta, ++j) {
        const int u = int(j & 1);
        if (j >= 2) {  // the epilogue of chunk j - 2 has read accumulator buffer u
          ok &= split_wait_bit(&acc_free[u], pfree, u, sa.abort);
        }
        tc::fence_after_sync();
        const uint32_t dq = tmem + 128 * u, de = dq + 64;
        for (int s = 0; s < kSlices; ++s, ++g) {
          const int b = int(g % kP3Ring);
          ok &= split_wait_bit(&ring_full[b], pf, b, sa.abort);
          tc::fence_after_sync();
          const uint32_t st = sbase + P3_RING + b * 32768;
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              // M = 128 from 8 KiB before the U_q block: its rows land in lanes 64..127
              const uint64_t ad = tc::smem_desc_sw128(st + h * 8192 - 8192 + 32 * kk, 16, 1024);
              // N = 64: the two state halves are the two 32-column atoms, 8 KiB apart
              const uint64_t bd = tc::smem_desc_sw64(st + 16384 + (64 * h + 16 * kk) * 64, 8192, 512);
              tc::mma_ss(dq, ad, bd, id, s > 0 || h > 0 || kk > 0);
            }
          tc::mma_commit(&ring_empty[b]);
        }
        ok &= split_wait_bit(&small_full[u], psf, u, sa.abort);
        tc::fence_after_sync();
        const uint32_t sm_small = sbase + P3_SMALL + u * P3_SMALL_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::mma_ss(de, tc::smem_desc_sw128(sm_small - 8192 + 32 * kk, 16, 1024),
                     tc::smem_desc_sw64(sm_small + 8192 + 16 * kk * 64, 4096, 512), id, kk > 0);
        tc::mma_commit(&acc_full[u]);
      }
    }
    __syncwarp();
  } else if (warp < 4) {
    // ================================================================ epilogue (q-row lanes)
    const uint32_t lane_off = uint32_t(warp * 32) << 16;  // warps 2, 3: lanes 64..127
    const int i = (warp - 2) * 32 + lane;                  // token row within the chunk
    uint32_t pa = 0;  // phase bits per slot
    int64_t j = 0;
    for (int64_t idx = cta; idx < total; idx += ncta, ++j) {
      const int64_t c = idx / N, n = idx % N;
      const int u = int(j & 1);
      ok &= split_wait_bit(&acc_full[u], pa, u, sa.abort);
      tc::fence_after_sync();
      const float yqs = reinterpret_cast<const float*>(sm + P3_SMALL + u * P3_SMALL_BYTES + 16384)[i];
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&small_empty[u]);
      const int64_t t = c * kC + i;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float yq[32], ye[32];
        tc::tmem_ld32(tmem + lane_off + 128 * u + 32 * hh, yq);
        tc::tmem_ld32(tmem + lane_off + 128 * u + 64 + 32 * hh, ye);
        tc::tmem_ld_wait();
        if (t < a.T) {
          const int64_t o = (n * a.T + t) * kDV + 32 * hh;
#pragma unroll
          for (int q = 0; q < 32; ++q) yq[q] = fmaf(yqs, yq[q], ye[q]);
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
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_free[u]);
    }
  }
}


// ================================================================ kernels
// One shared-memory size for all launches of this path (the largest role); the TMEM
// address slot sits above every role's layout.
constexpr uint32_t kSplitTslot = 225536;
constexpr uint32_t kSplitSmem = kSplitTslot + 16 + 1024;
static_assert(kP1Smem <= kSplitSmem && kP2Smem <= kSplitSmem && kP3Smem <= kSplitSmem,
              "a role's shared memory exceeds the launch's");
static_assert(kSplitTslot >= P2_BAR + 8 * kP2Bars && kSplitTslot >= P1_FK + 256 && P1_FK >= P1_BAR + kP1Bars && kSplitTslot >= P3_BAR + 8 * 18,
              "TMEM slot overlaps a role's barriers");

__device__ __forceinline__ uint8_t* split_smem() {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t s = tc::smem_u32(smem_raw);
  return smem_raw + ((1024u - (s & 1023u)) & 1023u);
}

__device__ __forceinline__ uint32_t split_tmem_alloc(uint8_t* sm, uint32_t cols) {
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + kSplitTslot);
  if ((threadIdx.x >> 5) == 0) {
    tc::tmem_alloc(tslot, cols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  return *tslot;
}

__device__ __forceinline__ void split_finish(uint32_t tmem, uint32_t cols, bool ok) {
  if (!ok) record_device_error(&g_split_error, kErrSplitWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) tc::tmem_dealloc(tmem, cols);
}

__global__ void __launch_bounds__(kP1Thr, 1) chunk_prep_kernel(SplitArgs sa, ProjParams P) {
  uint8_t* sm = split_smem();
  const uint32_t tmem = split_tmem_alloc(sm, 512);
  bool ok = true;
  prep_role(sa, P, sm, tmem, blockIdx.x, gridDim.x, nullptr, ok);
  split_finish(tmem, 512, ok);
}

__global__ void __launch_bounds__(kP2Thr, 1) state_pass_kernel(SplitArgs sa) {
  uint8_t* sm = split_smem();
  const uint32_t tmem = split_tmem_alloc(sm, 512);
  bool ok = true;
  state_role(sa, sm, tmem, blockIdx.x, nullptr, nullptr, ok);
  split_finish(tmem, 512, ok);
}

__global__ void __launch_bounds__(kP3Thr, 1) output_pass_kernel(SplitArgs sa) {
  uint8_t* sm = split_smem();
  const uint32_t tmem = split_tmem_alloc(sm, 256);
  bool ok = true;
  output_role(sa, sm, tmem, blockIdx.x, gridDim.x, nullptr, ok);
  split_finish(tmem, 256, ok);
}

// All three phases in one cooperative launch (one CTA per SM, all resident): CTAs
// 0..n_state-1 run the state pass while the others prepare the records it waits for and
// then produce the outputs of the chunks it has finished.  Hand-over through the
// per-chunk flags (zeroed before the launch); every wait on them is bounded.
__global__ void __launch_bounds__(kP1Thr, 1) split_persistent_kernel(SplitArgs sa, ProjParams P, uint32_t* rec_ready,
                                                                      uint32_t* out_prog, int n_state) {
  uint8_t* sm = split_smem();
  const uint32_t tmem = split_tmem_alloc(sm, 512);
  bool ok = true;
  if (int(blockIdx.x) < n_state) {
    state_role(sa, sm, tmem, blockIdx.x, rec_ready, out_prog, ok);
  } else {
    const int64_t cta = int64_t(blockIdx.x) - n_state, ncta = int64_t(gridDim.x) - n_state;
    prep_role(sa, P, sm, tmem, cta, ncta, rec_ready, ok);
    output_role(sa, sm, tmem, cta, ncta, out_prog, ok);
  }
  split_finish(tmem, 512, ok);
}

}  // namespace

// records, then the hand-over words of the persistent launch: one per record, two per
// sequence, the abort word
size_t split_prefill_workspace(int64_t N, int64_t T) {
  const int64_t NC = (T + kC - 1) / kC;
  return size_t(N) * size_t(NC) * REC_BYTES + ((size_t(N) * (size_t(NC) + 2) * 4 + 4 + 255) & ~size_t(255));
}

cudaError_t launch_split_prefill(const PrefillProblem& p, const ProjParams& P, void* ws, size_t ws_bytes,
                                 cudaStream_t stream, LaunchMarks& marks) {
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
  sa.abort = nullptr;
  int dev = 0, sms = 0, coop = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess) return e;
  const int64_t total = p.N * int64_t(sa.a.NC);
  for (const void* f : {(const void*)chunk_prep_kernel, (const void*)state_pass_kernel, (const void*)output_pass_kernel,
                        (const void*)split_persistent_kernel})
    if ((e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSplitSmem))) != cudaSuccess)
      return e;
  // one launch for all phases when every CTA fits at once and the state pass leaves at least half
  // of the SMs for the other two (KDN_SPLIT_PERSISTENT=0 forces the three launches); measured at
  // T = 16384: 32 sequences 1.66 ms in one launch vs 1.73 ms in three, 48 sequences 3.9 vs 2.2 ms
  const int n_state = int(2 * p.N);
  int per_sm = 0;
  if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, split_persistent_kernel, kP1Thr, kSplitSmem)) !=
      cudaSuccess)
    return e;
  const char* env = getenv("KDN_SPLIT_PERSISTENT");
  const bool persistent = coop && per_sm >= 1 && 2 * n_state <= sms && !(env && strcmp(env, "0") == 0);
  if (persistent) {
    uint32_t* rec_ready = reinterpret_cast<uint32_t*>(sa.ws + size_t(total) * REC_BYTES);
    uint32_t* out_prog = rec_ready + total;
    sa.abort = out_prog + 2 * p.N;
    if ((e = cudaMemsetAsync(rec_ready, 0, (size_t(total) + 2 * p.N + 1) * 4, stream)) != cudaSuccess) return e;
    marks.begin(stream);
    void* args[] = {&sa, const_cast<ProjParams*>(&P), &rec_ready, &out_prog, const_cast<int*>(&n_state)};
    if ((e = cudaLaunchCooperativeKernel((const void*)split_persistent_kernel, dim3(unsigned(sms)), dim3(kP1Thr), args,
                                         kSplitSmem, stream)) != cudaSuccess)
      return e;
    marks.after(stream);
    return cudaSuccess;
  }
  const unsigned grid1 = unsigned(total < sms ? total : sms);
  marks.begin(stream);
  chunk_prep_kernel<<<grid1, kP1Thr, kSplitSmem, stream>>>(sa, P);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  marks.after(stream);
  state_pass_kernel<<<unsigned(2 * p.N), kP2Thr, kSplitSmem, stream>>>(sa);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  marks.after(stream);
  output_pass_kernel<<<grid1, kP3Thr, kSplitSmem, stream>>>(sa);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  marks.after(stream);
  return cudaSuccess;
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
