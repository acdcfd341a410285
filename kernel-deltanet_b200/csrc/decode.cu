// decode.cu -- single-token decode state update (kdn_decode_step).
//
// Per (token t, head h), with S = states[slot_mapping[t], h] ([dv, D]):
//   y   = S phi(q)                                    (pre-update readout)
//   S  <- lambda (S - beta (S phi(k)) phi(k)^T) + beta v phi(k)^T
//      =  lambda S + beta (v - lambda S phi(k)) phi(k)^T
//   post-update readout (optional): y = lambda S phi(q) + beta (v - lambda S phi(k)) (phi(k) . phi(q))
// (kernels/kernel_deltanet_fused.py:288-300; benchmarks/run_full_batch_decoding.py:43-54)
//
// The step reads and writes every state row once, so it is a streaming kernel: one
// persistent CTA per SM walks units (token, head) -- each as items of 16 state rows (32 KiB
// of fp32 state at D = 512, contiguous in the slot pool) -- through a ring of shared-memory
// stages.  A loader warp keeps bulk loads of the next items (state rows, v; q and k with a
// unit's first item) in flight (it fetches the slots and gates of 32 units at a time, one
// per lane, so that no per-item global load sits on its path); 4 lift warps compute the
// features of each unit once (two 64-wide blocks each) up to two units ahead; 8 row warps
// keep a unit's normalised features in registers, update each item's rows (2 rows per
// warp), write them back with coalesced stores straight from registers and release the
// stage.  (The step is instruction-bound, not DRAM-bound, so lifting once per head rather
// than once per 16 rows is what matters.)  Loads of later items overlap the stores of earlier
// ones continuously, where a CTA that holds its rows in registers for its whole life
// reads, computes and writes in series.
#include "kdn_internal.h"
#include "tc_prims.cuh"

namespace kdn {
namespace {

__device__ int g_decode_error;

constexpr int kDecWarps = 8;                    // row warps (0..7)
constexpr int kLiftWarp0 = kDecWarps;           // lift warps 8..11, two 64-wide feature blocks each
constexpr int kLiftWarps = 4;
constexpr int kDecLoader = kDecWarps + kLiftWarps;  // warp 12
constexpr int kDecThr = 32 * (kDecWarps + kLiftWarps + 1);
constexpr int kFeatBufs = 2;
static_assert(2 * kLiftWarps == kMaxBlocks, "two feature blocks per lift warp");
constexpr int kItemRows = 16;                   // state rows per work item
constexpr int kStages = 6;
constexpr uint32_t kStateBytes = kItemRows * kMaxBlocks * 64 * 4;  // 32 KiB: fp32 rows at D = 512
constexpr uint32_t kStageBytes = kStateBytes + 128;                 // + v of the item's rows (below)
constexpr uint32_t STG_V = kStateBytes;  // v of the item's 16 rows (64 B fp32 / 32 B bf16), bulk-loaded with them
constexpr uint32_t kWaitLimit = 1u << 24;

// shared memory layout
constexpr uint32_t DEC_STAGE = 0;                                   // kStages x 32 KiB
constexpr uint32_t DEC_PHI = kStages * kStageBytes;                 // [2 items][k, q][512] floats
constexpr uint32_t DEC_SS = DEC_PHI + 2 * 2 * kMaxBlocks * 64 * 4;  // [2 items][k, q][8] floats
constexpr uint32_t DEC_META = DEC_SS + 2 * 2 * kMaxBlocks * 4;      // [kStages] int64 slot (or < 0)
constexpr uint32_t DEC_GATE = DEC_META + kStages * 8;               // [kStages] {beta, decay}
constexpr uint32_t DEC_PH = DEC_GATE + kStages * 8;                 // phase b[D]
constexpr uint32_t DEC_QK = DEC_PH + kMaxBlocks * 64 * 4;           // [2 units][q, k][d_k] (fp32 or bf16)
constexpr uint32_t DEC_QKV = DEC_QK + 2 * 2 * kDk * 4;              // [2 units] int: the unit has a valid slot
constexpr uint32_t DEC_BAR = DEC_QKV + 16;                          // full, empty: [kStages] each, then
                                                                    // feat_ready, feat_free, qk_full, qk_free: [2] each
constexpr uint32_t kDecSmem = DEC_BAR + (2 * kStages + 4 * kFeatBufs) * 8;

template <typename ST>
struct StateIO;

template <>
struct StateIO<float> {
  static __device__ __forceinline__ float2 load(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static __device__ __forceinline__ void store(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  }
};

template <>
struct StateIO<__nv_bfloat16> {
  static __device__ __forceinline__ float2 load(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
  }
};

// bounded wait; after one wait has given up, the others of the CTA give up at once
__device__ __forceinline__ bool dec_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  uint32_t n = 0;
  while (!tc::mbar_try_wait(bar, parity)) {
    if ((++n & 1023u) == 0 && (n >= kWaitLimit || *abort)) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// the state rows of group g of unit (token, head) th = t * H + h
template <typename ST>
__device__ __forceinline__ int64_t rows_offset(int64_t slot, int64_t th, const DecodeProblem& p, int g, int D) {
  return ((slot * p.H + th % p.H) * int64_t(p.dv) + int64_t(g) * kItemRows) * D;
}

template <typename ST>
__global__ void __launch_bounds__(kDecThr, 1) decode_kernel(DecodeProblem p, ProjParams P) {
  extern __shared__ __align__(1024) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + DEC_BAR);
  uint64_t* empty = full + kStages;
  uint64_t* feat_ready = empty + kStages;      // [2] features of an item computed (8 lift warps)
  uint64_t* feat_free = feat_ready + kFeatBufs;  // [2] features copied to registers (8 row warps)
  uint64_t* qk_full = feat_free + kFeatBufs;     // [2] a unit's q and k loaded (bytes)
  uint64_t* qk_free = qk_full + kFeatBufs;       // [2] a unit's q and k read (8 lift warps)
  int* qk_valid = reinterpret_cast<int*>(sm + DEC_QKV);
  int64_t* meta = reinterpret_cast<int64_t*>(sm + DEC_META);
  __shared__ int abort_flag;
  volatile int* abort = &abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int D = 64 * P.M;
  const int G = p.dv / kItemRows;
  const uint32_t item_bytes = uint32_t(kItemRows) * uint32_t(D) * uint32_t(sizeof(ST));
  const int64_t units = p.num_tokens * p.H;  // (token, head) pairs
  bool ok = true;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], kDecWarps);  // the row warps are done with the stage
    }
    for (int b = 0; b < kFeatBufs; ++b) {
      tc::mbar_init(&feat_ready[b], kLiftWarps);
      tc::mbar_init(&feat_free[b], kDecWarps);
      tc::mbar_init(&qk_full[b], 1);
      tc::mbar_init(&qk_free[b], kLiftWarps);
    }
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  for (int f = tid; f < D; f += kDecThr) reinterpret_cast<float*>(sm + DEC_PH)[f] = P.phase[f];
  __syncthreads();

  if (warp == kDecLoader) {
    // ================================================================ loads
    uint32_t pe = 0, pq = 0;  // phase bits per stage / per q-k buffer
    int k = 0, n = 0;         // items, units so far
    const uint32_t esz = p.in_dtype == KDN_DTYPE_BF16 ? 2u : 4u;
    for (int64_t u0 = blockIdx.x; u0 < units; u0 += int64_t(gridDim.x) * 32) {
      // slots and gates of the next 32 units of this CTA, one per lane
      const int64_t mine = u0 + int64_t(lane) * gridDim.x;
      int64_t slot = -1;
      float gb = 0.f, gd = 1.f;
      if (mine < units) {
        const int64_t t = mine / p.H;
        slot = p.index_dtype == KDN_INDEX_I64 ? reinterpret_cast<const int64_t*>(p.slot_mapping)[t]
                                              : int64_t(reinterpret_cast<const int32_t*>(p.slot_mapping)[t]);
        if (slot >= p.num_slots && mine % p.H == 0) record_device_error(&g_decode_error, kErrSlotOutOfRange);
        gb = ld_as_f32(p.beta, p.gate_dtype, mine);
        gd = p.decay ? ld_as_f32(p.decay, p.gate_dtype, mine) : 1.f;
      }
      for (int j = 0; j < 32; ++j) {
        const int64_t th = u0 + int64_t(j) * gridDim.x;
        if (th >= units) break;
        const int64_t sj = __shfl_sync(0xffffffffu, slot, j);
        const float bj = __shfl_sync(0xffffffffu, gb, j), dj = __shfl_sync(0xffffffffu, gd, j);
        if (lane != 0) {
          k += G;
          ++n;
          continue;
        }
        const bool valid = sj >= 0 && sj < p.num_slots;
        {  // the unit's q and k, for its features
          const int b = n % kFeatBufs;
          if (n >= kFeatBufs) {
            ok &= dec_wait(&qk_free[b], (pq >> b) & 1u, abort);
            pq ^= 1u << b;
          }
          qk_valid[b] = valid ? 1 : 0;
          if (valid) {
            const uint32_t dst = tc::smem_u32(sm + DEC_QK) + b * 2 * kDk * 4;
            tc::mbar_arrive_expect_tx(&qk_full[b], 2 * kDk * esz);
            tc::bulk_load(dst, static_cast<const uint8_t*>(p.q) + th * kDk * esz, kDk * esz, &qk_full[b]);
            tc::bulk_load(dst + kDk * 4, static_cast<const uint8_t*>(p.k) + th * kDk * esz, kDk * esz, &qk_full[b]);
          } else {
            tc::mbar_arrive(&qk_full[b]);
          }
          ++n;
        }
        for (int g = 0; g < G; ++g, ++k) {
          const int st = k % kStages;
          if (k >= kStages) {
            ok &= dec_wait(&empty[st], (pe >> st) & 1u, abort);
            pe ^= 1u << st;
          }
          meta[st] = valid ? sj : -1;
          if (valid) {
            reinterpret_cast<float2*>(sm + DEC_GATE)[st] = make_float2(bj, dj);
            const uint8_t* src = reinterpret_cast<const uint8_t*>(p.states) +
                                 rows_offset<ST>(sj, th, p, g, D) * int64_t(sizeof(ST));
            const uint32_t stage = tc::smem_u32(sm + DEC_STAGE + st * kStageBytes);
            tc::mbar_arrive_expect_tx(&full[st], item_bytes + kItemRows * esz);
            for (uint32_t o = 0; o < item_bytes; o += 16384) {
              const uint32_t n = item_bytes - o < 16384 ? item_bytes - o : 16384;
              tc::bulk_load(stage + o, src + o, n, &full[st]);
            }
            tc::bulk_load(stage + STG_V,
                          static_cast<const uint8_t*>(p.v) + (th * int64_t(p.dv) + int64_t(g) * kItemRows) * esz,
                          kItemRows * esz, &full[st]);
          } else {
            tc::mbar_arrive(&full[st]);  // nothing to load: the row warps zero the outputs
          }
        }
      }
      __syncwarp();
    }
  } else if (warp >= kLiftWarp0 && warp < kLiftWarp0 + kLiftWarps) {
    // ================================================================ lift warps (blocks w, w + 4)
    const int w = warp - kLiftWarp0;
    const float* ph = reinterpret_cast<const float*>(sm + DEC_PH);
    uint64_t bits[2][3] = {};  // the blocks' sign words, selected with static indices (a run-time
#pragma unroll                // index into the parameter block would copy it to local memory)
    for (int mm = 0; mm < kMaxBlocks; ++mm)
#pragma unroll
      for (int e = 0; e < 2; ++e)
        if (mm == w + kLiftWarps * e)
          bits[e][0] = P.sign_bits[mm][0], bits[e][1] = P.sign_bits[mm][1], bits[e][2] = P.sign_bits[mm][2];
    uint32_t pq = 0, pfree = 0;
    int n = 0;  // units so far
    for (int64_t th = blockIdx.x; th < units; th += gridDim.x, ++n) {
      const int buf = n % kFeatBufs;
      if (n >= kFeatBufs) {  // the row warps have taken this buffer's previous features
        ok &= dec_wait(&feat_free[buf], (pfree >> buf) & 1u, abort);
        pfree ^= 1u << buf;
      }
      ok &= dec_wait(&qk_full[buf], (pq >> buf) & 1u, abort);
      pq ^= 1u << buf;
      float* phi = reinterpret_cast<float*>(sm + DEC_PHI) + buf * 2 * kMaxBlocks * 64;
      float* ss = reinterpret_cast<float*>(sm + DEC_SS) + buf * 2 * kMaxBlocks;
      const uint8_t* qk = sm + DEC_QK + buf * 2 * kDk * 4;
      if (qk_valid[buf]) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int m = w + kLiftWarps * e;
          if (m >= P.M) continue;
#pragma unroll
          for (int which = 0; which < 2; ++which) {
            const float2 xv = ld2_as_f32(qk + (which ? 0 : kDk * 4), p.in_dtype, 2 * lane);
            float u0, u1;
            structured_block(xv.x, xv.y, bits[e], lane, u0, u1);
            const int f = 64 * m + 2 * lane;
            const float c0 = P.amp * cosf(fmaf(u0, P.tau_inv, ph[f]));
            const float c1 = P.amp * cosf(fmaf(u1, P.tau_inv, ph[f + 1]));
            phi[which * kMaxBlocks * 64 + f] = c0;
            phi[which * kMaxBlocks * 64 + f + 1] = c1;
            const float sw = warp_sum(fmaf(c0, c0, c1 * c1));
            if (lane == 0) ss[which * kMaxBlocks + m] = sw;
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&qk_free[buf]);
        tc::mbar_arrive(&feat_ready[buf]);
      }
    }
  } else if (warp < kDecWarps) {
    // ================================================================ row warps (2 rows each)
    uint32_t pf = 0, pready = 0;
    int k = 0, n = 0;
    for (int64_t th = blockIdx.x; th < units; th += gridDim.x, ++n) {
      const int buf = n % kFeatBufs;
      float2 fk[kMaxBlocks], fq[kMaxBlocks];
      float kq = 0.f;
      for (int g = 0; g < G; ++g, ++k) {
        const int st = k % kStages;
        ok &= dec_wait(&full[st], (pf >> st) & 1u, abort);  // the item's state rows and v
        pf ^= 1u << st;
        const int64_t slot = meta[st];
        if (g == 0) {  // the unit's features: normalised into registers, then the buffer is released
          ok &= dec_wait(&feat_ready[buf], (pready >> buf) & 1u, abort);
          pready ^= 1u << buf;
          const float* phi = reinterpret_cast<const float*>(sm + DEC_PHI) + buf * 2 * kMaxBlocks * 64;
          const float* ss = reinterpret_cast<const float*>(sm + DEC_SS) + buf * 2 * kMaxBlocks;
          float nk = 0.f, nq = 0.f;
          for (int m = 0; m < P.M; ++m) {
            nk += ss[m];
            nq += ss[kMaxBlocks + m];
          }
          const float sk = 1.0f / (sqrtf(nk) + 1e-8f), sq = 1.0f / (sqrtf(nq) + 1e-8f);
          kq = 0.f;
#pragma unroll
          for (int m = 0; m < kMaxBlocks; ++m) {
            fk[m] = make_float2(0.f, 0.f);
            fq[m] = make_float2(0.f, 0.f);
            if (m < P.M) {
              const int f = 64 * m + 2 * lane;
              fk[m] = make_float2(phi[f] * sk, phi[f + 1] * sk);
              fq[m] = make_float2(phi[kMaxBlocks * 64 + f] * sq, phi[kMaxBlocks * 64 + f + 1] * sq);
              kq = fmaf(fk[m].x, fq[m].x, fmaf(fk[m].y, fq[m].y, kq));
            }
          }
          if (p.readout == KDN_READOUT_POST) kq = warp_sum(kq);
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&feat_free[buf]);
        }
        const uint8_t* stg = sm + DEC_STAGE + st * kStageBytes;
        const float2 gate = reinterpret_cast<const float2*>(sm + DEC_GATE)[st];
        const float beta = gate.x, lam = gate.y;
        const ST* stage = reinterpret_cast<const ST*>(stg);
        ST* gstate = slot >= 0 ? reinterpret_cast<ST*>(p.states) + rows_offset<ST>(slot, th, p, g, D) : nullptr;
        constexpr int kRowsPerWarp = kItemRows / kDecWarps;
        const int r0 = warp * kRowsPerWarp;  // this warp's first row within the item
        if (slot < 0) {  // padding token (or a slot out of range): zero outputs, state untouched
#pragma unroll
          for (int rr = 0; rr < kRowsPerWarp; ++rr)
            if (lane == 0) st_from_f32(p.out, p.out_dtype, th * p.dv + int64_t(g) * kItemRows + r0 + rr, 0.f);
        } else {
          // both rows in one block: their loads, dot products and warp reductions interleave
          float2 sv[kRowsPerWarp][kMaxBlocks];
          float dk[kRowsPerWarp], dq[kRowsPerWarp];
#pragma unroll
          for (int rr = 0; rr < kRowsPerWarp; ++rr) {
            const ST* row = stage + int64_t(r0 + rr) * D;
            dk[rr] = dq[rr] = 0.f;
#pragma unroll
            for (int m = 0; m < kMaxBlocks; ++m) {
              sv[rr][m] = (m < P.M) ? StateIO<ST>::load(row + 64 * m + 2 * lane) : make_float2(0.f, 0.f);
              dk[rr] = fmaf(sv[rr][m].x, fk[m].x, fmaf(sv[rr][m].y, fk[m].y, dk[rr]));
              dq[rr] = fmaf(sv[rr][m].x, fq[m].x, fmaf(sv[rr][m].y, fq[m].y, dq[rr]));
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int rr = 0; rr < kRowsPerWarp; ++rr) {
              dk[rr] += __shfl_xor_sync(0xffffffffu, dk[rr], o);
              dq[rr] += __shfl_xor_sync(0xffffffffu, dq[rr], o);
            }
#pragma unroll
          for (int rr = 0; rr < kRowsPerWarp; ++rr) {
            const int r = r0 + rr;
            const int64_t orow = th * p.dv + int64_t(g) * kItemRows + r;
            ST* grow = gstate + int64_t(r) * D;
            const float coef = beta * (ld_as_f32(stg + STG_V, p.in_dtype, r) - lam * dk[rr]);
#pragma unroll
            for (int m = 0; m < kMaxBlocks; ++m)  // written back straight to the slot pool
              if (m < P.M)
                StateIO<ST>::store(grow + 64 * m + 2 * lane, fmaf(lam, sv[rr][m].x, coef * fk[m].x),
                                   fmaf(lam, sv[rr][m].y, coef * fk[m].y));
            if (lane == 0) {
              const float yv = p.readout == KDN_READOUT_POST ? fmaf(lam, dq[rr], coef * kq) : dq[rr];
              st_from_f32(p.out, p.out_dtype, orow, yv);
            }
          }
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&empty[st]);  // this warp has read its rows of the stage
      }
    }
  }
  if (!ok) record_device_error(&g_decode_error, kErrDecodeWaitTimeout);
  __syncthreads();
}

}  // namespace

cudaError_t launch_decode(const DecodeProblem& p, const ProjParams& P, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  const int sms = current_sm_count();
  const int64_t units = p.num_tokens * p.H;  // (token, head) pairs, walked by persistent CTAs
  const unsigned grid = unsigned(units < sms ? units : sms);
  cudaError_t e;
  if (p.state_dtype == KDN_DTYPE_BF16) {
    e = cudaFuncSetAttribute(decode_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDecSmem));
    if (e != cudaSuccess) return e;
    decode_kernel<__nv_bfloat16><<<grid, kDecThr, kDecSmem, stream>>>(p, P);
  } else {
    e = cudaFuncSetAttribute(decode_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kDecSmem));
    if (e != cudaSuccess) return e;
    decode_kernel<float><<<grid, kDecThr, kDecSmem, stream>>>(p, P);
  }
  return cudaGetLastError();
}

cudaError_t decode_read_error(cudaStream_t stream, int* code) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_decode_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  if (h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_decode_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  }
  *code = h;
  return cudaSuccess;
}

}  // namespace kdn
