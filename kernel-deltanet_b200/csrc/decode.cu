// decode.cu -- single-token decode state update (kdn_decode_step).
//
// Per (token t, head h), with S = states[slot_mapping[t], h] ([dv, D]):
//   y   = S phi(q)                                    (pre-update readout)
//   S  <- lambda (S - beta (S phi(k)) phi(k)^T) + beta v phi(k)^T
//      =  lambda S + beta (v - lambda S phi(k)) phi(k)^T
//   post-update readout (optional): y = lambda S phi(q) + beta (v - lambda S phi(k)) (phi(k) . phi(q))
// (kernels/kernel_deltanet_fused.py:288-300; benchmarks/run_full_batch_decoding.py:43-54)
//
// Grid (dv/16, H, num_tokens), 128 threads: each CTA owns 16 rows of one head's
// state and streams them once (one read, one write -- the bandwidth floor).
// The lift of q and k is split over the 4 warps by 64-wide block, shared through
// shared memory; each lane then keeps the features of its columns in registers.
#include "kdn_internal.h"

namespace kdn {
namespace {

__device__ int g_decode_error;

constexpr int kWarps = 4;
constexpr int kRowsPerWarp = 4;
constexpr int kRowsPerCta = kWarps * kRowsPerWarp;  // 16

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

template <typename ST>
__global__ void __launch_bounds__(kWarps * 32) decode_kernel(DecodeProblem p, ProjParams P) {
  __shared__ float s_phi[2][kMaxBlocks * 64];  // un-normalised cos features of k (0) and q (1)
  __shared__ float s_ss[2][kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rg = blockIdx.x, h = blockIdx.y;
  const int64_t t = blockIdx.z;
  const int D = 64 * P.M;
  const int64_t th = t * p.H + h;
  const int row0 = rg * kRowsPerCta + warp * kRowsPerWarp;

  int64_t slot = p.index_dtype == KDN_INDEX_I64 ? reinterpret_cast<const int64_t*>(p.slot_mapping)[t]
                                                : int64_t(reinterpret_cast<const int32_t*>(p.slot_mapping)[t]);
  if (slot < 0 || slot >= p.num_slots) {
    if (slot >= p.num_slots && threadIdx.x == 0 && rg == 0) record_device_error(&g_decode_error, kErrSlotOutOfRange);
    if (lane < kRowsPerWarp) st_from_f32(p.out, p.out_dtype, th * p.dv + row0 + lane, 0.f);
    return;
  }
  ST* Srow = reinterpret_cast<ST*>(p.states) + ((slot * p.H + h) * int64_t(p.dv) + row0) * D;

  // 1. issue the state loads first; the lift below overlaps their latency
  float2 s[kRowsPerWarp][kMaxBlocks];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
    for (int m = 0; m < kMaxBlocks; ++m)
      s[r][m] = (m < P.M) ? StateIO<ST>::load(Srow + int64_t(r) * D + 64 * m + 2 * lane) : make_float2(0.f, 0.f);

  // 2. lift: warp w handles blocks m = w, w+4 of both k and q
  {
    float ss[2] = {0.f, 0.f};
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      const float2 xv = ld2_as_f32(which ? p.q : p.k, p.in_dtype, th * kDk + 2 * lane);
#pragma unroll
      for (int mm = 0; mm < kMaxBlocks / kWarps; ++mm) {
        const int m = warp + kWarps * mm;
        if (m < P.M) {
          float u0, u1;
          structured_block(xv.x, xv.y, P.sign_bits[m], lane, u0, u1);
          const int f = 64 * m + 2 * lane;
          const float c0 = P.amp * cosf(fmaf(u0, P.tau_inv, P.phase[f]));
          const float c1 = P.amp * cosf(fmaf(u1, P.tau_inv, P.phase[f + 1]));
          s_phi[which][f] = c0;
          s_phi[which][f + 1] = c1;
          ss[which] = fmaf(c0, c0, fmaf(c1, c1, ss[which]));
        }
      }
    }
    ss[0] = warp_sum(ss[0]);
    ss[1] = warp_sum(ss[1]);
    if (lane == 0) {
      s_ss[0][warp] = ss[0];
      s_ss[1][warp] = ss[1];
    }
  }
  __syncthreads();
  float nk = 0.f, nq = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    nk += s_ss[0][w];
    nq += s_ss[1][w];
  }
  const float sk = 1.0f / (sqrtf(nk) + 1e-8f), sq = 1.0f / (sqrtf(nq) + 1e-8f);
  float2 fk[kMaxBlocks], fq[kMaxBlocks];
  float kq = 0.f;
#pragma unroll
  for (int m = 0; m < kMaxBlocks; ++m) {
    fk[m] = make_float2(0.f, 0.f);
    fq[m] = make_float2(0.f, 0.f);
    if (m < P.M) {
      const int f = 64 * m + 2 * lane;
      fk[m] = make_float2(s_phi[0][f] * sk, s_phi[0][f + 1] * sk);
      fq[m] = make_float2(s_phi[1][f] * sq, s_phi[1][f + 1] * sq);
      kq = fmaf(fk[m].x, fq[m].x, fmaf(fk[m].y, fq[m].y, kq));
    }
  }
  if (p.readout == KDN_READOUT_POST) kq = warp_sum(kq);

  const float beta = ld_as_f32(p.beta, p.gate_dtype, th);
  const float lam = p.decay ? ld_as_f32(p.decay, p.gate_dtype, th) : 1.0f;

  // 3. per row: the two dot products, the rank-1 update, the write-back
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    float dk = 0.f, dq = 0.f;
#pragma unroll
    for (int m = 0; m < kMaxBlocks; ++m) {
      dk = fmaf(s[r][m].x, fk[m].x, fmaf(s[r][m].y, fk[m].y, dk));
      dq = fmaf(s[r][m].x, fq[m].x, fmaf(s[r][m].y, fq[m].y, dq));
    }
    dk = warp_sum(dk);
    dq = warp_sum(dq);
    const float vr = ld_as_f32(p.v, p.in_dtype, th * p.dv + row0 + r);
    const float coef = beta * (vr - lam * dk);
#pragma unroll
    for (int m = 0; m < kMaxBlocks; ++m)
      if (m < P.M)
        StateIO<ST>::store(Srow + int64_t(r) * D + 64 * m + 2 * lane, fmaf(lam, s[r][m].x, coef * fk[m].x),
                           fmaf(lam, s[r][m].y, coef * fk[m].y));
    if (lane == r) {
      const float yv = p.readout == KDN_READOUT_POST ? fmaf(lam, dq, coef * kq) : dq;
      st_from_f32(p.out, p.out_dtype, th * p.dv + row0 + r, yv);
    }
  }
}

}  // namespace

cudaError_t launch_decode(const DecodeProblem& p, const ProjParams& P, cudaStream_t stream) {
  if (p.num_tokens == 0) return cudaSuccess;
  dim3 grid(p.dv / kRowsPerCta, p.H, unsigned(p.num_tokens));
  if (p.state_dtype == KDN_DTYPE_BF16)
    decode_kernel<__nv_bfloat16><<<grid, kWarps * 32, 0, stream>>>(p, P);
  else
    decode_kernel<float><<<grid, kWarps * 32, 0, stream>>>(p, P);
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
