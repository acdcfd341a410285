// tp_proj.cu -- row-parallel output projection with the all-reduce fused into its epilogue.
//
// Head tensor parallelism (serving/tensor_parallel_runner.py:51-75,
// experiments/run_kaggle_dual_gpu_cluster.py:99-112): rank r holds the scan outputs of its
// heads, Y_r [M, K] (M tokens, K = local heads x d_v), and its slice of the output projection,
// W_r [N, K]; the layer output is sum_r Y_r W_r^T [M, N] on every rank.  The reference runs
// a local GEMM and then an all-reduce.  Here one kernel does both: each CTA computes a
// 128 x 256 tile on the tensor cores (bf16 operands, fp32 accumulation in TMEM) and its
// epilogue adds the tile into every rank's copy of the output through the NVSwitch multicast
// address of a symmetric buffer (`multimem.red.add`), so the reduction traffic of one tile
// overlaps the products of the next ones.  Without a multicast address (one rank) the tile
// is stored.  Before the launch the output must be zero on every rank, and after it a
// barrier across ranks makes the sums visible; the host wrapper does both.
//
// Operands are staged by cp.async into 128-byte-swizzled K-major tiles (3 stages of K = 64);
// one thread issues the MMAs; the accumulator goes through shared memory so that each warp
// writes whole rows (coalesced 16-byte vectors).
#include "kdn_internal.h"
#include "tc_prims.cuh"

namespace kdn {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStagesP = 3;
constexpr int kThrP = 128;
constexpr uint32_t kATile = kBM * kBK * 2;  // 16 KiB
constexpr uint32_t kBTile = kBN * kBK * 2;  // 32 KiB
constexpr uint32_t kStageP = kATile + kBTile;
constexpr int kOutLd = kBN + 4;  // padded row stride (floats) of the staged accumulator
constexpr uint32_t kOutBytes = kBM * kOutLd * 4;
constexpr uint32_t kMainBytes = kStageP * kStagesP > kOutBytes ? kStageP * kStagesP : kOutBytes;
constexpr uint32_t P_BAR = kMainBytes;  // consumed[3], done
constexpr uint32_t P_TSLOT = P_BAR + 8 * (kStagesP + 1);
constexpr uint32_t kProjSmem = P_TSLOT + 16 + 1024;
constexpr uint32_t kWaitLimitP = 1u << 24;

__device__ int g_proj_error;

struct ProjArgs {
  const __nv_bfloat16* Y;  // [M, K]
  const __nv_bfloat16* W;  // [N, K]
  float* out;              // [M, N] this rank's copy (stores when no multicast address)
  float* out_mc;           // [M, N] multicast address of the symmetric output, or null
  int64_t M;
  int N, K;
};

__device__ __forceinline__ bool proj_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t n = 0; n < kWaitLimitP; ++n)
    if (tc::mbar_try_wait(bar, parity)) return true;
  return false;
}

// stage k-block kt of the CTA's A rows [m0, m0+128) and B rows [n0, n0+256) (zero past M)
__device__ __forceinline__ void load_stage(const ProjArgs& a, uint32_t sbase, int64_t m0, int n0, int kt, int tid) {
  const int k0 = kt * kBK;
#pragma unroll
  for (int i = 0; i < (kBM * 8) / kThrP; ++i) {  // A: 128 rows x 8 chunks of 16 B
    const int e = tid + i * kThrP, r = e >> 3, c = e & 7;
    const int64_t row = m0 + r;
    const bool in = row < a.M;
    const __nv_bfloat16* src = a.Y + (in ? row * a.K + k0 + 8 * c : 0);
    tc::cp_async16(sbase + tc::sw128_offset(r, 8 * c), src, in ? 16 : 0);
  }
#pragma unroll
  for (int i = 0; i < (kBN * 8) / kThrP; ++i) {  // B: 256 rows x 8 chunks
    const int e = tid + i * kThrP, r = e >> 3, c = e & 7;
    tc::cp_async16(sbase + kATile + tc::sw128_offset(r, 8 * c), a.W + int64_t(n0 + r) * a.K + k0 + 8 * c, 16);
  }
}

__device__ __forceinline__ void red_v4(float* addr, float4 v) {
  asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(kThrP, 1) tp_proj_kernel(ProjArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = tc::smem_u32(sm);
  uint64_t* consumed = reinterpret_cast<uint64_t*>(sm + P_BAR);
  uint64_t* done = consumed + kStagesP;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + P_TSLOT);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kBN;
  const int64_t m0 = int64_t(blockIdx.y) * kBM;
  const int KT = a.K / kBK;
  bool ok = true;

  if (warp == 0) {
    tc::tmem_alloc(tslot, kBN);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kStagesP; ++s) tc::mbar_init(&consumed[s], 1);
    tc::mbar_init(done, 1);
    tc::fence_mbar_init();
  }
  for (int s = 0; s < kStagesP - 1; ++s) {
    if (s < KT) load_stage(a, sbase + s * kStageP, m0, n0, s, tid);
    tc::cp_async_commit();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t idesc = tc::idesc_bf16_f32(kBM, kBN, false, false);
  uint32_t pc = 0;  // phase bits of consumed[]

  for (int kt = 0; kt < KT; ++kt) {
    const int s = kt % kStagesP;
    asm volatile("cp.async.wait_group %0;" ::"n"(kStagesP - 2) : "memory");  // this thread's part of stage kt
    tc::fence_proxy_async_smem();
    __syncthreads();  // every thread's part
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t st = sbase + s * kStageP;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk)
        tc::mma_ss(tmem, tc::smem_desc_sw128(st + 32 * kk, 16, 1024), tc::smem_desc_sw128(st + kATile + 32 * kk, 16, 1024),
                   idesc, kt > 0 || kk > 0);
      tc::mma_commit(&consumed[s]);
    }
    // refill the stage the previous products read with k-block kt + 2
    const int nk = kt + kStagesP - 1;
    if (nk < KT) {
      const int ns = nk % kStagesP;
      if (kt >= 1) {  // stage ns was last read by the products of k-block kt - 1
        ok &= proj_wait(&consumed[ns], (pc >> ns) & 1u);
        pc ^= 1u << ns;
      }
      load_stage(a, sbase + ns * kStageP, m0, n0, nk, tid);
    }
    tc::cp_async_commit();
  }
  if (tid == 0) tc::mma_commit(done);
  ok &= proj_wait(done, 0);
  tc::fence_after_sync();

  // accumulator -> shared memory (row r = lane of warp r / 32), then whole rows out
  tc::cp_async_wait_all();  // (every staged load was consumed; nothing is in flight)
  float* Os = reinterpret_cast<float*>(sm);
  const int r = 32 * warp + lane;
#pragma unroll 1
  for (int c0 = 0; c0 < kBN; c0 += 32) {
    float v[32];
    tc::tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + c0, v);
    tc::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; j += 4)
      *reinterpret_cast<float4*>(Os + r * kOutLd + c0 + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
  }
  tc::fence_before_sync();
  __syncthreads();
#pragma unroll 1
  for (int rr = warp; rr < kBM; rr += kThrP / 32) {
    const int64_t row = m0 + rr;
    if (row >= a.M) break;
#pragma unroll
    for (int h = 0; h < kBN / 128; ++h) {
      const int col = 128 * h + 4 * lane;
      const float4 v = *reinterpret_cast<const float4*>(Os + rr * kOutLd + col);
      const int64_t off = row * a.N + n0 + col;
      if (a.out_mc)
        red_v4(a.out_mc + off, v);
      else
        *reinterpret_cast<float4*>(a.out + off) = v;
    }
  }
  if (a.out_mc) __threadfence_system();  // the reductions before the kernel's completion
  if (!ok) record_device_error(&g_proj_error, kErrProjWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kBN);
}

}  // namespace

cudaError_t launch_tp_proj(const void* Y, const void* W, float* out, float* out_mc, int64_t M, int N, int K,
                           cudaStream_t stream) {
  ProjArgs a;
  a.Y = static_cast<const __nv_bfloat16*>(Y);
  a.W = static_cast<const __nv_bfloat16*>(W);
  a.out = out;
  a.out_mc = out_mc;
  a.M = M;
  a.N = N;
  a.K = K;
  cudaError_t e = cudaFuncSetAttribute(tp_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kProjSmem));
  if (e != cudaSuccess) return e;
  dim3 grid(unsigned(N / kBN), unsigned((M + kBM - 1) / kBM));
  tp_proj_kernel<<<grid, kThrP, kProjSmem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t tp_proj_read_error(cudaStream_t stream, int* code) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_proj_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  if (h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_proj_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  }
  *code = h;
  return cudaSuccess;
}

}  // namespace kdn
