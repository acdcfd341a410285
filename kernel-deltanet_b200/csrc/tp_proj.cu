// tp_proj.cu -- row-parallel output projection with the all-reduce fused into the same kernel.
//
// Head tensor parallelism (serving/tensor_parallel_runner.py:51-75,
// experiments/run_kaggle_dual_gpu_cluster.py:99-112): rank r holds the scan outputs of its
// heads, Y_r [M, K] (M tokens, K = local heads x d_v), and its slice of the output projection,
// W_r [N, K]; the layer output is sum_r Y_r W_r^T [M, N] on every rank.  The reference runs
// a local GEMM and then an all-reduce.  Here one persistent kernel does both.  Each CTA walks
// 128 x 256 output tiles; a tile is computed on the tensor cores (bf16 operands, fp32
// accumulation in TMEM) and written out from registers in one of three ways:
//
//   kStore       one rank: plain stores into `out` (fp32 or bf16).
//   kMulticastAdd (one-shot) `multimem.red.add` through the NVSwitch multicast address of a
//                symmetric buffer adds the tile into every rank's copy.  One pass, no waits, but
//                every GPU receives world x the output bytes: the form for small M.
//   kReduceOwned (two-phase, the bandwidth-optimal form; fp32 or bf16 copies) the tile is stored
//                into this rank's copy of the symmetric buffer and announced by a release `multimem.red` on a
//                per-tile counter (every rank's copy of the counter goes up by one).  The tiles
//                this rank owns (t % world == rank) are reduced, while the tile warps go on
//                computing, by four reducer warps per CTA: each waits until every rank has
//                announced tile t, reads the sum of all copies with `multimem.ld_reduce` (the
//                switch adds) and writes it to every copy with `multimem.st`.  Each GPU sends
//                and receives about (1 + 1/world) x the output bytes over NVLink, whatever the
//                world size, and the reduction of early tiles overlaps the products of later ones.
//
// The peer form (kReduceOwnedPeer) runs the same owner scheme over peer pointers: the owner
// reads the tile from every rank's copy, adds in rank order in fp32 and stores the sum into
// every copy (fp32, or bf16 copies: half the bytes), 2 (world - 1) / world x the output bytes
// each way per GPU -- fewer than the multicast form at world 2, and no multicast needed.
//
// The grid is at most one CTA per SM (all resident) and the reducer warps only wait on tiles
// whose tile warps never wait on another rank, so every wait ends; each is bounded all the same
// and a timeout sets the error word.
// Operands are staged by cp.async into 128-byte-swizzled K-major tiles (4 stages of K = 64,
// the next tile's first three loading during this tile's epilogue); one thread issues the
// MMAs; each epilogue thread writes 32-column pieces of its accumulator row from registers.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "kdn_internal.h"
#include "tc_prims.cuh"

namespace kdn {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStagesP = 4;
constexpr int kThrP = 128;              // the tile warps (0-3): loads, MMA issue, epilogue
constexpr int kThrAll = kThrP + 128;    // + the reducer warps (4-7) of the two-phase form
constexpr uint32_t kATile = kBM * kBK * 2;  // 16 KiB
constexpr uint32_t kBTile = kBN * kBK * 2;  // 32 KiB
constexpr uint32_t kStageP = kATile + kBTile;
constexpr uint32_t kStagesBytes = kStageP * kStagesP;
constexpr uint32_t P_BAR = kStagesBytes;  // consumed[4], done
constexpr uint32_t P_TSLOT = P_BAR + 8 * (kStagesP + 1);
constexpr uint32_t P_FLAG = P_TSLOT + 16;
constexpr uint32_t kProjSmem = P_FLAG + 16 + 1024;
static_assert(kProjSmem <= 227 * 1024, "projection tiles exceed shared memory");
constexpr uint32_t kWaitLimitP = 1u << 24;
constexpr uint32_t kFlagPollLimit = 1u << 22;

__device__ int g_proj_error;

enum Mode : int { kStore = 0, kMulticastAdd = 1, kReduceOwned = 2, kReduceOwnedPeer = 3 };
constexpr int kMaxWorld = 8;

struct ProjArgs {
  const __nv_bfloat16* Y;  // [M, K]
  const __nv_bfloat16* W;  // [N, K]
  float* out;              // [M, N] this rank's copy (fp32, or bf16 when out_bf16)
  float* out_mc;           // [M, N] multicast address of the symmetric output (modes 1, 2)
  uint32_t* flags;         // [tiles] this rank's copy of the tile counters (mode 2)
  uint32_t* flags_mc;      // [tiles] their multicast address (mode 2)
  int64_t M;
  int N, K;
  int mode, rank, world;
  int out_bf16;  // modes 0 and 3: the output copies hold bf16 (the sum is still formed in fp32)
  int swiglu;    // store form: tile columns [0, 128) are gate and [128, 256) up; out = silu(gate) * up
  uint32_t target;  // counter value meaning "every rank has announced this tile" in this call
  float* peer_out[kMaxWorld];        // mode 3: every rank's copy of the output (this rank's included)
  uint32_t* peer_flags[kMaxWorld];   // mode 3: every rank's copy of the tile counters
};

__device__ __forceinline__ bool proj_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t n = 0; n < kWaitLimitP; ++n)
    if (tc::mbar_try_wait(bar, parity)) return true;
  return false;
}

// stage k-block kt of the A rows [m0, m0+128) and B rows [n0, n0+256) (zero past M)
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

__device__ __forceinline__ void red_add_v4(float* addr, float4 v) {
  asm volatile("multimem.red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ float4 ld_reduce_v4(const float* addr) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_v4_all(float* addr, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
// bf16 copies: eight values per 16 bytes, summed by the switch in fp32 and rounded once
__device__ __forceinline__ uint4 ld_reduce_bf16x8(const void* addr) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_bf16x8_all(void* addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.bf16x2 [%0], {%1, %2, %3, %4};" ::"l"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void announce(uint32_t* flag_mc) {
  asm volatile("multimem.red.release.sys.global.add.u32 [%0], 1;" ::"l"(flag_mc) : "memory");
}
__device__ __forceinline__ void announce_peer(uint32_t* flag) {
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(flag) : "memory");
}
__device__ __forceinline__ float4 ld_peer_v4(const float* p) {
  float4 v;
  asm volatile("ld.relaxed.sys.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Reduction of the owned tiles (owner forms): CTA b reduces the owned tiles j = b, b + grid, ... (tile
// t = rank + j * world), a quarter tile (32 rows) per unit, units claimed in production order from the
// CTA's shared counter `claim` by every warp that calls this (reducer warps from the start, tile warps
// once they have no tile left to compute).
__device__ __forceinline__ void reduce_owned(const ProjArgs& a, unsigned int* claim, int64_t tiles, int tiles_n, int lane,
                             bool& ok) {
  if (a.mode >= kReduceOwned && a.rank < tiles) {
    const int64_t owned = (tiles - a.rank + a.world - 1) / a.world;
    const int64_t mine = owned > blockIdx.x ? (owned - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const unsigned int units = unsigned(mine * 4);
#pragma unroll 1
    while (true) {
      unsigned int u = 0;
      if (lane == 0) u = atomicAdd(claim, 1u);
      u = __shfl_sync(0xffffffffu, u, 0);
      if (u >= units) break;
      const int64_t t = a.rank + (blockIdx.x + int64_t(u >> 2) * gridDim.x) * a.world;
      int good = 0;
      if (lane == 0)
        for (uint32_t n = 0; n < kFlagPollLimit; ++n)
          if (int32_t(ld_acquire_sys(a.flags + t) - a.target) >= 0) {
            good = 1;
            break;
          }
      good = __shfl_sync(0xffffffffu, good, 0);
      __syncwarp();  // the acquire before every lane's reads
      if (!good) {
        ok = false;
        continue;
      }
      const int n0 = int(t % tiles_n) * kBN;
      const int64_t m0 = (t / tiles_n) * kBM + 32 * (u & 3);
      if (a.mode == kReduceOwned && a.out_bf16) {  // bf16 copies: a lane takes 8 columns (16 B) of a row
        __nv_bfloat16* mc = reinterpret_cast<__nv_bfloat16*>(a.out_mc);
#pragma unroll 1
        for (int r0 = 0; r0 < 32; r0 += 8) {
          uint4 v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t row = m0 + r0 + i;
            if (row < a.M) v[i] = ld_reduce_bf16x8(mc + row * a.N + n0 + 8 * lane);
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t row = m0 + r0 + i;
            if (row < a.M) st_bf16x8_all(mc + row * a.N + n0 + 8 * lane, v[i]);
          }
        }
      } else if (a.mode == kReduceOwned) {
#pragma unroll 1
        for (int r0 = 0; r0 < 32; r0 += 8) {  // 8 rows x 2 vectors per lane in flight
          float4 v[8][2];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t row = m0 + r0 + i;
            if (row < a.M) {
#pragma unroll
              for (int h = 0; h < 2; ++h) v[i][h] = ld_reduce_v4(a.out_mc + row * a.N + n0 + 128 * h + 4 * lane);
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int64_t row = m0 + r0 + i;
            if (row < a.M) {
#pragma unroll
              for (int h = 0; h < 2; ++h) st_v4_all(a.out_mc + row * a.N + n0 + 128 * h + 4 * lane, v[i][h]);
            }
          }
        }
      } else if (a.out_bf16) {  // peer form, bf16 copies: a lane takes 8 columns (16 B) of a row
#pragma unroll 1
        for (int r0 = 0; r0 < 32; r0 += 8) {
          float acc[8][8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
#pragma unroll 1
          for (int p = 0; p < a.world; ++p) {
            const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.peer_out[p]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int64_t row = m0 + r0 + i;
              if (row < a.M) {
                const float4 raw = ld_peer_v4(reinterpret_cast<const float*>(src + row * a.N + n0 + 8 * lane));
                const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = __bfloat1622float2(h2[e]);
                  acc[i][2 * e] += f.x;
                  acc[i][2 * e + 1] += f.y;
                }
              }
            }
          }
          uint4 pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            uint32_t* w32 = reinterpret_cast<uint32_t*>(&pk[i]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 b = __floats2bfloat162_rn(acc[i][2 * e], acc[i][2 * e + 1]);
              w32[e] = *reinterpret_cast<const uint32_t*>(&b);
            }
          }
#pragma unroll 1
          for (int p = 0; p < a.world; ++p) {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.peer_out[p]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int64_t row = m0 + r0 + i;
              if (row < a.M) *reinterpret_cast<uint4*>(dst + row * a.N + n0 + 8 * lane) = pk[i];
            }
          }
        }
      } else {  // peer form: read every copy, add in rank order, write the sum into every copy
#pragma unroll 1
        for (int r0 = 0; r0 < 32; r0 += 8) {  // 8 rows x 2 vectors per lane, one copy at a time
          float4 v[8][2];
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int h = 0; h < 2; ++h) v[i][h] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
          for (int p = 0; p < a.world; ++p) {
            const float* src = a.peer_out[p];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int64_t row = m0 + r0 + i;
              if (row < a.M) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const float4 x = ld_peer_v4(src + row * a.N + n0 + 128 * h + 4 * lane);
                  v[i][h].x += x.x;
                  v[i][h].y += x.y;
                  v[i][h].z += x.z;
                  v[i][h].w += x.w;
                }
              }
            }
          }
#pragma unroll 1
          for (int p = 0; p < a.world; ++p) {
            float* dst = a.peer_out[p];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int64_t row = m0 + r0 + i;
              if (row < a.M) {
#pragma unroll
                for (int h = 0; h < 2; ++h)
                  *reinterpret_cast<float4*>(dst + row * a.N + n0 + 128 * h + 4 * lane) = v[i][h];
              }
            }
          }
        }
      }
    }
  }
}

__device__ __forceinline__ void tile_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kThrP) : "memory"); }

__global__ void __launch_bounds__(kThrAll, 1) tp_proj_kernel(ProjArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = tc::smem_u32(sm);
  uint64_t* consumed = reinterpret_cast<uint64_t*>(sm + P_BAR);
  uint64_t* done = consumed + kStagesP;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + P_TSLOT);
  unsigned int* claim = reinterpret_cast<unsigned int*>(sm + P_FLAG);  // next unit of this CTA's reduction list
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KT = a.K / kBK;
  const int tiles_n = a.N / kBN;
  const int64_t tiles = ((a.M + kBM - 1) / kBM) * tiles_n;
  bool ok = true;

  if (warp == 0) {
    tc::tmem_alloc(tslot, kBN);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kStagesP; ++s) tc::mbar_init(&consumed[s], 1);
    tc::mbar_init(done, 1);
    *claim = 0u;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  const uint32_t idesc = tc::idesc_bf16_f32(kBM, kBN, false, false);
  uint32_t issued = 0;  // bit s: parity of the commits made so far on consumed[s]
  uint32_t pd = 0;      // phase of `done`

  // ---------------------------------------------------------------- tile warps: compute the tiles
  if (warp < kThrP / 32) {
  auto prologue = [&](int64_t t) {  // the first k-blocks of tile t
    for (int s = 0; s < kStagesP - 1; ++s) {
      if (s < KT) load_stage(a, sbase + s * kStageP, (t / tiles_n) * kBM, int(t % tiles_n) * kBN, s, tid);
      tc::cp_async_commit();
    }
  };
  if (blockIdx.x < tiles) prologue(blockIdx.x);
#pragma unroll 1
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int n0 = int(t % tiles_n) * kBN;
    const int64_t m0 = (t / tiles_n) * kBM;
#pragma unroll 1
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % kStagesP;
      asm volatile("cp.async.wait_group %0;" ::"n"(kStagesP - 2) : "memory");  // this thread's part of stage kt
      tc::fence_proxy_async_smem();
      tile_sync();  // every thread's part
      if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t st = sbase + s * kStageP;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          tc::mma_ss(tmem, tc::smem_desc_sw128(st + 32 * kk, 16, 1024),
                     tc::smem_desc_sw128(st + kATile + 32 * kk, 16, 1024), idesc, kt > 0 || kk > 0);
        tc::mma_commit(&consumed[s]);
      }
      issued ^= 1u << s;
      // refill the stage the products of k-block kt - 1 read with k-block kt + 2
      const int nk = kt + kStagesP - 1;
      if (nk < KT) {
        const int ns = nk % kStagesP;
        if (kt >= 1) ok &= proj_wait(&consumed[ns], ((issued >> ns) & 1u) ^ 1u);  // its latest commit
        load_stage(a, sbase + ns * kStageP, m0, n0, nk, tid);
      }
      tc::cp_async_commit();
    }
    if (tid == 0) tc::mma_commit(done);
    ok &= proj_wait(done, pd);
    pd ^= 1u;
    tc::fence_after_sync();
    // every stage is free: the next tile's first k-blocks load while this one is written out
    if (t + gridDim.x < tiles) prologue(t + gridDim.x);

    // accumulator -> registers -> global: thread r writes 32-column pieces of row m0 + r (whole
    // 128-byte lines in fp32, 64 bytes in bf16); the next tile's first k-blocks are already loading
    const int r = 32 * warp + lane;
    const int64_t row = m0 + r;
    if (a.mode == kMulticastAdd) {
      // one-shot: through the last stage buffer (free until the next tile's k-block 3 loads, after
      // this epilogue), 64 columns at a time, so that a warp instruction adds two whole 256-byte row
      // pieces (scattered 16-byte adds starve the multicast path)
      float* Os = reinterpret_cast<float*>(sm + (kStagesP - 1) * kStageP);
      constexpr int kLd = 64 + 4;
      static_assert(kBM * kLd * 4 <= kStageP, "staging exceeds a stage buffer");
#pragma unroll 1
      for (int c0 = 0; c0 < kBN; c0 += 64) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float v[32];
          tc::tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + c0 + 32 * hh, v);
          tc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(Os + r * kLd + 32 * hh + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
        tile_sync();
#pragma unroll 4
        for (int rr = 2 * warp + (lane >> 4); rr < kBM; rr += 2 * (kThrP / 32)) {
          if (m0 + rr < a.M)
            red_add_v4(a.out_mc + (m0 + rr) * a.N + n0 + c0 + 4 * (lane & 15),
                       *reinterpret_cast<const float4*>(Os + rr * kLd + 4 * (lane & 15)));
        }
        tile_sync();
      }
    }
#pragma unroll 1
    for (int c0 = 0; c0 < kBN && a.mode != kMulticastAdd; c0 += 32) {
      float v[32];
      tc::tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + c0, v);
      tc::tmem_ld_wait();
      if (row < a.M) {
        const int64_t off = row * a.N + n0 + c0;
        if (a.out_bf16) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 pk;
            uint32_t* w32 = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __nv_bfloat162 b = __floats2bfloat162_rn(v[j + 2 * e], v[j + 2 * e + 1]);
              w32[e] = *reinterpret_cast<const uint32_t*>(&b);
            }
            *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + off + j) = pk;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(a.out + off + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
      }
    }
    tc::fence_before_sync();
    tile_sync();  // every row of the tile is written; TMEM may take the next tile's products
    if (a.mode >= kReduceOwned && tid == 0) {
      __threadfence_system();
      if (a.mode == kReduceOwned)
        announce(a.flags_mc + t);
      else
        for (int p = 0; p < a.world; ++p) announce_peer(a.peer_flags[p] + t);
    }
  }

  }

  reduce_owned(a, claim, tiles, tiles_n, lane, ok);
  if (a.mode != kStore) __threadfence_system();  // the remote writes before the kernel's completion
  if (!ok) record_device_error(&g_proj_error, kErrProjWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kBN);
}

// ---------------------------------------------------------------------------- TMA-fed form
// Same tiles and outputs (modes kStore, kReduceOwned, kReduceOwnedPeer), warp-specialised: warp 4
// issues the TMA loads of a 4-stage ring (one thread, two tensor-map copies per k-block), warp 5
// issues the MMAs into one of two 256-column TMEM accumulators, warps 0-3 drain the other
// accumulator through swizzled shared-memory blocks and TMA stores (so a tile's epilogue overlaps
// the next tile's products), warps 6-7 reduce owned
// tiles from the start, and every other warp joins the reduction once its role has no work left.
constexpr int kEpiWarps = 4, kProdWarp = 4, kMmaWarp = 5, kRedWarp0 = 6, kRedWarps = 2;
constexpr int kThrT = 32 * (kRedWarp0 + kRedWarps);
constexpr int kStagesT = 4;
constexpr uint32_t T_STG = kStageP * kStagesT;  // two 16 KiB output staging buffers (TMA stores)
constexpr uint32_t kStgBytes = 16384;
constexpr uint32_t T_BAR = T_STG + 2 * kStgBytes;  // full[4], empty[4], acc_full[2], acc_empty[2]
constexpr uint32_t T_TSLOT = T_BAR + 8 * (2 * kStagesT + 4);
constexpr uint32_t T_CLAIM = T_TSLOT + 16;
constexpr uint32_t kProjSmemT = T_CLAIM + 16 + 1024;
static_assert(kProjSmemT <= 227 * 1024, "TMA projection ring exceeds shared memory");

// 2-D tensor-map tile into shared memory; completion counted in bytes on `bar` (no multicast)
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_u32(bar))
      : "memory");
}

// shared -> global 2-D tensor-map store of a staged block (this CTA's bulk group)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

__global__ void __launch_bounds__(kThrT, 1) tp_proj_tma_kernel(ProjArgs a, const __grid_constant__ CUtensorMap mapA,
                                                               const __grid_constant__ CUtensorMap mapB,
                                                               const __grid_constant__ CUtensorMap mapO) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = tc::smem_u32(sm);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + T_BAR);
  uint64_t* empty = full + kStagesT;
  uint64_t* accf = empty + kStagesT;
  uint64_t* acce = accf + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + T_TSLOT);
  unsigned int* claim = reinterpret_cast<unsigned int*>(sm + T_CLAIM);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int KT = a.K / kBK;
  const int tiles_n = (a.N + kBN - 1) / kBN;  // the last tile column may be partial (store form only)
  const int64_t tiles = ((a.M + kBM - 1) / kBM) * tiles_n;
  bool ok = true;

  if (warp == kMmaWarp) {
    tc::tmem_alloc(tslot, 2 * kBN);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < kStagesT; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&accf[b], 1);
      tc::mbar_init(&acce[b], kEpiWarps);
    }
    *claim = 0u;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  if (warp == kProdWarp) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int n0 = int(t % tiles_n) * kBN;
        const int m0 = int((t / tiles_n) * kBM);
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const uint32_t s = it % kStagesT;
          if (it >= kStagesT) ok &= proj_wait(&empty[s], ((it / kStagesT) - 1) & 1u);  // its previous use is read
          tc::mbar_arrive_expect_tx(&full[s], kStageP);
          const uint32_t st = sbase + s * kStageP;
          tma_load_2d(st, &mapA, kt * kBK, m0, &full[s]);
          tma_load_2d(st + kATile, &mapB, kt * kBK, n0, &full[s]);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16_f32(kBM, kBN, false, false);
      uint32_t it = 0, tcount = 0;
      for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++tcount) {
        const uint32_t ab = tcount & 1u;
        if (tcount >= 2) ok &= proj_wait(&acce[ab], ((tcount >> 1) - 1) & 1u);  // drained two tiles ago
        tc::fence_after_sync();
        const uint32_t acc = tmem + kBN * ab;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const uint32_t s = it % kStagesT;
          ok &= proj_wait(&full[s], (it / kStagesT) & 1u);
          tc::fence_after_sync();
          const uint32_t st = sbase + s * kStageP;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc::mma_ss(acc, tc::smem_desc_sw128(st + 32 * kk, 16, 1024),
                       tc::smem_desc_sw128(st + kATile + 32 * kk, 16, 1024), idesc, kt > 0 || kk > 0);
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&accf[ab]);
      }
    }
  } else if (warp < kEpiWarps) {
    // accumulator -> registers -> a 128-byte-swizzled staging block in shared memory (thread r: row r,
    // eight 16-byte chunks) -> one TMA store per block of 32 fp32 / 64 bf16 columns x 128 rows
    uint32_t tcount = 0, sc = 0;
    const int r = 32 * warp + lane;
    const int cols = a.out_bf16 ? 64 : 32;  // columns per staged block (128 bytes a row)
    const int tile_cols = a.swiglu ? kBN / 2 : kBN;  // output columns of a tile
    const int n_lim = a.swiglu ? a.N / 2 : a.N;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++tcount) {
      const uint32_t ab = tcount & 1u;
      ok &= proj_wait(&accf[ab], (tcount >> 1) & 1u);
      tc::fence_after_sync();
      const int n0 = int(t % tiles_n) * tile_cols;  // first output column of the tile
      const int m0 = int((t / tiles_n) * kBM);
#pragma unroll 1
      for (int c0 = 0; c0 < tile_cols && n0 + c0 < n_lim; c0 += cols, ++sc) {  // blocks past N hold no output
        const uint32_t buf = sbase + T_STG + (sc & 1u) * kStgBytes;
        if (tid == 0 && sc >= 2) bulk_wait_read_le1();  // the store that last read this buffer is done
        tc::named_bar_sync(1, 32 * kEpiWarps);
        uint32_t w[32];  // the row's 128 bytes
        if (a.swiglu) {  // bf16 out: silu(gate) * up, gate in accumulator column c, up in c + 128
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float gv[32], uv[32];
            const uint32_t col = tmem + (uint32_t(32 * warp) << 16) + kBN * ab + c0 + 32 * h;
            tc::tmem_ld32(col, gv);
            tc::tmem_ld32(col + kBN / 2, uv);
            tc::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const float p0 = gv[2 * e] / (1.f + expf(-gv[2 * e])) * uv[2 * e];
              const float p1 = gv[2 * e + 1] / (1.f + expf(-gv[2 * e + 1])) * uv[2 * e + 1];
              const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
              w[16 * h + e] = *reinterpret_cast<const uint32_t*>(&b2);
            }
          }
        } else if (a.out_bf16) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v[32];
            tc::tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + kBN * ab + c0 + 32 * h, v);
            tc::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
              w[16 * h + e] = *reinterpret_cast<const uint32_t*>(&b2);
            }
          }
        } else {
          float v[32];
          tc::tmem_ld32(tmem + (uint32_t(32 * warp) << 16) + kBN * ab + c0, v);
          tc::tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(v[e]);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t dst = buf + uint32_t(r) * 128u + ((uint32_t(c) ^ (uint32_t(r) & 7u)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[4 * c]), "r"(w[4 * c + 1]),
                       "r"(w[4 * c + 2]), "r"(w[4 * c + 3])
                       : "memory");
        }
        tc::fence_proxy_async_smem();  // the block is visible to the TMA engine
        tc::named_bar_sync(1, 32 * kEpiWarps);
        if (tid == 0) {
          tma_store_2d(&mapO, buf, n0 + c0, m0);  // rows past M and columns past N are not written
          tc::bulk_commit();
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acce[ab]);  // this warp's TMEM lanes are read
      if (a.mode >= kReduceOwned && tid == 0) {
        tc::bulk_wait_all();  // every block of the tile is in global memory
        tc::fence_proxy_async_global();
        __threadfence_system();
        if (a.mode == kReduceOwned)
          announce(a.flags_mc + t);
        else
          for (int p = 0; p < a.world; ++p) announce_peer(a.peer_flags[p] + t);
      }
    }
    if (tid == 0) tc::bulk_wait_all();  // no store may still read shared memory when the CTA ends
  }
  reduce_owned(a, claim, tiles, tiles_n, lane, ok);  // every warp, once its own role has no work left
  if (a.mode != kStore) __threadfence_system();
  if (!ok) record_device_error(&g_proj_error, kErrProjWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) tc::tmem_dealloc(tmem, 2 * kBN);
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// the [M, N] output (fp32 or bf16, rows ld elements apart), boxes of 128 bytes x 128 rows, 128-byte
// swizzle (the staged blocks)
bool encode_output(CUtensorMap* map, void* base, int64_t M, int N, bool bf16, int64_t ld) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t es = bf16 ? 2 : 4;
  const cuuint64_t dims[2] = {cuuint64_t(N), cuuint64_t(M)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * es};
  const cuuint32_t box[2] = {cuuint32_t(128 / es), cuuint32_t(kBM)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides,
             box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 [rows, K] row-major, boxes of 64 (K) x box_rows, 128-byte swizzle (the MMA operand layout)
bool encode_operand(CUtensorMap* map, const void* base, int64_t rows, int K, int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kBK), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() { return current_sm_count(); }

cudaError_t launch(const ProjArgs& a, cudaStream_t stream) {
  const int64_t tiles = ((a.M + kBM - 1) / kBM) * (a.N / kBN);
  const int64_t grid = tiles < sm_count() ? tiles : sm_count();
  CUtensorMap mapA, mapB, mapO;
  if (a.mode != kMulticastAdd && encode_operand(&mapA, a.Y, a.M, a.K, kBM) &&
      encode_operand(&mapB, a.W, a.N, a.K, kBN) && encode_output(&mapO, a.out, a.M, a.N, a.out_bf16 != 0, a.N)) {
    cudaError_t e =
        cudaFuncSetAttribute(tp_proj_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kProjSmemT));
    if (e != cudaSuccess) return e;
    tp_proj_tma_kernel<<<unsigned(grid), kThrT, kProjSmemT, stream>>>(a, mapA, mapB, mapO);
    return cudaGetLastError();
  }
  // the one-shot multicast form (staged epilogue), or no tensor-map encoder: the cp.async kernel
  cudaError_t e = cudaFuncSetAttribute(tp_proj_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kProjSmem));
  if (e != cudaSuccess) return e;
  tp_proj_kernel<<<unsigned(grid), kThrAll, kProjSmem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

int64_t tp_proj_tiles(int64_t M, int N) { return ((M + kBM - 1) / kBM) * (N / kBN); }

cudaError_t launch_linear(const void* x, const void* w, void* out, bool out_bf16, int64_t M, int N, int K, int64_t ldo,
                          cudaStream_t stream, bool swiglu) {
  ProjArgs a{};
  a.swiglu = swiglu ? 1 : 0;
  a.Y = static_cast<const __nv_bfloat16*>(x);
  a.W = static_cast<const __nv_bfloat16*>(w);
  a.out = static_cast<float*>(out);
  a.out_bf16 = out_bf16 ? 1 : 0;
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = kStore;
  a.world = 1;
  CUtensorMap mapA, mapB, mapO;
  // operand rows past M / N read as zero; output rows and columns past them are clipped by the store
  if (!encode_operand(&mapA, x, M, K, kBM) || !encode_operand(&mapB, w, N, K, kBN) ||
      !encode_output(&mapO, out, M, swiglu ? N / 2 : N, out_bf16, ldo))
    return cudaErrorNotSupported;
  cudaError_t e =
      cudaFuncSetAttribute(tp_proj_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kProjSmemT));
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((M + kBM - 1) / kBM) * ((int64_t(N) + kBN - 1) / kBN);
  const int64_t grid = tiles < sm_count() ? tiles : sm_count();
  tp_proj_tma_kernel<<<unsigned(grid), kThrT, kProjSmemT, stream>>>(a, mapA, mapB, mapO);
  return cudaGetLastError();
}

cudaError_t launch_tp_proj(const void* Y, const void* W, void* out, bool out_bf16, float* out_mc, int64_t M, int N,
                           int K, cudaStream_t stream) {
  ProjArgs a{};
  a.Y = static_cast<const __nv_bfloat16*>(Y);
  a.W = static_cast<const __nv_bfloat16*>(W);
  a.out = static_cast<float*>(out);
  a.out_bf16 = out_bf16 ? 1 : 0;
  a.out_mc = out_mc;
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = out_mc ? kMulticastAdd : kStore;
  a.world = 1;
  return launch(a, stream);
}

cudaError_t launch_tp_proj_reduce(const void* Y, const void* W, void* out, void* out_mc, bool out_bf16,
                                  uint32_t* flags, uint32_t* flags_mc, uint32_t target, int rank, int world, int64_t M,
                                  int N, int K, cudaStream_t stream) {
  ProjArgs a{};
  a.Y = static_cast<const __nv_bfloat16*>(Y);
  a.W = static_cast<const __nv_bfloat16*>(W);
  a.out = static_cast<float*>(out);
  a.out_mc = static_cast<float*>(out_mc);
  a.out_bf16 = out_bf16 ? 1 : 0;
  a.flags = flags;
  a.flags_mc = flags_mc;
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = kReduceOwned;
  a.rank = rank;
  a.world = world;
  a.target = target;
  return launch(a, stream);
}

cudaError_t launch_tp_proj_reduce_peer(const void* Y, const void* W, void* const* outs, bool out_bf16,
                                       uint32_t* const* flags, uint32_t target, int rank, int world, int64_t M, int N,
                                       int K, cudaStream_t stream) {
  if (world < 1 || world > kMaxWorld) return cudaErrorInvalidValue;
  ProjArgs a{};
  a.Y = static_cast<const __nv_bfloat16*>(Y);
  a.W = static_cast<const __nv_bfloat16*>(W);
  a.out = static_cast<float*>(outs[rank]);
  a.out_bf16 = out_bf16 ? 1 : 0;
  a.flags = flags[rank];
  for (int p = 0; p < world; ++p) {
    a.peer_out[p] = static_cast<float*>(outs[p]);
    a.peer_flags[p] = flags[p];
  }
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = kReduceOwnedPeer;
  a.rank = rank;
  a.world = world;
  a.target = target;
  return launch(a, stream);
}

int tp_proj_max_world() { return kMaxWorld; }

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
