// anchor_attn.cu -- the softmax anchors of the hybrid LM: rotary q/k with the KV-cache fill, and a
// varlen causal attention on the tensor cores.
//
// The anchors are the full-attention layers the reference keeps at fixed depths of its hybrid
// models (models/upcycling_llama_bridge.py:240-249): multi-head causal softmax attention with
// rotate-half rotary positions (:138-140), d_head 64.  The reference runs them through torch SDPA.
//
// anchor_qkv_kernel: one warp per token.  The fused projection row [3, H, 64] (q | k | v) is split;
//   q and k are rotated at the token's position (lanes 0-15 take q, 16-31 take k; lane f covers the
//   frequency pair 2f, 2f + 1 and the element pairs at 2f and 32 + 2f), k and v are written into the
//   per-sequence KV cache [rows, H, L, 64] and q into [H, n, 64] (head-major, the attention's layout)
//   or [n, H, 64] (the one-token decode attention's layout).  The rotation is formed as the torch
//   restatement forms it: inv_freq = theta^(-2i/64) and angle = pos * inv_freq in fp32, then
//   x cos - x' sin with each product and the sum rounded to fp32.
//
// anchor_attn_kernel: one CTA per (sequence, head, block of 256 queries); grid.x = sequences x H,
//   grid.y = query blocks of the longest sequence, launched heaviest block first (a CTA whose block
//   starts past its sequence returns at once).  The block is two 128-row query tiles that share
//   every key/value tile; each has its own softmax warpgroup, so while one warpgroup turns S into P
//   the tensor core works on the other tile.  Per key tile j (128 keys):
//     producer warp   TMA: K_j, V_j into a 3-stage ring (Q tiles once);
//     MMA warp        S_q = Q_q K_j^T (128 x 128, TMEM), later O_q += P_q V_j (128 x 64, TMEM);
//     softmax warps   thread r owns query row r: row max over S (first pass over TMEM), rescale
//                     factor alpha = 2^(m_old - m_new); once P(j-1) V(j-1) has landed, the row of O
//                     is scaled by alpha in TMEM (skipped when no row of the warp changed its max);
//                     P = 2^(S log2e/8 - m_new) as bf16 into a 128-byte-swizzled K-major shared
//                     tile (second pass) and the row sum in fp32.
//   The causal mask applies on the diagonal tile only (key c > row r); key positions past the
//   sequence end are never reached by a valid query.  O / l goes to out [n, H, 64] (bf16).
//   TMEM: S tiles at columns 128 q, O tiles at 256 + 64 q (512 columns, one CTA per SM).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>

#include "kdn_internal.h"
#include "tc_prims.cuh"

namespace kdn {

__device__ int g_attn_error;

namespace {

constexpr int kD = 64;
constexpr int kBQ = 128, kQT = 2, kBKV = 128, kStages = 3;
constexpr int kSoftWarps = 4 * kQT, kProdWarp = kSoftWarps, kMmaWarp = kSoftWarps + 1;
constexpr int kThreads = 32 * (kSoftWarps + 2);
constexpr uint32_t kTile = kBQ * kD * 2;  // 16 KiB: 128 rows x 64 bf16 (128-byte rows)
constexpr uint32_t A_Q = 0;
constexpr uint32_t A_K = A_Q + kQT * kTile;
constexpr uint32_t A_V = A_K + kStages * kTile;
constexpr uint32_t A_P = A_V + kStages * kTile;  // per query tile: keys [0, 64) then [64, 128)
constexpr uint32_t A_BAR = A_P + kQT * 2 * kTile;
// q_full, k_full[S], v_full[S], kv_empty[S], s_full[QT], p_full[QT], o_full[QT], mma_done
constexpr int kBars = 2 + 3 * kStages + 3 * kQT;
constexpr uint32_t A_TSLOT = A_BAR + 8 * kBars;
constexpr uint32_t kSmem = A_TSLOT + 16 + 1024;
static_assert(kSmem <= 227 * 1024, "attention tiles exceed shared memory");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kWaitLimit = 1u << 24;
constexpr float kScaleLog2 = 0.18033688011112042f;  // log2(e) / sqrt(64)

struct AttnArgs {
  const int64_t* cu;    // [B + 1] token offsets of the sequences
  const int64_t* rows;  // [B] KV-cache row of each sequence (null: row b)
  __nv_bfloat16* out;   // [n, H, 64]
  int64_t n;            // total tokens
  int64_t cache_batch;  // KV-cache rows
  int64_t L;            // KV-cache positions per row
  int H;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(tc::smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// row max of the 128 scores of this thread's row (masked: key c > r excluded)
template <bool kMasked>
__device__ __forceinline__ float row_max(uint32_t t_s, int r) {
  float mx = -INFINITY;
#pragma unroll
  for (int c0 = 0; c0 < kBKV; c0 += 32) {
    float v[32];
    tc::tmem_ld32(t_s + c0, v);
    tc::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (!kMasked || c0 + i <= r) mx = fmaxf(mx, v[i]);
  }
  return mx;
}

// P = 2^(S log2e/8 - m) as bf16 into the K-major swizzled tile at p_base; returns the fp32 row sum
template <bool kMasked>
__device__ __forceinline__ float write_p(uint32_t t_s, uint32_t p_base, int r, float m) {
  float sum = 0.f;
#pragma unroll
  for (int c0 = 0; c0 < kBKV; c0 += 16) {  // 16 keys (two 16-byte chunks of P) at a time
    float v[16];
    tc::tmem_ld16(t_s + c0, v);
    tc::tmem_ld_wait();
    uint32_t pk[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float p0 = ex2(fmaf(v[2 * e], kScaleLog2, -m));
      float p1 = ex2(fmaf(v[2 * e + 1], kScaleLog2, -m));
      if (kMasked) {
        if (c0 + 2 * e > r) p0 = 0.f;
        if (c0 + 2 * e + 1 > r) p1 = 0.f;
      }
      sum += p0 + p1;
      pk[e] = pack_bf16(p0, p1);
    }
    const uint32_t region = p_base + uint32_t(c0 / 64) * kTile + uint32_t(r) * 128u;
    const uint32_t ch0 = uint32_t(c0 % 64) / 8;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const uint32_t dst = region + (((ch0 + t) ^ (uint32_t(r) & 7u)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(pk[4 * t]), "r"(pk[4 * t + 1]),
                   "r"(pk[4 * t + 2]), "r"(pk[4 * t + 3])
                   : "memory");
    }
  }
  return sum;
}

// O *= alpha for this thread's row of the PV accumulator (64 TMEM columns; warp-collective)
__device__ __forceinline__ void rescale_o(uint32_t t_o, float alpha) {
#pragma unroll
  for (int c0 = 0; c0 < kD; c0 += 16) {
    float t[16];
    tc::tmem_ld16(t_o + c0, t);
    tc::tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 16; ++i) t[i] *= alpha;
    tc::tmem_st16(t_o + c0, t);
  }
  tc::tmem_st_wait();
}

// S_q = Q_q K_j^T (128 x 128, K = 64), then arrive on `done`
__device__ __forceinline__ void issue_s(uint32_t sbase, uint32_t tmem, uint32_t id, int q, int j, uint64_t* done) {
  const uint32_t qa = sbase + A_Q + q * kTile, ka = sbase + A_K + (j % kStages) * kTile;
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk)
    tc::mma_ss(tmem + 128 * q, tc::smem_desc_sw128(qa + 32 * kk, 16, 1024), tc::smem_desc_sw128(ka + 32 * kk, 16, 1024),
               id, kk > 0);
  tc::mma_commit(done);
}

// O_q (+)= P_q V_j (128 x 64, K = 128 keys; V is the MN-major B operand), then arrive on `done`
__device__ __forceinline__ void issue_o(uint32_t sbase, uint32_t tmem, uint32_t id, int q, int j, uint64_t* done) {
  const uint32_t pa = sbase + A_P + q * 2 * kTile, va = sbase + A_V + (j % kStages) * kTile;
#pragma unroll
  for (int kk = 0; kk < kBKV / 16; ++kk)
    tc::mma_ss(tmem + 256 + 64 * q, tc::smem_desc_sw128(pa + (kk / 4) * kTile + 32 * (kk % 4), 16, 1024),
               tc::smem_desc_sw128(va + 128 * 16 * kk, 8192, 1024), id, j > 0 || kk > 0);
  tc::mma_commit(done);
}

__global__ void __launch_bounds__(kThreads, 1) anchor_attn_kernel(AttnArgs a, const __grid_constant__ CUtensorMap mq,
                                                                  const __grid_constant__ CUtensorMap mk,
                                                                  const __grid_constant__ CUtensorMap mv) {
  const int b = int(blockIdx.x / a.H), h = int(blockIdx.x % a.H);
  const int64_t c0 = a.cu[b];
  const int64_t T = a.cu[b + 1] - c0;
  const int qb = int(gridDim.y - 1 - blockIdx.y);
  const int64_t q0 = int64_t(qb) * (kQT * kBQ);
  const int64_t row = a.rows ? a.rows[b] : b;
  if (threadIdx.x == 0 && qb == 0 && (T > int64_t(gridDim.y) * kQT * kBQ || T > a.L || c0 < 0 || T < 0 ||
                                      c0 + T > a.n || row < 0 || row >= a.cache_batch))
    record_device_error(&g_attn_error, kErrSlotOutOfRange);  // a bound the host could not check
  if (q0 >= T || row < 0 || row >= a.cache_batch || c0 < 0 || c0 + T > a.n || T > a.L) return;  // whole CTA
  const bool has1 = q0 + kBQ < T;
  const int nj0 = 2 * qb + 1, nj1 = has1 ? 2 * qb + 2 : 0;
  const int nkv = has1 ? nj1 : nj0;
  const int kv_y = int((row * a.H + h) * a.L);
  const int q_y = int(int64_t(h) * a.n + c0 + q0);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = tc::smem_u32(sm);
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sm + A_BAR);
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + kStages;
  uint64_t* kv_empty = v_full + kStages;
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* p_full = s_full + kQT;
  uint64_t* o_full = p_full + kQT;
  uint64_t* mma_done = o_full + kQT;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + A_TSLOT);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  bool ok = true;

  if (warp == kMmaWarp) {
    tc::tmem_alloc(tslot, kTmemCols);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&k_full[s], 1);
      tc::mbar_init(&v_full[s], 1);
      tc::mbar_init(&kv_empty[s], 1);
    }
    for (int q = 0; q < kQT; ++q) {
      tc::mbar_init(&s_full[q], 1);
      tc::mbar_init(&p_full[q], 128);
      tc::mbar_init(&o_full[q], 1);
    }
    tc::mbar_init(mma_done, 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;

  if (warp == kProdWarp) {
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(q_full, kTile * (has1 ? 2u : 1u));
      tma_load_2d(sbase + A_Q, &mq, 0, q_y, q_full);
      if (has1) tma_load_2d(sbase + A_Q + kTile, &mq, 0, q_y + kBQ, q_full);
      for (int j = 0; j < nkv && ok; ++j) {  // a wait that gave up ends the role (the error word is set)
        const int s = j % kStages;
        if (j >= kStages) ok &= tc::mbar_wait_bounded(&kv_empty[s], ((j / kStages) - 1) & 1, kWaitLimit);
        tc::mbar_arrive_expect_tx(&k_full[s], kTile);
        tma_load_2d(sbase + A_K + s * kTile, &mk, 0, kv_y + kBKV * j, &k_full[s]);
        tc::mbar_arrive_expect_tx(&v_full[s], kTile);
        tma_load_2d(sbase + A_V + s * kTile, &mv, 0, kv_y + kBKV * j, &v_full[s]);
      }
      // every commit on the ring's empty barriers has arrived before the CTA may exit
      for (int j = nkv > kStages ? nkv - kStages : 0; j < nkv && ok; ++j)
        ok &= tc::mbar_wait_bounded(&kv_empty[j % kStages], (j / kStages) & 1, kWaitLimit);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_bf16_f32(kBQ, kBKV, false, false);
      const uint32_t id_o = tc::idesc_bf16_f32(kBQ, kD, false, true);  // V is the MN-major B operand
      ok &= tc::mbar_wait_bounded(q_full, 0, kWaitLimit);
      ok &= tc::mbar_wait_bounded(&k_full[0], 0, kWaitLimit);
      tc::fence_after_sync();
      issue_s(sbase, tmem, id_s, 0, 0, &s_full[0]);
      if (has1) issue_s(sbase, tmem, id_s, 1, 0, &s_full[1]);
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j % kStages;
        const int s1 = (j + 1) % kStages;
        const uint32_t ph1 = ((j + 1) / kStages) & 1;
        ok &= tc::mbar_wait_bounded(&v_full[s], (j / kStages) & 1, kWaitLimit);
        if (j < nj0) {
          ok &= tc::mbar_wait_bounded(&p_full[0], j & 1, kWaitLimit);
          tc::fence_after_sync();
          issue_o(sbase, tmem, id_o, 0, j, &o_full[0]);
          if (j + 1 < nj0) {
            ok &= tc::mbar_wait_bounded(&k_full[s1], ph1, kWaitLimit);
            tc::fence_after_sync();
            issue_s(sbase, tmem, id_s, 0, j + 1, &s_full[0]);
          }
        }
        if (has1) {
          ok &= tc::mbar_wait_bounded(&p_full[1], j & 1, kWaitLimit);
          tc::fence_after_sync();
          issue_o(sbase, tmem, id_o, 1, j, &o_full[1]);
        }
        tc::mma_commit(&kv_empty[s]);  // K_j and V_j are read once these products complete
        if (has1 && j + 1 < nj1) {
          ok &= tc::mbar_wait_bounded(&k_full[s1], ph1, kWaitLimit);
          tc::fence_after_sync();
          issue_s(sbase, tmem, id_s, 1, j + 1, &s_full[1]);
        }
      }
      tc::mma_commit(mma_done);  // every product this thread issued is complete before TMEM is freed
      ok &= tc::mbar_wait_bounded(mma_done, 0, kWaitLimit);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int q = warp >> 2, r = 32 * (warp & 3) + lane;
    const int nj = q == 0 ? nj0 : nj1;
    const int jd = 2 * qb + q;  // the diagonal key tile of this query tile
    const uint32_t lane_off = uint32_t(32 * (warp & 3)) << 16;
    const uint32_t t_s = tmem + lane_off + 128 * q, t_o = tmem + lane_off + 256 + 64 * q;
    const uint32_t p_base = sbase + A_P + q * 2 * kTile;
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < nj && ok; ++j) {
      ok = __all_sync(0xffffffffu, ok && tc::mbar_wait_bounded(&s_full[q], j & 1, kWaitLimit));  // warp-uniform
      if (!ok) break;
      tc::fence_after_sync();
      const bool diag = j == jd;
      const float mx = diag ? row_max<true>(t_s, r) : row_max<false>(t_s, r);
      const float m_new = fmaxf(m, mx * kScaleLog2);
      const float alpha = ex2(m - m_new);
      if (j > 0) {  // P(j-1) V(j-1) has landed in O: P's tile is free, and O is rescaled to the new max
        ok = __all_sync(0xffffffffu, tc::mbar_wait_bounded(&o_full[q], (j - 1) & 1, kWaitLimit));
        if (!ok) break;
        tc::fence_after_sync();
        if (__any_sync(0xffffffffu, alpha != 1.f)) rescale_o(t_o, alpha);
      }
      const float sum = diag ? write_p<true>(t_s, p_base, r, m_new) : write_p<false>(t_s, p_base, r, m_new);
      l = l * alpha + sum;
      m = m_new;
      tc::fence_proxy_async_smem();  // P is visible to the tensor core
      tc::fence_before_sync();
      tc::mbar_arrive(&p_full[q]);
    }
    if (nj > 0 && ok) ok = __all_sync(0xffffffffu, tc::mbar_wait_bounded(&o_full[q], (nj - 1) & 1, kWaitLimit));
    if (nj > 0 && ok) {
      tc::fence_after_sync();
      const int64_t qpos = q0 + kBQ * q + r;
      const float inv = 1.f / l;
      uint4* dst = reinterpret_cast<uint4*>(a.out + ((c0 + (qpos < T ? qpos : 0)) * a.H + h) * kD);
#pragma unroll
      for (int c0 = 0; c0 < kD; c0 += 16) {  // every lane loads (warp-collective); valid rows store
        float v[16];
        tc::tmem_ld16(t_o + c0, v);
        tc::tmem_ld_wait();
        if (qpos < T) {
#pragma unroll
          for (int u = 0; u < 2; ++u)
            dst[c0 / 8 + u] = make_uint4(pack_bf16(v[8 * u] * inv, v[8 * u + 1] * inv),
                                         pack_bf16(v[8 * u + 2] * inv, v[8 * u + 3] * inv),
                                         pack_bf16(v[8 * u + 4] * inv, v[8 * u + 5] * inv),
                                         pack_bf16(v[8 * u + 6] * inv, v[8 * u + 7] * inv));
        }
      }
    }
  }

  if (!ok) record_device_error(&g_attn_error, kErrAttnWaitTimeout);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------- rotary + cache fill
__global__ void __launch_bounds__(256) anchor_qkv_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                         const int64_t* __restrict__ cu,
                                                         const int64_t* __restrict__ start,
                                                         const int64_t* __restrict__ rows, int64_t B, int64_t n, int H,
                                                         float theta, __nv_bfloat16* __restrict__ q_out,
                                                         int q_head_major, __nv_bfloat16* __restrict__ kc,
                                                         __nv_bfloat16* __restrict__ vc, int64_t cache_batch,
                                                         int64_t L) {
  const int64_t tok = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (tok >= n) return;
  int64_t lo = 0, hi = B - 1;  // the sequence holding the token: the last b with cu[b] <= tok
  while (lo < hi) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= tok) lo = mid;
    else hi = mid - 1;
  }
  const int64_t b = lo;
  const int64_t pos = tok - cu[b] + (start ? start[b] : 0);
  const int64_t row = rows ? rows[b] : b;
  const bool cache_ok = pos >= 0 && pos < L && row >= 0 && row < cache_batch;
  if (!cache_ok && lane == 0) record_device_error(&g_attn_error, kErrSlotOutOfRange);
  const int f = lane & 15;  // frequencies 2f, 2f + 1
  float cs[2], sn[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float inv = powf(theta, -float(2 * (2 * f + i)) / float(kD));
    const float ang = __fmul_rn(float(pos), inv);
    cs[i] = cosf(ang);
    sn[i] = sinf(ang);
  }
  const int64_t rowlen = int64_t(3) * H * kD;
  const bool is_k = lane >= 16;
  for (int h = 0; h < H; ++h) {
    const __nv_bfloat16* src = qkv + tok * rowlen + (is_k ? H * kD : 0) + h * kD;
    const float2 lo2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + 2 * f));
    const float2 hi2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + 32 + 2 * f));
    const float ol0 = __fadd_rn(__fmul_rn(lo2.x, cs[0]), -__fmul_rn(hi2.x, sn[0]));
    const float ol1 = __fadd_rn(__fmul_rn(lo2.y, cs[1]), -__fmul_rn(hi2.y, sn[1]));
    const float oh0 = __fadd_rn(__fmul_rn(hi2.x, cs[0]), __fmul_rn(lo2.x, sn[0]));
    const float oh1 = __fadd_rn(__fmul_rn(hi2.y, cs[1]), __fmul_rn(lo2.y, sn[1]));
    __nv_bfloat16* dst;
    if (is_k) {
      dst = cache_ok ? kc + ((row * H + h) * L + pos) * kD : nullptr;
    } else {
      dst = q_out + (q_head_major ? (int64_t(h) * n + tok) : (tok * H + h)) * kD;
    }
    if (dst) {
      *reinterpret_cast<__nv_bfloat162*>(dst + 2 * f) = __floats2bfloat162_rn(ol0, ol1);
      *reinterpret_cast<__nv_bfloat162*>(dst + 32 + 2 * f) = __floats2bfloat162_rn(oh0, oh1);
    }
    if (cache_ok) {
      const __nv_bfloat16* vs = qkv + tok * rowlen + 2 * H * kD + h * kD;
      *reinterpret_cast<__nv_bfloat162*>(vc + ((row * H + h) * L + pos) * kD + 2 * lane) =
          *reinterpret_cast<const __nv_bfloat162*>(vs + 2 * lane);
    }
  }
}

PFN_cuTensorMapEncodeTiled_v12000 map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// bf16 [rows, 64] row-major, boxes of 64 x 128 rows, 128-byte swizzle (the MMA operand layout)
bool encode_rows64(CUtensorMap* map, const void* base, int64_t rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = map_encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cuuint64_t(kD), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(kD) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kD), cuuint32_t(kBQ)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_anchor_qkv(const void* qkv, const int64_t* cu, const int64_t* start, const int64_t* rows, int64_t B,
                              int64_t n, int H, float theta, void* q_out, bool q_head_major, void* k_cache,
                              void* v_cache, int64_t cache_batch, int64_t L, cudaStream_t stream) {
  const int64_t grid = (n + 7) / 8;
  anchor_qkv_kernel<<<unsigned(grid), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(qkv), cu, start, rows, B, n, H, theta, static_cast<__nv_bfloat16*>(q_out),
      q_head_major ? 1 : 0, static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), cache_batch,
      L);
  return cudaGetLastError();
}

cudaError_t launch_anchor_attention(const void* q, const void* k_cache, const void* v_cache, const int64_t* cu,
                                    const int64_t* rows, int64_t B, int64_t n, int H, int64_t cache_batch, int64_t L,
                                    int64_t max_seqlen, void* out, cudaStream_t stream) {
  CUtensorMap mq, mk, mv;
  if (!encode_rows64(&mq, q, int64_t(H) * n) || !encode_rows64(&mk, k_cache, cache_batch * H * L) ||
      !encode_rows64(&mv, v_cache, cache_batch * H * L))
    return cudaErrorNotSupported;
  cudaError_t e = cudaFuncSetAttribute(anchor_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmem));
  if (e != cudaSuccess) return e;
  AttnArgs a{cu, rows, static_cast<__nv_bfloat16*>(out), n, cache_batch, L, H};
  const int64_t blocks = (max_seqlen + kQT * kBQ - 1) / (kQT * kBQ);
  anchor_attn_kernel<<<dim3(unsigned(B * H), unsigned(blocks)), kThreads, kSmem, stream>>>(a, mq, mk, mv);
  return cudaGetLastError();
}

int64_t anchor_attention_max_blocks() { return 65535; }

cudaError_t attn_read_error(cudaStream_t stream, int* code) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_attn_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  if (h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_attn_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return e;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  }
  *code = h;
  return cudaSuccess;
}

}  // namespace kdn
