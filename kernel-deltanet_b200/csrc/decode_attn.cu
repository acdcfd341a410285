// decode_attn.cu -- one-token softmax attention over a KV cache (the anchor layers' decode step).
//
// The hybrid model's anchor layers (models/upcycling_llama_bridge.py:240-249) attend, at every
// decode step, from one query per (sequence, head) to every cached key of that sequence.  That is
// a pure streaming read of K and V (256 bytes per key at d = 64, bf16); with a few sequences the
// (sequence, head) pairs alone cannot fill the GPU, so the key range is split: CTA (b, h, s) reduces
// keys [s*kKeys, (s+1)*kKeys) of sequence b to a partial (running max, sum of exponentials, weighted
// value sum), and a second kernel merges the partials of (b, h).  CTAs past a sequence's length
// exit at once, so the cost follows the live lengths even when the launch (e.g. inside a CUDA graph)
// is sized for the cache's capacity.
//
// In a CTA a warp takes groups of 32 keys: 8 lanes share a key and its value row (8 elements each, so a
// warp instruction reads four whole contiguous rows) and finish the key's dot product with 3 shuffles.
// The warp keeps an online softmax over its keys; each lane accumulates its 8 value dimensions over its
// own keys, and the 4 key subgroups of a warp are summed once, at the end.  All of a group's key and
// value chunks are loaded before any is used, so 16 loads per lane are in flight at once.
#include <math.h>

#include "kdn_common.cuh"
#include "kdn_internal.h"

namespace kdn {
namespace {

constexpr int kHd = 64;        // head dimension
constexpr int kKeys = 1024;    // keys per CTA
constexpr int kWarps = 4;
constexpr int kPart = kHd + 2; // partial record: m, l, acc[64]

// 8 consecutive elements of a cache row (16 bytes of bf16, 32 of fp32)
template <typename T>
struct Chunk;
template <>
struct Chunk<__nv_bfloat16> {
  uint4 u;
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { u = *reinterpret_cast<const uint4*>(p); }
  __device__ __forceinline__ void zero() { u = make_uint4(0u, 0u, 0u, 0u); }
  __device__ __forceinline__ void to_float(float* f) const {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
      f[2 * e] = t.x;
      f[2 * e + 1] = t.y;
    }
  }
};
template <>
struct Chunk<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = reinterpret_cast<const float4*>(p)[0];
    b = reinterpret_cast<const float4*>(p)[1];
  }
  __device__ __forceinline__ void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void to_float(float* f) const {
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
};

template <typename T>
__global__ void __launch_bounds__(32 * kWarps) decode_attn_partial_kernel(const T* __restrict__ q,
                                                                          const T* __restrict__ kc,
                                                                          const T* __restrict__ vc,
                                                                          const int64_t* __restrict__ lengths,
                                                                          float* __restrict__ part, int H,
                                                                          int64_t max_len, int splits, float scale) {
  __shared__ float red[kWarps][kPart];
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nkeys = lengths[b] + 1;  // positions [0, lengths[b]]
  const int64_t k0 = int64_t(s) * kKeys;
  float* out = part + ((int64_t(b) * H + h) * splits + s) * kPart;
  if (k0 >= nkeys || nkeys > max_len) {  // nothing of this sequence here (or a length out of range)
    if (threadIdx.x == 0) {
      out[0] = -INFINITY;
      out[1] = 0.f;
    }
    if (threadIdx.x < kHd) out[2 + threadIdx.x] = 0.f;
    return;
  }
  const int64_t k1 = (k0 + kKeys < nkeys) ? k0 + kKeys : nkeys;
  const int64_t bh = int64_t(b) * H + h;
  // lane l takes the 16-byte chunk sub = l % 8 of keys (l / 8) + 4 i (i < 8): a warp instruction reads four
  // whole contiguous key rows, and the 8 lanes of a key finish its dot product with 3 shuffles
  const int sub = lane & 7, grp = lane >> 3;
  float qs[8];  // this lane's 8 query elements [8 sub, 8 sub + 8)
  {
    Chunk<T> qc;
    qc.load(q + bh * kHd + 8 * sub);
    qc.to_float(qs);
  }
  const T* kb = kc + bh * max_len * kHd;
  const T* vb = vc + bh * max_len * kHd;
  float m = -INFINITY, l = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // dims [8 sub, 8 sub + 8)
  for (int64_t j0 = k0 + 32 * warp; j0 < k1; j0 += 32 * kWarps) {
    const int cnt = int((k1 - j0) < 32 ? (k1 - j0) : 32);
    // all of this lane's key and value chunks of the group in flight at once
    Chunk<T> kr[8], vr[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int kk = grp + 4 * i;  // key within the group
      if (kk < cnt) {
        kr[i].load(kb + (j0 + kk) * kHd + 8 * sub);
        vr[i].load(vb + (j0 + kk) * kHd + 8 * sub);
      } else {
        kr[i].zero();
        vr[i].zero();
      }
    }
    float sc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float kf[8];
      kr[i].to_float(kf);
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) dot = fmaf(qs[e], kf[e], dot);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      sc[i] = grp + 4 * i < cnt ? dot * scale : -INFINITY;
    }
    float mx = sc[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, sc[i]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float mn = fmaxf(m, mx);  // finite: the group has at least one key
    const float corr = expf(m - mn);
    float ps = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] *= corr;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float p = (grp + 4 * i < cnt) ? expf(sc[i] - mn) : 0.f;
      ps += p;
      float vf[8];
      vr[i].to_float(vf);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(p, vf[e], acc[e]);
    }
    // a key's probability sits in all 8 of its lanes: sum one lane per key subgroup (lanes 0, 8, 16, 24)
    ps = (sub == 0) ? ps : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l = l * corr + ps;
    m = mn;
  }
  // the 4 key subgroups share the running max, so their value sums add directly
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 8);
    acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], 16);
  }
  if (lane == 0) {
    red[warp][0] = m;
    red[warp][1] = l;
  }
  if (grp == 0) {
#pragma unroll
    for (int e = 0; e < 8; ++e) red[warp][2 + 8 * sub + e] = acc[e];
  }
  __syncthreads();
  if (warp == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red[w][0]);
    float L = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = red[w][0] == -INFINITY ? 0.f : expf(red[w][0] - M);
      L = fmaf(red[w][1], f, L);
      o0 = fmaf(red[w][2 + 2 * lane], f, o0);
      o1 = fmaf(red[w][3 + 2 * lane], f, o1);
    }
    if (lane == 0) {
      out[0] = M;
      out[1] = L;
    }
    out[2 + 2 * lane] = o0;
    out[3 + 2 * lane] = o1;
  }
}

// one warp per (b, h): merge the partials, o = sum_s acc_s e^{m_s - M} / sum_s l_s e^{m_s - M}
template <typename T>
__global__ void __launch_bounds__(256) decode_attn_merge_kernel(const float* __restrict__ part, T* __restrict__ o,
                                                                int64_t BH, int splits) {
  const int64_t bh = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (bh >= BH) return;
  const float* p = part + bh * splits * kPart;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, p[s * kPart]);
  float L = 0.f, o0 = 0.f, o1 = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = p[s * kPart];
    if (ms == -INFINITY) continue;
    const float f = expf(ms - M);
    L = fmaf(p[s * kPart + 1], f, L);
    o0 = fmaf(p[s * kPart + 2 + 2 * lane], f, o0);
    o1 = fmaf(p[s * kPart + 3 + 2 * lane], f, o1);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  if constexpr (sizeof(T) == 2)
    reinterpret_cast<__nv_bfloat162*>(o + bh * kHd)[lane] = __floats2bfloat162_rn(o0 * inv, o1 * inv);
  else
    reinterpret_cast<float2*>(o + bh * kHd)[lane] = make_float2(o0 * inv, o1 * inv);
}

}  // namespace

int decode_attn_splits(int64_t max_len) { return int((max_len + kKeys - 1) / kKeys); }

size_t decode_attn_workspace(int64_t B, int H, int64_t max_len) {
  return sizeof(float) * size_t(B) * H * decode_attn_splits(max_len) * kPart;
}

cudaError_t launch_decode_attn(const void* q, const void* k_cache, const void* v_cache, const int64_t* lengths,
                               void* out, int dt, int64_t B, int H, int64_t max_len, float* part,
                               cudaStream_t stream) {
  const int splits = decode_attn_splits(max_len);
  const dim3 grid{unsigned(splits), unsigned(H), unsigned(B)};
  const float scale = 0.125f;  // 1 / sqrt(64)
  if (dt == KDN_DTYPE_BF16) {
    decode_attn_partial_kernel<__nv_bfloat16><<<grid, 32 * kWarps, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k_cache),
        static_cast<const __nv_bfloat16*>(v_cache), lengths, part, H, max_len, splits, scale);
  } else {
    decode_attn_partial_kernel<float><<<grid, 32 * kWarps, 0, stream>>>(
        static_cast<const float*>(q), static_cast<const float*>(k_cache), static_cast<const float*>(v_cache), lengths,
        part, H, max_len, splits, scale);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int64_t BH = B * H;
  const unsigned mg = unsigned((BH + 7) / 8);
  if (dt == KDN_DTYPE_BF16)
    decode_attn_merge_kernel<__nv_bfloat16><<<mg, 256, 0, stream>>>(part, static_cast<__nv_bfloat16*>(out), BH,
                                                                    splits);
  else
    decode_attn_merge_kernel<float><<<mg, 256, 0, stream>>>(part, static_cast<float*>(out), BH, splits);
  return cudaGetLastError();
}

}  // namespace kdn
