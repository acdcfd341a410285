// glue.cu -- the element-wise steps between the hybrid LM's GEMMs, one HBM pass each.
//
// A pre-norm hybrid block (layers/hybrid_kernel_deltanet_block.py:85-96) surrounds its GEMMs
// with residual adds and RMSNorm (:23-25; an add and the norm after it are one kernel), SwiGLU's silu(gate) * up (:45-46) and, in the Kernel-DeltaNet mixer,
// the split of the fused q|k|v|beta projection into unit-norm q and k per head
// (layers/kernel_deltanet_layer.py:98-99), v, beta = sigmoid(.) (serving/tensor_parallel_runner.py:62)
// and the per-head decay sigmoid(logit_decay) (kernel_deltanet_layer.py:71-73).  Written as
// separate framework element-wise ops these are 5-8 passes over each activation; here each is
// one kernel that reads its input once and writes its outputs once (fp32 arithmetic, bf16 or
// fp32 storage, 16-byte vectors).
#include "kdn_common.cuh"
#include "kdn_internal.h"

namespace kdn {
namespace {

template <typename T>
struct V16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* f) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  } else {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u = make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), __float_as_uint(f[3]));
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<const uint32_t*>(&t);
    }
    u = make_uint4(w[0], w[1], w[2], w[3]);
  }
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename T>
__device__ __forceinline__ float round_to(float v) {  // the value a T tensor would hold
  if constexpr (sizeof(T) == 2) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}

// one warp per row: h = x + res (when res is given: rounded to T and stored to h_out, as a separate
// add would leave it), out = h * rsqrt(mean(h^2) + eps) * w.  The first kRowVecs 16-byte vectors of
// each lane stay in registers between the two passes (d <= 2048 bf16 / 1024 fp32 is one read of the
// row); the rest is read again from h_out (or x).  h_out may be x; out must not alias x, res or h_out.
constexpr int kRowVecs = 8;

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const T* x, const T* res,
                                                      const void* __restrict__ w, int wdt, bool wvec, T* h_out,
                                                      T* __restrict__ out, int64_t n, int d, float eps) {
  constexpr int V = V16<T>::N;
  const int64_t row = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const int nv = d / V;
  const T* xr = x + row * d;
  const T* rr = res ? res + row * d : nullptr;
  T* hr = res ? h_out + row * d : nullptr;
  auto load_h = [&](int vi, float* f) {
    load16(xr + vi * V, f);
    if (rr) {
      float r[V];
      load16(rr + vi * V, r);
#pragma unroll
      for (int j = 0; j < V; ++j) f[j] = round_to<T>(f[j] + r[j]);
    }
  };
  float keep[kRowVecs][V];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRowVecs; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
      load_h(vi, keep[i]);
#pragma unroll
      for (int j = 0; j < V; ++j) ss = fmaf(keep[i][j], keep[i][j], ss);
    }
  }
  for (int vi = lane + 32 * kRowVecs; vi < nv; vi += 32) {  // long rows
    float f[V];
    load_h(vi, f);
#pragma unroll
    for (int j = 0; j < V; ++j) ss = fmaf(f[j], f[j], ss);
    if (hr) store16(hr + vi * V, f);
  }
  const float r = rsqrtf(warp_sum(ss) / float(d) + eps);
  T* orow = out + row * d;
  auto finish = [&](int vi, float* f) {
    float wf[V];
    if (wvec) {
      load16(static_cast<const T*>(w) + vi * V, wf);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) wf[j] = ld_as_f32(w, wdt, vi * V + j);
    }
#pragma unroll
    for (int j = 0; j < V; ++j) f[j] = f[j] * r * wf[j];
    store16(orow + vi * V, f);
  };
#pragma unroll
  for (int i = 0; i < kRowVecs; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nv) {
      if (hr) store16(hr + vi * V, keep[i]);
      finish(vi, keep[i]);
    }
  }
  for (int vi = lane + 32 * kRowVecs; vi < nv; vi += 32) {
    float f[V];
    load16((hr ? hr : xr) + vi * V, f);  // this lane's own earlier store when h is written
    finish(vi, f);
  }
}

__device__ __forceinline__ float silu(float g) { return g / (1.f + expf(-g)); }

// out[r, j] = silu(gu[r, j]) * gu[r, f + j]
template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* __restrict__ gu, T* __restrict__ out, int64_t n, int f) {
  constexpr int V = V16<T>::N;
  const int per_row = f / V;
  const int64_t total = n * per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row;
    const int c = int(i - r * per_row) * V;
    float g[V], u[V];
    load16(gu + r * 2 * f + c, g);
    load16(gu + r * 2 * f + f + c, u);
#pragma unroll
    for (int j = 0; j < V; ++j) g[j] = silu(g[j]) * u[j];
    store16(out + r * f + c, g);
  }
}

// one warp per (token, head): z row = [q (H*64) | k (H*64) | v (H*64) | beta logits (H)]
__global__ void __launch_bounds__(256) mixer_inputs_kernel(const void* __restrict__ z, int dt, int64_t n, int H,
                                                           int64_t ld, const void* __restrict__ logit_decay, int lddt,
                                                           const int64_t* __restrict__ cu, int64_t num_seqs,
                                                           void* __restrict__ q, void* __restrict__ k,
                                                           void* __restrict__ v, float* __restrict__ beta,
                                                           float* __restrict__ decay) {
  const int64_t item = int64_t(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= n * H) return;
  const int64_t r = item / H;
  const int h = int(item - r * H);
  const int64_t zr = r * ld;  // z row stride (elements)
  int64_t dst = item;         // output row: [n, H] token-major, or head-major per sequence
  if (cu) {
    int64_t lo = 0, hi = num_seqs - 1;  // the sequence holding token r: the last b with cu[b] <= r
    while (lo < hi) {
      const int64_t mid = (lo + hi + 1) >> 1;
      if (cu[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    const int64_t c0 = cu[lo];
    dst = c0 * H + int64_t(h) * (cu[lo + 1] - c0) + (r - c0);
  }
  const int64_t o = dst * kDk + 2 * lane;
  float2 qv, kv, vv;
  if ((ld & 1) == 0) {
    qv = ld2_as_f32(z, dt, zr + int64_t(h) * kDk + 2 * lane);
    kv = ld2_as_f32(z, dt, zr + int64_t(H + h) * kDk + 2 * lane);
    vv = ld2_as_f32(z, dt, zr + int64_t(2 * H + h) * kDk + 2 * lane);
  } else {  // odd row length: element loads
    const int64_t b = 2 * lane;
    qv = make_float2(ld_as_f32(z, dt, zr + int64_t(h) * kDk + b), ld_as_f32(z, dt, zr + int64_t(h) * kDk + b + 1));
    kv = make_float2(ld_as_f32(z, dt, zr + int64_t(H + h) * kDk + b),
                     ld_as_f32(z, dt, zr + int64_t(H + h) * kDk + b + 1));
    vv = make_float2(ld_as_f32(z, dt, zr + int64_t(2 * H + h) * kDk + b),
                     ld_as_f32(z, dt, zr + int64_t(2 * H + h) * kDk + b + 1));
  }
  // unit norm per head, as F.normalize: x / max(||x||, 1e-12)
  const float qs = 1.f / fmaxf(sqrtf(warp_sum(qv.x * qv.x + qv.y * qv.y)), 1e-12f);
  const float ks = 1.f / fmaxf(sqrtf(warp_sum(kv.x * kv.x + kv.y * kv.y)), 1e-12f);
  st2_from_f32(q, dt, o, qv.x * qs, qv.y * qs);
  st2_from_f32(k, dt, o, kv.x * ks, kv.y * ks);
  st2_from_f32(v, dt, o, vv.x, vv.y);
  if (lane == 0) {
    const float bl = ld_as_f32(z, dt, zr + int64_t(3) * H * kDk + h);
    beta[dst] = 1.f / (1.f + expf(-bl));
    decay[dst] = 1.f / (1.f + expf(-ld_as_f32(logit_decay, lddt, h)));
  }
}

int grid_for(int64_t items, int per_block) {
  const int64_t g = (items + per_block - 1) / per_block;
  return int(g < 1 ? 1 : (g > (int64_t(1) << 30) ? (int64_t(1) << 30) : g));
}

}  // namespace

cudaError_t launch_rmsnorm(const void* x, const void* res, const void* w, int wdt, void* h_out, void* out, int dt,
                           int64_t n, int d, float eps, cudaStream_t stream) {
  const int grid = grid_for(n, 8);
  const bool wvec = wdt == dt && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  if (dt == KDN_DTYPE_BF16)
    rmsnorm_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(res), w, wdt, wvec,
        static_cast<__nv_bfloat16*>(h_out), static_cast<__nv_bfloat16*>(out), n, d, eps);
  else
    rmsnorm_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(x), static_cast<const float*>(res), w,
                                                     wdt, wvec, static_cast<float*>(h_out), static_cast<float*>(out),
                                                     n, d, eps);
  return cudaGetLastError();
}

cudaError_t launch_swiglu(const void* gu, void* out, int dt, int64_t n, int f, cudaStream_t stream) {
  const int64_t vecs = n * (f / (dt == KDN_DTYPE_BF16 ? 8 : 4));
  const int grid = int(vecs / 256 + 1 < 148 * 16 ? vecs / 256 + 1 : 148 * 16);
  if (dt == KDN_DTYPE_BF16)
    swiglu_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(gu),
                                                            static_cast<__nv_bfloat16*>(out), n, f);
  else
    swiglu_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float*>(gu), static_cast<float*>(out), n, f);
  return cudaGetLastError();
}

cudaError_t launch_mixer_inputs(const void* z, int dt, int64_t n, int H, int64_t z_ld, const void* logit_decay,
                                int lddt, const int64_t* cu, int64_t num_seqs, void* q, void* k, void* v, float* beta,
                                float* decay, cudaStream_t stream) {
  mixer_inputs_kernel<<<grid_for(n * H, 8), 256, 0, stream>>>(z, dt, n, H, z_ld, logit_decay, lddt, cu, num_seqs, q,
                                                              k, v, beta, decay);
  return cudaGetLastError();
}

}  // namespace kdn
