// prefill_simt.cu -- exact fp32 chunked delta-rule prefill on CUDA cores (KDN_MODE_F32).
//
// Chunk algebra (tokens i,j of one chunk, 0-based; g_i = sum_{l<=i} log clamp(decay_l);
// k_i, q_i the lifted features; S_0 the state entering the chunk):
//
//   A_ij  = beta_i exp(g_i - g_j) (k_i . k_j)        j < i      (the reference's L_c,
//   T     = (I + A)^-1                                           fused_kernel_deltanet.py:113-116)
//   R_i   = beta_i (v_i - exp(g_i) k_i S_0^T)                     pseudo-value right-hand side
//   E     = T R                                                   (rows e_i of new values)
//   y_i   = exp(g_{i-1}) q_i S_0^T + sum_{j<i} exp(g_{i-1} - g_j) (q_i . k_j) e_j
//   S_C   = exp(g_{C-1}) S_0 + sum_j exp(g_{C-1} - g_j) e_j^T k_j
//
// This is the same map as kernels/fused_kernel_deltanet.py:99-149 (the reference's
// decay-free upper resolvent inv_U equals diag(1/gamma) T diag(gamma) transposed);
// here the S_0-dependent and value-dependent parts share one triangular product.
//
// Launches: (1) lift k and q into the workspace, (2) per (chunk, sequence):
// Gram matrices, gates, T and the decayed q.k matrix, (3) per (sequence,
// tile of 4, 8 or 16 rows of S): the serial pass over chunks.
#include <math.h>

#include "kdn_internal.h"
#include "lift.cuh"
#include "tc_prims.cuh"

namespace kdn {
namespace {

constexpr int kThreads = 256;
// padded rows (floats) of the chunk-64 chain's shared tiles: T and Aq (16-byte row reads), the feature
// slices and the state (8-byte fragment reads: a row stride of 8 mod 32 words keeps them conflict-free)
constexpr int kChainLd = 68, kChainRingLd = 72, kChainSd = 520;

struct Workspace {
  float* phik;   // [N, Tp, D]
  float* phiq;   // [N, Tp, D]
  float* Tinv;   // [N, NC, C, C]
  float* Aq;     // [N, NC, C, C]
  float* gates;  // [N, NC, C, 4] = exp(g_{i-1}), exp(g_i), exp(g_{C-1} - g_i), beta_i
  int64_t Tp;
  int NC;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---- exact-fp32 products on the tensor cores: x = hi + lo with hi = x truncated to tf32 and lo the
// exact remainder (which the tensor core reads at tf32 precision, within 2^-20 |x|), and
// a b ~ hi_a hi_b + hi_a lo_b + lo_a hi_b (the split-tf32 scheme of Markidis et al., 2018): each tf32
// product is exact in the fp32 accumulator and the dropped terms are about 2^-20 |a b|, near the
// accuracy of an fp32 dot product.
__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = __float_as_uint(x) & 0xffffe000u;        // tf32 by truncation: the top 19 bits
  lo = __float_as_uint(x - __uint_as_float(hi));  // the exact remainder, below 2^-10 |x|, read as tf32
}
// c += a b for a 16 x 8 tile of a (row-major fragment a[4]) and an 8 x 8 tile of b (b0, b1)
__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_3xtf32(float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                           const uint32_t (&bh)[2], const uint32_t (&bl)[2]) {
  mma_tf32(c, al, bh[0], bh[1]);  // the small terms first
  mma_tf32(c, ah, bl[0], bl[1]);
  mma_tf32(c, ah, bh[0], bh[1]);
}

Workspace carve(void* base, int64_t N, int64_t T, int dv, int C, int D, size_t* total) {
  (void)dv;
  Workspace w;
  w.NC = int((T + C - 1) / C);
  w.Tp = int64_t(w.NC) * C;
  size_t off = 0;
  char* b = static_cast<char*>(base);
  auto take = [&](size_t bytes) {
    char* p = b ? b + off : nullptr;
    off = align256(off + bytes);
    return reinterpret_cast<float*>(p);
  };
  w.phik = take(sizeof(float) * size_t(N) * w.Tp * D);
  w.phiq = take(sizeof(float) * size_t(N) * w.Tp * D);
  w.Tinv = take(sizeof(float) * size_t(N) * w.NC * C * C);
  w.Aq = take(sizeof(float) * size_t(N) * w.NC * C * C);
  w.gates = take(sizeof(float) * size_t(N) * w.NC * C * 4);
  if (total) *total = off;
  return w;
}

// (1) lift k and q rows into [N, Tp, D]; padded rows (t >= T) become zeros.  Without a
// readout (y null) only k is lifted.
__global__ void __launch_bounds__(kThreads) simt_lift_kernel(PrefillProblem p, Workspace w, ProjParams P) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t rows = p.N * w.Tp;
  const int D = p.D;
  const int64_t total = (p.y || p.with_q) ? 2 * rows : rows;
  for (int64_t r = warp; r < total; r += nwarps) {
    const bool isq = r >= rows;
    const int64_t row = isq ? r - rows : r;
    const int64_t n = row / w.Tp, t = row % w.Tp;
    float* dst = (isq ? w.phiq : w.phik) + row * D;
    if (t >= p.T) {
      for (int d = 2 * lane; d < D; d += 64) *reinterpret_cast<float2*>(dst + d) = make_float2(0.f, 0.f);
      continue;
    }
    const float2 xv = ld2_as_f32(isq ? p.q : p.k, p.in_dtype, (n * p.T + t) * kDk + 2 * lane);
    float c[kMaxBlocks][2];
    lift_warp(xv.x, xv.y, P, lane, c);
#pragma unroll
    for (int m = 0; m < kMaxBlocks; ++m)
      if (m < P.M) *reinterpret_cast<float2*>(dst + 64 * m + 2 * lane) = make_float2(c[m][0], c[m][1]);
  }
}

// floats of one staged 64-feature slice in the preparation: feature-major rows of 68 (16-byte reads of
// a thread's 4 token rows) for chunk 64, token-major rows of 65 otherwise
template <int C>
constexpr int prep_stage_floats() {
  return C == 64 ? 64 * 68 : C * 65;
}

// (2) per (chunk c, sequence n): G = K K^T, P = Q K^T, gates, T = (I + A)^-1, Aq.
// kQ = false (no readout): P and Aq are skipped (Aq is written as zeros).
template <int C, bool kQ>
__global__ void __launch_bounds__(kThreads) simt_prep_kernel(PrefillProblem p, Workspace w) {
  constexpr int R = C / 16;  // each thread owns an R x R tile of G and of P
  constexpr int LD = C + 1;
  constexpr int SL = prep_stage_floats<C>();  // floats of one staged slice
  extern __shared__ float sm[];
  float* Ks = sm;            // chunk 64: [64 features][68] (feature-major); else [C][65]
  float* Qs = Ks + SL;
  float* G = Qs + SL;        // [C][LD], becomes A
  float* Pm = G + C * LD;    // [C][LD], becomes Aq
  float* Tm = Pm + C * LD;   // [C][LD]
  float* gl = Tm + C * LD;   // [C]
  float* bt = gl + C;        // [C]

  const int c = blockIdx.x;
  const int64_t n = blockIdx.y;
  const int tid = threadIdx.x;
  const int ti = tid / 16, tj = tid % 16;
  const int D = p.D;
  const float* Kg = w.phik + (n * w.Tp + int64_t(c) * C) * D;
  const float* Qg = w.phiq + (n * w.Tp + int64_t(c) * C) * D;

  float g[R][R], pq[R][R];
#pragma unroll
  for (int a = 0; a < R; ++a)
#pragma unroll
    for (int b = 0; b < R; ++b) g[a][b] = pq[a][b] = 0.f;

  for (int d0 = 0; d0 < D; d0 += 64) {
    for (int e = tid; e < C * 64; e += kThreads) {
      const int r = e >> 6, cc = e & 63;
      if constexpr (C == 64) {  // feature-major: a thread's 4 rows at one feature are one 16-byte read
        Ks[cc * 68 + r] = Kg[int64_t(r) * D + d0 + cc];
        if (kQ) Qs[cc * 68 + r] = Qg[int64_t(r) * D + d0 + cc];
      } else {
        Ks[r * 65 + cc] = Kg[int64_t(r) * D + d0 + cc];
        if (kQ) Qs[r * 65 + cc] = Qg[int64_t(r) * D + d0 + cc];
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int dd = 0; dd < 64; ++dd) {
      float a[R], qq[R], b[R];
      if constexpr (C == 64) {
        const float4 a4 = *reinterpret_cast<const float4*>(Ks + dd * 68 + ti * R);
        const float4 b4 = *reinterpret_cast<const float4*>(Ks + dd * 68 + tj * R);
        a[0] = a4.x, a[1] = a4.y, a[2] = a4.z, a[3] = a4.w;
        b[0] = b4.x, b[1] = b4.y, b[2] = b4.z, b[3] = b4.w;
        if (kQ) {
          const float4 q4 = *reinterpret_cast<const float4*>(Qs + dd * 68 + ti * R);
          qq[0] = q4.x, qq[1] = q4.y, qq[2] = q4.z, qq[3] = q4.w;
        } else {
          qq[0] = qq[1] = qq[2] = qq[3] = 0.f;
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          a[r] = Ks[(ti * R + r) * 65 + dd];
          qq[r] = kQ ? Qs[(ti * R + r) * 65 + dd] : 0.f;
          b[r] = Ks[(tj * R + r) * 65 + dd];
        }
      }
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int s = 0; s < R; ++s) {
          g[r][s] = fmaf(a[r], b[s], g[r][s]);
          if (kQ) pq[r][s] = fmaf(qq[r], b[s], pq[r][s]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int s = 0; s < R; ++s) {
      G[(ti * R + r) * LD + tj * R + s] = g[r][s];
      Pm[(ti * R + r) * LD + tj * R + s] = pq[r][s];
    }

  // gates: beta and log clamp(decay, 1e-5, 1) (fused_kernel_deltanet.py:74); padded rows beta=0, decay=1
  if (tid < C) {
    const int64_t t = int64_t(c) * C + tid;
    float b = 0.f, dec = 1.f;
    if (t < p.T) {
      b = ld_as_f32(p.beta, p.gate_dtype, n * p.T + t);
      if (p.decay) dec = ld_as_f32(p.decay, p.gate_dtype, n * p.T + t);
    }
    bt[tid] = b;
    gl[tid] = logf(fminf(fmaxf(dec, 1e-5f), 1.0f));
  }
  __syncthreads();
  if (tid == 0) {  // sequential inclusive prefix sum, same order as the reference's cumsum
    float s = 0.f;
    for (int i = 0; i < C; ++i) {
      s += gl[i];
      gl[i] = s;
    }
  }
  __syncthreads();

  for (int e = tid; e < C * C; e += kThreads) {
    const int i = e / C, j = e % C;
    float a = 0.f, aq = 0.f;
    if (j < i) {
      a = bt[i] * expf(gl[i] - gl[j]) * G[i * LD + j];
      aq = Pm[i * LD + j] * expf(gl[i - 1] - gl[j]);
    }
    G[i * LD + j] = a;
    Pm[i * LD + j] = aq;
    Tm[i * LD + j] = (i == j) ? 1.f : 0.f;
  }
  __syncthreads();
  // forward substitution T_ij = -sum_{l=j}^{i-1} A_il T_lj (j < i): the columns of T are independent,
  // so thread j takes column j down the rows with the column so far in registers (A_il read by all
  // column threads at once: a broadcast)
  if (tid < C) {
    const int j = tid;
    float col[C];
#pragma unroll
    for (int l = 0; l < C; ++l) col[l] = (l == j) ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < C; ++i) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int l = 0; l < i; l += 2) {
        s0 = fmaf(G[i * LD + l], col[l], s0);
        if (l + 1 < i) s1 = fmaf(G[i * LD + l + 1], col[l + 1], s1);
      }
      if (i > j) col[i] = -(s0 + s1);
    }
#pragma unroll
    for (int l = 0; l < C; ++l) Tm[l * LD + j] = col[l];
  }
  __syncthreads();

  float* To = w.Tinv + (n * w.NC + c) * int64_t(C) * C;
  float* Ao = w.Aq + (n * w.NC + c) * int64_t(C) * C;
  for (int e = tid; e < C * C; e += kThreads) {
    const int i = e / C, j = e % C;
    To[e] = Tm[i * LD + j];
    Ao[e] = Pm[i * LD + j];
  }
  float* go = w.gates + (n * w.NC + c) * int64_t(C) * 4;
  if (tid < C) {
    const int i = tid;
    const float gprev = i > 0 ? gl[i - 1] : 0.f;
    go[4 * i + 0] = expf(gprev);
    go[4 * i + 1] = expf(gl[i]);
    go[4 * i + 2] = expf(gl[C - 1] - gl[i]);
    go[4 * i + 3] = bt[i];
  }
}

template <int C>
constexpr size_t prep_smem_bytes() {
  return sizeof(float) * (2 * prep_stage_floats<C>() + 3 * C * (C + 1) + 2 * C);
}

// (3) per (tile of RT rows of S, sequence n): the serial pass over chunks (RT = 16, or 8 when the
// tiles of 16 would leave SMs idle).  Tiles below
// p.a_rows belong to the block transition's homogeneous map (identity start, v = 0,
// no readout, result to A_out); the others are value rows (S0, v, y, S_out).
template <int C, int RT>
__global__ void __launch_bounds__(kThreads) simt_chain_kernel(PrefillProblem p, Workspace w) {
  constexpr int TPR = kThreads / C;    // threads per chunk row
  constexpr int VPT = RT / TPR;  // state rows per thread in the (C x RT) phases
  constexpr int LD = C + 1;
  const int D = p.D;
  const int SD = D + 1;  // padded row stride of the S tile
  extern __shared__ float sm[];
  float* S = sm;                     // [RT][SD]
  float* Ks = S + RT * SD;     // [C][65]
  float* Qs = Ks + C * 65;           // [C][65]
  float* Tm = Qs + C * 65;           // [C][LD]
  float* Am = Tm + C * LD;           // [C][LD]
  float* gt = Am + C * LD;           // [C][4]
  float* Rs = gt + C * 4;            // [C][16]
  float* Es = Rs + C * RT;     // [C][16]

  const int vt = blockIdx.x;
  const int64_t n = blockIdx.y;
  const int tid = threadIdx.x;
  const int i = tid / TPR;
  const int v0 = (tid % TPR) * VPT;
  const bool a_tile = vt * RT < p.a_rows;
  const int row0 = a_tile ? vt * RT : vt * RT - p.a_rows;
  const bool readout = !a_tile && p.y != nullptr;  // uniform per CTA

  for (int e = tid; e < RT * D; e += kThreads) {
    const int r = e / D, d = e % D;
    float s0 = 0.f;
    if (a_tile)
      s0 = (row0 + r == d) ? 1.f : 0.f;
    else if (p.S0)
      s0 = p.S0[(n * p.dv + row0 + r) * int64_t(D) + d];
    S[r * SD + d] = s0;
  }
  __syncthreads();

  for (int c = 0; c < w.NC; ++c) {
    if (p.S_chunks && !a_tile) {  // checkpoint: the state entering chunk c
      float* Sc = p.S_chunks + ((n * w.NC + c) * p.dv + row0) * int64_t(D);
      for (int e = tid; e < RT * D; e += kThreads) Sc[e] = S[(e / D) * SD + e % D];
    }
    const float* Tg = w.Tinv + (n * w.NC + c) * int64_t(C) * C;
    const float* Ag = w.Aq + (n * w.NC + c) * int64_t(C) * C;
    const float* Gg = w.gates + (n * w.NC + c) * int64_t(C) * 4;
    for (int e = tid; e < C * C; e += kThreads) {
      Tm[(e / C) * LD + (e % C)] = Tg[e];
      Am[(e / C) * LD + (e % C)] = Ag[e];
    }
    for (int e = tid; e < C * 4; e += kThreads) gt[e] = Gg[e];

    // X = K S^T, Yq = Q S^T   (C x 16)
    const float* Kg = w.phik + (n * w.Tp + int64_t(c) * C) * D;
    const float* Qg = w.phiq + (n * w.Tp + int64_t(c) * C) * D;
    float x[VPT], yq[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) x[u] = yq[u] = 0.f;
    for (int d0 = 0; d0 < D; d0 += 64) {
      __syncthreads();
      for (int e = tid; e < C * 64; e += kThreads) {
        const int r = e >> 6, cc = e & 63;
        Ks[r * 65 + cc] = Kg[int64_t(r) * D + d0 + cc];
        if (readout) Qs[r * 65 + cc] = Qg[int64_t(r) * D + d0 + cc];
      }
      __syncthreads();
      if (readout) {
#pragma unroll 4
        for (int dd = 0; dd < 64; ++dd) {
          const float kd = Ks[i * 65 + dd], qd = Qs[i * 65 + dd];
#pragma unroll
          for (int u = 0; u < VPT; ++u) {
            const float s = S[(v0 + u) * SD + d0 + dd];
            x[u] = fmaf(kd, s, x[u]);
            yq[u] = fmaf(qd, s, yq[u]);
          }
        }
      } else {
#pragma unroll 4
        for (int dd = 0; dd < 64; ++dd) {
          const float kd = Ks[i * 65 + dd];
#pragma unroll
          for (int u = 0; u < VPT; ++u) x[u] = fmaf(kd, S[(v0 + u) * SD + d0 + dd], x[u]);
        }
      }
    }
    // R_i = beta_i (v_i - exp(g_i) x_i)
    const int64_t t = int64_t(c) * C + i;
    const float beta_i = gt[4 * i + 3], gi = gt[4 * i + 1], gprev = gt[4 * i + 0], wi = gt[4 * i + 2];
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      float vv = 0.f;
      if (!a_tile && t < p.T) vv = ld_as_f32(p.v, p.in_dtype, (n * p.T + t) * p.dv + row0 + v0 + u);
      Rs[i * RT + v0 + u] = beta_i * (vv - gi * x[u]);
    }
    __syncthreads();
    // E = T R  (T unit lower triangular)
    float e_[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) e_[u] = Rs[i * RT + v0 + u];
    for (int j = 0; j < i; ++j) {
      const float tij = Tm[i * LD + j];
#pragma unroll
      for (int u = 0; u < VPT; ++u) e_[u] = fmaf(tij, Rs[j * RT + v0 + u], e_[u]);
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Es[i * RT + v0 + u] = e_[u];
    if (p.E_rows && !a_tile) {
#pragma unroll
      for (int u = 0; u < VPT; ++u) p.E_rows[(n * w.Tp + t) * p.dv + row0 + v0 + u] = e_[u];
    }
    __syncthreads();
    // y_i = exp(g_{i-1}) yq_i + sum_{j<i} Aq_ij e_j ;  then E''_i = exp(g_{C-1} - g_i) e_i into Rs
    if (readout) {
      float yv[VPT];
#pragma unroll
      for (int u = 0; u < VPT; ++u) yv[u] = gprev * yq[u];
      for (int j = 0; j < i; ++j) {
        const float aij = Am[i * LD + j];
#pragma unroll
        for (int u = 0; u < VPT; ++u) yv[u] = fmaf(aij, Es[j * RT + v0 + u], yv[u]);
      }
      if (t < p.T) {
#pragma unroll
        for (int u = 0; u < VPT; ++u) st_from_f32(p.y, p.y_dtype, (n * p.T + t) * p.dv + row0 + v0 + u, yv[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Rs[i * RT + v0 + u] = wi * e_[u];
    __syncthreads();
    // S <- exp(g_{C-1}) S + E''^T K
    const float gC = gt[4 * (C - 1) + 1];
    for (int d = tid; d < D; d += kThreads) {
      float acc[RT];
#pragma unroll
      for (int r = 0; r < RT; ++r) acc[r] = gC * S[r * SD + d];
      for (int j = 0; j < C; ++j) {
        const float kv = Kg[int64_t(j) * D + d];
#pragma unroll
        for (int r = 0; r < RT; ++r) acc[r] = fmaf(Rs[j * RT + r], kv, acc[r]);
      }
#pragma unroll
      for (int r = 0; r < RT; ++r) S[r * SD + d] = acc[r];
    }
    __syncthreads();
  }

  float* dst = a_tile ? p.A_out + (n * p.a_rows + row0) * int64_t(D) : p.S_out + (n * p.dv + row0) * int64_t(D);
  for (int e = tid; e < RT * D; e += kThreads) {
    const int r = e / D, d = e % D;
    dst[int64_t(r) * D + d] = S[r * SD + d];
  }
}

template <int C, int RT>
size_t chain_smem_bytes(int D) {
  return sizeof(float) * (size_t(RT) * (D + 1) + 2 * C * 65 + 2 * C * (C + 1) + 4 * C + 2 * C * RT);
}

// (3) for chunk 64 and D = 512: the same serial pass with its loads off the chain.  The K and Q
// features of a chunk stream through a 3-stage cp.async ring of 64-feature slices ([64 tokens x 64]
// fp32, rows padded to 68 floats so that a 16-byte row read and the S reads are conflict-free),
// the chunk's T, Aq and gates load into one of two buffers with its first slice, and the
// products read 16 bytes at a time.  The state update reads the chunk's K rows from global memory
// (L2) as float4 with sixteen loads in flight per thread and a 4 x (RT/2) register block per thread.
// The arithmetic is the kernel above's (exact fp32), in another summation order.
template <int RT>
__global__ void __launch_bounds__(kThreads, 1) simt_chain64_kernel(PrefillProblem p, Workspace w) {
  constexpr int C = 64;
  constexpr int TPR = kThreads / C;  // threads per chunk row
  constexpr int VPT = RT / TPR;      // state rows per thread in the products
  constexpr int LD = kChainLd;       // padded row of the staged T and Aq (floats)
  constexpr int LDK = kChainRingLd;  // padded row of the staged feature slices
  constexpr int kStages = 3;
  constexpr int kSlice = C * LDK;    // floats of one staged 64-feature slice
  constexpr int D = 512, SD = kChainSd, kNsl = D / 64;
  constexpr int RPT = RT / 2;        // state rows per thread in the update (two row groups)
  constexpr int NT = RT / 8;         // 8-row tiles of the state in the tensor-core products
  static_assert(kThreads == 256 && RT % 8 == 0, "the products take 8 warps: 4 token tiles x 2 feature halves");
  extern __shared__ __align__(16) float sm[];
  float* S = sm;                              // [RT][SD]
  float* ring = S + RT * SD;                  // [kStages][K | Q][C][LDK]
  float* Tb = ring + kStages * 2 * kSlice;    // [2][T | Aq][C][LD]
  float* gb = Tb + 4 * C * LD;                // [2][C][4]
  float* Rs = gb + 2 * C * 4;                 // [C][RT]
  float* Es = Rs + C * RT;                    // [C][RT]

  const int vt = blockIdx.x;
  const int64_t n = blockIdx.y;
  const int tid = threadIdx.x;
  const int i = tid / TPR;
  const int v0 = (tid % TPR) * VPT;
  const bool a_tile = vt * RT < p.a_rows;
  const int row0 = a_tile ? vt * RT : vt * RT - p.a_rows;
  const bool readout = !a_tile && p.y != nullptr;  // uniform per CTA
  const int NC = w.NC;
  const int64_t items = int64_t(NC) * kNsl;

  for (int e = tid; e < RT * D; e += kThreads) {
    const int r = e / D, d = e % D;
    float s0 = 0.f;
    if (a_tile)
      s0 = (row0 + r == d) ? 1.f : 0.f;
    else if (p.S0)
      s0 = p.S0[(n * p.dv + row0 + r) * int64_t(D) + d];
    S[r * SD + d] = s0;
  }
  // item g: slice g % 8 of chunk g / 8 into stage g % 3 (and, for the first slice, the chunk's
  // T, Aq and gates into buffer c & 1); every call commits one group, possibly empty
  auto issue = [&](int64_t g) {
    if (g < items) {
      const int c = int(g / kNsl), s = int(g % kNsl);
      const int64_t rowbase = (n * w.Tp + int64_t(c) * C) * D + 64 * s;
      float* st = ring + int(g % kStages) * 2 * kSlice;
      for (int e = tid; e < C * 16; e += kThreads) {
        const int r = e >> 4, q = e & 15;
        tc::cp_async16(tc::smem_u32(st + r * LDK + 4 * q), w.phik + rowbase + int64_t(r) * D + 4 * q, 16);
        if (readout)
          tc::cp_async16(tc::smem_u32(st + kSlice + r * LDK + 4 * q), w.phiq + rowbase + int64_t(r) * D + 4 * q, 16);
      }
      if (s == 0) {
        const int64_t cm = (n * NC + c) * int64_t(C) * C;
        float* tb = Tb + (c & 1) * 2 * C * LD;
        for (int e = tid; e < C * 16; e += kThreads) {
          const int r = e >> 4, q = e & 15;
          tc::cp_async16(tc::smem_u32(tb + r * LD + 4 * q), w.Tinv + cm + r * C + 4 * q, 16);
          if (readout) tc::cp_async16(tc::smem_u32(tb + C * LD + r * LD + 4 * q), w.Aq + cm + r * C + 4 * q, 16);
        }
        const float* Gg = w.gates + (n * NC + c) * int64_t(C) * 4;
        for (int e = tid; e < C; e += kThreads) tc::cp_async16(tc::smem_u32(gb + (c & 1) * C * 4 + 4 * e), Gg + 4 * e, 16);
      }
    }
    tc::cp_async_commit();
  };
  for (int g = 0; g < kStages - 1; ++g) issue(g);
  __syncthreads();

  const int fb = tid % (D / 4);   // update: features 4 fb .. 4 fb + 3
  const int rb = tid / (D / 4);   //         rows RPT rb .. RPT rb + RPT - 1
  for (int c = 0; c < NC; ++c) {
    if (p.S_chunks && !a_tile) {  // checkpoint: the state entering chunk c
      float* Sc = p.S_chunks + ((n * NC + c) * p.dv + row0) * int64_t(D);
      for (int e = tid; e < RT * D; e += kThreads) Sc[e] = S[(e / D) * SD + e % D];
    }
    // X = K S^T, Yq = Q S^T (C x RT), slice by slice from the ring, on the tensor cores in split tf32:
    // warp w takes token rows 16 (w & 3) .. + 15 and the k-steps 4 (w >> 2) .. + 3 (8 features each) of
    // every slice; the two halves of the features meet in shared memory (Rs, Es are free until R and E).
    // A k-step's fragment slots t and t + 4 take the adjacent features 2t and 2t + 1 (the same order in
    // A and B, so the sum is unchanged): one 8-byte shared load per row, conflict-free with the padded
    // rows.  Two accumulators per product (even and odd k-steps) halve the dependent chain.
    {
      const int wq = tid >> 5, g8 = (tid & 31) >> 2, t4 = tid & 3;
      const int mrow = 16 * (wq & 3) + g8, kh = wq >> 2;
      float xa[2][NT][4], ya[2][NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) xa[h][nt][e] = ya[h][nt][e] = 0.f;
#pragma unroll 1
      for (int s = 0; s < kNsl; ++s) {
        const int64_t g = int64_t(c) * kNsl + s;
        tc::cp_async_wait_group<kStages - 2>();  // item g has landed (this thread's copies) ...
        __syncthreads();                         // ... everyone's; item g - 1's stage is free
        issue(g + kStages - 1);
        const float* Ks = ring + int(g % kStages) * 2 * kSlice;
        const float* Qs = Ks + kSlice;
        const float* Sd = S + 64 * s;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int kb = 8 * (4 * kh + kk) + 2 * t4;  // this lane's features kb, kb + 1 of the slice
          uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {  // B = S^T: state row 8 nt + g8
            const float2 s2 = *reinterpret_cast<const float2*>(Sd + (8 * nt + g8) * SD + kb);
            split_tf32(s2.x, bh[nt][0], bl[nt][0]);
            split_tf32(s2.y, bh[nt][1], bl[nt][1]);
          }
          uint32_t ah[4], al[4];
          {
            const float2 r0 = *reinterpret_cast<const float2*>(Ks + mrow * LDK + kb);
            const float2 r1 = *reinterpret_cast<const float2*>(Ks + (mrow + 8) * LDK + kb);
            split_tf32(r0.x, ah[0], al[0]);
            split_tf32(r1.x, ah[1], al[1]);
            split_tf32(r0.y, ah[2], al[2]);
            split_tf32(r1.y, ah[3], al[3]);
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_3xtf32(xa[kk & 1][nt], ah, al, bh[nt], bl[nt]);
          if (readout) {
            const float2 r0 = *reinterpret_cast<const float2*>(Qs + mrow * LDK + kb);
            const float2 r1 = *reinterpret_cast<const float2*>(Qs + (mrow + 8) * LDK + kb);
            split_tf32(r0.x, ah[0], al[0]);
            split_tf32(r1.x, ah[1], al[1]);
            split_tf32(r0.y, ah[2], al[2]);
            split_tf32(r1.y, ah[3], al[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) mma_3xtf32(ya[kk & 1][nt], ah, al, bh[nt], bl[nt]);
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          xa[0][nt][e] += xa[1][nt][e];
          ya[0][nt][e] += ya[1][nt][e];
        }
      // fragment element e of n-tile nt: token mrow + 8 (e >> 1), state row 8 nt + 2 t4 + (e & 1)
      if (kh == 1) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int o = (mrow + 8 * (e >> 1)) * RT + 8 * nt + 2 * t4 + (e & 1);
            Rs[o] = xa[0][nt][e];
            Es[o] = ya[0][nt][e];
          }
      }
      __syncthreads();
      if (kh == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int o = (mrow + 8 * (e >> 1)) * RT + 8 * nt + 2 * t4 + (e & 1);
            Rs[o] += xa[0][nt][e];
            Es[o] += ya[0][nt][e];
          }
      }
      __syncthreads();
    }
    float x[VPT], yq[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      x[u] = Rs[i * RT + v0 + u];
      yq[u] = Es[i * RT + v0 + u];
    }
    const float* Tm = Tb + (c & 1) * 2 * C * LD;
    const float* Am = Tm + C * LD;
    const float* gt = gb + (c & 1) * C * 4;
    // R_i = beta_i (v_i - exp(g_i) x_i)
    const int64_t t = int64_t(c) * C + i;
    const float beta_i = gt[4 * i + 3], gi = gt[4 * i + 1], gprev = gt[4 * i + 0], wi = gt[4 * i + 2];
    const float gC = gt[4 * (C - 1) + 1];
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      float vv = 0.f;
      if (!a_tile && t < p.T) vv = ld_as_f32(p.v, p.in_dtype, (n * p.T + t) * p.dv + row0 + v0 + u);
      Rs[i * RT + v0 + u] = beta_i * (vv - gi * x[u]);
    }
    __syncthreads();
    // E = T R over all 64 j (T is stored whole: unit diagonal, zeros above), four partial sums
    float e_[VPT];
    {
      float ep[4][VPT];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int u = 0; u < VPT; ++u) ep[a][u] = 0.f;
#pragma unroll 4
      for (int j = 0; j < C; j += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(Tm + i * LD + j);
        const float tv[4] = {t4.x, t4.y, t4.z, t4.w};
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int u = 0; u < VPT; ++u) ep[a][u] = fmaf(tv[a], Rs[(j + a) * RT + v0 + u], ep[a][u]);
      }
#pragma unroll
      for (int u = 0; u < VPT; ++u) e_[u] = (ep[0][u] + ep[1][u]) + (ep[2][u] + ep[3][u]);
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Es[i * RT + v0 + u] = e_[u];
    if (p.E_rows && !a_tile) {
#pragma unroll
      for (int u = 0; u < VPT; ++u) p.E_rows[(n * w.Tp + t) * p.dv + row0 + v0 + u] = e_[u];
    }
    __syncthreads();
    // y_i = exp(g_{i-1}) yq_i + sum_{j<i} Aq_ij e_j ;  then E''_i = exp(g_{C-1} - g_i) e_i into Rs
    if (readout) {  // Aq is strictly lower triangular as stored: all 64 j, four partial sums
      float yv[VPT];
      float yp[4][VPT];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int u = 0; u < VPT; ++u) yp[a][u] = 0.f;
#pragma unroll 4
      for (int j = 0; j < C; j += 4) {
        const float4 a4 = *reinterpret_cast<const float4*>(Am + i * LD + j);
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int u = 0; u < VPT; ++u) yp[a][u] = fmaf(av[a], Es[(j + a) * RT + v0 + u], yp[a][u]);
      }
#pragma unroll
      for (int u = 0; u < VPT; ++u) yv[u] = fmaf(gprev, yq[u], (yp[0][u] + yp[1][u]) + (yp[2][u] + yp[3][u]));
      if (t < p.T) {
#pragma unroll
        for (int u = 0; u < VPT; ++u) st_from_f32(p.y, p.y_dtype, (n * p.T + t) * p.dv + row0 + v0 + u, yv[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Rs[i * RT + v0 + u] = wi * e_[u];
    __syncthreads();
    // S <- exp(g_{C-1}) S + E''^T K: features 4 fb .. + 3, rows RPT rb .. + RPT - 1
    {
      const float* Kg = w.phik + (n * w.Tp + int64_t(c) * C) * D + 4 * fb;
      float acc[RPT][4];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const float4 s4 = *reinterpret_cast<const float4*>(S + (RPT * rb + r) * SD + 4 * fb);
        acc[r][0] = gC * s4.x, acc[r][1] = gC * s4.y, acc[r][2] = gC * s4.z, acc[r][3] = gC * s4.w;
      }
#pragma unroll
      for (int j0 = 0; j0 < C; j0 += 16) {
        float4 kv[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) kv[jj] = __ldcg(reinterpret_cast<const float4*>(Kg + int64_t(j0 + jj) * D));
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
#pragma unroll
          for (int r = 0; r < RPT; ++r) {
            const float ev = Rs[(j0 + jj) * RT + RPT * rb + r];
            acc[r][0] = fmaf(ev, kv[jj].x, acc[r][0]);
            acc[r][1] = fmaf(ev, kv[jj].y, acc[r][1]);
            acc[r][2] = fmaf(ev, kv[jj].z, acc[r][2]);
            acc[r][3] = fmaf(ev, kv[jj].w, acc[r][3]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RPT; ++r)
        *reinterpret_cast<float4*>(S + (RPT * rb + r) * SD + 4 * fb) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    }
    __syncthreads();
  }
  tc::cp_async_wait_all();

  float* dst = a_tile ? p.A_out + (n * p.a_rows + row0) * int64_t(D) : p.S_out + (n * p.dv + row0) * int64_t(D);
  for (int e = tid; e < RT * D; e += kThreads) {
    const int r = e / D, d = e % D;
    dst[int64_t(r) * D + d] = S[r * SD + d];
  }
}

template <int RT>
size_t chain64_smem_bytes() {
  return sizeof(float) *
         (size_t(RT) * kChainSd + 3 * 2 * 64 * kChainRingLd + 4 * 64 * kChainLd + 2 * 64 * 4 + 2 * 64 * RT);
}

// rows of S per chain CTA: 16, or 8 when 16-row tiles would leave SMs idle (few sequences), or 4
// (chunk 64) when 8-row tiles would too; the chains are latency-bound, so more CTAs -- on more SMs,
// then two per SM -- shorten them
int chain_rows(int64_t rows, int64_t N, int C) {
  const int sms = current_sm_count();
  if ((rows / 16) * N >= sms) return 16;
  return (C == 64 && (rows / 8) * N < sms) ? 4 : 8;
}

template <int C>
cudaError_t launch_c(const PrefillProblem& p, const Workspace& w, const ProjParams& P, cudaStream_t stream,
                     LaunchMarks& marks) {
  cudaError_t err;
  marks.begin(stream);
  {
    int64_t vecs = 2 * p.N * w.Tp;
    int64_t blocks = (vecs + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    simt_lift_kernel<<<unsigned(blocks), kThreads, 0, stream>>>(p, w, P);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    marks.after(stream);
  }
  {
    const size_t smem = prep_smem_bytes<C>();
    auto prep = (p.y || p.with_q) ? simt_prep_kernel<C, true> : simt_prep_kernel<C, false>;
    err = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    prep<<<dim3(w.NC, unsigned(p.N)), kThreads, smem, stream>>>(p, w);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    marks.after(stream);
  }
  if (C == 64 && p.D == 512) {  // pipelined pass: 16-row tiles when they fill the SMs, else 8
    const int rows = p.a_rows + p.dv;
    const bool r16 = (rows / 16) * p.N >= current_sm_count();
    const size_t smem = r16 ? chain64_smem_bytes<16>() : chain64_smem_bytes<8>();
    auto chain = r16 ? simt_chain64_kernel<16> : simt_chain64_kernel<8>;
    err = cudaFuncSetAttribute(chain, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    chain<<<dim3(rows / (r16 ? 16 : 8), unsigned(p.N)), kThreads, smem, stream>>>(p, w);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    marks.after(stream);
  } else {
    const int rt = chain_rows(p.a_rows + p.dv, p.N, C);
    const size_t smem = rt == 4   ? chain_smem_bytes<C, (C == 64 ? 4 : 8)>(p.D)
                        : rt == 8 ? chain_smem_bytes<C, 8>(p.D)
                                  : chain_smem_bytes<C, 16>(p.D);
    auto chain = rt == 4 ? simt_chain_kernel<C, (C == 64 ? 4 : 8)>
                 : rt == 8 ? simt_chain_kernel<C, 8>
                           : simt_chain_kernel<C, 16>;
    err = cudaFuncSetAttribute(chain, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    chain<<<dim3((p.a_rows + p.dv) / rt, unsigned(p.N)), kThreads, smem, stream>>>(p, w);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    marks.after(stream);
  }
  return cudaSuccess;
}

// ============================================================================ backward
//
// Gradient of the chunked prefill (the reference differentiates it by recompute + autograd,
// kernels/fused_kernel_deltanet.py:158-179).  With the chunk algebra of the file header
// (R_i the pseudo-value right-hand side, E = T R the new-value rows, P_ij = Aq_ij,
// Gs_i = exp(g_{i-1}), G_i = exp(g_i), Rg_i = exp(g_{C-1} - g_i)) and dY, dS_C the adjoints of the
// chunk's outputs and of the state leaving it, reverse-mode gives
//
//   dE_i  = Rg_i (dS_C k_i) + sum_{i'>i} P_{i'i} dY_{i'}          dR = T^T dE
//   dS_0  = G_{C-1} dS_C + sum_i (Gs_i dY_i q_i^T - beta_i G_i dR_i k_i^T)
//   dA_ij = -(dR_i . E_j)  (j < i)                                  (T = (I + A)^-1)
//   dq_i  = Gs_i (dY_i S_0) + sum_j Mq_ij k_j,   Mq_ij = (dY_i . E_j) exp(g_{i-1} - g_j)
//   dk_i  = sum_i' Mq_{i'i} q_i' - beta_i G_i (dR_i S_0) + Rg_i (E_i dS_C) + sum_j (Ab_ij + Ab_ji) k_j,
//           Ab_ij = dA_ij beta_i exp(g_i - g_j)
//   dv_i  = beta_i dR_i,   dbeta_i = dR_i . (v_i - G_i S_0 k_i) + sum_j dA_ij exp(g_i - g_j) k_i . k_j
//   d g_i collects every exp(g .) factor; d log decay_l = sum_{i >= l} d g_i (within the chunk),
//   zero where the decay is clamped (outside [1e-5, 1]).
// The feature gradients go back through the lift (lift_backward_kernel).  Passes: the forward
// chain with checkpoints (S entering each chunk, E rows), (B1) the reverse pass over chunks for
// dS (sequential, per tile of 8 or 16 rows), (B2) the per-chunk gradients (parallel), (B3) the lift.

// (B1) per (sequence, tile of RT rows of dS): chunks in reverse; stores dS_C of every chunk and dR
template <int C, int RT>
__global__ void __launch_bounds__(kThreads) simt_adjoint_kernel(BackwardProblem b, Workspace w,
                                                                float* __restrict__ dS_chunks,
                                                                float* __restrict__ dR_rows) {
  constexpr int TPR = kThreads / C;
  constexpr int VPT = RT / TPR;
  constexpr int LD = C + 1;
  const PrefillProblem& p = b.fwd;
  const int D = p.D;
  const int SD = D + 1;
  extern __shared__ float sm[];
  float* dS = sm;                    // [RT][SD]
  float* Ks = dS + RT * SD;    // [C][65]
  float* Tm = Ks + C * 65;           // [C][LD]
  float* Am = Tm + C * LD;           // [C][LD]
  float* gt = Am + C * LD;           // [C][4]
  float* Ys = gt + C * 4;            // [C][RT]: dY, then Gs_i dY_i
  float* Ws = Ys + C * RT;     // [C][RT]: dE, then beta_i G_i dR_i

  const int64_t n = blockIdx.y;
  const int tid = threadIdx.x;
  const int i = tid / TPR;
  const int v0 = (tid % TPR) * VPT;
  const int row0 = blockIdx.x * RT;

  for (int e = tid; e < RT * D; e += kThreads) {
    const int r = e / D, d = e % D;
    dS[r * SD + d] = b.dS_final ? b.dS_final[(n * p.dv + row0 + r) * int64_t(D) + d] : 0.f;
  }
  __syncthreads();

  for (int c = w.NC - 1; c >= 0; --c) {
    float* dSc = dS_chunks + ((n * w.NC + c) * p.dv + row0) * int64_t(D);
    for (int e = tid; e < RT * D; e += kThreads) dSc[e] = dS[(e / D) * SD + e % D];
    const float* Tg = w.Tinv + (n * w.NC + c) * int64_t(C) * C;
    const float* Ag = w.Aq + (n * w.NC + c) * int64_t(C) * C;
    const float* Gg = w.gates + (n * w.NC + c) * int64_t(C) * 4;
    for (int e = tid; e < C * C; e += kThreads) {
      Tm[(e / C) * LD + (e % C)] = Tg[e];
      Am[(e / C) * LD + (e % C)] = Ag[e];
    }
    for (int e = tid; e < C * 4; e += kThreads) gt[e] = Gg[e];

    // x_i = k_i . dS_v  (C x 16)
    const float* Kg = w.phik + (n * w.Tp + int64_t(c) * C) * D;
    const float* Qg = w.phiq + (n * w.Tp + int64_t(c) * C) * D;
    float x[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) x[u] = 0.f;
    for (int d0 = 0; d0 < D; d0 += 64) {
      __syncthreads();
      for (int e = tid; e < C * 64; e += kThreads) {
        const int r = e >> 6, cc = e & 63;
        Ks[r * 65 + cc] = Kg[int64_t(r) * D + d0 + cc];
      }
      __syncthreads();
#pragma unroll 4
      for (int dd = 0; dd < 64; ++dd) {
        const float kd = Ks[i * 65 + dd];
#pragma unroll
        for (int u = 0; u < VPT; ++u) x[u] = fmaf(kd, dS[(v0 + u) * SD + d0 + dd], x[u]);
      }
    }
    const int64_t t = int64_t(c) * C + i;
#pragma unroll
    for (int u = 0; u < VPT; ++u)
      Ys[i * RT + v0 + u] = t < p.T ? ld_as_f32(b.dy, b.dy_dtype, (n * p.T + t) * p.dv + row0 + v0 + u) : 0.f;
    __syncthreads();
    // dE_i = Rg_i x_i + sum_{i'>i} P_{i'i} dY_{i'}
    const float rg = gt[4 * i + 2];
    float de[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) de[u] = rg * x[u];
    for (int j = i + 1; j < C; ++j) {
      const float a = Am[j * LD + i];
#pragma unroll
      for (int u = 0; u < VPT; ++u) de[u] = fmaf(a, Ys[j * RT + v0 + u], de[u]);
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Ws[i * RT + v0 + u] = de[u];
    __syncthreads();
    // dR_i = dE_i + sum_{i'>i} T_{i'i} dE_{i'}
    float dr[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) dr[u] = de[u];
    for (int j = i + 1; j < C; ++j) {
      const float tj = Tm[j * LD + i];
#pragma unroll
      for (int u = 0; u < VPT; ++u) dr[u] = fmaf(tj, Ws[j * RT + v0 + u], dr[u]);
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) dR_rows[(n * w.Tp + t) * p.dv + row0 + v0 + u] = dr[u];
    __syncthreads();  // every read of dE and dY is done
    const float gprev = gt[4 * i + 0], gi = gt[4 * i + 1], beta_i = gt[4 * i + 3];
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      Ws[i * RT + v0 + u] = beta_i * gi * dr[u];
      Ys[i * RT + v0 + u] *= gprev;
    }
    __syncthreads();
    // dS <- G_{C-1} dS + sum_i (Gs_i dY_i q_i^T - beta_i G_i dR_i k_i^T)
    const float gC = gt[4 * (C - 1) + 1];
    for (int d = tid; d < D; d += kThreads) {
      float acc[RT];
#pragma unroll
      for (int r = 0; r < RT; ++r) acc[r] = gC * dS[r * SD + d];
      for (int j = 0; j < C; ++j) {
        const float kv = Kg[int64_t(j) * D + d], qv = Qg[int64_t(j) * D + d];
#pragma unroll
        for (int r = 0; r < RT; ++r)
          acc[r] = fmaf(Ys[j * RT + r], qv, fmaf(-Ws[j * RT + r], kv, acc[r]));
      }
#pragma unroll
      for (int r = 0; r < RT; ++r) dS[r * SD + d] = acc[r];
    }
    __syncthreads();
  }
  if (b.dS0) {
    for (int e = tid; e < RT * D; e += kThreads) {
      const int r = e / D, d = e % D;
      b.dS0[(n * p.dv + row0 + r) * int64_t(D) + d] = dS[r * SD + d];
    }
  }
}

// (B1) for chunk 64 and D = 512: the same reverse pass with the loads of `simt_chain64_kernel`: the
// chunk's K slices through a 3-stage cp.async ring for x = K dS^T, its T, Aq and gates into one of two
// buffers with its first slice, the triangular products over all 64 rows with four partial sums
// (T and Aq are stored whole, zeros where the sums skip), and the update reading K and Q rows from L2
// as float4, eight rows of each in flight, into a 4 features x RT/2 rows block per thread.
template <int RT>
__global__ void __launch_bounds__(kThreads, 1) simt_adjoint64_kernel(BackwardProblem b, Workspace w,
                                                                     float* __restrict__ dS_chunks,
                                                                     float* __restrict__ dR_rows) {
  constexpr int C = 64;
  constexpr int TPR = kThreads / C;
  constexpr int VPT = RT / TPR;
  constexpr int LD = kChainLd;
  constexpr int LDK = kChainRingLd;
  constexpr int kStages = 3;
  constexpr int kSlice = C * LDK;
  constexpr int D = 512, SD = kChainSd, kNsl = D / 64;
  constexpr int RPT = RT / 2;
  constexpr int NT = RT / 8;
  static_assert(kThreads == 256 && RT % 8 == 0, "the products take 8 warps: 4 token tiles x 2 feature halves");
  const PrefillProblem& p = b.fwd;
  extern __shared__ __align__(16) float sm[];
  float* dS = sm;                          // [RT][SD]
  float* ring = dS + RT * SD;              // [kStages][C][LDK] K slices
  float* Tb = ring + kStages * kSlice;     // [2][T | Aq][C][LD]
  float* gb = Tb + 4 * C * LD;             // [2][C][4]
  float* Ys = gb + 2 * C * 4;              // [C][RT]: dY, then Gs_i dY_i
  float* Ws = Ys + C * RT;                 // [C][RT]: dE, then beta_i G_i dR_i

  const int64_t n = blockIdx.y;
  const int tid = threadIdx.x;
  const int i = tid / TPR;
  const int v0 = (tid % TPR) * VPT;
  const int row0 = blockIdx.x * RT;
  const int NC = w.NC;
  const int64_t items = int64_t(NC) * kNsl;

  for (int e = tid; e < RT * D; e += kThreads) {
    const int r = e / D, d = e % D;
    dS[r * SD + d] = b.dS_final ? b.dS_final[(n * p.dv + row0 + r) * int64_t(D) + d] : 0.f;
  }
  // item g: slice g % 8 of chunk NC - 1 - g / 8 (chunks in reverse) into stage g % 3; the first slice
  // also brings the chunk's T, Aq and gates into buffer (g / 8) & 1
  auto issue = [&](int64_t g) {
    if (g < items) {
      const int ci = int(g / kNsl), s = int(g % kNsl), c = NC - 1 - ci;
      const int64_t rowbase = (n * w.Tp + int64_t(c) * C) * D + 64 * s;
      float* st = ring + int(g % kStages) * kSlice;
      for (int e = tid; e < C * 16; e += kThreads) {
        const int r = e >> 4, q = e & 15;
        tc::cp_async16(tc::smem_u32(st + r * LDK + 4 * q), w.phik + rowbase + int64_t(r) * D + 4 * q, 16);
      }
      if (s == 0) {
        const int64_t cm = (n * NC + c) * int64_t(C) * C;
        float* tb = Tb + (ci & 1) * 2 * C * LD;
        for (int e = tid; e < C * 16; e += kThreads) {
          const int r = e >> 4, q = e & 15;
          tc::cp_async16(tc::smem_u32(tb + r * LD + 4 * q), w.Tinv + cm + r * C + 4 * q, 16);
          tc::cp_async16(tc::smem_u32(tb + C * LD + r * LD + 4 * q), w.Aq + cm + r * C + 4 * q, 16);
        }
        const float* Gg = w.gates + (n * NC + c) * int64_t(C) * 4;
        for (int e = tid; e < C; e += kThreads) tc::cp_async16(tc::smem_u32(gb + (ci & 1) * C * 4 + 4 * e), Gg + 4 * e, 16);
      }
    }
    tc::cp_async_commit();
  };
  for (int g = 0; g < kStages - 1; ++g) issue(g);
  __syncthreads();

  const int fb = tid % (D / 4);
  const int rb = tid / (D / 4);
  for (int ci = 0; ci < NC; ++ci) {
    const int c = NC - 1 - ci;
    float* dSc = dS_chunks + ((n * NC + c) * p.dv + row0) * int64_t(D);
    for (int e = tid; e < RT * D; e += kThreads) dSc[e] = dS[(e / D) * SD + e % D];
    // x_i = k_i . dS_v  (C x RT), slice by slice from the ring, on the tensor cores in split tf32 with
    // the warp layout of simt_chain64_kernel's X; the two feature halves meet in Ws (free until dE)
    {
      const int wq = tid >> 5, g8 = (tid & 31) >> 2, t4 = tid & 3;
      const int mrow = 16 * (wq & 3) + g8, kh = wq >> 2;
      float xa[2][NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) xa[h][nt][e] = 0.f;
#pragma unroll 1
      for (int s = 0; s < kNsl; ++s) {
        const int64_t g = int64_t(ci) * kNsl + s;
        tc::cp_async_wait_group<kStages - 2>();
        __syncthreads();
        issue(g + kStages - 1);
        const float* Ks = ring + int(g % kStages) * kSlice;
        const float* Sd = dS + 64 * s;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int kb = 8 * (4 * kh + kk) + 2 * t4;
          uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float2 s2 = *reinterpret_cast<const float2*>(Sd + (8 * nt + g8) * SD + kb);
            split_tf32(s2.x, bh[nt][0], bl[nt][0]);
            split_tf32(s2.y, bh[nt][1], bl[nt][1]);
          }
          const float2 r0 = *reinterpret_cast<const float2*>(Ks + mrow * LDK + kb);
          const float2 r1 = *reinterpret_cast<const float2*>(Ks + (mrow + 8) * LDK + kb);
          uint32_t ah[4], al[4];
          split_tf32(r0.x, ah[0], al[0]);
          split_tf32(r1.x, ah[1], al[1]);
          split_tf32(r0.y, ah[2], al[2]);
          split_tf32(r1.y, ah[3], al[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma_3xtf32(xa[kk & 1][nt], ah, al, bh[nt], bl[nt]);
        }
      }
      if (kh == 1) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            Ws[(mrow + 8 * (e >> 1)) * RT + 8 * nt + 2 * t4 + (e & 1)] = xa[0][nt][e] + xa[1][nt][e];
      }
      __syncthreads();
      if (kh == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            Ws[(mrow + 8 * (e >> 1)) * RT + 8 * nt + 2 * t4 + (e & 1)] += xa[0][nt][e] + xa[1][nt][e];
      }
      __syncthreads();
    }
    float x[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) x[u] = Ws[i * RT + v0 + u];
    const float* Tm = Tb + (ci & 1) * 2 * C * LD;
    const float* Am = Tm + C * LD;
    const float* gt = gb + (ci & 1) * C * 4;
    const int64_t t = int64_t(c) * C + i;
#pragma unroll
    for (int u = 0; u < VPT; ++u)
      Ys[i * RT + v0 + u] = t < p.T ? ld_as_f32(b.dy, b.dy_dtype, (n * p.T + t) * p.dv + row0 + v0 + u) : 0.f;
    __syncthreads();
    // dE_i = Rg_i x_i + sum_j Aq_ji dY_j  (Aq_ji = 0 for j <= i)
    const float rg = gt[4 * i + 2];
    float de[VPT];
    {
      float dp[4][VPT];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int u = 0; u < VPT; ++u) dp[a][u] = 0.f;
#pragma unroll 4
      for (int j = 0; j < C; j += 4) {
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float aq = Am[(j + a) * LD + i];
#pragma unroll
          for (int u = 0; u < VPT; ++u) dp[a][u] = fmaf(aq, Ys[(j + a) * RT + v0 + u], dp[a][u]);
        }
      }
#pragma unroll
      for (int u = 0; u < VPT; ++u) de[u] = fmaf(rg, x[u], (dp[0][u] + dp[1][u]) + (dp[2][u] + dp[3][u]));
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Ws[i * RT + v0 + u] = de[u];
    __syncthreads();
    // dR_i = sum_j T_ji dE_j  (T_ii = 1, T_ji = 0 for j < i)
    float dr[VPT];
    {
      float dp[4][VPT];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int u = 0; u < VPT; ++u) dp[a][u] = 0.f;
#pragma unroll 4
      for (int j = 0; j < C; j += 4) {
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float tv = Tm[(j + a) * LD + i];
#pragma unroll
          for (int u = 0; u < VPT; ++u) dp[a][u] = fmaf(tv, Ws[(j + a) * RT + v0 + u], dp[a][u]);
        }
      }
#pragma unroll
      for (int u = 0; u < VPT; ++u) dr[u] = (dp[0][u] + dp[1][u]) + (dp[2][u] + dp[3][u]);
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) dR_rows[(n * w.Tp + t) * p.dv + row0 + v0 + u] = dr[u];
    const float gprev = gt[4 * i + 0], gi = gt[4 * i + 1], beta_i = gt[4 * i + 3];
    const float gC = gt[4 * (C - 1) + 1];
    __syncthreads();  // every read of dE and dY is done
#pragma unroll
    for (int u = 0; u < VPT; ++u) {
      Ws[i * RT + v0 + u] = beta_i * gi * dr[u];
      Ys[i * RT + v0 + u] *= gprev;
    }
    __syncthreads();
    // dS <- G_{C-1} dS + sum_j (Gs_j dY_j q_j^T - beta_j G_j dR_j k_j^T): features 4 fb.., rows RPT rb..
    {
      const int64_t base = (n * w.Tp + int64_t(c) * C) * D + 4 * fb;
      float acc[RPT][4];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const float4 s4 = *reinterpret_cast<const float4*>(dS + (RPT * rb + r) * SD + 4 * fb);
        acc[r][0] = gC * s4.x, acc[r][1] = gC * s4.y, acc[r][2] = gC * s4.z, acc[r][3] = gC * s4.w;
      }
#pragma unroll
      for (int j0 = 0; j0 < C; j0 += 8) {
        float4 kv[8], qv[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          kv[jj] = __ldcg(reinterpret_cast<const float4*>(w.phik + base + int64_t(j0 + jj) * D));
          qv[jj] = __ldcg(reinterpret_cast<const float4*>(w.phiq + base + int64_t(j0 + jj) * D));
        }
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
          for (int r = 0; r < RPT; ++r) {
            const float yv = Ys[(j0 + jj) * RT + RPT * rb + r], wv = -Ws[(j0 + jj) * RT + RPT * rb + r];
            acc[r][0] = fmaf(yv, qv[jj].x, fmaf(wv, kv[jj].x, acc[r][0]));
            acc[r][1] = fmaf(yv, qv[jj].y, fmaf(wv, kv[jj].y, acc[r][1]));
            acc[r][2] = fmaf(yv, qv[jj].z, fmaf(wv, kv[jj].z, acc[r][2]));
            acc[r][3] = fmaf(yv, qv[jj].w, fmaf(wv, kv[jj].w, acc[r][3]));
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RPT; ++r)
        *reinterpret_cast<float4*>(dS + (RPT * rb + r) * SD + 4 * fb) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    }
    __syncthreads();
  }
  tc::cp_async_wait_all();
  if (b.dS0) {
    for (int e = tid; e < RT * D; e += kThreads) {
      const int r = e / D, d = e % D;
      b.dS0[(n * p.dv + row0 + r) * int64_t(D) + d] = dS[r * SD + d];
    }
  }
}

template <int RT>
size_t adjoint64_smem_bytes() {
  return sizeof(float) * (size_t(RT) * kChainSd + 3 * 64 * kChainRingLd + 4 * 64 * kChainLd + 2 * 64 * 4 + 2 * 64 * RT);
}

// (B2) per (chunk, sequence): the gradients of the chunk's tokens.  The feature gradients
// overwrite the chunk's lifted features in the workspace (dq -> phiq rows, dk -> phik rows).
constexpr int kSlab = 32;

constexpr int kSlabLd = kSlab + 4;  // staged slab rows: 16-byte aligned for cp.async

// threads of the gradient kernel: 16 warps at C = 64 (the kernel is one CTA per SM, so the extra warps
// hide the shared-memory latency of its loops), 8 at C = 32
template <int C>
__host__ __device__ constexpr int grad_threads() {
  return C == 64 ? 512 : 256;
}

template <int C>
size_t grad_smem_bytes(int dv) {
  // rows, the two C x C matrices, two stages of [K | Q | S_0 | dS_C] slabs, the per-token vectors
  return sizeof(float) * (size_t(3) * C * (dv + 1) + 2 * C * (C + 1) + 2 * (2 * C + 2 * size_t(dv)) * kSlabLd +
                          9 * C + grad_threads<C>() / 32);
}

template <int C>
__global__ void __launch_bounds__(grad_threads<C>()) simt_grad_kernel(BackwardProblem b, Workspace w,
                                                             const float* __restrict__ dS_chunks,
                                                             const float* __restrict__ dR_rows) {
  constexpr int kGT = grad_threads<C>();
  constexpr int TJ = kGT / 16;          // the C x C products: 16 x TJ threads, each an RI x RJ tile
  constexpr int RI = C / 16, RJ = C / TJ;
  constexpr int LD = C + 1;
  constexpr int SL = kSlab + 1;
  constexpr int TPR2 = kGT / C;         // threads per token row in the slab phase
  constexpr int CPT = kSlab / TPR2;     // slab columns per thread
  const PrefillProblem& p = b.fwd;
  const int D = p.D, dv = p.dv, LV = dv + 1;
  extern __shared__ float sm[];
  float* Em = sm;                  // [C][LV] E rows
  float* Xm = Em + C * LV;         // [C][LV] dR rows
  float* Ym = Xm + C * LV;         // [C][LV] dY rows
  float* M1 = Ym + C * LV;         // [C][LD] Gram k.k, then Ab + Ab^T
  float* M2 = M1 + C * LD;         // [C][LD] Mq
  float* ring = M2 + C * LD;       // 2 stages of [K | Q | S_0 | dS_C] slabs, rows kSlabLd floats apart
  const int kStage = (2 * C + 2 * dv) * kSlabLd;
  float* Ks = ring;                // sweep 1: the K slab in stage 0, [C][SL]
  float* gl = ring + 2 * kStage;   // [C] g_i
  float* bt = gl + C;              // [C] beta_i
  float* lm = bt + C;              // [C] decay as given (1 past T)
  float* dg = lm + C;              // [C] d g_i
  float* dbA = dg + C;             // [C] the Gram part of d beta_i
  float* s1 = dbA + C;             // [C] dR_i . (S_0 k_i)
  float* s2 = s1 + C;              // [C] dY_i . (S_0 q_i)
  float* s3 = s2 + C;              // [C] E_i . (dS_C k_i)
  float* xv = s3 + C;              // [C] dR_i . v_i
  float* red = xv + C;             // [warps] <dS_C, S_0> partials

  const int c = blockIdx.x;
  const int64_t n = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t t0 = int64_t(c) * C;
  float* Kg = w.phik + (n * w.Tp + t0) * D;
  float* Qg = w.phiq + (n * w.Tp + t0) * D;
  const float* S0g = p.S_chunks + (n * w.NC + c) * int64_t(dv) * D;
  const float* dSg = dS_chunks + (n * w.NC + c) * int64_t(dv) * D;

  if (tid < 32) {  // gates in log space, as the prep pass forms them (pads: beta 0, decay 1)
    float gsum = 0.f;
    for (int base = 0; base < C; base += 32) {
      const int ii = base + lane;
      const int64_t t = t0 + ii;
      float dec = 1.f, be = 0.f;
      if (t < p.T) {
        dec = p.decay ? ld_as_f32(p.decay, p.gate_dtype, n * p.T + t) : 1.f;
        be = ld_as_f32(p.beta, p.gate_dtype, n * p.T + t);
      }
      float lg = logf(fminf(fmaxf(dec, 1e-5f), 1.0f));
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {  // inclusive scan over the warp
        const float y = __shfl_up_sync(0xffffffffu, lg, o);
        if (lane >= o) lg += y;
      }
      gl[ii] = gsum + lg;
      gsum += __shfl_sync(0xffffffffu, lg, 31);
      bt[ii] = be;
      lm[ii] = dec;
    }
  }
  for (int e = tid; e < C * dv; e += kGT) {
    const int ii = e / dv, v = e % dv;
    const int64_t t = t0 + ii;
    Em[ii * LV + v] = p.E_rows[(n * w.Tp + t) * dv + v];
    Xm[ii * LV + v] = dR_rows[(n * w.Tp + t) * dv + v];
    Ym[ii * LV + v] = t < p.T ? ld_as_f32(b.dy, b.dy_dtype, (n * p.T + t) * dv + v) : 0.f;
  }
  for (int e = tid; e < C; e += kGT) dg[e] = dbA[e] = s1[e] = s2[e] = s3[e] = 0.f;
  __syncthreads();

  // ---- sweep 1: Gram k.k and <dS_C, S_0>
  const int ti = tid / TJ, tj = tid % TJ;
  float gk[RI][RJ];
#pragma unroll
  for (int a = 0; a < RI; ++a)
#pragma unroll
    for (int q = 0; q < RJ; ++q) gk[a][q] = 0.f;
  float dss = 0.f;
  for (int d0 = 0; d0 < D; d0 += kSlab) {
    for (int e = tid; e < C * kSlab; e += kGT) {
      const int r = e / kSlab, cc = e % kSlab;
      Ks[r * SL + cc] = Kg[int64_t(r) * D + d0 + cc];
    }
    __syncthreads();
#pragma unroll 4
    for (int dd = 0; dd < kSlab; ++dd) {
      float ka[RI], kb[RJ];
#pragma unroll
      for (int a = 0; a < RI; ++a) ka[a] = Ks[(RI * ti + a) * SL + dd];
#pragma unroll
      for (int q = 0; q < RJ; ++q) kb[q] = Ks[(RJ * tj + q) * SL + dd];
#pragma unroll
      for (int a = 0; a < RI; ++a)
#pragma unroll
        for (int q = 0; q < RJ; ++q) gk[a][q] = fmaf(ka[a], kb[q], gk[a][q]);
    }
    __syncthreads();
  }

  // the slabs of sweep 2 through a 2-stage cp.async ring (slab m + 1 loads while slab m is used);
  // <dS_C, S_0> is taken from the staged slabs too
  const int nslab = D / kSlab;
  auto issue = [&](int m) {
    if (m < nslab) {
      float* st = ring + (m & 1) * kStage;
      const int dm = m * kSlab;
      constexpr int kq = kSlab / 4;  // 16-byte pieces per slab row
      for (int e = tid; e < (2 * C + 2 * dv) * kq; e += kGT) {
        const int r = e / kq, q4 = e % kq;
        const float* src = r < C       ? Kg + int64_t(r) * D
                           : r < 2 * C ? Qg + int64_t(r - C) * D
                           : r < 2 * C + dv ? S0g + int64_t(r - 2 * C) * D
                                            : dSg + int64_t(r - 2 * C - dv) * D;
        tc::cp_async16(tc::smem_u32(st + r * kSlabLd + 4 * q4), src + dm + 4 * q4, 16);
      }
    }
    tc::cp_async_commit();
  };
  issue(0);  // sweep 1 is over with stage 0 (its last barrier); slab 0 lands during the C x C phase

  // ---- C x C phase: dA, dY.E, the exp(g) factors, d g and d beta contributions
  float dA[RI][RJ], dP[RI][RJ];
#pragma unroll
  for (int a = 0; a < RI; ++a)
#pragma unroll
    for (int q = 0; q < RJ; ++q) dA[a][q] = dP[a][q] = 0.f;
  for (int v = 0; v < dv; ++v) {
    float xa[RI], ya[RI], eb[RJ];
#pragma unroll
    for (int a = 0; a < RI; ++a) {
      xa[a] = Xm[(RI * ti + a) * LV + v];
      ya[a] = Ym[(RI * ti + a) * LV + v];
    }
#pragma unroll
    for (int q = 0; q < RJ; ++q) eb[q] = Em[(RJ * tj + q) * LV + v];
#pragma unroll
    for (int a = 0; a < RI; ++a)
#pragma unroll
      for (int q = 0; q < RJ; ++q) {
        dA[a][q] = fmaf(-xa[a], eb[q], dA[a][q]);
        dP[a][q] = fmaf(ya[a], eb[q], dP[a][q]);
      }
  }
  const float* Pg = w.Aq + (n * w.NC + c) * int64_t(C) * C;
  float ab[RI][RJ], mq[RI][RJ];
#pragma unroll
  for (int a = 0; a < RI; ++a) {
    const int ii = RI * ti + a;
    float sg = 0.f, sb = 0.f, sp = 0.f;  // this row's d g_i, d beta_i and d g_{i-1} terms
#pragma unroll
    for (int q = 0; q < RJ; ++q) {
      const int jj = RJ * tj + q;
      ab[a][q] = mq[a][q] = 0.f;
      if (jj < ii) {
        const float eij = expf(gl[ii] - gl[jj]);
        const float aij = bt[ii] * eij * gk[a][q];
        const float ca = dA[a][q] * aij;              // d g through A
        const float cp = dP[a][q] * Pg[ii * C + jj];  // d g through P
        sg += ca;
        sb += dA[a][q] * eij * gk[a][q];
        sp += cp;
        atomicAdd(&dg[jj], -(ca + cp));
        mq[a][q] = dP[a][q] * expf(gl[ii - 1] - gl[jj]);
        ab[a][q] = dA[a][q] * bt[ii] * eij;
      }
    }
    // the TJ threads of a row group share row ii: one atomic each per group
#pragma unroll
    for (int o = TJ / 2; o > 0; o >>= 1) {
      sg += __shfl_xor_sync(0xffffffffu, sg, o);
      sb += __shfl_xor_sync(0xffffffffu, sb, o);
      sp += __shfl_xor_sync(0xffffffffu, sp, o);
    }
    if (tj == 0 && ii > 0) {
      atomicAdd(&dg[ii], sg);
      atomicAdd(&dbA[ii], sb);
      atomicAdd(&dg[ii - 1], sp);
    }
  }
#pragma unroll
  for (int a = 0; a < RI; ++a)
#pragma unroll
    for (int q = 0; q < RJ; ++q) {
      M1[(RI * ti + a) * LD + RJ * tj + q] = ab[a][q];
      M2[(RI * ti + a) * LD + RJ * tj + q] = mq[a][q];
    }
  __syncthreads();
  float sym[RI][RJ];
#pragma unroll
  for (int a = 0; a < RI; ++a)
#pragma unroll
    for (int q = 0; q < RJ; ++q) sym[a][q] = ab[a][q] + M1[(RJ * tj + q) * LD + RI * ti + a];
  __syncthreads();
#pragma unroll
  for (int a = 0; a < RI; ++a)
#pragma unroll
    for (int q = 0; q < RJ; ++q) M1[(RI * ti + a) * LD + RJ * tj + q] = sym[a][q];

  // ---- sweep 2: feature gradients, 32 columns at a time
  const int i = tid / TPR2;
  const int cb = (tid % TPR2) * CPT;
  const float Gs_i = i > 0 ? expf(gl[i - 1]) : 1.f;
  const float G_i = expf(gl[i]);
  const float Rg_i = expf(gl[C - 1] - gl[i]);
  const float bG = bt[i] * G_i;
  float p1 = 0.f, p2 = 0.f, p3 = 0.f;
  for (int m = 0; m < nslab; ++m) {
    const int d0 = m * kSlab;
    tc::cp_async_wait_group<0>();
    __syncthreads();  // slab m has landed everywhere; the stage of slab m - 1 is free
    issue(m + 1);
    const float* st = ring + (m & 1) * kStage;
    const float* Kst = st;
    const float* Qst = st + C * kSlabLd;
    const float* S0s = st + 2 * C * kSlabLd;
    const float* dSs = S0s + dv * kSlabLd;
    for (int e = tid; e < dv * kSlab; e += kGT) {
      const int r = e / kSlab, cc = e % kSlab;
      dss = fmaf(S0s[r * kSlabLd + cc], dSs[r * kSlabLd + cc], dss);
    }
    float yS[CPT], xS[CPT], wS[CPT], mK[CPT], mQ[CPT], aK[CPT];
#pragma unroll
    for (int q = 0; q < CPT; ++q) yS[q] = xS[q] = wS[q] = mK[q] = mQ[q] = aK[q] = 0.f;
    // the staged rows are read 16 bytes at a time (cb is a multiple of 4, rows are 16-byte aligned)
    auto row4 = [&](const float* rowp, float (&o)[CPT]) {
#pragma unroll
      for (int q = 0; q < CPT; q += 4) {
        const float4 f = *reinterpret_cast<const float4*>(rowp + cb + q);
        o[q] = f.x;
        o[q + 1] = f.y;
        o[q + 2] = f.z;
        o[q + 3] = f.w;
      }
    };
    for (int v = 0; v < dv; ++v) {
      const float yi = Ym[i * LV + v], xi = Xm[i * LV + v], ei = Em[i * LV + v];
      float s0[CPT], ds[CPT];
      row4(S0s + v * kSlabLd, s0);
      row4(dSs + v * kSlabLd, ds);
#pragma unroll
      for (int q = 0; q < CPT; ++q) {
        yS[q] = fmaf(yi, s0[q], yS[q]);
        xS[q] = fmaf(xi, s0[q], xS[q]);
        wS[q] = fmaf(ei, ds[q], wS[q]);
      }
    }
    for (int j = 0; j < C; ++j) {
      const float m_ij = M2[i * LD + j], m_ji = M2[j * LD + i], a_ij = M1[i * LD + j];
      float kj[CPT], qj[CPT];
      row4(Kst + j * kSlabLd, kj);
      row4(Qst + j * kSlabLd, qj);
#pragma unroll
      for (int q = 0; q < CPT; ++q) {
        mK[q] = fmaf(m_ij, kj[q], mK[q]);
        aK[q] = fmaf(a_ij, kj[q], aK[q]);
        mQ[q] = fmaf(m_ji, qj[q], mQ[q]);
      }
    }
    float oq[CPT], ok_[CPT], kr[CPT], qr[CPT];
    row4(Kst + i * kSlabLd, kr);
    row4(Qst + i * kSlabLd, qr);
#pragma unroll
    for (int q = 0; q < CPT; ++q) {
      const float ki = kr[q], qi = qr[q];
      p1 = fmaf(ki, xS[q], p1);
      p2 = fmaf(qi, yS[q], p2);
      p3 = fmaf(ki, wS[q], p3);
      oq[q] = fmaf(Gs_i, yS[q], mK[q]);
      ok_[q] = mQ[q] - bG * xS[q] + Rg_i * wS[q] + aK[q];
    }
    // the gradients overwrite this chunk's features (its slab is staged already), 16 bytes at a time
#pragma unroll
    for (int q = 0; q < CPT; q += 4) {
      *reinterpret_cast<float4*>(Qg + int64_t(i) * D + d0 + cb + q) = make_float4(oq[q], oq[q + 1], oq[q + 2], oq[q + 3]);
      *reinterpret_cast<float4*>(Kg + int64_t(i) * D + d0 + cb + q) =
          make_float4(ok_[q], ok_[q + 1], ok_[q + 2], ok_[q + 3]);
    }
  }
  tc::cp_async_wait_all();
  dss = warp_sum(dss);
  if (lane == 0) red[warp] = dss;
#pragma unroll
  for (int o = TPR2 / 2; o > 0; o >>= 1) {
    p1 += __shfl_xor_sync(0xffffffffu, p1, o);
    p2 += __shfl_xor_sync(0xffffffffu, p2, o);
    p3 += __shfl_xor_sync(0xffffffffu, p3, o);
  }
  if (tid % TPR2 == 0) {
    s1[i] = p1;
    s2[i] = p2;
    s3[i] = p3;
  }
  if (tid < C) {
    float acc = 0.f;
    for (int v = 0; v < dv; ++v) {
      const int64_t t = t0 + tid;
      const float vv = t < p.T ? ld_as_f32(p.v, p.in_dtype, (n * p.T + t) * dv + v) : 0.f;
      acc = fmaf(Xm[tid * LV + v], vv, acc);
    }
    xv[tid] = acc;
  }
  __syncthreads();
  if (tid < C) {  // per-token d g terms
    const int ii = tid;
    const float e_i = expf(gl[C - 1] - gl[ii]) * s3[ii];
    atomicAdd(&dg[C - 1], e_i);
    atomicAdd(&dg[ii], -e_i - bt[ii] * expf(gl[ii]) * s1[ii]);
    if (ii > 0) atomicAdd(&dg[ii - 1], expf(gl[ii - 1]) * s2[ii]);
    if (ii == C - 1) {
      float tot = 0.f;
      for (int q = 0; q < kGT / 32; ++q) tot += red[q];
      atomicAdd(&dg[C - 1], expf(gl[C - 1]) * tot);
    }
  }
  __syncthreads();
  if (tid < C) {
    const int ii = tid;
    const int64_t t = t0 + ii;
    if (t < p.T) {
      float dlog = 0.f;
      for (int q = ii; q < C; ++q) dlog += dg[q];
      b.dbeta[n * p.T + t] = xv[ii] - expf(gl[ii]) * s1[ii] + dbA[ii];
      if (b.ddecay) {
        const float dec = lm[ii];
        b.ddecay[n * p.T + t] = (dec >= 1e-5f && dec <= 1.0f) ? dlog / dec : 0.f;
      }
    }
  }
  for (int e = tid; e < C * dv; e += kGT) {
    const int ii = e / dv, v = e % dv;
    const int64_t t = t0 + ii;
    if (t < p.T) b.dv_out[(n * p.T + t) * dv + v] = bt[ii] * Xm[ii * LV + v];
  }
}

// transpose of structured_block: x = D1 H D2 H D3 H y / 8 (per-lane pairs, as the forward)
__device__ __forceinline__ void structured_block_t(float y0, float y1, const uint64_t (&bits)[3], int lane,
                                                   float& x0, float& x1) {
  float v0 = y0, v1 = y1;
  fwht64(v0, v1, lane);
  apply_signs(v0, v1, bits[2], lane);
  fwht64(v0, v1, lane);
  apply_signs(v0, v1, bits[1], lane);
  fwht64(v0, v1, lane);
  apply_signs(v0, v1, bits[0], lane);
  x0 = v0 * 0.125f;
  x1 = v1 * 0.125f;
}

// (B3) one warp per token row of q or k: dx = tau_inv Omega^T dz with
// dz = -amp sin(z) (dphi / e - u (u . dphi) / (|u| e^2)),  e = |u| + 1e-8
__global__ void __launch_bounds__(kThreads) lift_backward_kernel(BackwardProblem b, Workspace w, ProjParams P) {
  const PrefillProblem& p = b.fwd;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t rows = p.N * p.T;
  const int D = p.D;
  for (int64_t r = warp; r < 2 * rows; r += nwarps) {
    const bool isq = r >= rows;
    const int64_t row = isq ? r - rows : r;
    const int64_t n = row / p.T, t = row % p.T;
    const float2 xv = ld2_as_f32(isq ? p.q : p.k, p.in_dtype, row * kDk + 2 * lane);
    const float* g = (isq ? w.phiq : w.phik) + (n * w.Tp + t) * D;
    float sn[kMaxBlocks][2], u[kMaxBlocks][2], gg[kMaxBlocks][2];  // sin z, amp cos z, the incoming gradient
    float ss = 0.f, ug = 0.f;
#pragma unroll
    for (int m = 0; m < kMaxBlocks; ++m) {
      sn[m][0] = sn[m][1] = u[m][0] = u[m][1] = gg[m][0] = gg[m][1] = 0.f;
      if (m < P.M) {
        float a0, a1;
        structured_block(xv.x, xv.y, P.sign_bits[m], lane, a0, a1);
        const int f = 64 * m + 2 * lane;
        const float2 ph = *reinterpret_cast<const float2*>(P.phase + f);
        float c0, c1;  // one range reduction for the sine and the cosine of each argument
        sincosf(fmaf(a0, P.tau_inv, ph.x), &sn[m][0], &c0);
        sincosf(fmaf(a1, P.tau_inv, ph.y), &sn[m][1], &c1);
        u[m][0] = P.amp * c0;
        u[m][1] = P.amp * c1;
        const float2 gv = *reinterpret_cast<const float2*>(g + f);
        gg[m][0] = gv.x;
        gg[m][1] = gv.y;
        ss = fmaf(u[m][0], u[m][0], fmaf(u[m][1], u[m][1], ss));
        ug = fmaf(u[m][0], gv.x, fmaf(u[m][1], gv.y, ug));
      }
    }
    ss = warp_sum(ss);
    ug = warp_sum(ug);
    const float nrm = sqrtf(ss);
    const float e = nrm + 1e-8f;
    const float c1 = 1.f / e, c2 = ug / (fmaxf(nrm, 1e-30f) * e * e);
    float dx0 = 0.f, dx1 = 0.f;
#pragma unroll
    for (int m = 0; m < kMaxBlocks; ++m) {
      if (m < P.M) {
        const float dz0 = -(gg[m][0] * c1 - u[m][0] * c2) * P.amp * sn[m][0];
        const float dz1 = -(gg[m][1] * c1 - u[m][1] * c2) * P.amp * sn[m][1];
        float a0, a1;
        structured_block_t(dz0, dz1, P.sign_bits[m], lane, a0, a1);
        dx0 += a0;
        dx1 += a1;
      }
    }
    float* dst = (isq ? b.dq : b.dk) + row * kDk + 2 * lane;
    dst[0] = dx0 * P.tau_inv;
    dst[1] = dx1 * P.tau_inv;
  }
}

template <int C, int RT>
size_t adjoint_smem_bytes(int D) {
  return sizeof(float) * (size_t(RT) * (D + 1) + C * 65 + 2 * C * (C + 1) + 4 * C + 2 * C * RT);
}

struct BackwardExtra {
  float* S_chunks;
  float* dS_chunks;
  float* E_rows;
  float* dR_rows;
  float* S_scratch;
};

BackwardExtra carve_backward(void* base, int64_t N, int64_t T, int dv, int C, int D, size_t* total) {
  size_t off = 0;
  Workspace w = carve(base, N, T, dv, C, D, &off);
  char* bp = static_cast<char*>(base);
  auto take = [&](size_t bytes) {
    char* q = bp ? bp + off : nullptr;
    off = align256(off + bytes);
    return reinterpret_cast<float*>(q);
  };
  BackwardExtra x;
  x.S_chunks = take(sizeof(float) * size_t(N) * w.NC * dv * D);
  x.dS_chunks = take(sizeof(float) * size_t(N) * w.NC * dv * D);
  x.E_rows = take(sizeof(float) * size_t(N) * w.Tp * dv);
  x.dR_rows = take(sizeof(float) * size_t(N) * w.Tp * dv);
  x.S_scratch = take(sizeof(float) * size_t(N) * dv * D);
  if (total) *total = off;
  return x;
}

template <int C>
cudaError_t launch_backward_c(BackwardProblem b, const Workspace& w, const BackwardExtra& x, const ProjParams& P,
                              cudaStream_t stream) {
  LaunchMarks none;
  b.fwd.y = nullptr;
  b.fwd.with_q = true;
  b.fwd.S_chunks = x.S_chunks;
  b.fwd.E_rows = x.E_rows;
  b.fwd.S_out = x.S_scratch;
  b.fwd.a_rows = 0;
  b.fwd.A_out = nullptr;
  cudaError_t err = launch_c<C>(b.fwd, w, P, stream, none);  // lift, prep, chain with checkpoints
  if (err != cudaSuccess) return err;
  if (C == 64 && b.fwd.D == 512) {  // pipelined reverse pass
    const bool r16 = chain_rows(b.fwd.dv, b.fwd.N, C) == 16;
    const size_t smem = r16 ? adjoint64_smem_bytes<16>() : adjoint64_smem_bytes<8>();
    auto adjoint = r16 ? simt_adjoint64_kernel<16> : simt_adjoint64_kernel<8>;
    err = cudaFuncSetAttribute(adjoint, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    adjoint<<<dim3(b.fwd.dv / (r16 ? 16 : 8), unsigned(b.fwd.N)), kThreads, smem, stream>>>(b, w, x.dS_chunks,
                                                                                            x.dR_rows);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  } else {
    // tiles of at least 8 rows here: the adjoint loads K and Q per chunk, and 4-row tiles measured slower
    const int rt = chain_rows(b.fwd.dv, b.fwd.N, C) == 16 ? 16 : 8;
    const size_t smem = rt == 8 ? adjoint_smem_bytes<C, 8>(b.fwd.D) : adjoint_smem_bytes<C, 16>(b.fwd.D);
    auto adjoint = rt == 8 ? simt_adjoint_kernel<C, 8> : simt_adjoint_kernel<C, 16>;
    err = cudaFuncSetAttribute(adjoint, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    adjoint<<<dim3(b.fwd.dv / rt, unsigned(b.fwd.N)), kThreads, smem, stream>>>(b, w, x.dS_chunks, x.dR_rows);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  {
    const size_t smem = grad_smem_bytes<C>(b.fwd.dv);
    err = cudaFuncSetAttribute(simt_grad_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    simt_grad_kernel<C><<<dim3(w.NC, unsigned(b.fwd.N)), grad_threads<C>(), smem, stream>>>(b, w, x.dS_chunks,
                                                                                          x.dR_rows);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  {
    int64_t blocks = (2 * b.fwd.N * b.fwd.T + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    if (blocks < 1) blocks = 1;
    lift_backward_kernel<<<unsigned(blocks), kThreads, 0, stream>>>(b, w, P);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
  }
  return cudaSuccess;
}

}  // namespace

size_t simt_prefill_workspace(int64_t N, int64_t T, int dv, int C, int D) {
  size_t total = 0;
  carve(nullptr, N, T, dv, C, D, &total);
  return total;
}

cudaError_t launch_simt_prefill(const PrefillProblem& p, const ProjParams& P, void* ws, size_t ws_bytes,
                                cudaStream_t stream, LaunchMarks& marks) {
  size_t need = 0;
  Workspace w = carve(ws, p.N, p.T, p.dv, p.C, p.D, &need);
  if (ws_bytes < need) return cudaErrorInvalidValue;
  if (p.C == 64) return launch_c<64>(p, w, P, stream, marks);
  return launch_c<32>(p, w, P, stream, marks);
}

size_t simt_backward_workspace(int64_t N, int64_t T, int dv, int C, int D) {
  size_t total = 0;
  carve_backward(nullptr, N, T, dv, C, D, &total);
  return total;
}

cudaError_t launch_simt_backward(const BackwardProblem& b, const ProjParams& P, void* ws, size_t ws_bytes,
                                 cudaStream_t stream) {
  size_t need = 0;
  BackwardExtra x = carve_backward(ws, b.fwd.N, b.fwd.T, b.fwd.dv, b.fwd.C, b.fwd.D, &need);
  if (ws_bytes < need) return cudaErrorInvalidValue;
  Workspace w = carve(ws, b.fwd.N, b.fwd.T, b.fwd.dv, b.fwd.C, b.fwd.D, nullptr);
  if (b.fwd.C == 64) return launch_backward_c<64>(b, w, x, P, stream);
  return launch_backward_c<32>(b, w, x, P, stream);
}

}  // namespace kdn
