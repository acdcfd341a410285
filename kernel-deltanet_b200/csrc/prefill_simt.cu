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
// 16-row tile of S): the serial pass over chunks.
#include <math.h>

#include "kdn_internal.h"
#include "lift.cuh"

namespace kdn {
namespace {

constexpr int kThreads = 256;
constexpr int kRowTile = 16;  // rows of S per chain CTA

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
  const int64_t total = p.y ? 2 * rows : rows;
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

// (2) per (chunk c, sequence n): G = K K^T, P = Q K^T, gates, T = (I + A)^-1, Aq.
// kQ = false (no readout): P and Aq are skipped (Aq is written as zeros).
template <int C, bool kQ>
__global__ void __launch_bounds__(kThreads) simt_prep_kernel(PrefillProblem p, Workspace w) {
  constexpr int R = C / 16;  // each thread owns an R x R tile of G and of P
  constexpr int LD = C + 1;
  extern __shared__ float sm[];
  float* Ks = sm;            // [C][65]
  float* Qs = Ks + C * 65;   // [C][65]
  float* G = Qs + C * 65;    // [C][LD], becomes A
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
      Ks[r * 65 + cc] = Kg[int64_t(r) * D + d0 + cc];
      if (kQ) Qs[r * 65 + cc] = Qg[int64_t(r) * D + d0 + cc];
    }
    __syncthreads();
#pragma unroll 4
    for (int dd = 0; dd < 64; ++dd) {
      float a[R], qq[R], b[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        a[r] = Ks[(ti * R + r) * 65 + dd];
        qq[r] = kQ ? Qs[(ti * R + r) * 65 + dd] : 0.f;
        b[r] = Ks[(tj * R + r) * 65 + dd];
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
  // forward substitution, row by row: T_ij = -sum_{l=j}^{i-1} A_il T_lj  (j < i)
  for (int i = 1; i < C; ++i) {
    if (tid < i) {
      const int j = tid;
      float s = 0.f;
      for (int l = j; l < i; ++l) s = fmaf(G[i * LD + l], Tm[l * LD + j], s);
      Tm[i * LD + j] = -s;
    }
    __syncthreads();
  }

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
  return sizeof(float) * (2 * C * 65 + 3 * C * (C + 1) + 2 * C);
}

// (3) per (16-row tile of S, sequence n): the serial pass over chunks.  Tiles below
// p.a_rows belong to the block transition's homogeneous map (identity start, v = 0,
// no readout, result to A_out); the others are value rows (S0, v, y, S_out).
template <int C>
__global__ void __launch_bounds__(kThreads) simt_chain_kernel(PrefillProblem p, Workspace w) {
  constexpr int TPR = kThreads / C;    // threads per chunk row
  constexpr int VPT = kRowTile / TPR;  // state rows per thread in the (C x 16) phases
  constexpr int LD = C + 1;
  const int D = p.D;
  const int SD = D + 1;  // padded row stride of the S tile
  extern __shared__ float sm[];
  float* S = sm;                     // [16][SD]
  float* Ks = S + kRowTile * SD;     // [C][65]
  float* Qs = Ks + C * 65;           // [C][65]
  float* Tm = Qs + C * 65;           // [C][LD]
  float* Am = Tm + C * LD;           // [C][LD]
  float* gt = Am + C * LD;           // [C][4]
  float* Rs = gt + C * 4;            // [C][16]
  float* Es = Rs + C * kRowTile;     // [C][16]

  const int vt = blockIdx.x;
  const int64_t n = blockIdx.y;
  const int tid = threadIdx.x;
  const int i = tid / TPR;
  const int v0 = (tid % TPR) * VPT;
  const bool a_tile = vt * kRowTile < p.a_rows;
  const int row0 = a_tile ? vt * kRowTile : vt * kRowTile - p.a_rows;
  const bool readout = !a_tile && p.y != nullptr;  // uniform per CTA

  for (int e = tid; e < kRowTile * D; e += kThreads) {
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
      Rs[i * kRowTile + v0 + u] = beta_i * (vv - gi * x[u]);
    }
    __syncthreads();
    // E = T R  (T unit lower triangular)
    float e_[VPT];
#pragma unroll
    for (int u = 0; u < VPT; ++u) e_[u] = Rs[i * kRowTile + v0 + u];
    for (int j = 0; j < i; ++j) {
      const float tij = Tm[i * LD + j];
#pragma unroll
      for (int u = 0; u < VPT; ++u) e_[u] = fmaf(tij, Rs[j * kRowTile + v0 + u], e_[u]);
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Es[i * kRowTile + v0 + u] = e_[u];
    __syncthreads();
    // y_i = exp(g_{i-1}) yq_i + sum_{j<i} Aq_ij e_j ;  then E''_i = exp(g_{C-1} - g_i) e_i into Rs
    if (readout) {
      float yv[VPT];
#pragma unroll
      for (int u = 0; u < VPT; ++u) yv[u] = gprev * yq[u];
      for (int j = 0; j < i; ++j) {
        const float aij = Am[i * LD + j];
#pragma unroll
        for (int u = 0; u < VPT; ++u) yv[u] = fmaf(aij, Es[j * kRowTile + v0 + u], yv[u]);
      }
      if (t < p.T) {
#pragma unroll
        for (int u = 0; u < VPT; ++u) st_from_f32(p.y, p.y_dtype, (n * p.T + t) * p.dv + row0 + v0 + u, yv[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < VPT; ++u) Rs[i * kRowTile + v0 + u] = wi * e_[u];
    __syncthreads();
    // S <- exp(g_{C-1}) S + E''^T K
    const float gC = gt[4 * (C - 1) + 1];
    for (int d = tid; d < D; d += kThreads) {
      float acc[kRowTile];
#pragma unroll
      for (int r = 0; r < kRowTile; ++r) acc[r] = gC * S[r * SD + d];
      for (int j = 0; j < C; ++j) {
        const float kv = Kg[int64_t(j) * D + d];
#pragma unroll
        for (int r = 0; r < kRowTile; ++r) acc[r] = fmaf(Rs[j * kRowTile + r], kv, acc[r]);
      }
#pragma unroll
      for (int r = 0; r < kRowTile; ++r) S[r * SD + d] = acc[r];
    }
    __syncthreads();
  }

  float* dst = a_tile ? p.A_out + (n * p.a_rows + row0) * int64_t(D) : p.S_out + (n * p.dv + row0) * int64_t(D);
  for (int e = tid; e < kRowTile * D; e += kThreads) {
    const int r = e / D, d = e % D;
    dst[int64_t(r) * D + d] = S[r * SD + d];
  }
}

template <int C>
size_t chain_smem_bytes(int D) {
  return sizeof(float) * (size_t(kRowTile) * (D + 1) + 2 * C * 65 + 2 * C * (C + 1) + 4 * C + 2 * C * kRowTile);
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
    auto prep = p.y ? simt_prep_kernel<C, true> : simt_prep_kernel<C, false>;
    err = cudaFuncSetAttribute(prep, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    prep<<<dim3(w.NC, unsigned(p.N)), kThreads, smem, stream>>>(p, w);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    marks.after(stream);
  }
  {
    const size_t smem = chain_smem_bytes<C>(p.D);
    err = cudaFuncSetAttribute(simt_chain_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (err != cudaSuccess) return err;
    simt_chain_kernel<C><<<dim3((p.a_rows + p.dv) / kRowTile, unsigned(p.N)), kThreads, smem, stream>>>(p, w);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    marks.after(stream);
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

}  // namespace kdn
