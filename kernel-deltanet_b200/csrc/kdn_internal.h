// kdn_internal.h -- host-side declarations shared by libkdn's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "kdn.h"
#include "kdn_common.cuh"

namespace kdn {

// Multiprocessor count of the current device, looked up once per device and cached in a
// table of atomics (safe when several host threads drive several devices); 148 if the
// lookup fails.
int current_sm_count();

// ------------------------------------------------------------------ lift.cu
cudaError_t launch_lift(const void* x, int x_dtype, void* out, int out_dtype, int64_t n, const ProjParams& P,
                        bool omega_bf16_exact, cudaStream_t stream);
cudaError_t lift_read_error(cudaStream_t stream, int* code);

// ------------------------------------------------------------ prefill paths
struct PrefillProblem {
  const void* q;
  const void* k;
  const void* v;
  int in_dtype;
  const void* beta;
  const void* decay;  // may be null (== 1)
  int gate_dtype;
  const float* S0;  // may be null (zeros)
  void* y;          // may be null on the CUDA-core path (no readout: q is not lifted)
  int y_dtype;
  float* S_out;
  int64_t N, T;
  int dv, C, D;
  // Block transition (CUDA-core path only): a_rows extra state rows, started at the
  // identity and driven with v = 0, run ahead of the dv value rows; after the pass they
  // hold the homogeneous part A of the block's affine map, written to A_out [N, a_rows, D].
  int a_rows = 0;
  float* A_out = nullptr;
  // Backward recompute (CUDA-core path): lift and pair q even without a readout, and keep
  // the state entering every chunk, S_chunks [N, NC, dv, D], and the chunk-local new-value
  // rows e_i, E_rows [N, NC * C, dv].
  bool with_q = false;
  float* S_chunks = nullptr;
  float* E_rows = nullptr;
  // Varlen batch (fused tensor-core path only): see TcArgs::var_off
  const int64_t* var_off = nullptr;
  const int64_t* var_len = nullptr;
  int64_t var_rows = 0;
};

// Per-launch event marks of one prefill call (measurement hook behind
// kdn_set_prefill_events): ev[0] is recorded before the first launch and ev[i] after
// launch i while i < cap; `launches` counts the kernels the call launched.
struct LaunchMarks {
  cudaEvent_t* ev = nullptr;
  int cap = 0;
  int launches = 0;
  void begin(cudaStream_t s) {
    launches = 0;
    if (cap > 0) cudaEventRecord(ev[0], s);
  }
  void after(cudaStream_t s) {
    ++launches;
    if (launches < cap) cudaEventRecord(ev[launches], s);
  }
};

// prefill_simt.cu: exact fp32 arithmetic on CUDA cores, three launches over a workspace.
size_t simt_prefill_workspace(int64_t N, int64_t T, int dv, int C, int D);
// Backward of the chunked prefill (exact fp32; forward recompute with checkpoints, reverse
// adjoint pass over chunks, per-chunk gradients, lift backward).  Outputs fp32.
struct BackwardProblem {
  PrefillProblem fwd;     // q, k, v, beta, decay, S0, N, T, dv, C, D (y unused)
  const void* dy;         // [N, T, dv]
  int dy_dtype;
  const float* dS_final;  // [N, dv, D] or null (zero)
  float* dq;              // [N, T, d_k]
  float* dk;
  float* dv_out;          // [N, T, dv]
  float* dbeta;           // [N, T]
  float* ddecay;          // [N, T] or null
  float* dS0;             // [N, dv, D] or null
  const float* omega;     // unused (the lift is differentiated through its butterfly)
};
size_t simt_backward_workspace(int64_t N, int64_t T, int dv, int C, int D);
cudaError_t launch_simt_backward(const BackwardProblem& b, const ProjParams& P, void* ws, size_t ws_bytes,
                                 cudaStream_t stream);
cudaError_t launch_simt_prefill(const PrefillProblem& p, const ProjParams& P, void* ws, size_t ws_bytes,
                                cudaStream_t stream, LaunchMarks& marks);

// prefill_static.cu: device address of the library's fixed prefill scratch
// (KDN_STATIC_SCRATCH_BYTES) on the current device, looked up on first use and again
// whenever the device's current context has changed (after a device reset).
cudaError_t static_prefill_scratch(void** out);

// prefill_tc.cu: fused tensor-core path (bf16 operands, fp32 accumulation/state),
// one CTA per sequence; needs D=512, dv=64, C=64 and Omega exact in bf16.
bool tc_prefill_supported(int D, int dv, int C, const ProjParams& P);
cudaError_t launch_tc_prefill(const PrefillProblem& p, const ProjParams& P, cudaStream_t stream, LaunchMarks& marks);
cudaError_t tc_read_error(cudaStream_t stream, int* code);

// prefill_split.cu: the same arithmetic in two phases for few, long sequences -- a
// chunk-parallel preparation pass writing one record per chunk to the workspace, then
// a serial state pass per sequence.  Same shape requirements as the fused path.
size_t split_prefill_workspace(int64_t N, int64_t T);
cudaError_t launch_split_prefill(const PrefillProblem& p, const ProjParams& P, void* ws, size_t ws_bytes,
                                 cudaStream_t stream, LaunchMarks& marks);
cudaError_t split_read_error(cudaStream_t stream, int* code);

// ---------------------------------------------------------------- affine.cu
// (A1,B1) o (A2,B2) = (A1 A2, B1 A2 + B2), batched; A_out or B_out may be null (not computed).
cudaError_t launch_affine_compose(const float* A1, const float* B1, const float* A2, const float* B2, float* A_out,
                                  float* B_out, int64_t batch, int D, int dv, cudaStream_t stream);
// A [batch, D, D] = identity
cudaError_t launch_affine_identity(float* A, int64_t batch, int D, cudaStream_t stream);
// states[0] = S0 (zeros if null), states[c+1] = states[c] A_c + B_c; final = states[n_c-1] A + B.
cudaError_t launch_affine_prefix_states(const float* A, const float* B, const float* S0, float* states,
                                        float* final_state, int64_t n_c, int64_t batch, int D, int dv,
                                        cudaStream_t stream);

// ---------------------------------------------------------------- tp_proj.cu
// out (+)= Y W^T across ranks: stores into `out`, or adds into every rank's copy through the
// multicast address `out_mc` when given.  N % 256 == 0, K % 64 == 0.
cudaError_t launch_tp_proj(const void* Y, const void* W, void* out, bool out_bf16, float* out_mc, int64_t M, int N,
                           int K, cudaStream_t stream);
// two-phase form: tiles stored into `out` (this rank's copy) and announced on the tile counters;
// the owner (tile % world == rank) reduces each tile once every counter reaches `target`.
cudaError_t launch_tp_proj_reduce(const void* Y, const void* W, void* out, void* out_mc, bool out_bf16,
                                  uint32_t* flags, uint32_t* flags_mc, uint32_t target, int rank, int world, int64_t M,
                                  int N, int K, cudaStream_t stream);
// peer form: every rank's copies of the output and the counters by their peer pointers (world <= 8)
cudaError_t launch_tp_proj_reduce_peer(const void* Y, const void* W, void* const* outs, bool out_bf16,
                                       uint32_t* const* flags, uint32_t target, int rank, int world, int64_t M, int N,
                                       int K, cudaStream_t stream);
int tp_proj_max_world();
int64_t tp_proj_tiles(int64_t M, int N);
// y = x w^T of one rank (store form, any N >= 1, output row stride ldo): the TMA-fed tcgen05 GEMM.
// swiglu: w holds gate/up row blocks of 128 interleaved (N = 2 d_ff, d_ff % 128 == 0) and the epilogue
// stores silu(gate) * up, [M, d_ff] bf16 (ldo elements apart)
cudaError_t launch_linear(const void* x, const void* w, void* out, bool out_bf16, int64_t M, int N, int K, int64_t ldo,
                          cudaStream_t stream, bool swiglu = false);
cudaError_t tp_proj_read_error(cudaStream_t stream, int* code);

// ---------------------------------------------------------------- gemv.cu
// y = x w^T for a few rows (bf16 in, fp32 accumulation, output row stride ldo); rows are taken in
// groups of gemv_max_rows(), the weight streamed once per group
int gemv_max_rows();
cudaError_t launch_gemv(const void* x, const void* w, void* y, bool y_bf16, int64_t M, int N, int K, int64_t ldo,
                        cudaStream_t stream);

// ---------------------------------------------------------------- glue.cu
// element-wise steps of the hybrid block: RMSNorm, SwiGLU, the mixer-input split
cudaError_t launch_rmsnorm(const void* x, const void* res, const void* w, int wdt, void* h_out, void* out, int dt,
                           int64_t n, int d, float eps, cudaStream_t stream);
cudaError_t launch_swiglu(const void* gu, void* out, int dt, int64_t n, int f, cudaStream_t stream);
cudaError_t launch_mixer_inputs(const void* z, int dt, int64_t n, int H, int64_t z_ld, const void* logit_decay,
                                int lddt, const int64_t* cu, int64_t num_seqs, void* q, void* k, void* v, float* beta,
                                float* decay, cudaStream_t stream);

// ---------------------------------------------------------------- anchor_attn.cu
// rotary q/k of the anchors' fused q|k|v rows, k/v into the KV cache, q head-major [H, n, 64] or [n, H, 64]
cudaError_t launch_anchor_qkv(const void* qkv, const int64_t* cu, const int64_t* start, const int64_t* rows, int64_t B,
                              int64_t n, int H, float theta, void* q_out, bool q_head_major, void* k_cache,
                              void* v_cache, int64_t cache_batch, int64_t L, cudaStream_t stream);
// varlen causal softmax attention (d = 64, bf16) of head-major q against the KV cache rows
cudaError_t launch_anchor_attention(const void* q, const void* k_cache, const void* v_cache, const int64_t* cu,
                                    const int64_t* rows, int64_t B, int64_t n, int H, int64_t cache_batch, int64_t L,
                                    int64_t max_seqlen, void* out, cudaStream_t stream);
cudaError_t attn_read_error(cudaStream_t stream, int* code);

// ---------------------------------------------------------------- decode_attn.cu
// one query per (sequence, head) against its cached keys [0, lengths[b]] (d = 64), split-K
int decode_attn_splits(int64_t max_len);
size_t decode_attn_workspace(int64_t B, int H, int64_t max_len);
cudaError_t launch_decode_attn(const void* q, const void* k_cache, const void* v_cache, const int64_t* lengths,
                               void* out, int dt, int64_t B, int H, int64_t max_len, float* part,
                               cudaStream_t stream);

// ---------------------------------------------------------------- ragged.cu
// rows of a packed [total, H, w] batch <-> per-sequence head-major [H, T_i, w] blocks
cudaError_t launch_ragged_transpose(const void* src, void* dst, const void* cu_seqlens, int index_dtype,
                                    int64_t num_seqs, int64_t total_tokens, int H, int64_t row_bytes,
                                    int to_head_major, cudaStream_t stream);

// ---------------------------------------------------------------- decode.cu
struct DecodeProblem {
  const void* q;
  const void* k;
  const void* v;
  int in_dtype;
  const void* beta;
  const void* decay;
  int gate_dtype;
  void* states;
  int state_dtype;
  int64_t num_slots;
  const void* slot_mapping;
  int index_dtype;
  void* out;
  int out_dtype;
  int64_t num_tokens;
  int H, dv, D;
  int readout;
};
cudaError_t launch_decode(const DecodeProblem& p, const ProjParams& P, cudaStream_t stream);
// reads and clears the decode kernels' device error word (synchronises stream)
cudaError_t decode_read_error(cudaStream_t stream, int* code);

}  // namespace kdn
