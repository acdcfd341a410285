/*
 * kdn.h -- C ABI of libkdn, the B200 (sm_100a) implementation of the
 * Kernel-DeltaNet hot path:
 *
 *   structured-FWHT feature lift (d_k = 64 -> D = 512, spherical renorm)
 *     -> exact gated delta-rule chunked prefill
 *     -> single-token decode state update
 *
 * Conventions shared by every entry point:
 *   - all tensor arguments are DEVICE pointers to contiguous row-major arrays;
 *     shapes are given by the int64 size arguments;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *     all work is enqueued on it, nothing synchronises the host;
 *   - the caller owns every buffer; no entry point allocates device memory;
 *   - the return value is a status code (KDN_OK == 0); on failure
 *     kdn_last_error() returns a message for the calling thread; nothing aborts.
 */
#ifndef KDN_H_
#define KDN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDN_ABI_VERSION 1

/* status codes */
#define KDN_OK 0
#define KDN_ERR_INVALID 1     /* bad argument: null pointer, shape, alignment */
#define KDN_ERR_UNSUPPORTED 2 /* valid but not implemented (e.g. d_k != 64) */
#define KDN_ERR_CUDA 3        /* a CUDA runtime call or launch failed */
#define KDN_ERR_WORKSPACE 4   /* workspace too small */
#define KDN_ERR_DEVICE 5      /* a kernel's own bounds check recorded a bad index */

/* element types */
#define KDN_DTYPE_F32 0
#define KDN_DTYPE_BF16 1

/* index types (slot_mapping) */
#define KDN_INDEX_I32 0
#define KDN_INDEX_I64 1

/* prefill arithmetic modes */
#define KDN_MODE_F32 0  /* fp32 arithmetic: CUDA cores, and split-tf32 tensor-core products
                           (three tf32 products per term, fp32 accumulation) for K S^T and
                           Q S^T at chunk 64 / D 512 */
#define KDN_MODE_BF16 1 /* bf16 tensor-core products, fp32 accumulation, fp32 state */

/* decode readout order */
#define KDN_READOUT_PRE 0  /* y = S_{t-1} phi(q_t), then update (module semantics) */
#define KDN_READOUT_POST 1 /* update, then y = S_t phi(q_t) (decode benchmark variant) */

/*
 * Constants of one structured projection (the reference's
 * FastWalshHadamardProjection, kernels/fwht.py:48-111).  Block m of the dense
 * map is H diag(d3[m]) H diag(d2[m]) H diag(d1[m]) / sqrt(d_k) with H the +-1
 * Sylvester matrix of order d_k.
 *
 *   sign_bits[m][s] bit i == 1  <=>  stage s (0:d1, 1:d2, 2:d3) sign of block m,
 *                                    element i, is -1
 *   phase: device pointer to D floats (the reference's buffer `b`)
 *   tau_inv = 1 / d_k^(1/4); amp = sqrt(2 / D)
 */
typedef struct kdn_projection {
  int32_t d_k;
  int32_t D;
  float tau_inv;
  float amp;
  uint64_t sign_bits[8][3];
  const float* phase;
} kdn_projection;

/* ABI version (KDN_ABI_VERSION) of the loaded library. */
int kdn_abi_version(void);

/* Message describing the last failure on the calling thread ("" if none). */
const char* kdn_last_error(void);

/*
 * Feature lift phi(x) = u / (||u|| + 1e-8), u = amp * cos(Omega x * tau_inv + phase).
 * x: [n, d_k] (x_dtype), out: [n, D] (out_dtype).
 * Replaces FastWalshHadamardProjection.forward, kernels/fwht.py:113-130
 * (and the pybind fwht_forward of kernels/fwht_cuda.cpp:8-30).
 * bf16 inputs with D = 512, 16-byte aligned x and out, and an Omega exact in bf16 run on the
 * tensor cores; other cases on CUDA cores (environment KDN_LIFT_PATH=pair forces the CUDA-core
 * kernel).  A tensor-core wait that gives up is reported by kdn_device_error (code 6).
 */
int kdn_fwht_lift(const void* x, int x_dtype, void* out, int out_dtype, int64_t n,
                  const kdn_projection* proj, void* stream);

/*
 * Bytes of device workspace kdn_chunked_prefill needs for these sizes
 * (0 when the selected path keeps everything on chip).
 */
size_t kdn_chunked_prefill_workspace_size(int64_t N, int64_t T, int32_t dv, int32_t chunk,
                                          const kdn_projection* proj, int mode);

/*
 * Exact gated delta-rule prefill over N independent sequences (heads
 * flattened into N):
 *   S_t = decay_t S_{t-1} (I - beta_t phi(k_t) phi(k_t)^T) + beta_t v_t phi(k_t)^T
 *   y_t = S_{t-1} phi(q_t)
 * q, k: [N, T, d_k]; v, y: [N, T, dv] (in_dtype / y_dtype); beta, decay: [N, T]
 * (gate_dtype; decay may be NULL meaning 1); initial_state: [N, dv, D] fp32 or
 * NULL (zeros); final_state: [N, dv, D] fp32 (may alias initial_state).
 * chunk: 32 or 64.  mode: KDN_MODE_F32 or KDN_MODE_BF16.
 * Replaces fused_chunked_deltanet_forward, kernels/fused_kernel_deltanet.py:31-155.
 */
int kdn_chunked_prefill(const void* q, const void* k, const void* v, int in_dtype,
                        const void* beta, const void* decay, int gate_dtype,
                        const float* initial_state, void* y, int y_dtype, float* final_state,
                        int64_t N, int64_t T, int32_t dv, int32_t chunk,
                        const kdn_projection* proj, int mode,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Measurement hook (no counterpart in the reference): the next kdn_chunked_prefill
 * call made by this thread records events[0] (cudaEvent_t, created by the caller) on
 * its stream before its first kernel launch and events[i] after launch i, for i <
 * count; later calls record nothing until the hook is set again.  count = 0 disarms.
 */
int kdn_set_prefill_events(void* const* events, int count);

/* Number of kernels the last kdn_chunked_prefill call of this thread launched. */
int kdn_prefill_launch_count(void);

/*
 * Size of the scratch array compiled into libkdn for kdn_chunked_prefill_static:
 * 64 MiB of device memory per device, reserved when the library's module is
 * loaded there.  Each sequence is padded to whole chunks, so the limit is on
 * N * Tp with Tp = T rounded up to a multiple of the chunk: at D = 512 and
 * d_v = 64, N * Tp up to 14,336 tokens (chunk 64) or 15,360 (chunk 32) -- for
 * example N = 224 sequences of T <= 64, but N = 14,336 of T = 1 do not fit.
 * kdn_chunked_prefill_workspace_size(..., KDN_MODE_F32) gives the exact need.
 */
#define KDN_STATIC_SCRATCH_BYTES (64u * 1024u * 1024u)

/*
 * kdn_chunked_prefill without a workspace argument, for callers that may not
 * allocate device memory when they run a prefill (an engine that reserved
 * nearly all device memory for its own pool up front, a step loop that cannot
 * take cudaFree's implicit device synchronisation).  It always runs the exact
 * fp32 path (KDN_MODE_F32); its scratch is the fixed
 * KDN_STATIC_SCRATCH_BYTES array above, so nothing is allocated per call.
 *   - Sizes whose scratch need exceeds KDN_STATIC_SCRATCH_BYTES are rejected
 *     with KDN_ERR_WORKSPACE before any work is enqueued.
 *   - The first call on each device looks the array's address up
 *     (cudaGetSymbolAddress with that device current), and looks it up again
 *     if the device's context has changed since (a device reset); make the
 *     first call on a device before any stream capture begins.
 *   - All calls on one device share the array: calls whose kernels overlap
 *     (unordered streams, several host threads) race.  Serialise them.
 * Arguments and results are those of kdn_chunked_prefill.  This entry point has
 * no counterpart in the reference (kernels/fused_kernel_deltanet.py allocates
 * its temporaries through PyTorch on every call).
 */
int kdn_chunked_prefill_static(const void* q, const void* k, const void* v, int in_dtype,
                               const void* beta, const void* decay, int gate_dtype,
                               const float* initial_state, void* y, int y_dtype,
                               float* final_state, int64_t N, int64_t T, int32_t dv,
                               int32_t chunk, const kdn_projection* proj, void* stream);

/*
 * Row-parallel output projection with its all-reduce fused in (head tensor parallelism,
 * serving/tensor_parallel_runner.py:51-75; experiments/run_kaggle_dual_gpu_cluster.py:99-112
 * run a local GEMM and then an all-reduce).  y: [M, K] bf16 (this rank's heads' outputs),
 * w: [N, K] bf16 (this rank's slice of the projection), both row-major; the kernel computes
 * y w^T on the tensor cores with fp32 accumulation and
 *   - with out_multicast (the NVSwitch multicast address of a symmetric [M, N] fp32 buffer):
 *     adds each tile into every member's copy (multimem.red); the buffer must be zero on
 *     every rank before any rank launches, and a barrier across ranks must follow before
 *     the sum is read -- the caller owns both steps;
 *   - otherwise stores y w^T into out ([M, N], out_dtype KDN_DTYPE_F32 or KDN_DTYPE_BF16).
 * N % 256 == 0, K % 64 == 0, pointers 16-byte aligned.  No reference entry point.
 */
int kdn_tp_out_proj(const void* y, const void* w, void* out, int out_dtype, float* out_multicast, int64_t M, int32_t N,
                    int32_t K, void* stream);

/*
 * Dense projection of one GPU, out = x w^T: the hybrid LM's q|k|v|beta, anchor q|k|v, output,
 * SwiGLU and head projections (the bias-free nn.Linear layers of layers/kernel_deltanet_layer.py:
 * 46-49, layers/hybrid_kernel_deltanet_block.py:43-45 and models/kernel_deltanet_lm.py:65).  x: [M, K] bf16, w: [N, K] bf16, both
 * row-major and 16-byte aligned; fp32 accumulation; out: [M, ldo] (ldo = 0 means N; ldo >= N,
 * ldo * element size a multiple of 16 bytes), columns [0, N) written, out_dtype KDN_DTYPE_F32 or
 * KDN_DTYPE_BF16.  K % 64 == 0, any N >= 1.  M <= 64 streams the weight through a GEMV kernel
 * (16 rows per pass); larger M runs the TMA-fed tcgen05 GEMM of kdn_tp_out_proj (128 x 256 tiles,
 * partial tiles at the M and N edges).  No reference entry point.
 */
int kdn_linear(const void* x, const void* w, void* out, int out_dtype, int64_t M, int32_t N, int32_t K, int64_t ldo,
               void* stream);

/*
 * SwiGLU's gate and up projections with the product fused into the GEMM epilogue
 * (layers/hybrid_kernel_deltanet_block.py:43-46: silu(x W_gate^T) * (x W_up^T)): out[m, j] =
 * silu(g) * u with g = x[m] . W_gate[j], u = x[m] . W_up[j] accumulated in fp32, stored as bf16
 * [M, ldo] (ldo = 0 means d_ff).  w_interleaved [2 d_ff, K] bf16 holds the two weights in row
 * blocks of 128: rows [256 t, 256 t + 128) are W_gate rows [128 t, 128 t + 128) and the next 128
 * the same W_up rows.  d_ff % 128 == 0, K % 64 == 0, pointers 16-byte aligned.  The gate/up product
 * never reaches memory.  No reference entry point.
 */
int kdn_linear_swiglu(const void* x, const void* w_interleaved, void* out, int64_t M, int32_t d_ff, int32_t K,
                      int64_t ldo, void* stream);

/*
 * The two-phase (bandwidth-optimal) form of kdn_tp_out_proj for the same sum over ranks.
 * Every rank stores its tiles of y w^T into its own copy `out` of the symmetric [M, N] buffer
 * (out_dtype KDN_DTYPE_F32, or KDN_DTYPE_BF16: the switch sums the bf16 copies in fp32 and the
 * sum is rounded once) and announces each tile by adding 1 to every rank's copy of that tile's counter
 * (tile_counters: a symmetric uint32 buffer of kdn_tp_out_proj_tiles(M, N) entries; its
 * multicast address alongside).  The owner of tile t (t % world == rank) waits until its copy
 * of counter t reaches `target`, then writes the sum of all copies of the tile into every copy
 * (multimem.ld_reduce + multimem.st).  The counters only grow: they start at zero on every
 * rank and call number c (1, 2, ...) passes target = c * world.  A barrier across ranks must
 * follow before the sum is read or `out` is written again.  No reference entry point.
 */
int64_t kdn_tp_out_proj_tiles(int64_t M, int32_t N);
int kdn_tp_out_proj_allreduce(const void* y, const void* w, void* out, void* out_multicast, int out_dtype,
                              uint32_t* tile_counters, uint32_t* tile_counters_multicast, uint32_t target, int32_t rank,
                              int32_t world, int64_t M, int32_t N, int32_t K, void* stream);

/*
 * The same two-phase projection over peer pointers instead of a multicast address (for
 * world 2, where it moves fewer bytes, and for GPUs without NVSwitch multicast).  outs and
 * tile_counters are HOST arrays of `world` device pointers (world <= 8): every rank's copy of
 * the [M, N] output and of the counters, index = rank, all mapped into this process (a
 * symmetric allocation's peer pointers).  Tiles are announced by adding 1 to every rank's
 * counter; the owner of tile t reads the tile from every copy, adds them in rank order (fp32)
 * and stores the sum into every copy.  out_dtype KDN_DTYPE_BF16: the copies hold bf16 (each
 * rank's product rounded once, the sum rounded once), half the bytes.  Same counter and barrier rules as
 * kdn_tp_out_proj_allreduce.  No reference entry point.
 */
int kdn_tp_out_proj_allreduce_peer(const void* y, const void* w, void* const* outs, int out_dtype,
                                   uint32_t* const* tile_counters, uint32_t target, int32_t rank, int32_t world,
                                   int64_t M, int32_t N, int32_t K, void* stream);

/*
 * Varlen form of kdn_chunked_prefill (tensor-core arithmetic, KDN_MODE_BF16; D = 512, dv = 64,
 * chunk 64): N independent scans of different lengths in one launch, one CTA per scan.  Scan n
 * reads rows [scan_offsets[n], scan_offsets[n] + scan_lengths[n]) of q, k [total_rows, 64],
 * v [total_rows, dv], beta / decay [total_rows] and writes the same rows of y; its state is row n
 * of initial_state / final_state [N, dv, D] (fp32).  scan_offsets / scan_lengths: int64 arrays on
 * the device; a scan whose rows fall outside [0, total_rows) is not run (its state is copied
 * through) and kdn_device_error reports it.  Give the longest scans the lowest indices: CTAs start
 * in index order.  The serving batch of the reference (serving/vllm_ragged_batching.py:41-103)
 * runs its requests one after another instead.
 */
int kdn_chunked_prefill_varlen(const void* q, const void* k, const void* v, int in_dtype, const void* beta,
                               const void* decay, int gate_dtype, const float* initial_state, void* y, int y_dtype,
                               float* final_state, const int64_t* scan_offsets, const int64_t* scan_lengths,
                               int64_t N, int64_t total_rows, int32_t dv, int32_t chunk, const kdn_projection* proj,
                               void* stream);

/*
 * Backward of kdn_chunked_prefill (the reference differentiates its prefill by recompute +
 * autograd, kernels/fused_kernel_deltanet.py:158-179; this is that gradient, computed directly).
 * Given the forward's inputs and dy = dL/dY [N, T, dv] (dy_dtype), optionally dL/d(final
 * state) [N, dv, D] fp32, it writes fp32 gradients: dq, dk [N, T, d_k], dv_out [N, T, dv],
 * dbeta [N, T], ddecay [N, T] (when decay is given; zero where the decay is clamped, i.e.
 * outside [1e-5, 1]) and, if d_initial_state is not NULL, dL/d(initial state) [N, dv, D].
 * fp32 arithmetic (KDN_MODE_F32's kernels): the forward is recomputed with checkpoints (the state entering
 * every chunk), then one reverse pass over chunks carries the state's adjoint, one parallel
 * pass forms every chunk's gradients, and the lift is differentiated through its butterfly.
 * dv a multiple of 16 up to 128; chunk 32 or 64; workspace from
 * kdn_chunked_prefill_backward_workspace_size (256-byte aligned).
 */
size_t kdn_chunked_prefill_backward_workspace_size(int64_t N, int64_t T, int32_t dv, int32_t chunk,
                                                   const kdn_projection* proj);
int kdn_chunked_prefill_backward(const void* q, const void* k, const void* v, int in_dtype, const void* beta,
                                 const void* decay, int gate_dtype, const float* initial_state, const void* dy,
                                 int dy_dtype, const float* d_final_state, float* dq, float* dk, float* dv_out,
                                 float* dbeta, float* ddecay, float* d_initial_state, int64_t N, int64_t T,
                                 int32_t dv, int32_t chunk, const kdn_projection* proj, void* workspace,
                                 size_t workspace_bytes, void* stream);

/*
 * One-token softmax attention over a KV cache (the anchor layers' decode step in the hybrid
 * model; the reference keeps those layers as Llama attention, models/upcycling_llama_bridge.py:240-249).
 * q [B, H, 64], k_cache / v_cache [B, H, max_len, 64] (dtype), lengths [B] int64 on the device:
 * query (b, h) attends to cache positions [0, lengths[b]] with scale 1/8; out [B, H, 64].
 * Positions past a sequence's length cost nothing.  A length >= max_len yields a zero output
 * row (the positions it names do not exist).  workspace: kdn_decode_attention_workspace_size.
 */
size_t kdn_decode_attention_workspace_size(int64_t B, int32_t H, int64_t max_len);
int kdn_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int64_t* lengths, void* out,
                         int dtype, int64_t B, int32_t H, int64_t max_len, int32_t d_head, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Element-wise steps of the hybrid decoder block (layers/hybrid_kernel_deltanet_block.py),
 * each one pass over its data; fp32 arithmetic, dtype KDN_DTYPE_F32 or KDN_DTYPE_BF16 storage.
 *   kdn_rmsnorm: out[r] = x[r] * rsqrt(mean(x[r]^2) + eps) * weight  (RMSNorm, :16-25); x, out
 *     [n, d] (same dtype, 16-byte aligned, d a multiple of 8 for bf16 / 4 for fp32).
 *   kdn_add_rmsnorm: h = x + residual, rounded to dtype and stored to h_out (the residual add
 *     of :89 / :96), then out = RMSNorm(h) as kdn_rmsnorm; residual NULL is kdn_rmsnorm.  h_out
 *     may be x; with a residual, out must not alias x, residual or h_out.
 *   kdn_swiglu: out[r, j] = silu(gate_up[r, j]) * gate_up[r, d_ff + j]  (SwiGLU, :45-46);
 *     gate_up [n, 2 d_ff], out [n, d_ff].
 *   kdn_mixer_inputs: z [n, 3 H 64 + H] (the fused q|k|v|beta projection; rows z_ld elements
 *     apart, z_ld = 0 meaning contiguous, z_ld even for 2-element loads) -> q, k [n, H, 64]
 *     L2-normalised per head (layers/kernel_deltanet_layer.py:98-99), v [n, H, 64], and fp32
 *     beta = sigmoid(z_beta) [n, H] (serving/tensor_parallel_runner.py:62) and decay =
 *     sigmoid(logit_decay[h]) [n, H] (kernel_deltanet_layer.py:71-73).  d_head must be 64.  With
 *     cu_seqlens (device int64 [num_seqs + 1], the packing of kdn_ragged_transpose) the outputs are
 *     written in the head-major per-sequence layout instead (row cu[i] H + h T_i + t), the layout
 *     kdn_chunked_prefill_varlen reads, so no separate transpose is needed; NULL keeps [n, H].
 * No reference entry points (the reference runs these as separate torch ops).
 */
int kdn_rmsnorm(const void* x, int dtype, const void* weight, int weight_dtype, void* out, int64_t n, int32_t d,
                float eps, void* stream);
int kdn_add_rmsnorm(const void* x, const void* residual, int dtype, const void* weight, int weight_dtype, void* h_out,
                    void* out, int64_t n, int32_t d, float eps, void* stream);
int kdn_swiglu(const void* gate_up, void* out, int dtype, int64_t n, int32_t d_ff, void* stream);
int kdn_mixer_inputs(const void* z, int dtype, int64_t n, int32_t H, int32_t d_head, int64_t z_ld,
                     const void* logit_decay, int logit_dtype, const int64_t* cu_seqlens, int64_t num_seqs, void* q,
                     void* k, void* v, float* beta, float* decay, void* stream);

/*
 * The softmax anchors of the hybrid LM (models/upcycling_llama_bridge.py:138-140, 240-249: causal
 * multi-head attention with rotate-half rotary positions; the reference calls torch SDPA), bf16,
 * d_head 64.  Sequences are packed back to back: sequence i holds tokens [cu[i], cu[i + 1]) of the
 * batch (cu_seqlens: device int64 [num_seqs + 1]); its keys and values live in row cache_rows[i]
 * (device int64 [num_seqs], NULL = row i) of the caches [cache_batch, H, max_len, 64].
 *   kdn_anchor_qkv: qkv [total_tokens, 3, H, 64] (the fused q|k|v projection) -> q and k rotated
 *     at position t - cu[i] + start_pos[i] (start_pos: device int64 [num_seqs], NULL = 0) with
 *     inv_freq = rope_theta^(-2j/64), angle = position * inv_freq in fp32; k and v are stored at
 *     that position of the cache row, q into q_out: [H, total_tokens, 64] (q_head_major = 1, the
 *     layout kdn_varlen_causal_attention reads) or [total_tokens, H, 64] (0, the layout of
 *     kdn_decode_attention).  A position or row outside the cache is skipped and recorded for
 *     kdn_device_error (code 1).
 *   kdn_varlen_causal_attention: out[t, h] = softmax(q_t K^T / 8 over positions <= t) V for every
 *     token t of every sequence, q head-major [H, total_tokens, 64], the keys/values read from the
 *     cache rows (positions [0, T_i)); out [total_tokens, H, 64].  max_seqlen (host) bounds every
 *     T_i and is at most max_len; a longer sequence is recorded for kdn_device_error (code 1).
 *     fp32 accumulation of both products, P rounded to bf16, 2^x via ex2.approx.
 * No reference entry points.
 */
int kdn_anchor_qkv(const void* qkv, int dtype, const int64_t* cu_seqlens, const int64_t* start_pos,
                   const int64_t* cache_rows, int64_t num_seqs, int64_t total_tokens, int32_t H, int32_t d_head,
                   float rope_theta, void* q_out, int q_head_major, void* k_cache, void* v_cache, int64_t cache_batch,
                   int64_t max_len, void* stream);
int kdn_varlen_causal_attention(const void* q, const void* k_cache, const void* v_cache, int dtype,
                                const int64_t* cu_seqlens, const int64_t* cache_rows, int64_t num_seqs,
                                int64_t total_tokens, int32_t H, int32_t d_head, int64_t cache_batch, int64_t max_len,
                                int64_t max_seqlen, void* out, void* stream);

/*
 * Layout change of a ragged serving batch (no reference counterpart; the reference packs
 * requests the same way, serving/vllm_ragged_batching.py:57-67, then loops over them).
 * Element (sequence i, token t, head h) of the packed [total_tokens, H, row] tensor sits at
 * ((cu[i] + t) * H + h); in the head-major form sequence i is one [H, T_i, row] block
 * starting at cu[i] * H, the layout kdn_chunked_prefill reads.  to_head_major = 1 packs ->
 * head-major, 0 the reverse.  cu_seqlens: device [num_seqs + 1] (index_dtype), nondecreasing
 * from 0 to total_tokens (rows outside that are left untouched).  row_bytes: bytes per (token,
 * head) row.  src and dst must not overlap.
 */
int kdn_ragged_transpose(const void* src, void* dst, const void* cu_seqlens, int index_dtype, int64_t num_seqs,
                         int64_t total_tokens, int32_t H, int64_t row_bytes, int to_head_major, void* stream);

/*
 * Strided block copy for streaming a sequence segment between host and device (no
 * reference counterpart): `rows` blocks of `width_bytes`, `src_pitch` / `dst_pitch` bytes
 * apart, copied on `stream` in either direction (host memory should be pinned for the copy
 * to be asynchronous).  One [B, T_seg, d] slice of a [B, T, d] tensor is one call.
 */
int kdn_copy_rows(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes, size_t rows,
                  void* stream);

/*
 * Affine semigroup of block state maps (exact fp32 on CUDA cores).  The state map of
 * a block of tokens is affine, S_out = S_in A + B, with S [dv, D], A [D, D], B [dv, D];
 * blocks compose as (A1, B1) o (A2, B2) = (A1 A2, B1 A2 + B2).
 *
 * kdn_affine_compose: batched composition over [batch] pairs.  A1, A2, A_out:
 * [batch, D, D]; B1, B2, B_out: [batch, dv, D].  A_out (with A1) or B_out (with B1) may
 * be NULL to skip that half; B2 may be NULL (zero).  Outputs must not overlap inputs.
 * D, dv: multiples of 16; every pointer 16-byte aligned.
 * Replaces compose_transitions, kernels/blelloch_scan.py:42-56 (also
 * AffineSemigroupVerifier.compose, core/associative_algebra.py:45-60).
 */
int kdn_affine_compose(const float* A1, const float* B1, const float* A2, const float* B2, float* A_out,
                       float* B_out, int64_t batch, int32_t D, int32_t dv, void* stream);

/*
 * Exclusive prefix states of a sequence of n_c block maps applied to S0:
 *   states[0] = S0 (zeros if NULL),  states[c+1] = states[c] A[c] + B[c]
 * and, if final_state is not NULL, final_state = states[n_c-1] A[n_c-1] + B[n_c-1].
 * A: [n_c, batch, D, D]; B: [n_c, batch, dv, D]; S0, final_state: [batch, dv, D];
 * states: [n_c, batch, dv, D] (S0 may be states itself).  n_c = 0 copies S0 (or
 * zeros) to final_state.  Outputs must not overlap A, B or each other.
 * Replaces blelloch_prefix_scan / sequential_prefix_scan, kernels/blelloch_scan.py:59-150
 * (same result: the state-only chain needs dv x D x D products per block where the
 * tree composes D x D transitions).
 */
int kdn_affine_prefix_states(const float* A, const float* B, const float* S0, float* states, float* final_state,
                             int64_t n_c, int64_t batch, int32_t D, int32_t dv, void* stream);

/*
 * Affine map of one block of T tokens of each of N sequences (exact fp32):
 *   A[n] = prod_t decay_t (I - beta_t phi(k_t) phi(k_t)^T)   (the homogeneous part)
 *   B[n] = the state the block leaves when it starts from zeros
 * so that for every entering state S_out = S_in A + B.  k, v, beta, decay as in
 * kdn_chunked_prefill (no q: nothing is read out).  A_out [N, D, D] or B_out [N, dv, D]
 * may be NULL (not computed; v may be NULL when B_out is).  Workspace:
 * kdn_block_transition_workspace_size.  T = 0 gives A = I, B = 0.
 * The reference forms these maps per chunk for its sequence-parallel scan
 * (kernels/blelloch_scan.py:8-12: A_c = gamma (I - phi_k^T W phi_k), B_c = V^T W_c phi_k).
 */
size_t kdn_block_transition_workspace_size(int64_t N, int64_t T, int32_t chunk, const kdn_projection* proj);
int kdn_block_transition(const void* k, const void* v, int in_dtype, const void* beta, const void* decay,
                         int gate_dtype, float* A_out, float* B_out, int64_t N, int64_t T, int32_t dv,
                         int32_t chunk, const kdn_projection* proj, void* workspace, size_t workspace_bytes,
                         void* stream);

/*
 * One decode token per (token, head), states addressed through slot_mapping:
 * q, k: [num_tokens, H, d_k]; v, out: [num_tokens, H, dv] (in_dtype / out_dtype);
 * beta, decay: [num_tokens, H] (gate_dtype, decay may be NULL);
 * states: [num_slots, H, dv, D] (state_dtype), updated in place;
 * slot_mapping: [num_tokens] (index_dtype); a negative slot marks a padding
 * token: its output row is zeroed and no state is touched.  A slot >= num_slots
 * is skipped the same way and recorded for kdn_device_error().
 * Two tokens mapped to the same slot in one call race: map each slot once.
 * Replaces the hybrid_recurrent_forward op, serving/vllm_kernel_deltanet_op.cpp:11-34
 * (semantics of kernels/kernel_deltanet_fused.py:288-300).
 */
int kdn_decode_step(const void* q, const void* k, const void* v, int in_dtype,
                    const void* beta, const void* decay, int gate_dtype,
                    void* states, int state_dtype, int64_t num_slots,
                    const void* slot_mapping, int index_dtype,
                    void* out, int out_dtype,
                    int64_t num_tokens, int32_t H, int32_t dv,
                    const kdn_projection* proj, int readout, void* stream);

/*
 * Copy slot `parent` of a slot-major state pool onto slot `child` on `stream`.
 * Replaces fork_recurrent_state, serving/vllm_kernel_deltanet_op.cpp:39-58.
 */
int kdn_fork_state(void* states, int64_t num_slots, int64_t bytes_per_slot,
                   int64_t parent, int64_t child, void* stream);

/*
 * Read and clear the device-side error word of the current device (written by
 * kernels whose bounds checks skipped a bad index, or whose bounded waits gave up).
 * Synchronises `stream`.  *code_out = 0 when nothing was recorded; otherwise 1 = a slot,
 * length or offset out of range, 2 = fused tensor-core prefill wait, 3 = two-phase prefill
 * wait, 4 = decode wait, 5 = tensor-parallel projection wait, 6 = tensor-core lift wait,
 * 7 = anchor attention wait.
 */
int kdn_device_error(void* stream, int* code_out);

#ifdef __cplusplus
}
#endif

#endif /* KDN_H_ */
