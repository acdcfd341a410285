// capi.cu -- the extern "C" surface of libkdn (declared in include/kdn.h).
//
// Every entry point validates its arguments, enqueues work on the caller's
// stream and returns a status code; failures leave a message in a thread-local
// buffer read by kdn_last_error().  Nothing here allocates device memory.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <string>

#include "kdn_internal.h"

namespace kdn {

int current_sm_count() {
  constexpr int kDevs = 64;
  static std::atomic<int> cache[kDevs] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < kDevs) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  if (dev >= 0 && dev < kDevs) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace kdn

namespace {

thread_local std::string g_last_error;
thread_local kdn::LaunchMarks g_marks;       // armed by kdn_set_prefill_events for the next prefill
thread_local int g_last_prefill_launches = 0;

// kdn_linear: row counts up to this stream the weight through the GEMV kernel (in groups of 16 rows);
// above it the tcgen05 GEMM's 128-row tiles are the better use of the weight bytes
constexpr int64_t kLinearGemvRows = 64;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return KDN_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(KDN_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool valid_dtype(int d) { return d == KDN_DTYPE_F32 || d == KDN_DTYPE_BF16; }

int check_projection(const kdn_projection* proj) {
  if (!proj) return fail(KDN_ERR_INVALID, "projection is NULL");
  if (proj->d_k != 64) return fail(KDN_ERR_UNSUPPORTED, "d_k=%d: only d_k=64 is implemented", proj->d_k);
  if (proj->D < 64 || proj->D > 512 || proj->D % 64 != 0)
    return fail(KDN_ERR_UNSUPPORTED, "D=%d: D must be a multiple of 64 in [64, 512]", proj->D);
  if (!proj->phase) return fail(KDN_ERR_INVALID, "projection phase pointer is NULL");
  if (!aligned(proj->phase, 8)) return fail(KDN_ERR_INVALID, "projection phase pointer must be 8-byte aligned");
  return KDN_OK;
}

// The bf16 tensor-core path applies when the shape matches and the dense Omega
// is exact in bf16; the exactness check walks the butterfly on the host, so its
// result is cached per sign pattern.
bool use_tc_path(const kdn_projection* proj, int32_t dv, int32_t chunk, int mode) {
  if (mode != KDN_MODE_BF16) return false;
  static thread_local uint64_t cached_bits[8][3];
  static thread_local int cached_D = -1;
  static thread_local bool cached_ok = false;
  const kdn::ProjParams P = kdn::make_proj_params(*proj);
  if (cached_D != proj->D || memcmp(cached_bits, proj->sign_bits, sizeof(cached_bits)) != 0) {
    cached_ok = kdn::tc_prefill_supported(proj->D, 64, 64, P);
    cached_D = proj->D;
    memcpy(cached_bits, proj->sign_bits, sizeof(cached_bits));
  }
  return cached_ok && proj->D == 512 && dv == 64 && chunk == 64;
}

// Which tensor-core prefill runs: the fused kernel (one CTA per sequence) keeps
// everything on chip and suits many sequences; the two-phase kernels spread each
// sequence's chunks over all SMs and suit up to half as many sequences as SMs.  KDN_PREFILL_PATH
// = "fused" or "split" forces one (both give the same results up to rounding).
bool use_split_path(int64_t N) {
  const char* env = getenv("KDN_PREFILL_PATH");
  if (env && strcmp(env, "fused") == 0) return false;
  if (env && strcmp(env, "split") == 0) return true;
  // Measured on B200 (T = 16384, bf16): the one-CTA-per-sequence kernel takes about the same time
  // for any N up to the SM count (one wave, latency bound), while the two-phase path grows with N
  // (its preparation shares the SMs); the two cross between N = 64 (split 2.7 ms, fused 3.5 ms)
  // and N = 96 (split 4.3 ms, fused 3.5 ms).
  return N <= kdn::current_sm_count() / 2;
}

bool overlaps(const void* a, size_t abytes, const void* b, size_t bbytes) {
  if (!a || !b || abytes == 0 || bbytes == 0) return false;
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + bbytes && pb < pa + abytes;
}

int check_affine_dims(int64_t batch, int32_t D, int32_t dv, bool need_dv) {
  if (batch < 1 || batch > 65535) return fail(KDN_ERR_INVALID, "batch=%lld outside [1, 65535]", (long long)batch);
  if (D < 16 || D > 8192 || D % 16 != 0) return fail(KDN_ERR_UNSUPPORTED, "D=%d: a multiple of 16 in [16, 8192]", D);
  if (need_dv && (dv < 16 || dv > 8192 || dv % 16 != 0))
    return fail(KDN_ERR_UNSUPPORTED, "dv=%d: a multiple of 16 in [16, 8192]", dv);
  return KDN_OK;
}

}  // namespace

extern "C" {

int kdn_abi_version(void) { return KDN_ABI_VERSION; }

const char* kdn_last_error(void) { return g_last_error.c_str(); }

int kdn_fwht_lift(const void* x, int x_dtype, void* out, int out_dtype, int64_t n, const kdn_projection* proj,
                  void* stream) {
  if (int rc = check_projection(proj)) return rc;
  if (n < 0) return fail(KDN_ERR_INVALID, "n=%lld < 0", (long long)n);
  if (n > 0 && (!x || !out)) return fail(KDN_ERR_INVALID, "x/out is NULL");
  if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype)) return fail(KDN_ERR_INVALID, "bad dtype");
  if (!aligned(x, 8) || !aligned(out, 8)) return fail(KDN_ERR_INVALID, "x/out must be 8-byte aligned");
  const kdn::ProjParams P = kdn::make_proj_params(*proj);
  // the tensor-core lift needs the dense Omega exact in bf16: the same condition as the tensor-core prefill
  const bool omega_exact = proj->D == 512 && use_tc_path(proj, 64, 64, KDN_MODE_BF16);
  cudaError_t e = kdn::launch_lift(x, x_dtype, out, out_dtype, n, P, omega_exact, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "lift launch");
  return ok();
}

size_t kdn_chunked_prefill_workspace_size(int64_t N, int64_t T, int32_t dv, int32_t chunk,
                                          const kdn_projection* proj, int mode) {
  if (!proj || N <= 0 || T <= 0 || (chunk != 32 && chunk != 64)) return 0;
  if (proj->D >= 64 && proj->D <= 512 && proj->d_k == 64 && use_tc_path(proj, dv, chunk, mode))
    return use_split_path(N) ? kdn::split_prefill_workspace(N, T) : 0;
  return kdn::simt_prefill_workspace(N, T, dv, chunk, proj->D);
}

int kdn_chunked_prefill(const void* q, const void* k, const void* v, int in_dtype, const void* beta,
                        const void* decay, int gate_dtype, const float* initial_state, void* y, int y_dtype,
                        float* final_state, int64_t N, int64_t T, int32_t dv, int32_t chunk,
                        const kdn_projection* proj, int mode, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (int rc = check_projection(proj)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N < 1 || N > 65535) return fail(KDN_ERR_INVALID, "N=%lld outside [1, 65535]", (long long)N);
  if (T < 0) return fail(KDN_ERR_INVALID, "T=%lld < 0", (long long)T);
  if (dv < 16 || dv > 512 || dv % 16 != 0)
    return fail(KDN_ERR_UNSUPPORTED, "dv=%d: dv must be a multiple of 16 in [16, 512]", dv);
  if (chunk != 32 && chunk != 64) return fail(KDN_ERR_UNSUPPORTED, "chunk=%d: chunk must be 32 or 64", chunk);
  if (mode != KDN_MODE_F32 && mode != KDN_MODE_BF16) return fail(KDN_ERR_INVALID, "bad mode %d", mode);
  if (!valid_dtype(in_dtype) || !valid_dtype(gate_dtype) || !valid_dtype(y_dtype))
    return fail(KDN_ERR_INVALID, "bad dtype");
  if (!final_state) return fail(KDN_ERR_INVALID, "final_state is NULL");
  const size_t state_bytes = sizeof(float) * size_t(N) * dv * proj->D;
  if (T == 0) {  // nothing to scan: S_out = S_in
    cudaError_t e = initial_state ? (initial_state == final_state
                                         ? cudaSuccess
                                         : cudaMemcpyAsync(final_state, initial_state, state_bytes,
                                                           cudaMemcpyDeviceToDevice, st))
                                  : cudaMemsetAsync(final_state, 0, state_bytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "empty prefill state copy");
    return ok();
  }
  if (!q || !k || !v || !beta || !y) return fail(KDN_ERR_INVALID, "q/k/v/beta/y is NULL");
  if (!aligned(q, 8) || !aligned(k, 8)) return fail(KDN_ERR_INVALID, "q/k must be 8-byte aligned");
  const bool tc = use_tc_path(proj, dv, chunk, mode);
  if (tc && (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(y, 16)))
    return fail(KDN_ERR_INVALID, "q/k/v/y must be 16-byte aligned for the tensor-core path");
  const bool split = tc && use_split_path(N);
  const size_t need = tc ? (split ? kdn::split_prefill_workspace(N, T) : 0)
                         : kdn::simt_prefill_workspace(N, T, dv, chunk, proj->D);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(KDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes, need);
  if (need > 0 && !aligned(workspace, 256)) return fail(KDN_ERR_INVALID, "workspace must be 256-byte aligned");

  kdn::PrefillProblem p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.in_dtype = in_dtype;
  p.beta = beta;
  p.decay = decay;
  p.gate_dtype = gate_dtype;
  p.S0 = initial_state;
  p.y = y;
  p.y_dtype = y_dtype;
  p.S_out = final_state;
  p.N = N;
  p.T = T;
  p.dv = dv;
  p.C = chunk;
  p.D = proj->D;
  const kdn::ProjParams P = kdn::make_proj_params(*proj);
  kdn::LaunchMarks marks = g_marks;
  g_marks = kdn::LaunchMarks();
  cudaError_t e = split ? kdn::launch_split_prefill(p, P, workspace, workspace_bytes, st, marks)
                  : tc  ? kdn::launch_tc_prefill(p, P, st, marks)
                        : kdn::launch_simt_prefill(p, P, workspace, workspace_bytes, st, marks);
  g_last_prefill_launches = marks.launches;
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return ok();
}

int kdn_chunked_prefill_varlen(const void* q, const void* k, const void* v, int in_dtype, const void* beta,
                               const void* decay, int gate_dtype, const float* initial_state, void* y, int y_dtype,
                               float* final_state, const int64_t* scan_offsets, const int64_t* scan_lengths,
                               int64_t N, int64_t total_rows, int32_t dv, int32_t chunk, const kdn_projection* proj,
                               void* stream) {
  if (int rc = check_projection(proj)) return rc;
  if (N < 1 || N > (int64_t(1) << 31) - 1) return fail(KDN_ERR_INVALID, "N=%lld", (long long)N);
  if (total_rows < 0) return fail(KDN_ERR_INVALID, "total_rows=%lld", (long long)total_rows);
  if (!valid_dtype(in_dtype) || !valid_dtype(gate_dtype) || !valid_dtype(y_dtype))
    return fail(KDN_ERR_INVALID, "bad dtype");
  if (!use_tc_path(proj, dv, chunk, KDN_MODE_BF16))
    return fail(KDN_ERR_UNSUPPORTED, "the varlen prefill runs the tensor-core path only (D=512, dv=64, chunk=64)");
  if (!q || !k || !v || !beta || !y || !final_state || !scan_offsets || !scan_lengths)
    return fail(KDN_ERR_INVALID, "q/k/v/beta/y/final_state/scan_offsets/scan_lengths is NULL");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(y, 16) || !aligned(scan_offsets, 8) ||
      !aligned(scan_lengths, 8))
    return fail(KDN_ERR_INVALID, "q/k/v/y must be 16-byte aligned, the scan arrays 8-byte aligned");
  kdn::PrefillProblem p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.in_dtype = in_dtype;
  p.beta = beta;
  p.decay = decay;
  p.gate_dtype = gate_dtype;
  p.S0 = initial_state;
  p.y = y;
  p.y_dtype = y_dtype;
  p.S_out = final_state;
  p.N = N;
  p.T = 0;
  p.dv = dv;
  p.C = chunk;
  p.D = proj->D;
  p.var_off = scan_offsets;
  p.var_len = scan_lengths;
  p.var_rows = total_rows;
  const kdn::ProjParams P = kdn::make_proj_params(*proj);
  kdn::LaunchMarks marks = g_marks;
  g_marks = kdn::LaunchMarks();
  cudaError_t e = kdn::launch_tc_prefill(p, P, static_cast<cudaStream_t>(stream), marks);
  g_last_prefill_launches = marks.launches;
  if (e != cudaSuccess) return cuda_fail(e, "varlen prefill launch");
  return ok();
}

size_t kdn_chunked_prefill_backward_workspace_size(int64_t N, int64_t T, int32_t dv, int32_t chunk,
                                                   const kdn_projection* proj) {
  if (!proj || N < 1 || T < 1 || dv < 16 || (chunk != 32 && chunk != 64)) return 0;
  return kdn::simt_backward_workspace(N, T, dv, chunk, proj->D);
}

int kdn_chunked_prefill_backward(const void* q, const void* k, const void* v, int in_dtype, const void* beta,
                                 const void* decay, int gate_dtype, const float* initial_state, const void* dy,
                                 int dy_dtype, const float* d_final_state, float* dq, float* dk, float* dv_out,
                                 float* dbeta, float* ddecay, float* d_initial_state, int64_t N, int64_t T,
                                 int32_t dv, int32_t chunk, const kdn_projection* proj, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (int rc = check_projection(proj)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N < 1 || N > 65535) return fail(KDN_ERR_INVALID, "N=%lld outside [1, 65535]", (long long)N);
  if (T < 0) return fail(KDN_ERR_INVALID, "T=%lld < 0", (long long)T);
  if (dv < 16 || dv > 128 || dv % 16 != 0)
    return fail(KDN_ERR_UNSUPPORTED, "dv=%d: the backward takes a multiple of 16 in [16, 128]", dv);
  if (chunk != 32 && chunk != 64) return fail(KDN_ERR_UNSUPPORTED, "chunk=%d: chunk must be 32 or 64", chunk);
  if (!valid_dtype(in_dtype) || !valid_dtype(gate_dtype) || !valid_dtype(dy_dtype))
    return fail(KDN_ERR_INVALID, "bad dtype");
  const size_t state_bytes = sizeof(float) * size_t(N) * dv * proj->D;
  if (T == 0) {  // no tokens: the initial state's gradient is the final state's
    if (!d_initial_state) return ok();
    cudaError_t e = d_final_state ? cudaMemcpyAsync(d_initial_state, d_final_state, state_bytes,
                                                    cudaMemcpyDeviceToDevice, st)
                                  : cudaMemsetAsync(d_initial_state, 0, state_bytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "empty backward state copy");
    return ok();
  }
  if (!q || !k || !v || !beta || !dy || !dq || !dk || !dv_out || !dbeta)
    return fail(KDN_ERR_INVALID, "q/k/v/beta/dy or a gradient output is NULL");
  if (!aligned(q, 8) || !aligned(k, 8)) return fail(KDN_ERR_INVALID, "q/k must be 8-byte aligned");
  if (!aligned(dq, 8) || !aligned(dk, 8)) return fail(KDN_ERR_INVALID, "dq/dk must be 8-byte aligned");
  const size_t need = kdn::simt_backward_workspace(N, T, dv, chunk, proj->D);
  if (!workspace || workspace_bytes < need)
    return fail(KDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(KDN_ERR_INVALID, "workspace must be 256-byte aligned");
  kdn::BackwardProblem b;
  b.fwd.q = q;
  b.fwd.k = k;
  b.fwd.v = v;
  b.fwd.in_dtype = in_dtype;
  b.fwd.beta = beta;
  b.fwd.decay = decay;
  b.fwd.gate_dtype = gate_dtype;
  b.fwd.S0 = initial_state;
  b.fwd.y = nullptr;
  b.fwd.y_dtype = KDN_DTYPE_F32;
  b.fwd.S_out = nullptr;
  b.fwd.N = N;
  b.fwd.T = T;
  b.fwd.dv = dv;
  b.fwd.C = chunk;
  b.fwd.D = proj->D;
  b.dy = dy;
  b.dy_dtype = dy_dtype;
  b.dS_final = d_final_state;
  b.dq = dq;
  b.dk = dk;
  b.dv_out = dv_out;
  b.dbeta = dbeta;
  b.ddecay = decay ? ddecay : nullptr;
  b.dS0 = d_initial_state;
  b.omega = nullptr;
  const kdn::ProjParams P = kdn::make_proj_params(*proj);
  cudaError_t e = kdn::launch_simt_backward(b, P, workspace, workspace_bytes, st);
  if (e != cudaSuccess) return cuda_fail(e, "backward launch");
  return ok();
}

// Same checks and kernels as kdn_chunked_prefill in KDN_MODE_F32; the workspace is the
// library's fixed scratch array (prefill_static.cu), for callers that cannot allocate.
int kdn_chunked_prefill_static(const void* q, const void* k, const void* v, int in_dtype, const void* beta,
                               const void* decay, int gate_dtype, const float* initial_state, void* y, int y_dtype,
                               float* final_state, int64_t N, int64_t T, int32_t dv, int32_t chunk,
                               const kdn_projection* proj, void* stream) {
  if (int rc = check_projection(proj)) return rc;
  // bound the sizes first so that the scratch computation below cannot overflow
  if (N < 1 || N > 65535) return fail(KDN_ERR_INVALID, "N=%lld outside [1, 65535]", (long long)N);
  if (T < 0) return fail(KDN_ERR_INVALID, "T=%lld < 0", (long long)T);
  if (T > int64_t(KDN_STATIC_SCRATCH_BYTES))
    return fail(KDN_ERR_WORKSPACE, "T=%lld: far beyond the %u-byte static scratch; use kdn_chunked_prefill",
                (long long)T, KDN_STATIC_SCRATCH_BYTES);
  const size_t need = kdn_chunked_prefill_workspace_size(N, T, dv, chunk, proj, KDN_MODE_F32);
  if (need > size_t(KDN_STATIC_SCRATCH_BYTES))
    return fail(KDN_ERR_WORKSPACE,
                "N=%lld T=%lld needs %zu bytes of scratch, more than the %u-byte static scratch "
                "(KDN_STATIC_SCRATCH_BYTES); split the call or use kdn_chunked_prefill with a workspace",
                (long long)N, (long long)T, need, KDN_STATIC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need > 0) {
    cudaError_t e = kdn::static_prefill_scratch(&scratch);
    if (e != cudaSuccess) return cuda_fail(e, "static scratch address");
  }
  return kdn_chunked_prefill(q, k, v, in_dtype, beta, decay, gate_dtype, initial_state, y, y_dtype, final_state, N, T,
                             dv, chunk, proj, KDN_MODE_F32, scratch, scratch ? size_t(KDN_STATIC_SCRATCH_BYTES) : 0,
                             stream);
}

int kdn_set_prefill_events(void* const* events, int count) {
  if (count < 0 || (count > 0 && !events)) return fail(KDN_ERR_INVALID, "events/count");
  g_marks = kdn::LaunchMarks();
  g_marks.ev = count > 0 ? reinterpret_cast<cudaEvent_t*>(const_cast<void**>(events)) : nullptr;
  g_marks.cap = count;
  return ok();
}

int kdn_prefill_launch_count(void) { return g_last_prefill_launches; }

int kdn_tp_out_proj(const void* y, const void* w, void* out, int out_dtype, float* out_multicast, int64_t M, int32_t N,
                    int32_t K, void* stream) {
  if (M < 0 || M > (int64_t(65535) * 128)) return fail(KDN_ERR_INVALID, "M=%lld outside [0, 65535*128]", (long long)M);
  if (M == 0) return ok();
  if (N < 256 || N % 256 != 0 || N > 65535 * 256) return fail(KDN_ERR_UNSUPPORTED, "N=%d: a positive multiple of 256", N);
  if (K < 64 || K % 64 != 0) return fail(KDN_ERR_UNSUPPORTED, "K=%d: a positive multiple of 64", K);
  if (!y || !w || (!out && !out_multicast)) return fail(KDN_ERR_INVALID, "y/w/out is NULL");
  if (out_dtype != KDN_DTYPE_F32 && out_dtype != KDN_DTYPE_BF16) return fail(KDN_ERR_INVALID, "bad output dtype");
  if (out_multicast && out_dtype != KDN_DTYPE_F32)
    return fail(KDN_ERR_UNSUPPORTED, "the multicast sum is formed in the fp32 output");
  if (!aligned(y, 16) || !aligned(w, 16) || !aligned(out, 16) || !aligned(out_multicast, 16))
    return fail(KDN_ERR_INVALID, "y/w/out must be 16-byte aligned");
  cudaError_t e = kdn::launch_tp_proj(y, w, out, out_dtype == KDN_DTYPE_BF16, out_multicast, M, N, K,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tensor-parallel projection launch");
  return ok();
}

int kdn_linear(const void* x, const void* w, void* out, int out_dtype, int64_t M, int32_t N, int32_t K, int64_t ldo,
               void* stream) {
  if (M < 0 || M > int64_t(0x7fffff00)) return fail(KDN_ERR_INVALID, "M=%lld outside [0, 2^31 - 256]", (long long)M);
  if (N < 1 || K < 1) return fail(KDN_ERR_INVALID, "N=%d K=%d", N, K);
  if (M == 0) return ok();
  if (K % 64 != 0) return fail(KDN_ERR_UNSUPPORTED, "K=%d: a positive multiple of 64", K);
  if (!x || !w || !out) return fail(KDN_ERR_INVALID, "x/w/out is NULL");
  if (out_dtype != KDN_DTYPE_F32 && out_dtype != KDN_DTYPE_BF16) return fail(KDN_ERR_INVALID, "bad output dtype");
  const int64_t es = out_dtype == KDN_DTYPE_BF16 ? 2 : 4;
  if (ldo == 0) ldo = N;
  if (ldo < N || (ldo * es) % 16 != 0)
    return fail(KDN_ERR_INVALID, "ldo=%lld: at least N and a multiple of 16 bytes", (long long)ldo);
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16)) return fail(KDN_ERR_INVALID, "x/w/out must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = M <= kLinearGemvRows
                      ? kdn::launch_gemv(x, w, out, out_dtype == KDN_DTYPE_BF16, M, N, K, ldo, st)
                      : kdn::launch_linear(x, w, out, out_dtype == KDN_DTYPE_BF16, M, N, K, ldo, st);
  if (e == cudaErrorNotSupported) return fail(KDN_ERR_UNSUPPORTED, "no tensor-map encoder in this driver");
  if (e != cudaSuccess) return cuda_fail(e, "linear launch");
  return ok();
}

int kdn_linear_swiglu(const void* x, const void* w_interleaved, void* out, int64_t M, int32_t d_ff, int32_t K,
                      int64_t ldo, void* stream) {
  if (M < 0 || M > int64_t(0x7fffff00)) return fail(KDN_ERR_INVALID, "M=%lld outside [0, 2^31 - 256]", (long long)M);
  if (d_ff < 128 || d_ff % 128 != 0) return fail(KDN_ERR_UNSUPPORTED, "d_ff=%d: a positive multiple of 128", d_ff);
  if (K < 64 || K % 64 != 0) return fail(KDN_ERR_UNSUPPORTED, "K=%d: a positive multiple of 64", K);
  if (M == 0) return ok();
  if (!x || !w_interleaved || !out) return fail(KDN_ERR_INVALID, "x/w/out is NULL");
  if (ldo == 0) ldo = d_ff;
  if (ldo < d_ff || (ldo * 2) % 16 != 0)
    return fail(KDN_ERR_INVALID, "ldo=%lld: at least d_ff and a multiple of 16 bytes", (long long)ldo);
  if (!aligned(x, 16) || !aligned(w_interleaved, 16) || !aligned(out, 16))
    return fail(KDN_ERR_INVALID, "x/w/out must be 16-byte aligned");
  cudaError_t e = kdn::launch_linear(x, w_interleaved, out, true, M, 2 * d_ff, K, ldo, static_cast<cudaStream_t>(stream),
                                     true);
  if (e == cudaErrorNotSupported) return fail(KDN_ERR_UNSUPPORTED, "no tensor-map encoder in this driver");
  if (e != cudaSuccess) return cuda_fail(e, "linear-swiglu launch");
  return ok();
}

int64_t kdn_tp_out_proj_tiles(int64_t M, int32_t N) {
  if (M < 0 || N < 256 || N % 256 != 0) return 0;
  return kdn::tp_proj_tiles(M, N);
}

int kdn_tp_out_proj_allreduce(const void* y, const void* w, void* out, void* out_multicast, int out_dtype,
                              uint32_t* tile_counters, uint32_t* tile_counters_multicast, uint32_t target, int32_t rank,
                              int32_t world, int64_t M, int32_t N, int32_t K, void* stream) {
  if (M < 0 || M > (int64_t(65535) * 128)) return fail(KDN_ERR_INVALID, "M=%lld outside [0, 65535*128]", (long long)M);
  if (world < 1 || rank < 0 || rank >= world) return fail(KDN_ERR_INVALID, "rank=%d world=%d", rank, world);
  if (M == 0) return ok();
  if (N < 256 || N % 256 != 0 || N > 65535 * 256) return fail(KDN_ERR_UNSUPPORTED, "N=%d: a positive multiple of 256", N);
  if (K < 64 || K % 64 != 0) return fail(KDN_ERR_UNSUPPORTED, "K=%d: a positive multiple of 64", K);
  if (!y || !w || !out || !out_multicast || !tile_counters || !tile_counters_multicast)
    return fail(KDN_ERR_INVALID, "y/w/out/out_multicast/tile_counters is NULL");
  if (!aligned(y, 16) || !aligned(w, 16) || !aligned(out, 16) || !aligned(out_multicast, 16) ||
      !aligned(tile_counters, 4) || !aligned(tile_counters_multicast, 4))
    return fail(KDN_ERR_INVALID, "y/w/out must be 16-byte aligned, the counters 4-byte aligned");
  if (out_dtype != KDN_DTYPE_F32 && out_dtype != KDN_DTYPE_BF16) return fail(KDN_ERR_INVALID, "bad output dtype");
  cudaError_t e = kdn::launch_tp_proj_reduce(y, w, out, out_multicast, out_dtype == KDN_DTYPE_BF16, tile_counters,
                                             tile_counters_multicast, target, rank, world, M, N, K,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tensor-parallel projection launch");
  return ok();
}

int kdn_tp_out_proj_allreduce_peer(const void* y, const void* w, void* const* outs, int out_dtype,
                                   uint32_t* const* tile_counters, uint32_t target, int32_t rank, int32_t world,
                                   int64_t M, int32_t N, int32_t K, void* stream) {
  if (M < 0 || M > (int64_t(65535) * 128)) return fail(KDN_ERR_INVALID, "M=%lld outside [0, 65535*128]", (long long)M);
  if (world < 1 || world > kdn::tp_proj_max_world() || rank < 0 || rank >= world)
    return fail(KDN_ERR_INVALID, "rank=%d world=%d (world <= %d)", rank, world, kdn::tp_proj_max_world());
  if (M == 0) return ok();
  if (N < 256 || N % 256 != 0 || N > 65535 * 256) return fail(KDN_ERR_UNSUPPORTED, "N=%d: a positive multiple of 256", N);
  if (K < 64 || K % 64 != 0) return fail(KDN_ERR_UNSUPPORTED, "K=%d: a positive multiple of 64", K);
  if (!y || !w || !outs || !tile_counters) return fail(KDN_ERR_INVALID, "y/w/outs/tile_counters is NULL");
  if (out_dtype != KDN_DTYPE_F32 && out_dtype != KDN_DTYPE_BF16) return fail(KDN_ERR_INVALID, "bad output dtype");
  if (!aligned(y, 16) || !aligned(w, 16)) return fail(KDN_ERR_INVALID, "y/w must be 16-byte aligned");
  for (int p = 0; p < world; ++p)
    if (!outs[p] || !tile_counters[p] || !aligned(outs[p], 16) || !aligned(tile_counters[p], 4))
      return fail(KDN_ERR_INVALID, "copy %d of the output/counters is NULL or misaligned", p);
  cudaError_t e = kdn::launch_tp_proj_reduce_peer(y, w, outs, out_dtype == KDN_DTYPE_BF16, tile_counters, target, rank,
                                                  world, M, N, K, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tensor-parallel projection launch");
  return ok();
}

static bool float_dtype(int dt) { return dt == KDN_DTYPE_F32 || dt == KDN_DTYPE_BF16; }

size_t kdn_decode_attention_workspace_size(int64_t B, int32_t H, int64_t max_len) {
  if (B < 1 || H < 1 || max_len < 1) return 0;
  return kdn::decode_attn_workspace(B, H, max_len);
}

int kdn_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int64_t* lengths, void* out,
                         int dtype, int64_t B, int32_t H, int64_t max_len, int32_t d_head, void* workspace,
                         size_t workspace_bytes, void* stream) {
  if (B < 0 || H < 1 || max_len < 1) return fail(KDN_ERR_INVALID, "B=%lld H=%d max_len=%lld", (long long)B, H,
                                                 (long long)max_len);
  if (d_head != 64) return fail(KDN_ERR_UNSUPPORTED, "d_head=%d (64 only)", d_head);
  if (B == 0) return ok();
  if (B > 65535 || H > 65535 || kdn::decode_attn_splits(max_len) > (1 << 30))
    return fail(KDN_ERR_UNSUPPORTED, "grid too large");
  if (!q || !k_cache || !v_cache || !lengths || !out) return fail(KDN_ERR_INVALID, "a pointer is NULL");
  if (!float_dtype(dtype)) return fail(KDN_ERR_INVALID, "bad dtype");
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 8) || !aligned(lengths, 8))
    return fail(KDN_ERR_INVALID, "q/k_cache/v_cache must be 16-byte aligned");
  const size_t need = kdn::decode_attn_workspace(B, H, max_len);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
    return fail(KDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes, need);
  cudaError_t e = kdn::launch_decode_attn(q, k_cache, v_cache, lengths, out, dtype, B, H, max_len,
                                          static_cast<float*>(workspace), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode attention launch");
  return ok();
}
static int vec_elems(int dt) { return dt == KDN_DTYPE_BF16 ? 8 : 4; }

int kdn_rmsnorm(const void* x, int dtype, const void* weight, int weight_dtype, void* out, int64_t n, int32_t d,
                float eps, void* stream) {
  return kdn_add_rmsnorm(x, nullptr, dtype, weight, weight_dtype, nullptr, out, n, d, eps, stream);
}

int kdn_add_rmsnorm(const void* x, const void* residual, int dtype, const void* weight, int weight_dtype, void* h_out,
                    void* out, int64_t n, int32_t d, float eps, void* stream) {
  if (n < 0 || d < 1) return fail(KDN_ERR_INVALID, "n=%lld d=%d", (long long)n, d);
  if (n == 0) return ok();
  if (!x || !weight || !out) return fail(KDN_ERR_INVALID, "x/weight/out is NULL");
  if (residual && !h_out) return fail(KDN_ERR_INVALID, "h_out is NULL (needed with a residual)");
  if (!float_dtype(dtype) || !float_dtype(weight_dtype)) return fail(KDN_ERR_INVALID, "bad dtype");
  if (d % vec_elems(dtype) != 0) return fail(KDN_ERR_UNSUPPORTED, "d=%d: a multiple of %d", d, vec_elems(dtype));
  if (!aligned(x, 16) || !aligned(out, 16) || (residual && (!aligned(residual, 16) || !aligned(h_out, 16))))
    return fail(KDN_ERR_INVALID, "x/residual/h_out/out must be 16-byte aligned");
  if (residual && (out == x || out == residual || out == h_out))
    return fail(KDN_ERR_INVALID, "out must not alias x, residual or h_out");
  cudaError_t e = kdn::launch_rmsnorm(x, residual, weight, weight_dtype, residual ? h_out : nullptr, out, dtype, n, d,
                                      eps, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rmsnorm launch");
  return ok();
}

int kdn_swiglu(const void* gate_up, void* out, int dtype, int64_t n, int32_t d_ff, void* stream) {
  if (n < 0 || d_ff < 1) return fail(KDN_ERR_INVALID, "n=%lld d_ff=%d", (long long)n, d_ff);
  if (n == 0) return ok();
  if (!gate_up || !out) return fail(KDN_ERR_INVALID, "gate_up/out is NULL");
  if (!float_dtype(dtype)) return fail(KDN_ERR_INVALID, "bad dtype");
  if (d_ff % vec_elems(dtype) != 0) return fail(KDN_ERR_UNSUPPORTED, "d_ff=%d: a multiple of %d", d_ff, vec_elems(dtype));
  if (!aligned(gate_up, 16) || !aligned(out, 16)) return fail(KDN_ERR_INVALID, "gate_up/out must be 16-byte aligned");
  cudaError_t e = kdn::launch_swiglu(gate_up, out, dtype, n, d_ff, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "swiglu launch");
  return ok();
}

int kdn_mixer_inputs(const void* z, int dtype, int64_t n, int32_t H, int32_t d_head, int64_t z_ld,
                     const void* logit_decay, int logit_dtype, const int64_t* cu_seqlens, int64_t num_seqs, void* q,
                     void* k, void* v, float* beta, float* decay, void* stream) {
  if (n < 0 || H < 1) return fail(KDN_ERR_INVALID, "n=%lld H=%d", (long long)n, H);
  if (d_head != 64) return fail(KDN_ERR_UNSUPPORTED, "d_head=%d (the lift takes 64)", d_head);
  const int64_t row = int64_t(3) * H * d_head + H;
  if (z_ld == 0) z_ld = row;
  if (z_ld < row) return fail(KDN_ERR_INVALID, "z_ld=%lld below the row length %lld", (long long)z_ld, (long long)row);
  if (n == 0) return ok();
  if (!z || !logit_decay || !q || !k || !v || !beta || !decay) return fail(KDN_ERR_INVALID, "a pointer is NULL");
  if (!float_dtype(dtype) || !float_dtype(logit_dtype)) return fail(KDN_ERR_INVALID, "bad dtype");
  if (!aligned(z, 4) || !aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16))
    return fail(KDN_ERR_INVALID, "z must be 4-byte, q/k/v 16-byte aligned");
  if (cu_seqlens && num_seqs < 1) return fail(KDN_ERR_INVALID, "num_seqs=%lld with cu_seqlens", (long long)num_seqs);
  cudaError_t e = kdn::launch_mixer_inputs(z, dtype, n, H, z_ld, logit_decay, logit_dtype, cu_seqlens, num_seqs, q, k,
                                           v, beta, decay,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "mixer-input launch");
  return ok();
}

int kdn_anchor_qkv(const void* qkv, int dtype, const int64_t* cu_seqlens, const int64_t* start_pos,
                   const int64_t* cache_rows, int64_t num_seqs, int64_t total_tokens, int32_t H, int32_t d_head,
                   float rope_theta, void* q_out, int q_head_major, void* k_cache, void* v_cache, int64_t cache_batch,
                   int64_t max_len, void* stream) {
  if (num_seqs < 1 || total_tokens < 0 || H < 1 || cache_batch < 1 || max_len < 1)
    return fail(KDN_ERR_INVALID, "num_seqs=%lld total=%lld H=%d cache_batch=%lld max_len=%lld", (long long)num_seqs,
                (long long)total_tokens, H, (long long)cache_batch, (long long)max_len);
  if (d_head != 64) return fail(KDN_ERR_UNSUPPORTED, "d_head=%d (64 only)", d_head);
  if (dtype != KDN_DTYPE_BF16) return fail(KDN_ERR_UNSUPPORTED, "bf16 only");
  if (!(rope_theta > 0.f)) return fail(KDN_ERR_INVALID, "rope_theta must be positive");
  if (total_tokens == 0) return ok();
  if (!qkv || !cu_seqlens || !q_out || !k_cache || !v_cache) return fail(KDN_ERR_INVALID, "a pointer is NULL");
  if (!aligned(qkv, 4) || !aligned(q_out, 4) || !aligned(k_cache, 4) || !aligned(v_cache, 4))
    return fail(KDN_ERR_INVALID, "qkv/q_out/caches must be 4-byte aligned");
  cudaError_t e = kdn::launch_anchor_qkv(qkv, cu_seqlens, start_pos, cache_rows, num_seqs, total_tokens, H, rope_theta,
                                         q_out, q_head_major != 0, k_cache, v_cache, cache_batch, max_len,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "anchor q/k/v launch");
  return ok();
}

int kdn_varlen_causal_attention(const void* q, const void* k_cache, const void* v_cache, int dtype,
                                const int64_t* cu_seqlens, const int64_t* cache_rows, int64_t num_seqs,
                                int64_t total_tokens, int32_t H, int32_t d_head, int64_t cache_batch, int64_t max_len,
                                int64_t max_seqlen, void* out, void* stream) {
  if (num_seqs < 1 || total_tokens < 0 || H < 1 || cache_batch < 1 || max_len < 1 || max_seqlen < 0)
    return fail(KDN_ERR_INVALID, "num_seqs=%lld total=%lld H=%d cache_batch=%lld max_len=%lld max_seqlen=%lld",
                (long long)num_seqs, (long long)total_tokens, H, (long long)cache_batch, (long long)max_len,
                (long long)max_seqlen);
  if (d_head != 64) return fail(KDN_ERR_UNSUPPORTED, "d_head=%d (64 only)", d_head);
  if (dtype != KDN_DTYPE_BF16) return fail(KDN_ERR_UNSUPPORTED, "bf16 only");
  if (max_seqlen > max_len) return fail(KDN_ERR_INVALID, "max_seqlen=%lld exceeds the cache (%lld)",
                                        (long long)max_seqlen, (long long)max_len);
  const int64_t lim = (int64_t(1) << 31) - 1024;  // tensor-map row coordinates are 32-bit
  if (int64_t(H) * total_tokens > lim || cache_batch * H * max_len > lim)
    return fail(KDN_ERR_UNSUPPORTED, "more than 2^31 - 1024 rows of 64 in q or the cache");
  if (num_seqs * H > int64_t(0x7fffffff) || (max_seqlen + 255) / 256 > 65535)
    return fail(KDN_ERR_UNSUPPORTED, "grid too large");
  if (total_tokens == 0 || max_seqlen == 0) return ok();
  if (!q || !k_cache || !v_cache || !cu_seqlens || !out) return fail(KDN_ERR_INVALID, "a pointer is NULL");
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 16))
    return fail(KDN_ERR_INVALID, "q/caches/out must be 16-byte aligned");
  cudaError_t e = kdn::launch_anchor_attention(q, k_cache, v_cache, cu_seqlens, cache_rows, num_seqs, total_tokens, H,
                                               cache_batch, max_len, max_seqlen, out, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported) return fail(KDN_ERR_UNSUPPORTED, "no tensor-map encoder in this driver");
  if (e != cudaSuccess) return cuda_fail(e, "attention launch");
  return ok();
}

int kdn_ragged_transpose(const void* src, void* dst, const void* cu_seqlens, int index_dtype, int64_t num_seqs,
                         int64_t total_tokens, int32_t H, int64_t row_bytes, int to_head_major, void* stream) {
  if (total_tokens == 0) return ok();
  if (!src || !dst || !cu_seqlens) return fail(KDN_ERR_INVALID, "src/dst/cu_seqlens is NULL");
  if (num_seqs < 1 || total_tokens < 0 || H < 1 || row_bytes < 1)
    return fail(KDN_ERR_INVALID, "num_seqs=%lld total=%lld H=%d row_bytes=%lld", (long long)num_seqs,
                (long long)total_tokens, H, (long long)row_bytes);
  if (index_dtype != KDN_INDEX_I32 && index_dtype != KDN_INDEX_I64) return fail(KDN_ERR_INVALID, "bad index dtype");
  const size_t bytes = size_t(total_tokens) * H * size_t(row_bytes);
  if (overlaps(src, bytes, dst, bytes)) return fail(KDN_ERR_INVALID, "src and dst overlap");
  cudaError_t e = kdn::launch_ragged_transpose(src, dst, cu_seqlens, index_dtype, num_seqs, total_tokens, H, row_bytes,
                                               to_head_major, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "ragged transpose launch");
  return ok();
}

int kdn_copy_rows(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes, size_t rows,
                  void* stream) {
  if (rows == 0 || width_bytes == 0) return ok();
  if (!dst || !src) return fail(KDN_ERR_INVALID, "dst/src is NULL");
  if (dst_pitch < width_bytes || src_pitch < width_bytes)
    return fail(KDN_ERR_INVALID, "pitch below the row width (%zu, %zu < %zu)", dst_pitch, src_pitch, width_bytes);
  cudaError_t e = cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, rows, cudaMemcpyDefault,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "strided copy");
  return ok();
}

int kdn_affine_compose(const float* A1, const float* B1, const float* A2, const float* B2, float* A_out,
                       float* B_out, int64_t batch, int32_t D, int32_t dv, void* stream) {
  if (!A_out && !B_out) return ok();
  if (int rc = check_affine_dims(batch, D, dv, B_out != nullptr)) return rc;
  if (!A2) return fail(KDN_ERR_INVALID, "A2 is NULL");
  if (A_out && !A1) return fail(KDN_ERR_INVALID, "A1 is NULL but A_out is not");
  if (B_out && !B1) return fail(KDN_ERR_INVALID, "B1 is NULL but B_out is not");
  for (const void* p : {static_cast<const void*>(A1), static_cast<const void*>(B1), static_cast<const void*>(A2),
                        static_cast<const void*>(B2), static_cast<const void*>(A_out), static_cast<const void*>(B_out)})
    if (!aligned(p, 16)) return fail(KDN_ERR_INVALID, "affine operands must be 16-byte aligned");
  const size_t abytes = sizeof(float) * size_t(batch) * D * D;
  const size_t bbytes = B_out ? sizeof(float) * size_t(batch) * dv * D : 0;
  const void* ins[4] = {A1, B1, A2, B2};
  const size_t insz[4] = {A_out ? abytes : 0, bbytes, abytes, bbytes};
  for (int i = 0; i < 4; ++i)
    if (overlaps(A_out, A_out ? abytes : 0, ins[i], insz[i]) || overlaps(B_out, bbytes, ins[i], insz[i]))
      return fail(KDN_ERR_INVALID, "affine compose outputs overlap an input");
  if (overlaps(A_out, A_out ? abytes : 0, B_out, bbytes)) return fail(KDN_ERR_INVALID, "A_out overlaps B_out");
  cudaError_t e = kdn::launch_affine_compose(A1, B1, A2, B2, A_out, B_out, batch, D, dv,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "affine compose launch");
  return ok();
}

int kdn_affine_prefix_states(const float* A, const float* B, const float* S0, float* states, float* final_state,
                             int64_t n_c, int64_t batch, int32_t D, int32_t dv, void* stream) {
  if (int rc = check_affine_dims(batch, D, dv, true)) return rc;
  if (n_c < 0 || n_c > (int64_t(1) << 20)) return fail(KDN_ERR_INVALID, "n_c=%lld outside [0, 2^20]", (long long)n_c);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t sbytes = sizeof(float) * size_t(batch) * dv * D;
  if (n_c == 0) {
    if (!final_state) return ok();
    cudaError_t e = S0 ? (S0 == final_state ? cudaSuccess
                                            : cudaMemcpyAsync(final_state, S0, sbytes, cudaMemcpyDeviceToDevice, st))
                       : cudaMemsetAsync(final_state, 0, sbytes, st);
    if (e != cudaSuccess) return cuda_fail(e, "prefix state copy");
    return ok();
  }
  if (!A || !B || !states) return fail(KDN_ERR_INVALID, "A/B/states is NULL");
  for (const void* p : {static_cast<const void*>(A), static_cast<const void*>(B), static_cast<const void*>(S0),
                        static_cast<const void*>(states), static_cast<const void*>(final_state)})
    if (!aligned(p, 16)) return fail(KDN_ERR_INVALID, "affine operands must be 16-byte aligned");
  const size_t abytes = sizeof(float) * size_t(n_c) * batch * D * D, bbytes = sbytes * size_t(n_c);
  if (overlaps(states, bbytes, A, abytes) || overlaps(states, bbytes, B, bbytes) ||
      overlaps(final_state, sbytes, A, abytes) || overlaps(final_state, sbytes, B, bbytes) ||
      overlaps(final_state, sbytes, states, bbytes))
    return fail(KDN_ERR_INVALID, "prefix-state outputs overlap A, B or each other");
  if (S0 && S0 != states && overlaps(S0, sbytes, states, bbytes))
    return fail(KDN_ERR_INVALID, "S0 overlaps states without being states[0]");
  cudaError_t e = kdn::launch_affine_prefix_states(A, B, S0, states, final_state, n_c, batch, D, dv, st);
  if (e != cudaSuccess) return cuda_fail(e, "prefix states launch");
  return ok();
}

size_t kdn_block_transition_workspace_size(int64_t N, int64_t T, int32_t chunk, const kdn_projection* proj) {
  if (!proj || N <= 0 || T <= 0 || (chunk != 32 && chunk != 64) || proj->D < 64 || proj->D > 512) return 0;
  return kdn::simt_prefill_workspace(N, T, 0, chunk, proj->D);
}

int kdn_block_transition(const void* k, const void* v, int in_dtype, const void* beta, const void* decay,
                         int gate_dtype, float* A_out, float* B_out, int64_t N, int64_t T, int32_t dv, int32_t chunk,
                         const kdn_projection* proj, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_projection(proj)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N < 1 || N > 65535) return fail(KDN_ERR_INVALID, "N=%lld outside [1, 65535]", (long long)N);
  if (T < 0) return fail(KDN_ERR_INVALID, "T=%lld < 0", (long long)T);
  if (B_out && (dv < 16 || dv > 512 || dv % 16 != 0))
    return fail(KDN_ERR_UNSUPPORTED, "dv=%d: dv must be a multiple of 16 in [16, 512]", dv);
  if (chunk != 32 && chunk != 64) return fail(KDN_ERR_UNSUPPORTED, "chunk=%d: chunk must be 32 or 64", chunk);
  if (!valid_dtype(in_dtype) || !valid_dtype(gate_dtype)) return fail(KDN_ERR_INVALID, "bad dtype");
  if (!A_out && !B_out) return ok();
  const int D = proj->D;
  if (T == 0) {
    if (A_out) {
      cudaError_t e = kdn::launch_affine_identity(A_out, N, D, st);
      if (e != cudaSuccess) return cuda_fail(e, "identity launch");
    }
    if (B_out) {
      cudaError_t e = cudaMemsetAsync(B_out, 0, sizeof(float) * size_t(N) * dv * D, st);
      if (e != cudaSuccess) return cuda_fail(e, "zero state");
    }
    return ok();
  }
  if (!k || !beta) return fail(KDN_ERR_INVALID, "k/beta is NULL");
  if (B_out && !v) return fail(KDN_ERR_INVALID, "v is NULL but B_out is not");
  if (!aligned(k, 8)) return fail(KDN_ERR_INVALID, "k must be 8-byte aligned");
  const size_t need = kdn::simt_prefill_workspace(N, T, 0, chunk, D);
  if (!workspace || workspace_bytes < need)
    return fail(KDN_ERR_WORKSPACE, "workspace of %zu bytes given, %zu needed", workspace_bytes, need);
  if (!aligned(workspace, 256)) return fail(KDN_ERR_INVALID, "workspace must be 256-byte aligned");
  kdn::PrefillProblem p;
  p.q = nullptr;
  p.k = k;
  p.v = v;
  p.in_dtype = in_dtype;
  p.beta = beta;
  p.decay = decay;
  p.gate_dtype = gate_dtype;
  p.S0 = nullptr;
  p.y = nullptr;
  p.y_dtype = KDN_DTYPE_F32;
  p.S_out = B_out;
  p.N = N;
  p.T = T;
  p.dv = B_out ? dv : 0;
  p.C = chunk;
  p.D = D;
  p.a_rows = A_out ? D : 0;
  p.A_out = A_out;
  const kdn::ProjParams P = kdn::make_proj_params(*proj);
  kdn::LaunchMarks marks;
  cudaError_t e = kdn::launch_simt_prefill(p, P, workspace, workspace_bytes, st, marks);
  if (e != cudaSuccess) return cuda_fail(e, "block transition launch");
  return ok();
}

int kdn_decode_step(const void* q, const void* k, const void* v, int in_dtype, const void* beta, const void* decay,
                    int gate_dtype, void* states, int state_dtype, int64_t num_slots, const void* slot_mapping,
                    int index_dtype, void* out, int out_dtype, int64_t num_tokens, int32_t H, int32_t dv,
                    const kdn_projection* proj, int readout, void* stream) {
  if (int rc = check_projection(proj)) return rc;
  if (num_tokens < 0 || num_tokens > 65535)
    return fail(KDN_ERR_INVALID, "num_tokens=%lld outside [0, 65535]", (long long)num_tokens);
  if (num_tokens == 0) return ok();
  if (H < 1 || H > 65535) return fail(KDN_ERR_INVALID, "H=%d outside [1, 65535]", H);
  if (dv < 16 || dv % 16 != 0) return fail(KDN_ERR_UNSUPPORTED, "dv=%d: dv must be a positive multiple of 16", dv);
  if (num_slots < 1) return fail(KDN_ERR_INVALID, "num_slots=%lld < 1", (long long)num_slots);
  if (!q || !k || !v || !beta || !states || !slot_mapping || !out)
    return fail(KDN_ERR_INVALID, "a required pointer is NULL");
  if (!valid_dtype(in_dtype) || !valid_dtype(gate_dtype) || !valid_dtype(state_dtype) || !valid_dtype(out_dtype))
    return fail(KDN_ERR_INVALID, "bad dtype");
  if (index_dtype != KDN_INDEX_I32 && index_dtype != KDN_INDEX_I64) return fail(KDN_ERR_INVALID, "bad index dtype");
  if (readout != KDN_READOUT_PRE && readout != KDN_READOUT_POST) return fail(KDN_ERR_INVALID, "bad readout");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(states, 16))
    return fail(KDN_ERR_INVALID, "q/k/v/states must be 16-byte aligned (they are moved by bulk copies)");
  kdn::DecodeProblem p;
  p.q = q;
  p.k = k;
  p.v = v;
  p.in_dtype = in_dtype;
  p.beta = beta;
  p.decay = decay;
  p.gate_dtype = gate_dtype;
  p.states = states;
  p.state_dtype = state_dtype;
  p.num_slots = num_slots;
  p.slot_mapping = slot_mapping;
  p.index_dtype = index_dtype;
  p.out = out;
  p.out_dtype = out_dtype;
  p.num_tokens = num_tokens;
  p.H = H;
  p.dv = dv;
  p.D = proj->D;
  p.readout = readout;
  const kdn::ProjParams P = kdn::make_proj_params(*proj);
  cudaError_t e = kdn::launch_decode(p, P, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return ok();
}

int kdn_fork_state(void* states, int64_t num_slots, int64_t bytes_per_slot, int64_t parent, int64_t child,
                   void* stream) {
  if (!states) return fail(KDN_ERR_INVALID, "states is NULL");
  if (bytes_per_slot <= 0) return fail(KDN_ERR_INVALID, "bytes_per_slot=%lld", (long long)bytes_per_slot);
  if (parent < 0 || parent >= num_slots || child < 0 || child >= num_slots)
    return fail(KDN_ERR_INVALID, "slot out of range: parent=%lld child=%lld num_slots=%lld", (long long)parent,
                (long long)child, (long long)num_slots);
  if (parent == child) return ok();
  char* base = static_cast<char*>(states);
  cudaError_t e = cudaMemcpyAsync(base + child * bytes_per_slot, base + parent * bytes_per_slot,
                                  size_t(bytes_per_slot), cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "fork copy");
  return ok();
}

int kdn_device_error(void* stream, int* code_out) {
  if (!code_out) return fail(KDN_ERR_INVALID, "code_out is NULL");
  int code = 0, code_tc = 0, code_split = 0;
  cudaError_t e = kdn::decode_read_error(static_cast<cudaStream_t>(stream), &code);
  if (e != cudaSuccess) return cuda_fail(e, "device error read");
  e = kdn::tc_read_error(static_cast<cudaStream_t>(stream), &code_tc);
  if (e != cudaSuccess) return cuda_fail(e, "device error read");
  e = kdn::split_read_error(static_cast<cudaStream_t>(stream), &code_split);
  if (e != cudaSuccess) return cuda_fail(e, "device error read");
  int code_proj = 0;
  e = kdn::tp_proj_read_error(static_cast<cudaStream_t>(stream), &code_proj);
  if (e != cudaSuccess) return cuda_fail(e, "device error read");
  int code_lift = 0;
  e = kdn::lift_read_error(static_cast<cudaStream_t>(stream), &code_lift);
  if (e != cudaSuccess) return cuda_fail(e, "device error read");
  int code_attn = 0;
  e = kdn::attn_read_error(static_cast<cudaStream_t>(stream), &code_attn);
  if (e != cudaSuccess) return cuda_fail(e, "device error read");
  *code_out = code ? code
                   : (code_tc ? code_tc
                              : (code_split ? code_split : (code_proj ? code_proj : (code_lift ? code_lift : code_attn))));
  return ok();
}

}  // extern "C"
