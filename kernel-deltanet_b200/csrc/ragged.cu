// ragged.cu -- layout change of a ragged (packed) batch for the prefill kernels.
//
// A serving batch packs sequences back to back: element (sequence i, token t, head h) of a
// [total_tokens, H, w] tensor sits at ((cu[i] + t) * H + h) * w, with cu the cumulative
// sequence lengths (cu[0] = 0, cu[num_seqs] = total_tokens).  The prefill kernels read one
// sequence's heads as [H, T_i, w] (head-major); this kernel moves rows between the two
// layouts without padding: sequence i's head-major block starts at cu[i] * H * w.
//   to_head_major = 1: packed -> head-major;  0: head-major -> packed.
// One warp per token row; each (token, head) row is w contiguous elements in both layouts.
#include "kdn_internal.h"

namespace kdn {
namespace {

template <typename IDX>
__device__ __forceinline__ int64_t seq_of(const IDX* cu, int64_t num_seqs, int64_t row) {
  int64_t lo = 0, hi = num_seqs;  // largest i with cu[i] <= row
  while (hi - lo > 1) {
    const int64_t mid = (lo + hi) >> 1;
    if (int64_t(cu[mid]) <= row) lo = mid;
    else hi = mid;
  }
  return lo;
}

template <typename IDX>
__global__ void __launch_bounds__(256) ragged_transpose_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                                                             const IDX* __restrict__ cu, int64_t num_seqs,
                                                             int64_t total, int H, int64_t row_bytes,
                                                             int to_head_major, bool vec16) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t row = warp; row < total; row += nwarps) {
    const int64_t i = seq_of(cu, num_seqs, row);
    const int64_t c0 = int64_t(cu[i]), c1 = int64_t(cu[i + 1]), Ti = c1 - c0, t = row - c0;
    // malformed offsets (negative, decreasing or past the end): touch nothing
    if (c0 < 0 || c1 < c0 || c1 > total || t < 0 || t >= Ti) continue;
    for (int h = 0; h < H; ++h) {
      const int64_t packed = (row * H + h) * row_bytes;
      const int64_t hm = (c0 * H + int64_t(h) * Ti + t) * row_bytes;
      const uint8_t* s = src + (to_head_major ? packed : hm);
      uint8_t* d = dst + (to_head_major ? hm : packed);
      if (vec16) {  // rows of whole 16-byte vectors on 16-byte aligned bases
        for (int64_t o = 16 * lane; o < row_bytes; o += 512)
          *reinterpret_cast<uint4*>(d + o) = *reinterpret_cast<const uint4*>(s + o);
      } else {
        for (int64_t o = lane; o < row_bytes; o += 32) d[o] = s[o];
      }
    }
  }
}

}  // namespace

cudaError_t launch_ragged_transpose(const void* src, void* dst, const void* cu_seqlens, int index_dtype,
                                    int64_t num_seqs, int64_t total_tokens, int H, int64_t row_bytes,
                                    int to_head_major, cudaStream_t stream) {
  if (total_tokens == 0) return cudaSuccess;
  int64_t blocks = (total_tokens + 7) / 8;  // 8 warps per block, one row each
  if (blocks > 148 * 16) blocks = 148 * 16;
  const uint8_t* s = static_cast<const uint8_t*>(src);
  uint8_t* d = static_cast<uint8_t*>(dst);
  const bool vec16 = (row_bytes % 16) == 0 && (reinterpret_cast<uintptr_t>(s) % 16) == 0 &&
                     (reinterpret_cast<uintptr_t>(d) % 16) == 0;
  if (index_dtype == KDN_INDEX_I64)
    ragged_transpose_kernel<int64_t><<<unsigned(blocks), 256, 0, stream>>>(
        s, d, static_cast<const int64_t*>(cu_seqlens), num_seqs, total_tokens, H, row_bytes, to_head_major, vec16);
  else
    ragged_transpose_kernel<int32_t><<<unsigned(blocks), 256, 0, stream>>>(
        s, d, static_cast<const int32_t*>(cu_seqlens), num_seqs, total_tokens, H, row_bytes, to_head_major, vec16);
  return cudaGetLastError();
}

}  // namespace kdn
