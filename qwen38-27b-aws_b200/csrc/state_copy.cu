// Save / restore of one slot's recurrent states for prefix reuse: row `src_row` of every state buffer
// of the step (each gated-delta layer's recurrent state and conv state) copied to row `dst_row`, in
// one launch. Replaces GatedDeltaNetStep.copy_states (qwen38_inf2/model.py:456-464) as
// Qwen38Step.forward applies it to every layer (model.py:987-990).
//
// The copy is HBM-bound: 1.6 MB per gated-delta layer at full width (the bf16 state tile of 48 value
// heads plus the conv window), read once and written once. Blocks take 32 KB pieces of one buffer's
// row with 16-byte accesses (bytes one at a time where a row is not 16-byte aligned).
#include "q38_common.cuh"

namespace {

constexpr int kCopyBuffers = 96;        // buffers per launch (kernel parameter space); more take more launches
constexpr int kCopyThreads = 256;
constexpr int64_t kPieceBytes = 32768;  // row bytes per block

struct CopyArgs {
  uint8_t* base[kCopyBuffers];
  int64_t row_bytes[kCopyBuffers];
  int n;
  int64_t src_row, dst_row;
};

__global__ void __launch_bounds__(kCopyThreads) copy_rows_kernel(const __grid_constant__ CopyArgs a) {
  const int b = blockIdx.y;
  const int64_t rb = a.row_bytes[b];
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * kPieceBytes;
  if (b >= a.n || p0 >= rb) return;
  const int64_t p1 = min(rb, p0 + kPieceBytes);
  const uint8_t* src = a.base[b] + a.src_row * rb;
  uint8_t* dst = a.base[b] + a.dst_row * rb;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | static_cast<uintptr_t>(rb)) & 15u) == 0) {
    // Four independent 16-byte loads per thread before any store: one round trip per 16 KB.
    const int4* s = reinterpret_cast<const int4*>(src + p0);
    int4* d = reinterpret_cast<int4*>(dst + p0);
    const int64_t n = (p1 - p0) / 16;
    for (int64_t i = threadIdx.x; i < n; i += 4 * kCopyThreads) {
      int4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = i + u * kCopyThreads;
        if (j < n) v[u] = __ldcs(s + j);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t j = i + u * kCopyThreads;
        if (j < n) __stcs(d + j, v[u]);
      }
    }
  } else {
    for (int64_t i = p0 + threadIdx.x; i < p1; i += kCopyThreads) dst[i] = src[i];
  }
}

}  // namespace

extern "C" int q38_copy_state_rows(void* const* buffers, const int64_t* row_bytes, const int64_t* rows, int n_buffers,
                                   int64_t src_row, int64_t dst_row, q38_stream_t stream) {
  using namespace q38host;
  if (n_buffers < 0 || (n_buffers > 0 && (!buffers || !row_bytes || !rows)))
    return set_error("q38_copy_state_rows: %d buffers without their arrays", n_buffers), Q38_ERR_ARG;
  for (int i = 0; i < n_buffers; ++i) {
    if (!buffers[i] || row_bytes[i] <= 0 || rows[i] <= 0)
      return set_error("q38_copy_state_rows: buffer %d is null or empty", i), Q38_ERR_ARG;
    if (src_row < 0 || dst_row < 0 || src_row >= rows[i] || dst_row >= rows[i])
      return set_error("q38_copy_state_rows: rows %lld -> %lld outside buffer %d's %lld rows", (long long)src_row,
                       (long long)dst_row, i, (long long)rows[i]),
             Q38_ERR_ARG;
  }
  if (n_buffers == 0 || src_row == dst_row) return Q38_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int first = 0; first < n_buffers; first += kCopyBuffers) {
    CopyArgs a{};
    a.n = n_buffers - first < kCopyBuffers ? n_buffers - first : kCopyBuffers;
    a.src_row = src_row;
    a.dst_row = dst_row;
    int64_t wide = 0;
    for (int i = 0; i < a.n; ++i) {
      a.base[i] = static_cast<uint8_t*>(buffers[first + i]);
      a.row_bytes[i] = row_bytes[first + i];
      wide = a.row_bytes[i] > wide ? a.row_bytes[i] : wide;
    }
    const dim3 grid(static_cast<unsigned>((wide + kPieceBytes - 1) / kPieceBytes), static_cast<unsigned>(a.n));
    copy_rows_kernel<<<grid, kCopyThreads, 0, s>>>(a);
    const int st = cuda_status(cudaGetLastError(), "copy_rows_kernel launch");
    if (st != Q38_OK) return st;
  }
  return Q38_OK;
}
