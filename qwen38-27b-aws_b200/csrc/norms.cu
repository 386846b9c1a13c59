// Element-wise and row kernels around the FP8 GEMMs, each rounding where the reference rounds:
//   q38_rmsnorm_quant      rms_norm (model.py:54-57) -> bf16, and e5m2 for the next FP8 linear
//   q38_rmsnorm_divide     rms_norm, then divided by (1 + w_div): the MTP layer's output (model.py:858-860)
//   q38_silu_mul_quant     silu(gate) * up in bf16 steps (model.py:48-51, :259) -> e5m2
// All are HBM-bound; rows are read with 16-byte vector loads.
#include "q38_common.cuh"

namespace {

using namespace q38;

constexpr int kNormThreads = 256;

union Pack8 {
  uint4 u;
  __nv_bfloat16 h[8];
};

// Rows too long for registers: one CTA per row, two passes over the row (sum of squares, then scale;
// the second read hits L1/L2).
__global__ void __launch_bounds__(kNormThreads) rmsnorm_quant_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                      const __nv_bfloat16* __restrict__ w, int n,
                                                                      float eps, __nv_bfloat16* __restrict__ y,
                                                                      int64_t ldy, uint8_t* __restrict__ q,
                                                                      int64_t ldq) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  const int chunks = n / 8;
  float ss = 0.f;
  for (int c = threadIdx.x; c < chunks; c += kNormThreads) {
    Pack8 p;
    p.u = *reinterpret_cast<const uint4*>(xr + c * 8);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float f = __bfloat162float(p.h[i]);
      ss += f * f;
    }
  }
  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) total += red[i];
  const float r = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  for (int c = threadIdx.x; c < chunks; c += kNormThreads) {
    Pack8 p, pw, out;
    p.u = *reinterpret_cast<const uint4*>(xr + c * 8);
    pw.u = *reinterpret_cast<const uint4*>(w + c * 8);
    float h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float scaled = __fmul_rn(__bfloat162float(p.h[i]), r);
      h[i] = bf16r(__fmul_rn(scaled, __fadd_rn(1.0f, __bfloat162float(pw.h[i]))));
      out.h[i] = __float2bfloat16_rn(h[i]);
    }
    if (y) *reinterpret_cast<uint4*>(y + row * ldy + c * 8) = out.u;
    if (q) {
      uint2 o;
      o.x = pack4_e5m2(h[0], h[1], h[2], h[3]);
      o.y = pack4_e5m2(h[4], h[5], h[6], h[7]);
      *reinterpret_cast<uint2*>(q + row * ldq + c * 8) = o;
    }
  }
}

// One CTA of kRegThreads per row with the whole row in registers: each thread loads its PER 8-column
// chunks of x and of the weight in one batch (a single round trip), then the sum of squares, one block
// reduction, and the outputs from registers.
constexpr int kRegThreads = 128;

template <int PER>
__global__ void __launch_bounds__(kRegThreads) rmsnorm_quant_reg_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                       const __nv_bfloat16* __restrict__ w, int n,
                                                                       float eps, __nv_bfloat16* __restrict__ y,
                                                                       int64_t ldy, uint8_t* __restrict__ q, int64_t ldq) {
  pdl_wait();
  pdl_trigger();
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  const int chunks = n / 8;
  Pack8 px[PER], pw[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = threadIdx.x + k * kRegThreads;
    if (c < chunks) {
      px[k].u = *reinterpret_cast<const uint4*>(xr + c * 8);
      pw[k].u = *reinterpret_cast<const uint4*>(w + c * 8);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    if (threadIdx.x + k * kRegThreads < chunks) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float f = __bfloat162float(px[k].h[i]);
        ss += f * f;
      }
    }
  }
  __shared__ float red[kRegThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kRegThreads / 32; ++i) total += red[i];
  const float r = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = threadIdx.x + k * kRegThreads;
    if (c >= chunks) continue;
    Pack8 out;
    float h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float scaled = __fmul_rn(__bfloat162float(px[k].h[i]), r);
      h[i] = bf16r(__fmul_rn(scaled, __fadd_rn(1.0f, __bfloat162float(pw[k].h[i]))));
      out.h[i] = __float2bfloat16_rn(h[i]);
    }
    if (y) *reinterpret_cast<uint4*>(y + row * ldy + c * 8) = out.u;
    if (q) {
      uint2 o;
      o.x = pack4_e5m2(h[0], h[1], h[2], h[3]);
      o.y = pack4_e5m2(h[4], h[5], h[6], h[7]);
      *reinterpret_cast<uint2*>(q + row * ldq + c * 8) = o;
    }
  }
}

// Grid-stride over (row, 8-column chunk).
__global__ void silu_mul_quant_kernel(const __nv_bfloat16* __restrict__ gu, int64_t ld, int rows, int n,
                                      uint8_t* __restrict__ y, int64_t ldy) {
  const int chunks = n / 8;
  const int64_t total = static_cast<int64_t>(rows) * chunks;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(i / chunks);
    const int c = static_cast<int>(i % chunks);
    Pack8 g, u;
    g.u = *reinterpret_cast<const uint4*>(gu + row * ld + c * 8);
    u.u = *reinterpret_cast<const uint4*>(gu + row * ld + n + c * 8);
    float h[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) h[k] = silu_mul_bf16(__bfloat162float(g.h[k]), __bfloat162float(u.h[k]));
    uint2 o;
    o.x = pack4_e5m2(h[0], h[1], h[2], h[3]);
    o.y = pack4_e5m2(h[4], h[5], h[6], h[7]);
    *reinterpret_cast<uint2*>(y + row * ldy + c * 8) = o;
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int q38_rmsnorm_quant(const void* x, int64_t ldx, const void* w, int64_t rows, int64_t n, float eps,
                                 void* y_bf16, int64_t ldy, void* y_e5m2, int64_t ldq, q38_stream_t stream) {
  using namespace q38host;
  if (!x || !w || (!y_bf16 && !y_e5m2)) return set_error("q38_rmsnorm_quant: null pointer"), Q38_ERR_ARG;
  if (rows <= 0 || n <= 0 || n % 8 != 0 || rows > (1 << 30) || ldx < n || (y_bf16 && ldy < n) || (y_e5m2 && ldq < n))
    return set_error("q38_rmsnorm_quant: bad sizes"), Q38_ERR_ARG;
  if (!al16(x) || !al16(w) || (y_bf16 && !al16(y_bf16)) || (y_e5m2 && reinterpret_cast<uintptr_t>(y_e5m2) % 8) ||
      ldx % 8 || (y_bf16 && ldy % 8) || (y_e5m2 && ldq % 8))
    return set_error("q38_rmsnorm_quant: misaligned pointer or leading dimension"), Q38_ERR_ARG;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* yb = static_cast<__nv_bfloat16*>(y_bf16);
  auto* qb = static_cast<uint8_t*>(y_e5m2);
  const unsigned grid = static_cast<unsigned>(rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int per = static_cast<int>((n / 8 + kRegThreads - 1) / kRegThreads);
  const int ni = static_cast<int>(n);
  cudaError_t e = cudaSuccess;
  switch (per) {  // rows up to 8 * 128 * 8 = 8192 columns live in registers
    case 1: e = launch_pdl(rmsnorm_quant_reg_kernel<1>, dim3(grid), dim3(kRegThreads), 0, s, xb, ldx, wb, ni, eps, yb, ldy, qb, ldq); break;
    case 2: e = launch_pdl(rmsnorm_quant_reg_kernel<2>, dim3(grid), dim3(kRegThreads), 0, s, xb, ldx, wb, ni, eps, yb, ldy, qb, ldq); break;
    case 3: e = launch_pdl(rmsnorm_quant_reg_kernel<3>, dim3(grid), dim3(kRegThreads), 0, s, xb, ldx, wb, ni, eps, yb, ldy, qb, ldq); break;
    case 4: e = launch_pdl(rmsnorm_quant_reg_kernel<4>, dim3(grid), dim3(kRegThreads), 0, s, xb, ldx, wb, ni, eps, yb, ldy, qb, ldq); break;
    case 5: e = launch_pdl(rmsnorm_quant_reg_kernel<5>, dim3(grid), dim3(kRegThreads), 0, s, xb, ldx, wb, ni, eps, yb, ldy, qb, ldq); break;
    case 6:
    case 7:
    case 8: e = launch_pdl(rmsnorm_quant_reg_kernel<8>, dim3(grid), dim3(kRegThreads), 0, s, xb, ldx, wb, ni, eps, yb, ldy, qb, ldq); break;
    default:
      e = launch_pdl(rmsnorm_quant_kernel, dim3(grid), dim3(kNormThreads), 0, s, xb, ldx, wb, ni, eps, yb, ldy, qb, ldq);
  }
  return cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "rmsnorm_quant launch");
}

extern "C" int q38_silu_mul_quant(const void* gu, int64_t ld, int64_t rows, int64_t n, void* y_e5m2, int64_t ldy,
                                  q38_stream_t stream) {
  using namespace q38host;
  if (!gu || !y_e5m2) return set_error("q38_silu_mul_quant: null pointer"), Q38_ERR_ARG;
  if (rows <= 0 || n <= 0 || n % 8 || ld < 2 * n || ldy < n || ld % 8 || ldy % 8 || !al16(gu) ||
      reinterpret_cast<uintptr_t>(y_e5m2) % 8)
    return set_error("q38_silu_mul_quant: bad sizes or alignment"), Q38_ERR_ARG;
  const int64_t work = rows * (n / 8);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((work + 255) / 256, 148 * 16));
  silu_mul_quant_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gu), ld, static_cast<int>(rows), static_cast<int>(n),
      static_cast<uint8_t*>(y_e5m2), ldy);
  return cuda_status(cudaGetLastError(), "silu_mul_quant launch");
}

// y = bf16(bf16(rms_norm(x) * (1 + w)) / (1 + w_div)) per row: MTPStep's output, its own norm divided by
// (1 + the final norm's weight) in fp32 (qwen38_inf2/model.py:858-860), so the head's final norm recovers
// what the layer predicts.
namespace {
__global__ void __launch_bounds__(kNormThreads) rmsnorm_divide_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                                                      const __nv_bfloat16* __restrict__ w,
                                                                      const __nv_bfloat16* __restrict__ w_div, int n,
                                                                      float eps, __nv_bfloat16* __restrict__ y,
                                                                      int64_t ldy) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += kNormThreads) {
    const float f = __bfloat162float(xr[i]);
    ss += f * f;
  }
  __shared__ float red[kNormThreads / 32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) total += red[i];
  const float r = 1.0f / sqrtf(total / static_cast<float>(n) + eps);
  for (int i = threadIdx.x; i < n; i += kNormThreads) {
    const float h = bf16r(__fmul_rn(__fmul_rn(__bfloat162float(xr[i]), r), __fadd_rn(1.0f, __bfloat162float(w[i]))));
    y[row * ldy + i] = __float2bfloat16_rn(__fdiv_rn(h, __fadd_rn(1.0f, __bfloat162float(w_div[i]))));
  }
}
}  // namespace

extern "C" int q38_rmsnorm_divide(const void* x, int64_t ldx, const void* w, const void* w_div, int64_t rows, int64_t n,
                                  float eps, void* y, int64_t ldy, q38_stream_t stream) {
  using namespace q38host;
  if (!x || !w || !w_div || !y) return set_error("q38_rmsnorm_divide: null pointer"), Q38_ERR_ARG;
  if (rows <= 0 || rows > (1 << 30) || n <= 0 || n > (1 << 20) || ldx < n || ldy < n)
    return set_error("q38_rmsnorm_divide: bad sizes"), Q38_ERR_ARG;
  const cudaError_t e = launch_pdl(rmsnorm_divide_kernel, dim3(static_cast<unsigned>(rows)), dim3(kNormThreads), 0,
                                   static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x), ldx,
                                   static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(w_div),
                                   static_cast<int>(n), eps, static_cast<__nv_bfloat16*>(y), ldy);
  return cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "rmsnorm_divide launch");
}
