// Pieces shared by the decode and prefill attention kernels.
#pragma once

#include <cuda_fp8.h>

#include "q38_common.cuh"

namespace q38 {

// The FP8 e4m3 KV cache with static scales (qwen38_inf2/model.py:579-593): the cache holds e4m3 bytes of
// value / scale clamped to +-240 (the reference's FP8_E4M3_MAX, model.py:37-41), and reads back as
// bf16(e4m3 * scale).
constexpr float kKvFp8Max = 240.0f;
__device__ __forceinline__ float fp8_load(uint8_t b, float scale) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(b), __NV_E4M3);
  return bf16r(__fmul_rn(__half2float(__half(h)), scale));
}
__device__ __forceinline__ uint8_t fp8_store(float x, float scale) {
  const float v = fminf(fmaxf(__fdiv_rn(x, scale), -kKvFp8Max), kKvFp8Max);
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
// Sixteen e4m3 bytes decoded to sixteen bf16 values (two 16-byte pieces).
__device__ __forceinline__ void fp8_load16(const uint4& v, float scale, uint4& lo, uint4& hi) {
  const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
  uint32_t* l = reinterpret_cast<uint32_t*>(&lo);
  uint32_t* h = reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    l[e] = pack_bf16x2(fp8_load(b[2 * e], scale), fp8_load(b[2 * e + 1], scale));
    h[e] = pack_bf16x2(fp8_load(b[8 + 2 * e], scale), fp8_load(b[8 + 2 * e + 1], scale));
  }
}

// RMS norm (1 + w) of one head held by a warp (values in smem, in place), then partial rotary on
// the first `rot` dims: bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)) (model.py:54-57, :70-82).
template <int HD>
__device__ void norm_rope_head(float* x, const __nv_bfloat16* w, const __nv_bfloat16* cs, const __nv_bfloat16* sn,
                               int rot, float eps, int lane) {
  float ss = 0.f;
  for (int d = lane; d < HD; d += 32) ss = __fadd_rn(ss, __fmul_rn(x[d], x[d]));
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(HD)), eps));
  for (int d = lane; d < HD; d += 32)
    x[d] = bf16r(__fmul_rn(__fmul_rn(x[d], r), __fadd_rn(1.0f, __bfloat162float(w[d]))));
  __syncwarp();
  float roped[HD / 32 > 0 ? HD / 32 : 1];
  const int half = rot / 2;
  int n = 0;
  for (int d = lane; d < HD; d += 32, ++n) {
    if (d < rot) {
      const float rh = d < half ? -x[d + half] : x[d - half];
      roped[n] = bf16r(__fadd_rn(bf16r(__fmul_rn(x[d], __bfloat162float(cs[d]))),
                                 bf16r(__fmul_rn(rh, __bfloat162float(sn[d])))));
    } else {
      roped[n] = x[d];
    }
  }
  __syncwarp();
  n = 0;
  for (int d = lane; d < HD; d += 32, ++n) x[d] = roped[n];
  __syncwarp();
}

// ---------------------------------------------------------------------------------------------
// Warp-level BF16 tensor-core pieces (mma.sync m16n8k16, fp32 accumulate) and cp.async.
// ---------------------------------------------------------------------------------------------
// Four 8x8 b16 matrices from shared memory; lane l gives the address of row l % 8 of matrix l / 8.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
// D[16x8] += A[16x16] (row) * B[16x8] (col), bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 16-byte asynchronous copy global -> shared; src_bytes 0 fills the destination with zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace q38
