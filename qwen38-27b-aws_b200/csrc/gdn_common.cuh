// Pieces shared by the gated-delta decode and verify kernels.
#pragma once

#include "q38_common.cuh"

namespace q38 {

__device__ __forceinline__ void group_bar(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }

// CPL consecutive bf16 of a state row, as one vector access when CPL == 4 (8 bytes, conflict-free
// across a warp's 32 lanes), element by element otherwise.
template <int CPL>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[CPL]) {
  if constexpr (CPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    v[0] = __low2float(a);
    v[1] = __high2float(a);
    v[2] = __low2float(b);
    v[3] = __high2float(b);
  } else {
#pragma unroll
    for (int t = 0; t < CPL; ++t) v[t] = __bfloat162float(p[t]);
  }
}
template <int CPL>
__device__ __forceinline__ void store_row(__nv_bfloat16* p, const float (&v)[CPL]) {
  if constexpr (CPL == 4) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
#pragma unroll
    for (int t = 0; t < CPL; ++t) p[t] = __float2bfloat16_rn(v[t]);
  }
}

}  // namespace q38
