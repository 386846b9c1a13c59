// Pieces shared by the decode and prefill attention kernels.
#pragma once

#include "q38_common.cuh"

namespace q38 {

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

}  // namespace q38
