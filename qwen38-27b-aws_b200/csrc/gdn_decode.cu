// Gated delta rule, one decode token per row: GatedDeltaNetStep.forward (qwen38_inf2/model.py:347-374).
//
// One CTA per (row, key head). A key head's q and k feed R = num_v_heads / num_k_heads value heads
// (repeat_interleave, model.py:64-67, :329-330), so the CTA convolves the key head's q/k channels
// once and owns its R value heads' state tiles and conv channels outright: no two CTAs touch the
// same state or conv state, so everything updates in place.
//
// The bf16 state tiles [R][DK][DV] (32 KB each at DK = DV = 128) stream in by one bulk copy per
// value head as soon as the CTA starts, are updated in shared memory (fp32 math), and stream back
// out by bulk copy; two CTAs fit per SM, so each SM keeps ~190 KB of state traffic in flight.
// This is the decode step's dominant HBM stream (1.57 MB per row per layer at full width).
//
// Rounding follows the reference's CPU branch: bf16 conv products and sum, bf16 SiLU; fp32 L2 norms,
// gates and recurrence (products and sums unfused, as PyTorch evaluates them); the output o rounded
// to bf16 before the gated RMS norm; bf16 after the norm, after the norm weight, and after the SiLU(z)
// gate; finally e5m2 for out_proj.
#include "gdn_common.cuh"

namespace {

using namespace q38;

struct GdnArgs {
  const __nv_bfloat16* qkvz;
  int64_t ld_qkvz;
  const __nv_bfloat16* ab;
  int64_t ld_ab;
  __nv_bfloat16* conv_state;
  const __nv_bfloat16* conv_w;
  const __nv_bfloat16* a_log;
  const __nv_bfloat16* dt_bias;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* state;
  const int32_t* position;
  const float* active;
  uint8_t* out;
  int64_t ld_out;
  int num_k_heads, num_v_heads;
  float eps;
};

template <int DK, int DV, int R>
struct GdnSmem {
  static constexpr int KCONV = 4;
  static constexpr int CH = 2 * DK + R * DV;  // channels this CTA convolves
  static constexpr size_t STATE = static_cast<size_t>(R) * DK * DV * 2;
  static constexpr size_t TOTAL = STATE + sizeof(float) * (CH + 2 * DK + 2 * R * 4 * DV + 4 * R) + 8 * R + 4 * R + 64;
};

template <int DK, int DV, int R>
__global__ void __launch_bounds__(R * 128) gdn_decode_kernel(GdnArgs a) {
  using S = GdnSmem<DK, DV, R>;
  constexpr int ROWS_W = DK / 4;   // state rows per warp of a value-head group
  constexpr int CPL = DV / 32;     // state columns per lane
  constexpr uint32_t TILE_BYTES = DK * DV * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(smem);                  // [R][DK][DV]
  float* xs = reinterpret_cast<float*>(smem + S::STATE);                        // conv+SiLU outputs [CH]
  float* qn = xs + S::CH;                                                       // [DK]
  float* kn = qn + DK;                                                          // [DK]
  float* red = kn + DK;                                                         // [R][4][DV]
  float* red2 = red + R * 4 * DV;                                               // [R][4][DV]
  float* gates = red2 + R * 4 * DV;                                             // [R][4]: beta, decay, -, -
  uint64_t* bars = reinterpret_cast<uint64_t*>(gates + 4 * R);

  const int tid = threadIdx.x;
  const int kh = blockIdx.x;
  const int b = blockIdx.y;
  const int pos = a.position[b];
  const bool on = a.active[b] > 0.5f;
  const float act = a.active[b];
  const float keep = (pos == 0 && on) ? 0.0f : 1.0f;
  const int key_dim = a.num_k_heads * DK;
  const int conv_dim = 2 * key_dim + a.num_v_heads * DV;
  const int h0 = kh * R;  // first value head of this CTA

  if (tid == 0) {
    for (int j = 0; j < R; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0 && keep != 0.0f) {
    for (int j = 0; j < R; ++j) {
      mbar_arrive_expect_tx(&bars[j], TILE_BYTES);
      bulk_load(st + static_cast<size_t>(j) * DK * DV,
                a.state + (static_cast<int64_t>(b) * a.num_v_heads + h0 + j) * DK * DV, TILE_BYTES, &bars[j]);
    }
  }

  // Causal conv over the window [conv_state * keep, new] and SiLU, for q, k and the R heads' v.
  const __nv_bfloat16* xrow = a.qkvz + b * a.ld_qkvz;
  for (int i = tid; i < S::CH; i += R * 128) {
    int c;
    if (i < DK) c = kh * DK + i;
    else if (i < 2 * DK) c = key_dim + kh * DK + (i - DK);
    else c = 2 * key_dim + h0 * DV + (i - 2 * DK);
    __nv_bfloat16* cs = a.conv_state + (static_cast<int64_t>(b) * conv_dim + c) * (S::KCONV - 1);
    const __nv_bfloat16* cw = a.conv_w + static_cast<int64_t>(c) * S::KCONV;
    float win[S::KCONV];
#pragma unroll
    for (int j = 0; j < S::KCONV - 1; ++j) win[j] = __bfloat162float(cs[j]) * keep;
    win[S::KCONV - 1] = __bfloat162float(xrow[c]);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < S::KCONV; ++j) acc = __fadd_rn(acc, bf16r(__fmul_rn(win[j], __bfloat162float(cw[j]))));
    const float conv = bf16r(acc);
    xs[i] = bf16r(__fmul_rn(conv, bf16r(sigmoidf_(conv))));
    if (on) {
#pragma unroll
      for (int j = 0; j < S::KCONV - 1; ++j) cs[j] = __float2bfloat16_rn(win[j + 1]);
    }
  }
  // Gates per value head: beta = bf16(sigmoid(b)) * active, g = -exp(A_log) * softplus(a + dt_bias) * active.
  if (tid < R) {
    const int h = h0 + tid;
    const float braw = __bfloat162float(a.ab[b * a.ld_ab + h]);
    const float araw = __bfloat162float(a.ab[b * a.ld_ab + a.num_v_heads + h]);
    const float beta = __fmul_rn(bf16r(sigmoidf_(braw)), act);
    const float g = __fmul_rn(__fmul_rn(-expf(__bfloat162float(a.a_log[h])),
                                        softplusf_(__fadd_rn(araw, __bfloat162float(a.dt_bias[h])))),
                              act);
    gates[tid * 4 + 0] = beta;
    gates[tid * 4 + 1] = expf(g);
  }
  __syncthreads();
  // L2 norms of q (then / sqrt(dk)) and k.
  const int warp = tid >> 5, lane = tid & 31;
  if (warp < 2) {
    const float* src = xs + warp * DK;
    float* dst = warp == 0 ? qn : kn;
    float ss = 0.f;
    for (int i = lane; i < DK; i += 32) ss = __fadd_rn(ss, __fmul_rn(src[i], src[i]));
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + 1e-6f);
    const float inv_scale = static_cast<float>(sqrt(static_cast<double>(DK)));  // math.sqrt(k_head) as fp32
    for (int i = lane; i < DK; i += 32) {
      const float v = __fmul_rn(src[i], r);
      dst[i] = warp == 0 ? __fdiv_rn(v, inv_scale) : v;
    }
  }
  __syncthreads();

  // Recurrence for value head j = this thread's group.
  const int j = tid >> 7;
  const int gl = tid & 127;
  const int gw = gl >> 5;  // warp within the group: rows gw*ROWS_W ..
  const int c0 = lane * CPL;
  const float beta = gates[j * 4 + 0];
  const float decay = gates[j * 4 + 1];
  // Every thread of the group observes the copy itself; a timeout in any of them is voted through
  // shared memory so the whole group leaves together (state untouched, no output).
  volatile int* failed = reinterpret_cast<volatile int*>(bars + R);
  if (gl == 0) failed[j] = 0;
  group_bar(1 + j);
  if (keep != 0.0f && !mbar_wait(&bars[j], 0)) failed[j] = 1;
  group_bar(1 + j);
  if (failed[j]) return;
  __nv_bfloat16* tile = st + static_cast<size_t>(j) * DK * DV;
  const float* vj = xs + 2 * DK + j * DV;
  float kv[CPL];
#pragma unroll
  for (int t = 0; t < CPL; ++t) kv[t] = 0.f;
#pragma unroll 4
  for (int r = 0; r < ROWS_W; ++r) {
    const int i = gw * ROWS_W + r;
    const float ki = kn[i];
    float sv[CPL];
    load_row<CPL>(tile + i * DV + c0, sv);
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const float s = keep != 0.0f ? __fmul_rn(sv[t], decay) : 0.0f;
      kv[t] = __fadd_rn(kv[t], __fmul_rn(s, ki));
    }
  }
#pragma unroll
  for (int t = 0; t < CPL; ++t) red[(j * 4 + gw) * DV + c0 + t] = kv[t];
  group_bar(1 + j);
  float delta[CPL];
#pragma unroll
  for (int t = 0; t < CPL; ++t) {
    const int c = c0 + t;
    const float kvs = __fadd_rn(__fadd_rn(__fadd_rn(red[(j * 4 + 0) * DV + c], red[(j * 4 + 1) * DV + c]),
                                          red[(j * 4 + 2) * DV + c]),
                                red[(j * 4 + 3) * DV + c]);
    delta[t] = __fmul_rn(__fsub_rn(vj[c], kvs), beta);
  }
  float o[CPL];
#pragma unroll
  for (int t = 0; t < CPL; ++t) o[t] = 0.f;
#pragma unroll 4
  for (int r = 0; r < ROWS_W; ++r) {
    const int i = gw * ROWS_W + r;
    const float ki = kn[i], qi = qn[i];
    float sv[CPL];
    load_row<CPL>(tile + i * DV + c0, sv);
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const float s = keep != 0.0f ? __fmul_rn(sv[t], decay) : 0.0f;
      sv[t] = __fadd_rn(s, __fmul_rn(ki, delta[t]));
      o[t] = __fadd_rn(o[t], __fmul_rn(sv[t], qi));
    }
    store_row<CPL>(tile + i * DV + c0, sv);
  }
#pragma unroll
  for (int t = 0; t < CPL; ++t) red2[(j * 4 + gw) * DV + c0 + t] = o[t];
  fence_proxy_async_shared();  // make the updated tile visible to the bulk copy engine
  group_bar(1 + j);
  if (gl == 0 && on) {
    bulk_store(a.state + (static_cast<int64_t>(b) * a.num_v_heads + h0 + j) * DK * DV, tile, TILE_BYTES);
    bulk_commit();
  }
  // Gated RMS norm of this head's o (bf16), times the norm weight, times SiLU(z); e5m2 out.
  if (gw == 0) {
    float ob[CPL];
    float ss = 0.f;
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const int c = c0 + t;
      const float os = __fadd_rn(__fadd_rn(__fadd_rn(red2[(j * 4 + 0) * DV + c], red2[(j * 4 + 1) * DV + c]),
                                           red2[(j * 4 + 2) * DV + c]),
                                 red2[(j * 4 + 3) * DV + c]);
      ob[t] = bf16r(os);
      ss = __fadd_rn(ss, __fmul_rn(ob[t], ob[t]));
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(DV)), a.eps));
    const __nv_bfloat16* zrow = xrow + conv_dim + (h0 + j) * DV;
    uint8_t* orow = a.out + b * a.ld_out + (h0 + j) * DV;
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const int c = c0 + t;
      const float n1 = bf16r(__fmul_rn(ob[t], r));
      const float n2 = bf16r(__fmul_rn(__bfloat162float(a.norm_w[c]), n1));
      const float z = __bfloat162float(zrow[c]);
      const float sz = __fmul_rn(z, sigmoidf_(z));
      orow[c] = f32_to_e5m2(bf16r(__fmul_rn(n2, sz)));
    }
  }
  if (gl == 0 && on) bulk_wait_read0();  // the tile must stay until the copy engine has read it
}

template <int DK, int DV, int R>
int launch_gdn(const GdnArgs& a, int64_t batch, cudaStream_t stream) {
  using S = GdnSmem<DK, DV, R>;
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gdn_decode_kernel<DK, DV, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(S::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(gdn_decode)");
    done_mask |= 1ull << dev;
  }
  dim3 grid(static_cast<unsigned>(a.num_k_heads), static_cast<unsigned>(batch));
  gdn_decode_kernel<DK, DV, R><<<grid, R * 128, S::TOTAL, stream>>>(a);
  return q38host::cuda_status(cudaGetLastError(), "gdn_decode launch");
}

}  // namespace

extern "C" int q38_gdn_decode(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                              const void* conv_weight, const void* a_log, const void* dt_bias, const void* norm_weight,
                              void* state, const int32_t* position, const float* active, void* out, int64_t ld_out,
                              int64_t batch, int num_k_heads, int num_v_heads, int head_k, int head_v,
                              int conv_kernel, float eps, q38_stream_t stream) {
  using namespace q38host;
  if (!qkvz || !ab || !conv_state || !conv_weight || !a_log || !dt_bias || !norm_weight || !state || !position ||
      !active || !out)
    return set_error("q38_gdn_decode: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads)
    return set_error("q38_gdn_decode: bad batch or head counts"), Q38_ERR_ARG;
  if (conv_kernel != 4) return set_error("q38_gdn_decode: conv kernel %d not built (4 is)", conv_kernel), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(state) & 15u) != 0)
    return set_error("q38_gdn_decode: state must be 16-byte aligned"), Q38_ERR_ARG;
  const int rep = num_v_heads / num_k_heads;
  const int64_t conv_dim = 2LL * num_k_heads * head_k + static_cast<int64_t>(num_v_heads) * head_v;
  if (ld_qkvz < conv_dim + static_cast<int64_t>(num_v_heads) * head_v || ld_ab < 2 * num_v_heads ||
      ld_out < static_cast<int64_t>(num_v_heads) * head_v)
    return set_error("q38_gdn_decode: leading dimension too small"), Q38_ERR_ARG;
  GdnArgs a{};
  a.qkvz = static_cast<const __nv_bfloat16*>(qkvz);
  a.ld_qkvz = ld_qkvz;
  a.ab = static_cast<const __nv_bfloat16*>(ab);
  a.ld_ab = ld_ab;
  a.conv_state = static_cast<__nv_bfloat16*>(conv_state);
  a.conv_w = static_cast<const __nv_bfloat16*>(conv_weight);
  a.a_log = static_cast<const __nv_bfloat16*>(a_log);
  a.dt_bias = static_cast<const __nv_bfloat16*>(dt_bias);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_weight);
  a.state = static_cast<__nv_bfloat16*>(state);
  a.position = position;
  a.active = active;
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_k_heads = num_k_heads;
  a.num_v_heads = num_v_heads;
  a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_k == 128 && head_v == 128 && rep == 3) return launch_gdn<128, 128, 3>(a, batch, s);
  if (head_k == 32 && head_v == 32 && rep == 3) return launch_gdn<32, 32, 3>(a, batch, s);
  return set_error("q38_gdn_decode: head dims %d/%d with %d value heads per key head not built", head_k, head_v, rep),
         Q38_ERR_UNSUPPORTED;
}
