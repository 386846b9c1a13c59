// Gated delta rule, one decode token per row: GatedDeltaNetStep.forward (qwen38_inf2/model.py:347-374).
//
// Two launches. First, one small CTA per (row, key head) convolves the key head's q and k channels
// once (A key head's q and k feed R = num_v_heads / num_k_heads value heads: repeat_interleave,
// model.py:64-67, :329-330), L2-normalises them into a workspace and updates their conv state.
// Then one CTA of 128 threads per (row, value head) owns that head's state tile and v channels
// outright, so everything updates in place with no race: its bf16 state tile (32 KB at DK = DV = 128)
// streams in by one bulk copy, is updated in shared memory (fp32 math) and streams back out. A CTA
// holds ~37 KB of shared memory, so several share an SM and the state traffic of some overlaps the
// arithmetic of others; this is the decode step's dominant HBM stream (1.57 MB per row per layer at
// full width).
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
  int num_k_heads, num_v_heads, head_v;
  float eps;
};

// Kernel 1, one CTA of DK threads per (row, key head): the causal conv and SiLU of the key head's
// q and k channels, their L2 norms, the normalised q (/ sqrt(dk)) and k into the workspace
// [row][key head][q | k][DK] (fp32), and the q/k channels' conv-state update.
template <int DK>
__global__ void __launch_bounds__(DK) gdn_qk_kernel(GdnArgs a, float* qk) {
  constexpr int KCONV = 4;
  constexpr int NW = DK / 32;
  __shared__ float part[2][NW];
  pdl_wait();
  pdl_trigger();
  const int kh = blockIdx.x, b = blockIdx.y, i = threadIdx.x, warp = i >> 5, lane = i & 31;
  const int pos = a.position[b];
  const bool on = a.active[b] > 0.5f;
  const float keep = (pos == 0 && on) ? 0.0f : 1.0f;
  const int key_dim = a.num_k_heads * DK;
  const int conv_dim = 2 * key_dim + a.num_v_heads * a.head_v;
  const __nv_bfloat16* xrow = a.qkvz + b * a.ld_qkvz;
  // Both channels' loads before any store: one round trip.
  float win[2][KCONV], cwv[2][KCONV];
  __nv_bfloat16* cs[2];
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const int c = which * key_dim + kh * DK + i;
    cs[which] = a.conv_state + (static_cast<int64_t>(b) * conv_dim + c) * (KCONV - 1);
    const __nv_bfloat16* cw = a.conv_w + static_cast<int64_t>(c) * KCONV;
#pragma unroll
    for (int j = 0; j < KCONV - 1; ++j) win[which][j] = __bfloat162float(cs[which][j]) * keep;
    win[which][KCONV - 1] = __bfloat162float(xrow[c]);
#pragma unroll
    for (int j = 0; j < KCONV; ++j) cwv[which][j] = __bfloat162float(cw[j]);
  }
  float val[2];
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < KCONV; ++j) acc = __fadd_rn(acc, bf16r(__fmul_rn(win[which][j], cwv[which][j])));
    const float conv = bf16r(acc);
    val[which] = bf16r(__fmul_rn(conv, bf16r(sigmoidf_(conv))));
    if (on) {
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) cs[which][j] = __float2bfloat16_rn(win[which][j + 1]);
    }
  }
  float sq = warp_sum(__fmul_rn(val[0], val[0])), sk = warp_sum(__fmul_rn(val[1], val[1]));
  if (lane == 0) {
    part[0][warp] = sq;
    part[1][warp] = sk;
  }
  __syncthreads();
  sq = 0.f;
  sk = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    sq = __fadd_rn(sq, part[0][w]);
    sk = __fadd_rn(sk, part[1][w]);
  }
  const float inv_scale = static_cast<float>(sqrt(static_cast<double>(DK)));  // math.sqrt(k_head) as fp32
  float* dst = qk + (static_cast<int64_t>(b) * a.num_k_heads + kh) * 2 * DK;
  dst[i] = __fdiv_rn(__fmul_rn(val[0], 1.0f / sqrtf(sq + 1e-6f)), inv_scale);
  dst[DK + i] = __fmul_rn(val[1], 1.0f / sqrtf(sk + 1e-6f));
}

template <int DK, int DV>
struct GdnSmem {
  static constexpr size_t TILE = static_cast<size_t>(DK) * DV * 2;
  static constexpr size_t TOTAL = TILE + sizeof(float) * (DV + 2 * DK + 4 * DV + 4) + 2 * 2 * DV + 16;
};

// Kernel 2, one CTA of 128 threads per (row, value head): the head's v conv, gates, the recurrence on
// its 32 KB state tile (bulk copy in, fp32 math in shared memory, bulk copy out), and the gated norm.
// Small CTAs, several per SM, so the state traffic of some overlaps the arithmetic of others.
template <int DK, int DV>
__global__ void __launch_bounds__(128) gdn_decode_kernel(GdnArgs a, const float* qk) {
  using S = GdnSmem<DK, DV>;
  constexpr int KCONV = 4;
  constexpr int ROWS_W = DK / 4;  // state rows per warp
  constexpr int CPL = DV / 32;    // state columns per lane
  constexpr uint32_t TILE_BYTES = DK * DV * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(smem);
  float* xv = reinterpret_cast<float*>(smem + S::TILE);  // [DV] conv + SiLU of v
  float* qn = xv + DV;                                   // [DK]
  float* kn = qn + DK;                                   // [DK]
  float* red = kn + DK;                                  // [4][DV], both reductions in turn
  float* gates = red + 4 * DV;                           // beta, decay
  __nv_bfloat16* nws = reinterpret_cast<__nv_bfloat16*>(gates + 4);  // [DV] norm weight
  __nv_bfloat16* zs = nws + DV;                                      // [DV] z
  uint64_t* bar = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(zs + DV) + 7) & ~uintptr_t(7));

  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int R = a.num_v_heads / a.num_k_heads;
  const int kh = h / R;
  const int pos = a.position[b];
  const bool on = a.active[b] > 0.5f;
  const float act = a.active[b];
  const float keep = (pos == 0 && on) ? 0.0f : 1.0f;
  const int key_dim = a.num_k_heads * DK;
  const int conv_dim = 2 * key_dim + a.num_v_heads * DV;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    if (keep != 0.0f) {
      mbar_arrive_expect_tx(bar, TILE_BYTES);
      bulk_load(tile, a.state + (static_cast<int64_t>(b) * a.num_v_heads + h) * DK * DV, TILE_BYTES, bar);
    }
  }
  // Every input of the head, loaded into registers before any store so the whole prologue is one
  // round trip: the v channels' conv window and weights, the normalised q / k, the norm weight, z and
  // the gate inputs.
  constexpr int VN = (DV + 127) / 128;      // v channels per thread
  constexpr int QN = (2 * DK + 127) / 128;  // q / k values per thread
  const __nv_bfloat16* xrow = a.qkvz + b * a.ld_qkvz;
  const __nv_bfloat16* zrow = xrow + conv_dim + h * DV;
  const float* qkrow = qk + (static_cast<int64_t>(b) * a.num_k_heads + kh) * 2 * DK;
  float win[VN][KCONV], cwv[VN][KCONV], qkr[QN], graw[4];
  __nv_bfloat16 nwr[VN], zr[VN];
  __nv_bfloat16* csp[VN];
#pragma unroll
  for (int v = 0; v < VN; ++v) {
    const int i = tid + 128 * v;
    if (i < DV) {
      const int c = 2 * key_dim + h * DV + i;
      csp[v] = a.conv_state + (static_cast<int64_t>(b) * conv_dim + c) * (KCONV - 1);
      const __nv_bfloat16* cw = a.conv_w + static_cast<int64_t>(c) * KCONV;
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) win[v][j] = __bfloat162float(csp[v][j]) * keep;
      win[v][KCONV - 1] = __bfloat162float(xrow[c]);
#pragma unroll
      for (int j = 0; j < KCONV; ++j) cwv[v][j] = __bfloat162float(cw[j]);
      nwr[v] = a.norm_w[i];
      zr[v] = zrow[i];
    }
  }
#pragma unroll
  for (int k = 0; k < QN; ++k)
    if (tid + 128 * k < 2 * DK) qkr[k] = qkrow[tid + 128 * k];
  if (tid == 0) {
    graw[0] = __bfloat162float(a.ab[b * a.ld_ab + h]);
    graw[1] = __bfloat162float(a.ab[b * a.ld_ab + a.num_v_heads + h]);
    graw[2] = __bfloat162float(a.a_log[h]);
    graw[3] = __bfloat162float(a.dt_bias[h]);
  }
  // Thread 0's barrier initialisation is visible to every thread before any waits on it (an mbarrier
  // must be initialised before any other operation on it; the shared memory may still hold a previous
  // CTA's data).
  __syncthreads();
  // v conv + SiLU for this head's DV channels; the conv state moves on.
#pragma unroll
  for (int v = 0; v < VN; ++v) {
    const int i = tid + 128 * v;
    if (i < DV) {
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < KCONV; ++j) acc = __fadd_rn(acc, bf16r(__fmul_rn(win[v][j], cwv[v][j])));
      const float conv = bf16r(acc);
      xv[i] = bf16r(__fmul_rn(conv, bf16r(sigmoidf_(conv))));
      nws[i] = nwr[v];
      zs[i] = zr[v];
      if (on) {
#pragma unroll
        for (int j = 0; j < KCONV - 1; ++j) csp[v][j] = __float2bfloat16_rn(win[v][j + 1]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < QN; ++k)
    if (tid + 128 * k < 2 * DK) qn[tid + 128 * k] = qkr[k];  // qn then kn, adjacent
  // Gates: beta = bf16(sigmoid(b)) * active, g = -exp(A_log) * softplus(a + dt_bias) * active.
  if (tid == 0) {
    const float beta = __fmul_rn(bf16r(sigmoidf_(graw[0])), act);
    const float g = __fmul_rn(__fmul_rn(-expf(graw[2]), softplusf_(__fadd_rn(graw[1], graw[3]))), act);
    gates[0] = beta;
    gates[1] = expf(g);
  }
  const bool ok = keep == 0.0f || mbar_wait(bar, 0);
  if (__syncthreads_or(!ok)) return;  // the copy timed out (recorded): state untouched, no output

  const int c0 = lane * CPL;
  const float beta = gates[0];
  const float decay = gates[1];
  float kv[CPL];
#pragma unroll
  for (int t = 0; t < CPL; ++t) kv[t] = 0.f;
#pragma unroll 4
  for (int r = 0; r < ROWS_W; ++r) {
    const int i = warp * ROWS_W + r;
    const float ki = kn[i];
    float sv[CPL];
    load_row<CPL>(tile + i * DV + c0, sv);
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const float sx = keep != 0.0f ? __fmul_rn(sv[t], decay) : 0.0f;
      kv[t] = __fadd_rn(kv[t], __fmul_rn(sx, ki));
    }
  }
#pragma unroll
  for (int t = 0; t < CPL; ++t) red[warp * DV + c0 + t] = kv[t];
  __syncthreads();
  float delta[CPL];
#pragma unroll
  for (int t = 0; t < CPL; ++t) {
    const int c = c0 + t;
    const float kvs = __fadd_rn(__fadd_rn(__fadd_rn(red[0 * DV + c], red[1 * DV + c]), red[2 * DV + c]), red[3 * DV + c]);
    delta[t] = __fmul_rn(__fsub_rn(xv[c], kvs), beta);
  }
  __syncthreads();  // the reduction buffer is read; the second reduction reuses it
  float o[CPL];
#pragma unroll
  for (int t = 0; t < CPL; ++t) o[t] = 0.f;
#pragma unroll 4
  for (int r = 0; r < ROWS_W; ++r) {
    const int i = warp * ROWS_W + r;
    const float ki = kn[i], qi = qn[i];
    float sv[CPL];
    load_row<CPL>(tile + i * DV + c0, sv);
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const float sx = keep != 0.0f ? __fmul_rn(sv[t], decay) : 0.0f;
      sv[t] = __fadd_rn(sx, __fmul_rn(ki, delta[t]));
      o[t] = __fadd_rn(o[t], __fmul_rn(sv[t], qi));
    }
    store_row<CPL>(tile + i * DV + c0, sv);
  }
#pragma unroll
  for (int t = 0; t < CPL; ++t) red[warp * DV + c0 + t] = o[t];
  fence_proxy_async_shared();  // make the updated tile visible to the bulk copy engine
  __syncthreads();
  if (tid == 0 && on) {
    bulk_store(a.state + (static_cast<int64_t>(b) * a.num_v_heads + h) * DK * DV, tile, TILE_BYTES);
    bulk_commit();
  }
  // Gated RMS norm of this head's o (bf16), times the norm weight, times SiLU(z); e5m2 out.
  if (warp == 0) {
    float ob[CPL];
    float ss = 0.f;
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const int c = c0 + t;
      const float os = __fadd_rn(__fadd_rn(__fadd_rn(red[0 * DV + c], red[1 * DV + c]), red[2 * DV + c]), red[3 * DV + c]);
      ob[t] = bf16r(os);
      ss = __fadd_rn(ss, __fmul_rn(ob[t], ob[t]));
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(DV)), a.eps));
    uint8_t* orow = a.out + b * a.ld_out + h * DV;
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const int c = c0 + t;
      const float n1 = bf16r(__fmul_rn(ob[t], r));
      const float n2 = bf16r(__fmul_rn(__bfloat162float(nws[c]), n1));
      const float z = __bfloat162float(zs[c]);
      const float sz = __fmul_rn(z, sigmoidf_(z));
      orow[c] = f32_to_e5m2(bf16r(__fmul_rn(n2, sz)));
    }
  }
  if (tid == 0 && on) bulk_wait_read0();  // the tile must stay until the copy engine has read it
}

template <int DK, int DV>
int launch_gdn(const GdnArgs& a, int64_t batch, float* qk, cudaStream_t stream) {
  using S = GdnSmem<DK, DV>;
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gdn_decode_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(S::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(gdn_decode)");
    done_mask |= 1ull << dev;
  }
  e = q38host::launch_pdl(gdn_qk_kernel<DK>, dim3(a.num_k_heads, static_cast<unsigned>(batch)), dim3(DK), 0, stream, a,
                          qk);
  if (e != cudaSuccess) return q38host::cuda_status(e, "gdn_qk launch");
  e = q38host::launch_pdl(gdn_decode_kernel<DK, DV>, dim3(a.num_v_heads, static_cast<unsigned>(batch)), dim3(128),
                          S::TOTAL, stream, a, static_cast<const float*>(qk));
  return q38host::cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "gdn_decode launch");
}

}  // namespace

extern "C" size_t q38_gdn_decode_workspace_bytes(int64_t batch, int num_k_heads, int head_k) {
  if (batch <= 0 || num_k_heads <= 0 || head_k <= 0) return 0;
  return sizeof(float) * static_cast<size_t>(batch) * num_k_heads * 2 * head_k;
}

extern "C" int q38_gdn_decode(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                              const void* conv_weight, const void* a_log, const void* dt_bias, const void* norm_weight,
                              void* state, const int32_t* position, const float* active, void* out, int64_t ld_out,
                              int64_t batch, int num_k_heads, int num_v_heads, int head_k, int head_v,
                              int conv_kernel, float eps, void* workspace, size_t workspace_bytes,
                              q38_stream_t stream) {
  using namespace q38host;
  if (!qkvz || !ab || !conv_state || !conv_weight || !a_log || !dt_bias || !norm_weight || !state || !position ||
      !active || !out || !workspace)
    return set_error("q38_gdn_decode: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads)
    return set_error("q38_gdn_decode: bad batch or head counts"), Q38_ERR_ARG;
  if (conv_kernel != 4) return set_error("q38_gdn_decode: conv kernel %d not built (4 is)", conv_kernel), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(state) & 15u) != 0)
    return set_error("q38_gdn_decode: state must be 16-byte aligned"), Q38_ERR_ARG;
  if (workspace_bytes < q38_gdn_decode_workspace_bytes(batch, num_k_heads, head_k) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15u) != 0)
    return set_error("q38_gdn_decode: workspace needs %zu bytes, 16-byte aligned",
                     q38_gdn_decode_workspace_bytes(batch, num_k_heads, head_k)),
           Q38_ERR_ARG;
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
  a.head_v = head_v;
  a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* qk = static_cast<float*>(workspace);
  if (head_k == 128 && head_v == 128 && rep == 3) return launch_gdn<128, 128>(a, batch, qk, s);
  if (head_k == 32 && head_v == 32 && rep == 3) return launch_gdn<32, 32>(a, batch, qk, s);
  return set_error("q38_gdn_decode: head dims %d/%d with %d value heads per key head not built", head_k, head_v, rep),
         Q38_ERR_UNSUPPORTED;
}
