// Gated full attention, one decode token per row over a BF16 KV cache:
// FullAttentionStep._project + forward (qwen38_inf2/model.py:565-577, :610-639).
//
// One CTA per (row, KV head) with its G query heads. The reference computes the scores as a BF16
// matmul (fp32 sums rounded to bf16), a fp32 softmax over cache positions < position plus the
// token's own key, weights rounded to bf16, and the output as a BF16 matmul plus the own value's
// bf16 term. This kernel keeps those rounding points, so it takes two passes: scores for every
// visible position into shared memory (K streamed once), then the normalised weights against V
// (V streamed once). It is HBM-bound on the cache: position * head_dim * 4 bytes per (row, KV head).
#include "attn_common.cuh"

namespace {

using namespace q38;

constexpr int kThreads = 256;
constexpr int kMaxGroups = 8;

struct AttnArgs {
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t max_seq;
  const int32_t* position;
  const float* active;
  uint8_t* out;
  int64_t ld_out;
  int num_q_heads, num_kv_heads, groups, rot;
  float eps;
};

template <int HD>
struct AttnSmem {
  static constexpr int DPL = HD / 32;               // dims per lane in pass 1
  static constexpr int CHUNKS = HD / 8;             // 8-dim chunks of a row
  static constexpr int PGROUPS = kThreads / CHUNKS; // position groups in pass 2
  static size_t bytes(int groups, int64_t max_seq) {
    return sizeof(float) * (static_cast<size_t>(groups) * HD * 2 + 2 * HD + static_cast<size_t>(groups) * max_seq +
                            static_cast<size_t>(PGROUPS) * groups * HD + 4 * kMaxGroups);
  }
};

union Pack8 {
  uint4 u;
  __nv_bfloat16 h[8];
};

template <int HD>
__global__ void __launch_bounds__(kThreads) attn_decode_kernel(AttnArgs a) {
  using S = AttnSmem<HD>;
  extern __shared__ __align__(16) float sm[];
  const int G = a.groups;
  float* qf = sm;                              // [G][HD] normed, roped queries
  float* gate = qf + G * HD;                   // [G][HD] gate values
  float* kown = gate + G * HD;                 // [HD]
  float* vown = kown + HD;                     // [HD]
  float* sc = vown + HD;                       // [G][max_seq] scores, then weights
  float* part = sc + G * a.max_seq;            // [PGROUPS][G][HD]
  float* hs = part + S::PGROUPS * G * HD;      // [kMaxGroups] own weights; [kMaxGroups..] spare

  const int g = blockIdx.x;
  const int b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool on = a.active[b] > 0.5f;
  const int pos = a.position[b];
  const int64_t pos64 = pos < 0 ? 0 : pos;
  const int n_read = on ? static_cast<int>(pos64 < a.max_seq ? pos64 : a.max_seq) : 0;
  const int64_t where = on ? (pos64 < a.max_seq - 1 ? pos64 : a.max_seq - 1) : a.max_seq - 1;
  const __nv_bfloat16* row = a.qkv + b * a.ld_qkv;
  const int qh0 = g * G;

  // Stage the raw query heads, gates, own key and value.
  for (int i = tid; i < G * HD; i += kThreads) {
    const int h = i / HD, d = i % HD;
    const __nv_bfloat16* base = row + static_cast<int64_t>(qh0 + h) * 2 * HD;
    qf[i] = __bfloat162float(base[d]);
    gate[i] = __bfloat162float(base[HD + d]);
  }
  const __nv_bfloat16* kraw = row + static_cast<int64_t>(a.num_q_heads) * 2 * HD + static_cast<int64_t>(g) * HD;
  const __nv_bfloat16* vraw = kraw + static_cast<int64_t>(a.num_kv_heads) * HD;
  for (int d = tid; d < HD; d += kThreads) {
    kown[d] = __bfloat162float(kraw[d]);
    vown[d] = __bfloat162float(vraw[d]);
  }
  __syncthreads();
  const __nv_bfloat16* cs = a.cos + b * a.rot;
  const __nv_bfloat16* sn = a.sin + b * a.rot;
  for (int h = warp; h <= G; h += kThreads / 32) {
    if (h < G) norm_rope_head<HD>(qf + h * HD, a.q_norm_w, cs, sn, a.rot, a.eps, lane);
    else norm_rope_head<HD>(kown, a.k_norm_w, cs, sn, a.rot, a.eps, lane);
  }
  __syncthreads();

  // Pass 1: bf16-rounded scores of every visible cached position, one position per warp step.
  const __nv_bfloat16* kc = a.k_cache + (static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq * HD;
  const __nv_bfloat16* vc = a.v_cache + (static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq * HD;
  {
    float qreg[kMaxGroups][S::DPL];
#pragma unroll
    for (int h = 0; h < kMaxGroups; ++h)
#pragma unroll
      for (int e = 0; e < S::DPL; ++e) qreg[h][e] = h < G ? qf[h * HD + lane * S::DPL + e] : 0.f;
    // Each warp takes 4 consecutive positions per step and loads their K rows before using them, so
    // each warp keeps 4 rows (2 KB at head_dim 256) in flight.
    constexpr int PW = 4;
    for (int p0 = warp * PW; p0 < n_read; p0 += (kThreads / 32) * PW) {
      float kv[PW][S::DPL];
#pragma unroll
      for (int u = 0; u < PW; ++u) {
        const int p = min(p0 + u, n_read - 1);
        if constexpr (S::DPL == 8) {
          Pack8 pk;
          pk.u = __ldg(reinterpret_cast<const uint4*>(kc + static_cast<int64_t>(p) * HD + lane * 8));
#pragma unroll
          for (int e = 0; e < 8; ++e) kv[u][e] = __bfloat162float(pk.h[e]);
        } else {
#pragma unroll
          for (int e = 0; e < S::DPL; ++e) kv[u][e] = __bfloat162float(kc[static_cast<int64_t>(p) * HD + lane * S::DPL + e]);
        }
      }
#pragma unroll
      for (int u = 0; u < PW; ++u) {
        const int p = p0 + u;
#pragma unroll
        for (int h = 0; h < kMaxGroups; ++h) {
          if (h >= G) break;
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < S::DPL; ++e) d += qreg[h][e] * kv[u][e];
          d = warp_sum(d);
          if (lane == 0 && p < n_read) sc[h * a.max_seq + p] = bf16r(d);
        }
      }
    }
    // Own scores.
    if (warp < G) {
      float d = 0.f;
      for (int e = lane; e < HD; e += 32) d += qf[warp * HD + e] * kown[e];
      d = warp_sum(d);
      if (lane == 0) hs[warp] = bf16r(d);
    }
  }
  __syncthreads();

  // Softmax of (scores / sqrt(head_dim)) per head; weights rounded to bf16.
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));  // head**-0.5 as fp32
  if (warp < G) {
    float* s = sc + warp * a.max_seq;
    const float own = __fmul_rn(hs[warp], scale);
    float m = own;
    for (int p = lane; p < n_read; p += 32) m = fmaxf(m, __fmul_rn(s[p], scale));
    m = warp_max(m);
    float sum = 0.f;
    for (int p = lane; p < n_read; p += 32) sum += expf(__fsub_rn(__fmul_rn(s[p], scale), m));
    sum = warp_sum(sum);
    const float eown = expf(__fsub_rn(own, m));
    sum = __fadd_rn(sum, eown);
    for (int p = lane; p < n_read; p += 32) s[p] = bf16r(__fdiv_rn(expf(__fsub_rn(__fmul_rn(s[p], scale), m)), sum));
    __syncwarp();
    if (lane == 0) hs[kMaxGroups + warp] = bf16r(__fdiv_rn(eown, sum));
  }
  __syncthreads();

  // Pass 2: sum_p w[h][p] * V[p], thread = (8-dim chunk, position group).
  {
    const int chunk = tid % S::CHUNKS;
    const int pg = tid / S::CHUNKS;
    float acc[kMaxGroups][8];
#pragma unroll
    for (int h = 0; h < kMaxGroups; ++h)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] = 0.f;
    // 8 positions per step per thread, loaded before use (128 B in flight per thread).
    constexpr int PV = 8;
    for (int p0 = pg; p0 < n_read; p0 += S::PGROUPS * PV) {
      Pack8 pv[PV];
#pragma unroll
      for (int u = 0; u < PV; ++u) {
        const int p = min(p0 + u * S::PGROUPS, n_read - 1);
        pv[u].u = __ldg(reinterpret_cast<const uint4*>(vc + static_cast<int64_t>(p) * HD + chunk * 8));
      }
#pragma unroll
      for (int u = 0; u < PV; ++u) {
        const int p = p0 + u * S::PGROUPS;
        if (p >= n_read) break;
#pragma unroll
        for (int h = 0; h < kMaxGroups; ++h) {
          if (h >= G) break;
          const float w = sc[h * a.max_seq + p];
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[h][e] += w * __bfloat162float(pv[u].h[e]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroups; ++h) {
      if (h >= G) break;
#pragma unroll
      for (int e = 0; e < 8; ++e) part[(pg * G + h) * HD + chunk * 8 + e] = acc[h][e];
    }
  }
  __syncthreads();

  // Final: bf16(bf16(sum) + bf16(w_own * v_own)), times bf16(sigmoid(gate)), to e5m2.
  uint8_t* orow = a.out + b * a.ld_out;
  for (int i = tid; i < G * HD; i += kThreads) {
    const int h = i / HD, d = i % HD;
    float s = 0.f;
    for (int pg = 0; pg < S::PGROUPS; ++pg) s += part[(pg * G + h) * HD + d];
    const float o = bf16r(__fadd_rn(bf16r(s), bf16r(__fmul_rn(hs[kMaxGroups + h], vown[d]))));
    const float gt = bf16r(sigmoidf_(gate[i]));
    orow[static_cast<int64_t>(qh0 + h) * HD + d] = f32_to_e5m2(bf16r(__fmul_rn(o, gt)));
  }
  // The token's key and value go to the cache at `where` (nothing above read that position).
  __nv_bfloat16* kw = a.k_cache + ((static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq + where) * HD;
  __nv_bfloat16* vw = a.v_cache + ((static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq + where) * HD;
  for (int d = tid; d < HD; d += kThreads) {
    kw[d] = __float2bfloat16_rn(kown[d]);
    vw[d] = __float2bfloat16_rn(vown[d]);
  }
}

template <int HD>
int launch_attn(const AttnArgs& a, int64_t batch, cudaStream_t stream) {
  const size_t smem = AttnSmem<HD>::bytes(a.groups, a.max_seq);
  if (smem > 220 * 1024)
    return q38host::set_error("q38_attn_decode: max_seq %lld needs %zu bytes of shared memory", (long long)a.max_seq, smem),
           Q38_ERR_UNSUPPORTED;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(attn_decode)");
  }
  dim3 grid(static_cast<unsigned>(a.num_kv_heads), static_cast<unsigned>(batch));
  attn_decode_kernel<HD><<<grid, kThreads, smem, stream>>>(a);
  return q38host::cuda_status(cudaGetLastError(), "attn_decode launch");
}

}  // namespace

extern "C" int q38_attn_decode(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w,
                               const void* cos, const void* sin, void* k_cache, void* v_cache, int64_t max_seq,
                               const int32_t* position, const float* active, void* out, int64_t ld_out,
                               int64_t batch, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                               q38_stream_t stream) {
  using namespace q38host;
  if (!qkv || !q_norm_w || !k_norm_w || !cos || !sin || !k_cache || !v_cache || !position || !active || !out)
    return set_error("q38_attn_decode: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads ||
      num_q_heads / num_kv_heads > kMaxGroups || max_seq <= 0 || rot_dim < 0 || rot_dim > head_dim || rot_dim % 2)
    return set_error("q38_attn_decode: bad sizes"), Q38_ERR_ARG;
  if (ld_qkv < static_cast<int64_t>(2 * num_q_heads + 2 * num_kv_heads) * head_dim ||
      ld_out < static_cast<int64_t>(num_q_heads) * head_dim || ld_qkv % 8)
    return set_error("q38_attn_decode: leading dimension too small"), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(qkv)) & 15u)
    return set_error("q38_attn_decode: qkv and caches must be 16-byte aligned"), Q38_ERR_ARG;
  AttnArgs a{};
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ld_qkv = ld_qkv;
  a.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  a.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.max_seq = max_seq;
  a.position = position;
  a.active = active;
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.groups = num_q_heads / num_kv_heads;
  a.rot = rot_dim;
  a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 256) return launch_attn<256>(a, batch, s);
  if (head_dim == 32) return launch_attn<32>(a, batch, s);
  return set_error("q38_attn_decode: head_dim %d not built (256, 32 are)", head_dim), Q38_ERR_UNSUPPORTED;
}
