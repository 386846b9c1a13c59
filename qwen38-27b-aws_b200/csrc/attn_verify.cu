// Gated full attention for K verify tokens per row over a BF16 KV cache: FullAttentionStep.verify
// (qwen38_inf2/model.py:641-675, BF16 cache branch).
//
// One CTA per (KV head, row) with its G query heads for the K tokens (G * K query rows). Token t of a
// row attends to cache positions < position (the cache as it was before the step) and to the step's
// own keys 0 .. t. The reference's rounding points stay: scores are bf16-rounded fp32 dot products,
// one fp32 softmax of (score * head_dim^-0.5) over [cache, own] per query row, weights rounded to bf16,
// and the output is bf16(weights_cache @ V_cache) + bf16(weights_own @ V_own) in bf16, times
// bf16(sigmoid(gate)), then e5m2 for o_proj. The K tokens' keys and values are written from position
// on (rows with active 0 write at the cache's last K positions, which no sequence reads).
#include "attn_common.cuh"

namespace {

using namespace q38;

constexpr int kThreads = 256;
constexpr int KMAX = 8;      // verify tokens per row built
constexpr int kMaxRows = 48; // G * K query rows per CTA
constexpr int RG = 6;        // query rows per pass of the weighted-value sum

struct VerifyAttnArgs {
  const __nv_bfloat16* qkv;  // [batch * K, ld_qkv]
  int64_t ld_qkv;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* cos;  // [batch * K, rot]
  const __nv_bfloat16* sin;
  __nv_bfloat16* k_cache;  // [batch, num_kv_heads, max_seq, HD]
  __nv_bfloat16* v_cache;
  int64_t max_seq;
  const int32_t* position;
  const float* active;
  uint8_t* out;  // [batch * K, ld_out]
  int64_t ld_out;
  int num_q_heads, num_kv_heads, groups, rot, K;
  float eps;
};

template <int HD>
struct VerifyAttnSmem {
  static constexpr int CHUNKS = HD / 8;
  static constexpr int PGROUPS = kThreads / CHUNKS;
  static size_t bytes(int rows, int K, int64_t max_seq) {
    return sizeof(float) * (static_cast<size_t>(rows) * HD + 2 * static_cast<size_t>(K) * HD + 2 * rows * KMAX +
                            static_cast<size_t>(PGROUPS) * RG * HD) +
           2 * static_cast<size_t>(rows) * max_seq;
  }
};

union Pack8 {
  uint4 u;
  __nv_bfloat16 h[8];
};

template <int HD>
__global__ void __launch_bounds__(kThreads) attn_verify_kernel(VerifyAttnArgs a) {
  using S = VerifyAttnSmem<HD>;
  constexpr int DPL = HD / 32;
  extern __shared__ __align__(16) float sm[];
  const int G = a.groups, K = a.K, QR = G * K;
  float* qf = sm;                               // [QR][HD] normed, roped queries (row r = h * K + t)
  float* kown = qf + QR * HD;                   // [K][HD]
  float* vown = kown + K * HD;                  // [K][HD]
  float* sown = vown + K * HD;                  // [QR][KMAX] own scores, then own weights
  float* wown = sown + QR * KMAX;               // [QR][KMAX]
  float* part = wown + QR * KMAX;               // [PGROUPS][RG][HD]
  __nv_bfloat16* sc = reinterpret_cast<__nv_bfloat16*>(part + S::PGROUPS * RG * HD);  // [QR][max_seq]

  const int g = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool on = a.active[b] > 0.5f;
  const int pos = a.position[b];
  const int64_t pos64 = pos < 0 ? 0 : pos;
  const int n_read = on ? static_cast<int>(pos64 < a.max_seq ? pos64 : a.max_seq) : 0;
  const int qh0 = g * G;

  // Stage raw queries, own keys and values of the K tokens.
  for (int i = tid; i < QR * HD; i += kThreads) {
    const int r = i / HD, d = i % HD;
    const int h = r / K, t = r % K;
    qf[i] = __bfloat162float(a.qkv[(static_cast<int64_t>(b) * K + t) * a.ld_qkv + static_cast<int64_t>(qh0 + h) * 2 * HD + d]);
  }
  for (int i = tid; i < K * HD; i += kThreads) {
    const int t = i / HD, d = i % HD;
    const __nv_bfloat16* kraw = a.qkv + (static_cast<int64_t>(b) * K + t) * a.ld_qkv +
                                static_cast<int64_t>(a.num_q_heads) * 2 * HD + static_cast<int64_t>(g) * HD;
    kown[i] = __bfloat162float(kraw[d]);
    vown[i] = __bfloat162float(kraw[static_cast<int64_t>(a.num_kv_heads) * HD + d]);
  }
  __syncthreads();
  for (int p = warp; p < QR + K; p += kThreads / 32) {
    const int t = p < QR ? p % K : p - QR;
    const __nv_bfloat16* cs = a.cos + (static_cast<int64_t>(b) * K + t) * a.rot;
    const __nv_bfloat16* sn = a.sin + (static_cast<int64_t>(b) * K + t) * a.rot;
    if (p < QR) norm_rope_head<HD>(qf + p * HD, a.q_norm_w, cs, sn, a.rot, a.eps, lane);
    else norm_rope_head<HD>(kown + t * HD, a.k_norm_w, cs, sn, a.rot, a.eps, lane);
  }
  __syncthreads();

  // Pass 1: bf16-rounded scores of every visible cached position; 4 positions per warp step in flight.
  const __nv_bfloat16* kc = a.k_cache + (static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq * HD;
  const __nv_bfloat16* vc = a.v_cache + (static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq * HD;
  {
    constexpr int PW = 4;
    for (int p0 = warp * PW; p0 < n_read; p0 += (kThreads / 32) * PW) {
      float kv[PW][DPL];
#pragma unroll
      for (int u = 0; u < PW; ++u) {
        const int p = min(p0 + u, n_read - 1);
        if constexpr (DPL == 8) {
          Pack8 pk;
          pk.u = __ldg(reinterpret_cast<const uint4*>(kc + static_cast<int64_t>(p) * HD + lane * 8));
#pragma unroll
          for (int e = 0; e < 8; ++e) kv[u][e] = __bfloat162float(pk.h[e]);
        } else {
#pragma unroll
          for (int e = 0; e < DPL; ++e) kv[u][e] = __bfloat162float(kc[static_cast<int64_t>(p) * HD + lane * DPL + e]);
        }
      }
      for (int r = 0; r < QR; ++r) {
        float q[DPL];
#pragma unroll
        for (int e = 0; e < DPL; ++e) q[e] = qf[r * HD + lane * DPL + e];
#pragma unroll
        for (int u = 0; u < PW; ++u) {
          float d = 0.f;
#pragma unroll
          for (int e = 0; e < DPL; ++e) d += q[e] * kv[u][e];
          d = warp_sum(d);
          if (lane == 0 && p0 + u < n_read) sc[static_cast<int64_t>(r) * a.max_seq + p0 + u] = __float2bfloat16_rn(d);
        }
      }
    }
    // Own scores: query row (h, t) against own keys s <= t.
    for (int p = warp; p < QR * K; p += kThreads / 32) {
      const int r = p / K, s = p % K, t = r % K;
      if (s > t) continue;
      float d = 0.f;
      for (int e = lane; e < HD; e += 32) d += qf[r * HD + e] * kown[s * HD + e];
      d = warp_sum(d);
      if (lane == 0) sown[r * KMAX + s] = bf16r(d);
    }
  }
  __syncthreads();

  // Softmax of (score * head_dim^-0.5) per query row over [cache < position, own <= t]; bf16 weights.
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));
  for (int r = warp; r < QR; r += kThreads / 32) {
    const int t = r % K;
    __nv_bfloat16* s = sc + static_cast<int64_t>(r) * a.max_seq;
    float m = -INFINITY;
    for (int p = lane; p < n_read; p += 32) m = fmaxf(m, __fmul_rn(__bfloat162float(s[p]), scale));
    for (int j = 0; j <= t; ++j) m = fmaxf(m, __fmul_rn(sown[r * KMAX + j], scale));
    m = warp_max(m);
    float sum = 0.f;
    for (int p = lane; p < n_read; p += 32) sum += expf(__fsub_rn(__fmul_rn(__bfloat162float(s[p]), scale), m));
    sum = warp_sum(sum);
    for (int j = 0; j <= t; ++j) sum = __fadd_rn(sum, expf(__fsub_rn(__fmul_rn(sown[r * KMAX + j], scale), m)));
    for (int p = lane; p < n_read; p += 32)
      s[p] = __float2bfloat16_rn(__fdiv_rn(expf(__fsub_rn(__fmul_rn(__bfloat162float(s[p]), scale), m)), sum));
    __syncwarp();
    if (lane < K) wown[r * KMAX + lane] = lane <= t ? bf16r(__fdiv_rn(expf(__fsub_rn(__fmul_rn(sown[r * KMAX + lane], scale), m)), sum)) : 0.f;
  }
  __syncthreads();

  // Pass 2, RG query rows at a time: sum_p w[r][p] V[p], thread = (8-dim chunk, position group).
  const int chunk = tid % S::CHUNKS, pg = tid / S::CHUNKS;
  for (int r0 = 0; r0 < QR; r0 += RG) {
    const int nr = min(RG, QR - r0);
    float acc[RG][8];
#pragma unroll
    for (int x = 0; x < RG; ++x)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[x][e] = 0.f;
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
        for (int x = 0; x < RG; ++x) {
          if (x >= nr) break;
          const float w = __bfloat162float(sc[static_cast<int64_t>(r0 + x) * a.max_seq + p]);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[x][e] += w * __bfloat162float(pv[u].h[e]);
        }
      }
    }
#pragma unroll
    for (int x = 0; x < RG; ++x) {
      if (x >= nr) break;
#pragma unroll
      for (int e = 0; e < 8; ++e) part[(pg * RG + x) * HD + chunk * 8 + e] = acc[x][e];
    }
    __syncthreads();
    for (int i = tid; i < nr * HD; i += kThreads) {
      const int x = i / HD, d = i % HD;
      const int r = r0 + x, h = r / K, t = r % K;
      float s = 0.f;
      for (int q = 0; q < S::PGROUPS; ++q) s += part[(q * RG + x) * HD + d];
      float own = 0.f;
      for (int j = 0; j <= t; ++j) own = fmaf(wown[r * KMAX + j], vown[j * HD + d], own);
      const float o = bf16r(__fadd_rn(bf16r(s), bf16r(own)));
      const int64_t row = static_cast<int64_t>(b) * K + t;
      const float gate = __bfloat162float(a.qkv[row * a.ld_qkv + static_cast<int64_t>(qh0 + h) * 2 * HD + HD + d]);
      const float gt = bf16r(sigmoidf_(gate));
      a.out[row * a.ld_out + static_cast<int64_t>(qh0 + h) * HD + d] = f32_to_e5m2(bf16r(__fmul_rn(o, gt)));
    }
    __syncthreads();
  }
  // The tokens' keys and values go to the cache (nothing above read those positions).
  for (int i = tid; i < K * HD; i += kThreads) {
    const int t = i / HD, d = i % HD;
    const int64_t where = on ? pos64 + t : a.max_seq - K + t;
    const int64_t at = ((static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq + where) * HD + d;
    a.k_cache[at] = __float2bfloat16_rn(kown[i]);
    a.v_cache[at] = __float2bfloat16_rn(vown[i]);
  }
}

template <int HD>
int launch_attn_verify(const VerifyAttnArgs& a, int64_t batch, cudaStream_t stream) {
  const size_t smem = VerifyAttnSmem<HD>::bytes(a.groups * a.K, a.K, a.max_seq);
  if (smem > 220 * 1024)
    return q38host::set_error("q38_attn_verify: max_seq %lld with %d x %d query rows needs %zu bytes of shared memory",
                              static_cast<long long>(a.max_seq), a.groups, a.K, smem),
           Q38_ERR_UNSUPPORTED;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(attn_verify_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(attn_verify)");
  }
  dim3 grid(static_cast<unsigned>(a.num_kv_heads), static_cast<unsigned>(batch));
  attn_verify_kernel<HD><<<grid, kThreads, smem, stream>>>(a);
  return q38host::cuda_status(cudaGetLastError(), "attn_verify launch");
}

}  // namespace

extern "C" int q38_attn_verify(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w,
                               const void* cos, const void* sin, void* k_cache, void* v_cache, int64_t max_seq,
                               const int32_t* position, const float* active, void* out, int64_t ld_out, int64_t batch,
                               int tokens, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                               q38_stream_t stream) {
  using namespace q38host;
  if (!qkv || !q_norm_w || !k_norm_w || !cos || !sin || !k_cache || !v_cache || !position || !active || !out)
    return set_error("q38_attn_verify: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || tokens < 1 || tokens > KMAX || max_seq < tokens)
    return set_error("q38_attn_verify: batch %lld, %d tokens per row (1..%d built), max_seq %lld",
                     static_cast<long long>(batch), tokens, KMAX, static_cast<long long>(max_seq)),
           Q38_ERR_ARG;
  if (num_kv_heads <= 0 || num_q_heads % num_kv_heads || (num_q_heads / num_kv_heads) * tokens > kMaxRows)
    return set_error("q38_attn_verify: %d query heads per KV head x %d tokens exceeds %d rows", num_q_heads / num_kv_heads,
                     tokens, kMaxRows),
           Q38_ERR_UNSUPPORTED;
  if (rot_dim <= 0 || rot_dim > head_dim || rot_dim % 2) return set_error("q38_attn_verify: bad rotary dim"), Q38_ERR_ARG;
  if (ld_qkv < static_cast<int64_t>(num_q_heads) * 2 * head_dim + 2LL * num_kv_heads * head_dim ||
      ld_out < static_cast<int64_t>(num_q_heads) * head_dim)
    return set_error("q38_attn_verify: leading dimension too small"), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u)
    return set_error("q38_attn_verify: caches must be 16-byte aligned"), Q38_ERR_ARG;
  VerifyAttnArgs a{};
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
  a.K = tokens;
  a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 256) return launch_attn_verify<256>(a, batch, s);
  if (head_dim == 32) return launch_attn_verify<32>(a, batch, s);
  return set_error("q38_attn_verify: head_dim %d not built (256, 32 are)", head_dim), Q38_ERR_UNSUPPORTED;
}
