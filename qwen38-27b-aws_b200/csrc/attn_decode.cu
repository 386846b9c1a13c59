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

constexpr int kWarps = 4;
constexpr int KT = 32;     // cache positions per tile
constexpr int STAGES = 4;  // tiles in flight
constexpr int MROWS = 16;  // the MMA's M: query heads, padded

template <int HD>
struct AttnSmem {
  static constexpr int ROWP = HD + 8;  // padded row (bf16): ldmatrix rows land in distinct banks
  static constexpr int NPAD = 8;       // extra weight columns past max_seq
  static size_t bytes(int groups, int64_t max_seq) {
    const size_t wcols = static_cast<size_t>((max_seq + KT - 1) / KT * KT + NPAD);
    return 2 * (static_cast<size_t>(MROWS) * ROWP   // q (bf16)
                + STAGES * static_cast<size_t>(KT) * ROWP  // K / V tile ring
                + MROWS * wcols)                      // scores, then weights (bf16)
           + sizeof(float) * (static_cast<size_t>(groups) * HD + 2 * HD + 2 * kMaxGroups);
  }
};

template <int HD>
__global__ void __launch_bounds__(kWarps * 32) attn_decode_kernel(AttnArgs a) {
  using S = AttnSmem<HD>;
  constexpr int ROWP = S::ROWP;
  constexpr int KSTEPS = HD / 16;          // MMA k-steps over head_dim
  constexpr int NT2 = HD / 8 / kWarps;     // pass-2 n-tiles (8 dims) per warp
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int G = a.groups;
  const int wcols = static_cast<int>((a.max_seq + KT - 1) / KT * KT) + S::NPAD;
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem_raw);       // [16][ROWP]
  __nv_bfloat16* ring = qs + MROWS * ROWP;                               // [STAGES][KT][ROWP]
  __nv_bfloat16* wb = ring + STAGES * KT * ROWP;                         // [16][wcols]
  float* qf = reinterpret_cast<float*>(wb + MROWS * wcols);             // [G][HD]
  float* kown = qf + G * HD;                                             // [HD]
  float* vown = kown + HD;                                               // [HD]
  float* hs = vown + HD;                                                 // [2][kMaxGroups]

  const int g = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool on = a.active[b] > 0.5f;
  const int pos = a.position[b];
  const int64_t pos64 = pos < 0 ? 0 : pos;
  const int n_read = on ? static_cast<int>(pos64 < a.max_seq ? pos64 : a.max_seq) : 0;
  const int64_t where = on ? (pos64 < a.max_seq - 1 ? pos64 : a.max_seq - 1) : a.max_seq - 1;
  const __nv_bfloat16* row = a.qkv + b * a.ld_qkv;
  const int qh0 = g * G;
  const __nv_bfloat16* kc = a.k_cache + (static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq * HD;
  const __nv_bfloat16* vc = a.v_cache + (static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq * HD;
  const int ntiles = (n_read + KT - 1) / KT;

  // Tile i of the stream: K tiles 0 .. ntiles-1, then V tiles. Rows past n_read are zero-filled.
  auto load_tile = [&](int i) {
    const bool is_v = i >= ntiles;
    const int p0 = (is_v ? i - ntiles : i) * KT;
    const __nv_bfloat16* src = is_v ? vc : kc;
    __nv_bfloat16* dst = ring + (i % STAGES) * KT * ROWP;
    for (int c = tid; c < KT * (HD / 8); c += kWarps * 32) {
      const int r = c / (HD / 8), cc = c % (HD / 8);
      const int p = p0 + r;
      const bool ok = p < n_read;
      cp_async16(smem_u32(dst + r * ROWP + cc * 8), src + static_cast<int64_t>(ok ? p : 0) * HD + cc * 8, ok ? 16u : 0u);
    }
    cp_async_commit();
  };
  for (int i = 0; i < STAGES - 1; ++i) {
    if (i < 2 * ntiles) load_tile(i);
    else cp_async_commit();  // empty groups keep the wait counts uniform
  }

  // Stage the raw query heads, own key and value; norm + rotary; queries to bf16 MMA rows.
  for (int i = tid; i < G * HD; i += kWarps * 32) {
    const int h = i / HD, d = i % HD;
    qf[i] = __bfloat162float(row[static_cast<int64_t>(qh0 + h) * 2 * HD + d]);
  }
  const __nv_bfloat16* kraw = row + static_cast<int64_t>(a.num_q_heads) * 2 * HD + static_cast<int64_t>(g) * HD;
  const __nv_bfloat16* vraw = kraw + static_cast<int64_t>(a.num_kv_heads) * HD;
  for (int d = tid; d < HD; d += kWarps * 32) {
    kown[d] = __bfloat162float(kraw[d]);
    vown[d] = __bfloat162float(vraw[d]);
  }
  __syncthreads();
  const __nv_bfloat16* cs = a.cos + b * a.rot;
  const __nv_bfloat16* sn = a.sin + b * a.rot;
  for (int h = warp; h <= G; h += kWarps) {
    if (h < G) norm_rope_head<HD>(qf + h * HD, a.q_norm_w, cs, sn, a.rot, a.eps, lane);
    else norm_rope_head<HD>(kown, a.k_norm_w, cs, sn, a.rot, a.eps, lane);
  }
  __syncthreads();
  for (int i = tid; i < MROWS * HD; i += kWarps * 32) {
    const int h = i / HD, d = i % HD;
    qs[h * ROWP + d] = __float2bfloat16_rn(h < G ? qf[i] : 0.f);
  }
  for (int i = tid; i < MROWS * wcols; i += kWarps * 32) wb[i] = __float2bfloat16_rn(0.f);
  // Own scores (fp32 dot, bf16-rounded like the reference's matmul output).
  for (int h = warp; h < G; h += kWarps) {
    float d = 0.f;
    for (int e = lane; e < HD; e += 32) d += qf[h * HD + e] * kown[e];
    d = warp_sum(d);
    if (lane == 0) hs[h] = bf16r(d);
  }
  __syncthreads();

  // Query fragments for every k-step, kept in registers for pass 1.
  uint32_t qa[KSTEPS][4];
  {
    const int r = lane & 15, co = (lane >> 4) * 8;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks)
      ldsm_x4(smem_u32(qs + r * ROWP + ks * 16 + co), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }

  float acc2[NT2][4];
#pragma unroll
  for (int n = 0; n < NT2; ++n) acc2[n][0] = acc2[n][1] = acc2[n][2] = acc2[n][3] = 0.f;
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));  // head**-0.5 as fp32

  for (int i = 0; i < 2 * ntiles; ++i) {
    if (i + STAGES - 1 < 2 * ntiles) load_tile(i + STAGES - 1);
    else cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncthreads();  // tile i is in shared memory for every thread
    const __nv_bfloat16* tile = ring + (i % STAGES) * KT * ROWP;
    if (i < ntiles) {
      // Pass 1: S[16 x 8] for this warp's 8 positions of the tile.
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      const int n0 = warp * 8;
      const int r = n0 + (lane & 7), co = (lane >> 3) * 8;  // x4: four k-chunks of 8
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ks += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(tile + r * ROWP + ks * 16 + co), b0, b1, b2, b3);
        mma_bf16_16816(s, qa[ks], b0, b1);
        mma_bf16_16816(s, qa[ks + 1], b2, b3);
      }
      // C fragment: rows lane/4 (+8) = heads, columns 2*(lane%4) + {0,1} = positions.
      const int h = lane >> 2, p = i * KT + n0 + 2 * (lane & 3);
      if (h < G) {
        if (p < n_read) wb[h * wcols + p] = __float2bfloat16_rn(s[0]);
        if (p + 1 < n_read) wb[h * wcols + p + 1] = __float2bfloat16_rn(s[1]);
      }
    } else {
      if (i == ntiles) {
        // All scores are in: softmax of (score * head_dim^-0.5) per head over [cache, own];
        // weights rounded to bf16 in place. (The barrier above ordered the last score writes.)
        for (int h = warp; h < G; h += kWarps) {
          __nv_bfloat16* w = wb + h * wcols;
          const float own = __fmul_rn(hs[h], scale);
          float m = own;
          for (int p = lane; p < n_read; p += 32) m = fmaxf(m, __fmul_rn(__bfloat162float(w[p]), scale));
          m = warp_max(m);
          float sum = 0.f;
          for (int p = lane; p < n_read; p += 32) sum += expf(__fsub_rn(__fmul_rn(__bfloat162float(w[p]), scale), m));
          sum = warp_sum(sum);
          const float eown = expf(__fsub_rn(own, m));
          sum = __fadd_rn(sum, eown);
          for (int p = lane; p < n_read; p += 32)
            w[p] = __float2bfloat16_rn(__fdiv_rn(expf(__fsub_rn(__fmul_rn(__bfloat162float(w[p]), scale), m)), sum));
          if (lane == 0) hs[kMaxGroups + h] = bf16r(__fdiv_rn(eown, sum));
        }
        __syncthreads();
      }
      // Pass 2: O[16 x this warp's dims] += W[16 x 32 positions] * V[32 x dims].
      const int t = i - ntiles;
#pragma unroll
      for (int ks = 0; ks < KT / 16; ++ks) {
        uint32_t wa[4];
        ldsm_x4(smem_u32(wb + (lane & 15) * wcols + t * KT + ks * 16 + (lane >> 4) * 8), wa[0], wa[1], wa[2], wa[3]);
        const int vr = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;  // x4.trans: (k 0-7 | 8-15) x (n 0-7 | 8-15)
#pragma unroll
        for (int n = 0; n < NT2; n += 2) {
          const int d0 = (warp * NT2 + n) * 8 + (lane >> 4) * 8;
          uint32_t b0, b1, b2, b3;
          if constexpr (NT2 >= 2) {
            ldsm_x4_t(smem_u32(tile + vr * ROWP + d0), b0, b1, b2, b3);
            mma_bf16_16816(acc2[n], wa, b0, b1);
            mma_bf16_16816(acc2[n + 1], wa, b2, b3);
          } else {
            ldsm_x2_t(smem_u32(tile + vr * ROWP + (warp * NT2 + n) * 8), b0, b1);
            mma_bf16_16816(acc2[n], wa, b0, b1);
          }
        }
      }
    }
    __syncthreads();  // every warp is done with tile i before its buffer is refilled
  }
  if (ntiles == 0) {
    // No cached positions: only the own key; its weight is exp(0) / exp(0) = 1.
    if (tid < G) hs[kMaxGroups + tid] = 1.0f;
    __syncthreads();
  }

  // Final: bf16(bf16(W V) + bf16(w_own * v_own)) * bf16(sigmoid(gate)), to e5m2.
  uint8_t* orow = a.out + b * a.ld_out;
  const int h = lane >> 2;
  if (h < G) {
#pragma unroll
    for (int n = 0; n < NT2; ++n) {
      const int d = (warp * NT2 + n) * 8 + 2 * (lane & 3);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float o = bf16r(__fadd_rn(bf16r(acc2[n][e]), bf16r(__fmul_rn(hs[kMaxGroups + h], vown[d + e]))));
        const float gv = __bfloat162float(row[static_cast<int64_t>(qh0 + h) * 2 * HD + HD + d + e]);
        orow[static_cast<int64_t>(qh0 + h) * HD + d + e] = f32_to_e5m2(bf16r(__fmul_rn(o, bf16r(sigmoidf_(gv)))));
      }
    }
  }
  // The token's key and value go to the cache at `where` (nothing above read that position).
  __nv_bfloat16* kw = a.k_cache + ((static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq + where) * HD;
  __nv_bfloat16* vw = a.v_cache + ((static_cast<int64_t>(b) * a.num_kv_heads + g) * a.max_seq + where) * HD;
  for (int d = tid; d < HD; d += kWarps * 32) {
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
  attn_decode_kernel<HD><<<grid, kWarps * 32, smem, stream>>>(a);
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
