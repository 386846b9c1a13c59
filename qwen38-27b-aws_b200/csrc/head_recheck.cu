// The head's exact recheck on the device: ChipHead.next_tokens (qwen38_inf2/generate.py:186-208) after
// the group-of-32 maxima. For each batch row: the `candidates` groups with the largest maxima (ties to
// the lower group index), then every vocabulary row of those groups scored exactly, in fp32, against
// the row's fp32-normed hidden state rms_norm(hidden.float(), w) (generate.py:198), and the best token:
// the largest logit inside a group (its first row on ties), the groups taken in candidate order with a
// strictly larger logit replacing the best so far (generate.py:199-204). Only the token ids go back to
// the host: 4 bytes per row instead of the maxima's 4 bytes per group of 32.
//
// With the vocabulary sliced over ranks, each rank scores the candidate groups that fall in its slice
// and leaves the others at -inf; a max across ranks (the ranks' slots are disjoint) and q38_lm_head_pick
// then choose as the single-rank kernel does.
//
// One CTA of 256 threads per batch row. The lm_head rows come from the BF16 linear's tiled layout
// (16 KB tiles of 128 rows x 64 values, 128-byte swizzled), so no second copy of the lm_head is kept.
#include <cmath>

#include "q38_common.cuh"

namespace {

using namespace q38;

constexpr int kThreads = 256;
constexpr int kMaxCandidates = 8;
constexpr int kGroup = 32;

struct RecheckArgs {
  const __nv_bfloat16* hidden;
  int64_t ldh;
  const __nv_bfloat16* norm_w;
  float eps;
  const float* maxima;  // [rows][groups] over the whole vocabulary
  int64_t ldm, groups;
  const uint8_t* lm_head;      // this rank's slice, tiled
  int64_t vocab_first, vocab_rows, hidden_size;
  int candidates;
  float* slot_logits;   // [rows][candidates] or null
  int32_t* slot_tokens;  // [rows][candidates] or null
  int32_t* tokens;      // [rows] or null
};

// Byte address of BF16 element (v, k) in the tiled layout: tile (v / 128, 2k / 128), row v % 128, the
// 16-byte chunk (2k % 128) / 16 stored at chunk ^ (v % 8).
__device__ __forceinline__ const uint8_t* tiled_at(const uint8_t* base, int64_t v, int64_t kbytes, int64_t ktiles) {
  const int64_t r = v & 127, c = (kbytes & 127) >> 4;
  return base + ((v >> 7) * ktiles + (kbytes >> 7)) * 16384 + r * 128 + ((c ^ (r & 7)) << 4) + (kbytes & 15);
}

__device__ __forceinline__ bool better(float v, int64_t i, float bv, int64_t bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(kThreads) recheck_kernel(RecheckArgs a) {
  extern __shared__ float norm[];  // [hidden_size] fp32
  __shared__ float red_v[kThreads / 32];
  __shared__ int64_t red_i[kThreads / 32];
  __shared__ int64_t chosen[kMaxCandidates];
  __shared__ float logits[kGroup];
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t H = a.hidden_size;
  // fp32 RMS norm of the hidden row (not rounded: the reference norms hidden.float()).
  const __nv_bfloat16* h = a.hidden + row * a.ldh;
  float ss = 0.f;
  for (int64_t k = tid; k < H; k += kThreads) {
    const float f = __bfloat162float(h[k]);
    norm[k] = f;
    ss += f * f;
  }
  ss = warp_sum(ss);
  if (lane == 0) red_v[warp] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) total += red_v[w];
  const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), a.eps));
  for (int64_t k = tid; k < H; k += kThreads)
    norm[k] = __fmul_rn(__fmul_rn(norm[k], r), __fadd_rn(1.0f, __bfloat162float(a.norm_w[k])));
  __syncthreads();

  // The candidate groups, largest maximum first (lower index on ties; NaN maxima never chosen).
  const float* m = a.maxima + row * a.ldm;
  for (int j = 0; j < a.candidates; ++j) {
    float bv = -INFINITY;
    int64_t bi = INT64_MAX;
    for (int64_t g = tid; g < a.groups; g += kThreads) {
      bool taken = false;
      for (int q = 0; q < j; ++q) taken |= chosen[q] == g;
      const float v = m[g];
      if (!taken && !isnan(v) && better(v, g, bv, bi)) {
        bv = v;
        bi = g;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      red_v[warp] = bv;
      red_i[warp] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float v = red_v[0];
      int64_t i = red_i[0];
      for (int w = 1; w < kThreads / 32; ++w)
        if (better(red_v[w], red_i[w], v, i)) {
          v = red_v[w];
          i = red_i[w];
        }
      chosen[j] = i == INT64_MAX ? -1 : i;
    }
    __syncthreads();
  }

  // Each candidate group: 32 exact fp32 logits (4 rows per warp), its best row, then the running best.
  const int64_t ktiles = (2 * H + 127) / 128;
  float best = -INFINITY;
  int32_t best_token = -1;
  for (int j = 0; j < a.candidates; ++j) {
    const int64_t g = chosen[j];
    const int64_t first = g * kGroup;
    const bool mine = g >= 0 && first >= a.vocab_first && first + kGroup <= a.vocab_first + a.vocab_rows;
    float gl = -INFINITY;
    int32_t gt = -1;
    if (mine) {
      for (int rr = warp; rr < kGroup; rr += kThreads / 32) {
        const int64_t v = first - a.vocab_first + rr;
        float d = 0.f;
        for (int64_t k8 = lane * 8; k8 < H; k8 += 32 * 8) {  // 8 values (one 16-byte piece) per lane
          const uint4 u = *reinterpret_cast<const uint4*>(tiled_at(a.lm_head, v, 2 * k8, ktiles));
          const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
          for (int e = 0; e < 8; ++e) d = __fmaf_rn(__bfloat162float(w[e]), norm[k8 + e], d);
        }
        d = warp_sum(d);
        if (lane == 0) logits[rr] = d;
      }
      __syncthreads();
      if (tid == 0) {
        for (int rr = 0; rr < kGroup; ++rr)
          if (logits[rr] > gl || (gt < 0 && !isnan(logits[rr]))) {
            gl = logits[rr];
            gt = static_cast<int32_t>(first + rr);
          }
      }
      __syncthreads();
    }
    if (tid == 0) {
      if (a.slot_logits) {
        a.slot_logits[row * a.candidates + j] = gl;
        a.slot_tokens[row * a.candidates + j] = gt;
      }
      if (gt >= 0 && (best_token < 0 || gl > best)) {
        best = gl;
        best_token = gt;
      }
    }
  }
  if (tid == 0 && a.tokens) a.tokens[row] = best_token;
}

// The token from per-slot results (after a max across ranks): the candidate slots in order, a strictly
// larger logit replacing the best so far.
__global__ void pick_kernel(const float* slot_logits, const int32_t* slot_tokens, int candidates, int64_t rows,
                            int32_t* tokens) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float best = -INFINITY;
  int32_t tok = -1;
  for (int j = 0; j < candidates; ++j) {
    const int32_t t = slot_tokens[row * candidates + j];
    const float v = slot_logits[row * candidates + j];
    if (t >= 0 && (tok < 0 || v > best)) {
      best = v;
      tok = t;
    }
  }
  tokens[row] = tok;
}

}  // namespace

extern "C" int q38_lm_head_recheck(const void* hidden, int64_t ldh, const void* norm_w, float eps, const float* maxima,
                                   int64_t ldm, int64_t groups, const void* lm_head, int64_t vocab_first,
                                   int64_t vocab_rows, int64_t hidden_size, int group, int candidates, int64_t rows,
                                   float* slot_logits, int32_t* slot_tokens, int32_t* tokens, q38_stream_t stream) {
  using namespace q38host;
  if (!hidden || !norm_w || !maxima || !lm_head || (!tokens && !slot_logits) || (!slot_logits != !slot_tokens))
    return set_error("q38_lm_head_recheck: null pointer"), Q38_ERR_ARG;
  if (group != kGroup || candidates < 1 || candidates > kMaxCandidates || rows <= 0 || rows > (1 << 30) ||
      hidden_size <= 0 || hidden_size % 8 || hidden_size > 65536 || groups <= 0 || ldm < groups || ldh < hidden_size ||
      vocab_first < 0 || vocab_rows <= 0 || vocab_first % kGroup || vocab_rows % kGroup ||
      vocab_first + vocab_rows > groups * kGroup)
    return set_error("q38_lm_head_recheck: bad sizes (group 32, 1..%d candidates)", kMaxCandidates), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(lm_head) & 15u) || (reinterpret_cast<uintptr_t>(hidden) & 15u) || ldh % 8)
    return set_error("q38_lm_head_recheck: lm_head and hidden rows must be 16-byte aligned"), Q38_ERR_ARG;
  RecheckArgs a{};
  a.hidden = static_cast<const __nv_bfloat16*>(hidden);
  a.ldh = ldh;
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  a.eps = eps;
  a.maxima = maxima;
  a.ldm = ldm;
  a.groups = groups;
  a.lm_head = static_cast<const uint8_t*>(lm_head);
  a.vocab_first = vocab_first;
  a.vocab_rows = vocab_rows;
  a.hidden_size = hidden_size;
  a.candidates = candidates;
  a.slot_logits = slot_logits;
  a.slot_tokens = slot_tokens;
  a.tokens = tokens;
  const size_t smem = static_cast<size_t>(hidden_size) * sizeof(float);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(recheck_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(recheck)");
  }
  const cudaError_t e = launch_pdl(recheck_kernel, dim3(static_cast<unsigned>(rows)), dim3(kThreads), smem,
                                   static_cast<cudaStream_t>(stream), a);
  return cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "lm_head_recheck launch");
}

extern "C" int q38_lm_head_pick(const float* slot_logits, const int32_t* slot_tokens, int candidates, int64_t rows,
                                int32_t* tokens, q38_stream_t stream) {
  using namespace q38host;
  if (!slot_logits || !slot_tokens || !tokens) return set_error("q38_lm_head_pick: null pointer"), Q38_ERR_ARG;
  if (candidates < 1 || candidates > kMaxCandidates || rows <= 0 || rows > (1 << 30))
    return set_error("q38_lm_head_pick: bad sizes"), Q38_ERR_ARG;
  const unsigned blocks = static_cast<unsigned>((rows + 127) / 128);
  const cudaError_t e = launch_pdl(pick_kernel, dim3(blocks), dim3(128), 0, static_cast<cudaStream_t>(stream),
                                   slot_logits, slot_tokens, candidates, rows, tokens);
  return cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "lm_head_pick launch");
}

// ---- embeddings ------------------------------------------------------------------------------------
// out[i] = table[ids[i]] (bf16 rows of hidden_size), ChipHead.embed_batch (generate.py:183-184) on the
// device: one 16-byte piece per thread. An id outside the table writes a zero row and records
// Q38_ERR_ARG in the device error word.
namespace {
__global__ void embed_kernel(const __nv_bfloat16* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n,
                             __nv_bfloat16* out, int64_t ldo) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = blockIdx.y;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // 8-value piece
  if (i >= n || c * 8 >= hidden) return;
  const int64_t id = ids[i];
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (id >= 0 && id < vocab) v = *reinterpret_cast<const uint4*>(table + id * hidden + c * 8);
  else if (c == 0) record_error(Q38_ERR_ARG);
  *reinterpret_cast<uint4*>(out + i * ldo + c * 8) = v;
}
}  // namespace

extern "C" int q38_embed_rows(const void* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t n, void* out,
                              int64_t ldo, q38_stream_t stream) {
  using namespace q38host;
  if (!table || !ids || !out) return set_error("q38_embed_rows: null pointer"), Q38_ERR_ARG;
  if (vocab <= 0 || hidden <= 0 || hidden % 8 || n <= 0 || n > 65535 || ldo < hidden || ldo % 8)
    return set_error("q38_embed_rows: bad sizes (hidden a multiple of 8, at most 65535 ids)"), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return set_error("q38_embed_rows: table and out must be 16-byte aligned"), Q38_ERR_ARG;
  const dim3 grid(static_cast<unsigned>((hidden / 8 + 127) / 128), static_cast<unsigned>(n));
  const cudaError_t e = launch_pdl(embed_kernel, grid, dim3(128), 0, static_cast<cudaStream_t>(stream),
                                   static_cast<const __nv_bfloat16*>(table), vocab, hidden, ids, n,
                                   static_cast<__nv_bfloat16*>(out), ldo);
  return cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "embed_rows launch");
}
