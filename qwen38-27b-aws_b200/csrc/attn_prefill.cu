// Keys-first gated attention over a prefill chunk of one row: FullAttentionStep.prefill
// (qwen38_inf2/model.py:732-786) with the online softmax of blocked_attention (model.py:170-191).
//
// Two launches on the caller's stream:
//   prep       one CTA per token: q/k RMS norms (1 + w), partial rotary, the scaled query
//              bf16(q * head_dim^-0.5) into the workspace, and the chunk's own keys and values into
//              the row's cache at start .. start + tokens - 1 (model.py:780-781). The reference
//              attends to its own keys from registers and writes them afterwards; the values are the
//              same bf16 numbers, so writing first lets the attention read one key range.
//   attention  one CTA per (KV head, 48 / G-token tile) holding that KV head's G query heads for those
//              tokens (48 query rows), so each key and value tile is read once for G heads. Token t sees
//              cache positions 0 .. start + t. The arithmetic keeps the reference's rounding points:
//              scores are bf16-rounded fp32 dot products (its BF16 matmul); the online softmax walks the
//              reference's own blocks of 2048 keys of [cache, chunk], each in two passes (the block's
//              maximum, then weights exp(s - max) summed in fp32 and, rounded to bf16, multiplied into
//              the values); the block's weighted values are rounded to bf16 (its BF16 matmul output)
//              before the fp32 rescale-and-add. Output: bf16(out / total) * bf16(sigmoid(gate)) in
//              bf16, then e5m2 for o_proj.
#include "attn_common.cuh"

namespace {

using namespace q38;

constexpr int kThreads = 256;
constexpr int KT = 32;  // keys per tile (one per lane)

struct AttnPrefillArgs {
  const __nv_bfloat16* qkv;  // [tokens, ld_qkv]: per q head [query | gate], then k, then v
  int64_t ld_qkv;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* cos;  // [tokens, rot]
  const __nv_bfloat16* sin;
  __nv_bfloat16* k_cache;  // this row: [num_kv_heads][max_seq][HD]
  __nv_bfloat16* v_cache;
  int64_t max_seq;
  int tokens, start;
  uint8_t* out;
  int64_t ld_out;
  int num_q_heads, num_kv_heads, groups, rot;
  float eps, scale;
  __nv_bfloat16* qs;  // workspace [num_kv_heads][groups][tokens][HD]
};

template <int HD>
__global__ void __launch_bounds__(kThreads) attn_prefill_prep_kernel(AttnPrefillArgs a) {
  extern __shared__ __align__(16) float xs[];  // [heads + kv heads][HD]
  const int t = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* row = a.qkv + static_cast<int64_t>(t) * a.ld_qkv;
  const int nh = a.num_q_heads + a.num_kv_heads;
  for (int i = tid; i < nh * HD; i += kThreads) {
    const int h = i / HD, d = i % HD;
    xs[i] = __bfloat162float(h < a.num_q_heads ? row[static_cast<int64_t>(h) * 2 * HD + d]
                                               : row[static_cast<int64_t>(a.num_q_heads) * 2 * HD +
                                                     static_cast<int64_t>(h - a.num_q_heads) * HD + d]);
  }
  __syncthreads();
  const __nv_bfloat16* cs = a.cos + static_cast<int64_t>(t) * a.rot;
  const __nv_bfloat16* sn = a.sin + static_cast<int64_t>(t) * a.rot;
  const int64_t pos = a.start + t;
  for (int h = warp; h < nh; h += kThreads / 32) {
    float* x = xs + h * HD;
    const bool is_q = h < a.num_q_heads;
    norm_rope_head<HD>(x, is_q ? a.q_norm_w : a.k_norm_w, cs, sn, a.rot, a.eps, lane);
    if (is_q) {
      const int kvh = h / a.groups, g = h % a.groups;
      __nv_bfloat16* dst = a.qs + ((static_cast<int64_t>(kvh) * a.groups + g) * a.tokens + t) * HD;
      for (int d = lane; d < HD; d += 32) dst[d] = __float2bfloat16_rn(__fmul_rn(x[d], a.scale));
    } else {
      const int kvh = h - a.num_q_heads;
      __nv_bfloat16* kd = a.k_cache + (static_cast<int64_t>(kvh) * a.max_seq + pos) * HD;
      __nv_bfloat16* vd = a.v_cache + (static_cast<int64_t>(kvh) * a.max_seq + pos) * HD;
      const __nv_bfloat16* vraw = row + static_cast<int64_t>(a.num_q_heads) * 2 * HD +
                                  static_cast<int64_t>(a.num_kv_heads + kvh) * HD;
      for (int d = lane; d < HD; d += 32) {
        kd[d] = __float2bfloat16_rn(x[d]);
        vd[d] = vraw[d];
      }
    }
  }
}

constexpr int RPW = 6;                       // query rows per warp
constexpr int ROWS = RPW * (kThreads / 32);  // query rows per CTA: G heads x (ROWS / G) tokens
constexpr int REF_BLOCK = 2048;              // keys per block of the reference's online softmax

template <int HD>
struct PrefillSmem {
  static constexpr size_t QF = 0;                                  // [ROWS][HD] fp32 queries
  static constexpr size_t KTR = QF + sizeof(float) * ROWS * HD;    // [HD][KT] keys, transposed
  static constexpr size_t VT = KTR + sizeof(float) * HD * KT;      // [KT][HD] values
  static constexpr size_t PW = VT + sizeof(float) * KT * HD;       // [ROWS][KT] bf16-rounded weights
  static constexpr size_t TOTAL = PW + sizeof(float) * ROWS * KT;
};

// The reference's softmax block of a key: it concatenates the row's cache (max_seq positions, those
// < start visible) and the chunk's own keys, then walks that sequence in blocks of REF_BLOCK. Here the
// chunk's keys sit in the cache at start .., so key index k < start is cache position k and k >= start
// is own token k - start, at sequence index max_seq + k - start.
__device__ __forceinline__ int64_t ref_block(int64_t key, int64_t start, int64_t max_seq) {
  return (key < start ? key : max_seq + key - start) / REF_BLOCK;
}

// Rows of the CTA: r = g * tq + tt (query head g of the KV head, token t0 + tt); warp w owns rows
// w * RPW .. w * RPW + RPW - 1.
template <int HD>
__global__ void __launch_bounds__(kThreads, 1) attn_prefill_kernel(AttnPrefillArgs a) {
  using S = PrefillSmem<HD>;
  constexpr int DPL = HD / 32;  // output dims per lane
  extern __shared__ __align__(16) uint8_t smem[];
  float* qf = reinterpret_cast<float*>(smem + S::QF);
  float* kT = reinterpret_cast<float*>(smem + S::KTR);
  float* vt = reinterpret_cast<float*>(smem + S::VT);
  float* pw = reinterpret_cast<float*>(smem + S::PW);
  const int G = a.groups;
  const int tq = ROWS / G;
  const int kvh = blockIdx.x;
  const int t0 = blockIdx.y * tq;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int i = tid; i < ROWS * HD; i += kThreads) {
    const int r = i / HD, d = i % HD;
    const int g = r / tq, t = t0 + r % tq;
    qf[i] = t < a.tokens ? __bfloat162float(a.qs[((static_cast<int64_t>(kvh) * G + g) * a.tokens + t) * HD + d]) : 0.f;
  }
  const int t_last = min(t0 + tq, a.tokens) - 1;
  const int n_keys = a.start + t_last + 1;
  const __nv_bfloat16* kc = a.k_cache + static_cast<int64_t>(kvh) * a.max_seq * HD;
  const __nv_bfloat16* vc = a.v_cache + static_cast<int64_t>(kvh) * a.max_seq * HD;

  const int r0 = warp * RPW;
  int tok[RPW];
  float best[RPW], total[RPW], out[RPW][DPL];
#pragma unroll
  for (int x = 0; x < RPW; ++x) {
    tok[x] = t0 + (r0 + x) % tq;
    best[x] = -INFINITY;
    total[x] = 0.f;
#pragma unroll
    for (int d = 0; d < DPL; ++d) out[x][d] = 0.f;
  }

  // Stages keys [kb, kb + KT) (and values) of this KV head; zero past n_keys.
  auto load_tile = [&](int kb, bool values) {
    __syncthreads();  // the previous tile is consumed (and, the first time, the queries are staged)
    for (int i = tid; i < KT * (HD / 8); i += kThreads) {
      const int j = i / (HD / 8), c = (i % (HD / 8)) * 8;
      uint4 ku = make_uint4(0, 0, 0, 0), vu = make_uint4(0, 0, 0, 0);
      if (kb + j < n_keys) {
        ku = __ldg(reinterpret_cast<const uint4*>(kc + static_cast<int64_t>(kb + j) * HD + c));
        if (values) vu = __ldg(reinterpret_cast<const uint4*>(vc + static_cast<int64_t>(kb + j) * HD + c));
      }
      const __nv_bfloat16* kh = reinterpret_cast<const __nv_bfloat16*>(&ku);
      const __nv_bfloat16* vh = reinterpret_cast<const __nv_bfloat16*>(&vu);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        kT[(c + e) * KT + j] = __bfloat162float(kh[e]);
        if (values) vt[j * HD + c + e] = __bfloat162float(vh[e]);
      }
    }
    __syncthreads();
  };
  // Scores of this warp's rows against the staged keys (lane = key), bf16-rounded, -inf where hidden.
  auto scores = [&](int kb, float (&s)[RPW]) {
    float acc[RPW];
#pragma unroll
    for (int x = 0; x < RPW; ++x) acc[x] = 0.f;
#pragma unroll 2
    for (int d = 0; d < HD; d += 4) {
      const float k0 = kT[(d + 0) * KT + lane], k1 = kT[(d + 1) * KT + lane];
      const float k2 = kT[(d + 2) * KT + lane], k3 = kT[(d + 3) * KT + lane];
#pragma unroll
      for (int x = 0; x < RPW; ++x) {
        const float4 q = *reinterpret_cast<const float4*>(qf + (r0 + x) * HD + d);
        acc[x] = fmaf(q.x, k0, acc[x]);
        acc[x] = fmaf(q.y, k1, acc[x]);
        acc[x] = fmaf(q.z, k2, acc[x]);
        acc[x] = fmaf(q.w, k3, acc[x]);
      }
    }
    const int key = kb + lane;
#pragma unroll
    for (int x = 0; x < RPW; ++x) {
      const bool vis = tok[x] < a.tokens && key < n_keys && key <= a.start + tok[x];
      s[x] = vis ? bf16r(acc[x]) : -INFINITY;
    }
  };

  for (int seg = 0; seg < n_keys;) {
    // The keys of one reference block: [seg, seg_end).
    const int64_t blk = ref_block(seg, a.start, a.max_seq);
    int seg_end = seg + 1;
    {
      // ref_block is nondecreasing in the key index: find where it moves past blk.
      int64_t lo = seg, hi = n_keys;  // blk(lo) == blk, answer in (lo, hi]
      while (hi - lo > 1) {
        const int64_t mid = (lo + hi) / 2;
        if (ref_block(mid, a.start, a.max_seq) == blk) lo = mid;
        else hi = mid;
      }
      seg_end = static_cast<int>(hi);
    }
    // Pass 1: the block's maximum per row.
    float bm[RPW];
#pragma unroll
    for (int x = 0; x < RPW; ++x) bm[x] = -INFINITY;
    for (int kb = seg; kb < seg_end; kb += KT) {
      load_tile(kb, false);
      float s[RPW];
      scores(kb, s);
#pragma unroll
      for (int x = 0; x < RPW; ++x) {
        const bool in = kb + lane < seg_end;
        bm[x] = fmaxf(bm[x], warp_max(in ? s[x] : -INFINITY));
      }
    }
    // Pass 2: weights exp(s - nb), their fp32 sum, and the weighted values with bf16 weights.
    float nb[RPW], bsum[RPW], acc[RPW][DPL];
#pragma unroll
    for (int x = 0; x < RPW; ++x) {
      nb[x] = fmaxf(best[x], bm[x]);
      bsum[x] = 0.f;
#pragma unroll
      for (int d = 0; d < DPL; ++d) acc[x][d] = 0.f;
    }
    for (int kb = seg; kb < seg_end; kb += KT) {
      load_tile(kb, true);
      float s[RPW];
      scores(kb, s);
#pragma unroll
      for (int x = 0; x < RPW; ++x) {
        const bool in = kb + lane < seg_end && s[x] != -INFINITY;
        const float p = in ? expf(__fsub_rn(s[x], nb[x])) : 0.f;
        bsum[x] = __fadd_rn(bsum[x], warp_sum(p));
        pw[(r0 + x) * KT + lane] = bf16r(p);
      }
      __syncwarp();
#pragma unroll 4
      for (int j = 0; j < KT; ++j) {
        float vv[DPL];
#pragma unroll
        for (int d = 0; d < DPL; ++d) vv[d] = vt[j * HD + lane * DPL + d];
#pragma unroll
        for (int x = 0; x < RPW; ++x) {
          const float p = pw[(r0 + x) * KT + j];
#pragma unroll
          for (int d = 0; d < DPL; ++d) acc[x][d] = fmaf(p, vv[d], acc[x][d]);
        }
      }
      __syncwarp();
    }
    // Merge the block (the reference's out * rescale + bf16(wts @ values)); rows that see nothing in
    // this block are unchanged (their weights there are exactly zero).
#pragma unroll
    for (int x = 0; x < RPW; ++x) {
      if (bm[x] == -INFINITY) continue;
      const float rescale = best[x] == -INFINITY ? 0.f : expf(__fsub_rn(best[x], nb[x]));
      total[x] = __fadd_rn(__fmul_rn(total[x], rescale), bsum[x]);
#pragma unroll
      for (int d = 0; d < DPL; ++d) out[x][d] = __fadd_rn(__fmul_rn(out[x][d], rescale), bf16r(acc[x][d]));
      best[x] = nb[x];
    }
    seg = seg_end;
  }
  // Epilogue: bf16(out / total) * bf16(sigmoid(gate)), e5m2.
#pragma unroll
  for (int x = 0; x < RPW; ++x) {
    const int t = tok[x];
    if (t >= a.tokens) continue;
    const int h = kvh * G + (r0 + x) / tq;
    const __nv_bfloat16* gate = a.qkv + static_cast<int64_t>(t) * a.ld_qkv + static_cast<int64_t>(h) * 2 * HD + HD;
    uint8_t* dst = a.out + static_cast<int64_t>(t) * a.ld_out + static_cast<int64_t>(h) * HD;
#pragma unroll
    for (int d = 0; d < DPL; ++d) {
      const int dd = lane * DPL + d;
      const float ob = bf16r(__fdiv_rn(out[x][d], total[x]));
      const float gs = bf16r(sigmoidf_(__bfloat162float(gate[dd])));
      dst[dd] = f32_to_e5m2(bf16r(__fmul_rn(ob, gs)));
    }
  }
}

template <int HD>
int launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t stream) {
  using S = PrefillSmem<HD>;
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(attn_prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(S::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(attn_prefill)");
    done_mask |= 1ull << dev;
  }
  const size_t prep_smem = sizeof(float) * (a.num_q_heads + a.num_kv_heads) * HD;
  attn_prefill_prep_kernel<HD><<<a.tokens, kThreads, prep_smem, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "attn_prefill_prep launch");
  const int tq = ROWS / a.groups;
  dim3 grid(a.num_kv_heads, (a.tokens + tq - 1) / tq);
  attn_prefill_kernel<HD><<<grid, kThreads, S::TOTAL, stream>>>(a);
  return q38host::cuda_status(cudaGetLastError(), "attn_prefill launch");
}

}  // namespace

extern "C" size_t q38_attn_prefill_workspace_bytes(int64_t tokens, int num_q_heads, int head_dim) {
  if (tokens <= 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
  return 2 * static_cast<size_t>(tokens) * num_q_heads * head_dim;
}

extern "C" int q38_attn_prefill(const void* qkv, int64_t ld_qkv, const void* q_norm_weight, const void* k_norm_weight,
                                const void* cos, const void* sin, void* k_cache, void* v_cache, int64_t slot,
                                int64_t cache_rows, int64_t max_seq, int64_t tokens, int64_t start, void* out,
                                int64_t ld_out, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                                void* workspace, size_t workspace_bytes, q38_stream_t stream) {
  using namespace q38host;
  if (!qkv || !q_norm_weight || !k_norm_weight || !cos || !sin || !k_cache || !v_cache || !out || !workspace)
    return set_error("q38_attn_prefill: null pointer"), Q38_ERR_ARG;
  if (tokens <= 0 || tokens > 65535 || start < 0 || start + tokens > max_seq)
    return set_error("q38_attn_prefill: chunk %lld + %lld does not fit the cache of %lld positions",
                     static_cast<long long>(start), static_cast<long long>(tokens), static_cast<long long>(max_seq)),
           Q38_ERR_ARG;
  if (slot < 0 || slot >= cache_rows) return set_error("q38_attn_prefill: slot out of range"), Q38_ERR_ARG;
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads)
    return set_error("q38_attn_prefill: bad head counts"), Q38_ERR_ARG;
  if (rot_dim <= 0 || rot_dim > head_dim || rot_dim % 2)
    return set_error("q38_attn_prefill: bad rotary dim %d", rot_dim), Q38_ERR_ARG;
  if (ld_qkv < static_cast<int64_t>(num_q_heads) * 2 * head_dim + 2LL * num_kv_heads * head_dim ||
      ld_out < static_cast<int64_t>(num_q_heads) * head_dim)
    return set_error("q38_attn_prefill: leading dimension too small"), Q38_ERR_ARG;
  if (workspace_bytes < q38_attn_prefill_workspace_bytes(tokens, num_q_heads, head_dim))
    return set_error("q38_attn_prefill: workspace too small"), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u)
    return set_error("q38_attn_prefill: caches must be 16-byte aligned"), Q38_ERR_ARG;
  AttnPrefillArgs a{};
  const int64_t row_elems = static_cast<int64_t>(num_kv_heads) * max_seq * head_dim;
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ld_qkv = ld_qkv;
  a.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_weight);
  a.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_weight);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache) + slot * row_elems;
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache) + slot * row_elems;
  a.max_seq = max_seq;
  a.tokens = static_cast<int>(tokens);
  a.start = static_cast<int>(start);
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.groups = num_q_heads / num_kv_heads;
  a.rot = rot_dim;
  a.eps = eps;
  a.scale = static_cast<float>(1.0 / sqrt(static_cast<double>(head_dim)));
  a.qs = static_cast<__nv_bfloat16*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ROWS % a.groups != 0)
    return set_error("q38_attn_prefill: %d query heads per KV head do not divide %d rows", a.groups, ROWS), Q38_ERR_UNSUPPORTED;
  if (head_dim == 256) return launch_attn_prefill<256>(a, s);
  if (head_dim == 32) return launch_attn_prefill<32>(a, s);
  return set_error("q38_attn_prefill: head_dim %d not built (256, 32 are)", head_dim), Q38_ERR_UNSUPPORTED;
}
