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
//              cache positions 0 .. start + t. Scores and weighted values are mma.sync tensor-core
//              products (BF16 in, fp32 accumulate) over 64-key tiles double-buffered by cp.async. The
//              arithmetic keeps the reference's rounding points: scores are bf16-rounded fp32 dot
//              products (its BF16 matmul); the online softmax walks the reference's own blocks of 2048
//              keys of [cache, chunk], each in two passes (the block's maximum, then weights
//              exp(s - max) summed in fp32 and, rounded to bf16, multiplied into the values); the
//              block's weighted values are rounded to bf16 (its BF16 matmul output) before the fp32
//              rescale-and-add. Output: bf16(out / total) * bf16(sigmoid(gate)) in bf16, then e5m2 for
//              o_proj.
// With the FP8 e4m3 cache (q38_attn_prefill_e4m3) the prep kernel writes the chunk's keys and values as
// cache bytes, and the attention decodes every 64-key tile to bf16(e4m3 * scale) on its way into shared
// memory, so the chunk's own keys and values are read as the cache's round trip of them, as the
// reference attends to them (model.py:748-752).
#include <cmath>

#include "attn_common.cuh"

namespace {

using namespace q38;

constexpr int kThreads = 256;  // prep

struct AttnPrefillArgs {
  const __nv_bfloat16* qkv;  // [tokens, ld_qkv]: per q head [query | gate], then k, then v
  int64_t ld_qkv;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* cos;  // [tokens, rot]
  const __nv_bfloat16* sin;
  uint8_t* k_cache;  // this row: [num_kv_heads][max_seq][HD], bf16 or e4m3 bytes
  uint8_t* v_cache;
  float k_scale, v_scale;  // e4m3 cache
  int64_t max_seq;
  int tokens, start;
  uint8_t* out;
  int64_t ld_out;
  int num_q_heads, num_kv_heads, groups, rot;
  float eps, scale;
  __nv_bfloat16* qs;  // workspace [num_kv_heads][groups][tokens][HD]
};

template <int HD, bool FP8>
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
      const int64_t at = (static_cast<int64_t>(kvh) * a.max_seq + pos) * HD;
      const __nv_bfloat16* vraw = row + static_cast<int64_t>(a.num_q_heads) * 2 * HD +
                                  static_cast<int64_t>(a.num_kv_heads + kvh) * HD;
      for (int d = lane; d < HD; d += 32) {
        if constexpr (FP8) {
          a.k_cache[at + d] = fp8_store(x[d], a.k_scale);
          a.v_cache[at + d] = fp8_store(__bfloat162float(vraw[d]), a.v_scale);
        } else {
          reinterpret_cast<__nv_bfloat16*>(a.k_cache)[at + d] = __float2bfloat16_rn(x[d]);
          reinterpret_cast<__nv_bfloat16*>(a.v_cache)[at + d] = vraw[d];
        }
      }
    }
  }
}

constexpr int PF_WARPS = 6;                   // two per 16-row MMA tile of the CTA's 48 query rows
constexpr int PF_THREADS = PF_WARPS * 32;
constexpr int ROWS = 48;                      // query rows per CTA: G heads x (ROWS / G) tokens
constexpr int KB = 64;                        // keys per tile
constexpr int REF_BLOCK = 2048;               // keys per block of the reference's online softmax

template <int HD>
struct PrefillSmem {
  static constexpr int QP = HD + 8;  // padded bf16 rows: the 8 rows of an ldmatrix land in distinct banks
  static constexpr int PP = KB + 8;
  static constexpr size_t QS = 0;                                      // [ROWS][QP] bf16 queries
  static constexpr size_t KS = QS + 2 * ROWS * QP;                     // [2][KB][QP] bf16 key tiles
  static constexpr size_t VS = KS + 2 * 2 * KB * QP;                   // [2][KB][QP] bf16 value tiles
  static constexpr size_t PS = VS + 2 * 2 * KB * QP;                   // [ROWS][PP] bf16 weights
  static constexpr size_t RED = PS + 2 * ROWS * PP;                    // [2][ROWS] fp32, per half-warp pair
  static constexpr size_t TOTAL = RED + sizeof(float) * 2 * ROWS;
  static_assert(KS % 16 == 0 && VS % 16 == 0 && PS % 16 == 0 && RED % 16 == 0, "16-byte aligned regions");
};

// The reference's softmax block of a key: it concatenates the row's cache (max_seq positions, those
// < start visible) and the chunk's own keys, then walks that sequence in blocks of REF_BLOCK. Here the
// chunk's keys sit in the cache at start .., so key index k < start is cache position k and k >= start
// is own token k - start, at sequence index max_seq + k - start.
__device__ __forceinline__ int64_t ref_block(int64_t key, int64_t start, int64_t max_seq) {
  return (key < start ? key : max_seq + key - start) / REF_BLOCK;
}

// Rows of the CTA: r = g * tq + tt (query head g of the KV head, token t0 + tt), 3 MMA row tiles;
// warp w holds row tile w / 2 and, of each 64-key tile, keys 32 (w % 2) .. + 31 for the scores and
// head dims (w % 2) HD / 2 .. + HD / 2 - 1 for the weighted values. Scores and weighted values run on
// mma.sync (BF16 in, fp32 accumulate): the reference's BF16 matmuls.
template <int HD, bool FP8>
__global__ void __launch_bounds__(PF_THREADS, 1) attn_prefill_kernel(AttnPrefillArgs a) {
  using S = PrefillSmem<HD>;
  constexpr int QP = S::QP, PP = S::PP;
  constexpr int KSTEPS = HD / 16;  // score k-steps over head_dim
  constexpr int NTW = HD / 16;     // weighted-value n-tiles (8 dims) per warp: half the head
  static_assert(NTW % 2 == 0, "n-tiles in pairs per ldmatrix");
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem + S::QS);
  __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(smem + S::KS);
  __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(smem + S::VS);
  __nv_bfloat16* ps = reinterpret_cast<__nv_bfloat16*>(smem + S::PS);
  float* red = reinterpret_cast<float*>(smem + S::RED);
  const int G = a.groups;
  const int tq = ROWS / G;
  const int kvh = blockIdx.x;
  const int t0 = blockIdx.y * tq;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wm = warp >> 1, wh = warp & 1;
  const int t_last = min(t0 + tq, a.tokens) - 1;
  const int n_keys = a.start + t_last + 1;
  const __nv_bfloat16* kc = reinterpret_cast<const __nv_bfloat16*>(a.k_cache) + static_cast<int64_t>(kvh) * a.max_seq * HD;
  const __nv_bfloat16* vc = reinterpret_cast<const __nv_bfloat16*>(a.v_cache) + static_cast<int64_t>(kvh) * a.max_seq * HD;
  const uint8_t* kc8 = a.k_cache + static_cast<int64_t>(kvh) * a.max_seq * HD;  // e4m3 cache
  const uint8_t* vc8 = a.v_cache + static_cast<int64_t>(kvh) * a.max_seq * HD;

  // Queries (rows past the chunk are zero).
  for (int i = tid; i < ROWS * (HD / 8); i += PF_THREADS) {
    const int r = i / (HD / 8), c = i % (HD / 8);
    const int g = r / tq, t = t0 + r % tq;
    const __nv_bfloat16* src = a.qs + ((static_cast<int64_t>(kvh) * G + g) * a.tokens + min(t, a.tokens - 1)) * HD + 8 * c;
    cp_async16(smem_u32(qs + r * QP + 8 * c), src, t < a.tokens ? 16u : 0u);
  }
  cp_async_commit();

  // This thread's two rows (MMA fragment rows lane / 4 and + 8 of its row tile): key bounds.
  const int rlo = 16 * wm + (lane >> 2), rhi = rlo + 8;
  const int tlo = t0 + rlo % tq, thi = t0 + rhi % tq;
  const int lim_lo = tlo < a.tokens ? a.start + tlo + 1 : 0;  // keys < lim are visible to the row
  const int lim_hi = thi < a.tokens ? a.start + thi + 1 : 0;

  // Keys [kb, kb + KB) (and values) into buffer `buf`; zero past n_keys.
  auto load_tile = [&](int kb, int buf, bool values) {
    __nv_bfloat16* kd = ks + buf * KB * QP;
    __nv_bfloat16* vd = vs + buf * KB * QP;
    if constexpr (FP8) {
      // Decoded on the way in: every 16-byte piece loaded before any is stored.
      constexpr int PIECES = KB * (HD / 16), PER = (PIECES + PF_THREADS - 1) / PF_THREADS;
      uint4 rk[PER], rv[PER];
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int i = tid + u * PF_THREADS, j = i / (HD / 16), c = i % (HD / 16);
        const bool in = i < PIECES && kb + j < n_keys;
        const int64_t off = static_cast<int64_t>(kb + j) * HD + 16 * c;
        rk[u] = in ? *reinterpret_cast<const uint4*>(kc8 + off) : make_uint4(0u, 0u, 0u, 0u);
        rv[u] = in && values ? *reinterpret_cast<const uint4*>(vc8 + off) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        const int i = tid + u * PF_THREADS, j = i / (HD / 16), c = i % (HD / 16);
        if (i >= PIECES) break;
        uint4 lo, hi;
        fp8_load16(rk[u], a.k_scale, lo, hi);
        *reinterpret_cast<uint4*>(kd + j * QP + 16 * c) = lo;
        *reinterpret_cast<uint4*>(kd + j * QP + 16 * c + 8) = hi;
        if (values) {
          fp8_load16(rv[u], a.v_scale, lo, hi);
          *reinterpret_cast<uint4*>(vd + j * QP + 16 * c) = lo;
          *reinterpret_cast<uint4*>(vd + j * QP + 16 * c + 8) = hi;
        }
      }
      return;
    }
    for (int i = tid; i < KB * (HD / 8); i += PF_THREADS) {
      const int j = i / (HD / 8), c = i % (HD / 8);
      const int key = kb + j;
      const bool in = key < n_keys;
      const int64_t off = static_cast<int64_t>(in ? key : 0) * HD + 8 * c;
      cp_async16(smem_u32(kd + j * QP + 8 * c), kc + off, in ? 16u : 0u);
      if (values) cp_async16(smem_u32(vd + j * QP + 8 * c), vc + off, in ? 16u : 0u);
    }
    cp_async_commit();
  };
  // This warp's scores: its 16 rows x 32 keys of the tile in buffer `buf`, bf16-rounded, -inf where
  // the key is hidden from the row or outside [kb, kend).
  auto scores = [&](int buf, int kb, int kend, float (&s)[4][4]) {
    const __nv_bfloat16* kt = ks + buf * KB * QP;
    float acc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    const uint32_t abase = smem_u32(qs + (16 * wm + (lane & 15)) * QP + 8 * (lane >> 4));
    const int krow = 32 * wh + (lane & 7) + 8 * (lane >> 4);
#pragma unroll
    for (int k = 0; k < KSTEPS; ++k) {
      uint32_t af[4];
      ldsm_x4(abase + k * 32, af[0], af[1], af[2], af[3]);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;  // keys 16 np + 0..7 (b0, b1) and + 8..15 (b2, b3), dims 16 k .. + 15
        ldsm_x4(smem_u32(kt + (krow + 16 * np) * QP + 16 * k + 8 * ((lane >> 3) & 1)), b0, b1, b2, b3);
        mma_bf16_16816(acc[2 * np], af, b0, b1);
        mma_bf16_16816(acc[2 * np + 1], af, b2, b3);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int key = kb + 32 * wh + 8 * nt + 2 * (lane & 3);
      s[nt][0] = key < kend && key < lim_lo ? bf16r(acc[nt][0]) : -INFINITY;
      s[nt][1] = key + 1 < kend && key + 1 < lim_lo ? bf16r(acc[nt][1]) : -INFINITY;
      s[nt][2] = key < kend && key < lim_hi ? bf16r(acc[nt][2]) : -INFINITY;
      s[nt][3] = key + 1 < kend && key + 1 < lim_hi ? bf16r(acc[nt][3]) : -INFINITY;
    }
  };
  // Per row across the two warps of a row tile: red[half][row], combined half 0 then half 1.
  auto pair_combine = [&](float lo, float hi, bool is_max, float& out_lo, float& out_hi) {
    if ((lane & 3) == 0) {
      red[wh * ROWS + rlo] = lo;
      red[wh * ROWS + rhi] = hi;
    }
    __syncthreads();
    out_lo = is_max ? fmaxf(red[rlo], red[ROWS + rlo]) : __fadd_rn(red[rlo], red[ROWS + rlo]);
    out_hi = is_max ? fmaxf(red[rhi], red[ROWS + rhi]) : __fadd_rn(red[rhi], red[ROWS + rhi]);
    __syncthreads();  // red is read before it is written again
  };

  float out[NTW][4];
#pragma unroll
  for (int n = 0; n < NTW; ++n) out[n][0] = out[n][1] = out[n][2] = out[n][3] = 0.f;
  float best_lo = -INFINITY, best_hi = -INFINITY, tot_lo = 0.f, tot_hi = 0.f;

  for (int seg = 0; seg < n_keys;) {
    // The keys of one reference block: [seg, seg_end).
    const int64_t blk = ref_block(seg, a.start, a.max_seq);
    int seg_end;
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
    // Pass 1: the block's maximum score per row.
    float bm_lo = -INFINITY, bm_hi = -INFINITY;
    load_tile(seg, 0, false);
    for (int kb = seg, buf = 0; kb < seg_end; kb += KB, buf ^= 1) {
      if (kb + KB < seg_end) {
        load_tile(kb + KB, buf ^ 1, false);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      float sc[4][4];
      scores(buf, kb, seg_end, sc);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        bm_lo = fmaxf(bm_lo, fmaxf(sc[nt][0], sc[nt][1]));
        bm_hi = fmaxf(bm_hi, fmaxf(sc[nt][2], sc[nt][3]));
      }
      __syncthreads();  // the tile is consumed before its buffer is refilled
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      bm_lo = fmaxf(bm_lo, __shfl_xor_sync(0xffffffffu, bm_lo, o));
      bm_hi = fmaxf(bm_hi, __shfl_xor_sync(0xffffffffu, bm_hi, o));
    }
    pair_combine(bm_lo, bm_hi, true, bm_lo, bm_hi);
    // Pass 2: weights exp(s - nb), their fp32 sum, and the weighted values with bf16 weights.
    const float nb_lo = fmaxf(best_lo, bm_lo), nb_hi = fmaxf(best_hi, bm_hi);
    float acc[NTW][4];
#pragma unroll
    for (int n = 0; n < NTW; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    float bs_lo = 0.f, bs_hi = 0.f;
    load_tile(seg, 0, true);
    for (int kb = seg, buf = 0; kb < seg_end; kb += KB, buf ^= 1) {
      if (kb + KB < seg_end) {
        load_tile(kb + KB, buf ^ 1, true);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncthreads();
      float sc[4][4];
      scores(buf, kb, seg_end, sc);
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const float p0 = sc[nt][0] == -INFINITY ? 0.f : expf(__fsub_rn(sc[nt][0], nb_lo));
        const float p1 = sc[nt][1] == -INFINITY ? 0.f : expf(__fsub_rn(sc[nt][1], nb_lo));
        const float p2 = sc[nt][2] == -INFINITY ? 0.f : expf(__fsub_rn(sc[nt][2], nb_hi));
        const float p3 = sc[nt][3] == -INFINITY ? 0.f : expf(__fsub_rn(sc[nt][3], nb_hi));
        bs_lo = __fadd_rn(__fadd_rn(bs_lo, p0), p1);
        bs_hi = __fadd_rn(__fadd_rn(bs_hi, p2), p3);
        const int col = 32 * wh + 8 * nt + 2 * (lane & 3);
        *reinterpret_cast<uint32_t*>(ps + rlo * PP + col) = pack_bf16x2(p0, p1);
        *reinterpret_cast<uint32_t*>(ps + rhi * PP + col) = pack_bf16x2(p2, p3);
      }
      // The two warps of this row tile have written its weights.
      asm volatile("bar.sync %0, %1;" ::"r"(1 + wm), "r"(64) : "memory");
      const uint32_t pbase = smem_u32(ps + (16 * wm + (lane & 15)) * PP + 8 * (lane >> 4));
      const __nv_bfloat16* vt = vs + buf * KB * QP;
#pragma unroll
      for (int k = 0; k < KB / 16; ++k) {
        uint32_t pa[4];
        ldsm_x4(pbase + k * 32, pa[0], pa[1], pa[2], pa[3]);
        const int vr = 16 * k + (lane & 7) + 8 * ((lane >> 3) & 1);  // x4.trans: (keys 0-7 | 8-15) x (n | n + 1)
#pragma unroll
        for (int n = 0; n < NTW; n += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(smem_u32(vt + vr * QP + wh * (HD / 2) + 8 * (n + (lane >> 4))), b0, b1, b2, b3);
          mma_bf16_16816(acc[n], pa, b0, b1);
          mma_bf16_16816(acc[n + 1], pa, b2, b3);
        }
      }
      __syncthreads();  // keys, values and weights are consumed before the buffers are refilled
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      bs_lo = __fadd_rn(bs_lo, __shfl_xor_sync(0xffffffffu, bs_lo, o));
      bs_hi = __fadd_rn(bs_hi, __shfl_xor_sync(0xffffffffu, bs_hi, o));
    }
    pair_combine(bs_lo, bs_hi, false, bs_lo, bs_hi);
    // Merge the block (the reference's out * rescale + bf16(wts @ values)); rows that see nothing in
    // this block are unchanged (their weights there are exactly zero).
    if (bm_lo != -INFINITY) {
      const float rescale = best_lo == -INFINITY ? 0.f : expf(__fsub_rn(best_lo, nb_lo));
      tot_lo = __fadd_rn(__fmul_rn(tot_lo, rescale), bs_lo);
#pragma unroll
      for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) out[n][e] = __fadd_rn(__fmul_rn(out[n][e], rescale), bf16r(acc[n][e]));
      best_lo = nb_lo;
    }
    if (bm_hi != -INFINITY) {
      const float rescale = best_hi == -INFINITY ? 0.f : expf(__fsub_rn(best_hi, nb_hi));
      tot_hi = __fadd_rn(__fmul_rn(tot_hi, rescale), bs_hi);
#pragma unroll
      for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 2; e < 4; ++e) out[n][e] = __fadd_rn(__fmul_rn(out[n][e], rescale), bf16r(acc[n][e]));
      best_hi = nb_hi;
    }
    seg = seg_end;
  }
  // Epilogue: bf16(out / total) * bf16(sigmoid(gate)), e5m2.
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = half ? rhi : rlo;
    const int t = half ? thi : tlo;
    if (t >= a.tokens) continue;
    const float total = half ? tot_hi : tot_lo;
    const int h = kvh * G + r / tq;
    const __nv_bfloat16* gate = a.qkv + static_cast<int64_t>(t) * a.ld_qkv + static_cast<int64_t>(h) * 2 * HD + HD;
    uint8_t* dst = a.out + static_cast<int64_t>(t) * a.ld_out + static_cast<int64_t>(h) * HD;
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int dd = wh * (HD / 2) + 8 * n + 2 * (lane & 3) + e;
        const float ob = bf16r(__fdiv_rn(out[n][2 * half + e], total));
        const float gs = bf16r(sigmoidf_(__bfloat162float(gate[dd])));
        dst[dd] = f32_to_e5m2(bf16r(__fmul_rn(ob, gs)));
      }
  }
}

template <int HD, bool FP8>
int launch_attn_prefill(const AttnPrefillArgs& a, cudaStream_t stream) {
  using S = PrefillSmem<HD>;
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(attn_prefill_kernel<HD, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(S::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(attn_prefill)");
    done_mask |= 1ull << dev;
  }
  const size_t prep_smem = sizeof(float) * (a.num_q_heads + a.num_kv_heads) * HD;
  attn_prefill_prep_kernel<HD, FP8><<<a.tokens, kThreads, prep_smem, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "attn_prefill_prep launch");
  const int tq = ROWS / a.groups;
  dim3 grid(a.num_kv_heads, (a.tokens + tq - 1) / tq);
  attn_prefill_kernel<HD, FP8><<<grid, PF_THREADS, S::TOTAL, stream>>>(a);
  return q38host::cuda_status(cudaGetLastError(), "attn_prefill launch");
}

}  // namespace

extern "C" size_t q38_attn_prefill_workspace_bytes(int64_t tokens, int num_q_heads, int head_dim) {
  if (tokens <= 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
  return 2 * static_cast<size_t>(tokens) * num_q_heads * head_dim;
}

namespace {

int attn_prefill_any(const void* qkv, int64_t ld_qkv, const void* q_norm_weight, const void* k_norm_weight,
                     const void* cos, const void* sin, void* k_cache, void* v_cache, bool fp8, float k_scale,
                     float v_scale, int64_t slot, int64_t cache_rows, int64_t max_seq, int64_t tokens, int64_t start,
                     void* out, int64_t ld_out, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
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
  if (fp8 && !(k_scale > 0.f && v_scale > 0.f && std::isfinite(k_scale) && std::isfinite(v_scale)))
    return set_error("q38_attn_prefill_e4m3: scales must be positive"), Q38_ERR_ARG;
  AttnPrefillArgs a{};
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * max_seq * head_dim * (fp8 ? 1 : 2);
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ld_qkv = ld_qkv;
  a.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_weight);
  a.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_weight);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.k_cache = static_cast<uint8_t*>(k_cache) + slot * row_bytes;
  a.v_cache = static_cast<uint8_t*>(v_cache) + slot * row_bytes;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
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
  if (head_dim == 256) return fp8 ? launch_attn_prefill<256, true>(a, s) : launch_attn_prefill<256, false>(a, s);
  if (head_dim == 32) return fp8 ? launch_attn_prefill<32, true>(a, s) : launch_attn_prefill<32, false>(a, s);
  return set_error("q38_attn_prefill: head_dim %d not built (256, 32 are)", head_dim), Q38_ERR_UNSUPPORTED;
}

}  // namespace

extern "C" int q38_attn_prefill(const void* qkv, int64_t ld_qkv, const void* q_norm_weight, const void* k_norm_weight,
                                const void* cos, const void* sin, void* k_cache, void* v_cache, int64_t slot,
                                int64_t cache_rows, int64_t max_seq, int64_t tokens, int64_t start, void* out,
                                int64_t ld_out, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                                void* workspace, size_t workspace_bytes, q38_stream_t stream) {
  return attn_prefill_any(qkv, ld_qkv, q_norm_weight, k_norm_weight, cos, sin, k_cache, v_cache, false, 1.f, 1.f, slot,
                          cache_rows, max_seq, tokens, start, out, ld_out, num_q_heads, num_kv_heads, head_dim, rot_dim,
                          eps, workspace, workspace_bytes, stream);
}

extern "C" int q38_attn_prefill_e4m3(const void* qkv, int64_t ld_qkv, const void* q_norm_weight,
                                     const void* k_norm_weight, const void* cos, const void* sin, void* k_cache,
                                     void* v_cache, float k_scale, float v_scale, int64_t slot, int64_t cache_rows,
                                     int64_t max_seq, int64_t tokens, int64_t start, void* out, int64_t ld_out,
                                     int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                                     void* workspace, size_t workspace_bytes, q38_stream_t stream) {
  return attn_prefill_any(qkv, ld_qkv, q_norm_weight, k_norm_weight, cos, sin, k_cache, v_cache, true, k_scale, v_scale,
                          slot, cache_rows, max_seq, tokens, start, out, ld_out, num_q_heads, num_kv_heads, head_dim,
                          rot_dim, eps, workspace, workspace_bytes, stream);
}
