// Gated full attention over long caches, split along the cache: decode (one token per row) and
// verify (K tokens per row) against a BF16 or an FP8 e4m3 cache with static scales, for any cache
// length. FullAttentionStep.forward / verify (qwen38_inf2/model.py:610-675) with the cache formats
// of _store / _load / _round_trip (:579-593).
//
// The reference rounds the scores to bf16 (BF16 matmul), takes a fp32 softmax over the whole row
// (cache positions < position, then the step's own keys, causal among themselves), rounds the
// normalised weights to bf16 and multiplies them into the values as a BF16 matmul:
// out = bf16(bf16(W_cache V) + bf16(W_own V_own)). A weight can only be rounded once the row's maximum
// and sum are known, so the row is split into chunks of the cache and taken in three launches:
//   1. scores: per (chunk, row, KV head) CTA, the bf16 scores of its positions for the G x K query
//      rows (queries normed and rotated in the CTA), stored in the workspace, with the chunk's maximum
//      and sum of exponentials; chunk 0 also stores the own-key scores;
//   2. values: per (chunk, row, KV head) CTA, the row's maximum and sum from every chunk's statistics
//      (the same order in every CTA), the bf16 weights of its positions, and their product with its V
//      positions as a fp32 partial;
//   3. finish: per (row, KV head), the partials summed in chunk order and rounded once, the own term,
//      the gate, e5m2 out; then the step's keys and values go into the cache.
// The cache is streamed once for K and once for V over as many CTAs as fill the GPU, so a few rows at
// 32K positions run at HBM speed. FP8 cache tiles arrive as bytes (one bulk copy per 32 positions) and
// are decoded to bf16(e4m3 * scale) in shared memory before the tensor cores read them.
#include <cmath>

#include "attn_common.cuh"

namespace {

using namespace q38;

constexpr int kWarps = 4;                      // compute warps
constexpr int kThreads = (kWarps + 1) * 32;    // + one copy warp
constexpr int KT = 32;                         // cache positions per tile
constexpr int kStages = 4;                     // tiles in flight per CTA
constexpr int kMaxRows = 32;                   // query rows per (row, KV head): groups x tokens
constexpr int kMaxTokens = 8;                  // verify tokens
constexpr int kMaxChunk = 512;                 // cache positions per chunk
constexpr int kFinishThreads = 512;            // threads of a finishing CTA
constexpr int kFinishSlices = 4;               // finishing CTAs per (row, KV head)

__host__ __device__ constexpr size_t al16(size_t x) { return (x + 15) & ~size_t(15); }

struct SplitArgs {
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  const __nv_bfloat16* q_norm_w;
  const __nv_bfloat16* k_norm_w;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  uint8_t* k_cache;  // bf16 or e4m3 [batch][kv heads][max_seq][HD]
  uint8_t* v_cache;
  float k_scale, v_scale;  // FP8 cache: the static scales (bf16 values)
  int64_t max_seq;
  const int32_t* position;
  const float* active;
  uint8_t* out;
  int64_t ld_out;
  int num_q_heads, num_kv_heads, groups, tokens, rows, rot;  // rows = groups * tokens
  float eps;
  int chunk, nchunks;
  int64_t seq_pad;        // score row length in the workspace
  __nv_bfloat16* scores;  // [pairs][rows][seq_pad]
  float* stats;           // [pairs][nchunks][rows][2]: chunk maximum, sum of exp(score - maximum)
  float* own;             // [pairs][rows][tokens]: own-key scores (bf16 values), -inf where not visible
  float* part;            // [pairs][nchunks][rows][HD]: fp32 partial products W V
};

template <int HD>
struct Geom {
  static constexpr bool kSwizzle = HD >= 64;
  static constexpr int kBoxCols = kSwizzle ? 64 : HD;
  static constexpr int kBoxes = HD / kBoxCols;
  static constexpr int kBoxBytes = KT * kBoxCols * 2;
  static constexpr int kTileBytes = KT * HD * 2;  // bf16 tile
  static constexpr int kRawBytes = KT * HD;       // e4m3 tile
  // Byte offset of 16-byte chunk `c` (8 dims) of position row `r` in a bf16 tile (the tensor copy's
  // 128-byte swizzle: chunk c of a 128-byte row r stored at chunk c ^ (r % 8)).
  __device__ static __forceinline__ uint32_t at(int r, int c) {
    if constexpr (kSwizzle) return static_cast<uint32_t>((c >> 3) * kBoxBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
    else return static_cast<uint32_t>(r * HD * 2 + c * 16);
  }
};

__device__ __forceinline__ void compute_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kWarps * 32) : "memory"); }

// One (row, KV head) pair: its rows' visible cache length, and where token t's key and value go.
struct Pair {
  int b, g, pair, n_read;
  bool on;
  int64_t pos;
};
__device__ __forceinline__ Pair pair_of(const SplitArgs& a, int g, int b) {
  Pair p;
  p.b = b;
  p.g = g;
  p.pair = b * a.num_kv_heads + g;
  p.on = a.active[b] > 0.5f;
  p.pos = a.position[b] < 0 ? 0 : a.position[b];
  p.n_read = p.on ? static_cast<int>(p.pos < a.max_seq ? p.pos : a.max_seq) : 0;
  return p;
}
__device__ __forceinline__ int64_t write_position(const SplitArgs& a, const Pair& p, int t) {
  const int64_t w = p.on ? p.pos + t : a.max_seq - a.tokens + t;
  return w < a.max_seq ? w : a.max_seq - 1;
}

// The row's softmax statistics over every chunk and the own keys, in one fixed order (the same in
// every CTA that needs them): maximum m and sum of exp(score * scale - m).
__device__ __forceinline__ void row_stats(const SplitArgs& a, int pair, int r, int live, float scale, int lane, float& m,
                                          float& sum) {
  const float* st = a.stats + (static_cast<int64_t>(pair) * a.nchunks) * a.rows * 2;
  const float* own = a.own + (static_cast<int64_t>(pair) * a.rows + r) * a.tokens;
  float mx = -INFINITY;
  for (int c = lane; c < live; c += 32) mx = fmaxf(mx, st[(static_cast<int64_t>(c) * a.rows + r) * 2]);
  for (int t = lane; t < a.tokens; t += 32) mx = fmaxf(mx, __fmul_rn(own[t], scale));
  mx = warp_max(mx);
  float s = 0.f;
  for (int c = lane; c < live; c += 32) {
    const float* e = st + (static_cast<int64_t>(c) * a.rows + r) * 2;
    if (e[1] > 0.f) s += e[1] * expf(__fsub_rn(e[0], mx));
  }
  for (int t = lane; t < a.tokens; t += 32)
    if (own[t] > -INFINITY) s += expf(__fsub_rn(__fmul_rn(own[t], scale), mx));
  m = mx;
  sum = warp_sum(s);
}

// Shared memory layout of the two streaming kernels (offsets from a 1024-byte aligned base).
template <int HD, bool FP8>
struct Layout {
  size_t ring, work, q, qf, prm, sc, kown, bars, total;
  int rowp, scw;
  // mrows: the query rows the MMA tiles cover (16 x MT), which the query and score buffers hold.
  __host__ __device__ Layout(int rows, int tokens, int chunk, int rot, int mrows) {
    rowp = HD + 8;
    scw = chunk + 8;
    size_t off = 0;
    auto take = [&](size_t bytes) {
      const size_t at = off;
      off = al16(off + bytes);
      return at;
    };
    ring = take(static_cast<size_t>(kStages) * (FP8 ? Geom<HD>::kRawBytes : Geom<HD>::kTileBytes));
    work = FP8 ? take(2 * static_cast<size_t>(Geom<HD>::kTileBytes)) : 0;  // decoded tiles (double buffered)
    q = take(static_cast<size_t>(mrows) * rowp * 2);                     // queries bf16 (scores kernel)
    qf = take(static_cast<size_t>(rows) * HD * 4);                        // query staging fp32
    prm = take(static_cast<size_t>(2) * HD * 2 + static_cast<size_t>(2) * tokens * (rot > 0 ? rot : 1) * 2);
    sc = take(static_cast<size_t>(mrows) * scw * 2);                      // scores / weights bf16
    kown = take(static_cast<size_t>(tokens) * HD * 4);                    // own keys fp32
    bars = take(2 * kStages * 8);
    total = off + 1024;
  }
};

// Decodes raw e4m3 tile rows [0, valid) into the bf16 tile (rows from `valid` on: zeros).
template <int HD>
__device__ __forceinline__ void decode_tile(const uint8_t* raw, uint8_t* tile, int valid, float scale, int tid) {
  using T = Geom<HD>;
  constexpr int CPR = HD / 16;  // raw 16-byte chunks per row
  for (int i = tid; i < KT * CPR; i += kWarps * 32) {
    const int r = i / CPR, c = i % CPR;
    uint4 lo = make_uint4(0u, 0u, 0u, 0u), hi = lo;
    if (r < valid) fp8_load16(*reinterpret_cast<const uint4*>(raw + r * HD + c * 16), scale, lo, hi);
    *reinterpret_cast<uint4*>(tile + T::at(r, 2 * c)) = lo;
    *reinterpret_cast<uint4*>(tile + T::at(r, 2 * c + 1)) = hi;
  }
}

// Copy warp: the tiles [p0, p1) of one (row, KV head)'s K or V cache into the ring. BF16: tensor
// copies (the box past the cache's end is zero-filled). FP8: one bulk copy of the valid rows.
template <int HD, bool FP8>
__device__ void copy_tiles(const CUtensorMap* map, const uint8_t* cache, int64_t row0, int p0, int p1, uint8_t* ring,
                           uint64_t* full, uint64_t* empty) {
  using T = Geom<HD>;
  const int ntiles = (p1 - p0 + KT - 1) / KT;
  if (!FP8) prefetch_tmap(map);
  for (int i = 0; i < ntiles; ++i) {
    const int s = i % kStages;
    if (i >= kStages && !mbar_wait(&empty[s], ((i / kStages) - 1) & 1)) break;
    const int p = p0 + i * KT;
    if constexpr (FP8) {
      const int valid = min(KT, p1 - p);
      const uint32_t bytes = static_cast<uint32_t>(valid * HD);
      mbar_arrive_expect_tx(&full[s], bytes);
      bulk_load(ring + s * T::kRawBytes, cache + (row0 + p) * HD, bytes, &full[s]);
    } else {
      mbar_arrive_expect_tx(&full[s], T::kTileBytes);
#pragma unroll
      for (int bx = 0; bx < T::kBoxes; ++bx)
        tma_load_2d(ring + s * T::kTileBytes + bx * T::kBoxBytes, map, &full[s], bx * T::kBoxCols, static_cast<int>(row0 + p));
    }
  }
  // Never leave with copies in flight.
  for (int i = max(0, ntiles - kStages); i < ntiles; ++i) mbar_wait(&full[i % kStages], (i / kStages) & 1);
}

// The bf16 tile of ring slot s for tile index i (FP8: decoded into one of two work tiles first; every
// compute warp takes part, and the barrier after the decode also orders the previous tile's reads of
// the other work tile before its next reuse).
template <int HD, bool FP8>
__device__ __forceinline__ uint32_t tile_for(uint8_t* ring, uint8_t* work, uint64_t* full, uint64_t* empty, int i, int valid,
                                             float scale, int tid, int lane) {
  using T = Geom<HD>;
  const int s = i % kStages;
  mbar_wait(&full[s], (i / kStages) & 1);
  if constexpr (FP8) {
    uint8_t* tile = work + (i & 1) * T::kTileBytes;
    decode_tile<HD>(ring + s * T::kRawBytes, tile, valid, scale, tid);
    compute_bar();
    if (lane == 0) mbar_arrive(&empty[s]);
    return smem_u32(tile);
  } else {
    return smem_u32(ring + s * T::kTileBytes);
  }
}

// Queries of the pair's rows (r = t * groups + h) normed and rotated into `qs` (bf16, rows past `rows`
// zero), with the fp32 copies in `qf`; with `keys`, the step's own keys too (as the cache holds them).
template <int HD, bool FP8>
__device__ void stage_queries(const SplitArgs& a, const Pair& p, __nv_bfloat16* qs, int rowp, int mrows, float* qf,
                              __nv_bfloat16* prm, float* kown, bool keys, int tid, int warp, int lane) {
  const int G = a.groups, K = a.tokens, rot = a.rot > 0 ? a.rot : 1;
  __nv_bfloat16* wq = prm;
  __nv_bfloat16* wk = wq + HD;
  __nv_bfloat16* cs = wk + HD;  // [K][rot]
  __nv_bfloat16* sn = cs + K * rot;
  for (int i = tid; i < HD; i += kWarps * 32) {
    wq[i] = a.q_norm_w[i];
    wk[i] = a.k_norm_w[i];
  }
  for (int i = tid; i < K * a.rot; i += kWarps * 32) {
    const int t = i / a.rot, d = i % a.rot;
    cs[t * rot + d] = a.cos[(static_cast<int64_t>(p.b) * K + t) * a.rot + d];
    sn[t * rot + d] = a.sin[(static_cast<int64_t>(p.b) * K + t) * a.rot + d];
  }
  for (int i = tid; i < a.rows * HD; i += kWarps * 32) {
    const int r = i / HD, d = i % HD, t = r / G, h = r % G;
    const __nv_bfloat16* row = a.qkv + (static_cast<int64_t>(p.b) * K + t) * a.ld_qkv;
    qf[i] = __bfloat162float(row[static_cast<int64_t>(p.g * G + h) * 2 * HD + d]);
  }
  if (keys) {
    for (int i = tid; i < K * HD; i += kWarps * 32) {
      const int t = i / HD, d = i % HD;
      const __nv_bfloat16* row = a.qkv + (static_cast<int64_t>(p.b) * K + t) * a.ld_qkv;
      kown[i] = __bfloat162float(row[static_cast<int64_t>(a.num_q_heads) * 2 * HD + static_cast<int64_t>(p.g) * HD + d]);
    }
  }
  compute_bar();
  const int nrows = a.rows + (keys ? K : 0);
  for (int r = warp; r < nrows; r += kWarps) {
    const bool is_q = r < a.rows;
    const int t = is_q ? r / G : r - a.rows;
    float* x = is_q ? qf + r * HD : kown + t * HD;
    norm_rope_head<HD>(x, is_q ? wq : wk, cs + t * rot, sn + t * rot, a.rot, a.eps, lane);
    if (!is_q && FP8) {
      for (int d = lane; d < HD; d += 32) x[d] = fp8_load(fp8_store(x[d], a.k_scale), a.k_scale);
      __syncwarp();
    }
  }
  compute_bar();
  for (int i = tid; i < mrows * HD; i += kWarps * 32) {
    const int r = i / HD, d = i % HD;
    qs[r * rowp + d] = __float2bfloat16_rn(r < a.rows ? qf[i] : 0.f);
  }
  compute_bar();
}

// ---- launch 1: scores and their per-chunk statistics --------------------------------------------
template <int HD, int MT, bool FP8>
__global__ void __launch_bounds__(kThreads, 1) split_scores_kernel(const __grid_constant__ CUtensorMap tmap_k, SplitArgs a) {
  using T = Geom<HD>;
  constexpr int KSTEPS = HD / 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout<HD, FP8> L(a.rows, a.tokens, a.chunk, a.rot, MT * 16);
  uint8_t* ring = smem + L.ring;
  uint8_t* work = smem + L.work;
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem + L.q);
  float* qf = reinterpret_cast<float*>(smem + L.qf);
  __nv_bfloat16* prm = reinterpret_cast<__nv_bfloat16*>(smem + L.prm);
  __nv_bfloat16* sc = reinterpret_cast<__nv_bfloat16*>(smem + L.sc);
  float* kown = reinterpret_cast<float*>(smem + L.kown);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kStages;

  pdl_wait();
  pdl_trigger();
  const Pair p = pair_of(a, blockIdx.y, blockIdx.z);
  const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int p0 = c * a.chunk, p1 = min(p0 + a.chunk, p.n_read);
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));
  float* stats = a.stats + ((static_cast<int64_t>(p.pair) * a.nchunks + c) * a.rows) * 2;
  if (p0 >= p1 && c != 0) return;  // past the row's visible cache: nothing to read, no statistics used

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t row0 = static_cast<int64_t>(p.pair) * a.max_seq;
  if (warp == kWarps) {
    if (lane == 0 && p0 < p1) copy_tiles<HD, FP8>(&tmap_k, a.k_cache, row0, p0, p1, ring, full, empty);
    return;
  }
  stage_queries<HD, FP8>(a, p, qs, L.rowp, MT * 16, qf, prm, kown, c == 0, tid, warp, lane);
  if (c == 0) {
    // Own-key scores: bf16(q . k_own) for the visible own keys (token t sees own tokens 0 .. t).
    for (int i = warp; i < a.rows * a.tokens; i += kWarps) {
      const int r = i / a.tokens, t2 = i % a.tokens;
      float d = 0.f;
      for (int e = lane; e < HD; e += 32) d += qf[r * HD + e] * kown[t2 * HD + e];
      d = warp_sum(d);
      if (lane == 0)
        a.own[(static_cast<int64_t>(p.pair) * a.rows + r) * a.tokens + t2] = t2 <= r / a.groups ? bf16r(d) : -INFINITY;
    }
  }

  // Scores of this chunk: S[rows x 8 positions] per warp and tile, bf16 into sc.
  const int ntiles = (p1 - p0 + KT - 1) / KT;
  const int n0 = warp * 8;
  for (int i = 0; i < ntiles; ++i) {
    const uint32_t tile = tile_for<HD, FP8>(ring, work, full, empty, i, min(KT, p1 - p0 - i * KT), a.k_scale, tid, lane);
    float acc[MT][4] = {};
    const int r = n0 + (lane & 7);
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ks += 2) {
      uint32_t b0, b1, b2, b3;
      ldsm_x4(tile + T::at(r, 2 * ks + (lane >> 3)), b0, b1, b2, b3);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t qa[4], qb[4];
        const uint32_t qaddr = smem_u32(qs + (mt * 16 + (lane & 15)) * L.rowp + (lane >> 4) * 8);
        ldsm_x4(qaddr + ks * 32, qa[0], qa[1], qa[2], qa[3]);
        ldsm_x4(qaddr + (ks + 1) * 32, qb[0], qb[1], qb[2], qb[3]);
        mma_bf16_16816(acc[mt], qa, b0, b1);
        mma_bf16_16816(acc[mt], qb, b2, b3);
      }
    }
    if constexpr (!FP8) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[i % kStages]);
    }
    const int pl = i * KT + n0 + 2 * (lane & 3);  // position within the chunk
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int qr = mt * 16 + (lane >> 2) + hh * 8;
        if (qr < a.rows) {
          if (p0 + pl < p1) sc[qr * L.scw + pl] = __float2bfloat16_rn(acc[mt][2 * hh]);
          if (p0 + pl + 1 < p1) sc[qr * L.scw + pl + 1] = __float2bfloat16_rn(acc[mt][2 * hh + 1]);
        }
      }
  }
  compute_bar();
  // Per query row: the chunk's maximum of score * scale and sum of exp(. - maximum); the scores go to
  // the workspace (16-byte pieces: chunk starts are multiples of 32 positions).
  const int n = p1 - p0;
  for (int r = warp; r < a.rows; r += kWarps) {
    const __nv_bfloat16* row = sc + r * L.scw;
    float m = -INFINITY;
    for (int q = lane; q < n; q += 32) m = fmaxf(m, __fmul_rn(__bfloat162float(row[q]), scale));
    m = warp_max(m);
    float s = 0.f;
    for (int q = lane; q < n; q += 32) s += expf(__fsub_rn(__fmul_rn(__bfloat162float(row[q]), scale), m));
    s = warp_sum(s);
    if (lane == 0) {
      stats[r * 2] = n > 0 ? m : -INFINITY;
      stats[r * 2 + 1] = n > 0 ? s : 0.f;
    }
    __nv_bfloat16* dst = a.scores + (static_cast<int64_t>(p.pair) * a.rows + r) * a.seq_pad + p0;
    for (int q = lane * 8; q < n; q += 32 * 8) {
      if (q + 8 <= n) *reinterpret_cast<uint4*>(dst + q) = *reinterpret_cast<const uint4*>(row + q);
      else
        for (int e = q; e < n; ++e) dst[e] = row[e];
    }
  }
}

// ---- launch 2: weights of the chunk times its values ---------------------------------------------
template <int HD, int MT, bool FP8>
__global__ void __launch_bounds__(kThreads, 1) split_values_kernel(const __grid_constant__ CUtensorMap tmap_v, SplitArgs a) {
  using T = Geom<HD>;
  constexpr int NT2 = HD / 8 / kWarps;  // 8-dim output tiles per warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout<HD, FP8> L(a.rows, a.tokens, a.chunk, a.rot, MT * 16);
  uint8_t* ring = smem + L.ring;
  uint8_t* work = smem + L.work;
  __nv_bfloat16* wt = reinterpret_cast<__nv_bfloat16*>(smem + L.sc);
  float* rs = reinterpret_cast<float*>(smem + L.qf);  // [rows][2]: the row's maximum and sum
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + kStages;

  pdl_wait();
  pdl_trigger();
  const Pair p = pair_of(a, blockIdx.y, blockIdx.z);
  const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int p0 = c * a.chunk, p1 = min(p0 + a.chunk, p.n_read);
  if (p0 >= p1) return;
  const int live = (p.n_read + a.chunk - 1) / a.chunk;
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t row0 = static_cast<int64_t>(p.pair) * a.max_seq;
  if (warp == kWarps) {
    if (lane == 0) copy_tiles<HD, FP8>(&tmap_v, a.v_cache, row0, p0, p1, ring, full, empty);
    return;
  }
  for (int r = warp; r < a.rows; r += kWarps) {
    float m, s;
    row_stats(a, p.pair, r, live, scale, lane, m, s);
    if (lane == 0) {
      rs[2 * r] = m;
      rs[2 * r + 1] = s;
    }
  }
  compute_bar();
  // bf16 weights of the chunk's positions; rows past `rows` and positions past p1 are zero.
  const int n = p1 - p0, ntiles = (n + KT - 1) / KT;
  for (int i = tid; i < MT * 16 * ntiles * KT; i += kWarps * 32) {
    const int r = i / (ntiles * KT), q = i % (ntiles * KT);
    float w = 0.f;
    if (r < a.rows && q < n) {
      const float sv = __bfloat162float(a.scores[(static_cast<int64_t>(p.pair) * a.rows + r) * a.seq_pad + p0 + q]);
      w = __fdiv_rn(expf(__fsub_rn(__fmul_rn(sv, scale), rs[2 * r])), rs[2 * r + 1]);
    }
    wt[r * L.scw + q] = __float2bfloat16_rn(w);
  }
  compute_bar();

  float acc[MT][NT2][4] = {};
  const int c0 = warp * NT2;  // this warp's first 8-dim chunk
  for (int i = 0; i < ntiles; ++i) {
    const int valid = min(KT, n - i * KT);
    uint32_t tile = tile_for<HD, FP8>(ring, work, full, empty, i, valid, a.v_scale, tid, lane);
    if constexpr (!FP8) {
      if (valid < KT) {
        // Positions past the row's visible cache (zero weight) must not bring non-finite values into 0 x V.
        uint8_t* tp = ring + (i % kStages) * T::kTileBytes;
        for (int e = lane; e < (KT - valid) * NT2; e += 32)
          *reinterpret_cast<uint4*>(tp + T::at(valid + e / NT2, c0 + e % NT2)) = make_uint4(0u, 0u, 0u, 0u);
        fence_proxy_async_shared();  // ordered before the slot's next tensor copy
        __syncwarp();
      }
    }
#pragma unroll
    for (int ks = 0; ks < KT / 16; ++ks) {
      const int vr = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t wa[4];
        ldsm_x4(smem_u32(wt + (mt * 16 + (lane & 15)) * L.scw + i * KT + ks * 16 + (lane >> 4) * 8), wa[0], wa[1], wa[2],
                wa[3]);
#pragma unroll
        for (int nn = 0; nn < NT2; nn += 2) {
          uint32_t b0, b1, b2, b3;
          if constexpr (NT2 >= 2) {
            ldsm_x4_t(tile + T::at(vr, c0 + nn + (lane >> 4)), b0, b1, b2, b3);
            mma_bf16_16816(acc[mt][nn], wa, b0, b1);
            mma_bf16_16816(acc[mt][nn + 1], wa, b2, b3);
          } else {
            ldsm_x2_t(tile + T::at(vr, c0 + nn), b0, b1);
            mma_bf16_16816(acc[mt][nn], wa, b0, b1);
          }
        }
      }
    }
    if constexpr (!FP8) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[i % kStages]);
    }
  }
  float* part = a.part + ((static_cast<int64_t>(p.pair) * a.nchunks + c) * a.rows) * HD;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int qr = mt * 16 + (lane >> 2) + hh * 8;
      if (qr >= a.rows) continue;
#pragma unroll
      for (int nn = 0; nn < NT2; ++nn) {
        const int d = (c0 + nn) * 8 + 2 * (lane & 3);
        *reinterpret_cast<float2*>(part + qr * HD + d) = make_float2(acc[mt][nn][2 * hh], acc[mt][nn][2 * hh + 1]);
      }
    }
}

// ---- launch 3: the output rows and the cache writes ----------------------------------------------
// One CTA of kFinishThreads per (row, KV head, slice of the rows x HD outputs): the softmax statistics
// and the step's own keys and values are recomputed by every slice (a few hundred values), the
// chunks' partial sums are read for the slice's outputs only, eight chunks' loads in flight at a time
// and added in chunk order; slice 0 writes the step's keys and values into the cache.
template <int HD, bool FP8>
__global__ void __launch_bounds__(kFinishThreads) split_finish_kernel(SplitArgs a) {
  extern __shared__ uint8_t smem_raw[];
  float* rs = reinterpret_cast<float*>(smem_raw);   // [rows][2]
  float* wown = rs + 2 * kMaxRows;                  // [rows][tokens] own weights (bf16 values)
  float* kown = wown + kMaxRows * kMaxTokens;       // [tokens][HD] own keys (as the cache holds them)
  float* vown = kown + kMaxTokens * HD;             // [tokens][HD] own values
  __nv_bfloat16* prm = reinterpret_cast<__nv_bfloat16*>(vown + kMaxTokens * HD);  // norm weights, cos, sin

  pdl_wait();
  pdl_trigger();
  const Pair p = pair_of(a, blockIdx.x, blockIdx.y);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NT = kFinishThreads, NW = kFinishThreads / 32;
  const int K = a.tokens, G = a.groups, rot = a.rot > 0 ? a.rot : 1;
  const int live = (p.n_read + a.chunk - 1) / a.chunk;
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));
  for (int r = warp; r < a.rows; r += NW) {
    float m, s;
    row_stats(a, p.pair, r, live, scale, lane, m, s);
    if (lane < K) {
      const float o = a.own[(static_cast<int64_t>(p.pair) * a.rows + r) * K + lane];
      wown[r * kMaxTokens + lane] = o > -INFINITY ? bf16r(__fdiv_rn(expf(__fsub_rn(__fmul_rn(o, scale), m)), s)) : 0.f;
    }
  }
  // Own keys (normed, rotated, as the cache holds them) and values.
  __nv_bfloat16* wk = prm;
  __nv_bfloat16* cs = wk + HD;
  __nv_bfloat16* sn = cs + K * rot;
  for (int i = tid; i < HD; i += NT) wk[i] = a.k_norm_w[i];
  for (int i = tid; i < K * a.rot; i += NT) {
    const int t = i / a.rot, d = i % a.rot;
    cs[t * rot + d] = a.cos[(static_cast<int64_t>(p.b) * K + t) * a.rot + d];
    sn[t * rot + d] = a.sin[(static_cast<int64_t>(p.b) * K + t) * a.rot + d];
  }
  for (int i = tid; i < K * HD; i += NT) {
    const int t = i / HD, d = i % HD;
    const __nv_bfloat16* row = a.qkv + (static_cast<int64_t>(p.b) * K + t) * a.ld_qkv +
                               static_cast<int64_t>(a.num_q_heads) * 2 * HD + static_cast<int64_t>(p.g) * HD + d;
    kown[i] = __bfloat162float(row[0]);
    const float v = __bfloat162float(row[static_cast<int64_t>(a.num_kv_heads) * HD]);
    vown[i] = FP8 ? fp8_load(fp8_store(v, a.v_scale), a.v_scale) : v;
  }
  __syncthreads();
  for (int t = warp; t < K; t += NW) norm_rope_head<HD>(kown + t * HD, wk, cs + t * rot, sn + t * rot, a.rot, a.eps, lane);
  __syncthreads();

  // out = bf16(bf16(sum over chunks of W V) + bf16(W_own V_own)) * bf16(sigmoid(gate)), to e5m2.
  const float* part = a.part + (static_cast<int64_t>(p.pair) * a.nchunks) * a.rows * HD;
  const int64_t cstride = static_cast<int64_t>(a.rows) * HD;
  const int n_out = a.rows * HD;
  const int lo = static_cast<int>(static_cast<int64_t>(blockIdx.z) * n_out / gridDim.z);
  const int hi = static_cast<int>(static_cast<int64_t>(blockIdx.z + 1) * n_out / gridDim.z);
  for (int i = lo + tid; i < hi; i += NT) {
    const int r = i / HD, d = i % HD, t = r / G, h = r % G;
    float cache_part = 0.f;
    int c = 0;
    for (; c + 8 <= live; c += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = part[(c + u) * cstride + i];
#pragma unroll
      for (int u = 0; u < 8; ++u) cache_part += v[u];
    }
    for (; c < live; ++c) cache_part += part[c * cstride + i];
    float own_part = 0.f;
    for (int t2 = 0; t2 < K; ++t2) own_part = __fmaf_rn(wown[r * kMaxTokens + t2], vown[t2 * HD + d], own_part);
    const float o = bf16r(__fadd_rn(bf16r(cache_part), bf16r(own_part)));
    const int64_t qrow = static_cast<int64_t>(p.b) * K + t;
    const int qh = p.g * G + h;
    const float gv = __bfloat162float(a.qkv[qrow * a.ld_qkv + static_cast<int64_t>(qh) * 2 * HD + HD + d]);
    a.out[qrow * a.ld_out + static_cast<int64_t>(qh) * HD + d] = f32_to_e5m2(bf16r(__fmul_rn(o, bf16r(sigmoidf_(gv)))));
  }
  // The step's keys and values into the cache: every read of it this step is in the earlier launches.
  if (blockIdx.z != 0) return;
  for (int i = tid; i < K * HD; i += NT) {
    const int t = i / HD, d = i % HD;
    const int64_t at = (static_cast<int64_t>(p.pair) * a.max_seq + write_position(a, p, t)) * HD + d;
    const float k = kown[i];
    const float v = __bfloat162float(a.qkv[(static_cast<int64_t>(p.b) * K + t) * a.ld_qkv +
                                           static_cast<int64_t>(a.num_q_heads) * 2 * HD +
                                           static_cast<int64_t>(a.num_kv_heads + p.g) * HD + d]);
    if constexpr (FP8) {
      a.k_cache[at] = fp8_store(k, a.k_scale);
      a.v_cache[at] = fp8_store(v, a.v_scale);
    } else {
      reinterpret_cast<__nv_bfloat16*>(a.k_cache)[at] = __float2bfloat16_rn(k);
      reinterpret_cast<__nv_bfloat16*>(a.v_cache)[at] = __float2bfloat16_rn(v);
    }
  }
}

// ---- host ----------------------------------------------------------------------------------------
struct Plan {
  int chunk, nchunks;
  int64_t seq_pad;
  size_t scores, stats, own, part, total;
};

// Chunks per (row, KV head): enough CTAs for about four per SM over all pairs, each chunk a multiple
// of 32 positions and at most kMaxChunk.
Plan plan_for(int64_t batch, int kv_heads, int rows, int tokens, int64_t max_seq, int hd) {
  Plan pl{};
  const int64_t pairs = batch * kv_heads;
  const int64_t tiles = (max_seq + KT - 1) / KT;
  int64_t want = (4 * 148 + pairs - 1) / pairs;
  want = want < 1 ? 1 : (want > tiles ? tiles : want);
  int64_t chunk = ((tiles + want - 1) / want) * KT;
  if (chunk > kMaxChunk) chunk = kMaxChunk;
  pl.chunk = static_cast<int>(chunk);
  pl.nchunks = static_cast<int>((max_seq + chunk - 1) / chunk);
  pl.seq_pad = (max_seq + 31) / 32 * 32;
  auto a256 = [](size_t x) { return (x + 255) & ~size_t(255); };
  pl.scores = a256(static_cast<size_t>(pairs) * rows * pl.seq_pad * 2);
  pl.stats = a256(static_cast<size_t>(pairs) * pl.nchunks * rows * 2 * 4);
  pl.own = a256(static_cast<size_t>(pairs) * rows * tokens * 4);
  pl.part = a256(static_cast<size_t>(pairs) * pl.nchunks * rows * hd * 4);
  pl.total = pl.scores + pl.stats + pl.own + pl.part;
  return pl;
}

template <int HD, int MT, bool FP8>
int launch_split(SplitArgs a, int64_t batch, cudaStream_t stream) {
  using T = Geom<HD>;
  const uint64_t cache_rows = static_cast<uint64_t>(batch) * a.num_kv_heads * a.max_seq;
  CUtensorMap tk{}, tv{};
  if (!FP8) {
    if (cache_rows + KT > (1ull << 31))
      return q38host::set_error("q38_attn_split: cache of %llu rows too large", (unsigned long long)cache_rows),
             Q38_ERR_UNSUPPORTED;
    int st = q38host::encode_tmap_2d(&tk, a.k_cache, cache_rows, HD, 2, KT, T::kBoxCols, T::kSwizzle);
    if (st == Q38_OK) st = q38host::encode_tmap_2d(&tv, a.v_cache, cache_rows, HD, 2, KT, T::kBoxCols, T::kSwizzle);
    if (st != Q38_OK) return st;
  }
  const size_t smem = Layout<HD, FP8>(a.rows, a.tokens, a.chunk, a.rot, MT * 16).total;
  cudaError_t e = cudaFuncSetAttribute(split_scores_kernel<HD, MT, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(split_values_kernel<HD, MT, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(attn_split)");
  const dim3 grid(static_cast<unsigned>(a.nchunks), static_cast<unsigned>(a.num_kv_heads), static_cast<unsigned>(batch));
  e = q38host::launch_pdl(split_scores_kernel<HD, MT, FP8>, grid, dim3(kThreads), smem, stream, tk, a);
  if (e == cudaSuccess) e = q38host::launch_pdl(split_values_kernel<HD, MT, FP8>, grid, dim3(kThreads), smem, stream, tv, a);
  const size_t fsmem = (2 * kMaxRows + kMaxRows * kMaxTokens + 2 * kMaxTokens * HD) * 4 +
                       (HD + 2 * kMaxTokens * (a.rot > 0 ? a.rot : 1)) * 2;
  if (e == cudaSuccess)
    e = q38host::launch_pdl(split_finish_kernel<HD, FP8>, dim3(a.num_kv_heads, static_cast<unsigned>(batch), kFinishSlices),
                            dim3(kFinishThreads), fsmem, stream, a);
  return q38host::cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "attn_split launch");
}

template <int HD>
int dispatch(const SplitArgs& a, int64_t batch, bool fp8, cudaStream_t s) {
  if (a.rows <= 16) return fp8 ? launch_split<HD, 1, true>(a, batch, s) : launch_split<HD, 1, false>(a, batch, s);
  return fp8 ? launch_split<HD, 2, true>(a, batch, s) : launch_split<HD, 2, false>(a, batch, s);
}

}  // namespace

extern "C" size_t q38_attn_split_workspace_bytes(int64_t batch, int num_q_heads, int num_kv_heads, int tokens,
                                                 int64_t max_seq, int head_dim) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || tokens <= 0 || max_seq <= 0 || head_dim <= 0 ||
      num_q_heads % num_kv_heads)
    return 0;
  return plan_for(batch, num_kv_heads, num_q_heads / num_kv_heads * tokens, tokens, max_seq, head_dim).total;
}

extern "C" int q38_attn_split(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w,
                              const void* cos, const void* sin, void* k_cache, void* v_cache, int kv_format,
                              float k_scale, float v_scale, int64_t max_seq, const int32_t* position,
                              const float* active, void* out, int64_t ld_out, int64_t batch, int tokens,
                              int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps, void* workspace,
                              size_t workspace_bytes, q38_stream_t stream) {
  using namespace q38host;
  if (!qkv || !q_norm_w || !k_norm_w || !cos || !sin || !k_cache || !v_cache || !position || !active || !out ||
      !workspace)
    return set_error("q38_attn_split: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads ||
      tokens < 1 || tokens > kMaxTokens || num_q_heads / num_kv_heads * tokens > kMaxRows || max_seq < tokens ||
      max_seq > (1 << 24) || rot_dim < 0 || rot_dim > head_dim || rot_dim % 2)
    return set_error("q38_attn_split: bad sizes (groups x tokens <= %d, tokens <= %d)", kMaxRows, kMaxTokens), Q38_ERR_ARG;
  if (kv_format != Q38_KV_BF16 && kv_format != Q38_KV_E4M3)
    return set_error("q38_attn_split: unknown cache format %d", kv_format), Q38_ERR_ARG;
  const bool fp8 = kv_format == Q38_KV_E4M3;
  if (fp8 && !(k_scale > 0.f && v_scale > 0.f && std::isfinite(k_scale) && std::isfinite(v_scale)))
    return set_error("q38_attn_split: FP8 cache scales must be positive"), Q38_ERR_ARG;
  if (ld_qkv < static_cast<int64_t>(2 * num_q_heads + 2 * num_kv_heads) * head_dim ||
      ld_out < static_cast<int64_t>(num_q_heads) * head_dim)
    return set_error("q38_attn_split: leading dimension too small"), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
       reinterpret_cast<uintptr_t>(workspace)) & 15u)
    return set_error("q38_attn_split: caches and workspace must be 16-byte aligned"), Q38_ERR_ARG;
  const int rows = num_q_heads / num_kv_heads * tokens;
  const Plan pl = plan_for(batch, num_kv_heads, rows, tokens, max_seq, head_dim);
  if (workspace_bytes < pl.total)
    return set_error("q38_attn_split: workspace of %zu bytes, needs %zu", workspace_bytes, pl.total), Q38_ERR_ARG;
  SplitArgs a{};
  a.qkv = static_cast<const __nv_bfloat16*>(qkv);
  a.ld_qkv = ld_qkv;
  a.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  a.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.k_cache = static_cast<uint8_t*>(k_cache);
  a.v_cache = static_cast<uint8_t*>(v_cache);
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.max_seq = max_seq;
  a.position = position;
  a.active = active;
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.groups = num_q_heads / num_kv_heads;
  a.tokens = tokens;
  a.rows = rows;
  a.rot = rot_dim;
  a.eps = eps;
  a.chunk = pl.chunk;
  a.nchunks = pl.nchunks;
  a.seq_pad = pl.seq_pad;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.scores = reinterpret_cast<__nv_bfloat16*>(ws);
  a.stats = reinterpret_cast<float*>(ws + pl.scores);
  a.own = reinterpret_cast<float*>(ws + pl.scores + pl.stats);
  a.part = reinterpret_cast<float*>(ws + pl.scores + pl.stats + pl.own);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 256) return dispatch<256>(a, batch, fp8, s);
  if (head_dim == 32) return dispatch<32>(a, batch, fp8, s);
  return set_error("q38_attn_split: head_dim %d not built (256, 32 are)", head_dim), Q38_ERR_UNSUPPORTED;
}
