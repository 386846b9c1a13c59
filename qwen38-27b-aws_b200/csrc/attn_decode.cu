// Gated full attention, one decode token per row over a BF16 KV cache:
// FullAttentionStep._project + forward (qwen38_inf2/model.py:565-577, :610-639).
//
// One CTA per (row, KV head) with its G query heads. The reference computes the scores as a BF16
// matmul (fp32 sums rounded to bf16), a fp32 softmax over cache positions < position plus the
// token's own key, weights rounded to bf16 after normalisation, and the output as a BF16 matmul plus
// the own value's bf16 term. This kernel keeps those rounding points, so it takes two passes: scores
// for every visible position into shared memory (K streamed once), then the normalised weights
// against V (V streamed once).
//
// It is HBM-bound on the cache (position * head_dim * 4 bytes per (row, KV head)), so the CTA is
// built around the copy stream: a copy warp keeps a ring of tiles of 32 positions in flight (tensor
// copies of 64-dim boxes with 128-byte swizzle), K tiles then V tiles, handed over through full /
// empty mbarriers, so it runs ahead into V while the four compute warps finish the softmax; the
// compute warps multiply on mma.sync (BF16, fp32 accumulate) and never wait on a CTA-wide barrier per
// tile. Every other input of the row (queries, own key / value, gates, norm weights, cos / sin) is
// fetched in one round trip at the start. Four CTAs per SM (two tiles in flight each).
//
// Rows differ in length (each streams position * head_dim * 4 bytes per KV head), and a CTA streams
// at a fraction of the SM's bandwidth, so a long row that starts in the grid's last wave sets the
// kernel's end. With a row order (attn_row_order_kernel, once per step) the CTAs take the rows
// longest first; any order gives the same bytes.
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
  const int32_t* order;  // row for each blockIdx.y (a permutation), or null: blockIdx.y itself
  int num_q_heads, num_kv_heads, groups, rot;
  float eps;
};

constexpr int kComputeWarps = 4;
constexpr int kThreads = (kComputeWarps + 1) * 32;  // compute warps + one copy warp
constexpr int KT = 32;                               // cache positions per tile
constexpr int kStages = 2;                           // tiles in flight per CTA (four CTAs per SM)
constexpr int MROWS = 16;                            // the MMA's M: query heads, padded by a zero row

__host__ __device__ constexpr size_t al16(size_t x) { return (x + 15) & ~size_t(15); }

// K / V tile geometry: [KT positions][HD] bf16 as boxes of up to 64 dims (128-byte rows), written by
// the tensor copy with 128-byte swizzle (16-byte chunk c of row r stored at chunk c ^ (r % 8)), so
// ldmatrix reads of 8 rows at one chunk hit 8 distinct bank groups. Heads narrower than 64 dims
// (the test config) use one unswizzled box.
template <int HD>
struct TileGeom {
  static constexpr bool kSwizzle = HD >= 64;
  static constexpr int kBoxCols = kSwizzle ? 64 : HD;
  static constexpr int kBoxes = HD / kBoxCols;
  static constexpr int kBoxBytes = KT * kBoxCols * 2;
  static constexpr int kTileBytes = KT * HD * 2;
  // Byte offset of 16-byte chunk `c` (8 dims) of position row `r` within a tile.
  __device__ static __forceinline__ uint32_t at(int r, int c) {
    if constexpr (kSwizzle) {
      return static_cast<uint32_t>((c >> 3) * kBoxBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
    } else {
      return static_cast<uint32_t>(r * HD * 2 + c * 16);
    }
  }
};

// Shared memory of one CTA (byte offsets from a 1024-byte aligned base; the same arithmetic on host
// and device).
template <int HD, int STAGES>
struct DecLayout {
  int rowp;      // padded q row (bf16): ldmatrix rows land in distinct banks
  int wcols;     // score / weight row length (bf16)
  size_t ring;   // [STAGES] tiles        K tiles, then V tiles
  size_t q;      // [groups][rowp] bf16   queries after norm + rotary
  size_t sc;     // [groups][wcols] bf16  scores, then weights in place
  size_t qf;     // [groups][hd] fp32     query staging
  size_t kown;   // [hd] fp32             own key staging
  size_t prm;    // [4][hd] bf16          q / k norm weights, cos, sin
  size_t gate;   // [groups][hd] bf16     output gates
  size_t vown;   // [hd] bf16             own value
  size_t zero;   // 16 zero bytes: the MMA rows past the group
  size_t bars;   // full[STAGES], empty[STAGES]
  size_t stats;  // [kMaxGroups] fp32 own scores, then own weights
  size_t total;  // including the alignment slack of the base
  __host__ __device__ DecLayout(int groups, int64_t max_seq) {
    rowp = HD + 8;
    wcols = static_cast<int>((max_seq + KT - 1) / KT * KT) + 8;
    size_t off = 0;
    auto take = [&](size_t bytes) {
      const size_t at = off;
      off = al16(off + bytes);
      return at;
    };
    ring = take(static_cast<size_t>(STAGES) * TileGeom<HD>::kTileBytes);
    q = take(static_cast<size_t>(groups) * rowp * 2);
    sc = take(static_cast<size_t>(groups) * wcols * 2);
    qf = take(static_cast<size_t>(groups) * HD * 4);
    kown = take(static_cast<size_t>(HD) * 4);
    prm = take(static_cast<size_t>(4) * HD * 2);
    gate = take(static_cast<size_t>(groups) * HD * 2);
    vown = take(static_cast<size_t>(HD) * 2);
    zero = take(16);
    bars = take(2 * STAGES * 8);
    stats = take(kMaxGroups * 4);
    total = off + 1024;
  }
};

// Barrier among the compute warps only (the copy warp runs on its own).
__device__ __forceinline__ void compute_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32) : "memory");
}

template <int HD, int STAGES>
__global__ void __launch_bounds__(kThreads, 4) attn_decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                               const __grid_constant__ CUtensorMap tmap_v, AttnArgs a) {
  using T = TileGeom<HD>;
  constexpr int KSTEPS = HD / 16;                  // MMA k-steps over head_dim
  constexpr int NT2 = HD / 8 / kComputeWarps;      // pass-2 n-tiles (8 dims) per warp
  static_assert(KT == 8 * kComputeWarps, "one 8-position n-tile per compute warp in pass 1");
  static_assert(KSTEPS % 2 == 0 && NT2 >= 1, "head_dim");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int G = a.groups;
  const DecLayout<HD, STAGES> L(G, a.max_seq);
  const int ROWP = L.rowp, wcols = L.wcols;
  uint8_t* ring = smem + L.ring;
  __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(smem + L.q);
  __nv_bfloat16* sc = reinterpret_cast<__nv_bfloat16*>(smem + L.sc);
  float* qf = reinterpret_cast<float*>(smem + L.qf);
  float* kown = reinterpret_cast<float*>(smem + L.kown);
  __nv_bfloat16* wq = reinterpret_cast<__nv_bfloat16*>(smem + L.prm);
  __nv_bfloat16* wk = wq + HD;
  __nv_bfloat16* cs = wk + HD;
  __nv_bfloat16* sn = cs + HD;
  __nv_bfloat16* gates = reinterpret_cast<__nv_bfloat16*>(smem + L.gate);
  __nv_bfloat16* vown = reinterpret_cast<__nv_bfloat16*>(smem + L.vown);
  uint32_t* zero = reinterpret_cast<uint32_t*>(smem + L.zero);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + STAGES;
  float* stats = reinterpret_cast<float*>(smem + L.stats);

  pdl_wait();
  pdl_trigger();
  const int g = blockIdx.x, b = a.order ? a.order[blockIdx.y] : static_cast<int>(blockIdx.y);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t head_row = static_cast<int64_t>(b) * a.num_kv_heads + g;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kComputeWarps);
    }
    fence_mbar_init();
  }
  if (tid < 4) zero[tid] = 0u;
  const bool on = a.active[b] > 0.5f;
  const int pos = a.position[b];
  const int64_t pos64 = pos < 0 ? 0 : pos;
  const int n_read = on ? static_cast<int>(pos64 < a.max_seq ? pos64 : a.max_seq) : 0;
  const int64_t where = on ? (pos64 < a.max_seq - 1 ? pos64 : a.max_seq - 1) : a.max_seq - 1;
  const int ntiles = (n_read + KT - 1) / KT;
  __syncthreads();

  if (warp == kComputeWarps) {
    // Copy warp: K tiles 0 .. ntiles-1, then V tiles, each as T::kBoxes tensor copies of [KT rows x
    // box] at row head_row * max_seq + p0. Rows past n_read bring other positions' (finite) data or
    // zeros past the cache's end; the compute warps ignore or clear them.
    if (lane == 0) {
      prefetch_tmap(&tmap_k);
      prefetch_tmap(&tmap_v);
      const int y0 = static_cast<int>(head_row * a.max_seq);
      for (int i = 0; i < 2 * ntiles; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait(&empty[s], ((i / STAGES) - 1) & 1)) break;
        const bool is_v = i >= ntiles;
        const int p0 = (is_v ? i - ntiles : i) * KT;
        uint8_t* dst = ring + s * T::kTileBytes;
        mbar_arrive_expect_tx(&full[s], T::kTileBytes);
#pragma unroll
        for (int bx = 0; bx < T::kBoxes; ++bx)
          tma_load_2d(dst + bx * T::kBoxBytes, is_v ? &tmap_v : &tmap_k, &full[s], bx * T::kBoxCols, y0 + p0);
      }
    }
    return;
  }

  // ---- compute warps: every input of the row in one round trip (queries, own key and value, norm
  // weights, cos / sin, gates), then norm + rotary.
  // All loads are issued before any store (16-byte vectors into registers), so the staging costs one
  // round trip instead of one per loop iteration.
  constexpr int CT = kComputeWarps * 32;
  constexpr int HV = HD / 8;  // 16-byte vectors per head row
  static_assert(kMaxGroups * HV <= 2 * CT && 4 * HV <= CT, "staging covers a group in two vectors per thread");
  const __nv_bfloat16* row = a.qkv + b * a.ld_qkv;
  const int qh0 = g * G;
  const __nv_bfloat16* kraw = row + static_cast<int64_t>(a.num_q_heads) * 2 * HD + static_cast<int64_t>(g) * HD;
  const __nv_bfloat16* vraw = kraw + static_cast<int64_t>(a.num_kv_heads) * HD;
  {
    uint4 rq[2], rg[2], rp;
    __nv_bfloat16 rc[2], rs[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + k * CT;
      if (i < G * HV) {
        const uint4* src = reinterpret_cast<const uint4*>(row + static_cast<int64_t>(qh0 + i / HV) * 2 * HD);
        rq[k] = src[i % HV];
        rg[k] = src[HV + i % HV];
      }
      const int d = tid + k * CT;
      if (d < a.rot) {
        rc[k] = a.cos[b * a.rot + d];
        rs[k] = a.sin[b * a.rot + d];
      }
    }
    // Threads 0..4*HV-1: the own key, own value, q and k norm weights (one vector each).
    const int which = tid / HV, c = tid % HV;
    if (which < 4) {
      const __nv_bfloat16* src = which == 0 ? kraw : which == 1 ? vraw : which == 2 ? a.q_norm_w : a.k_norm_w;
      rp = reinterpret_cast<const uint4*>(src)[c];
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + k * CT;
      if (i < G * HV) {
        const __nv_bfloat16* qv = reinterpret_cast<const __nv_bfloat16*>(&rq[k]);
#pragma unroll
        for (int e = 0; e < 8; ++e) qf[i * 8 + e] = __bfloat162float(qv[e]);
        reinterpret_cast<uint4*>(gates)[i] = rg[k];
      }
      const int d = tid + k * CT;
      if (d < a.rot) {
        cs[d] = rc[k];
        sn[d] = rs[k];
      }
    }
    if (which == 0) {
      const __nv_bfloat16* kv = reinterpret_cast<const __nv_bfloat16*>(&rp);
#pragma unroll
      for (int e = 0; e < 8; ++e) kown[c * 8 + e] = __bfloat162float(kv[e]);
    } else if (which < 4) {
      reinterpret_cast<uint4*>(which == 1 ? vown : which == 2 ? wq : wk)[c] = rp;
    }
  }
  // Weights past n_read in the last tile are zero.
  for (int i = tid; i < G * KT; i += kComputeWarps * 32) {
    const int h = i / KT, p = n_read + i % KT;
    if (p < ntiles * KT) sc[h * wcols + p] = __float2bfloat16_rn(0.f);
  }
  compute_bar();
  for (int h = warp; h <= G; h += kComputeWarps) {
    if (h < G) norm_rope_head<HD>(qf + h * HD, wq, cs, sn, a.rot, a.eps, lane);
    else norm_rope_head<HD>(kown, wk, cs, sn, a.rot, a.eps, lane);
  }
  compute_bar();
  for (int i = tid; i < G * HD; i += kComputeWarps * 32) qs[(i / HD) * ROWP + i % HD] = __float2bfloat16_rn(qf[i]);
  // Own scores (fp32 dot, bf16-rounded like the reference's matmul output).
  for (int h = warp; h < G; h += kComputeWarps) {
    float d = 0.f;
    for (int e = lane; e < HD; e += 32) d += qf[h * HD + e] * kown[e];
    d = warp_sum(d);
    if (lane == 0) stats[h] = bf16r(d);
  }
  compute_bar();

  // Query fragments for every k-step (A rows past the group read the zero chunk).
  uint32_t qa[KSTEPS][4];
  {
    const int qr = lane & 15;
    const uint32_t base = qr < G ? smem_u32(qs + qr * ROWP + (lane >> 4) * 8) : smem_u32(zero);
    const uint32_t step = qr < G ? 32u : 0u;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) ldsm_x4(base + ks * step, qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }

  // ---- pass 1: S[16 x 8] per warp and K tile (this warp's 8 positions), bf16 into the score rows.
  // Two accumulators (even / odd k-step pairs) halve the dependent MMA chain.
  const int n0 = warp * 8;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % STAGES;
    mbar_wait(&full[s], (t / STAGES) & 1);
    const uint32_t tile = smem_u32(ring + s * T::kTileBytes);
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int r = n0 + (lane & 7);
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ks += 2) {
      uint32_t b0, b1, b2, b3;  // x4: k 0-7, 8-15 of k-step ks, then of ks + 1
      ldsm_x4(tile + T::at(r, 2 * ks + (lane >> 3)), b0, b1, b2, b3);
      mma_bf16_16816(acc[(ks >> 1) & 1], qa[ks], b0, b1);
      mma_bf16_16816(acc[(ks >> 1) & 1], qa[ks + 1], b2, b3);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // C fragment: rows lane/4 (+8) = heads, columns 2*(lane%4) + {0,1} = positions.
    const int h = lane >> 2, p = t * KT + n0 + 2 * (lane & 3);
    if (h < G) {
      if (p < n_read) sc[h * wcols + p] = __float2bfloat16_rn(__fadd_rn(acc[0][0], acc[1][0]));
      if (p + 1 < n_read) sc[h * wcols + p + 1] = __float2bfloat16_rn(__fadd_rn(acc[0][1], acc[1][1]));
    }
  }
  compute_bar();

  // ---- softmax of (score * head_dim^-0.5) per head over [cache, own]; weights bf16 in place.
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));  // head**-0.5 as fp32
  for (int h = warp; h < G; h += kComputeWarps) {
    __nv_bfloat16* w = sc + h * wcols;
    const float own = __fmul_rn(stats[h], scale);
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
    __syncwarp();
    if (lane == 0) stats[h] = bf16r(__fdiv_rn(eown, sum));  // now the own key's weight
  }
  compute_bar();

  // ---- pass 2: O[16 x this warp's dims] += W[16 x 32 positions] * V[32 x dims] per V tile.
  float acc2[NT2][4];
#pragma unroll
  for (int n = 0; n < NT2; ++n) acc2[n][0] = acc2[n][1] = acc2[n][2] = acc2[n][3] = 0.f;
  const int wr = lane & 15;
  const uint32_t wbase = wr < G ? smem_u32(sc + wr * wcols + (lane >> 4) * 8) : smem_u32(zero);
  const uint32_t wstep = wr < G ? 32u : 0u;  // bytes per 16 positions
  const int c0 = warp * NT2;                 // this warp's first 8-dim chunk
  for (int t = 0; t < ntiles; ++t) {
    const int i = ntiles + t, s = i % STAGES;
    mbar_wait(&full[s], (i / STAGES) & 1);
    uint8_t* tp = ring + s * T::kTileBytes;
    const uint32_t tile = smem_u32(tp);
    const int rows = min(KT, n_read - t * KT);
    if (rows < KT) {
      // Positions past n_read (zero weight) must not bring stale non-finite values into 0 x V.
      for (int e = lane; e < (KT - rows) * NT2; e += 32)
        *reinterpret_cast<uint4*>(tp + T::at(rows + e / NT2, c0 + e % NT2)) = make_uint4(0u, 0u, 0u, 0u);
      fence_proxy_async_shared();  // ordered before the slot's next tensor copy
      __syncwarp();
    }
#pragma unroll
    for (int ks = 0; ks < KT / 16; ++ks) {
      uint32_t wa[4];
      ldsm_x4(wbase + (t * (KT / 16) + ks) * wstep, wa[0], wa[1], wa[2], wa[3]);
      const int vr = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;  // x4.trans: (k 0-7 | 8-15) x (n 0-7 | 8-15)
#pragma unroll
      for (int n = 0; n < NT2; n += 2) {
        uint32_t b0, b1, b2, b3;
        if constexpr (NT2 >= 2) {
          ldsm_x4_t(tile + T::at(vr, c0 + n + (lane >> 4)), b0, b1, b2, b3);
          mma_bf16_16816(acc2[n], wa, b0, b1);
          mma_bf16_16816(acc2[n + 1], wa, b2, b3);
        } else {
          ldsm_x2_t(tile + T::at(vr, c0 + n), b0, b1);
          mma_bf16_16816(acc2[n], wa, b0, b1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // Final: bf16(bf16(W V) + bf16(w_own * v_own)) * bf16(sigmoid(gate)), to e5m2.
  uint8_t* orow = a.out + b * a.ld_out;
  const int h = lane >> 2;
  if (h < G) {
#pragma unroll
    for (int n = 0; n < NT2; ++n) {
      const int d = (c0 + n) * 8 + 2 * (lane & 3);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float o = bf16r(__fadd_rn(bf16r(acc2[n][e]), bf16r(__fmul_rn(stats[h], __bfloat162float(vown[d + e])))));
        const float gv = __bfloat162float(gates[h * HD + d + e]);
        orow[static_cast<int64_t>(qh0 + h) * HD + d + e] = f32_to_e5m2(bf16r(__fmul_rn(o, bf16r(sigmoidf_(gv)))));
      }
    }
  }
  // The token's key and value go to the cache at `where`: every read of this (row, KV head)'s cache
  // this step has completed above.
  __nv_bfloat16* kw = a.k_cache + (head_row * a.max_seq + where) * HD;
  __nv_bfloat16* vw = a.v_cache + (head_row * a.max_seq + where) * HD;
  for (int d = tid; d < HD; d += kComputeWarps * 32) {
    kw[d] = __float2bfloat16_rn(kown[d]);
    vw[d] = vown[d];
  }
}

// The longest-first row order for attn_decode_kernel: rows by decreasing count of visible cache tiles
// (KT positions; inactive rows see none), ties by row index. One CTA; each thread ranks its rows
// against all others, O(batch^2) comparisons (a few microseconds at 4096 rows).
constexpr int kOrderMaxRows = 4096;
__global__ void __launch_bounds__(1024) attn_row_order_kernel(const int32_t* position, const float* active,
                                                              int64_t max_seq, int batch, int32_t* order) {
  __shared__ int tiles[kOrderMaxRows];
  pdl_wait();
  pdl_trigger();
  for (int r = threadIdx.x; r < batch; r += blockDim.x) {
    const int64_t p = position[r] < 0 ? 0 : position[r];
    const int64_t n = active[r] > 0.5f ? (p < max_seq ? p : max_seq) : 0;
    tiles[r] = static_cast<int>((n + KT - 1) / KT);
  }
  __syncthreads();
  for (int r = threadIdx.x; r < batch; r += blockDim.x) {
    const int tr = tiles[r];
    int rank = 0;
    for (int j = 0; j < batch; ++j) {
      const int tj = tiles[j];
      rank += (tj > tr) || (tj == tr && j < r);
    }
    order[rank] = r;
  }
}

template <int HD>
int launch_attn(const AttnArgs& a, int64_t batch, cudaStream_t stream) {
  using T = TileGeom<HD>;
  const size_t smem = DecLayout<HD, kStages>(a.groups, a.max_seq).total;
  if (smem > 220 * 1024)
    return q38host::set_error("q38_attn_decode: max_seq %lld needs %zu bytes of shared memory", (long long)a.max_seq, smem),
           Q38_ERR_UNSUPPORTED;
  const uint64_t rows = static_cast<uint64_t>(batch) * a.num_kv_heads * a.max_seq;
  if (rows + KT > (1ull << 31))
    return q38host::set_error("q38_attn_decode: cache of %llu rows too large", (unsigned long long)rows), Q38_ERR_UNSUPPORTED;
  CUtensorMap tk, tv;
  int st = q38host::encode_tmap_2d(&tk, a.k_cache, rows, HD, 2, KT, T::kBoxCols, T::kSwizzle);
  if (st == Q38_OK) st = q38host::encode_tmap_2d(&tv, a.v_cache, rows, HD, 2, KT, T::kBoxCols, T::kSwizzle);
  if (st != Q38_OK) return st;
  cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<HD, kStages>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(attn_decode)");
  dim3 grid(static_cast<unsigned>(a.num_kv_heads), static_cast<unsigned>(batch));
  e = q38host::launch_pdl(attn_decode_kernel<HD, kStages>, grid, dim3(kThreads), smem, stream, tk, tv, a);
  return q38host::cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "attn_decode launch");
}

}  // namespace

extern "C" int q38_attn_decode(const void* qkv, int64_t ld_qkv, const void* q_norm_w, const void* k_norm_w,
                               const void* cos, const void* sin, void* k_cache, void* v_cache, int64_t max_seq,
                               const int32_t* position, const float* active, void* out, int64_t ld_out,
                               int64_t batch, int num_q_heads, int num_kv_heads, int head_dim, int rot_dim, float eps,
                               const int32_t* row_order, q38_stream_t stream) {
  using namespace q38host;
  if (!qkv || !q_norm_w || !k_norm_w || !cos || !sin || !k_cache || !v_cache || !position || !active || !out)
    return set_error("q38_attn_decode: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads ||
      num_q_heads / num_kv_heads > kMaxGroups || max_seq <= 0 || rot_dim < 0 || rot_dim > head_dim || rot_dim % 2)
    return set_error("q38_attn_decode: bad sizes"), Q38_ERR_ARG;
  if (ld_qkv < static_cast<int64_t>(2 * num_q_heads + 2 * num_kv_heads) * head_dim ||
      ld_out < static_cast<int64_t>(num_q_heads) * head_dim || ld_qkv % 8)
    return set_error("q38_attn_decode: leading dimension too small"), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(qkv) |
       reinterpret_cast<uintptr_t>(q_norm_w) | reinterpret_cast<uintptr_t>(k_norm_w)) & 15u)
    return set_error("q38_attn_decode: qkv, caches and norm weights must be 16-byte aligned"), Q38_ERR_ARG;
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
  a.order = row_order;
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

extern "C" int q38_attn_row_order(const int32_t* position, const float* active, int64_t max_seq, int64_t batch,
                                  int32_t* row_order, q38_stream_t stream) {
  using namespace q38host;
  if (!position || !active || !row_order) return set_error("q38_attn_row_order: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > kOrderMaxRows || max_seq <= 0)
    return set_error("q38_attn_row_order: batch must be 1..%d", kOrderMaxRows), Q38_ERR_ARG;
  const unsigned threads = static_cast<unsigned>(batch >= 1024 ? 1024 : (batch + 31) / 32 * 32);
  const cudaError_t e = launch_pdl(attn_row_order_kernel, dim3(1), dim3(threads), 0, static_cast<cudaStream_t>(stream),
                                   position, active, max_seq, static_cast<int>(batch), row_order);
  return cuda_status(e != cudaSuccess ? e : cudaGetLastError(), "attn_row_order launch");
}
