// Gated delta rule, K verify tokens per row with commit-on-accept: GatedDeltaNetStep.verify
// (qwen38_inf2/model.py:376-454) and the CPU form of _commit_and_read (model.py:262-271).
//
// One CTA per (row, key head), owning its R value heads' state tiles, conv channels and pending
// slices outright (the decode kernel's partition), R * 128 threads. In one pass:
//   1. commit: S' = bf16(S * e^{sum of the accepted tokens' log decays} * keep
//                         + sum_s (k_s e^{decays after s}) delta_s^T)   from the pending buffers the
//      last verify step kept (the closed form of applying those tokens one by one); the conv history
//      moves past the accepted tokens' inputs. A row with active 0 keeps both exactly.
//   2. the K new tokens: causal conv from that history, SiLU, L2 norms, gates; [k_t; q_t]^T S' for each
//      token, then the K x K chunk: delta_t = beta_t (v_t - e^{c_t} k_t^T S' - sum_{s<t} e^{c_t - c_s}
//      (k_t.k_s) delta_s), o_t = e^{c_t} q_t^T S' + sum_{s<=t} e^{c_t - c_s} (q_t.k_s) delta_s, with c
//      the running sum of log decays. S' itself is stored; the new tokens' k, delta, log decay and conv
//      inputs become the pending buffers for the next step to commit.
//   3. the gated RMS norm times SiLU(z), e5m2 for out_proj.
// Rounding follows the reference's CPU branch: the conv as decode (fp32 sum of bf16 products, one
// rounding), the committed state rounded to bf16 before it is read, fp32 elsewhere.
#include "gdn_common.cuh"

namespace {

using namespace q38;

constexpr int KCONV = 4;
constexpr int KMAX = 4;  // verify tokens per row built (the reference drafts K = 4)

struct VerifyArgs {
  const __nv_bfloat16* qkvz;  // [batch * K, ld_qkvz]: row b * K + t
  int64_t ld_qkvz;
  const __nv_bfloat16* ab;  // [batch * K, ld_ab]
  int64_t ld_ab;
  __nv_bfloat16* conv_state;  // [rows, conv_dim, KCONV - 1]
  const __nv_bfloat16* conv_w;
  const __nv_bfloat16* a_log;
  const __nv_bfloat16* dt_bias;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* state;  // [rows, num_v_heads, DK, DV]
  float* pending_key;    // [batch, K, num_v_heads, DK]
  float* pending_delta;  // [batch, K, num_v_heads, DV]
  float* pending_decay;  // [batch, K, num_v_heads]
  __nv_bfloat16* pending_input;  // [batch, K, conv_dim]
  const int32_t* position;
  const float* active;
  const int32_t* accepted;
  uint8_t* out;  // [batch * K, ld_out]
  int64_t ld_out;
  int num_k_heads, num_v_heads, K;
  float eps;
};

template <int DK, int DV, int R>
struct VerifySmem {
  static constexpr int CH = 2 * DK + R * DV;
  static constexpr size_t STATE = static_cast<size_t>(R) * DK * DV * 2;
  static constexpr size_t XS = STATE;                                          // [KMAX][CH] conv + SiLU
  static constexpr size_t QN = XS + sizeof(float) * KMAX * CH;                 // [KMAX][DK]
  static constexpr size_t KN = QN + sizeof(float) * KMAX * DK;                 // [KMAX][DK]
  static constexpr size_t WK = KN + sizeof(float) * KMAX * DK;                 // [R][KMAX][DK] weighted pending keys
  static constexpr size_t DL = WK + sizeof(float) * R * KMAX * DK;             // [R][KMAX][DV] pending deltas
  static constexpr size_t RED = DL + sizeof(float) * R * KMAX * DV;            // [R][4][2 KMAX][DV]
  static constexpr size_t OB = RED + sizeof(float) * R * 4 * 2 * KMAX * DV;    // [R][KMAX][DV] outputs
  static constexpr size_t DOT = OB + sizeof(float) * R * KMAX * DV;            // [2][KMAX][KMAX] k.k, q.k
  static constexpr size_t GT = DOT + sizeof(float) * 2 * KMAX * KMAX;          // [R][KMAX][2] beta, log decay
  static constexpr size_t SC = GT + sizeof(float) * R * KMAX * 2;              // [R] commit scale
  static constexpr size_t BAR = (SC + sizeof(float) * R + 7) & ~size_t(7);     // [R] mbarriers, then [R] flags
  static constexpr size_t TOTAL = BAR + 8 * R + 4 * R + 16;
};

template <int DK, int DV, int R>
__global__ void __launch_bounds__(R * 128) gdn_verify_kernel(VerifyArgs a) {
  using S = VerifySmem<DK, DV, R>;
  constexpr int ROWS_W = DK / 4;  // state rows per warp of a value-head group
  constexpr int CPL = DV / 32;    // state columns per lane
  constexpr uint32_t TILE_BYTES = DK * DV * 2;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* st = reinterpret_cast<__nv_bfloat16*>(smem);
  float* xs = reinterpret_cast<float*>(smem + S::XS);
  float* qn = reinterpret_cast<float*>(smem + S::QN);
  float* kn = reinterpret_cast<float*>(smem + S::KN);
  float* wk = reinterpret_cast<float*>(smem + S::WK);
  float* dl = reinterpret_cast<float*>(smem + S::DL);
  float* red = reinterpret_cast<float*>(smem + S::RED);
  float* ob = reinterpret_cast<float*>(smem + S::OB);
  float* dots = reinterpret_cast<float*>(smem + S::DOT);
  float* gt = reinterpret_cast<float*>(smem + S::GT);
  float* scl = reinterpret_cast<float*>(smem + S::SC);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::BAR);
  volatile int* failed = reinterpret_cast<volatile int*>(bars + R);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kh = blockIdx.x, b = blockIdx.y;
  const int K = a.K;
  const int pos = a.position[b];
  const bool on = a.active[b] > 0.5f;
  const float act = a.active[b];
  const float keep = (pos == 0 && on) ? 0.0f : 1.0f;
  int acc = a.accepted[b];
  acc = acc < 0 ? 0 : (acc > K ? K : acc);
  const int key_dim = a.num_k_heads * DK;
  const int conv_dim = 2 * key_dim + a.num_v_heads * DV;
  const int h0 = kh * R;

  if (tid == 0) {
    for (int j = 0; j < R; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    for (int j = 0; j < R; ++j) {
      mbar_arrive_expect_tx(&bars[j], TILE_BYTES);
      bulk_load(st + static_cast<size_t>(j) * DK * DV,
                a.state + (static_cast<int64_t>(b) * a.num_v_heads + h0 + j) * DK * DV, TILE_BYTES, &bars[j]);
    }
  }

  // Commit factors and the pending slices of this CTA's heads (read before this step overwrites them).
  if (tid < R) {
    const int h = h0 + tid;
    float d[KMAX];
    float total = 0.f;
#pragma unroll
    for (int s = 0; s < KMAX; ++s) {
      d[s] = s < K ? __fmul_rn(a.pending_decay[(static_cast<int64_t>(b) * K + s) * a.num_v_heads + h], s < acc ? 1.f : 0.f)
                   : 0.f;
      if (s < K) total = __fadd_rn(total, d[s]);
    }
    scl[tid] = on ? __fmul_rn(expf(total), keep) : 1.0f;
    float rem = total;
#pragma unroll
    for (int s = 0; s < KMAX; ++s) {
      if (s >= K) break;
      rem = __fsub_rn(rem, d[s]);
      const float f = __fmul_rn(__fmul_rn(__fmul_rn(expf(rem), s < acc ? 1.f : 0.f), keep), on ? 1.f : 0.f);
      gt[(tid * KMAX + s) * 2] = f;  // weight of pending token s (reuses the gate slot until the gates below)
    }
  }
  __syncthreads();
  for (int i = tid; i < R * K * (DK + DV); i += blockDim.x) {
    const int j = i / (K * (DK + DV)), rest = i % (K * (DK + DV));
    const int s = rest / (DK + DV), e = rest % (DK + DV);
    const int64_t base = (static_cast<int64_t>(b) * K + s) * a.num_v_heads + h0 + j;
    if (e < DK) wk[(j * KMAX + s) * DK + e] = __fmul_rn(a.pending_key[base * DK + e], gt[(j * KMAX + s) * 2]);
    else dl[(j * KMAX + s) * DV + (e - DK)] = a.pending_delta[base * DV + (e - DK)];
  }

  // Conv: history = the KCONV - 1 inputs before the first uncommitted token (times keep), then the K tokens.
  for (int i = tid; i < S::CH; i += blockDim.x) {
    int c;
    if (i < DK) c = kh * DK + i;
    else if (i < 2 * DK) c = key_dim + kh * DK + (i - DK);
    else c = 2 * key_dim + h0 * DV + (i - 2 * DK);
    __nv_bfloat16* cs = a.conv_state + (static_cast<int64_t>(b) * conv_dim + c) * (KCONV - 1);
    float win[KCONV - 1 + KMAX];
#pragma unroll
    for (int j = 0; j < KCONV - 1; ++j) win[j] = __bfloat162float(cs[j]);
    for (int s = 0; s < K; ++s) win[KCONV - 1 + s] = __bfloat162float(a.pending_input[(static_cast<int64_t>(b) * K + s) * conv_dim + c]);
    float hist[KCONV - 1];
#pragma unroll
    for (int j = 0; j < KCONV - 1; ++j) hist[j] = on ? __fmul_rn(win[acc + j], keep) : win[j];
    float cw[KCONV];
#pragma unroll
    for (int j = 0; j < KCONV; ++j) cw[j] = __bfloat162float(a.conv_w[static_cast<int64_t>(c) * KCONV + j]);
    float w2[KCONV - 1 + KMAX];
#pragma unroll
    for (int j = 0; j < KCONV - 1; ++j) w2[j] = hist[j];
    for (int t = 0; t < K; ++t) {
      const __nv_bfloat16 xin = a.qkvz[(static_cast<int64_t>(b) * K + t) * a.ld_qkvz + c];
      w2[KCONV - 1 + t] = __bfloat162float(xin);
      a.pending_input[(static_cast<int64_t>(b) * K + t) * conv_dim + c] = xin;
    }
    for (int t = 0; t < K; ++t) {
      float sacc = 0.f;
#pragma unroll
      for (int j = 0; j < KCONV; ++j) sacc = __fadd_rn(sacc, bf16r(__fmul_rn(w2[t + j], cw[j])));
      const float conv = bf16r(sacc);
      xs[t * S::CH + i] = bf16r(__fmul_rn(conv, bf16r(sigmoidf_(conv))));
    }
    if (on) {
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) cs[j] = __float2bfloat16_rn(hist[j]);
    }
  }
  __syncthreads();
  // Gates per (value head, token).
  if (tid < R * K) {
    const int j = tid / K, t = tid % K, h = h0 + j;
    const int64_t r = static_cast<int64_t>(b) * K + t;
    const float braw = __bfloat162float(a.ab[r * a.ld_ab + h]);
    const float araw = __bfloat162float(a.ab[r * a.ld_ab + a.num_v_heads + h]);
    gt[(j * KMAX + t) * 2 + 0] = __fmul_rn(bf16r(sigmoidf_(braw)), act);
    gt[(j * KMAX + t) * 2 + 1] = __fmul_rn(
        __fmul_rn(-expf(__bfloat162float(a.a_log[h])), softplusf_(__fadd_rn(araw, __bfloat162float(a.dt_bias[h])))), act);
  }
  // L2 norms of q (then / sqrt(dk)) and k per token.
  const float inv_scale = static_cast<float>(sqrt(static_cast<double>(DK)));
  for (int p = warp; p < 2 * K; p += blockDim.x / 32) {
    const int t = p >> 1, which = p & 1;
    const float* src = xs + t * S::CH + which * DK;
    float* dst = (which ? kn : qn) + t * DK;
    float ss = 0.f;
    for (int i = lane; i < DK; i += 32) ss = __fadd_rn(ss, __fmul_rn(src[i], src[i]));
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + 1e-6f);
    for (int i = lane; i < DK; i += 32) {
      const float v = __fmul_rn(src[i], r);
      dst[i] = which == 0 ? __fdiv_rn(v, inv_scale) : v;
    }
  }
  __syncthreads();
  // k_t . k_s (s < t) and q_t . k_s (s <= t).
  for (int p = warp; p < 2 * K * K; p += blockDim.x / 32) {
    const int which = p / (K * K), t = (p / K) % K, s = p % K;
    const float* x = (which ? qn : kn) + t * DK;
    const float* y = kn + s * DK;
    float d = 0.f;
    for (int i = lane; i < DK; i += 32) d = fmaf(x[i], y[i], d);
    d = warp_sum(d);
    if (lane == 0) dots[(which * KMAX + t) * KMAX + s] = d;
  }

  // Per value head group: commit, products, the chunk, pending, output.
  const int j = tid >> 7;
  const int gl = tid & 127;
  const int gw = gl >> 5;
  const int c0 = lane * CPL;
  const int h = h0 + j;
  __syncthreads();  // the dots and norms above are complete
  if (gl == 0) failed[j] = 0;
  group_bar(1 + j);
  if (!mbar_wait(&bars[j], 0)) failed[j] = 1;
  group_bar(1 + j);
  if (failed[j]) return;  // no block-wide barrier follows: each group leaves on its own
  __nv_bfloat16* tile = st + static_cast<size_t>(j) * DK * DV;
  const float scale = scl[j];
  float prod[2 * KMAX][CPL];
#pragma unroll
  for (int t = 0; t < 2 * KMAX; ++t)
#pragma unroll
    for (int e = 0; e < CPL; ++e) prod[t][e] = 0.f;
  for (int r = 0; r < ROWS_W; ++r) {
    const int i = gw * ROWS_W + r;
    float sv[CPL];
    load_row<CPL>(tile + i * DV + c0, sv);
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      float w = 0.f;
      for (int s = 0; s < K; ++s) w = fmaf(wk[(j * KMAX + s) * DK + i], dl[(j * KMAX + s) * DV + c0 + e], w);
      sv[e] = bf16r(__fadd_rn(__fmul_rn(sv[e], scale), w));
    }
    if (on) store_row<CPL>(tile + i * DV + c0, sv);
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      if (t >= K) break;
      const float kt = kn[t * DK + i], qt = qn[t * DK + i];
#pragma unroll
      for (int e = 0; e < CPL; ++e) {
        prod[t][e] = fmaf(kt, sv[e], prod[t][e]);
        prod[KMAX + t][e] = fmaf(qt, sv[e], prod[KMAX + t][e]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < KMAX; ++t) {
    if (t >= K) break;
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      red[((j * 4 + gw) * 2 * KMAX + t) * DV + c0 + e] = prod[t][e];
      red[((j * 4 + gw) * 2 * KMAX + KMAX + t) * DV + c0 + e] = prod[KMAX + t][e];
    }
  }
  fence_proxy_async_shared();  // the committed tile is visible to the bulk copy engine
  group_bar(1 + j);
  if (gl == 0 && on) {
    bulk_store(a.state + (static_cast<int64_t>(b) * a.num_v_heads + h) * DK * DV, tile, TILE_BYTES);
    bulk_commit();
  }
  // The K x K chunk, one state column per thread.
  if (gl < DV) {
    const int c = gl;
    float cum[KMAX], dlt[KMAX];
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      cum[t] = t == 0 ? gt[(j * KMAX) * 2 + 1] : __fadd_rn(cum[t - 1], gt[(j * KMAX + t) * 2 + 1]);
      dlt[t] = 0.f;
    }
#pragma unroll
    for (int t = 0; t < KMAX; ++t) {
      if (t >= K) break;
      float ks = 0.f, qs = 0.f;
      for (int w = 0; w < 4; ++w) {
        ks = __fadd_rn(ks, red[((j * 4 + w) * 2 * KMAX + t) * DV + c]);
        qs = __fadd_rn(qs, red[((j * 4 + w) * 2 * KMAX + KMAX + t) * DV + c]);
      }
      const float v = xs[t * S::CH + 2 * DK + j * DV + c];
      float d = __fsub_rn(v, __fmul_rn(expf(cum[t]), ks));
#pragma unroll
      for (int s = 0; s < t; ++s)
        d = __fsub_rn(d, __fmul_rn(__fmul_rn(expf(__fsub_rn(cum[t], cum[s])), dots[(0 * KMAX + t) * KMAX + s]), dlt[s]));
      dlt[t] = __fmul_rn(d, gt[(j * KMAX + t) * 2 + 0]);
      float o = __fmul_rn(expf(cum[t]), qs);
#pragma unroll
      for (int s = 0; s <= t; ++s)
        o = __fadd_rn(o, __fmul_rn(__fmul_rn(expf(__fsub_rn(cum[t], cum[s])), dots[(1 * KMAX + t) * KMAX + s]), dlt[s]));
      ob[(j * KMAX + t) * DV + c] = bf16r(o);
      a.pending_delta[((static_cast<int64_t>(b) * K + t) * a.num_v_heads + h) * DV + c] = dlt[t];
    }
  }
  for (int i = gl; i < K * DK; i += 128) {
    const int t = i / DK, e = i % DK;
    a.pending_key[((static_cast<int64_t>(b) * K + t) * a.num_v_heads + h) * DK + e] = kn[t * DK + e];
  }
  if (gl < K) a.pending_decay[(static_cast<int64_t>(b) * K + gl) * a.num_v_heads + h] = gt[(j * KMAX + gl) * 2 + 1];
  group_bar(1 + j);
  // Gated RMS norm of each token's output for this head, times SiLU(z); e5m2 out.
  for (int t = gw; t < K; t += 4) {
    float o[CPL];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      o[e] = ob[(j * KMAX + t) * DV + c0 + e];
      ss = __fadd_rn(ss, __fmul_rn(o[e], o[e]));
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(DV)), a.eps));
    const int64_t row = static_cast<int64_t>(b) * K + t;
    const __nv_bfloat16* zrow = a.qkvz + row * a.ld_qkvz + conv_dim + h * DV;
    uint8_t* orow = a.out + row * a.ld_out + h * DV;
#pragma unroll
    for (int e = 0; e < CPL; ++e) {
      const int c = c0 + e;
      const float n1 = bf16r(__fmul_rn(o[e], r));
      const float n2 = bf16r(__fmul_rn(__bfloat162float(a.norm_w[c]), n1));
      const float z = __bfloat162float(zrow[c]);
      orow[c] = f32_to_e5m2(bf16r(__fmul_rn(n2, __fmul_rn(z, sigmoidf_(z)))));
    }
  }
  if (gl == 0 && on) bulk_wait_read0();  // the tile must stay until the copy engine has read it
}

template <int DK, int DV, int R>
int launch_verify(const VerifyArgs& a, int64_t batch, cudaStream_t stream) {
  using S = VerifySmem<DK, DV, R>;
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gdn_verify_kernel<DK, DV, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(S::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(gdn_verify)");
    done_mask |= 1ull << dev;
  }
  dim3 grid(static_cast<unsigned>(a.num_k_heads), static_cast<unsigned>(batch));
  gdn_verify_kernel<DK, DV, R><<<grid, R * 128, S::TOTAL, stream>>>(a);
  return q38host::cuda_status(cudaGetLastError(), "gdn_verify launch");
}

}  // namespace

extern "C" int q38_gdn_verify_commit(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                                     const void* conv_weight, const void* a_log, const void* dt_bias,
                                     const void* norm_weight, void* state, void* pending_key, void* pending_delta,
                                     void* pending_decay, void* pending_input, const int32_t* position,
                                     const float* active, const int32_t* accepted, void* out, int64_t ld_out,
                                     int64_t batch, int tokens, int num_k_heads, int num_v_heads, int head_k,
                                     int head_v, int conv_kernel, float eps, q38_stream_t stream) {
  using namespace q38host;
  if (!qkvz || !ab || !conv_state || !conv_weight || !a_log || !dt_bias || !norm_weight || !state || !pending_key ||
      !pending_delta || !pending_decay || !pending_input || !position || !active || !accepted || !out)
    return set_error("q38_gdn_verify_commit: null pointer"), Q38_ERR_ARG;
  if (batch <= 0 || batch > 65535 || tokens < 1 || tokens > KMAX)
    return set_error("q38_gdn_verify_commit: batch %lld / %d tokens per row (1..%d built)", static_cast<long long>(batch),
                     tokens, KMAX),
           Q38_ERR_ARG;
  if (num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads)
    return set_error("q38_gdn_verify_commit: bad head counts"), Q38_ERR_ARG;
  if (conv_kernel != KCONV) return set_error("q38_gdn_verify_commit: conv kernel %d not built (4 is)", conv_kernel), Q38_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(state) & 15u) != 0)
    return set_error("q38_gdn_verify_commit: state must be 16-byte aligned"), Q38_ERR_ARG;
  const int64_t conv_dim = 2LL * num_k_heads * head_k + static_cast<int64_t>(num_v_heads) * head_v;
  if (ld_qkvz < conv_dim + static_cast<int64_t>(num_v_heads) * head_v || ld_ab < 2 * num_v_heads ||
      ld_out < static_cast<int64_t>(num_v_heads) * head_v)
    return set_error("q38_gdn_verify_commit: leading dimension too small"), Q38_ERR_ARG;
  VerifyArgs a{};
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
  a.pending_key = static_cast<float*>(pending_key);
  a.pending_delta = static_cast<float*>(pending_delta);
  a.pending_decay = static_cast<float*>(pending_decay);
  a.pending_input = static_cast<__nv_bfloat16*>(pending_input);
  a.position = position;
  a.active = active;
  a.accepted = accepted;
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_k_heads = num_k_heads;
  a.num_v_heads = num_v_heads;
  a.K = tokens;
  a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rep = num_v_heads / num_k_heads;
  if (head_k == 128 && head_v == 128 && rep == 3) return launch_verify<128, 128, 3>(a, batch, s);
  if (head_k == 32 && head_v == 32 && rep == 3) return launch_verify<32, 32, 3>(a, batch, s);
  return set_error("q38_gdn_verify_commit: head dims %d/%d with %d value heads per key head not built", head_k, head_v,
                   rep),
         Q38_ERR_UNSUPPORTED;
}
