// Gated delta rule over a prefill chunk of one row: GatedDeltaNetStep.prefill
// (qwen38_inf2/model.py:476-521) with the chunked rule of model.py:90-128.
//
// Three launches per call, all on the caller's stream:
//   prep   one CTA per (32-token tile, key head): the causal conv over [history * keep, chunk] with
//          the CPU branch's rounding (bf16 products summed left to right in bf16, model.py:513),
//          bf16 SiLU, fp32 L2 norms of q (then / sqrt(dk)) and k, and the gates beta, log decay
//          (masked to the valid tokens). q and k are written transposed, [key head][dk][tokens], so
//          the delta kernel's loads of a sub-chunk are contiguous runs of 256 bytes.
//   delta  one CTA per (value head, 32-column slice of the state). The state's value columns evolve
//          independently given k, beta and g, so the slices need no exchange; each CTA keeps its
//          [dk x 32] fp32 slice in shared memory across the chunk and walks it in sub-chunks of 64
//          tokens:   r  = beta * (v - e^g (k . S))            o_in = e^g (q . S)
//                    (I + N) vn = r,  N = strictly_lower(beta (k k^T) * decay)   (blocked solve)
//                    o  = o_in + ((q k^T) * decay) vn
//                    S  = e^{g_last} S + (k e^{g_last - g})^T vn
//          which is the reference's u - w S with u = A (v beta), w = A (k beta e^g), A = (I + N)^-1,
//          regrouped as A (beta (v - e^g k S)) (same values, fp32 sums in another order). The sub-chunk
//          length is 64 instead of the CPU branch's 128 (model.py:34): the rule is exact for any split.
//   norm   one CTA per token: the gated RMS norm of each value head (model.py:339-344), times SiLU(z),
//          e5m2 for out_proj; one more CTA carries the last conv_kernel-1 valid inputs into the conv
//          state (model.py:490-492) after the prep CTAs have read the old history.
#include "q38_common.cuh"

namespace {

using namespace q38;

constexpr int KCONV = 4;
constexpr int PREP_TOK = 32;  // tokens per prep CTA
constexpr int SUB = 64;       // tokens per sub-chunk of the delta rule
constexpr int SUBP = SUB + 4; // padded row of the transposed [dk][SUB] tiles (keeps float4 alignment)
constexpr int DVS = 32;       // state columns per delta CTA

struct PrefillArgs {
  const __nv_bfloat16* qkvz;  // [tokens, ld_qkvz]: q | k | v | z
  int64_t ld_qkvz;
  const __nv_bfloat16* ab;  // [tokens, ld_ab]: b | a
  int64_t ld_ab;
  __nv_bfloat16* conv_state;  // this slot's row [conv_dim][KCONV - 1]
  const __nv_bfloat16* conv_w;
  const __nv_bfloat16* a_log;
  const __nv_bfloat16* dt_bias;
  const __nv_bfloat16* norm_w;
  __nv_bfloat16* state;  // this slot's row [num_v_heads][dk][dv]
  int tokens, n_valid;
  float keep;  // 1 when start > 0, else the history and state are zero
  uint8_t* out;
  int64_t ld_out;
  int num_k_heads, num_v_heads;
  float eps;
  // workspace
  float* qT;    // [num_k_heads][dk][tokens]
  float* kT;    // [num_k_heads][dk][tokens]
  float* v;     // [num_v_heads][tokens][dv]
  float* beta;  // [num_v_heads][tokens]
  float* g;     // [num_v_heads][tokens]
  __nv_bfloat16* o;  // [tokens][num_v_heads * dv]
};

// ---------------------------------------------------------------------------------------------
// prep
// ---------------------------------------------------------------------------------------------
template <int DK, int DV, int R>
__global__ void __launch_bounds__(256) gdn_prefill_prep_kernel(PrefillArgs a) {
  constexpr int CH = 2 * DK + R * DV;
  extern __shared__ __align__(16) uint8_t smem[];
  float* xs = reinterpret_cast<float*>(smem);  // [CH][PREP_TOK + 1]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kh = blockIdx.y;
  const int t0 = blockIdx.x * PREP_TOK;
  const int key_dim = a.num_k_heads * DK;
  const int h0 = kh * R;

  for (int i = tid; i < CH; i += blockDim.x) {
    int c;
    if (i < DK) c = kh * DK + i;
    else if (i < 2 * DK) c = key_dim + kh * DK + (i - DK);
    else c = 2 * key_dim + h0 * DV + (i - 2 * DK);
    float w[KCONV];
#pragma unroll
    for (int j = 0; j < KCONV; ++j) w[j] = __bfloat162float(a.conv_w[static_cast<int64_t>(c) * KCONV + j]);
    // win[j] = input at token t - (KCONV - 1) + j; inputs before token 0 come from the history.
    float win[KCONV];
#pragma unroll
    for (int j = 0; j < KCONV - 1; ++j) {
      const int t = t0 - (KCONV - 1) + j;
      win[j] = t >= 0 ? __bfloat162float(a.qkvz[static_cast<int64_t>(t) * a.ld_qkvz + c])
                      : __bfloat162float(a.conv_state[static_cast<int64_t>(c) * (KCONV - 1) + (t + KCONV - 1)]) * a.keep;
    }
    for (int tt = 0; tt < PREP_TOK; ++tt) {
      const int t = t0 + tt;
      if (t >= a.tokens) {
        xs[i * (PREP_TOK + 1) + tt] = 0.f;
        continue;
      }
      win[KCONV - 1] = __bfloat162float(a.qkvz[static_cast<int64_t>(t) * a.ld_qkvz + c]);
      // Python's sum over the taps: each addition rounds to bf16.
      float s = bf16r(__fmul_rn(win[0], w[0]));
#pragma unroll
      for (int j = 1; j < KCONV; ++j) s = bf16r(__fadd_rn(s, bf16r(__fmul_rn(win[j], w[j]))));
      xs[i * (PREP_TOK + 1) + tt] = bf16r(__fmul_rn(s, bf16r(sigmoidf_(s))));
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) win[j] = win[j + 1];
    }
  }
  __syncthreads();
  // L2 norms per (token, q|k), in place.
  const float inv_scale = static_cast<float>(sqrt(static_cast<double>(DK)));  // math.sqrt(k_head) as fp32
  for (int p = warp; p < 2 * PREP_TOK; p += blockDim.x / 32) {
    const int tt = p >> 1, which = p & 1;
    float* col = xs + (which * DK) * (PREP_TOK + 1) + tt;
    float ss = 0.f;
    for (int d = lane; d < DK; d += 32) ss = __fadd_rn(ss, __fmul_rn(col[d * (PREP_TOK + 1)], col[d * (PREP_TOK + 1)]));
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss + 1e-6f);
    for (int d = lane; d < DK; d += 32) {
      const float v = __fmul_rn(col[d * (PREP_TOK + 1)], r);
      col[d * (PREP_TOK + 1)] = which == 0 ? __fdiv_rn(v, inv_scale) : v;
    }
  }
  __syncthreads();
  // q, k transposed: lane = token, so each row of 32 tokens is one 128-byte store.
  {
    const int t = t0 + lane;
    for (int d = warp; d < 2 * DK; d += blockDim.x / 32) {
      const int which = d >= DK, dd = d - which * DK;
      float* dst = (which ? a.kT : a.qT) + (static_cast<int64_t>(kh) * DK + dd) * a.tokens;
      if (t < a.tokens) dst[t] = xs[d * (PREP_TOK + 1) + lane];
    }
  }
  // v per value head, [head][token][dv].
  for (int idx = tid; idx < R * PREP_TOK * DV; idx += blockDim.x) {
    const int d = idx % DV, rest = idx / DV;
    const int tt = rest % PREP_TOK, j = rest / PREP_TOK;
    const int t = t0 + tt;
    if (t < a.tokens)
      a.v[(static_cast<int64_t>(h0 + j) * a.tokens + t) * DV + d] = xs[(2 * DK + j * DV + d) * (PREP_TOK + 1) + tt];
  }
  // Gates: beta = bf16(sigmoid(b)) * valid, g = -exp(A_log) * softplus(a + dt_bias) * valid.
  for (int idx = tid; idx < R * PREP_TOK; idx += blockDim.x) {
    const int j = idx / PREP_TOK, tt = idx % PREP_TOK;
    const int t = t0 + tt, h = h0 + j;
    if (t >= a.tokens) continue;
    const float valid = t < a.n_valid ? 1.0f : 0.0f;
    const float braw = __bfloat162float(a.ab[static_cast<int64_t>(t) * a.ld_ab + h]);
    const float araw = __bfloat162float(a.ab[static_cast<int64_t>(t) * a.ld_ab + a.num_v_heads + h]);
    a.beta[static_cast<int64_t>(h) * a.tokens + t] = __fmul_rn(bf16r(sigmoidf_(braw)), valid);
    a.g[static_cast<int64_t>(h) * a.tokens + t] =
        __fmul_rn(__fmul_rn(-expf(__bfloat162float(a.a_log[h])), softplusf_(__fadd_rn(araw, __bfloat162float(a.dt_bias[h])))),
                  valid);
  }
}

// ---------------------------------------------------------------------------------------------
// delta
// ---------------------------------------------------------------------------------------------
template <int DK>
struct DeltaSmem {
  static constexpr int KDP = DK + 4;
  static constexpr size_t QT = 0;                                  // [DK][SUBP]
  static constexpr size_t KT = QT + sizeof(float) * DK * SUBP;     // [DK][SUBP]
  static constexpr size_t KD = KT + sizeof(float) * DK * SUBP;     // [SUB][KDP] k_a[d] e^{g_last - g_a}
  static constexpr size_t ST = KD + sizeof(float) * SUB * KDP;     // [DK][DVS]
  static constexpr size_t VS = ST + sizeof(float) * DK * DVS;      // [SUB][DVS]
  static constexpr size_t RR = VS + sizeof(float) * SUB * DVS;     // [SUB][DVS] r
  static constexpr size_t OI = RR + sizeof(float) * SUB * DVS;     // [SUB][DVS] o_in
  static constexpr size_t VN = OI + sizeof(float) * SUB * DVS;     // [SUB][DVS]
  static constexpr size_t TB = VN + sizeof(float) * SUB * DVS;     // [16][DVS]
  static constexpr size_t AT = TB + sizeof(float) * 16 * DVS;      // [SUB][SUBP] (q k^T * decay)^T
  static constexpr size_t NT = AT + sizeof(float) * SUB * SUBP;    // [SUB][SUBP] N^T
  static constexpr size_t INV = NT + sizeof(float) * SUB * SUBP;   // [4][16][16]
  static constexpr size_t VEC = INV + sizeof(float) * 4 * 16 * 16; // gc, eg, beta, graw, wl [SUB] each
  static constexpr size_t TOTAL = VEC + sizeof(float) * 5 * SUB;
};

template <int DK, int DV>
__global__ void __launch_bounds__(256, 1) gdn_prefill_delta_kernel(PrefillArgs a) {
  using S = DeltaSmem<DK>;
  extern __shared__ __align__(16) uint8_t smem[];
  float* qT = reinterpret_cast<float*>(smem + S::QT);
  float* kT = reinterpret_cast<float*>(smem + S::KT);
  float* kd = reinterpret_cast<float*>(smem + S::KD);
  float* st = reinterpret_cast<float*>(smem + S::ST);
  float* vs = reinterpret_cast<float*>(smem + S::VS);
  float* rr = reinterpret_cast<float*>(smem + S::RR);
  float* oi = reinterpret_cast<float*>(smem + S::OI);
  float* vn = reinterpret_cast<float*>(smem + S::VN);
  float* tb = reinterpret_cast<float*>(smem + S::TB);
  float* atT = reinterpret_cast<float*>(smem + S::AT);
  float* nT = reinterpret_cast<float*>(smem + S::NT);
  float* inv = reinterpret_cast<float*>(smem + S::INV);
  float* gc = reinterpret_cast<float*>(smem + S::VEC);
  float* eg = gc + SUB;
  float* be = eg + SUB;
  float* graw = be + SUB;
  float* wl = graw + SUB;

  const int tid = threadIdx.x;
  const int h = blockIdx.x;
  const int c0 = blockIdx.y * DVS;  // first state column of this CTA
  const int R = a.num_v_heads / a.num_k_heads;
  const int kh = h / R;
  const int T = a.tokens;
  const int64_t vd_all = static_cast<int64_t>(a.num_v_heads) * DV;

  // The state slice, fp32, zero unless the row continues (start > 0).
  __nv_bfloat16* srow = a.state + static_cast<int64_t>(h) * DK * DV;
  for (int i = tid; i < DK * DVS; i += 256) {
    const int d = i / DVS, j = i % DVS;
    st[i] = __fmul_rn(__bfloat162float(srow[d * DV + c0 + j]), a.keep);
  }

  // Thread tilings (256 threads):
  //   C: the 64 x 64 products, 4 x 4 per thread.
  const int ai = tid >> 4, bi = tid & 15;
  //   D, F: [SUB][DVS], RPT rows x 4 columns per thread.
  constexpr int CG = DVS / 4, RG = 256 / CG, RPT = SUB / RG;
  const int ri = tid / CG, ci = tid % CG;
  //   G: [DK][DVS], DPT rows x 4 columns per thread.
  constexpr int DG = 256 / CG, DPT = DK / DG;
  static_assert(RPT >= 1 && DPT >= 1 && DK % DG == 0, "tiling");

  for (int s0 = 0; s0 < T; s0 += SUB) {
    const int n = min(SUB, T - s0);
    __syncthreads();  // the previous sub-chunk is done with every buffer
    for (int i = tid; i < DK * SUB; i += 256) {
      const int d = i / SUB, c = i % SUB;
      const int64_t src = (static_cast<int64_t>(kh) * DK + d) * T + s0 + c;
      qT[d * SUBP + c] = c < n ? a.qT[src] : 0.f;
      kT[d * SUBP + c] = c < n ? a.kT[src] : 0.f;
    }
    for (int i = tid; i < SUB * DVS; i += 256) {
      const int c = i / DVS, j = i % DVS;
      vs[i] = c < n ? a.v[(static_cast<int64_t>(h) * T + s0 + c) * DV + c0 + j] : 0.f;
    }
    if (tid < SUB) {
      be[tid] = tid < n ? a.beta[static_cast<int64_t>(h) * T + s0 + tid] : 0.f;
      graw[tid] = tid < n ? a.g[static_cast<int64_t>(h) * T + s0 + tid] : 0.f;
    }
    __syncthreads();
    if (tid == 0) {
      // Inclusive cumulative sum of the log decays (accumulated in double, rounded per element).
      double acc = 0.0;
      for (int c = 0; c < SUB; ++c) {
        acc += graw[c];
        gc[c] = static_cast<float>(acc);
      }
    }
    __syncthreads();
    if (tid < SUB) {
      eg[tid] = expf(gc[tid]);
      wl[tid] = expf(__fsub_rn(gc[SUB - 1], gc[tid]));
    }

    // C: attT[b][a] = (q_a . k_b) e^{g_a - g_b} for a >= b; nT[b][a] = beta_a (k_a . k_b) e^{g_a - g_b} for a > b.
    {
      float accq[4][4], acck[4][4];
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) accq[x][y] = acck[x][y] = 0.f;
#pragma unroll 4
      for (int d = 0; d < DK; ++d) {
        const float4 qa = *reinterpret_cast<const float4*>(qT + d * SUBP + 4 * ai);
        const float4 ka = *reinterpret_cast<const float4*>(kT + d * SUBP + 4 * ai);
        const float4 kb = *reinterpret_cast<const float4*>(kT + d * SUBP + 4 * bi);
        const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {ka.x, ka.y, ka.z, ka.w}, bv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
        for (int x = 0; x < 4; ++x)
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            accq[x][y] = fmaf(qv[x], bv[y], accq[x][y]);
            acck[x][y] = fmaf(kv[x], bv[y], acck[x][y]);
          }
      }
#pragma unroll
      for (int y = 0; y < 4; ++y) {
        const int b = 4 * bi + y;
        float at[4], nn[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int a_ = 4 * ai + x;
          const float dec = a_ >= b ? expf(__fsub_rn(gc[a_], gc[b])) : 0.f;
          at[x] = a_ >= b ? __fmul_rn(accq[x][y], dec) : 0.f;
          nn[x] = a_ > b ? __fmul_rn(__fmul_rn(be[a_], acck[x][y]), dec) : 0.f;
        }
        *reinterpret_cast<float4*>(atT + b * SUBP + 4 * ai) = make_float4(at[0], at[1], at[2], at[3]);
        *reinterpret_cast<float4*>(nT + b * SUBP + 4 * ai) = make_float4(nn[0], nn[1], nn[2], nn[3]);
      }
    }
    __syncthreads();  // eg, wl visible
    // D: r = beta (v - e^g (k . S)), o_in = e^g (q . S); and kd = k e^{g_last - g}.
    {
      float accr[RPT][4], acco[RPT][4];
#pragma unroll
      for (int x = 0; x < RPT; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) accr[x][y] = acco[x][y] = 0.f;
      const int a0 = ri * RPT;
#pragma unroll 4
      for (int d = 0; d < DK; ++d) {
        const float4 sv = *reinterpret_cast<const float4*>(st + d * DVS + 4 * ci);
        const float s4[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int x = 0; x < RPT; ++x) {
          const float kx = kT[d * SUBP + a0 + x], qx = qT[d * SUBP + a0 + x];
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            accr[x][y] = fmaf(kx, s4[y], accr[x][y]);
            acco[x][y] = fmaf(qx, s4[y], acco[x][y]);
          }
        }
      }
#pragma unroll
      for (int x = 0; x < RPT; ++x) {
        const int a_ = a0 + x;
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          const int j = 4 * ci + y;
          rr[a_ * DVS + j] = __fmul_rn(be[a_], __fsub_rn(vs[a_ * DVS + j], __fmul_rn(eg[a_], accr[x][y])));
          oi[a_ * DVS + j] = __fmul_rn(eg[a_], acco[x][y]);
        }
      }
      for (int i = tid; i < SUB * DK; i += 256) {
        const int a_ = i / DK, d = i % DK;
        kd[a_ * S::KDP + d] = __fmul_rn(kT[d * SUBP + a_], wl[a_]);
      }
    }
    // E0: inverses of the four 16 x 16 unit lower diagonal blocks of I + N (two warps, a column per lane).
    if (tid < 64) {
      const int blk = tid >> 4, c = tid & 15, base = blk * 16;
      float col[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float s = 0.f;
#pragma unroll
        for (int b = 0; b < r; ++b) s = fmaf(nT[(base + b) * SUBP + base + r], col[b], s);
        col[r] = r < c ? 0.f : (r == c ? 1.f : -s);
      }
#pragma unroll
      for (int r = 0; r < 16; ++r) inv[(blk * 16 + r) * 16 + c] = col[r];
    }
    __syncthreads();
    // E: (I + N) vn = r, block by block.
    {
      constexpr int JPT = DVS / 16;
      const int ar = tid >> 4, j0 = (tid & 15) * JPT;
      for (int blk = 0; blk < 4; ++blk) {
        const int a_ = blk * 16 + ar;
        float t[JPT];
#pragma unroll
        for (int y = 0; y < JPT; ++y) t[y] = rr[a_ * DVS + j0 + y];
        for (int b = 0; b < blk * 16; ++b) {
          const float nab = nT[b * SUBP + a_];
#pragma unroll
          for (int y = 0; y < JPT; ++y) t[y] = fmaf(-nab, vn[b * DVS + j0 + y], t[y]);
        }
#pragma unroll
        for (int y = 0; y < JPT; ++y) tb[ar * DVS + j0 + y] = t[y];
        __syncthreads();
        float v[JPT];
#pragma unroll
        for (int y = 0; y < JPT; ++y) v[y] = 0.f;
        for (int c = 0; c <= ar; ++c) {
          const float m = inv[(blk * 16 + ar) * 16 + c];
#pragma unroll
          for (int y = 0; y < JPT; ++y) v[y] = fmaf(m, tb[c * DVS + j0 + y], v[y]);
        }
#pragma unroll
        for (int y = 0; y < JPT; ++y) vn[a_ * DVS + j0 + y] = v[y];
        __syncthreads();
      }
    }
    // F: o = o_in + attn vn, bf16 out. G: S = e^{g_last} S + kd^T vn.
    {
      const int a0 = ri * RPT;
      float acc[RPT][4];
#pragma unroll
      for (int x = 0; x < RPT; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
      for (int b = 0; b < a0 + RPT; ++b) {
        const float4 vv = *reinterpret_cast<const float4*>(vn + b * DVS + 4 * ci);
        const float v4[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int x = 0; x < RPT; ++x) {
          const float m = atT[b * SUBP + a0 + x];
#pragma unroll
          for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(m, v4[y], acc[x][y]);
        }
      }
#pragma unroll
      for (int x = 0; x < RPT; ++x) {
        const int a_ = a0 + x;
        if (a_ < n) {
          __nv_bfloat16* orow = a.o + static_cast<int64_t>(s0 + a_) * vd_all + static_cast<int64_t>(h) * DV + c0 + 4 * ci;
#pragma unroll
          for (int y = 0; y < 4; ++y) orow[y] = __float2bfloat16_rn(__fadd_rn(oi[a_ * DVS + 4 * ci + y], acc[x][y]));
        }
      }
    }
    {
      const int di = tid / CG, d0 = di * DPT;
      const float el = eg[SUB - 1];
      float acc[DPT][4];
#pragma unroll
      for (int x = 0; x < DPT; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = 0.f;
#pragma unroll 4
      for (int a_ = 0; a_ < SUB; ++a_) {
        const float4 vv = *reinterpret_cast<const float4*>(vn + a_ * DVS + 4 * ci);
        const float v4[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int x = 0; x < DPT; ++x) {
          const float kx = kd[a_ * S::KDP + d0 + x];
#pragma unroll
          for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(kx, v4[y], acc[x][y]);
        }
      }
#pragma unroll
      for (int x = 0; x < DPT; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) {
          float* p = st + (d0 + x) * DVS + 4 * ci + y;
          *p = __fadd_rn(__fmul_rn(*p, el), acc[x][y]);
        }
    }
  }
  __syncthreads();
  for (int i = tid; i < DK * DVS; i += 256) {
    const int d = i / DVS, j = i % DVS;
    srow[d * DV + c0 + j] = __float2bfloat16_rn(st[i]);
  }
}

// ---------------------------------------------------------------------------------------------
// norm (+ conv carry)
// ---------------------------------------------------------------------------------------------
template <int DV>
__global__ void __launch_bounds__(256) gdn_prefill_norm_kernel(PrefillArgs a, int conv_dim) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x;
  if (t == a.tokens) {
    // The conv state keeps window rows n_valid .. n_valid + KCONV - 2 of [history * keep, chunk].
    for (int c = tid; c < conv_dim; c += blockDim.x) {
      __nv_bfloat16* cs = a.conv_state + static_cast<int64_t>(c) * (KCONV - 1);
      __nv_bfloat16 val[KCONV - 1];
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) {
        const int w = a.n_valid + j;
        val[j] = w < KCONV - 1 ? __float2bfloat16_rn(__bfloat162float(cs[w]) * a.keep)
                               : a.qkvz[static_cast<int64_t>(w - (KCONV - 1)) * a.ld_qkvz + c];
      }
#pragma unroll
      for (int j = 0; j < KCONV - 1; ++j) cs[j] = val[j];
    }
    return;
  }
  constexpr int CPL = DV / 32;
  const int64_t vd_all = static_cast<int64_t>(a.num_v_heads) * DV;
  const __nv_bfloat16* orow = a.o + static_cast<int64_t>(t) * vd_all;
  const __nv_bfloat16* zrow = a.qkvz + static_cast<int64_t>(t) * a.ld_qkvz + conv_dim;
  uint8_t* out = a.out + static_cast<int64_t>(t) * a.ld_out;
  for (int h = warp; h < a.num_v_heads; h += blockDim.x / 32) {
    float ob[CPL];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      ob[i] = __bfloat162float(orow[h * DV + lane * CPL + i]);
      ss = __fadd_rn(ss, __fmul_rn(ob[i], ob[i]));
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(DV)), a.eps));
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
      const int c = lane * CPL + i;
      const float n1 = bf16r(__fmul_rn(ob[i], r));
      const float n2 = bf16r(__fmul_rn(__bfloat162float(a.norm_w[c]), n1));
      const float z = __bfloat162float(zrow[h * DV + c]);
      out[h * DV + c] = f32_to_e5m2(bf16r(__fmul_rn(n2, __fmul_rn(z, sigmoidf_(z)))));
    }
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WsLayout {
  size_t qT, kT, v, beta, g, o, total;
};

WsLayout ws_layout(int64_t tokens, int hk, int hv, int dk, int dv) {
  WsLayout w{};
  size_t off = 0;
  w.qT = off;
  off = align256(off + sizeof(float) * hk * dk * tokens);
  w.kT = off;
  off = align256(off + sizeof(float) * hk * dk * tokens);
  w.v = off;
  off = align256(off + sizeof(float) * hv * tokens * dv);
  w.beta = off;
  off = align256(off + sizeof(float) * hv * tokens);
  w.g = off;
  off = align256(off + sizeof(float) * hv * tokens);
  w.o = off;
  off = align256(off + 2 * static_cast<size_t>(tokens) * hv * dv);
  w.total = off;
  return w;
}

template <int DK, int DV, int R>
int launch_prefill(PrefillArgs a, int conv_dim, cudaStream_t stream) {
  using S = DeltaSmem<DK>;
  static unsigned long long done_mask = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return q38host::cuda_status(e, "cudaGetDevice");
  const size_t prep_smem = sizeof(float) * (2 * DK + R * DV) * (PREP_TOK + 1);
  if (dev < 64 && !(done_mask & (1ull << dev))) {
    e = cudaFuncSetAttribute(gdn_prefill_prep_kernel<DK, DV, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(prep_smem));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gdn_prefill_delta_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(S::TOTAL));
    if (e != cudaSuccess) return q38host::cuda_status(e, "cudaFuncSetAttribute(gdn_prefill)");
    done_mask |= 1ull << dev;
  }
  dim3 gp((a.tokens + PREP_TOK - 1) / PREP_TOK, a.num_k_heads);
  gdn_prefill_prep_kernel<DK, DV, R><<<gp, 256, prep_smem, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "gdn_prefill_prep launch");
  dim3 gd(a.num_v_heads, DV / DVS);
  gdn_prefill_delta_kernel<DK, DV><<<gd, 256, S::TOTAL, stream>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return q38host::cuda_status(e, "gdn_prefill_delta launch");
  gdn_prefill_norm_kernel<DV><<<a.tokens + 1, 256, 0, stream>>>(a, conv_dim);
  return q38host::cuda_status(cudaGetLastError(), "gdn_prefill_norm launch");
}

}  // namespace

extern "C" size_t q38_gdn_prefill_workspace_bytes(int64_t tokens, int num_k_heads, int num_v_heads, int head_k,
                                                  int head_v) {
  if (tokens <= 0 || num_k_heads <= 0 || num_v_heads <= 0 || head_k <= 0 || head_v <= 0) return 0;
  return ws_layout(tokens, num_k_heads, num_v_heads, head_k, head_v).total;
}

extern "C" int q38_gdn_prefill_chunk(const void* qkvz, int64_t ld_qkvz, const void* ab, int64_t ld_ab, void* conv_state,
                                     const void* conv_weight, const void* a_log, const void* dt_bias,
                                     const void* norm_weight, void* state, int64_t slot, int64_t state_rows,
                                     int64_t tokens, int64_t start, int64_t n_valid, void* out, int64_t ld_out,
                                     int num_k_heads, int num_v_heads, int head_k, int head_v, int conv_kernel,
                                     float eps, void* workspace, size_t workspace_bytes, q38_stream_t stream) {
  using namespace q38host;
  if (!qkvz || !ab || !conv_state || !conv_weight || !a_log || !dt_bias || !norm_weight || !state || !out || !workspace)
    return set_error("q38_gdn_prefill_chunk: null pointer"), Q38_ERR_ARG;
  if (tokens <= 0 || tokens > 65535 || n_valid < 0 || n_valid > tokens || start < 0)
    return set_error("q38_gdn_prefill_chunk: bad tokens %lld / n_valid %lld / start %lld", static_cast<long long>(tokens),
                     static_cast<long long>(n_valid), static_cast<long long>(start)),
           Q38_ERR_ARG;
  if (slot < 0 || slot >= state_rows) return set_error("q38_gdn_prefill_chunk: slot %lld out of range", static_cast<long long>(slot)), Q38_ERR_ARG;
  if (num_k_heads <= 0 || num_v_heads <= 0 || num_v_heads % num_k_heads)
    return set_error("q38_gdn_prefill_chunk: bad head counts"), Q38_ERR_ARG;
  if (conv_kernel != KCONV) return set_error("q38_gdn_prefill_chunk: conv kernel %d not built (4 is)", conv_kernel), Q38_ERR_ARG;
  const int64_t conv_dim = 2LL * num_k_heads * head_k + static_cast<int64_t>(num_v_heads) * head_v;
  if (ld_qkvz < conv_dim + static_cast<int64_t>(num_v_heads) * head_v || ld_ab < 2 * num_v_heads ||
      ld_out < static_cast<int64_t>(num_v_heads) * head_v)
    return set_error("q38_gdn_prefill_chunk: leading dimension too small"), Q38_ERR_ARG;
  const WsLayout w = ws_layout(tokens, num_k_heads, num_v_heads, head_k, head_v);
  if (workspace_bytes < w.total || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error("q38_gdn_prefill_chunk: workspace needs %zu bytes, 256-byte aligned", w.total), Q38_ERR_ARG;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  PrefillArgs a{};
  a.qkvz = static_cast<const __nv_bfloat16*>(qkvz);
  a.ld_qkvz = ld_qkvz;
  a.ab = static_cast<const __nv_bfloat16*>(ab);
  a.ld_ab = ld_ab;
  a.conv_state = static_cast<__nv_bfloat16*>(conv_state) + slot * conv_dim * (KCONV - 1);
  a.conv_w = static_cast<const __nv_bfloat16*>(conv_weight);
  a.a_log = static_cast<const __nv_bfloat16*>(a_log);
  a.dt_bias = static_cast<const __nv_bfloat16*>(dt_bias);
  a.norm_w = static_cast<const __nv_bfloat16*>(norm_weight);
  a.state = static_cast<__nv_bfloat16*>(state) + slot * static_cast<int64_t>(num_v_heads) * head_k * head_v;
  a.tokens = static_cast<int>(tokens);
  a.n_valid = static_cast<int>(n_valid);
  a.keep = start > 0 ? 1.0f : 0.0f;
  a.out = static_cast<uint8_t*>(out);
  a.ld_out = ld_out;
  a.num_k_heads = num_k_heads;
  a.num_v_heads = num_v_heads;
  a.eps = eps;
  a.qT = reinterpret_cast<float*>(ws + w.qT);
  a.kT = reinterpret_cast<float*>(ws + w.kT);
  a.v = reinterpret_cast<float*>(ws + w.v);
  a.beta = reinterpret_cast<float*>(ws + w.beta);
  a.g = reinterpret_cast<float*>(ws + w.g);
  a.o = reinterpret_cast<__nv_bfloat16*>(ws + w.o);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rep = num_v_heads / num_k_heads;
  if (head_k == 128 && head_v == 128 && rep == 3) return launch_prefill<128, 128, 3>(a, static_cast<int>(conv_dim), s);
  if (head_k == 32 && head_v == 32 && rep == 3) return launch_prefill<32, 32, 3>(a, static_cast<int>(conv_dim), s);
  return set_error("q38_gdn_prefill_chunk: head dims %d/%d with %d value heads per key head not built", head_k, head_v, rep),
         Q38_ERR_UNSUPPORTED;
}
