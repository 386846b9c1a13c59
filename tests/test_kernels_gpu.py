"""Kernel-level parity of the sm_100a kernels against the CPU oracle (and float64 for the GEMM).

Tolerances, stated per check:
* bf16 outputs: within 1 bf16 ulp of the exact value, and exact for at least 98% of elements
  (differences come only from fp32 summation order before the final rounding).
* e5m2 outputs (FP8 linear inputs): codes equal or adjacent, adjacent for at most 2% of elements.
* gated-delta state: within 1e-2 absolute (BASELINE), and bit-equal for at least 95% of elements.
"""

import math

import pytest
import torch

from oracle import cpu_model as om

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16_ulp(x: torch.Tensor) -> torch.Tensor:
    a = x.float().abs().clamp_min(2.0**-126)
    return torch.ldexp(torch.ones_like(a), torch.floor(torch.log2(a)).int() - 7)


def assert_bf16_close(got, want, frac=0.02, what=""):
    got, want = got.float().cpu(), want.float().cpu()
    diff = (got - want).abs()
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    assert (diff <= bf16_ulp(want) * 1.01).all(), f"{what}: max diff {diff.max().item()} beyond 1 ulp"
    mism = (diff > 0).float().mean().item()
    assert mism <= frac, f"{what}: {mism:.4f} of elements differ"


def assert_gemm_close(got, exact, magnitude, what=""):
    """A GEMM with fp32 accumulation: within 1 bf16 ulp of the float64 result plus 2^-19 of
    sum_k |x_k w_k| (fp32 rounding of the running sum, visible only where the result cancels), and
    beyond 1 ulp for at most 0.5% of elements (and at most 8 of them in small outputs)."""
    got, exact, magnitude = got.double().cpu(), exact.cpu(), magnitude.cpu()
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    err = (got - exact).abs()
    ulp = bf16_ulp(exact).double()
    assert (err <= ulp * 1.01 + magnitude * 2.0**-19).all(), f"{what}: error {((err - ulp) / magnitude).max().item():.3g} of sum|xw|"
    beyond = int((err > ulp * 1.01).sum())
    assert beyond <= max(8, 5e-3 * err.numel()), f"{what}: {beyond} of {err.numel()} elements beyond 1 ulp"


def assert_attention_e5m2_close(got_bytes, want_bf16, what=""):
    """Attention outputs in e5m2: at most 2% of codes differ, 0.1% by more than one code, and every
    row within 2e-2 relative L2 of the oracle."""
    want_codes = want_bf16.float().to(torch.float8_e5m2).view(torch.uint8)
    d = (e5m2_code(got_bytes) - e5m2_code(want_codes)).abs()
    differ, far = (d > 0).float().mean().item(), (d > 1).float().mean().item()
    got = got_bytes.view(torch.float8_e5m2).float()
    want = want_codes.view(torch.float8_e5m2).float()
    rel = ((got - want).norm(dim=-1) / want.norm(dim=-1).clamp_min(1e-12)).max().item()
    msg = f"{what}: {differ:.4f} of codes differ, {far:.5f} by more than one, worst row relative L2 {rel:.3g}"
    assert differ <= 0.02 and far <= 1e-3 and rel <= 2e-2, msg


def e5m2_code(b: torch.Tensor) -> torch.Tensor:
    b = b.to(torch.int32)
    mag = b & 0x7F
    return torch.where(b >= 128, -mag, mag)


def assert_e5m2_close(got_bytes, want_bf16, frac=0.02, what=""):
    want = want_bf16.float().cpu().to(torch.float8_e5m2).view(torch.uint8)
    d = (e5m2_code(got_bytes.cpu()) - e5m2_code(want)).abs()
    assert d.max().item() <= 1, f"{what}: e5m2 codes differ by {d.max().item()}"
    mism = (d > 0).float().mean().item()
    assert mism <= frac, f"{what}: {mism:.4f} of e5m2 codes differ"


@pytest.fixture(scope="module")
def ops(pkg):
    mod = __import__(pkg.__name__ + ".ops", fromlist=["ops"])
    mod._lib.load()
    assert torch.cuda.is_available()
    return mod


def scaled_weight(pkg, rows, cols, gen, spread=12):
    """N(0,1) weights whose 32-groups carry independent power-of-two magnitudes, so every scale matters."""
    w = torch.randn(rows, cols, generator=gen)
    mags = torch.randint(-spread, 3, (rows, cols // 32), generator=gen).float()
    w = w * torch.exp2(mags).repeat_interleave(32, dim=1)
    return pkg.weights.FP8Weight.from_float(w)


GEMM_CASES = [
    # tokens, k, features, splits
    (3, 192, 320, 1),
    (8, 256, 384, 2),
    (64, 17408, 5120, 1),
    (64, 17408, 5120, 3),
    (200, 5120, 1024, 1),
    (256, 17408, 5120, 3),
    (300, 640, 520, 2),
    (512, 17408, 5120, 1),
    (256, 17408, 1024, 12),  # more splits than a portable cluster: the workspace path
    (40, 2048, 640, 8),
]


@pytest.mark.parametrize("tokens,k,features,splits", GEMM_CASES)
def test_fp8_gemm_matches_float64(pkg, ops, tokens, k, features, splits):
    gen = torch.Generator().manual_seed(tokens * 7 + k + features)
    w = scaled_weight(pkg, features, k, gen)
    x = torch.randn(tokens, k, generator=gen).to(torch.bfloat16)
    xq = pkg.codec.to_e5m2_bytes(x)
    lin = ops.DeviceLinear(w, DEV)
    y = torch.full((tokens, features), float("nan"), dtype=torch.bfloat16, device=DEV)
    ws = None
    if splits > 1:
        ws = torch.zeros(ops.gemm_workspace_bytes(tokens, features, splits), dtype=torch.uint8, device=DEV)
    ops.fp8_gemm(xq.to(DEV), lin, y, splits=splits, workspace=ws)
    torch.cuda.synchronize()
    xf, wf = pkg.codec.e5m2_bytes_to_float(xq).double().to(DEV), w.dequant().double().to(DEV)
    exact = xf @ wf.T
    magnitude = xf.abs() @ wf.abs().T  # sum_k |x_k w_k|, the scale of fp32 accumulation error
    assert_gemm_close(y, exact, magnitude, what=f"gemm {tokens}x{k}x{features}/{splits}")
    if splits > 1:
        # The kernel leaves the split counters at zero, so the same workspace serves the next call.
        counters = ws[: 4 * (-(-features // 128)) * (-(-tokens // ops.token_tile(tokens)))]
        assert int(counters.count_nonzero()) == 0
        y2 = torch.empty_like(y)
        ops.fp8_gemm(xq.to(DEV), lin, y2, splits=splits, workspace=ws)
        assert torch.equal(y, y2), "split-K result must not depend on which CTA finishes last"


STREAMK_CASES = [
    # tokens, k, features, residual
    (256, 17408, 5120, True),  # down_proj at TP = 1: every tile split between ~4 CTA pairs
    (256, 6144, 5120, True),  # out_proj / o_proj
    (64, 17408, 5120, False),  # 128-token tiles, one CTA per SM
    (8, 6144, 5120, True),
    (200, 3072, 1024, False),
    (512, 8704, 5120, True),  # two token tiles
    (37, 512, 384, True),  # fewer K steps than CTAs: some tiles whole
    (300, 640, 520, False),  # ragged features and tokens
]


@pytest.mark.parametrize("tokens,k,features,residual", STREAMK_CASES)
def test_fp8_gemm_streamk_matches_float64(pkg, ops, tokens, k, features, residual):
    """q38_fp8_gemm_streamk: within the GEMM tolerance of the float64 product; with the residual epilogue
    within 1 bf16 ulp of the split-K form's; the same bits on a second call (the last-arriver sum is in K
    order, and the counters are back at zero)."""
    gen = torch.Generator().manual_seed(tokens * 5 + k + features)
    w = scaled_weight(pkg, features, k, gen)
    x = torch.randn(tokens, k, generator=gen).to(torch.bfloat16)
    xq = pkg.codec.to_e5m2_bytes(x).to(DEV)
    lin = ops.DeviceLinear(w, DEV)
    res = (torch.randn(tokens, features, generator=gen) * 4).to(torch.bfloat16).to(DEV) if residual else None
    ws = torch.zeros(ops.streamk_workspace_bytes(tokens, features, k), dtype=torch.uint8, device=DEV)
    y = torch.full((tokens, features), float("nan"), dtype=torch.bfloat16, device=DEV)
    ops.fp8_gemm_streamk(xq, lin, y, ws, residual=res)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    xf, wf = pkg.codec.e5m2_bytes_to_float(xq.cpu()).double().to(DEV), w.dequant().double().to(DEV)
    exact = xf @ wf.T
    magnitude = xf.abs() @ wf.abs().T
    if residual:
        # bf16(residual + bf16(acc)) against the split-K form's residual epilogue on the same inputs: the
        # fp32 sums run in another order, so the two accumulators differ by up to twice the fp32 rounding
        # of the running sum (2^-19 of sum |x w| each, as assert_gemm_close allows) and bf16(acc) by up to
        # one more ulp; the sum with the residual then adds one ulp of the result.
        splits = ops.choose_splits(tokens, features, k)
        wsk = torch.zeros(max(256, ops.gemm_workspace_bytes(tokens, features, splits)), dtype=torch.uint8, device=DEV)
        ref = res.clone()
        ops.fp8_gemm(xq, lin, ref, residual=ref, splits=splits, workspace=wsk)
        torch.cuda.synchronize()
        got, want = y.double().cpu(), ref.double().cpu()
        diff = (got - want).abs()
        bound = bf16_ulp(want).double() + bf16_ulp(exact.cpu()).double() + 2 * magnitude.cpu() * 2.0**-19
        assert torch.isfinite(got).all() and (diff <= bound * 1.01).all(), f"streamk {tokens}x{k}x{features} + residual"
        assert (diff > 0).float().mean().item() <= 0.02, f"streamk {tokens}x{k}x{features}: too many elements differ"
    else:
        assert_gemm_close(y, exact, magnitude, what=f"streamk {tokens}x{k}x{features}")
    y2 = torch.empty_like(y)
    ops.fp8_gemm_streamk(xq, lin, y2, ws, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(y, y2), "stream-K result must not depend on which CTA finishes a tile last"


def test_fp8_gemm_residual_epilogue_and_oracle_linear(pkg, ops):
    gen = torch.Generator().manual_seed(3)
    tokens, k, features = 37, 512, 384
    w = pkg.weights.FP8Weight.from_float(torch.randn(features, k, generator=gen) * 0.02)
    x = torch.randn(tokens, k, generator=gen).to(torch.bfloat16)
    res = torch.randn(tokens, features, generator=gen).to(torch.bfloat16)
    lin = ops.DeviceLinear(w, DEV)
    y = res.to(DEV).clone()
    ops.fp8_gemm(pkg.codec.to_e5m2_bytes(x).to(DEV), lin, y, residual=y)
    torch.cuda.synchronize()
    want = res + om.linear_of(w)(x)  # the oracle's BF16 linear, then the BF16 residual add
    assert_bf16_close(y, want, what="residual epilogue")


def test_rmsnorm_quant_matches_oracle_and_torch_e5m2(pkg, ops):
    gen = torch.Generator().manual_seed(5)
    rows, n = 19, 5120
    x = (torch.randn(rows, n, generator=gen) * torch.exp2(torch.randint(-8, 8, (rows, 1), generator=gen).float())).to(torch.bfloat16)
    w = (torch.randn(n, generator=gen) * 0.3).to(torch.bfloat16)
    yb = torch.empty(rows, n, dtype=torch.bfloat16, device=DEV)
    yq = torch.empty(rows, n, dtype=torch.uint8, device=DEV)
    ops.rmsnorm_quant(x.to(DEV), w.to(DEV), 1e-6, yb, yq)
    torch.cuda.synchronize()
    assert_bf16_close(yb, om.rms_norm(x, w, 1e-6), what="rmsnorm")
    # The kernel's e5m2 of its own bf16 output equals torch's e5m2 rounding, bit for bit.
    assert torch.equal(yq.cpu(), yb.cpu().to(torch.float8_e5m2).view(torch.uint8))


def test_e5m2_rounding_of_every_bf16_value(pkg, ops):
    """Every finite bf16 up to e5m2's largest finite value through the kernels' e5m2 rounding, against
    torch's cast (the reference's fp8_round). silu_mul_quant with gate 1.28125 gives bf16(silu(g)) == 1.0,
    so its output is e5m2(u) exactly."""
    bits = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    v = bits[torch.isfinite(bits.float()) & (bits.float().abs() <= 57344)]
    v = v[: (v.numel() // 8) * 8].reshape(-1, 8)
    g = torch.full_like(v, 1.28125)
    assert torch.equal(om.silu(g), torch.ones_like(g)), "the gate must make bf16(silu(g)) exactly 1"
    y = torch.empty(v.shape, dtype=torch.uint8, device=DEV)
    ops.silu_mul_quant(torch.cat((g, v), dim=1).to(DEV), 8, y)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), v.to(torch.float8_e5m2).view(torch.uint8))


def test_silu_mul_quant_matches_oracle(pkg, ops):
    gen = torch.Generator().manual_seed(6)
    rows, n = 33, 1024
    g = (torch.randn(rows, n, generator=gen) * 3).to(torch.bfloat16)
    u = (torch.randn(rows, n, generator=gen) * 3).to(torch.bfloat16)
    y = torch.empty(rows, n, dtype=torch.uint8, device=DEV)
    ops.silu_mul_quant(torch.cat((g, u), 1).to(DEV), n, y)
    torch.cuda.synchronize()
    assert_e5m2_close(y, om.silu(g) * u, frac=0.002, what="silu*up")


@pytest.mark.parametrize("tokens,k,inter", [(8, 5120, 17408), (256, 5120, 17408), (37, 512, 256), (300, 1024, 640),
                                             (512, 5120, 8704)])
def test_fp8_gemm_silu_matches_oracle(pkg, ops, tokens, k, inter):
    """The gate/up GEMM with SiLU(gate) * up fused into its epilogue (weights interleaved in 64-row
    blocks) against (1) the unfused kernels on the same inputs, bit for bit, and (2) the oracle's
    BF16 gate_proj / up_proj then silu(gate) * up, in e5m2 codes."""
    gen = torch.Generator().manual_seed(tokens + inter)
    gate = pkg.weights.FP8Weight.from_float(torch.randn(inter, k, generator=gen) * 0.03)
    up = pkg.weights.FP8Weight.from_float(torch.randn(inter, k, generator=gen) * 0.03)
    x = torch.randn(tokens, k, generator=gen).to(torch.bfloat16)
    xq = pkg.codec.to_e5m2_bytes(x).to(DEV)
    fused = ops.DeviceLinear(pkg.weights.FP8Weight.interleave_rows(gate, up), DEV)
    y = torch.full((tokens, inter), 0x7F, dtype=torch.uint8, device=DEV)
    ops.fp8_gemm_silu(xq, fused, y)
    # Unfused: one GEMM over [gate; up] (single K split, the fused kernel's summation order), then silu*up.
    plain = ops.DeviceLinear(pkg.weights.FP8Weight.cat_rows([gate, up]), DEV)
    gu = torch.empty(tokens, 2 * inter, dtype=torch.bfloat16, device=DEV)
    ops.fp8_gemm(xq, plain, gu, splits=1)
    want = torch.empty_like(y)
    ops.silu_mul_quant(gu, inter, want)
    torch.cuda.synchronize()
    assert torch.equal(y, want), f"fused vs unfused: {(y != want).sum().item()} of {y.numel()} bytes differ"
    if tokens * k * inter <= 2e9:  # the oracle's CPU matmuls stay within seconds
        xd = pkg.codec.e5m2_bytes_to_float(xq.cpu()).to(torch.bfloat16)
        ref = om.silu(om.linear_of(gate)(xd)) * om.linear_of(up)(xd)
        assert_e5m2_close(y, ref, frac=0.01, what=f"fused silu {tokens}x{k}x{inter}")


@pytest.mark.parametrize("rows,k,n,splits", [(13, 5120, 96, 1), (256, 5120, 96, 40), (8, 128, 12, 2), (200, 640, 130, 3)])
def test_bf16_linear_matches_float64(pkg, ops, rows, k, n, splits):
    gen = torch.Generator().manual_seed(8 + rows)
    x = torch.randn(rows, k, generator=gen).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=gen) * 0.02).to(torch.bfloat16)
    y = torch.empty(rows, n, dtype=torch.bfloat16, device=DEV)
    lin = ops.DeviceBF16Linear(w, DEV)
    ws = torch.zeros(max(256, ops.gemm_workspace_bytes(rows, n, splits)), dtype=torch.uint8, device=DEV)
    ops.bf16_linear(x.to(DEV), lin, y, splits=splits, workspace=ws)
    torch.cuda.synchronize()
    exact = x.double() @ w.double().T
    assert_gemm_close(y, exact, x.double().abs() @ w.double().abs().T, what=f"bf16 linear {rows}x{k}x{n}/{splits}")


@pytest.mark.parametrize("rows,splits", [(8, 8), (100, 4), (256, 8), (256, 2)])
def test_bf16_linear_workspace_and_cluster_paths_agree_bitwise(pkg, ops, rows, splits):
    """Split partials through the workspace (independent CTA pairs) and through a cluster's shared
    memory are summed in the same split order: the outputs are the same bits. Run twice through the
    workspace, which must have reset its counters."""
    gen = torch.Generator().manual_seed(21 + rows)
    x = torch.randn(rows, 5120, generator=gen).to(torch.bfloat16).to(DEV)
    w = (torch.randn(96, 5120, generator=gen) * 0.02).to(torch.bfloat16)
    lin = ops.DeviceBF16Linear(w, DEV)
    ws = torch.zeros(max(256, ops.gemm_workspace_bytes(rows, 96, splits)), dtype=torch.uint8, device=DEV)
    y_ws, y_cl = (torch.empty(rows, 96, dtype=torch.bfloat16, device=DEV) for _ in range(2))
    for _ in range(2):
        ops.bf16_linear(x, lin, y_ws, splits=splits, workspace=ws)
    ops.bf16_linear(x, lin, y_cl, splits=splits, workspace=None)
    torch.cuda.synchronize()
    assert torch.equal(y_ws.view(torch.int16), y_cl.view(torch.int16))


@pytest.mark.parametrize("batch,max_seq", [(1, 64), (256, 512), (1000, 300), (4096, 2048)])
def test_attn_row_order_is_longest_first(ops, batch, max_seq):
    """The schedule is the permutation that sorts rows by decreasing visible 32-position tiles (inactive
    rows see none), ties by row index, as a stable CPU sort gives it."""
    gen = torch.Generator().manual_seed(batch)
    position = torch.randint(-3, max_seq + 40, (batch,), generator=gen, dtype=torch.int32)
    active = (torch.rand(batch, generator=gen) > 0.1).float()
    order = ops.attn_row_order(position.to(DEV), active.to(DEV), max_seq, torch.full((batch,), -1, dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    seen = torch.where(active > 0.5, position.clamp(0, max_seq), torch.zeros_like(position))
    tiles = (seen.long() + 31) // 32
    want = sorted(range(batch), key=lambda r: (-int(tiles[r]), r))
    assert order.cpu().tolist() == want


def _gdn_setup(pkg, cfg, batch, gen):
    w = pkg.weights.synthetic_layer(cfg, 0, seed=11, device="cpu", std=0.1)
    layer = om.GDNLayer(cfg, w, "layers.0", 1, batch, torch.bfloat16)
    layer.recurrent_state.copy_((torch.randn(layer.recurrent_state.shape, generator=gen) * 0.1).to(torch.bfloat16))
    layer.conv_state.copy_(torch.randn(layer.conv_state.shape, generator=gen).to(torch.bfloat16))
    return layer


@pytest.mark.parametrize("shape,batch", [("tiny", 5), ("full", 62)])
def test_gdn_decode_matches_oracle(pkg, ops, shape, batch):
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(12)
    layer = _gdn_setup(pkg, cfg, batch, gen)
    conv_dim, vd, hv = cfg.linear_conv_dim, cfg.linear_value_dim, cfg.linear_num_value_heads
    qkv = torch.randn(batch, conv_dim, generator=gen).to(torch.bfloat16)
    z = torch.randn(batch, vd, generator=gen).to(torch.bfloat16)
    b_raw = torch.randn(batch, hv, generator=gen).to(torch.bfloat16)
    a_raw = torch.randn(batch, hv, generator=gen).to(torch.bfloat16)
    position = torch.randint(1, 400, (batch,), generator=gen, dtype=torch.int32)
    position[0] = 0  # a fresh sequence
    active = torch.ones(batch)
    active[1] = 0.0  # an idle row keeps its state bit for bit
    state0 = layer.recurrent_state.clone()
    conv0 = layer.conv_state.clone()
    # GPU first (the oracle updates its buffers in place).
    d_state, d_conv = state0.to(DEV), conv0.to(DEV)
    out = torch.empty(batch, vd, dtype=torch.uint8, device=DEV)
    ab = torch.cat((b_raw, a_raw), 1).to(DEV)
    ops.gdn_decode(torch.cat((qkv, z), 1).to(DEV), ab, d_conv, layer.conv_w.to(DEV), layer.A_log.to(DEV),
                   layer.dt_bias.to(DEV), layer.norm_w.to(DEV), d_state, position.to(DEV), active.to(DEV), out,
                   batch=batch, num_k_heads=cfg.linear_num_key_heads, num_v_heads=hv, head_k=cfg.linear_key_head_dim,
                   head_v=cfg.linear_value_head_dim, eps=cfg.rms_norm_eps)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    h = layer.decode_core(qkv, z, b_raw, a_raw, position, active)
    on = active > 0.5
    assert_e5m2_close(out.cpu()[on], h[on], what="gdn out")
    got_state = d_state.cpu()
    assert torch.equal(got_state[1], state0[1]) and torch.equal(d_conv.cpu()[1], conv0[1]), "idle row changed"
    diff = (got_state.float() - layer.recurrent_state.float()).abs()
    assert diff.max().item() < 1e-2, f"state differs by {diff.max().item()}"
    assert (diff == 0).float().mean().item() > 0.95
    assert torch.equal(d_conv.cpu(), layer.conv_state)


@pytest.mark.parametrize("shape,batch,max_seq", [("tiny", 4, 64), ("full", 9, 512), ("full", 40, 512), ("tiny", 12, 200)])
def test_attn_decode_matches_oracle(pkg, ops, shape, batch, max_seq):
    """Against the oracle's decode, rows at positions on and around the 64- and 128-position chunk
    edges, the last position and inactive rows; a second call gives the same bytes (the kernels'
    chunk counters are back at zero)."""
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(13)
    w = pkg.weights.synthetic_layer(cfg, 3, seed=11, device="cpu", std=0.1)
    layer = om.AttentionLayer(cfg, w, "layers.3", 1, 0, batch, max_seq, torch.bfloat16)
    layer.k_cache.copy_(torch.randn(layer.k_cache.shape, generator=gen).to(torch.bfloat16))
    layer.v_cache.copy_(torch.randn(layer.v_cache.shape, generator=gen).to(torch.bfloat16))
    hd, heads, kvh = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    qg = torch.randn(batch, 1, heads * 2 * hd, generator=gen).to(torch.bfloat16)
    k = torch.randn(batch, 1, kvh * hd, generator=gen).to(torch.bfloat16)
    v = torch.randn(batch, 1, kvh * hd, generator=gen).to(torch.bfloat16)
    position = torch.randint(1, max_seq - 1, (batch,), generator=gen, dtype=torch.int32)
    edges = torch.tensor([0, 63, 64, 65, 127, 128, 129, 255, 256, max_seq - 2, max_seq - 1], dtype=torch.int32)
    edges = edges[edges < max_seq][: batch - 1]
    position[: edges.numel()] = edges
    active = torch.ones(batch)
    active[-1] = 0.0
    cos, sin = om.rotary(cfg, position, torch.bfloat16)
    kc0, vc0 = layer.k_cache.clone(), layer.v_cache.clone()
    d_k, d_v = kc0.to(DEV), vc0.to(DEV)
    out = torch.empty(batch, heads * hd, dtype=torch.uint8, device=DEV)
    ops.attn_decode(torch.cat((qg, k, v), -1).reshape(batch, -1).to(DEV), layer.q_norm.to(DEV), layer.k_norm.to(DEV),
                    cos.to(DEV), sin.to(DEV), d_k, d_v, position.to(DEV), active.to(DEV), out, batch=batch,
                    num_q_heads=heads, num_kv_heads=kvh, head_dim=hd, rot_dim=cfg.rotary_dim, eps=cfg.rms_norm_eps)
    torch.cuda.synchronize()
    # Again, scheduled longest row first: the same bytes (the order only places the rows' CTAs).
    out2 = torch.empty_like(out)
    order = ops.attn_row_order(position.to(DEV), active.to(DEV), max_seq, torch.empty(batch, dtype=torch.int32, device=DEV))
    ops.attn_decode(torch.cat((qg, k, v), -1).reshape(batch, -1).to(DEV), layer.q_norm.to(DEV), layer.k_norm.to(DEV),
                    cos.to(DEV), sin.to(DEV), d_k, d_v, position.to(DEV), active.to(DEV), out2, batch=batch,
                    num_q_heads=heads, num_kv_heads=kvh, head_dim=hd, rot_dim=cfg.rotary_dim, eps=cfg.rms_norm_eps,
                    row_order=order)
    torch.cuda.synchronize()
    assert sorted(order.cpu().tolist()) == list(range(batch))
    assert torch.equal(out, out2), "a repeated, reordered call must give the same bytes"
    want = layer.decode_core(qg, k, v, cos.unsqueeze(1), sin.unsqueeze(1), position, active).reshape(batch, -1)
    on = active > 0.5
    # fp32 summation order differs from the oracle's matmul: where W V nearly cancels the own value's
    # term the small result can move by more than one e5m2 code (rare, bounded in L2).
    assert_attention_e5m2_close(out.cpu()[on], want[on], what="attention out")
    assert_bf16_close(d_k.cpu(), layer.k_cache, frac=0.001, what="k cache")
    assert torch.equal(d_v.cpu(), layer.v_cache)


@pytest.mark.parametrize("rows,vocab", [(11, 4096), (64, 4224), (100, 3104), (256, 4096), (300, 4224), (256, 8192 + 96)])
def test_lm_head_groupmax_matches_oracle(pkg, ops, rows, vocab):
    """Group-of-32 maxima of the logits against float64: batch tiles of 64/128/256 and several of
    them (300 rows), an odd count of 128-row weight tiles (4224) and a partial last tile (3104)."""
    cfg = pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(14 + rows + vocab)
    h = cfg.hidden_size
    w = pkg.weights.FP8Weight.from_float(torch.randn(vocab, h, generator=gen) * 0.02)
    x = torch.randn(rows, h, generator=gen).to(torch.bfloat16)
    maxima = torch.full((rows, vocab // 32), float("nan"), device=DEV)  # every entry must be written
    ops.lm_head_groupmax(x.to(DEV), ops.DeviceBF16Linear(w.dequant().to(torch.bfloat16), DEV), maxima)
    torch.cuda.synchronize()
    logits = x.double() @ w.dequant().double().T
    want = logits.reshape(rows, -1, 32).amax(-1).float()
    got = maxima.cpu()
    assert ((got - want).abs() <= 1e-5 * want.abs().clamp_min(1e-3)).all()
    assert torch.equal(got.topk(4, -1).indices, want.topk(4, -1).indices)
