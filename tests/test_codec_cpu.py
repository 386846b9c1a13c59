"""FP8 codecs: the weight format is exact in BF16, scales tile as the GEMM kernel reads them."""

import torch


def test_mx_e4m3_dequantises_exactly_to_bf16(pkg):
    gen = torch.Generator().manual_seed(0)
    w = torch.randn(64, 256, generator=gen) * torch.exp2(torch.randint(-20, 4, (64, 1), generator=gen).float())
    q, s = pkg.codec.quantize_mx_e4m3(w)
    deq = pkg.codec.dequantize_mx_e4m3(q, s)
    assert torch.equal(deq, deq.to(torch.bfloat16).float()), "e4m3 * 2^s must be exact in bf16"
    # Scales are powers of two and no group saturates.
    m, _ = torch.frexp(s)
    assert torch.all(m == 0.5)
    groups = (w.reshape(64, 8, 32).abs().amax(-1) / s)
    assert groups.max() <= 448 and groups.max() > 224
    # Quantisation error is within e4m3's half-ulp (relative 2^-4) of each value, above the subnormals.
    big = w.abs() > s.repeat_interleave(32, 1) * 2.0**-6
    assert ((deq - w).abs()[big] <= w.abs()[big] * 2.0**-4 + 1e-30).all()


def test_zero_group_gets_unit_scale(pkg):
    w = torch.zeros(2, 64)
    w[1, 40] = 3.0
    q, s = pkg.codec.quantize_mx_e4m3(w)
    assert s[0, 0] == 1.0 and s[0, 1] == 1.0 and s[1, 0] == 1.0
    assert pkg.codec.dequantize_mx_e4m3(q, s)[1, 40] == 3.0


def test_scale_tiles_round_trip_and_layout(pkg):
    gen = torch.Generator().manual_seed(1)
    rows, groups = 300, 11
    ue = torch.randint(100, 140, (rows, groups), generator=gen, dtype=torch.int32).to(torch.uint8)
    tiles = pkg.codec.tile_scales(ue)
    assert tiles.numel() == 3 * 3 * 512
    assert torch.equal(pkg.codec.untile_scales(tiles, rows, groups), ue)
    # Row r, group g of tile (rt, kc) sits at byte (r % 32) * 16 + (r // 32) * 4 + g % 4.
    r, g = 165, 9
    rt, kc, rr = r // 128, g // 4, r % 128
    block = tiles[(rt * 3 + kc) * 512 : (rt * 3 + kc + 1) * 512]
    assert block[(rr % 32) * 16 + (rr // 32) * 4 + g % 4] == ue[r, g]
    # Padding is scale 1.0.
    assert tiles[(2 * 3 + 2) * 512 + 31 * 16 + 3 * 4 + 3] == 127


def test_ue8m0_bytes(pkg):
    s = torch.tensor([1.0, 2.0**-13, 2.0**5, 2.0**-127])
    assert pkg.codec.scale_to_ue8m0(s).tolist() == [127, 114, 132, 0]


def test_e5m2_round_matches_reference_codec(pkg):
    """round_e5m2 is the reference's fp8_round (model.py:85-87): torch's e5m2 cast."""
    x = torch.linspace(-300, 300, 10001).to(torch.bfloat16)
    assert torch.equal(pkg.codec.round_e5m2(x), x.to(torch.float8_e5m2).to(torch.bfloat16))


def test_weight_tiles_are_swizzled_16kb_blocks(pkg):
    """tile_weight: [row tile][K tile] blocks of 128 rows x 128 bytes, chunk c of row r stored at c ^ (r % 8)."""
    gen = torch.Generator().manual_seed(2)
    w = torch.randint(0, 256, (300, 400), generator=gen, dtype=torch.int32).to(torch.uint8)
    t = pkg.codec.tile_weight(w)
    assert t.numel() == 3 * 4 * 16384
    assert torch.equal(pkg.codec.untile_weight(t, 300, 400), w)
    rt, kt, r, c = 1, 2, 13, 5  # row 128 + 13, bytes 256 + 16*5 ...
    block = t[(rt * 4 + kt) * 16384 : (rt * 4 + kt + 1) * 16384].reshape(128, 128)
    stored = c ^ (r % 8)
    assert torch.equal(block[r, stored * 16 : stored * 16 + 16], w[rt * 128 + r, kt * 128 + c * 16 : kt * 128 + c * 16 + 16])
    # Padding is zero; BF16 weights tile on their bytes.
    assert int(t.reshape(3, 4, 128, 128)[2, :, 300 - 256 :].count_nonzero()) == 0
    wb = torch.randn(130, 96, generator=gen).to(torch.bfloat16)
    assert torch.equal(pkg.codec.untile_weight(pkg.codec.tile_weight(wb), 130, 192).view(torch.bfloat16), wb)
