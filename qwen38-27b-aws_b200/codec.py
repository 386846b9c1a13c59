"""FP8 number formats of the hot path, in PyTorch (CPU or CUDA tensors alike).

* Weights: FP8 e4m3 (OCP e4m3fn) bytes with one power-of-two scale per 32 input columns, kept as
  fp32 in host files and as UE8M0 bytes (exponent + 127) on the device. A power-of-two scale makes
  the dequantised weight e4m3 * 2^s exact in BF16, so dequantise-then-BF16-matmul (the reference's
  CPU path, qwen38_inf2/model.py:222-225) and the tensor cores' block-scaled MMA see the same values.
* Activations: FP8 e5m2, the rounding the reference applies to every FP8 linear's input
  (`fp8_round`, qwen38_inf2/model.py:85-87).
"""

from __future__ import annotations

import torch

GROUP = 32
E4M3_MAX = 448.0
UE8M0_BIAS = 127
# Scale bytes per (128 weight rows, 128 K) block, the unit the GEMM kernel loads per pipeline stage.
SF_TILE_ROWS = 128
SF_TILE_K = 128
SF_BLOCK_BYTES = 512


def round_e5m2(x: torch.Tensor) -> torch.Tensor:
    """Round to FP8 e5m2 and back, in x's dtype (round to nearest even)."""
    return x.to(torch.float8_e5m2).to(x.dtype)


def to_e5m2_bytes(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float8_e5m2).view(torch.uint8)


def e5m2_bytes_to_float(b: torch.Tensor) -> torch.Tensor:
    return b.view(torch.float8_e5m2).float()


def quantize_mx_e4m3(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise a float matrix ``[out, in]`` to (e4m3 bytes ``[out, in]``, fp32 power-of-two scales ``[out, in / 32]``).

    Each group of 32 along the input dimension gets the smallest power-of-two scale s with
    max|w| / s <= 448, so nothing saturates; an all-zero group gets scale 1.
    """
    if w.dim() != 2 or w.shape[1] % GROUP:
        raise ValueError(f"expected [out, in] with in a multiple of {GROUP}, got {tuple(w.shape)}")
    rows, cols = w.shape
    g = w.float().reshape(rows, cols // GROUP, GROUP)
    amax = g.abs().amax(dim=-1)
    mant, exp = torch.frexp(amax / E4M3_MAX)  # amax/448 = mant * 2^exp, mant in [0.5, 1)
    exponent = torch.where(mant == 0.5, exp - 1, exp)
    # Guard the rounding of amax / 448: step the exponent until the group fits exactly.
    exponent = torch.where(amax > E4M3_MAX * torch.ldexp(torch.ones_like(amax), exponent), exponent + 1, exponent)
    exponent = torch.where(amax == 0, torch.zeros_like(exponent), exponent).clamp(-UE8M0_BIAS, UE8M0_BIAS)
    scale = torch.ldexp(torch.ones_like(amax), exponent)
    q = (g / scale.unsqueeze(-1)).to(torch.float8_e4m3fn).view(torch.uint8).reshape(rows, cols)
    return q.contiguous(), scale.contiguous()


def dequantize_mx_e4m3(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 ``[out, in]`` values of e4m3 bytes times their per-32 scales."""
    return q.view(torch.float8_e4m3fn).float() * scale.repeat_interleave(GROUP, dim=1)


def scale_to_ue8m0(scale: torch.Tensor) -> torch.Tensor:
    """Power-of-two fp32 scales to UE8M0 bytes (exponent + 127)."""
    _, exp = torch.frexp(scale)
    return (exp - 1 + UE8M0_BIAS).to(torch.uint8)


def tile_scales(ue8m0: torch.Tensor) -> torch.Tensor:
    """UE8M0 scales ``[out, in / 32]`` to the GEMM kernel's tiled layout (flat uint8).

    One 512-byte block per (128 rows, 4 groups = 128 K): byte ``(r % 32) * 16 + (r // 32) * 4 + g % 4``
    holds row r's scale of group g, the layout tcgen05.cp 32x128b.warpx4 moves into tensor memory for
    the block-scaled MMA. Padding rows and groups hold 127 (scale 1.0).
    """
    rows, groups = ue8m0.shape
    rp = -(-rows // SF_TILE_ROWS) * SF_TILE_ROWS
    gp = -(-groups // 4) * 4
    padded = torch.full((rp, gp), UE8M0_BIAS, dtype=torch.uint8, device=ue8m0.device)
    padded[:rows, :groups] = ue8m0
    t = padded.reshape(rp // SF_TILE_ROWS, 4, 32, gp // 4, 4)  # [row tile, quarter, row, k chunk, group]
    return t.permute(0, 3, 2, 1, 4).contiguous().reshape(-1)


W_TILE_ROWS = 128
W_TILE_BYTES = 128  # bytes of K per tile row: one 128-byte swizzle row
W_TILE_SIZE = W_TILE_ROWS * W_TILE_BYTES


def tile_weight(w: torch.Tensor) -> torch.Tensor:
    """A weight [out, in] (any element size) to the GEMM kernel's tiled layout (flat uint8).

    Tiles of 128 rows x 128 bytes of K, ordered [row tile][K tile], each 16 KB tile contiguous and
    already 128-byte swizzled (16-byte chunk c of row r stored at chunk c ^ (r % 8)), which is the
    layout a TMA load with 128-byte swizzle would leave in shared memory. A pipeline stage then moves
    one contiguous 16 KB block with a single bulk copy, so HBM sees long sequential streams instead of
    128-byte pieces of thousands of rows. Padding rows and K bytes are zero.
    """
    b = w.contiguous().view(torch.uint8)
    rows, kb = b.shape
    rp = -(-rows // W_TILE_ROWS) * W_TILE_ROWS
    kp = -(-kb // W_TILE_BYTES) * W_TILE_BYTES
    padded = torch.zeros((rp, kp), dtype=torch.uint8, device=b.device)
    padded[:rows, :kb] = b
    t = padded.reshape(rp // W_TILE_ROWS, W_TILE_ROWS, kp // W_TILE_BYTES, 8, 16)  # [rt, r, kt, chunk, byte]
    r = torch.arange(W_TILE_ROWS, device=b.device)
    chunk = torch.arange(8, device=b.device)
    src = chunk.unsqueeze(0) ^ (r % 8).unsqueeze(1)  # stored chunk c holds logical chunk c ^ (r % 8)
    t = t.gather(3, src.reshape(1, W_TILE_ROWS, 1, 8, 1).expand(t.shape[0], -1, t.shape[2], -1, 16))
    return t.permute(0, 2, 1, 3, 4).contiguous().reshape(-1)


def untile_weight(tiles: torch.Tensor, rows: int, row_bytes: int) -> torch.Tensor:
    """Inverse of `tile_weight` on bytes (for tests)."""
    rp = -(-rows // W_TILE_ROWS) * W_TILE_ROWS
    kp = -(-row_bytes // W_TILE_BYTES) * W_TILE_BYTES
    t = tiles.reshape(rp // W_TILE_ROWS, kp // W_TILE_BYTES, W_TILE_ROWS, 8, 16)
    r = torch.arange(W_TILE_ROWS, device=tiles.device)
    chunk = torch.arange(8, device=tiles.device)
    src = chunk.unsqueeze(0) ^ (r % 8).unsqueeze(1)  # logical chunk c sits at stored chunk c ^ (r % 8)
    t = t.gather(3, src.reshape(1, 1, W_TILE_ROWS, 8, 1).expand(t.shape[0], t.shape[1], -1, -1, 16))
    return t.permute(0, 2, 1, 3, 4).reshape(rp, kp)[:rows, :row_bytes].contiguous()


def untile_scales(tiles: torch.Tensor, rows: int, groups: int) -> torch.Tensor:
    """Inverse of `tile_scales` (for tests)."""
    rp = -(-rows // SF_TILE_ROWS) * SF_TILE_ROWS
    gp = -(-groups // 4) * 4
    t = tiles.reshape(rp // SF_TILE_ROWS, gp // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(rp, gp)
    return t[:rows, :groups].contiguous()
