"""Synthetic model weights and their tensor-parallel cut.

Names follow the reference model's parameters (qwen38_inf2/model.py, as loaded by
checkpoint.layer_weights, qwen38_inf2/checkpoint.py:185-224), with each FP8 linear held as an
`FP8Weight` ([out, in] e4m3 bytes plus per-32 power-of-two scales) instead of the reference's
[in, out] e5m2 `weight_fp8`. The cutting rules are the reference's: column-parallel matrices by
output rows, row-parallel ones (down_proj, out_proj, o_proj) by input columns, in_proj_qkv and the
conv weight block by block over [q | k | v] (checkpoint.py:150-174), plus KV-head replication when
there are more ranks than KV heads.

Values are seeded N(0, 0.02) for every matrix and vector (BASELINE configs 0 and 3), drawn per
tensor from its own generator so any one layer can be regenerated alone, on CPU or on the GPU.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass, replace

import torch

from . import codec
from .config import FULL, LINEAR, TextConfig

STD = 0.02


@dataclass
class FP8Weight:
    q: torch.Tensor  # uint8 [out, in], e4m3 bytes
    scale: torch.Tensor  # float32 [out, in / 32], powers of two

    @property
    def shape(self) -> tuple[int, int]:
        return tuple(self.q.shape)

    def dequant(self) -> torch.Tensor:
        return codec.dequantize_mx_e4m3(self.q, self.scale)

    def rows(self, start: int, end: int) -> "FP8Weight":
        return FP8Weight(self.q[start:end], self.scale[start:end])

    def cols(self, start: int, end: int) -> "FP8Weight":
        if start % codec.GROUP or end % codec.GROUP:
            raise ValueError("a column cut must land on a 32-column scale group")
        return FP8Weight(self.q[:, start:end], self.scale[:, start // codec.GROUP : end // codec.GROUP])

    def to(self, device) -> "FP8Weight":
        return FP8Weight(self.q.to(device), self.scale.to(device))

    @staticmethod
    def cat_rows(parts: list["FP8Weight"]) -> "FP8Weight":
        return FP8Weight(torch.cat([p.q for p in parts]).contiguous(), torch.cat([p.scale for p in parts]).contiguous())

    @staticmethod
    def interleave_rows(a: "FP8Weight", b: "FP8Weight", block: int = 64) -> "FP8Weight":
        """Rows a[0:block], b[0:block], a[block:2 block], b[block:2 block], ...: the gate/up layout of the
        fused MLP GEMM, whose 128-row tiles each hold matching gate and up rows."""
        if a.shape != b.shape or a.shape[0] % block:
            raise ValueError(f"interleave needs equal shapes with rows a multiple of {block}: {a.shape}, {b.shape}")
        n = a.shape[0] // block
        q = torch.stack((a.q.reshape(n, block, -1), b.q.reshape(n, block, -1)), 1).reshape(2 * a.shape[0], -1)
        sc = torch.stack((a.scale.reshape(n, block, -1), b.scale.reshape(n, block, -1)), 1).reshape(2 * a.shape[0], -1)
        return FP8Weight(q.contiguous(), sc.contiguous())

    @staticmethod
    def from_float(w: torch.Tensor) -> "FP8Weight":
        q, s = codec.quantize_mx_e4m3(w)
        return FP8Weight(q, s)


def _seed(seed: int, name: str) -> int:
    return int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") & ((1 << 63) - 1)


def _normal(shape, seed: int, name: str, device, std: float = STD) -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed(seed, name))
    return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * std


def _fp8(shape, seed, name, device, std=STD) -> FP8Weight:
    # Drawn in row pieces so a 17408 x 5120 matrix never needs a second full fp32 copy.
    rows, cols = shape
    piece = max(1, (1 << 26) // cols)
    qs, ss = [], []
    gen = torch.Generator(device=device)
    gen.manual_seed(_seed(seed, name))
    for first in range(0, rows, piece):
        n = min(piece, rows - first)
        w = torch.randn(n, cols, generator=gen, device=device, dtype=torch.float32) * std
        q, s = codec.quantize_mx_e4m3(w)
        qs.append(q)
        ss.append(s)
    return FP8Weight(torch.cat(qs), torch.cat(ss))


def _bf16(shape, seed, name, device, std=STD) -> torch.Tensor:
    return _normal(shape, seed, name, device, std).to(torch.bfloat16)


def synthetic_layer(cfg: TextConfig, index: int, seed: int = 0, device="cpu", std: float = STD) -> dict:
    """All of one decoder layer's weights, unsharded, named as the reference's parameters."""
    h, inter = cfg.hidden_size, cfg.intermediate_size
    p = f"layers.{index}"
    out = {
        f"{p}.input_layernorm_weight": _bf16((h,), seed, f"{p}.input_layernorm", device, std),
        f"{p}.post_attention_layernorm_weight": _bf16((h,), seed, f"{p}.post_attention_layernorm", device, std),
        f"{p}.mlp.gate_proj": _fp8((inter, h), seed, f"{p}.mlp.gate_proj", device, std),
        f"{p}.mlp.up_proj": _fp8((inter, h), seed, f"{p}.mlp.up_proj", device, std),
        f"{p}.mlp.down_proj": _fp8((h, inter), seed, f"{p}.mlp.down_proj", device, std),
    }
    if cfg.layer_types[index] == LINEAR:
        la = f"{p}.linear_attn"
        hv = cfg.linear_num_value_heads
        out |= {
            f"{la}.in_proj_qkv": _fp8((cfg.linear_conv_dim, h), seed, f"{la}.in_proj_qkv", device, std),
            f"{la}.in_proj_z": _fp8((cfg.linear_value_dim, h), seed, f"{la}.in_proj_z", device, std),
            f"{la}.out_proj": _fp8((h, cfg.linear_value_dim), seed, f"{la}.out_proj", device, std),
            f"{la}.in_proj_b": _bf16((hv, h), seed, f"{la}.in_proj_b", device, std),
            f"{la}.in_proj_a": _bf16((hv, h), seed, f"{la}.in_proj_a", device, std),
            f"{la}.conv_weight": _bf16((cfg.linear_conv_dim, cfg.linear_conv_kernel_dim), seed, f"{la}.conv1d", device, std),
            f"{la}.A_log": _bf16((hv,), seed, f"{la}.A_log", device, std),
            f"{la}.dt_bias": _bf16((hv,), seed, f"{la}.dt_bias", device, std),
            f"{la}.norm_weight": _bf16((cfg.linear_value_head_dim,), seed, f"{la}.norm", device, std),
        }
    elif cfg.layer_types[index] == FULL:
        sa = f"{p}.self_attn"
        hd = cfg.head_dim
        out |= {
            f"{sa}.q_proj": _fp8((cfg.num_attention_heads * hd * 2, h), seed, f"{sa}.q_proj", device, std),
            f"{sa}.k_proj": _fp8((cfg.num_key_value_heads * hd, h), seed, f"{sa}.k_proj", device, std),
            f"{sa}.v_proj": _fp8((cfg.num_key_value_heads * hd, h), seed, f"{sa}.v_proj", device, std),
            f"{sa}.o_proj": _fp8((h, cfg.num_attention_heads * hd), seed, f"{sa}.o_proj", device, std),
            f"{sa}.q_norm_weight": _bf16((hd,), seed, f"{sa}.q_norm", device, std),
            f"{sa}.k_norm_weight": _bf16((hd,), seed, f"{sa}.k_norm", device, std),
        }
    else:
        raise ValueError(f"unknown layer type {cfg.layer_types[index]}")
    return out


def synthetic_head(cfg: TextConfig, seed: int = 0, device="cpu", std: float = STD) -> dict:
    """Final norm and lm_head ``[vocab, hidden]``."""
    return {
        "norm_weight": _bf16((cfg.hidden_size,), seed, "model.norm", device, std),
        "lm_head": _fp8((cfg.vocab_size, cfg.hidden_size), seed, "lm_head", device, std),
    }


MTP_SEED_OFFSET = 7919  # the MTP layer's tensors draw from their own seeds


def synthetic_mtp(cfg: TextConfig, seed: int = 0, device="cpu", std: float = STD) -> dict:
    """The MTP draft layer's weights (MTPStep, qwen38_inf2/model.py:812-860; checkpoint.mtp_weights
    :363-393 names): fc [hidden, 2 hidden] over [normed embedding | normed hidden state], the four norms
    (final_norm_weight is the model's final norm, the head's norm_weight) and one full-attention decoder
    layer under `layers.0.`."""
    h = cfg.hidden_size
    layer_cfg = replace(cfg, layer_types=(FULL,))
    out = {
        "fc": _fp8((h, 2 * h), seed, "mtp.fc", device, std),
        "embedding_norm_weight": _bf16((h,), seed, "mtp.pre_fc_norm_embedding", device, std),
        "hidden_norm_weight": _bf16((h,), seed, "mtp.pre_fc_norm_hidden", device, std),
        "norm_weight": _bf16((h,), seed, "mtp.norm", device, std),
        "final_norm_weight": _bf16((h,), seed, "model.norm", device, std),
    }
    return out | synthetic_layer(layer_cfg, 0, seed + MTP_SEED_OFFSET, device, std)


def shard_mtp(cfg: TextConfig, weights: dict, rank: int, tp: int) -> dict:
    """One rank's share of the MTP layer: fc by input columns in `tp` equal slices of [embedding | hidden]
    (any TP degree; the reference's rank_gate split, model.py:835-850, holds only for 2), the decoder layer
    as any full-attention layer."""
    layer_cfg = replace(cfg, layer_types=(FULL,))
    out = {k: v for k, v in weights.items() if not k.startswith("layers.") and k != "fc"}
    out["fc"] = _cols(weights["fc"], rank, tp) if tp > 1 else weights["fc"]
    return out | shard_layer(layer_cfg, weights, 0, rank, tp)


def synthetic_kv_scales(cfg: TextConfig, index: int) -> tuple[float, float]:
    """Static FP8 KV-cache scales (k_scale, v_scale) of attention layer `index` for synthetic weights:
    powers of two that put normed keys (|k| up to ~5) and the values of N(0, 0.02) projections (|v| up
    to ~7) inside e4m3's range of +-240, as a checkpoint's calibrated scales would."""
    if cfg.layer_types[index] != FULL:
        raise ValueError(f"layer {index} has no KV cache")
    return 2.0 ** -4, 2.0 ** -5


def synthetic_embedding_table(cfg: TextConfig, seed: int = 0, device="cuda", std: float = STD) -> torch.Tensor:
    """A seeded N(0, std) embedding table [vocab, hidden] bf16 drawn on `device` in one piece (its values are
    not embedding_rows', which draws a generator per token on the CPU; serving loops that need every row
    on the GPU use this one)."""
    return _bf16((cfg.vocab_size, cfg.hidden_size), seed, "embed.table", device, std)


def embedding_rows(cfg: TextConfig, token_ids, seed: int = 0, std: float = STD) -> torch.Tensor:
    """Rows of a seeded N(0, std) embedding table ``[vocab, hidden]``, generated per token, bf16 on CPU."""
    rows = [_normal((cfg.hidden_size,), seed, f"embed.{int(t)}", "cpu", std) for t in token_ids]
    return torch.stack(rows).to(torch.bfloat16)


# ----------------------------------------------------------------------------------------------
# Tensor-parallel cut (qwen38_inf2/checkpoint.py:150-224)
# ----------------------------------------------------------------------------------------------
def _span(total: int, rank: int, tp: int) -> tuple[int, int]:
    size = total // tp
    return rank * size, (rank + 1) * size


def _rows(t, rank, tp):
    a, b = _span(t.shape[0], rank, tp)
    return t.rows(a, b) if isinstance(t, FP8Weight) else t[a:b]


def _cols(t: FP8Weight, rank, tp):
    a, b = _span(t.shape[1], rank, tp)
    return t.cols(a, b)


def _qkv_rows(t, cfg: TextConfig, rank: int, tp: int):
    kd, vd = cfg.linear_key_dim, cfg.linear_value_dim
    blocks = [(0, kd), (kd, 2 * kd), (2 * kd, 2 * kd + vd)]
    parts = []
    for first, last in blocks:
        a, b = _span(last - first, rank, tp)
        parts.append(t.rows(first + a, first + b) if isinstance(t, FP8Weight) else t[first + a : first + b])
    return FP8Weight.cat_rows(parts) if isinstance(t, FP8Weight) else torch.cat(parts)


def _kv_rows(t, cfg: TextConfig, rank: int, tp: int):
    hd = cfg.head_dim
    first = cfg.kv_head_of_rank(rank, tp)
    n = cfg.kv_heads_per_rank(tp)
    return t.rows(first * hd, (first + n) * hd)


def shard_layer(cfg: TextConfig, weights: dict, index: int, rank: int, tp: int) -> dict:
    """One rank's share of layer `index`'s weights (all names kept)."""
    p = f"layers.{index}"
    out = {}
    for name, t in weights.items():
        if not name.startswith(p + "."):
            continue
        leaf = name[len(p) + 1 :]
        if tp == 1 or leaf.endswith("norm_weight") or leaf in ("self_attn.k_scale", "self_attn.v_scale"):
            out[name] = t
        elif leaf in ("mlp.gate_proj", "mlp.up_proj", "linear_attn.in_proj_z", "linear_attn.in_proj_b",
                      "linear_attn.in_proj_a", "linear_attn.A_log", "linear_attn.dt_bias", "self_attn.q_proj"):
            out[name] = _rows(t, rank, tp)
        elif leaf in ("mlp.down_proj", "linear_attn.out_proj", "self_attn.o_proj"):
            out[name] = _cols(t, rank, tp)
        elif leaf in ("linear_attn.in_proj_qkv", "linear_attn.conv_weight"):
            out[name] = _qkv_rows(t, cfg, rank, tp)
        elif leaf in ("self_attn.k_proj", "self_attn.v_proj"):
            out[name] = _kv_rows(t, cfg, rank, tp)
        else:
            raise KeyError(f"no TP rule for {name}")
    return out


def shard_head(cfg: TextConfig, head: dict, rank: int, tp: int) -> dict:
    a, b = _span(cfg.vocab_size, rank, tp)
    return {"norm_weight": head["norm_weight"], "lm_head": head["lm_head"].rows(a, b)}


# ----------------------------------------------------------------------------------------------
# On-disk weights: this package's per-rank shards, and the reference's own per-rank files
# ----------------------------------------------------------------------------------------------
SHARD_BLOCK = 4  # layers per shard file, the model's repeat


def _flatten(weights: dict) -> dict:
    out = {}
    for name, t in weights.items():
        if isinstance(t, FP8Weight):
            out[f"{name}.q"], out[f"{name}.scale"] = t.q.contiguous(), t.scale.contiguous()
        else:
            out[name] = t.contiguous()
    return out


def _unflatten(tensors: dict) -> dict:
    out = {}
    for name, t in tensors.items():
        if name.endswith(".q"):
            base = name[:-2]
            out[base] = FP8Weight(t, tensors[base + ".scale"])
        elif not name.endswith(".scale"):
            out[name] = t
    return out


def shard_file(weights_dir, kind: str, rank: int, block: int | None = None):
    from pathlib import Path

    stem = f"b200_block{block:02d}_tp{rank}" if kind == "block" else f"b200_{kind}_tp{rank}"
    return Path(weights_dir) / f"{stem}.safetensors"


def write_rank_shards(cfg: TextConfig, layer_weights, head: dict, weights_dir, tp: int, mtp: dict | None = None) -> None:
    """This package's on-disk format: for every rank r of `tp`, its TP cut (shard_layer, shard_head,
    shard_mtp: e4m3 bytes [out, in] as <name>.q with fp32 power-of-two scales [out, in / 32] as
    <name>.scale, bf16 vectors) in b200_block{b}_tp{r} files of SHARD_BLOCK layers, b200_head_tp{r} and
    b200_mtp_tp{r}, and build_info.json. `layer_weights(i)` gives layer i's unsharded weights. Loading a
    rank reads only its own files (RankShards)."""
    import json
    from pathlib import Path

    from safetensors.torch import save_file

    d = Path(weights_dir)
    d.mkdir(parents=True, exist_ok=True)
    L = cfg.num_hidden_layers
    for b in range(0, L, SHARD_BLOCK):
        full = {}
        for i in range(b, min(L, b + SHARD_BLOCK)):
            full |= layer_weights(i)
        for r in range(tp):
            cut = {}
            for i in range(b, min(L, b + SHARD_BLOCK)):
                cut |= shard_layer(cfg, full, i, r, tp)
            save_file(_flatten(cut), str(shard_file(d, "block", r, b // SHARD_BLOCK)))
    for r in range(tp):
        save_file(_flatten(shard_head(cfg, head, r, tp)), str(shard_file(d, "head", r)))
        if mtp is not None:
            save_file(_flatten(shard_mtp(cfg, mtp, r, tp)), str(shard_file(d, "mtp", r)))
    (d / "build_info.json").write_text(json.dumps({"format": "b200 e4m3 + fp32 per-32 scales, [out, in]", "tp_degree": tp,
                                                   "layers": L, "block_layers": SHARD_BLOCK, "mtp": mtp is not None}))


class RankShards:
    """One rank's weights from write_rank_shards' files: `layer(i)` (that rank's cut of layer i, names as
    synthetic_layer's), `head()`, `mtp()`; pass them to B200Step / B200Head / B200MTP with presharded=True."""

    def __init__(self, weights_dir, rank: int):
        import json
        from pathlib import Path

        self.dir, self.rank = Path(weights_dir), rank
        self.info = json.loads((self.dir / "build_info.json").read_text())
        if not 0 <= rank < self.info["tp_degree"]:
            raise ValueError(f"rank {rank} outside the files' {self.info['tp_degree']} ranks")
        self._block, self._cache = None, {}

    def _load(self, path) -> dict:
        from safetensors.torch import load_file

        return _unflatten(load_file(str(path)))

    def layer(self, i: int) -> dict:
        b = i // self.info["block_layers"]
        if self._block != b:
            self._cache, self._block = self._load(shard_file(self.dir, "block", self.rank, b)), b
        p = f"layers.{i}."
        return {k: v for k, v in self._cache.items() if k.startswith(p)}

    def head(self) -> dict:
        return self._load(shard_file(self.dir, "head", self.rank))

    def mtp(self) -> dict:
        return self._load(shard_file(self.dir, "mtp", self.rank))


def _e5m2_to_e4m3(weight_fp8: torch.Tensor, name: str) -> FP8Weight:
    """A reference weight_fp8 matrix (e5m2 bytes [in, out], scale folded in) as e4m3 [out, in] with per-32
    power-of-two scales, exactly: the reference's weights are MXFP4 values times a power of two per group of
    32 inputs (checkpoint._fp4_weights, fp4.to_fp8), and a group spanning under 16 binades converts without
    rounding. A group that would round raises."""
    w = weight_fp8.view(torch.float8_e5m2).float().transpose(0, 1).contiguous()
    q, scale = codec.quantize_mx_e4m3(w)
    back = codec.dequantize_mx_e4m3(q, scale)
    if not torch.equal(back, w):
        bad = int((back != w).sum())
        raise ValueError(f"{name}: {bad} values of the reference's e5m2 weights do not convert to e4m3 exactly")
    return FP8Weight(q, scale)


def reference_rank_files(weights_dir, cfg: TextConfig, block_layers: int, tp_ref: int):
    """The reference's own per-rank files (checkpoint.write_rank_weights: block{b:02d}_tp{r}.safetensors,
    checkpoint.py:282-292, :405-413) as layer_weights(i) -> layer i's unsharded weights in this package's
    form: the ranks' cuts joined again by the reference's rules (rows of column-parallel matrices, columns
    of row-parallel ones, [q | k | v] block by block, checkpoint.py:165-224), each weight_fp8 converted
    exactly to e4m3 with per-32 scales; KV-cache scales, when the files hold them, under
    self_attn.k_scale / v_scale. Re-cut it for any TP degree with shard_layer."""
    from pathlib import Path

    from safetensors.torch import load_file

    d = Path(weights_dir)
    cache: dict = {}

    def rank_block(b: int, r: int) -> dict:
        if (b, r) not in cache:
            if len(cache) >= 2 * tp_ref:
                cache.clear()
            cache[(b, r)] = load_file(str(d / f"block{b:02d}_tp{r}.safetensors"))
        return cache[(b, r)]

    def layer(i: int) -> dict:
        b, off = divmod(i, block_layers)
        parts = [rank_block(b, r) for r in range(tp_ref)]
        src, dst = f"layers.{off}.", f"layers.{i}."
        names = sorted({k[len(src):] for k in parts[0] if k.startswith(src)})
        kd, vd = cfg.linear_key_dim // tp_ref, cfg.linear_value_dim // tp_ref
        out = {}
        for leaf in names:
            ts = [p[src + leaf] for p in parts]
            base = leaf[: -len(".weight_fp8")] if leaf.endswith(".weight_fp8") else leaf
            if base in ("mlp.down_proj", "linear_attn.out_proj", "self_attn.o_proj"):
                full = torch.cat(ts, dim=0)  # [in / t, out] pieces: row-parallel, cut by input
            elif base == "linear_attn.in_proj_qkv":
                full = torch.cat([torch.cat([t[:, j * kd:(j + 1) * kd] if j < 2 else t[:, 2 * kd:2 * kd + vd] for t in ts], 1)
                                  for j in range(3)], dim=1)
            elif base == "linear_attn.conv_weight":
                full = torch.cat([torch.cat([t[j * kd:(j + 1) * kd] if j < 2 else t[2 * kd:2 * kd + vd] for t in ts], 0)
                                  for j in range(3)], dim=0)
            elif leaf.endswith(".weight_fp8"):
                full = torch.cat(ts, dim=1)  # [in, out / t] pieces: column-parallel, cut by output
            elif base in ("linear_attn.in_proj_b", "linear_attn.in_proj_a", "linear_attn.A_log", "linear_attn.dt_bias"):
                full = torch.cat(ts, dim=0)
            else:
                full = ts[0]  # norms and KV-cache scales are the same on every rank
            out[dst + base] = _e5m2_to_e4m3(full, dst + base) if leaf.endswith(".weight_fp8") else full
        return out

    return layer
