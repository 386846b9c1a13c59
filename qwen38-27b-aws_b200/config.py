"""Model shapes, mirroring the reference's TextConfig (qwen38_inf2/config.py:11-130).

Field names and derived sizes are the reference's, so a reference caller's config maps one to one.
Two differences, both for tensor parallelism on 8 GPUs: `kv_heads_per_rank` replicates the 4 KV
heads when tp_degree exceeds them (rank r uses KV head r // (tp / kv_heads)), which the reference's
`validate_tp` rejects (config.py:64-83), and `validate_tp` here checks FP8 group (32) boundaries of
the row-parallel inputs instead of FP4 ones, which is the same rule.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, replace
from pathlib import Path

LINEAR = "linear_attention"
FULL = "full_attention"


@dataclass(frozen=True)
class TextConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    layer_types: tuple[str, ...]
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    rms_norm_eps: float
    rope_theta: float
    partial_rotary_factor: float
    weight_format: str = "fp8"
    recurrent_state_format: str = "bf16"
    kv_cache_format: str = "bf16"

    @property
    def num_hidden_layers(self) -> int:
        return len(self.layer_types)

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def linear_key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def linear_value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def linear_conv_dim(self) -> int:
        return 2 * self.linear_key_dim + self.linear_value_dim

    @property
    def num_key_value_groups(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    @property
    def linear_key_repeat(self) -> int:
        return self.linear_num_value_heads // self.linear_num_key_heads

    def kv_heads_per_rank(self, tp_degree: int) -> int:
        return max(1, self.num_key_value_heads // tp_degree)

    def kv_head_of_rank(self, rank: int, tp_degree: int) -> int:
        """First KV head a rank holds. With more ranks than KV heads, neighbours share (replicate) one."""
        if tp_degree <= self.num_key_value_heads:
            return rank * (self.num_key_value_heads // tp_degree)
        return rank // (tp_degree // self.num_key_value_heads)

    def validate_tp(self, tp_degree: int) -> None:
        """Every split lands on a head boundary and a 32-element FP8 scale-group boundary."""
        must_divide = {
            "linear_num_key_heads": self.linear_num_key_heads,
            "linear_num_value_heads": self.linear_num_value_heads,
            "num_attention_heads": self.num_attention_heads,
            "intermediate_size": self.intermediate_size,
            "vocab_size": self.vocab_size,
        }
        for name, value in must_divide.items():
            if value % tp_degree:
                raise ValueError(f"{name}={value} is not divisible by tp_degree={tp_degree}")
        kv = self.num_key_value_heads
        if kv % tp_degree and tp_degree % kv:
            raise ValueError(f"num_key_value_heads={kv} neither divides nor is divided by tp_degree={tp_degree}")
        for name, cols in {
            "mlp.down_proj": self.intermediate_size,
            "linear_attn.out_proj": self.linear_value_dim,
            "self_attn.o_proj": self.num_attention_heads * self.head_dim,
        }.items():
            if cols % (32 * tp_degree):
                raise ValueError(f"{name} input width {cols} does not split on 32-wide scale groups at tp_degree={tp_degree}")
        if (self.vocab_size // tp_degree) % 32:
            raise ValueError(f"vocab slice {self.vocab_size // tp_degree} is not a whole number of 32-token groups")

    @classmethod
    def from_model_config(cls, config: dict) -> "TextConfig":
        text = config.get("text_config", config)
        rope = text.get("rope_parameters", text)
        return cls(
            vocab_size=text["vocab_size"],
            hidden_size=text["hidden_size"],
            intermediate_size=text["intermediate_size"],
            layer_types=tuple(text["layer_types"]),
            num_attention_heads=text["num_attention_heads"],
            num_key_value_heads=text["num_key_value_heads"],
            head_dim=text["head_dim"],
            linear_num_key_heads=text["linear_num_key_heads"],
            linear_num_value_heads=text["linear_num_value_heads"],
            linear_key_head_dim=text["linear_key_head_dim"],
            linear_value_head_dim=text["linear_value_head_dim"],
            linear_conv_kernel_dim=text["linear_conv_kernel_dim"],
            rms_norm_eps=text["rms_norm_eps"],
            rope_theta=rope["rope_theta"],
            partial_rotary_factor=rope["partial_rotary_factor"],
        )

    @classmethod
    def from_file(cls, path: str | Path) -> "TextConfig":
        return cls.from_model_config(json.loads(Path(path).read_text()))


def full_config(num_blocks: int = 16) -> TextConfig:
    """The Qwen3.8-27B text decoder: 16 repeats of 3 gated-delta layers and 1 attention layer."""
    return TextConfig(
        vocab_size=248320,
        hidden_size=5120,
        intermediate_size=17408,
        layer_types=(LINEAR, LINEAR, LINEAR, FULL) * num_blocks,
        num_attention_heads=24,
        num_key_value_heads=4,
        head_dim=256,
        linear_num_key_heads=16,
        linear_num_value_heads=48,
        linear_key_head_dim=128,
        linear_value_head_dim=128,
        linear_conv_kernel_dim=4,
        rms_norm_eps=1e-6,
        rope_theta=10000000.0,
        partial_rotary_factor=0.25,
    )


def tiny_config(num_blocks: int = 2) -> TextConfig:
    """The reference's test shape (qwen38_inf2/config.py:112-130): same ratios, CPU-sized."""
    return TextConfig(
        vocab_size=128,
        hidden_size=128,
        intermediate_size=256,
        layer_types=(LINEAR, LINEAR, LINEAR, FULL) * num_blocks,
        num_attention_heads=6,
        num_key_value_heads=2,
        head_dim=32,
        linear_num_key_heads=2,
        linear_num_value_heads=6,
        linear_key_head_dim=32,
        linear_value_head_dim=32,
        linear_conv_kernel_dim=4,
        rms_norm_eps=1e-6,
        rope_theta=10000000.0,
        partial_rotary_factor=0.25,
    )


def block_config(cfg: TextConfig, block_layers: int = 4) -> TextConfig:
    return replace(cfg, layer_types=cfg.layer_types[:block_layers])
