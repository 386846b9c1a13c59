"""The reference's own CPU step (from oracle/_ref, see build_ref.py) on synthetic weights: test and
baseline infrastructure, never the product.

`reference_block(cfg, batch, max_seq)` builds the reference's Qwen38Step for one full-width 4-layer block
with the weights of weights.synthetic_layer and the one codec swap BASELINE asks for, made the way the
reference's own test swaps `fp8_round` (tests/test_model_parity.py:255-257): FP8Linear.forward decodes
e4m3 bytes with per-32 power-of-two scales, keeping the reference's e5m2 input rounding and BF16 matmul
(model.py:222-225). `reference_head` builds its HeadStep (CPU branch, BF16 lm_head) the same way.
"""

from __future__ import annotations

import importlib
import sys
from dataclasses import fields
from pathlib import Path

import torch
import torch.nn.functional as F

REF = Path(__file__).resolve().parent / "_ref"
_pkg = importlib.import_module("qwen38-27b-aws_b200")


def available() -> bool:
    return (REF / "qwen38_inf2" / "model.py").is_file()


def _modules():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    rconfig = importlib.import_module("qwen38_inf2.config")
    rmodel = importlib.import_module("qwen38_inf2.model")
    rgen = importlib.import_module("qwen38_inf2.generate")

    def fp8_forward(self, x):
        x = rmodel.fp8_round(x)
        return F.linear(x, self._b200_weight.to(x.dtype))

    rmodel.FP8Linear.forward = fp8_forward
    return rconfig, rmodel, rgen


def ref_config(rconfig, cfg):
    names = [f.name for f in fields(rconfig.TextConfig) if f.name not in ("weight_format", "recurrent_state_format",
                                                                         "kv_cache_format")]
    return rconfig.TextConfig(**{n: getattr(cfg, n) for n in names}, weight_format="fp8", recurrent_state_format="bf16",
                              kv_cache_format="bf16")


def reference_block(cfg, batch: int, max_seq: int, seed: int = 0):
    """(the reference's Qwen38Step for cfg's layers, its config, its generate module)."""
    rconfig, rmodel, rgen = _modules()
    rcfg = ref_config(rconfig, cfg)
    model = rmodel.Qwen38Step(rcfg, max_seq, tp_degree=1, dtype=torch.bfloat16, batch_size=batch).eval()
    plain = {}
    for i in range(cfg.num_hidden_layers):
        for name, t in _pkg.weights.synthetic_layer(cfg, i, seed, "cpu").items():
            if isinstance(t, _pkg.weights.FP8Weight):
                model.get_submodule(name)._b200_weight = t.dequant()
            else:
                plain[name] = t
    model.load_state_dict(plain, strict=False)
    return model, rcfg, rgen


def reference_head(cfg, batch: int, seed: int = 0):
    """The reference's HeadStep (CPU branch) over the whole vocabulary with the synthetic lm_head."""
    rconfig, rmodel, _ = _modules()
    head = _pkg.weights.synthetic_head(cfg, seed, "cpu")
    hstep = rmodel.HeadStep(ref_config(rconfig, cfg), 1, batch, group_rows=32, head_format="bf16").eval()
    hstep.norm_weight.data = head["norm_weight"]
    hstep.lm_head.data = head["lm_head"].dequant().to(torch.bfloat16).transpose(0, 1).contiguous()
    hstep.rank_gate.data = torch.ones(1)
    return hstep
