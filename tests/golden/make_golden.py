"""Generates the golden vectors under tests/golden/ by running the reference itself.

Run in a checkout of the reference (read-only is fine), never on the GPU box:

    python tests/golden/make_golden.py --reference /path/to/reference

The reference's `Qwen38Step` and `HeadStep` run their CPU branches on seeded synthetic weights
(weights.synthetic_layer, tiny config). The one change is the weight codec, swapped the way the
reference's own test swaps `fp8_round` (tests/test_model_parity.py:255-257): `FP8Linear.forward`
decodes e4m3 bytes with per-32 power-of-two scales instead of scale-free e5m2 bytes, and keeps the
reference's e5m2 rounding of the input and its BF16 matmul. Weights are not stored: the fixture holds
their seed and a SHA-256 of their bytes, and the tests regenerate them.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import sys
from dataclasses import replace
from pathlib import Path

import torch
import torch.nn.functional as F
from safetensors.torch import save_file

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
pkg = importlib.import_module("qwen38-27b-aws_b200")

SEED = 7
STD = 0.1  # larger than the model's 0.02 so a 4-layer tiny block is far from linear
BATCH = 3
MAX_SEQ = 64
CHUNK = 16
VERIFY = 4  # tokens per verify step


def weights_digest(weights: dict) -> str:
    h = hashlib.sha256()
    for name in sorted(weights):
        t = weights[name]
        parts = (t.q, t.scale) if isinstance(t, pkg.weights.FP8Weight) else (t,)
        for p in parts:
            h.update(name.encode())
            h.update(p.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def tiny_weights(cfg) -> dict:
    out = {}
    for i in range(cfg.num_hidden_layers):
        out |= pkg.weights.synthetic_layer(cfg, i, SEED, "cpu", STD)
    return out


def decode_schedule():
    """(positions, active) per decode step, exercising fresh rows, idle rows and a refill."""
    return [
        ([0, 0, 5], [1, 0, 1]),
        ([1, 0, 6], [1, 1, 1]),
        ([2, 1, 7], [1, 1, 0]),
        ([3, 2, 7], [1, 1, 1]),
        ([0, 3, 8], [1, 1, 1]),  # row 0 starts a new sequence: its state must clear
        ([1, 4, 9], [1, 1, 1]),
    ]


def verify_schedule():
    """(positions, active, accepted) per verify step: the first after decode commits nothing; then rows
    accept different counts, a row idles, and a row starts a new sequence (its states must clear)."""
    return [
        ([2, 2, 2], [1, 1, 1], [0, 0, 0]),
        ([4, 6, 3], [1, 1, 1], [2, 4, 1]),
        ([7, 7, 3], [1, 1, 0], [3, 1, 0]),
        ([0, 9, 3], [1, 1, 1], [0, 2, 0]),
        ([1, 12, 5], [1, 1, 1], [1, 3, 2]),
    ]


def build_model(rmodel, ref_cfg, weights, verify_tokens=0):
    """The reference's Qwen38Step on CPU with the synthetic weights loaded (FP8 linears through the
    swapped codec of `fp8_forward` in main)."""
    model = rmodel.Qwen38Step(ref_cfg, MAX_SEQ, tp_degree=1, dtype=torch.bfloat16, batch_size=BATCH,
                              verify_tokens=verify_tokens).eval()
    plain = {}
    for name, t in weights.items():
        if isinstance(t, pkg.weights.FP8Weight):
            model.get_submodule(name)._b200_weight = t.dequant()
        else:
            plain[name] = t
    missing, unexpected = model.load_state_dict(plain, strict=False)
    assert not unexpected, unexpected
    assert all(n.endswith(("weight_fp8", "_cache", "_state")) for n in missing), missing
    return model


def verify_goldens(rgen, ref_cfg, model, ours):
    """Two decode steps, then the verify schedule, then a decode step; every output and the final buffers
    (recurrent, conv and pending states, KV caches) into tiny_verify.safetensors."""
    tensors: dict[str, torch.Tensor] = {}
    gen = torch.Generator().manual_seed(SEED + 1)
    with torch.no_grad():
        for step in range(2):
            x = torch.randn(BATCH, 1, ours.hidden_size, generator=gen).to(torch.bfloat16)
            inputs = rgen.batch_step_inputs(ref_cfg, [step] * BATCH, MAX_SEQ, torch.bfloat16, [True] * BATCH)
            tensors[f"decode{step}.x"] = x
            tensors.update({f"decode{step}.{k}": v for k, v in inputs.items()})
            tensors[f"decode{step}.y"] = model(inputs_embeds=x, **inputs)
        for step, (positions, active, accepted) in enumerate(verify_schedule()):
            x = torch.randn(BATCH, VERIFY, ours.hidden_size, generator=gen).to(torch.bfloat16)
            inputs = rgen.verify_inputs(ref_cfg, positions, VERIFY, MAX_SEQ, torch.bfloat16, [bool(a) for a in active],
                                        accepted)
            tensors[f"verify{step}.x"] = x
            tensors.update({f"verify{step}.{k}": v for k, v in inputs.items()})
            tensors[f"verify{step}.y"] = model(inputs_embeds=x, **inputs)
        x = torch.randn(BATCH, 1, ours.hidden_size, generator=gen).to(torch.bfloat16)
        inputs = rgen.batch_step_inputs(ref_cfg, [2, 15, 7], MAX_SEQ, torch.bfloat16, [True] * BATCH)
        tensors["after.x"] = x
        tensors.update({f"after.{k}": v for k, v in inputs.items()})
        tensors["after.y"] = model(inputs_embeds=x, **inputs)
        for name, buf in model.named_buffers():
            tensors[f"state.{name}"] = buf.clone()
    return tensors


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference (contains qwen38_inf2/)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    rconfig = importlib.import_module("qwen38_inf2.config")
    rmodel = importlib.import_module("qwen38_inf2.model")
    rgen = importlib.import_module("qwen38_inf2.generate")

    ours = pkg.config.tiny_config(num_blocks=1)
    ref_cfg = replace(rconfig.tiny_config(num_blocks=1), weight_format="fp8", recurrent_state_format="bf16", kv_cache_format="bf16")
    assert ref_cfg.layer_types == ours.layer_types and ref_cfg.hidden_size == ours.hidden_size
    weights = tiny_weights(ours)

    def fp8_forward(self, x):
        # The reference's CPU branch (model.py:222-225) with the weight decode swapped to e4m3 * 2^s.
        x = rmodel.fp8_round(x)
        return F.linear(x, self._b200_weight.to(x.dtype))

    rmodel.FP8Linear.forward = fp8_forward
    model = build_model(rmodel, ref_cfg, weights)

    tensors: dict[str, torch.Tensor] = {}
    gen = torch.Generator().manual_seed(SEED)
    with torch.no_grad():
        for step, (positions, active) in enumerate(decode_schedule()):
            x = (torch.randn(BATCH, 1, ours.hidden_size, generator=gen)).to(torch.bfloat16)
            inputs = rgen.batch_step_inputs(ref_cfg, positions, MAX_SEQ, torch.bfloat16, [bool(a) for a in active])
            y = model(inputs_embeds=x, **inputs)
            tensors[f"decode{step}.x"] = x
            for k, v in inputs.items():
                tensors[f"decode{step}.{k}"] = v
            tensors[f"decode{step}.y"] = y
        # A prompt prefilled into slot 1 in two chunks (the second partial), then decode for all rows.
        for c, (start, n_valid) in enumerate([(0, CHUNK), (CHUNK, 11)]):
            x = torch.randn(1, CHUNK, ours.hidden_size, generator=gen).to(torch.bfloat16)
            inputs = rgen.prefill_inputs(ref_cfg, 1, start, n_valid, CHUNK, torch.bfloat16)
            y = model(inputs_embeds=x, **inputs)
            tensors[f"prefill{c}.x"] = x
            for k, v in inputs.items():
                tensors[f"prefill{c}.{k}"] = v
            tensors[f"prefill{c}.y"] = y
        x = torch.randn(BATCH, 1, ours.hidden_size, generator=gen).to(torch.bfloat16)
        inputs = rgen.batch_step_inputs(ref_cfg, [2, CHUNK + 11, 10], MAX_SEQ, torch.bfloat16, [True, True, True])
        y = model(inputs_embeds=x, **inputs)
        tensors["after.x"] = x
        for k, v in inputs.items():
            tensors[f"after.{k}"] = v
        tensors["after.y"] = y
        for name, buf in model.named_buffers():
            tensors[f"state.{name}"] = buf.clone()

        # Head: HeadStep's CPU branch with the lm_head decoded the same way.
        head = pkg.weights.synthetic_head(ours, SEED, "cpu", STD)
        hstep = rmodel.HeadStep(ref_cfg, 1, BATCH, group_rows=32, head_format="bf16").eval()
        hstep.norm_weight.data = head["norm_weight"]
        hstep.lm_head.data = head["lm_head"].dequant().to(torch.bfloat16).transpose(0, 1).contiguous()
        hstep.rank_gate.data = torch.ones(1)
        hidden = torch.randn(BATCH, 1, ours.hidden_size, generator=gen).to(torch.bfloat16)
        tensors["head.hidden"] = hidden
        tensors["head.maxima"] = hstep(hidden)

        # Kernel-level pins of the chunked delta rule (model.py:90-128) and attention blocks (:170-191).
        heads, tokens, dim = 2, 64, 16
        q = F.normalize(torch.randn(heads, tokens, dim, generator=gen), dim=-1) / dim**0.5
        k = F.normalize(torch.randn(heads, tokens, dim, generator=gen), dim=-1)
        v = torch.randn(heads, tokens, dim, generator=gen)
        g = -torch.rand(heads, tokens, generator=gen) * 0.5
        b = torch.rand(heads, tokens, generator=gen)
        s0 = torch.randn(heads, dim, dim, generator=gen)
        out, s1 = rmodel.chunked_gated_delta(q, k, v, g, b, s0, chunk=32)
        for name, t in dict(q=q, k=k, v=v, g=g, b=b, s0=s0, out=out, s1=s1).items():
            tensors[f"delta.{name}"] = t
        lower = -torch.tril(torch.randn(2, 32, 32, generator=gen) * 0.3, diagonal=-1)
        tensors["inverse.lower"] = lower
        tensors["inverse.out"] = rmodel.unit_lower_inverse(lower)
        qa = torch.randn(2, 12, 16, generator=gen).to(torch.bfloat16)
        ka = torch.randn(2, 40, 16, generator=gen).to(torch.bfloat16)
        va = torch.randn(2, 40, 16, generator=gen).to(torch.bfloat16)
        vis = torch.rand(12, 40, generator=gen) > 0.3
        vis[:, 0] = True
        tensors.update({"attn.q": qa, "attn.k": ka, "attn.v": va, "attn.visible": vis, "attn.out": rmodel.blocked_attention(qa, ka, va, vis, 16)})

    meta = {"seed": str(SEED), "std": str(STD), "batch": str(BATCH), "max_seq": str(MAX_SEQ), "chunk": str(CHUNK),
            "weights_sha256": weights_digest(weights), "head_sha256": weights_digest(head),
            "decode_steps": str(len(decode_schedule())), "generator": "tests/golden/make_golden.py"}
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(HERE / "tiny_block.safetensors"), metadata=meta)
    print(json.dumps(meta, indent=1))
    print(f"{len(tensors)} tensors, {(HERE / 'tiny_block.safetensors').stat().st_size} bytes")

    vtensors = verify_goldens(rgen, ref_cfg, build_model(rmodel, ref_cfg, weights, VERIFY), ours)
    vmeta = dict(meta, verify_tokens=str(VERIFY), verify_steps=str(len(verify_schedule())))
    del vmeta["decode_steps"], vmeta["chunk"]
    save_file({k: v.contiguous() for k, v in vtensors.items()}, str(HERE / "tiny_verify.safetensors"), metadata=vmeta)
    print(f"{len(vtensors)} tensors, {(HERE / 'tiny_verify.safetensors').stat().st_size} bytes")


if __name__ == "__main__":
    main()
