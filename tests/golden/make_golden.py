"""Generates the golden vectors under tests/golden/ by running the reference itself.

Run in a checkout of the reference (read-only is fine), never on the GPU box:

    python tests/golden/make_golden.py --reference /path/to/reference [--full-width]

--full-width writes full_block.safetensors instead: BASELINE config 0 at full width (one 4-layer block,
batch 8, rows at positions uniform in [0, 512) over seeded cache and state contents), two greedy
decode steps through the reference's Qwen38Step, HeadStep maxima over the whole 248,320-token vocabulary
and ChipHead.next_tokens (the exact top-4 recheck). It takes a few minutes and ~20 GB of host memory.

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
    assert all(n.endswith(("weight_fp8", "_cache", "_state", "_scale")) for n in missing), missing
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


FP8_SCALES = (2.0 ** -5, 2.0 ** -6)  # k_scale, v_scale: the value scale clamps the largest values at 240


def fp8_cache_goldens(rconfig, rmodel, rgen, ours, weights):
    """The FP8 e4m3 KV cache (kv_cache_format "fp8", model.py:579-608): decode steps with fresh and idle
    rows, a prefill chunk, a decode step, then a verify model's decode and verify steps, every output and
    the final caches, into tiny_fp8.safetensors."""
    tensors: dict[str, torch.Tensor] = {}
    gen = torch.Generator().manual_seed(SEED + 2)
    for verify in (0, VERIFY):
        ref_cfg = replace(rconfig.tiny_config(num_blocks=1), weight_format="fp8", recurrent_state_format="bf16",
                          kv_cache_format="fp8")
        model = build_model(rmodel, ref_cfg, weights, verify)
        for layer in model.layers:
            if hasattr(layer, "self_attn"):
                layer.self_attn.k_scale.data.fill_(FP8_SCALES[0])
                layer.self_attn.v_scale.data.fill_(FP8_SCALES[1])
        tag = "v" if verify else "d"
        calls = []
        if not verify:
            for step, (positions, active) in enumerate(decode_schedule()[:4]):
                calls.append((f"{tag}decode{step}", BATCH, rgen.batch_step_inputs(ref_cfg, positions, MAX_SEQ, torch.bfloat16,
                                                                                   [bool(a) for a in active])))
            calls.append((f"{tag}prefill", 1, rgen.prefill_inputs(ref_cfg, 2, 9, CHUNK, CHUNK, torch.bfloat16)))
            calls.append((f"{tag}after", BATCH, rgen.batch_step_inputs(ref_cfg, [4, 3, CHUNK + 9], MAX_SEQ, torch.bfloat16,
                                                                        [True] * BATCH)))
        else:
            for step in range(2):
                calls.append((f"{tag}decode{step}", BATCH, rgen.batch_step_inputs(ref_cfg, [step] * BATCH, MAX_SEQ, torch.bfloat16,
                                                                                   [True] * BATCH)))
            for step, (positions, active, accepted) in enumerate(verify_schedule()):
                calls.append((f"{tag}verify{step}", BATCH, rgen.verify_inputs(ref_cfg, positions, VERIFY, MAX_SEQ, torch.bfloat16,
                                                                               [bool(a) for a in active], accepted)))
        with torch.no_grad():
            for name, rows, inputs in calls:
                width = VERIFY if "verify" in name else (CHUNK if "prefill" in name else 1)
                x = torch.randn(rows, width, ours.hidden_size, generator=gen).to(torch.bfloat16)
                tensors[f"{name}.x"] = x
                tensors.update({f"{name}.{k}": v for k, v in inputs.items()})
                tensors[f"{name}.y"] = model(inputs_embeds=x, **inputs)
            for bname, buf in model.named_buffers():
                if "_cache" in bname:
                    tensors[f"{tag}state.{bname}"] = buf.clone()
        tensors[f"{tag}calls"] = torch.tensor([len(calls)])
    return tensors


MTP_TOKENS = 4


def mtp_goldens(rconfig, rmodel, rgen, ours):
    """The MTP draft layer (MTPStep, model.py:812-860) with synthetic weights: a prompt chunk into slot 1
    (which only fills its cache), then two steps of MTP_TOKENS tokens per row from each row's MTP index,
    the second feeding its own outputs back, into tiny_mtp.safetensors."""
    ref_cfg = replace(rconfig.tiny_config(num_blocks=1), weight_format="fp8", recurrent_state_format="bf16",
                      kv_cache_format="bf16")
    weights = pkg.weights.synthetic_mtp(ours, SEED, "cpu", STD)
    mtp = rmodel.MTPStep(ref_cfg, 1, MAX_SEQ, torch.bfloat16, rmodel.identity_all_reduce, BATCH).eval()
    plain = {}
    for name, t in weights.items():
        ref_name = ("layer." + name[len("layers.0."):]) if name.startswith("layers.0.") else name
        if isinstance(t, pkg.weights.FP8Weight):
            mtp.get_submodule(ref_name)._b200_weight = t.dequant()
        else:
            plain[ref_name] = t
    missing, unexpected = mtp.load_state_dict(plain, strict=False)
    assert not unexpected, unexpected
    assert all(n.endswith(("weight_fp8", "_cache")) for n in missing), missing
    tensors = {}
    gen = torch.Generator().manual_seed(SEED + 3)
    with torch.no_grad():
        hidden = torch.randn(1, CHUNK, ours.hidden_size, generator=gen).to(torch.bfloat16)
        embeds = torch.randn(1, CHUNK, ours.hidden_size, generator=gen).to(torch.bfloat16)
        inputs = rgen.mtp_prefill_inputs(ref_cfg, 1, 0, CHUNK, CHUNK, torch.bfloat16)
        tensors.update({"prefill.hidden": hidden, "prefill.x": embeds} | {f"prefill.{k}": v for k, v in inputs.items()})
        tensors["prefill.y"] = mtp(hidden=hidden, inputs_embeds=embeds, **inputs)
        hidden = torch.randn(BATCH, MTP_TOKENS, ours.hidden_size, generator=gen).to(torch.bfloat16)
        for step, (indices, active) in enumerate([([3, CHUNK, 7], [True, True, False]), ([4, CHUNK + 2, 1], [True, True, True])]):
            embeds = torch.randn(BATCH, MTP_TOKENS, ours.hidden_size, generator=gen).to(torch.bfloat16)
            inputs = rgen.mtp_step_inputs(ref_cfg, indices, MTP_TOKENS, MAX_SEQ, torch.bfloat16, active)
            tensors.update({f"step{step}.hidden": hidden, f"step{step}.x": embeds} | {f"step{step}.{k}": v for k, v in inputs.items()})
            hidden = mtp(hidden=hidden, inputs_embeds=embeds, **inputs)
            tensors[f"step{step}.y"] = hidden.clone()
        tensors["state.k_cache"] = mtp.layer.self_attn.k_cache.clone()
        tensors["state.v_cache"] = mtp.layer.self_attn.v_cache.clone()
    meta = {"seed": str(SEED), "std": str(STD), "batch": str(BATCH), "max_seq": str(MAX_SEQ), "chunk": str(CHUNK),
            "tokens": str(MTP_TOKENS), "steps": "2", "weights_sha256": weights_digest(weights),
            "generator": "tests/golden/make_golden.py"}
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(HERE / "tiny_mtp.safetensors"), metadata=meta)
    print(f"{len(tensors)} tensors, {(HERE / 'tiny_mtp.safetensors').stat().st_size} bytes")


FULL_BATCH = 8
FULL_MAX_SEQ = 512
FULL_STATE_SEED = 1
FULL_STEPS = 2


def full_width_states(cfg, batch: int = FULL_BATCH, max_seq: int = FULL_MAX_SEQ, seed: int = FULL_STATE_SEED):
    """Seeded recurrent states and KV caches for a full-width block, in layer order: per gated-delta layer
    (recurrent state N(0, 0.1) [batch, heads, dk, dv], conv state N(0, 1) [batch, conv_dim, kernel - 1]),
    per attention layer (k_cache, v_cache N(0, 1) [batch, kv_heads, max_seq, head_dim]), all bf16."""
    gen = torch.Generator().manual_seed(seed)
    out = []
    for kind in cfg.layer_types:
        if kind == pkg.config.LINEAR:
            st = torch.randn(batch, cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim,
                             generator=gen) * 0.1
            conv = torch.randn(batch, cfg.linear_conv_dim, cfg.linear_conv_kernel_dim - 1, generator=gen)
            out.append((st.to(torch.bfloat16), conv.to(torch.bfloat16)))
        else:
            shape = (batch, cfg.num_key_value_heads, max_seq, cfg.head_dim)
            out.append((torch.randn(shape, generator=gen).to(torch.bfloat16), torch.randn(shape, generator=gen).to(torch.bfloat16)))
    return out


def full_width_schedule(cfg):
    """Step 0's token ids and positions (seed 0), as BASELINE config 0 draws them."""
    gen = torch.Generator().manual_seed(0)
    position = torch.randint(0, FULL_MAX_SEQ - FULL_STEPS, (FULL_BATCH,), generator=gen, dtype=torch.int32)
    tokens = torch.randint(0, cfg.vocab_size, (FULL_BATCH,), generator=gen)
    return tokens.tolist(), position


def full_width_golden(rconfig, rmodel, rgen, rcheckpoint):
    ours = pkg.config.full_config(num_blocks=1)
    fields = ("vocab_size", "hidden_size", "intermediate_size", "layer_types", "num_attention_heads",
              "num_key_value_heads", "head_dim", "linear_num_key_heads", "linear_num_value_heads", "linear_key_head_dim",
              "linear_value_head_dim", "linear_conv_kernel_dim", "rms_norm_eps", "rope_theta", "partial_rotary_factor")
    ref_cfg = rconfig.TextConfig(**{f: getattr(ours, f) for f in fields}, weight_format="fp8",
                                 recurrent_state_format="bf16", kv_cache_format="bf16")
    weights = {}
    for i in range(ours.num_hidden_layers):
        weights |= pkg.weights.synthetic_layer(ours, i, 0, "cpu")
    model = rmodel.Qwen38Step(ref_cfg, FULL_MAX_SEQ, tp_degree=1, dtype=torch.bfloat16, batch_size=FULL_BATCH).eval()
    plain = {}
    for name, t in weights.items():
        if isinstance(t, pkg.weights.FP8Weight):
            model.get_submodule(name)._b200_weight = t.dequant()
        else:
            plain[name] = t
    model.load_state_dict(plain, strict=False)
    for layer, (a, b) in zip(model.layers, full_width_states(ours)):
        if hasattr(layer, "linear_attn"):
            layer.linear_attn.recurrent_state = a.clone()
            layer.linear_attn.conv_state = b.clone()
        else:
            layer.self_attn.k_cache = a.clone()
            layer.self_attn.v_cache = b.clone()
    head = pkg.weights.synthetic_head(ours, 0, "cpu")
    lm_rows = head["lm_head"].dequant().to(torch.bfloat16)  # e4m3 x 2^s: exact in bf16
    hstep = rmodel.HeadStep(ref_cfg, 1, FULL_BATCH, group_rows=32, head_format="bf16").eval()
    hstep.norm_weight.data = head["norm_weight"]
    hstep.lm_head.data = lm_rows.transpose(0, 1).contiguous()
    hstep.rank_gate.data = torch.ones(1)
    source = rcheckpoint.DictSource({rcheckpoint.FINAL_NORM: head["norm_weight"], rcheckpoint.LM_HEAD: lm_rows})
    chip = rgen.ChipHead(source, ours.rms_norm_eps, lambda hidden: hstep(hidden), FULL_BATCH)

    tensors = {}
    tokens, position = full_width_schedule(ours)
    with torch.no_grad():
        for step in range(FULL_STEPS):
            x = pkg.weights.embedding_rows(ours, tokens).reshape(FULL_BATCH, 1, -1)
            inputs = rgen.batch_step_inputs(ref_cfg, (position + step).tolist(), FULL_MAX_SEQ, torch.bfloat16,
                                            [True] * FULL_BATCH)
            y = model(inputs_embeds=x, **inputs)
            maxima = hstep(y)
            tensors[f"step{step}.tokens_in"] = torch.tensor(tokens, dtype=torch.int64)
            tensors[f"step{step}.x"] = x
            tensors.update({f"step{step}.{k}": v for k, v in inputs.items()})
            tensors[f"step{step}.y"] = y
            tensors[f"step{step}.maxima"] = maxima
            tensors[f"step{step}.top4"] = maxima.float().topk(4, dim=-1).indices
            tokens = chip.next_tokens(y)
            tensors[f"step{step}.tokens_out"] = torch.tensor(tokens, dtype=torch.int64)
    meta = {"seed": "0", "std": str(pkg.weights.STD), "batch": str(FULL_BATCH), "max_seq": str(FULL_MAX_SEQ),
            "state_seed": str(FULL_STATE_SEED), "steps": str(FULL_STEPS), "weights_sha256": weights_digest(weights),
            "head_sha256": weights_digest(head), "generator": "tests/golden/make_golden.py --full-width"}
    path = HERE / "full_block.safetensors"
    save_file({k: v.contiguous() for k, v in tensors.items()}, str(path), metadata=meta)
    print(json.dumps(meta, indent=1))
    print(f"{len(tensors)} tensors, {path.stat().st_size} bytes")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference (contains qwen38_inf2/)")
    ap.add_argument("--full-width", action="store_true", help="write full_block.safetensors (config 0 at full width)")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    rconfig = importlib.import_module("qwen38_inf2.config")
    rmodel = importlib.import_module("qwen38_inf2.model")
    rgen = importlib.import_module("qwen38_inf2.generate")

    def fp8_forward(self, x):
        # The reference's CPU branch (model.py:222-225) with the weight decode swapped to e4m3 * 2^s.
        x = rmodel.fp8_round(x)
        return F.linear(x, self._b200_weight.to(x.dtype))

    rmodel.FP8Linear.forward = fp8_forward
    if args.full_width:
        full_width_golden(rconfig, rmodel, rgen, importlib.import_module("qwen38_inf2.checkpoint"))
        return

    ours = pkg.config.tiny_config(num_blocks=1)
    ref_cfg = replace(rconfig.tiny_config(num_blocks=1), weight_format="fp8", recurrent_state_format="bf16", kv_cache_format="bf16")
    assert ref_cfg.layer_types == ours.layer_types and ref_cfg.hidden_size == ours.hidden_size
    weights = tiny_weights(ours)
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

    mtp_goldens(rconfig, rmodel, rgen, ours)
    ftensors = fp8_cache_goldens(rconfig, rmodel, rgen, ours, weights)
    fmeta = dict(meta, k_scale=str(FP8_SCALES[0]), v_scale=str(FP8_SCALES[1]), verify_tokens=str(VERIFY))
    del fmeta["decode_steps"]
    save_file({k: v.contiguous() for k, v in ftensors.items()}, str(HERE / "tiny_fp8.safetensors"), metadata=fmeta)
    print(f"{len(ftensors)} tensors, {(HERE / 'tiny_fp8.safetensors').stat().st_size} bytes")

    vtensors = verify_goldens(rgen, ref_cfg, build_model(rmodel, ref_cfg, weights, VERIFY), ours)
    vmeta = dict(meta, verify_tokens=str(VERIFY), verify_steps=str(len(verify_schedule())))
    del vmeta["decode_steps"], vmeta["chunk"]
    save_file({k: v.contiguous() for k, v in vtensors.items()}, str(HERE / "tiny_verify.safetensors"), metadata=vmeta)
    print(f"{len(vtensors)} tensors, {(HERE / 'tiny_verify.safetensors').stat().st_size} bytes")


if __name__ == "__main__":
    main()
