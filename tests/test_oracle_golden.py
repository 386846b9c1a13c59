"""The CPU oracle against golden vectors made by the reference itself (tests/golden/make_golden.py).

These pin the oracle: every later GPU parity test compares the CUDA path with this oracle, so the
oracle must first reproduce the reference's own outputs on the same inputs.
"""

import hashlib
from pathlib import Path

import pytest
import torch
from safetensors import safe_open

from oracle import cpu_model as om

GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_block.safetensors"


def _digest(pkg, weights):
    h = hashlib.sha256()
    for name in sorted(weights):
        t = weights[name]
        parts = (t.q, t.scale) if isinstance(t, pkg.weights.FP8Weight) else (t,)
        for p in parts:
            h.update(name.encode())
            h.update(p.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


@pytest.fixture(scope="module")
def golden():
    with safe_open(str(GOLDEN), "pt") as f:
        return {k: f.get_tensor(k) for k in f.keys()}, f.metadata()


@pytest.fixture(scope="module")
def tiny(pkg, golden):
    tensors, meta = golden
    cfg = pkg.config.tiny_config(num_blocks=1)
    seed, std = int(meta["seed"]), float(meta["std"])
    weights = {}
    for i in range(cfg.num_hidden_layers):
        weights |= pkg.weights.synthetic_layer(cfg, i, seed, "cpu", std)
    head = pkg.weights.synthetic_head(cfg, seed, "cpu", std)
    assert _digest(pkg, weights) == meta["weights_sha256"], "synthetic weights drifted from the fixture"
    assert _digest(pkg, head) == meta["head_sha256"]
    return cfg, weights, head, meta


def _inputs(tensors, prefix):
    keys = ("cos", "sin", "position", "active", "slot", "start", "n_valid")
    return {k: tensors[f"{prefix}.{k}"] for k in keys if f"{prefix}.{k}" in tensors}


def test_oracle_reproduces_reference_decode_prefill_and_states(golden, tiny):
    tensors, _ = golden
    cfg, weights, _, meta = tiny
    step = om.OracleStep(cfg, weights, int(meta["max_seq"]), int(meta["batch"]))
    worst = 0.0
    for s in range(int(meta["decode_steps"])):
        y = step(inputs_embeds=tensors[f"decode{s}.x"], **_inputs(tensors, f"decode{s}"))
        want = tensors[f"decode{s}.y"]
        active = tensors[f"decode{s}.active"] > 0.5
        worst = max(worst, (y[active].float() - want[active].float()).abs().max().item())
    for c in range(2):
        y = step(inputs_embeds=tensors[f"prefill{c}.x"], **_inputs(tensors, f"prefill{c}"))
        n = int(tensors[f"prefill{c}.n_valid"])
        worst = max(worst, (y[:, :n].float() - tensors[f"prefill{c}.y"][:, :n].float()).abs().max().item())
    y = step(inputs_embeds=tensors["after.x"], **_inputs(tensors, "after"))
    worst = max(worst, (y.float() - tensors["after.y"].float()).abs().max().item())
    assert worst == 0.0, f"oracle differs from the reference by {worst}"

    # Final recurrent, conv and KV states, except the KV cache's junk tail (written by inactive rows).
    for i, (kind, mixer, *_rest) in enumerate(step.layers):
        if kind == om.LINEAR:
            assert torch.equal(mixer.recurrent_state, tensors[f"state.layers.{i}.linear_attn.recurrent_state"])
            assert torch.equal(mixer.conv_state, tensors[f"state.layers.{i}.linear_attn.conv_state"])
        else:
            tail = int(meta["chunk"])
            assert torch.equal(mixer.k_cache[:, :, :-tail], tensors[f"state.layers.{i}.self_attn.k_cache"][:, :, :-tail])
            assert torch.equal(mixer.v_cache[:, :, :-tail], tensors[f"state.layers.{i}.self_attn.v_cache"][:, :, :-tail])


def test_oracle_head_maxima_match_reference(golden, tiny):
    tensors, _ = golden
    cfg, _, head, _ = tiny
    got = om.head_maxima(cfg, tensors["head.hidden"], head["norm_weight"], head["lm_head"].q, head["lm_head"].scale)
    assert torch.equal(got, tensors["head.maxima"])


def test_oracle_kernels_match_reference(golden):
    tensors, _ = golden
    d = {k.split(".", 1)[1]: v for k, v in tensors.items() if k.startswith("delta.")}
    out, s1 = om.chunked_gated_delta(d["q"], d["k"], d["v"], d["g"], d["b"], d["s0"], chunk=32)
    assert torch.equal(out, d["out"]) and torch.equal(s1, d["s1"])
    assert torch.equal(om.unit_lower_inverse(tensors["inverse.lower"]), tensors["inverse.out"])
    got = om.blocked_attention(tensors["attn.q"], tensors["attn.k"], tensors["attn.v"], tensors["attn.visible"], 16)
    assert torch.equal(got, tensors["attn.out"])


def test_chunked_rule_matches_recurrent_rule():
    """The property the reference tests (tests/test_prefill.py:29-49), here on the oracle."""
    torch.manual_seed(0)
    heads, tokens, dim = 3, 128, 32
    q = torch.nn.functional.normalize(torch.randn(heads, tokens, dim), dim=-1) / dim**0.5
    k = torch.nn.functional.normalize(torch.randn(heads, tokens, dim), dim=-1)
    v = torch.randn(heads, tokens, dim)
    g = -torch.rand(heads, tokens) * 0.5
    b = torch.rand(heads, tokens)
    s = torch.randn(heads, dim, dim)
    want_o, want_s = om.recurrent_gated_delta(q, k, v, g, b, s)
    got_o, got_s = om.chunked_gated_delta(q, k, v, g, b, s, chunk=64)
    assert (got_o - want_o).abs().max() < 1e-3 and (got_s - want_s).abs().max() < 1e-3


VERIFY_GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_verify.safetensors"


def test_oracle_reproduces_reference_verify_steps(pkg):
    """Decode, five verify steps (commit-on-accept with different accepted counts, an idle row, a row
    starting over), then decode: every output and the final recurrent, conv, pending and KV buffers."""
    with safe_open(str(VERIFY_GOLDEN), "pt") as f:
        tensors, meta = {k: f.get_tensor(k) for k in f.keys()}, f.metadata()
    cfg = pkg.config.tiny_config(num_blocks=1)
    weights = {}
    for i in range(cfg.num_hidden_layers):
        weights |= pkg.weights.synthetic_layer(cfg, i, int(meta["seed"]), "cpu", float(meta["std"]))
    assert _digest(pkg, weights) == meta["weights_sha256"]
    K = int(meta["verify_tokens"])
    step = om.OracleStep(cfg, weights, int(meta["max_seq"]), int(meta["batch"]), verify_tokens=K)
    calls = [f"decode{s}" for s in range(2)] + [f"verify{s}" for s in range(int(meta["verify_steps"]))] + ["after"]
    for c in calls:
        y = step(inputs_embeds=tensors[f"{c}.x"], **_inputs(tensors, c) | ({"accepted": tensors[f"{c}.accepted"]} if f"{c}.accepted" in tensors else {}))
        active = tensors[f"{c}.active"] > 0.5
        assert torch.equal(y[active], tensors[f"{c}.y"][active]), f"{c}: oracle differs from the reference"
    for i, (kind, mixer, *_rest) in enumerate(step.layers):
        if kind == om.LINEAR:
            p = f"state.layers.{i}.linear_attn."
            assert torch.equal(mixer.recurrent_state, tensors[p + "recurrent_state"])
            assert torch.equal(mixer.conv_state, tensors[p + "conv_state"])
            assert torch.equal(mixer.pending_key, tensors[p + "pending_key_state"])
            assert torch.equal(mixer.pending_delta, tensors[p + "pending_delta_state"])
            assert torch.equal(mixer.pending_decay, tensors[p + "pending_decay_state"])
            assert torch.equal(mixer.pending_input, tensors[p + "pending_input_state"])
        else:
            tail = K  # the junk positions written by idle rows
            assert torch.equal(mixer.k_cache[:, :, :-tail], tensors[f"state.layers.{i}.self_attn.k_cache"][:, :, :-tail])
            assert torch.equal(mixer.v_cache[:, :, :-tail], tensors[f"state.layers.{i}.self_attn.v_cache"][:, :, :-tail])


FP8_GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_fp8.safetensors"


def test_oracle_reproduces_reference_fp8_kv_cache(pkg):
    """The FP8 e4m3 KV cache with static scales (model.py:579-608), made by the reference with its
    kv_cache_format "fp8": decode steps (fresh and idle rows), a prefill chunk, decode again, then a
    verify model's decode and verify steps; every output and the final cache bytes. The value scale
    is small enough that the largest values clamp at 240."""
    with safe_open(str(FP8_GOLDEN), "pt") as f:
        tensors, meta = {k: f.get_tensor(k) for k in f.keys()}, f.metadata()
    cfg = pkg.config.tiny_config(num_blocks=1)
    weights = {}
    for i in range(cfg.num_hidden_layers):
        weights |= pkg.weights.synthetic_layer(cfg, i, int(meta["seed"]), "cpu", float(meta["std"]))
    assert _digest(pkg, weights) == meta["weights_sha256"]
    scales = {i: (float(meta["k_scale"]), float(meta["v_scale"])) for i, kind in enumerate(cfg.layer_types) if kind == om.FULL}
    # The calls in the order they were made: decode steps, then the prefill chunk and the decode after it,
    # or the verify steps.
    order = {"decode": 0, "prefill": 1, "verify": 1, "after": 2}

    def rank(name):
        kind = name[1:].rstrip("0123456789")
        return order[kind], int(name[1 + len(kind):] or 0)

    clamped = False
    for tag, K in (("d", 0), ("v", int(meta["verify_tokens"]))):
        step = om.OracleStep(cfg, weights, int(meta["max_seq"]), int(meta["batch"]), verify_tokens=K, kv_scales=scales)
        names = sorted({k.rsplit(".", 1)[0] for k in tensors if k.startswith(tag) and k.endswith(".y")}, key=rank)
        assert len(names) == int(tensors[f"{tag}calls"])
        for name in names:
            keys = ("cos", "sin", "position", "active", "slot", "start", "n_valid", "accepted")
            inputs = {k: tensors[f"{name}.{k}"] for k in keys if f"{name}.{k}" in tensors}
            y = step(inputs_embeds=tensors[f"{name}.x"], **inputs)
            want = tensors[f"{name}.y"]
            if "active" in inputs:
                on = inputs["active"] > 0.5
                y, want = y[on], want[on]
            elif "n_valid" in inputs:
                n = int(inputs["n_valid"])
                y, want = y[:, :n], want[:, :n]
            assert torch.equal(y, want), f"{name}: oracle differs from the reference"
        for i, (kind, mixer, *_rest) in enumerate(step.layers):
            if kind == om.FULL:
                tail = max(K, 1) if tag == "v" else int(meta["chunk"])
                for which, cache in (("k_cache", mixer.k_cache), ("v_cache", mixer.v_cache)):
                    want = tensors[f"{tag}state.layers.{i}.self_attn.{which}"]
                    assert want.dtype == torch.uint8 and torch.equal(cache[:, :, :-tail], want[:, :, :-tail])
                    clamped |= bool((want.view(torch.float8_e4m3fn).float().abs() == 240).any())
    assert clamped, "no cached value reached the 240 clamp"


def test_oracle_reproduces_full_width_reference_steps_and_head(pkg):
    """BASELINE config 0 at full width, made by the reference (tests/golden/make_golden.py --full-width):
    two greedy decode steps of one 4-layer block at batch 8 over seeded states, each output bit for bit,
    then HeadStep's maxima over the whole 248,320-token vocabulary (fp32 logits in another summation
    layout: within 1e-5 relative) and ChipHead's tokens and top-4 groups exactly."""
    from tests import full_width as fw

    tensors, meta = fw.load()
    cfg, w, head = fw.model(pkg, meta)
    batch = int(meta["batch"])
    oracle = om.OracleStep(cfg, w, int(meta["max_seq"]), batch)
    fw.seed_oracle(oracle, cfg, meta)
    lm_rows = head["lm_head"].dequant()
    for s in range(int(meta["steps"])):
        y = oracle(inputs_embeds=tensors[f"step{s}.x"], **fw.inputs(tensors, s))
        assert torch.equal(y, tensors[f"step{s}.y"]), f"step {s}: oracle differs from the reference"
        maxima = om.head_maxima(cfg, y, head["norm_weight"], head["lm_head"].q, head["lm_head"].scale)
        want = tensors[f"step{s}.maxima"]
        rel = ((maxima - want).abs() / want.abs().amax(-1, keepdim=True)).max().item()
        assert rel <= 1e-5, f"step {s}: maxima differ by {rel:.3g} of the row peak"
        assert torch.equal(maxima.topk(4, dim=-1).indices, tensors[f"step{s}.top4"])
        tokens = om.recheck_tokens(cfg, y, head["norm_weight"], lm_rows, maxima)
        assert tokens == tensors[f"step{s}.tokens_out"].tolist()
        if s + 1 < int(meta["steps"]):
            assert tokens == tensors[f"step{s + 1}.tokens_in"].tolist()


MTP_GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_mtp.safetensors"


def _mtp_calls(tensors):
    return ["prefill"] + [f"step{s}" for s in range(sum(1 for k in tensors if k.startswith("step") and k.endswith(".y")))]


def test_oracle_reproduces_reference_mtp_layer(pkg):
    """The MTP draft layer (MTPStep), made by the reference: a prompt chunk (cache only), then two steps of
    4 tokens per row (the second on the first's outputs), each output and the layer's final KV cache."""
    with safe_open(str(MTP_GOLDEN), "pt") as f:
        tensors, meta = {k: f.get_tensor(k) for k in f.keys()}, f.metadata()
    cfg = pkg.config.tiny_config(num_blocks=1)
    weights = pkg.weights.synthetic_mtp(cfg, int(meta["seed"]), "cpu", float(meta["std"]))
    assert _digest(pkg, weights) == meta["weights_sha256"]
    mtp = om.OracleMTP(cfg, weights, int(meta["max_seq"]), int(meta["batch"]))
    for name in _mtp_calls(tensors):
        keys = ("cos", "sin", "position", "active", "slot", "start", "n_valid")
        inputs = {k: tensors[f"{name}.{k}"] for k in keys if f"{name}.{k}" in tensors}
        y = mtp(hidden=tensors[f"{name}.hidden"], inputs_embeds=tensors[f"{name}.x"], **inputs)
        want = tensors[f"{name}.y"]
        if "active" in inputs:
            on = inputs["active"] > 0.5
            y, want = y[on], want[on]
        assert torch.equal(y, want), f"{name}: oracle differs from the reference"
    tail = max(int(meta["tokens"]), int(meta["chunk"]))  # the junk positions of idle rows and of prefill's other rows
    assert torch.equal(mtp.attention.k_cache[:, :, :-tail], tensors["state.k_cache"][:, :, :-tail])
    assert torch.equal(mtp.attention.v_cache[:, :, :-tail], tensors["state.v_cache"][:, :, :-tail])
