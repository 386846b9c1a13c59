"""The full-width fixture (tests/golden/full_block.safetensors): BASELINE config 0 made by the reference.

One full-width 4-layer block (3 gated-delta + 1 attention layer) at batch 8, rows at positions uniform in
[0, 512) over seeded cache and state contents, two greedy decode steps through the reference's
Qwen38Step, its HeadStep maxima over the whole 248,320-token vocabulary and ChipHead.next_tokens (the
exact recheck of the best 4 groups). Weights and states are regenerated here from their seeds; the
fixture holds the inputs, the outputs and a SHA-256 of the weights.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import torch
from safetensors import safe_open

from tests.golden.make_golden import full_width_states

PATH = Path(__file__).resolve().parent / "golden" / "full_block.safetensors"


def load():
    with safe_open(str(PATH), "pt") as f:
        return {k: f.get_tensor(k) for k in f.keys()}, f.metadata()


def digest(pkg, weights) -> str:
    h = hashlib.sha256()
    for name in sorted(weights):
        t = weights[name]
        parts = (t.q, t.scale) if isinstance(t, pkg.weights.FP8Weight) else (t,)
        for p in parts:
            h.update(name.encode())
            h.update(p.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def model(pkg, meta):
    """(cfg, block weights, head weights) regenerated on the CPU and checked against the fixture."""
    cfg = pkg.config.full_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, int(meta["seed"]), "cpu")
    head = pkg.weights.synthetic_head(cfg, int(meta["seed"]), "cpu")
    assert digest(pkg, w) == meta["weights_sha256"], "synthetic weights drifted from the fixture"
    assert digest(pkg, head) == meta["head_sha256"], "synthetic head drifted from the fixture"
    return cfg, w, head


def seed_oracle(oracle, cfg, meta) -> None:
    """The fixture's starting states, into an oracle.OracleStep."""
    states = full_width_states(cfg, int(meta["batch"]), int(meta["max_seq"]), int(meta["state_seed"]))
    for (kind, mixer, *_r), (a, b) in zip(oracle.layers, states):
        if hasattr(mixer, "recurrent_state"):
            mixer.recurrent_state.copy_(a)
            mixer.conv_state.copy_(b)
        else:
            mixer.k_cache.copy_(a)
            mixer.v_cache.copy_(b)


def seed_step(step, cfg, meta) -> None:
    """The fixture's starting states, into a B200Step (TP = 1)."""
    states = full_width_states(cfg, int(meta["batch"]), int(meta["max_seq"]), int(meta["state_seed"]))
    for l, (a, b) in zip(step.layers, states):
        if hasattr(l.mixer, "state"):
            l.mixer.state[: a.shape[0]].copy_(a)
            l.mixer.conv_state[: b.shape[0]].copy_(b)
        else:
            l.mixer.k_cache.copy_(a)
            l.mixer.v_cache.copy_(b)


def inputs(tensors, step: int) -> dict:
    return {k: tensors[f"step{step}.{k}"] for k in ("cos", "sin", "position", "active")}
