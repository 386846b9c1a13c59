"""B200MTP (the MTP draft layer) against the reference's own MTPStep outputs.

The fixture tests/golden/tiny_mtp.safetensors was made by the reference's MTPStep (model.py:812-860)
with synthetic weights: a prompt chunk into slot 1 (which only fills the layer's cache), then two steps
of 4 tokens per row from each row's MTP index (an idle row in the first), the second step on the first
step's outputs. B200MTP runs the same calls: outputs within 2e-2 of the row peak and in relative L2
(BASELINE), the layer's cache keys within one bf16 ulp on at most 0.1% of values and values bit for bit.
"""

from pathlib import Path

import pytest
import torch
from safetensors import safe_open

from tests.test_kernels_gpu import assert_bf16_close
from tests.test_step_gpu import assert_hidden_close

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_mtp.safetensors"


def test_mtp_layer_matches_reference_golden(pkg):
    step_mod = __import__(pkg.__name__ + ".step", fromlist=["step"])
    with safe_open(str(GOLDEN), "pt") as f:
        tensors, meta = {k: f.get_tensor(k) for k in f.keys()}, f.metadata()
    cfg = pkg.config.tiny_config(num_blocks=1)
    weights = pkg.weights.synthetic_mtp(cfg, int(meta["seed"]), "cpu", float(meta["std"]))
    mtp = step_mod.B200MTP(cfg, weights, int(meta["max_seq"]), int(meta["batch"]), tokens=int(meta["tokens"]),
                           max_chunk=int(meta["chunk"]))
    calls = ["prefill"] + [f"step{s}" for s in range(int(meta["steps"]))]
    for name in calls:
        keys = ("cos", "sin", "position", "active", "slot", "start", "n_valid")
        inputs = {k: tensors[f"{name}.{k}"] for k in keys if f"{name}.{k}" in tensors}
        y = mtp(hidden=tensors[f"{name}.hidden"], inputs_embeds=tensors[f"{name}.x"], **inputs)
        want = tensors[f"{name}.y"]
        assert y.shape == want.shape, name
        if "active" in inputs:
            on = inputs["active"] > 0.5
            y, want = y[on], want[on]
        rows = want.shape[0] * want.shape[1]
        assert_hidden_close(y.reshape(rows, -1), want.reshape(rows, -1), what=name)
    tail = max(int(meta["tokens"]), int(meta["chunk"]))
    attn = mtp.layer.layers[0].mixer
    assert_bf16_close(attn.k_cache.cpu()[:, :, :-tail], tensors["state.k_cache"][:, :, :-tail], frac=0.001, what="k cache")
    assert torch.equal(attn.v_cache.cpu()[:, :, :-tail], tensors["state.v_cache"][:, :, :-tail])
