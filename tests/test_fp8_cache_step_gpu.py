"""B200Step with the FP8 e4m3 KV cache (kv_cache_format "fp8") against the reference's own outputs.

The fixture tests/golden/tiny_fp8.safetensors was made by the reference's Qwen38Step with
kv_cache_format "fp8" and static scales (k 2^-5, v 2^-6, small enough that the largest values clamp at
240): decode steps with fresh and idle rows, a prefill chunk into one row, a decode step after it, then
a verify-built step's decode steps and five verify steps with different accepted counts, an idle row and
a row starting over. B200Step runs the same calls: hidden states within 2e-2 of the row peak and in
relative L2 (BASELINE), and the final caches' e4m3 bytes equal or one code apart for at most 1% of them
(a key one bf16 ulp away can round to the neighbouring code).
"""

from pathlib import Path

import pytest
import torch
from safetensors import safe_open

from tests.test_kernels_gpu import e5m2_code
from tests.test_step_gpu import assert_hidden_close

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_fp8.safetensors"
ORDER = {"decode": 0, "prefill": 1, "verify": 1, "after": 2}


def _calls(tensors, tag):
    def rank(name):
        kind = name[1:].rstrip("0123456789")
        return ORDER[kind], int(name[1 + len(kind):] or 0)

    return sorted({k.rsplit(".", 1)[0] for k in tensors if k.startswith(tag) and k.endswith(".y")}, key=rank)


@pytest.mark.parametrize("use_graph", [False, True])
def test_fp8_cache_step_matches_reference_golden(pkg, use_graph):
    step_mod = __import__(pkg.__name__ + ".step", fromlist=["step"])
    with safe_open(str(GOLDEN), "pt") as f:
        tensors, meta = {k: f.get_tensor(k) for k in f.keys()}, f.metadata()
    cfg = pkg.config.tiny_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, int(meta["seed"]), "cpu", float(meta["std"]))
    scales = {i: (float(meta["k_scale"]), float(meta["v_scale"])) for i, kind in enumerate(cfg.layer_types)
              if kind == pkg.config.FULL}
    for tag, K in (("d", 0), ("v", int(meta["verify_tokens"]))):
        step = step_mod.B200Step(cfg, w, int(meta["max_seq"]), int(meta["batch"]), verify_tokens=K, use_graph=use_graph,
                                 kv_cache_format="fp8", kv_scales=scales)
        for name in _calls(tensors, tag):
            keys = ("cos", "sin", "position", "active", "slot", "start", "n_valid", "accepted")
            inputs = {k: tensors[f"{name}.{k}"] for k in keys if f"{name}.{k}" in tensors}
            y = step(inputs_embeds=tensors[f"{name}.x"], **inputs)
            want = tensors[f"{name}.y"]
            if "active" in inputs:
                on = inputs["active"] > 0.5
                y, want = y[on], want[on]
            else:
                n = int(inputs["n_valid"])
                y, want = y[:, :n], want[:, :n]
            rows = want.shape[0] * want.shape[1]
            assert_hidden_close(y.reshape(rows, -1), want.reshape(rows, -1), what=f"{name}")
        for i, l in enumerate(step.layers):
            if l.kind == pkg.config.FULL:
                tail = max(K, 1) if tag == "v" else int(meta["chunk"])
                for which, cache in (("k_cache", l.mixer.k_cache), ("v_cache", l.mixer.v_cache)):
                    want = tensors[f"{tag}state.layers.{i}.self_attn.{which}"][:, :, :-tail]
                    d = (e5m2_code(cache.cpu()[:, :, :-tail]) - e5m2_code(want)).abs()
                    assert d.max().item() <= 1 and (d > 0).float().mean().item() <= 1e-2, f"{which} of layer {i}"
