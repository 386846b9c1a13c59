"""On-disk weights: this package's per-rank shards, and the reference's own per-rank files (CPU only).

* write_rank_shards + RankShards: every rank reads back exactly its TP cut (shard_layer / shard_head /
  shard_mtp), including the KV-head replication at TP = 8 on the full-width shape's head counts.
* reference_rank_files: a checkpoint made by the reference's own tools (fp4.encode_host for an MXFP4
  source, checkpoint.write_rank_weights for its per-rank block files, as scripts/prepare_weights.py
  does), read back joined across its ranks and converted to e4m3 with per-32 scales: every matrix equals
  the reference's own decode of the MXFP4 source (fp4.decode_host) bit for bit, every vector the source.
"""

import sys
from dataclasses import replace

import pytest
import torch

from oracle import ref_step


def _tiny(pkg):
    cfg = pkg.config.tiny_config(num_blocks=2)
    return cfg, {i: pkg.weights.synthetic_layer(cfg, i, 3, "cpu", 0.1) for i in range(cfg.num_hidden_layers)}


def test_rank_shards_round_trip_every_rank(pkg, tmp_path):
    W = pkg.weights
    cfg, layers = _tiny(pkg)
    head = W.synthetic_head(cfg, 3, "cpu", 0.1)
    mtp = W.synthetic_mtp(cfg, 3, "cpu", 0.1)
    tp = 2
    W.write_rank_shards(cfg, lambda i: layers[i], head, tmp_path, tp, mtp)
    for r in range(tp):
        shards = W.RankShards(tmp_path, r)
        for i in range(cfg.num_hidden_layers):
            got, want = shards.layer(i), W.shard_layer(cfg, layers[i], i, r, tp)
            assert got.keys() == want.keys()
            for k in want:
                a, b = got[k], want[k]
                if isinstance(b, W.FP8Weight):
                    assert torch.equal(a.q, b.q) and torch.equal(a.scale, b.scale), k
                else:
                    assert torch.equal(a, b), k
        assert torch.equal(shards.head()["lm_head"].q, W.shard_head(cfg, head, r, tp)["lm_head"].q)
        assert torch.equal(shards.mtp()["fc"].q, W.shard_mtp(cfg, mtp, r, tp)["fc"].q)
    with pytest.raises(ValueError):
        W.RankShards(tmp_path, tp)


def test_rank_shards_keep_the_kv_replication_at_tp8(pkg, tmp_path):
    W = pkg.weights
    cfg = pkg.config.full_config(num_blocks=1)
    small = replace(cfg, hidden_size=256, intermediate_size=512)  # full head counts, small matrices
    w = W.synthetic_layer(small, 3, 0, "cpu")
    W.write_rank_shards(small, lambda i: W.synthetic_layer(small, i, 0, "cpu"), W.synthetic_head(replace(small, vocab_size=1024), 0),
                        tmp_path, 8)
    for r in (0, 1, 6, 7):
        got = W.RankShards(tmp_path, r).layer(3)["layers.3.self_attn.k_proj"]
        h = small.head_dim
        first = small.kv_head_of_rank(r, 8)
        assert torch.equal(got.q, w["layers.3.self_attn.k_proj"].q[first * h:(first + 1) * h])


def test_reference_rank_files_import_exactly(pkg, tmp_path):
    if not ref_step.available():
        pytest.skip("the reference's package is not in oracle/_ref")
    if str(ref_step.REF) not in sys.path:
        sys.path.insert(0, str(ref_step.REF))
    import qwen38_inf2.checkpoint as rcheck
    import qwen38_inf2.fp4 as rfp4

    rconfig, _, _ = ref_step._modules()
    cfg, layers = _tiny(pkg)
    rcfg = ref_step.ref_config(rconfig, cfg)
    P = rcheck.TEXT_PREFIX
    source, decoded = {}, {}
    matrices = {"mlp.gate_proj": "mlp.gate_proj", "mlp.up_proj": "mlp.up_proj", "mlp.down_proj": "mlp.down_proj",
                "linear_attn.in_proj_qkv": "linear_attn.in_proj_qkv", "linear_attn.in_proj_z": "linear_attn.in_proj_z",
                "linear_attn.out_proj": "linear_attn.out_proj", "self_attn.q_proj": "self_attn.q_proj",
                "self_attn.k_proj": "self_attn.k_proj", "self_attn.v_proj": "self_attn.v_proj",
                "self_attn.o_proj": "self_attn.o_proj"}
    vectors = {"input_layernorm_weight": "input_layernorm.weight",
               "post_attention_layernorm_weight": "post_attention_layernorm.weight",
               "linear_attn.in_proj_b": "linear_attn.in_proj_b.weight", "linear_attn.in_proj_a": "linear_attn.in_proj_a.weight",
               "linear_attn.A_log": "linear_attn.A_log", "linear_attn.dt_bias": "linear_attn.dt_bias",
               "linear_attn.norm_weight": "linear_attn.norm.weight", "self_attn.q_norm_weight": "self_attn.q_norm.weight",
               "self_attn.k_norm_weight": "self_attn.k_norm.weight"}
    for i, w in layers.items():
        for ours, hf in matrices.items():
            if f"layers.{i}.{ours}" in w:
                packed, scale = rfp4.encode_host(w[f"layers.{i}.{ours}"].dequant())
                source[f"{P}layers.{i}.{hf}.weight_packed"], source[f"{P}layers.{i}.{hf}.weight_scale"] = packed, scale
                decoded[f"layers.{i}.{ours}"] = rfp4.decode_host(packed, scale, torch.float32)
        for ours, hf in vectors.items():
            if f"layers.{i}.{ours}" in w:
                source[f"{P}layers.{i}.{hf}"] = w[f"layers.{i}.{ours}"]
        if f"layers.{i}.linear_attn.conv_weight" in w:
            source[f"{P}layers.{i}.linear_attn.conv1d.weight"] = w[f"layers.{i}.linear_attn.conv_weight"].unsqueeze(1)
    rcheck.write_rank_weights(rcheck.DictSource(source), rcfg, tmp_path, 4, tp_degree=2)
    layer = pkg.weights.reference_rank_files(tmp_path, cfg, 4, 2)
    for i, w in layers.items():
        got = layer(i)
        assert got.keys() == w.keys(), set(got) ^ set(w)
        for name, t in got.items():
            if isinstance(t, pkg.weights.FP8Weight):
                assert torch.equal(t.dequant(), decoded[name]), name
            else:
                assert torch.equal(t, w[name]), name
