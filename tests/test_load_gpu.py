"""B200Step / B200Head built from on-disk weights (weights.RankShards, presharded) give the same bytes as
when built from the same weights in memory; and from the reference's own per-rank files when its package
is in oracle/_ref (they convert exactly, so the same bytes again)."""

import pytest
import torch

from oracle import cpu_model as om

pytestmark = pytest.mark.gpu


def test_step_from_rank_shards_equals_step_from_memory(pkg, tmp_path):
    step_mod = __import__(pkg.__name__ + ".step", fromlist=["step"])
    W = pkg.weights
    cfg = pkg.config.tiny_config(num_blocks=1)
    layers = {i: W.synthetic_layer(cfg, i, 5, "cpu", 0.1) for i in range(cfg.num_hidden_layers)}
    head = W.synthetic_head(cfg, 5, "cpu", 0.1)
    W.write_rank_shards(cfg, lambda i: layers[i], head, tmp_path, 1)
    shards = W.RankShards(tmp_path, 0)
    batch = 3
    pos = torch.tensor([0, 7, 30], dtype=torch.int32)
    cos, sin = om.rotary(cfg, pos, torch.bfloat16)
    inputs = dict(cos=cos.unsqueeze(1), sin=sin.unsqueeze(1), position=pos, active=torch.ones(batch))
    x = torch.randn(batch, 1, cfg.hidden_size, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    outs = []
    for build in (lambda: (step_mod.B200Step(cfg, lambda i: layers[i], 64, batch), step_mod.B200Head(cfg, head, batch)),
                  lambda: (step_mod.B200Step(cfg, shards.layer, 64, batch, presharded=True),
                           step_mod.B200Head(cfg, shards.head(), batch, presharded=True))):
        step, hd = build()
        y = step(inputs_embeds=x, **inputs)
        outs.append((y, hd.run_graph(y), hd.next_tokens(y)))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1]) and outs[0][2] == outs[1][2]
