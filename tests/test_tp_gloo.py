"""Tensor parallelism's host logic on CPU ranks (gloo): the TP cut of weights.shard_layer plus a sum of the
row-parallel outputs across ranks must give the single-rank result, as the reference's own
test_tensor_parallel_ranks_match_single_rank checks (tests/test_model_parity.py:141-170), including the
case the reference cannot run: more ranks than KV heads, with KV heads replicated.
"""

import os
import socket
from dataclasses import replace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import cpu_model as om


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _config(pkg, wide):
    cfg = pkg.config.tiny_config(num_blocks=1)
    if wide == "tp8":  # the full model's head counts (24 query over 4 KV heads, 16 key / 48 value heads) at the
        # tiny head sizes: at 8 ranks 3 query heads per rank, each pair of ranks sharing one replicated KV head
        cfg = replace(cfg, num_attention_heads=24, num_key_value_heads=4, linear_num_key_heads=16, linear_num_value_heads=48)
    elif wide:  # 8 query heads over 2 KV heads, 4 key / 12 value heads: splits 4 ways with KV replication
        cfg = replace(cfg, num_attention_heads=8, num_key_value_heads=2, linear_num_key_heads=4, linear_num_value_heads=12)
    return cfg


def _run(rank, world, port, wide, out_q):
    import importlib

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.set_num_threads(1)
    pkg = importlib.import_module("qwen38-27b-aws_b200")
    cfg = _config(pkg, wide)
    weights = {}
    for i in range(cfg.num_hidden_layers):
        full = pkg.weights.synthetic_layer(cfg, i, seed=3, device="cpu", std=0.1)
        weights |= pkg.weights.shard_layer(cfg, full, i, rank, world)

    def all_reduce(t):
        s = t.float().clone()
        dist.all_reduce(s)
        return s.to(t.dtype)

    step = om.OracleStep(cfg, weights, 32, 2, tp_degree=world, rank=rank, all_reduce=all_reduce, dtype=torch.float32)
    outs = []
    gen = torch.Generator().manual_seed(0)
    for pos in range(5):
        x = torch.randn(2, 1, cfg.hidden_size, generator=gen)
        cos, sin = om.rotary(cfg, torch.tensor([pos, pos + 3]), torch.float32)
        outs.append(step(inputs_embeds=x, cos=cos.unsqueeze(1), sin=sin.unsqueeze(1),
                         position=torch.tensor([pos, pos + 3], dtype=torch.int32), active=torch.ones(2)))
    out_q.put((rank, torch.stack(outs).numpy()))  # by value: the worker may exit before the parent reads
    dist.destroy_process_group()


@pytest.mark.parametrize("world,wide", [(2, False), (4, True), (8, "tp8")])
def test_tensor_parallel_ranks_match_single_rank(pkg, world, wide):
    cfg = _config(pkg, wide)
    weights = {}
    for i in range(cfg.num_hidden_layers):
        weights |= pkg.weights.synthetic_layer(cfg, i, seed=3, device="cpu", std=0.1)
    single = om.OracleStep(cfg, weights, 32, 2, dtype=torch.float32)
    gen = torch.Generator().manual_seed(0)
    want = []
    for pos in range(5):
        x = torch.randn(2, 1, cfg.hidden_size, generator=gen)
        cos, sin = om.rotary(cfg, torch.tensor([pos, pos + 3]), torch.float32)
        want.append(single(inputs_embeds=x, cos=cos.unsqueeze(1), sin=sin.unsqueeze(1),
                           position=torch.tensor([pos, pos + 3], dtype=torch.int32), active=torch.ones(2)))
    want = torch.stack(want)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, wide, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {r: torch.from_numpy(a) for r, a in (q.get(timeout=300) for _ in range(world))}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert (results[r] - want).abs().max() < 1e-4, f"rank {r} differs by {(results[r] - want).abs().max()}"
