"""The fused GEMM + all-reduce over NVLink peer memory, and B200Step at TP = 2, 4 and 8 (each world
skipped when the box has fewer GPUs).

One spawned process per GPU, NCCL process group on 127.0.0.1 (used only to pass the IPC handles, for
the baseline and to compare ranks). Checks, per rank:
* q38_fp8_gemm_allreduce equals, bit for bit, its stated arithmetic: every rank's bf16 partial (the
  plain GEMM with the same K splits), summed in fp32 in rank order, rounded to bf16 once, added to the
  residual in bf16; for decode, verify and prefill shapes, over consecutive calls (both epoch
  parities) and inside a replayed CUDA graph.
* B200Step at TP = world with the fused all-reduce (one full-width 4-layer block; at TP = 8 two ranks
  share each of the 4 KV heads), layer by layer (the same input on both sides), against the oracle
  running the same TP arithmetic (world oracle ranks in threads whose all-reduce sums the bf16
  partials in fp32 in rank order): within 2e-2 (BASELINE). The oracle runs once, in the test process,
  before the GPU ranks start. Every rank's residual stream must equal rank 0's bit for bit. TP is not
  compared with TP = 1 end to end: rounding each rank's partial to bf16 moves later e5m2 roundings, as
  the reference's own TP test avoids by running in float32 (tests/test_model_parity.py:141-170).
* the same layer checks with the NCCL baseline instead of the fused all-reduce (within 1e-1 above two
  ranks, where NCCL's ring rounds every hop's partial sum to bf16);
* two whole steps back to back, as one CUDA graph and as eager launches: the same bits (the exchange
  has no host synchronisation between layers there).
Each worker bounds its collectives (a short process-group timeout) and the parent kills workers that
outlive their budget. NVLS stays off (NCCL_NVLS_ENABLE=0) and the fused kernels use plain peer stores.
"""

import importlib
import multiprocessing as mp
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue, oracle_path):
    try:
        sys.path.insert(0, str(ROOT))
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        import datetime

        torch.distributed.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                             timeout=datetime.timedelta(seconds=120))
        pkg = importlib.import_module("qwen38-27b-aws_b200")
        ops = importlib.import_module("qwen38-27b-aws_b200.ops")
        dev = torch.device(f"cuda:{rank}")
        results = []
        hidden = 5120
        comm = ops.Communicator(rank, world, 1024, hidden, dev)
        stream = torch.cuda.current_stream()

        def case(tokens, k, splits, seed):
            g = torch.Generator().manual_seed(seed * 10 + rank)
            w = pkg.weights.FP8Weight.from_float(torch.randn(hidden, k, generator=g) * 0.02)
            lin = ops.DeviceLinear(w, dev)
            xq = pkg.codec.to_e5m2_bytes(torch.randn(tokens, k, generator=g).to(torch.bfloat16)).to(dev)
            gr = torch.Generator().manual_seed(seed)  # the residual is the same on every rank
            res = torch.randn(tokens, hidden, generator=gr).to(torch.bfloat16).to(dev)
            part = torch.empty(tokens, hidden, dtype=torch.bfloat16, device=dev)
            ws = torch.zeros(max(256, ops.gemm_workspace_bytes(tokens, hidden, splits)), dtype=torch.uint8, device=dev)
            ops.fp8_gemm(xq, lin, part, splits=splits, workspace=ws)
            every = torch.empty(world * tokens, hidden, dtype=torch.bfloat16, device=dev)
            torch.distributed.all_gather_into_tensor(every, part)
            acc = torch.zeros(tokens, hidden, dtype=torch.float32, device=dev)
            for r in range(world):
                acc += every[r * tokens:(r + 1) * tokens].float()
            want = (res.float() + acc.to(torch.bfloat16).float()).to(torch.bfloat16)
            return lin, xq, res, want

        cases = [(8, 3072, 3, 1), (32, 3072, 3, 2), (256, 8704, 3, 3), (512, 8704, 1, 4), (200, 3072, 2, 5)]
        for tokens, k, splits, seed in cases:
            lin, xq, res, want = case(tokens, k, splits, seed)
            for rep in range(3):  # consecutive calls: both epoch parities, slots reused
                comm.x[:tokens].copy_(res)
                torch.distributed.barrier()
                ops.fp8_gemm_allreduce(xq, lin, comm, splits=splits)
                torch.cuda.synchronize()
                status = ops.device_status()
                ok = status == 0 and torch.equal(comm.x[:tokens], want)
                results.append((f"fused {tokens}x{k}/{splits} call {rep}", ok,
                                f"device status {status}, max diff {(comm.x[:tokens].float() - want.float()).abs().max().item()}"))
        # Inside a CUDA graph: the epoch advances on the device, so replays exchange correctly.
        lin, xq, res, want = case(256, 8704, 3, 6)
        graph = torch.cuda.CUDAGraph()
        comm.x[:256].copy_(res)
        torch.distributed.barrier()
        ops.fp8_gemm_allreduce(xq, lin, comm, splits=3)  # warm-up outside capture
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            ops.fp8_gemm_allreduce(xq, lin, comm, splits=3)
        for rep in range(3):
            comm.x[:256].copy_(res)
            torch.cuda.synchronize()
            torch.distributed.barrier()
            graph.replay()
            torch.cuda.synchronize()
            results.append((f"graph replay {rep}", torch.equal(comm.x[:256], want) and ops.device_status() == 0, ""))
        del graph
        torch.cuda.synchronize()
        comm.close()

        # B200Step at TP = world, with the fused all-reduce and with the NCCL baseline: layer by layer
        # against the oracle's layer outputs (computed by the parent).
        step_mod = importlib.import_module("qwen38-27b-aws_b200.step")
        ref = torch.load(oracle_path)
        cfg = pkg.config.full_config(num_blocks=1)
        w = _block_weights(pkg, cfg)
        emb, inputs, xs = ref["emb"], ref["inputs"], ref["layers"]
        batch = emb.shape[0]
        for name, fused in (("fused", True), ("nccl", False)):
            step = step_mod.B200Step(cfg, w, 512, batch, tp_degree=world, rank=rank, device=dev, use_graph=False,
                                     fused_allreduce=fused)
            step.load_decode_inputs(emb, inputs["cos"], inputs["sin"], inputs["position"], inputs["active"])
            for i in range(cfg.num_hidden_layers):
                step.x.copy_(xs[i].reshape(batch, -1))
                torch.distributed.barrier()
                step.run_layer(i)
                torch.cuda.synchronize()
                every = torch.empty(world * batch, cfg.hidden_size, dtype=torch.bfloat16, device=dev)
                torch.distributed.all_gather_into_tensor(every, step.x.contiguous())
                same = all(torch.equal(every[r * batch:(r + 1) * batch], step.x) for r in range(world))
                results.append((f"TP={world} {name} layer {i}: every rank's residual stream equals rank 0's", same, ""))
                got = step.x.float().cpu()
                want = xs[i + 1].float().reshape(batch, -1)
                peak = want.abs().amax(-1, keepdim=True)
                worst = ((got - want).abs() / peak).max().item()
                rel = ((got - want).norm(dim=-1) / want.norm(dim=-1)).max().item()
                # The NCCL baseline sums bf16 partials on a ring: above two ranks every hop rounds to bf16,
                # which the oracle's rank-order fp32 sum does not, and the layer's e5m2 roundings amplify
                # those ulps; it is the comparison baseline, held to 1e-1 there.
                bound = 1e-1 if (name == "nccl" and world > 2) else 2e-2
                results.append((f"TP={world} {name} layer {i} vs TP={world} oracle", worst <= bound and rel <= bound,
                                f"max {worst:.3g} of the row peak, relative L2 {rel:.3g}"))
            step.close()
            torch.distributed.barrier()
        # Whole steps back to back (no host synchronisation between the layers' exchanges): the CUDA graph
        # and the eager launches of the fused path give the same bits. End to end the fused path is not
        # compared with NCCL's: above two ranks NCCL rounds its partial sums to bf16 on every hop, and
        # four layers of e5m2 roundings amplify those ulps (the layer checks above bound each path).
        outs = {}
        for name, graph in (("graph", True), ("eager", False)):
            step = step_mod.B200Step(cfg, w, 512, batch, tp_degree=world, rank=rank, device=dev, use_graph=graph)
            outs[name] = [step(inputs_embeds=emb, **inputs).float() for _ in range(2)]
            step.close()
            torch.distributed.barrier()
        for s in range(2):
            same = torch.equal(outs["graph"][s], outs["eager"][s])
            diff = (outs["graph"][s] - outs["eager"][s]).abs().max().item()
            results.append((f"TP={world} step {s}: CUDA graph equals eager launches", same and ops.device_status() == 0,
                            f"max diff {diff:.3g}"))
        torch.distributed.destroy_process_group()
        queue.put((rank, results, None))
    except Exception:  # noqa: BLE001
        queue.put((rank, [], traceback.format_exc()))


def _block_weights(pkg, cfg) -> dict:
    """One full-width 4-layer block's unsharded weights, drawn on the CPU (the same values in every process)."""
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, seed=0, device="cpu")
    return w


def _oracle_layers(world: int, path: Path) -> None:
    """The TP = world oracle's output after each layer of the block, teacher-forced (layer i gets the
    oracle's own output of layer i - 1), with the decode inputs, saved for the GPU ranks."""
    import threading

    from oracle import cpu_model as om

    pkg = importlib.import_module("qwen38-27b-aws_b200")
    cfg = pkg.config.full_config(num_blocks=1)
    w = _block_weights(pkg, cfg)
    batch = 8
    g = torch.Generator().manual_seed(0)
    position = torch.randint(0, 510, (batch,), generator=g, dtype=torch.int32)
    emb = pkg.weights.embedding_rows(cfg, torch.randint(0, cfg.vocab_size, (batch,), generator=g).tolist())
    emb = emb.reshape(batch, 1, -1).to(torch.bfloat16)
    cos, sin = om.rotary(cfg, position, torch.bfloat16)
    inputs = dict(cos=cos.unsqueeze(1), sin=sin.unsqueeze(1), position=position, active=torch.ones(batch))

    class RankSum:
        """The TP all-reduce for oracle ranks in threads: fp32 sum in rank order, back to the dtype."""

        def __init__(self, n):
            self.vals, self.out = {}, None
            self.bar = threading.Barrier(n, action=self._sum)

        def _sum(self):
            acc = None
            for r in sorted(self.vals):
                acc = self.vals[r].float() if acc is None else acc + self.vals[r].float()
            self.out, self.vals = acc, {}

        def bind(self, r):
            def reduce(t):
                self.vals[r] = t
                self.bar.wait()
                return self.out.to(t.dtype)
            return reduce

    reducer = RankSum(world)
    oracles = []
    for rr in range(world):
        shard = {}
        for i in range(cfg.num_hidden_layers):
            shard |= pkg.weights.shard_layer(cfg, w, i, rr, world)
        oracles.append(om.OracleStep(cfg, shard, 512, batch, tp_degree=world, rank=rr, all_reduce=reducer.bind(rr)))
    xs = [emb]
    for i in range(cfg.num_hidden_layers):
        outs = {}

        def run(rr):
            outs[rr] = oracles[rr].layer(i, xs[-1], **inputs)

        threads = [threading.Thread(target=run, args=(rr,)) for rr in range(world)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        xs.append(outs[0])
    torch.save({"emb": emb, "inputs": inputs, "layers": xs}, path)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_gemm_allreduce_and_tp_step(world, tmp_path):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    oracle_path = tmp_path / f"oracle_tp{world}.pt"
    _oracle_layers(world, oracle_path)
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue, str(oracle_path))) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, results, err = queue.get(timeout=900)
            got[rank] = (results, err)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, (results, err) in sorted(got.items()):
        assert err is None, f"rank {rank}:\n{err}"
        bad = [(n, m) for n, ok, m in results if not ok]
        assert not bad, f"rank {rank}: {bad}"
