"""Benchmark of the hot path: decode steps of the 64-layer FP8 model (BASELINE config 3 shape).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--batch 256]

One step = one decode token for each of `--batch` rows through all 64 layers (48 gated-delta + 16
attention) plus the lm_head group-of-32 maxima, rows at positions spread over [0, 511) of a
512-position context, each advancing one position per step (a row reaching 511 restarts at 0 as a
new sequence, as the reference's batched loop refills rows). N GPUs run tensor parallel (TP = N,
heads and vocabulary sliced, row-parallel outputs summed): the total work is fixed, so scaling is
"strong". Weights are seeded random FP8 of the real architecture; cache and recurrent-state contents
are seeded random values (the bytes moved are the same as a real prompt's).

The JSON line's `value` is tokens/s with the step inputs already on the device; `e2e` is the same
through the reference-facing calls (B200Step(**host tensors) -> host hidden, B200Head.next_tokens ->
host token ids, as ChipHead.next_tokens returns them), host<->device copies included. `step_roofline` sets the algorithmic HBM bytes of one
whole decode step against the step time; `prefill` is one 512-token chunk of one row through all
layers, device-timed (the prefill half of the tokens/s metric). A step ends with each row's greedy token
(the exact recheck of the best 4 groups included). `--impl reference` times the reference's own CPU
branches (its Qwen38Step and HeadStep, copied into oracle/_ref by oracle/build_ref.py; the oracle's
restatement where that copy is absent) on this host's cores on a bounded sample: one 4-layer block per
step at the same batch, scaled to 64 layers, plus one head call.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import platform
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
PACKAGE = "qwen38-27b-aws_b200"
# BASELINE.json's metric. `value` is its decode half at config 3 (tokens/s of 64-layer decode steps with the
# lm_head maxima and each row's greedy token); `serve` is prefill + decode together; at N > 1
# `fused_allreduce` is config 1 (the fused GEMM + all-reduce against its roofline and against NCCL).
METRIC = "total tokens/s (prefill+decode) at 1/2/4/8 B200; fused GEMM+AR % of roofline"
MAX_SEQ = 512
GDN_TRAFFIC_B256 = 777.4e6  # dram__bytes per gdn_decode_kernel launch, batch 256, one GPU (ncu)
LAYERS = 64
SERVE_PROMPT = (32, 224)  # prompt lengths of the serving sample
SERVE_CHUNK = 256
SERVE_NEW = 32


def peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class ClockSampler:
    """nvidia-smi samples during the timed region (clocks and throttle reasons). The sampler starts
    before the region and is waited for until its first sample arrives (nvidia-smi takes a few hundred
    ms to start); samples are read by a thread with their arrival time, and those that arrive between
    `begin()` and `end()` (plus one sampling interval) are the region's."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    INTERVAL_MS = 20

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.t0 = self.t1 = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line))

    def start(self):
        import threading

        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.INTERVAL_MS)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.reader = threading.Thread(target=self._read, daemon=True)
        self.reader.start()
        deadline = time.monotonic() + 10.0
        while not self.lines and time.monotonic() < deadline and self.proc.poll() is None:
            time.sleep(0.01)

    def begin(self):
        self.t0 = time.monotonic()

    def end(self):
        self.t1 = time.monotonic()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(2 * self.INTERVAL_MS / 1e3)  # the region's last sample arrives after it is taken
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.reader.join(timeout=10)
        t0 = self.t0 if self.t0 is not None else float("-inf")
        t1 = (self.t1 if self.t1 is not None else float("inf")) + 2 * self.INTERVAL_MS / 1e3
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for when, line in self.lines:
            if not t0 <= when <= t1:
                continue
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def max_over_ranks(value: float, world: int, device) -> float:
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------------
def run_ours(args, world, rank, local):
    pkg = importlib.import_module(PACKAGE)
    step_mod = importlib.import_module(f"{PACKAGE}.step")
    ops = importlib.import_module(f"{PACKAGE}.ops")
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group("nccl", device_id=device, timeout=__import__("datetime").timedelta(seconds=300))
    cfg = pkg.config.full_config(num_blocks=LAYERS // 4)
    B = args.batch

    t0 = time.time()
    step = step_mod.B200Step(cfg, lambda i: pkg.weights.synthetic_layer(cfg, i, seed=0, device=device), MAX_SEQ, B,
                             tp_degree=world, rank=rank, device=device)
    head = step_mod.B200Head(cfg, pkg.weights.synthetic_head(cfg, seed=0, device=device), B, tp_degree=world, rank=rank,
                             device=device)
    torch.cuda.synchronize()
    build_s = time.time() - t0

    # Seeded cache and state contents.
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + rank)
    for l in step.layers:
        if l.kind == pkg.config.LINEAR:
            l.mixer.state.normal_(0.0, 0.1, generator=gen)
            l.mixer.conv_state.normal_(0.0, 1.0, generator=gen)
        else:
            l.mixer.k_cache.normal_(0.0, 1.0, generator=gen)
            l.mixer.v_cache.normal_(0.0, 1.0, generator=gen)

    # Step inputs for every warm-up and timed step, made up front (host and device copies).
    total = args.warmup + args.steps
    g_cpu = torch.Generator().manual_seed(99)
    pos0 = torch.randint(0, MAX_SEQ - 1, (B,), generator=g_cpu)
    positions = torch.stack([(pos0 + s) % (MAX_SEQ - 1) for s in range(total)]).to(torch.int32)
    embeds = (torch.randn(total, B, cfg.hidden_size, generator=g_cpu) * 0.02).to(torch.bfloat16)
    om_rot = lambda p: rotary(cfg, p)  # noqa: E731
    cs = [om_rot(positions[s]) for s in range(total)]
    host = [dict(inputs_embeds=embeds[s].reshape(B, 1, -1).pin_memory(), cos=cs[s][0].unsqueeze(1).pin_memory(),
                 sin=cs[s][1].unsqueeze(1).pin_memory(), position=positions[s].pin_memory(),
                 active=torch.ones(B).pin_memory()) for s in range(total)]
    dev_inputs = [{k: v.to(device) for k, v in h.items()} for h in host]

    tokens_dev = torch.zeros(B, dtype=torch.int32, device=device)
    slot_l = torch.zeros(B, 4, dtype=torch.float32, device=device)
    slot_t = torch.zeros(B, 4, dtype=torch.int32, device=device)

    def device_step(s):
        """One greedy token per row with everything resident: the 64 layers, the lm_head group maxima and
        the exact recheck of the best 4 groups, tokens left on the device."""
        d = dev_inputs[s]
        step.load_decode_inputs(d["inputs_embeds"], d["cos"], d["sin"], d["position"], d["active"])
        hidden = step.decode_device()
        head.hidden.copy_(hidden)
        maxima = head.maxima_device()
        if world == 1:
            ops.lm_head_recheck(head.hidden, head.norm_w, cfg.rms_norm_eps, maxima, head.lm_head, 0, 4, tokens=tokens_dev)
        else:
            ops.lm_head_recheck(head.hidden, head.norm_w, cfg.rms_norm_eps, maxima, head.lm_head, rank * head.vocab_local,
                                4, slot_logits=slot_l, slot_tokens=slot_t)
            torch.distributed.all_reduce(slot_l, op=torch.distributed.ReduceOp.MAX)
            torch.distributed.all_reduce(slot_t, op=torch.distributed.ReduceOp.MAX)
            ops.lm_head_pick(slot_l, slot_t, tokens_dev)
        return tokens_dev

    # Warm-up (also captures the decode graph).
    for s in range(args.warmup):
        device_step(s)
    torch.cuda.synchronize()

    # L2 note: every step streams ~24 GB of weights and ~40 GB of state, far above the 126 MB L2.
    sampler = ClockSampler(local)
    sampler.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.begin()
    start.record()
    for s in range(args.warmup, total):
        device_step(s)
    end.record()
    torch.cuda.synchronize()
    sampler.end()
    if world > 1:
        torch.distributed.barrier()
    dev_ms = max_over_ranks(start.elapsed_time(end), world, device)
    clocks = sampler.stop()

    # End to end through the reference-facing calls, host tensors in and out.
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e_start.record()
    for s in range(args.warmup, total):
        hidden = step(**host[s])  # NeuronStep's call: host tensors in, the hidden state back on the host
        head.next_tokens(hidden)  # ChipHead.next_tokens' call: group maxima and the exact recheck, token ids back
    e_end.record()
    torch.cuda.synchronize()
    wall_e2e = time.perf_counter() - w0
    e2e_ms = max_over_ranks(max(e_start.elapsed_time(e_end), wall_e2e * 1e3), world, device)
    h2d = sum(v.numel() * v.element_size() for v in host[0].values()) + B * cfg.hidden_size * 2
    d2h = B * cfg.hidden_size * 2 + B * 4

    # Roofline of the dominant kernel (gdn_decode): each launch moves the state tiles in and out,
    # the conv state in and out, and reads its qkvz/ab rows and writes the e5m2 output.
    gdn_ms = time_gdn_launches(step, ops, pkg, repeats=3)
    hv = cfg.linear_num_value_heads // world
    per_launch = (B * hv * cfg.linear_key_head_dim * cfg.linear_value_head_dim * 2 * 2
                  + B * (cfg.linear_conv_dim // world) * 3 * 2 * 2
                  + B * ((cfg.linear_conv_dim + cfg.linear_value_dim) // world + 2 * hv) * 2
                  + B * (cfg.linear_value_dim // world))
    peak, peak_kind = peaks()
    achieved = per_launch / (gdn_ms * 1e-3) / 1e9

    # Prefill: one MAX_SEQ-token chunk of one row (slot 0, position 0) through all layers, inputs
    # resident, timed on the device after one untimed chunk.
    C, chunks = MAX_SEQ, 3
    p_emb = (torch.randn(1, C, cfg.hidden_size, generator=g_cpu) * 0.02).to(torch.bfloat16).to(device)
    p_cos, p_sin = (t.unsqueeze(0).to(device) for t in rotary(cfg, torch.arange(C)))
    step.prefill(p_emb, p_cos, p_sin, slot=0, start=0, n_valid=C)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    p_start, p_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_start.record()
    for _ in range(chunks):
        step.prefill(p_emb, p_cos, p_sin, slot=0, start=0, n_valid=C)
    p_end.record()
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(p_start.elapsed_time(p_end), world, device) / chunks

    # Serving (the prefill half and the decode half of "total tokens/s" together): every slot takes a
    # seeded prompt, prefilled in chunks through the step's prefill call, then greedy decode steps; the
    # reference's Scheduler.run without speculation (serve.py), timed on the host clock end to end.
    serve_mod = importlib.import_module(f"{PACKAGE}.serve")
    table = pkg.weights.synthetic_embedding_table(cfg, seed=0, device=device)
    embeddings = serve_mod.Embeddings(table)
    g_serve = torch.Generator().manual_seed(7)
    lens = torch.randint(SERVE_PROMPT[0], SERVE_PROMPT[1] + 1, (B,), generator=g_serve).tolist()
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g_serve).tolist() for n in lens]
    serve_mod.serve(step, head, embeddings, prompts[:2], 2, chunk=SERVE_CHUNK)  # first use of the chunk size
    if world > 1:
        torch.distributed.barrier()
    served = serve_mod.serve(step, head, embeddings, prompts, SERVE_NEW, chunk=SERVE_CHUNK)
    serve_s = max_over_ranks(served.wall_s, world, device)
    del table, embeddings

    # BASELINE config 1 at TP = N: the fused GEMM + all-reduce against its roofline and against NCCL.
    fused_ar = None
    if world > 1:
        fused_ar = {"workload": "BASELINE config 1: down_proj (17408 / t -> 5120) at M rows: plain GEMM, fused GEMM + "
                                "all-reduce, GEMM + NCCL all-reduce; CUDA graphs of 20 launches, max over ranks",
                    "rows": allreduce_rows(world, rank, device, (64, 256, 512), (("down_proj", 17408 // world),), 20)}

    tokens = B * args.steps
    step_bytes = decode_step_bytes(step, head, pkg.config.LINEAR, positions[args.warmup:])
    line = {
        "metric": METRIC,
        "value": tokens / (dev_ms / 1e3),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dev_ms / args.steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8(e4m3 weights x e5m2 activations)+bf16",
        "data": "synthetic (seeded random FP8 weights of the architecture, random cache/state contents)",
        "config": {
            "workload": "BASELINE config 3: 64-layer decode steps, batch %d, 512-position context, rows at positions "
                        "spread over [0,511) (the metric's decode half; `serve` has prefill + decode)" % B,
            "global_batch": B,
            "seq_len": MAX_SEQ,
            "parallelism": f"tp{world}",
            "l2": "inputs larger than L2 (24 GB weights + ~40 GB state streamed per step)",
        },
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "roofline": {
            "kernel": "gdn_decode (q/k prep + per-value-head kernel, timed together)",
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            # dram__bytes_read.sum + dram__bytes_write.sum of one gdn_decode_kernel launch from an ncu capture
            # at batch 256 on one GPU (the shape this line times at N = 1); other shapes were not captured.
            "traffic": GDN_TRAFFIC_B256 if (B == 256 and world == 1) else None,
            "traffic_source": "ncu capture, batch 256, one GPU" if (B == 256 and world == 1) else None,
            "bytes_per_launch": per_launch,
            "launch_ms": gdn_ms,
        },
        # The whole step against HBM: the algorithmic bytes of one decode step (FP8 weights and scales,
        # the BF16 lm_head and in_proj_b/a, gated-delta and conv state in and out, the KV cache below
        # each row's position) over the measured step time.
        "step_roofline": {
            "bytes_per_step": step_bytes,
            "achieved": step_bytes / (dev_ms / args.steps * 1e-3) / 1e9,
            "peak": peak,
            "unit": "GB/s",
            "frac": step_bytes / (dev_ms / args.steps * 1e-3) / 1e9 / peak,
        },
        "prefill": {
            "workload": f"one {C}-token chunk of one row through all {LAYERS} layers (device-timed, {chunks} chunks)",
            "ms_per_chunk": prefill_ms,
            "tokens_per_s": C / (prefill_ms / 1e3),
        },
        "serve": {
            "workload": f"{B} prompts of U[{SERVE_PROMPT[0]}, {SERVE_PROMPT[1]}] seeded tokens, prefilled in "
                        f"{SERVE_CHUNK}-token chunks one row at a time, then {SERVE_NEW} greedy tokens each "
                        "(prefill-first slots, B200Step + B200Head.next_tokens, host clock)",
            "total_tokens_per_s": (served.prompt_tokens + served.generated_tokens) / serve_s,
            "prompt_tokens": served.prompt_tokens,
            "generated_tokens": served.generated_tokens,
            "seconds": serve_s,
            "prefill_seconds": served.prefill_s,
            "decode_seconds": served.decode_s,
            "prefill_calls": served.prefill_calls,
            "decode_steps": served.decode_steps,
        },
        "fused_allreduce": fused_ar,
        "clocks": clocks,
        # the step's kernels, then rmsnorm + group maxima + recheck (+ pick with TP > 1)
        "gpu_launches": (step.kernels_per_decode_step() + 3 + (world > 1)) * args.steps,
        "build_s": round(build_s, 1),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, pkg, B, samples=1)
    if rank == 0:
        print(json.dumps(line), flush=True)
    step.close()  # the decode graph and the communicator's peer mappings go before the process group
    del step, head
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def decode_step_bytes(step, head, linear_kind: str, positions: torch.Tensor) -> int:
    """HBM bytes one decode step must move on this rank, averaged over the timed steps' positions. The
    lm_head counts as FP8 with its scales (the checkpoint's format and the algorithmic figure), although
    the kernel streams it as BF16 (twice the bytes: at 256 rows it is bound by the BF16 tensor rate)."""
    fp8 = lambda lin: lin.out_features * lin.in_features * 33 // 32  # e4m3 bytes + UE8M0 per 32  # noqa: E731
    total = fp8(head.lm_head)
    kv_positions = positions.clamp(max=MAX_SEQ).long().sum(dim=1).float().mean().item()
    for l in step.layers:
        total += fp8(l.gate_up) + fp8(l.down)
        if l.kind == linear_kind:
            m = l.mixer
            total += fp8(m.qkvz) + fp8(m.out) + m.ab.out_features * m.ab.in_features * 2
            total += m.state.numel() * 2 * 2 + m.conv_state.numel() * 2 * 2
        else:
            m = l.mixer
            kvh, hd = m.k_cache.shape[1], m.k_cache.shape[3]
            total += fp8(m.qkv) + fp8(m.o) + int(kv_positions * kvh * hd * 2 * 2)
    return int(total)


def time_gdn_launches(step, ops, pkg, repeats: int) -> float:
    """Average duration of one layer's gated-delta decode (its q/k prep + decode launches) right after the
    timed region: the 48 layers' launches over their own states, captured as one CUDA graph as in the
    step (no host launch gaps between them), replayed `repeats` times between CUDA events on the
    launching stream."""
    cfg, tp = step.cfg, step.tp
    stream = torch.cuda.current_stream()
    layers = [l for l in step.layers if l.kind == pkg.config.LINEAR]

    def run():
        for l in layers:
            m = l.mixer
            ops.gdn_decode(step.proj, step.ab, m.conv_state, m.conv_w, m.a_log, m.dt_bias, m.norm_w, m.state,
                           step.position, step.active, step.mix_gdn, batch=step.batch,
                           num_k_heads=cfg.linear_num_key_heads // tp, num_v_heads=cfg.linear_num_value_heads // tp,
                           head_k=cfg.linear_key_head_dim, head_v=cfg.linear_value_head_dim, eps=cfg.rms_norm_eps,
                           workspace=step.gdn_workspace)

    run()  # outside capture first (module loading, attributes)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(repeats):
        graph.replay()
    b.record(stream)
    torch.cuda.synchronize()
    del graph
    return a.elapsed_time(b) / (repeats * len(layers))


def rotary(cfg, positions):
    dim = cfg.rotary_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    f = positions.float().unsqueeze(-1) * inv
    return f.cos().repeat(1, 2).to(torch.bfloat16), f.sin().repeat(1, 2).to(torch.bfloat16)


# ------------------------------------------------------------------------------------------------
def cpu_block_step(cfg, pkg, batch: int):
    """One decode step of one full-width 4-layer block (3 gated-delta + 1 attention layer) on the host's
    cores, at `batch` rows over seeded cache and state contents, and a function running it. The
    reference's own Qwen38Step CPU branch when its package is in oracle/_ref (oracle/build_ref.py), else
    the oracle's restatement of it. Returns (run, kind)."""
    from oracle import ref_step

    block = pkg.config.block_config(cfg, 4)
    gen = torch.Generator().manual_seed(5)
    pos = torch.randint(0, MAX_SEQ - 2, (batch,), generator=gen, dtype=torch.int32)
    x = (torch.randn(batch, 1, cfg.hidden_size, generator=gen) * 0.02).to(torch.bfloat16)
    if ref_step.available():
        model, rcfg, rgen = ref_step.reference_block(block, batch, MAX_SEQ)
        for layer in model.layers:
            if hasattr(layer, "linear_attn"):
                layer.linear_attn.recurrent_state.normal_(0.0, 0.1, generator=gen)
            else:
                layer.self_attn.k_cache.normal_(0.0, 1.0, generator=gen)
                layer.self_attn.v_cache.normal_(0.0, 1.0, generator=gen)
        inputs = rgen.batch_step_inputs(rcfg, pos.tolist(), MAX_SEQ, torch.bfloat16, [True] * batch)

        def run():
            with torch.no_grad():
                return model(inputs_embeds=x, **inputs)

        return run, "reference"
    from oracle import cpu_model as om

    w = {}
    for i in range(4):
        w |= pkg.weights.synthetic_layer(cfg, i, seed=0, device="cpu")
    st = om.OracleStep(block, w, MAX_SEQ, batch)
    for kind, mixer, *_ in st.layers:
        if kind == om.LINEAR:
            mixer.recurrent_state.normal_(0.0, 0.1, generator=gen)
        else:
            mixer.k_cache.normal_(0.0, 1.0, generator=gen)
            mixer.v_cache.normal_(0.0, 1.0, generator=gen)
    cos, sin = om.rotary(cfg, pos, torch.bfloat16)
    inputs = dict(cos=cos.unsqueeze(1), sin=sin.unsqueeze(1), position=pos, active=torch.ones(batch))
    return (lambda: st(inputs_embeds=x, **inputs)), "port"


def cpu_head_seconds(cfg, pkg, batch: int) -> tuple[float, str]:
    """One call of the head on the host's cores: the reference's HeadStep CPU branch (fp32 logits over the
    whole vocabulary and their group maxima) when available, else the oracle's restatement."""
    from oracle import ref_step

    x = (torch.randn(batch, 1, cfg.hidden_size, generator=torch.Generator().manual_seed(6))).to(torch.bfloat16)
    if ref_step.available():
        hstep = ref_step.reference_head(cfg, batch)
        with torch.no_grad():
            t0 = time.perf_counter()
            hstep(x)
            return time.perf_counter() - t0, "reference"
    from oracle import cpu_model as om

    head = pkg.weights.synthetic_head(cfg, 0, "cpu")
    t0 = time.perf_counter()
    om.head_maxima(cfg, x, head["norm_weight"], head["lm_head"].q, head["lm_head"].scale)
    return time.perf_counter() - t0, "port"


def cpu_step(cfg, pkg, batch: int, steps: int, warmup: int) -> dict:
    """The CPU baseline of one decode step of the 64-layer model at `batch` rows: one 4-layer block timed
    over `steps` runs (after `warmup`), times 16, plus one timed head call over the whole vocabulary."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    run, kind = cpu_block_step(cfg, pkg, batch)
    for _ in range(max(1, warmup)):
        run()
    t0 = time.perf_counter()
    for _ in range(steps):
        run()
    per_block = (time.perf_counter() - t0) / steps
    head_s, _ = cpu_head_seconds(cfg, pkg, batch)
    step_s = per_block * (LAYERS // 4) + head_s
    who = "the reference's own Qwen38Step / HeadStep CPU branches" if kind == "reference" else "the oracle's restatement"
    return {"value": batch / step_s, "unit": "tokens/s", "cores": threads, "kind": kind, "step_s": step_s,
            "sample": f"{who}: one full-width 4-layer block (3 gated-delta + 1 attention) decoding {batch} rows, "
                      f"{steps} runs at {per_block:.2f} s, x{LAYERS // 4} for 64 layers, plus one head call over the "
                      f"whole vocabulary ({head_s:.2f} s); CPU {platform.processor() or platform.machine()}"}


def cpu_baseline(cfg, pkg, batch: int, samples: int) -> dict:
    out = cpu_step(cfg, pkg, batch, samples, 1)
    out.pop("step_s")
    return out


def run_reference(args, world, rank, local):
    """The reference arm: the reference's own CPU implementation on this host's cores, rank 0 only."""
    if rank != 0:
        return
    pkg = importlib.import_module(PACKAGE)
    cfg = pkg.config.full_config(num_blocks=LAYERS // 4)
    base = cpu_step(cfg, pkg, args.batch, args.steps, args.warmup)
    step_s = base.pop("step_s")
    value = base["value"]
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp8 weights dequantised to bf16 (CPU)", "data": "synthetic", "impl": "reference",
        "config": {"workload": "BASELINE config 3 decode step, batch %d; per step one 4-layer block timed, x16, plus "
                               "the head" % args.batch,
                   "global_batch": args.batch, "seq_len": MAX_SEQ, "parallelism": "cpu"},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_micro(args):
    """One kernel alone, for profiling and per-kernel rooflines: `gdn` (BASELINE config 2 decode shape,
    48 value heads, dk = dv = 128) or `gemm` (config 1, the down_proj shape 17408 -> 5120)."""
    pkg = importlib.import_module(PACKAGE)
    ops = importlib.import_module(f"{PACKAGE}.ops")
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    cfg = pkg.config.full_config(1)
    B = args.batch
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    bf = lambda *s: (torch.randn(*s, device=dev, generator=gen)).to(torch.bfloat16)  # noqa: E731
    peak, peak_kind = peaks()
    if args.micro == "gdn":
        hv, dk, dv = cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        conv_dim = cfg.linear_conv_dim
        states = [(bf(B, hv, dk, dv) * 0.1, bf(B, conv_dim, 3)) for _ in range(args.copies)]
        qkvz, ab = bf(B, conv_dim + cfg.linear_value_dim), bf(B, 2 * hv)
        conv_w, a_log, dt, nw = bf(conv_dim, 4) * 0.1, bf(hv) * 0.1, bf(hv) * 0.1, bf(dv) * 0.1
        pos = torch.randint(1, 500, (B,), device=dev, dtype=torch.int32)
        act = torch.ones(B, device=dev)
        out = torch.empty(B, cfg.linear_value_dim, dtype=torch.uint8, device=dev)

        def launch(i):
            st, cs = states[i % len(states)]
            ops.gdn_decode(qkvz, ab, cs, conv_w, a_log, dt, nw, st, pos, act, out, batch=B, num_k_heads=cfg.linear_num_key_heads,
                           num_v_heads=hv, head_k=dk, head_v=dv, eps=1e-6)
        per = B * hv * dk * dv * 2 * 2 + B * conv_dim * 3 * 2 * 2 + B * (conv_dim + cfg.linear_value_dim + 2 * hv) * 2 + B * cfg.linear_value_dim
        unit, bound = "GB/s", "hbm"
    elif args.micro == "attn":
        # One attention layer's decode at BASELINE config 3: positions U[0, 512), BF16 cache of 512.
        heads, kvh, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        caches = [(bf(B, kvh, MAX_SEQ, hd), bf(B, kvh, MAX_SEQ, hd)) for _ in range(args.copies)]
        qkv = bf(B, heads * 2 * hd + 2 * kvh * hd)
        qn, kn = bf(hd) * 0.1, bf(hd) * 0.1
        pos = torch.randint(0, MAX_SEQ - 1, (B,), device=dev, dtype=torch.int32, generator=gen)
        cs, sn = bf(B, cfg.rotary_dim), bf(B, cfg.rotary_dim)
        act = torch.ones(B, device=dev)
        out = torch.empty(B, heads * hd, dtype=torch.uint8, device=dev)

        order = ops.attn_row_order(pos, act, MAX_SEQ, torch.empty(B, dtype=torch.int32, device=dev))

        def launch(i):
            kc, vc = caches[i % len(caches)]
            ops.attn_decode(qkv, qn, kn, cs, sn, kc, vc, pos, act, out, batch=B, num_q_heads=heads, num_kv_heads=kvh,
                            head_dim=hd, rot_dim=cfg.rotary_dim, eps=1e-6, row_order=order)
        per = int(pos.sum().item()) * kvh * hd * 2 * 2 + B * qkv.shape[1] * 2 + B * heads * hd + B * kvh * hd * 2 * 2
        unit, bound = "GB/s", "hbm"
    elif args.micro == "attn_long":
        # BASELINE config 4's attention decode (or K-token verify): 4 rows (--batch) at positions U[30000, 32000) of a
        # 32,768-position cache (the long-context agent workload), one layer at TP = --tp head counts,
        # split along the cache (q38_attn_split); --kv fp8 reads the FP8 e4m3 cache. Bytes: the K and V
        # rows below each position, plus the row's inputs and outputs.
        B = args.batch if args.batch_given else 4
        max_seq = 32768
        heads, kvh, hd = cfg.num_attention_heads // args.tp, cfg.kv_heads_per_rank(args.tp), cfg.head_dim
        fp8 = args.kv == "fp8"
        mk = (lambda: bf(B, kvh, max_seq, hd).float().to(torch.float8_e4m3fn).view(torch.uint8)) if fp8 else (
            lambda: bf(B, kvh, max_seq, hd))
        caches = [(mk(), mk()) for _ in range(args.copies)]
        K = args.verify_tokens
        qkv = bf(B * K, heads * 2 * hd + 2 * kvh * hd)
        qn, kn = bf(hd) * 0.1, bf(hd) * 0.1
        pos = torch.randint(30000, 32000, (B,), device=dev, dtype=torch.int32, generator=gen)
        cs, sn = bf(B * K, cfg.rotary_dim), bf(B * K, cfg.rotary_dim)
        act = torch.ones(B, device=dev)
        out = torch.empty(B * K, heads * hd, dtype=torch.uint8, device=dev)
        ws = torch.empty(ops.attn_split_workspace_bytes(B, heads, kvh, K, max_seq, hd), dtype=torch.uint8, device=dev)
        scales = (2.0 ** -4, 2.0 ** -5) if fp8 else None

        def launch(i):
            kc, vc = caches[i % len(caches)]
            ops.attn_split(qkv, qn, kn, cs, sn, kc, vc, pos, act, out, batch=B, tokens=K, num_q_heads=heads,
                           num_kv_heads=kvh, head_dim=hd, rot_dim=cfg.rotary_dim, eps=1e-6, kv_scales=scales, workspace=ws)
        per = int(pos.sum().item()) * kvh * hd * (1 if fp8 else 2) * 2 + B * K * (qkv.shape[1] * 2 + heads * hd)
        unit, bound = "GB/s", "hbm"
    elif args.micro == "gemm":
        k, n = cfg.intermediate_size // args.tp, cfg.hidden_size
        if args.shape:
            n, k = (int(v) for v in args.shape.split(","))
        lins = [ops.DeviceLinear(pkg.weights.FP8Weight.from_float(torch.randn(n, k, device=dev, generator=gen) * 0.02), dev)
                for _ in range(args.copies)]
        x = pkg.codec.to_e5m2_bytes(bf(B, k))
        y = torch.zeros(B, n, dtype=torch.bfloat16, device=dev)
        splits = args.splits or ops.choose_splits(B, n, k)
        if args.streamk:  # the row-parallel form at TP = 1: stream-K with the residual epilogue
            ws = torch.zeros(ops.streamk_workspace_bytes(B, n, k), dtype=torch.uint8, device=dev)

            def launch(i):
                ops.fp8_gemm_streamk(x, lins[i % len(lins)], y, ws, residual=y)
        else:
            ws = torch.zeros(max(256, ops.gemm_workspace_bytes(B, n, splits)), dtype=torch.uint8, device=dev)

            def launch(i):
                ops.fp8_gemm(x, lins[i % len(lins)], y, splits=splits, workspace=ws)
        per = n * k + n * (k // 32) + B * k + B * n * 2
        unit, bound = "GB/s", "hbm"
    elif args.micro == "gemm_silu":
        # The MLP's gate/up GEMM with SiLU(gate) * up in the epilogue (hidden -> 2 x intermediate).
        k, inter = cfg.hidden_size, cfg.intermediate_size // args.tp
        rnd = lambda: pkg.weights.FP8Weight.from_float(torch.randn(inter, k, device=dev, generator=gen) * 0.02)  # noqa: E731
        lins = [ops.DeviceLinear(pkg.weights.FP8Weight.interleave_rows(rnd(), rnd()), dev) for _ in range(args.copies)]
        x = pkg.codec.to_e5m2_bytes(bf(B, k))
        y = torch.empty(B, inter, dtype=torch.uint8, device=dev)

        def launch(i):
            ops.fp8_gemm_silu(x, lins[i % len(lins)], y)
        per = 2 * inter * k + 2 * inter * (k // 32) + B * k + B * inter
        unit, bound = "GB/s", "hbm"
    if args.micro == "gdn_prefill":
        # one 512-token prefill chunk through the gated delta rule (48 value heads,
        # dk = dv = 128), continuing a row (start > 0). Work: the chunked rule's fp32 products.
        T = 512
        hk, hv, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        conv_dim = cfg.linear_conv_dim
        states = [(bf(1, hv, dk, dv) * 0.1, bf(1, conv_dim, 3)) for _ in range(args.copies)]
        qkvz, ab = bf(T, conv_dim + cfg.linear_value_dim), bf(T, 2 * hv)
        conv_w, a_log, dt, nw = bf(conv_dim, 4) * 0.1, bf(hv) * 0.1, bf(hv) * 0.1, bf(dv) * 0.1
        out = torch.empty(T, cfg.linear_value_dim, dtype=torch.uint8, device=dev)
        ws = torch.empty(ops.gdn_prefill_workspace_bytes(T, hk, hv, dk, dv), dtype=torch.uint8, device=dev)

        def launch(i):
            st, cs = states[i % len(states)]
            ops.gdn_prefill(qkvz, ab, cs, conv_w, a_log, dt, nw, st, out, ws, slot=0, start=512, n_valid=T,
                            num_k_heads=hk, num_v_heads=hv, head_k=dk, head_v=dv, eps=1e-6)
        per = hv * dk * dv * 2 * 2 + T * (conv_dim + cfg.linear_value_dim + 2 * hv) * 2 + T * cfg.linear_value_dim
        # fp32 FLOPs per chunk (64-token sub-chunks): K K^T, Q K^T (2 C^2 dk) per 32-column slice, the
        # state products (3 C dk DVS), the solve and the attention-to-delta product, per head and slice.
        C, slices = 64, dv // 32
        flops = 2 * hv * slices * (T // C) * (2 * C * C * dk + 3 * C * dk * 32 + C * C * 32)
        unit, bound = "GB/s", "fp32 FMA (SIMT)"
    if args.micro == "attn_prefill":
        # BASELINE config 0's prefill attention: a 512-token chunk of a row continuing 512 positions
        # (cache of 1024), 24 query / 4 KV heads of 256.
        T, start, mseq = 512, 512, 1024
        heads, kvh, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        caches = [(bf(1, kvh, mseq, hd), bf(1, kvh, mseq, hd)) for _ in range(args.copies)]
        qkv = bf(T, heads * 2 * hd + 2 * kvh * hd)
        qn, kn = bf(hd) * 0.1, bf(hd) * 0.1
        cs, sn = bf(T, cfg.rotary_dim), bf(T, cfg.rotary_dim)
        out = torch.empty(T, heads * hd, dtype=torch.uint8, device=dev)
        ws = torch.empty(ops.attn_prefill_workspace_bytes(T, heads, hd), dtype=torch.uint8, device=dev)

        def launch(i):
            kc, vc = caches[i % len(caches)]
            ops.attn_prefill(qkv, qn, kn, cs, sn, kc, vc, out, ws, slot=0, start=start, num_q_heads=heads,
                             num_kv_heads=kvh, head_dim=hd, rot_dim=cfg.rotary_dim, eps=1e-6)
        per = (start + T) * kvh * hd * 2 * 2 + T * qkv.shape[1] * 2 + T * heads * hd
        keys = sum(start + t + 1 for t in range(T))  # visible keys summed over the chunk's tokens
        flops = 2 * heads * keys * hd * 3  # scores twice (two passes per block) and the weighted values
        unit, bound = "GB/s", "fp32 FMA (SIMT)"
    if args.micro == "verify":
        # One gated-delta layer's verify (K = 4 tokens per row, commit-on-accept) at batch B.
        K = 4
        hk, hv, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        conv_dim = cfg.linear_conv_dim
        f32 = lambda *s: torch.randn(*s, device=dev, generator=gen) * 0.1  # noqa: E731
        sets = [(bf(B, hv, dk, dv) * 0.1, bf(B, conv_dim, 3), f32(B, K, hv, dk), f32(B, K, hv, dv), -f32(B, K, hv).abs(),
                 bf(B, K, conv_dim)) for _ in range(args.copies)]
        qkvz, ab = bf(B * K, conv_dim + cfg.linear_value_dim), bf(B * K, 2 * hv)
        conv_w, a_log, dt, nw = bf(conv_dim, 4) * 0.1, bf(hv) * 0.1, bf(hv) * 0.1, bf(dv) * 0.1
        pos = torch.randint(1, 500, (B,), device=dev, dtype=torch.int32, generator=gen)
        act = torch.ones(B, device=dev)
        acc = torch.randint(0, K + 1, (B,), device=dev, dtype=torch.int32, generator=gen)
        out = torch.empty(B * K, cfg.linear_value_dim, dtype=torch.uint8, device=dev)

        def launch(i):
            st, cs, pk, pd, pg, pi = sets[i % len(sets)]
            ops.gdn_verify(qkvz, ab, cs, conv_w, a_log, dt, nw, st, pk, pd, pg, pi, pos, act, acc, out, batch=B,
                           tokens=K, num_k_heads=hk, num_v_heads=hv, head_k=dk, head_v=dv, eps=1e-6)
        per = (B * hv * dk * dv * 2 * 2 + B * conv_dim * 3 * 2 * 2 + B * K * hv * (dk + dv + 1) * 4 * 2
               + B * K * conv_dim * 2 * 2 + B * K * (conv_dim + cfg.linear_value_dim + 2 * hv) * 2)
        unit, bound = "GB/s", "hbm"
    if args.micro == "ab":
        # in_proj_b/a of one GDN layer: BF16 [B, 5120] x [96, 5120]^T.
        k, n = cfg.hidden_size, 2 * cfg.linear_num_value_heads
        lins = [ops.DeviceBF16Linear((torch.randn(n, k, device=dev, generator=gen) * 0.02).to(torch.bfloat16), dev)
                for _ in range(args.copies)]
        x = bf(B, k)
        y = torch.empty(B, n, dtype=torch.bfloat16, device=dev)
        splits = args.splits or ops.bf16_linear_splits(B, n, k)
        ws = torch.zeros(max(256, ops.gemm_workspace_bytes(B, n, splits)), dtype=torch.uint8, device=dev)

        def launch(i):
            ops.bf16_linear(x, lins[i % len(lins)], y, splits=splits, workspace=ws)
        per = n * k * 2 + B * k * 2 + B * n * 2
        unit, bound = "GB/s", "hbm"
    if args.micro == "head":
        # The lm_head group-of-32 maxima over the whole vocabulary (BF16 [vocab, 5120], one rank).
        k, n = cfg.hidden_size, cfg.vocab_size // args.tp
        lins = [ops.DeviceBF16Linear((torch.randn(n, k, device=dev, generator=gen) * 0.02).to(torch.bfloat16), dev)
                for _ in range(min(args.copies, 2))]
        x = bf(B, k)
        maxima = torch.empty(B, n // 32, dtype=torch.float32, device=dev)

        def launch(i):
            ops.lm_head_groupmax(x, lins[i % len(lins)], maxima)
        per = n * k * 2 + B * k * 2 + B * (n // 32) * 4
        flops = 2 * B * n * k
        unit, bound = "GB/s", "hbm"
    for i in range(args.warmup):
        launch(i)
    torch.cuda.synchronize()
    # The K launches are captured in one CUDA graph and timed as one replay, so the host's launch
    # cost never shows between kernels; consecutive launches cycle through `copies` buffers. --eager
    # launches them one by one instead (for profilers, which then see plain kernel launches).
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if args.eager:
        a.record()
        for i in range(args.steps):
            launch(i)
        b.record()
    else:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                launch(i)
        graph.replay()
        torch.cuda.synchronize()
        a.record()
        graph.replay()
        b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    achieved = per / (ms * 1e-3) / 1e9
    extra = {}
    if "flops" in locals():
        extra = {"gflop_per_launch": flops / 1e9, "achieved_tflops": flops / (ms * 1e-3) / 1e12}
    print(json.dumps({"micro": args.micro, "batch": B, "shape": args.shape, "launch_ms": ms, "bytes_per_launch": per, **extra,
                      "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": unit,
                                   "frac": achieved / peak}}), flush=True)


NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this pool (the profiling recipe's figure)


def allreduce_rows(world: int, rank: int, device, batches, shapes, steps: int) -> list[dict]:
    """the row-parallel projection at TP = world, alone, at M rows: the plain GEMM, the
    fused GEMM + all-reduce, and the GEMM followed by an NCCL all-reduce (the baseline), each timed as a
    CUDA graph of `steps` launches, max over ranks. Per shape: hidden = 1 - (fused - gemm) / (nccl - gemm),
    the share of the baseline's communication time the fused kernel hides, and the roofline of the fused
    call: the slowest of its HBM bytes at the measured HBM peak, its FLOPs at the FP8 tensor peak (twice
    the measured BF16 peak), and the all-reduce's NVLink bytes (2 (t - 1) / t x M x 5120 x 2 per rank,
    the reduce-scatter + all-gather minimum) at the measured 770 GB/s per direction."""
    pkg = importlib.import_module(PACKAGE)
    ops = importlib.import_module(f"{PACKAGE}.ops")
    H = 5120
    comm = ops.Communicator(rank, world, max(max(batches), 512), H, device)
    hbm, _ = peaks()
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    bf16_tf = float(json.loads(peaks_path.read_text())["bf16_tflops"]) if peaks_path.exists() else 1590.0
    rows = []
    for B in batches:
        for name, k in shapes:
            g = torch.Generator().manual_seed(rank)
            lin = ops.DeviceLinear(pkg.weights.FP8Weight.from_float(torch.randn(H, k, generator=g) * 0.02), device)
            xq = pkg.codec.to_e5m2_bytes(torch.randn(B, k, generator=g).to(torch.bfloat16)).to(device)
            splits = min(ops.choose_splits(B, H, k), 8)
            ws = torch.zeros(max(256, ops.gemm_workspace_bytes(B, H, splits)), dtype=torch.uint8, device=device)
            part = torch.zeros(B, H, dtype=torch.bfloat16, device=device)
            variants = {
                "gemm": lambda: ops.fp8_gemm(xq, lin, part, splits=splits, workspace=ws),
                "fused": lambda: ops.fp8_gemm_allreduce(xq, lin, comm, splits=splits),
                "gemm+nccl": lambda: (ops.fp8_gemm(xq, lin, part, splits=splits, workspace=ws),
                                      torch.distributed.all_reduce(part)),
            }
            t = {}
            for vname, fn in variants.items():
                for _ in range(3):
                    fn()
                torch.cuda.synchronize()
                torch.distributed.barrier()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for _ in range(steps):
                        fn()
                graph.replay()
                torch.cuda.synchronize()
                torch.distributed.barrier()
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record()
                graph.replay()
                ev1.record()
                torch.cuda.synchronize()
                t[vname] = max_over_ranks(ev0.elapsed_time(ev1), world, device) * 1e3 / steps
                del graph
                torch.distributed.barrier()
            hbm_bytes = H * k * 33 // 32 + B * k + 2 * B * H * 2  # weights + scales, x, residual in and out
            flops = 2 * B * k * H
            nvlink_bytes = 2 * (world - 1) / world * B * H * 2
            bounds = {"hbm_us": hbm_bytes / (hbm * 1e3), "tensor_us": flops / (2 * bf16_tf * 1e6),
                      "nvlink_us": nvlink_bytes / (NVLINK_GBS * 1e3)}
            target = max(bounds.values())
            comm_nccl = t["gemm+nccl"] - t["gemm"]
            rows.append({"shape": name, "M": B, "k": k, "splits": splits, "gemm_us": round(t["gemm"], 2),
                         "fused_us": round(t["fused"], 2), "nccl_us": round(t["gemm+nccl"], 2),
                         "hidden": round(1 - (t["fused"] - t["gemm"]) / comm_nccl, 3) if comm_nccl > 0 else None,
                         "roofline_us": round(target, 2), "roofline_bound": max(bounds, key=bounds.get)[:-3],
                         "roofline_frac": round(target / t["fused"], 3),
                         **{key: round(v, 2) for key, v in bounds.items()}})
    if ops.device_status() != 0:
        raise RuntimeError(f"device status {ops.device_status()} after the fused all-reduce sweep")
    comm.close()
    return rows


def run_micro_allreduce(args, world, rank, local):
    """The config-1 sweep alone (allreduce_rows) at M in {64, 256, 512} rows (or --batch), down_proj
    (17408 / world -> 5120) and o_proj (6144 / world -> 5120)."""
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    torch.distributed.init_process_group("nccl", device_id=device, timeout=__import__("datetime").timedelta(seconds=120))
    batches = [args.batch] if args.batch_given else [64, 256, 512]
    rows = allreduce_rows(world, rank, device, batches, (("down_proj", 17408 // world), ("o_proj", 6144 // world)),
                          args.steps)
    hbm, _ = peaks()
    peaks_path = ROOT / "MEASURED_PEAKS.json"
    bf16_tf = float(json.loads(peaks_path.read_text())["bf16_tflops"]) if peaks_path.exists() else 1590.0
    if rank == 0:
        print(json.dumps({"micro": "gemm_allreduce", "tp": world, "steps": args.steps, "device_status": 0,
                          "peaks": {"hbm_gbs": hbm, "fp8_tflops": 2 * bf16_tf, "nvlink_gbs": NVLINK_GBS},
                          "rows": rows}), flush=True)
    torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--kv", choices=["bf16", "fp8"], default="bf16", help="--micro attn_long: the KV cache format")
    ap.add_argument("--verify-tokens", type=int, default=1, help="--micro attn_long: query tokens per row (4: verify)")
    ap.add_argument("--micro", choices=["gdn", "gemm", "gemm_silu", "head", "attn", "attn_long", "ab", "gdn_prefill", "attn_prefill", "verify", "gemm_ar"],
                    help="time one kernel alone (profiling) instead of the step; gemm_ar: the fused all-reduce under torchrun")
    ap.add_argument("--copies", type=int, default=4, help="--micro: distinct weight/state copies cycled (defeat L2)")
    ap.add_argument("--tp", type=int, default=1, help="--micro gemm: K = 17408 / tp")
    ap.add_argument("--shape", help="--micro gemm: 'features,k' instead of the down_proj shape")
    ap.add_argument("--splits", type=int, default=0, help="--micro gemm/ab: K splits instead of the default choice")
    ap.add_argument("--streamk", action="store_true", help="--micro gemm: the stream-K form with the residual epilogue")
    ap.add_argument("--eager", action="store_true", help="--micro: launch one by one instead of one CUDA graph")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.batch_given = args.batch is not None
    if args.batch is None:
        args.batch = 256
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    world, rank, local = dist_env()
    if args.micro == "gemm_ar":
        run_micro_allreduce(args, world, rank, local)
        return
    if args.micro:
        run_micro(args)
        return
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}; launch N>1 with torch.distributed.run")
    if args.impl == "reference":
        run_reference(args, world, rank, local)
    else:
        run_ours(args, world, rank, local)


if __name__ == "__main__":
    main()
