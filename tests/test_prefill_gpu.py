"""Prefill chunks of one row: the gated-delta and attention prefill kernels against the oracle, and
B200Step's prefill call against the reference's golden vectors and, at full width, the oracle.

Tolerances, stated per check:
* gated-delta e5m2 output (out_proj's input): codes equal or adjacent, adjacent for at most 2%. The
  GPU's chunked rule regroups the CPU branch's fp32 sums (64-token sub-chunks instead of 128, a blocked
  triangular solve instead of the explicit inverse), so bf16 values can move by one ulp.
* attention e5m2 output (o_proj's input): the reference rounds scores to bf16, and scores reach ~16,
  so a one-ulp flip from fp32 summation order moves that key's weight by up to 6% and an output near
  zero by several e5m2 codes. So: codes equal for at least 98%, more than one code apart for at most
  0.1%, and the decoded values within 2e-2 relative L2 per token.
* gated-delta state after the chunk: within 1e-2 absolute (BASELINE) and equal for most elements.
* conv state: bit-exact (it is a copy of bf16 inputs). KV cache written by the chunk: keys within
  1 bf16 ulp (norm and rotary in fp32 sums), values bit-exact.
* hidden states through B200Step: within 2e-2 of the row peak and in relative L2 (BASELINE).
"""

from pathlib import Path

import pytest
import torch
from safetensors import safe_open

from oracle import cpu_model as om
from tests.test_kernels_gpu import assert_attention_e5m2_close, assert_bf16_close, assert_e5m2_close, e5m2_code
from tests.test_step_gpu import assert_hidden_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_block.safetensors"


@pytest.fixture(scope="module")
def ops(pkg):
    return __import__(pkg.__name__ + ".ops", fromlist=["ops"])


@pytest.fixture(scope="module")
def step_mod(pkg):
    return __import__(pkg.__name__ + ".step", fromlist=["step"])


def _scalar(v):
    return torch.tensor([v], dtype=torch.int32)


@pytest.mark.parametrize("shape,tokens,start,n_valid", [("tiny", 16, 0, 16), ("tiny", 16, 16, 11), ("full", 100, 40, 90),
                                                        ("full", 512, 512, 512), ("full", 512, 0, 300)])
def test_gdn_prefill_matches_oracle(pkg, ops, shape, tokens, start, n_valid):
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(21 + tokens + start)
    rows, slot = 3, 1
    w = pkg.weights.synthetic_layer(cfg, 0, seed=11, device="cpu", std=0.1)
    layer = om.GDNLayer(cfg, w, "layers.0", 1, rows, torch.bfloat16)
    layer.recurrent_state.copy_((torch.randn(layer.recurrent_state.shape, generator=gen) * 0.1).to(torch.bfloat16))
    layer.conv_state.copy_(torch.randn(layer.conv_state.shape, generator=gen).to(torch.bfloat16))
    conv_dim, vd, hv = cfg.linear_conv_dim, cfg.linear_value_dim, cfg.linear_num_value_heads
    qkv = torch.randn(tokens, conv_dim, generator=gen).to(torch.bfloat16)
    z = torch.randn(tokens, vd, generator=gen).to(torch.bfloat16)
    b_raw = torch.randn(tokens, hv, generator=gen).to(torch.bfloat16)
    a_raw = torch.randn(tokens, hv, generator=gen).to(torch.bfloat16)
    state0, conv0 = layer.recurrent_state.clone(), layer.conv_state.clone()
    d_state, d_conv = state0.to(DEV), conv0.to(DEV)
    out = torch.empty(tokens, vd, dtype=torch.uint8, device=DEV)
    heads = dict(num_k_heads=cfg.linear_num_key_heads, num_v_heads=hv, head_k=cfg.linear_key_head_dim,
                 head_v=cfg.linear_value_head_dim)
    ws = torch.empty(ops.gdn_prefill_workspace_bytes(tokens, **heads), dtype=torch.uint8, device=DEV)
    ops.gdn_prefill(torch.cat((qkv, z), 1).to(DEV), torch.cat((b_raw, a_raw), 1).to(DEV), d_conv, layer.conv_w.to(DEV),
                    layer.A_log.to(DEV), layer.dt_bias.to(DEV), layer.norm_w.to(DEV), d_state, out, ws, slot=slot,
                    start=start, n_valid=n_valid, eps=cfg.rms_norm_eps, **heads)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    want = layer.prefill_core(qkv, z, b_raw, a_raw, _scalar(slot), _scalar(start), _scalar(n_valid))
    assert_e5m2_close(out.cpu()[:n_valid], want[:n_valid], what="gdn prefill out")
    got_state = d_state.cpu()
    for r in range(rows):
        if r != slot:
            assert torch.equal(got_state[r], state0[r]) and torch.equal(d_conv.cpu()[r], conv0[r]), "another row changed"
    diff = (got_state[slot].float() - layer.recurrent_state[slot].float()).abs()
    assert diff.max().item() < 1e-2, f"state differs by {diff.max().item()}"
    assert (diff == 0).float().mean().item() > 0.9
    assert torch.equal(d_conv.cpu(), layer.conv_state)


@pytest.mark.parametrize("shape,tokens,start,max_seq", [("tiny", 16, 0, 64), ("tiny", 16, 16, 64), ("full", 100, 37, 512),
                                                        ("full", 512, 0, 1024), ("full", 256, 300, 1024)])
def test_attn_prefill_matches_oracle(pkg, ops, shape, tokens, start, max_seq):
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(31 + tokens + start)
    rows, slot = 2, 1
    w = pkg.weights.synthetic_layer(cfg, 3, seed=11, device="cpu", std=0.1)
    layer = om.AttentionLayer(cfg, w, "layers.3", 1, 0, rows, max_seq, torch.bfloat16)
    layer.k_cache.copy_(torch.randn(layer.k_cache.shape, generator=gen).to(torch.bfloat16))
    layer.v_cache.copy_(torch.randn(layer.v_cache.shape, generator=gen).to(torch.bfloat16))
    hd, heads, kvh = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    qg = torch.randn(1, tokens, heads * 2 * hd, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, tokens, kvh * hd, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, tokens, kvh * hd, generator=gen).to(torch.bfloat16)
    cos, sin = om.rotary(cfg, torch.arange(start, start + tokens), torch.bfloat16)
    d_k, d_v = layer.k_cache.to(DEV), layer.v_cache.to(DEV)
    out = torch.empty(tokens, heads * hd, dtype=torch.uint8, device=DEV)
    ws = torch.empty(ops.attn_prefill_workspace_bytes(tokens, heads, hd), dtype=torch.uint8, device=DEV)
    ops.attn_prefill(torch.cat((qg, k, v), -1).reshape(tokens, -1).to(DEV), layer.q_norm.to(DEV), layer.k_norm.to(DEV),
                     cos.to(DEV), sin.to(DEV), d_k, d_v, out, ws, slot=slot, start=start, num_q_heads=heads,
                     num_kv_heads=kvh, head_dim=hd, rot_dim=cfg.rotary_dim, eps=cfg.rms_norm_eps)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    want = layer.prefill_core(qg, k, v, cos.unsqueeze(0), sin.unsqueeze(0), _scalar(slot), _scalar(start))
    assert_attention_e5m2_close(out.cpu(), want.reshape(tokens, -1), what="attention prefill out")
    assert_bf16_close(d_k.cpu(), layer.k_cache, frac=0.001, what="k cache")
    assert torch.equal(d_v.cpu(), layer.v_cache)


@pytest.fixture(scope="module")
def golden():
    with safe_open(str(GOLDEN), "pt") as f:
        return {k: f.get_tensor(k) for k in f.keys()}, f.metadata()


def _inputs(tensors, prefix):
    keys = ("cos", "sin", "position", "active", "slot", "start", "n_valid")
    return {k: tensors[f"{prefix}.{k}"] for k in keys if f"{prefix}.{k}" in tensors}


@pytest.mark.parametrize("use_graph", [False, True])
def test_tiny_decode_prefill_decode_matches_reference_golden(pkg, step_mod, golden, use_graph):
    """The golden sequence: decode steps, a prompt prefilled into slot 1 in two chunks (the second
    partial), then one more decode step for all rows; every output and the final states."""
    tensors, meta = golden
    cfg = pkg.config.tiny_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, int(meta["seed"]), "cpu", float(meta["std"]))
    step = step_mod.B200Step(cfg, w, int(meta["max_seq"]), int(meta["batch"]), use_graph=use_graph)
    for s in range(int(meta["decode_steps"])):
        step(inputs_embeds=tensors[f"decode{s}.x"], **_inputs(tensors, f"decode{s}"))
    for c in range(2):
        y = step(inputs_embeds=tensors[f"prefill{c}.x"], **_inputs(tensors, f"prefill{c}"))
        n = int(tensors[f"prefill{c}.n_valid"])
        assert y.shape == tensors[f"prefill{c}.y"].shape
        assert_hidden_close(y[0, :n], tensors[f"prefill{c}.y"][0, :n], what=f"prefill chunk {c}")
    y = step(inputs_embeds=tensors["after.x"], **_inputs(tensors, "after"))
    assert_hidden_close(y, tensors["after.y"], what="decode after prefill")
    for i, l in enumerate(step.layers):
        if l.kind == om.LINEAR:
            want = tensors[f"state.layers.{i}.linear_attn.recurrent_state"].float()
            d = (l.mixer.state.cpu().float() - want).abs().max().item()
            assert d < 1e-2, f"layer {i} state differs by {d}"
            assert torch.equal(l.mixer.conv_state.cpu(), tensors[f"state.layers.{i}.linear_attn.conv_state"])


def assert_chunk_close(got, want, what=""):
    """Hidden states of a chunk [tokens, H]: within 2e-2 relative L2 over the chunk and for the median
    token; every token within 8%. Each FP8 linear rounds its input to e5m2 (2 mantissa bits), so one bf16
    ulp upstream can move a value by a whole e5m2 step: the oracle itself, with only its matmuls' sums
    reordered (linear_fp32), moves layer 0 of this chunk by 0.67% over the chunk but by up to 5.75% on
    single tokens (6.2% of a token's peak). 8% bounds that spread; the chunk-level 2e-2 is BASELINE's."""
    got, want = got.float().reshape(want.shape[0], -1), want.float().reshape(want.shape[0], -1)
    assert torch.isfinite(got).all(), f"{what}: non-finite"
    agg = ((got - want).norm() / want.norm()).item()
    tok = (got - want).norm(dim=-1) / want.norm(dim=-1).clamp_min(1e-12)
    msg = f"{what}: chunk relative L2 {agg:.3g}, median token {tok.median().item():.3g}, worst token {tok.max().item():.3g}"
    assert agg <= 2e-2 and tok.median().item() <= 2e-2 and tok.max().item() <= 8e-2, msg


def test_config0_prefill_chunk_layer_by_layer_matches_oracle(pkg, step_mod):
    """BASELINE config 0's prefill: one 512-token chunk of a row continuing a 512-position history (start
    512, cache of 1024), through each layer of the full-width block with the same input on both sides."""
    cfg = pkg.config.full_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, seed=0, device="cuda")
    wc = {k: v.to("cpu") for k, v in w.items()}
    gen = torch.Generator().manual_seed(5)
    rows, max_seq, tokens, start, slot = 2, 1024, 512, 512, 1
    step = step_mod.B200Step(cfg, w, max_seq, rows, use_graph=False)
    oracle = om.OracleStep(cfg, wc, max_seq, rows)
    for l, (kind, mixer, *_r) in zip(step.layers, oracle.layers):
        if kind == om.LINEAR:
            mixer.recurrent_state.copy_((torch.randn(mixer.recurrent_state.shape, generator=gen) * 0.1).to(torch.bfloat16))
            mixer.conv_state.copy_(torch.randn(mixer.conv_state.shape, generator=gen).to(torch.bfloat16))
            l.mixer.state.copy_(mixer.recurrent_state)
            l.mixer.conv_state.copy_(mixer.conv_state)
        else:
            mixer.k_cache.copy_(torch.randn(mixer.k_cache.shape, generator=gen).to(torch.bfloat16))
            mixer.v_cache.copy_(torch.randn(mixer.v_cache.shape, generator=gen).to(torch.bfloat16))
            l.mixer.k_cache.copy_(mixer.k_cache)
            l.mixer.v_cache.copy_(mixer.v_cache)
    ids = torch.randint(0, cfg.vocab_size, (tokens,), generator=gen).tolist()
    x = pkg.weights.embedding_rows(cfg, ids).reshape(1, tokens, -1).to(torch.bfloat16)
    cos, sin = om.rotary(cfg, torch.arange(start, start + tokens), torch.bfloat16)
    cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    chunk = dict(slot=_scalar(slot), start=_scalar(start), n_valid=_scalar(tokens))
    for i in range(cfg.num_hidden_layers):
        got = step.run_prefill_layer(i, x, cos, sin, slot, start, tokens).cpu().reshape(1, tokens, -1)
        want = oracle.layer(i, x, cos, sin, **chunk)
        assert_chunk_close(got[0], want[0], what=f"config 0 prefill layer {i}")
        kind, mixer, *_r = oracle.layers[i]
        if kind == om.LINEAR:
            d = (step.layers[i].mixer.state.cpu()[slot].float() - mixer.recurrent_state[slot].float()).abs().max().item()
            assert d < 1e-2, f"layer {i} gated-delta state differs by {d}"
        x = want
