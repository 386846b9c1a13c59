"""Speculative verify with commit-on-accept: the gated-delta and attention verify kernels against the
oracle, and B200Step's verify call against the reference's golden vectors (tests/golden/tiny_verify).

Tolerances, stated per check:
* gated-delta e5m2 output: codes equal or adjacent, adjacent for at most 2% (fp32 sums reordered).
* attention e5m2 output: as for prefill attention (bf16-rounded scores can flip by one ulp under fp32
  reordering): codes equal for 98%, more than one code apart for at most 0.1%, 2e-2 relative L2 per token.
* committed gated-delta state: within 1e-2 absolute (BASELINE), equal for most elements; conv state and
  the pending conv inputs bit-exact (copies of bf16 inputs); pending keys, deltas and log decays within
  1e-5 relative to their scale (fp32 values from reordered sums).
* KV written by the step: keys within one bf16 ulp, values bit-exact.
* hidden states through B200Step: within 2e-2 of the row peak and in relative L2 (BASELINE).
"""

from pathlib import Path

import pytest
import torch
from safetensors import safe_open

from oracle import cpu_model as om
from tests.test_kernels_gpu import assert_bf16_close, assert_e5m2_close
from tests.test_prefill_gpu import assert_attention_e5m2_close
from tests.test_step_gpu import assert_hidden_close

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden" / "tiny_verify.safetensors"
K = 4


@pytest.fixture(scope="module")
def ops(pkg):
    return __import__(pkg.__name__ + ".ops", fromlist=["ops"])


@pytest.fixture(scope="module")
def step_mod(pkg):
    return __import__(pkg.__name__ + ".step", fromlist=["step"])


def assert_f32_close(got, want, rel=1e-5, what=""):
    got, want = got.float().cpu(), want.float().cpu()
    scale = want.abs().max().clamp_min(1e-30)
    d = ((got - want).abs() / scale).max().item()
    assert d <= rel, f"{what}: differs by {d:.3g} of the largest magnitude"


def _row_inputs(batch, gen):
    position = torch.randint(1, 40, (batch,), generator=gen, dtype=torch.int32)
    position[0] = 0  # a fresh sequence: states clear
    active = torch.ones(batch)
    active[1] = 0.0  # an idle row keeps everything
    accepted = torch.randint(0, K + 1, (batch,), generator=gen, dtype=torch.int32)
    accepted[2] = K
    accepted[3 % batch] = 0
    return position, active, accepted


@pytest.mark.parametrize("shape,batch", [("tiny", 5), ("full", 9)])
def test_gdn_verify_matches_oracle(pkg, ops, shape, batch):
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(41)
    w = pkg.weights.synthetic_layer(cfg, 0, seed=11, device="cpu", std=0.1)
    layer = om.GDNLayer(cfg, w, "layers.0", 1, batch, torch.bfloat16, verify_tokens=K)
    layer.recurrent_state.copy_((torch.randn(layer.recurrent_state.shape, generator=gen) * 0.1).to(torch.bfloat16))
    layer.conv_state.copy_(torch.randn(layer.conv_state.shape, generator=gen).to(torch.bfloat16))
    layer.pending_key = torch.nn.functional.normalize(torch.randn(layer.pending_key.shape, generator=gen), dim=-1)
    layer.pending_delta = torch.randn(layer.pending_delta.shape, generator=gen) * 0.1
    layer.pending_decay = -torch.rand(layer.pending_decay.shape, generator=gen)
    layer.pending_input = torch.randn(layer.pending_input.shape, generator=gen).to(torch.bfloat16)
    conv_dim, vd, hv = cfg.linear_conv_dim, cfg.linear_value_dim, cfg.linear_num_value_heads
    qkv = torch.randn(batch, K, conv_dim, generator=gen).to(torch.bfloat16)
    z = torch.randn(batch, K, vd, generator=gen).to(torch.bfloat16)
    b_raw = torch.randn(batch, K, hv, generator=gen).to(torch.bfloat16)
    a_raw = torch.randn(batch, K, hv, generator=gen).to(torch.bfloat16)
    position, active, accepted = _row_inputs(batch, gen)
    d = {n: getattr(layer, n).clone().to(DEV) for n in ("recurrent_state", "conv_state", "pending_key", "pending_delta",
                                                       "pending_decay", "pending_input")}
    state0, conv0 = layer.recurrent_state.clone(), layer.conv_state.clone()
    out = torch.empty(batch * K, vd, dtype=torch.uint8, device=DEV)
    ops.gdn_verify(torch.cat((qkv, z), -1).reshape(batch * K, -1).to(DEV),
                   torch.cat((b_raw, a_raw), -1).reshape(batch * K, -1).to(DEV), d["conv_state"], layer.conv_w.to(DEV),
                   layer.A_log.to(DEV), layer.dt_bias.to(DEV), layer.norm_w.to(DEV), d["recurrent_state"],
                   d["pending_key"], d["pending_delta"], d["pending_decay"], d["pending_input"], position.to(DEV),
                   active.to(DEV), accepted.to(DEV), out, batch=batch, tokens=K, num_k_heads=cfg.linear_num_key_heads,
                   num_v_heads=hv, head_k=cfg.linear_key_head_dim, head_v=cfg.linear_value_head_dim, eps=cfg.rms_norm_eps)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    want = layer.verify_core(qkv, z, b_raw, a_raw, position, active, accepted)
    on = (active > 0.5).repeat_interleave(K)
    assert_e5m2_close(out.cpu()[on], want.reshape(batch * K, -1)[on], what="gdn verify out")
    got_state = d["recurrent_state"].cpu()
    assert torch.equal(got_state[1], state0[1]) and torch.equal(d["conv_state"].cpu()[1], conv0[1]), "idle row changed"
    diff = (got_state.float() - layer.recurrent_state.float()).abs()
    assert diff.max().item() < 1e-2, f"committed state differs by {diff.max().item()}"
    assert (diff == 0).float().mean().item() > 0.95
    assert torch.equal(d["conv_state"].cpu(), layer.conv_state)
    assert torch.equal(d["pending_input"].cpu(), layer.pending_input)
    assert_f32_close(d["pending_key"], layer.pending_key, what="pending keys")
    assert_f32_close(d["pending_decay"], layer.pending_decay, what="pending log decays")
    assert_f32_close(d["pending_delta"], layer.pending_delta, rel=1e-4, what="pending deltas")


@pytest.mark.parametrize("shape,batch,max_seq", [("tiny", 4, 64), ("full", 7, 512)])
def test_attn_verify_matches_oracle(pkg, ops, shape, batch, max_seq):
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(43)
    w = pkg.weights.synthetic_layer(cfg, 3, seed=11, device="cpu", std=0.1)
    layer = om.AttentionLayer(cfg, w, "layers.3", 1, 0, batch, max_seq, torch.bfloat16)
    layer.k_cache.copy_(torch.randn(layer.k_cache.shape, generator=gen).to(torch.bfloat16))
    layer.v_cache.copy_(torch.randn(layer.v_cache.shape, generator=gen).to(torch.bfloat16))
    hd, heads, kvh = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    qg = torch.randn(batch, K, heads * 2 * hd, generator=gen).to(torch.bfloat16)
    k = torch.randn(batch, K, kvh * hd, generator=gen).to(torch.bfloat16)
    v = torch.randn(batch, K, kvh * hd, generator=gen).to(torch.bfloat16)
    position = torch.randint(1, max_seq - K - 1, (batch,), generator=gen, dtype=torch.int32)
    position[0] = 0
    active = torch.ones(batch)
    active[-1] = 0.0
    cos, sin = om.rotary(cfg, (position.unsqueeze(-1) + torch.arange(K)).reshape(-1), torch.bfloat16)
    d_k, d_v = layer.k_cache.to(DEV), layer.v_cache.to(DEV)
    out = torch.empty(batch * K, heads * hd, dtype=torch.uint8, device=DEV)
    ops.attn_verify(torch.cat((qg, k, v), -1).reshape(batch * K, -1).to(DEV), layer.q_norm.to(DEV), layer.k_norm.to(DEV),
                    cos.to(DEV), sin.to(DEV), d_k, d_v, position.to(DEV), active.to(DEV), out, batch=batch, tokens=K,
                    num_q_heads=heads, num_kv_heads=kvh, head_dim=hd, rot_dim=cfg.rotary_dim, eps=cfg.rms_norm_eps)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    want = layer.verify_core(qg, k, v, cos.reshape(batch, K, -1), sin.reshape(batch, K, -1), position, active)
    on = (active > 0.5).repeat_interleave(K)
    assert_attention_e5m2_close(out.cpu()[on], want.reshape(batch * K, -1)[on], what="attention verify out")
    assert_bf16_close(d_k.cpu(), layer.k_cache, frac=0.001, what="k cache")
    assert torch.equal(d_v.cpu(), layer.v_cache)


def _inputs(tensors, prefix):
    keys = ("cos", "sin", "position", "active", "accepted")
    return {k: tensors[f"{prefix}.{k}"] for k in keys if f"{prefix}.{k}" in tensors}


def test_tiny_verify_sequence_matches_reference_golden(pkg, step_mod):
    """Two decode steps, five verify steps (different accepted counts, an idle row, a row starting over),
    then decode: every output and the final recurrent, conv, pending and KV buffers."""
    with safe_open(str(GOLDEN), "pt") as f:
        tensors, meta = {k: f.get_tensor(k) for k in f.keys()}, f.metadata()
    cfg = pkg.config.tiny_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, int(meta["seed"]), "cpu", float(meta["std"]))
    kv = int(meta["verify_tokens"])
    step = step_mod.B200Step(cfg, w, int(meta["max_seq"]), int(meta["batch"]), verify_tokens=kv)
    calls = [f"decode{s}" for s in range(2)] + [f"verify{s}" for s in range(int(meta["verify_steps"]))] + ["after"]
    for c in calls:
        y = step(inputs_embeds=tensors[f"{c}.x"], **_inputs(tensors, c))
        on = tensors[f"{c}.active"] > 0.5
        assert_hidden_close(y[on], tensors[f"{c}.y"][on], what=c)
    for i, l in enumerate(step.layers):
        p = f"state.layers.{i}."
        if l.kind == om.LINEAR:
            d = (l.mixer.state.cpu().float() - tensors[p + "linear_attn.recurrent_state"].float()).abs().max().item()
            assert d < 1e-2, f"layer {i} state differs by {d}"
            assert torch.equal(l.mixer.conv_state.cpu(), tensors[p + "linear_attn.conv_state"])
            assert torch.equal(l.mixer.pending[3].cpu(), tensors[p + "linear_attn.pending_input_state"])
        else:
            want = tensors[p + "self_attn.k_cache"][:, :, :-kv].float()
            got = l.mixer.k_cache.cpu()[:, :, :-kv].float()
            assert (got - want).abs().max().item() <= 2e-2 * want.abs().max().item()
