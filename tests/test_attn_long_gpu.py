"""Attention split along the cache (q38_attn_split): long caches and the FP8 e4m3 KV cache.

Against the oracle's decode_core / verify_core (FullAttentionStep.forward / verify, model.py:610-675,
with the FP8 cache's _store / _load / _round_trip, :579-593), on the same inputs:
* BASELINE config 4's shapes: caches of 32,768 positions with rows at ~16K and ~30K positions, at the
  head counts of one GPU (6 query heads per KV head, 4 KV heads) and of TP = 8 (3 query heads, 1 KV
  head), decode (1 token) and verify (4 tokens), BF16 and FP8 caches; an inactive row in every batch;
* the tiny test shape, and config 3's 512-position cache at batch 8 (where the one-CTA-per-row
  decode kernel also runs: both kernels must agree).
Tolerances as the other attention tests: e5m2 outputs with at most 2% of codes differing, 0.1% by more
than one code, every row within 2e-2 relative L2; the cache's new keys within one bf16 ulp (one e4m3
code for the FP8 cache) on at most 0.1% of values, the new values bit for bit.
"""

import pytest
import torch

from oracle import cpu_model as om
from tests.test_kernels_gpu import assert_attention_e5m2_close, assert_bf16_close, e5m2_code

pytestmark = pytest.mark.gpu
DEV = "cuda"
FP8_SCALES = (2.0 ** -4, 2.0 ** -5)


@pytest.fixture(scope="module")
def ops(pkg):
    return __import__(pkg.__name__ + ".ops", fromlist=["ops"])


def _case(pkg, shape, tp, batch, max_seq, tokens, fp8, positions):
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(17 + max_seq + tokens + tp)
    w = pkg.weights.synthetic_layer(cfg, 3, seed=11, device="cpu", std=0.1)
    layer = om.AttentionLayer(cfg, w, "layers.3", tp, 0, batch, max_seq, torch.bfloat16, FP8_SCALES if fp8 else None)
    for cache, which in ((layer.k_cache, 0), (layer.v_cache, 1)):
        cache.copy_(layer.store(torch.randn(cache.shape, generator=gen).to(torch.bfloat16), which))
    hd, heads, kvh = cfg.head_dim, layer.heads, layer.kv_heads
    qg = torch.randn(batch, tokens, heads * 2 * hd, generator=gen).to(torch.bfloat16)
    k = torch.randn(batch, tokens, kvh * hd, generator=gen).to(torch.bfloat16)
    v = torch.randn(batch, tokens, kvh * hd, generator=gen).to(torch.bfloat16)
    position = torch.tensor(positions, dtype=torch.int32)
    active = torch.ones(batch)
    active[-1] = 0.0
    cos, sin = om.rotary(cfg, (position.unsqueeze(-1) + torch.arange(tokens)).reshape(-1), torch.bfloat16)
    return cfg, layer, qg, k, v, position, active, cos, sin


def _run_split(ops, cfg, layer, qg, k, v, position, active, cos, sin, tokens, fp8):
    batch = qg.shape[0]
    hd = cfg.head_dim
    d_k, d_v = layer.k_cache.to(DEV), layer.v_cache.to(DEV)
    out = torch.empty(batch * tokens, layer.heads * hd, dtype=torch.uint8, device=DEV)
    ops.attn_split(torch.cat((qg, k, v), -1).reshape(batch * tokens, -1).to(DEV), layer.q_norm.to(DEV),
                   layer.k_norm.to(DEV), cos.to(DEV), sin.to(DEV), d_k, d_v, position.to(DEV), active.to(DEV), out,
                   batch=batch, tokens=tokens, num_q_heads=layer.heads, num_kv_heads=layer.kv_heads, head_dim=hd,
                   rot_dim=cfg.rotary_dim, eps=cfg.rms_norm_eps, kv_scales=FP8_SCALES if fp8 else None)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return out, d_k, d_v


LONG = [
    # shape, tp, batch, max_seq, tokens, fp8, positions (the last row inactive)
    ("tiny", 1, 3, 64, 1, False, [0, 37, 5]),
    ("tiny", 1, 3, 64, 1, True, [63, 31, 5]),
    ("tiny", 1, 3, 64, 4, True, [0, 33, 7]),
    ("full", 8, 3, 32768, 1, False, [16384, 30001, 100]),
    ("full", 8, 3, 32768, 4, True, [16000, 30717, 9]),
    ("full", 1, 3, 32768, 1, True, [15999, 29990, 4000]),
    ("full", 1, 3, 32768, 4, False, [16411, 30000, 20]),
]


@pytest.mark.parametrize("shape,tp,batch,max_seq,tokens,fp8,positions", LONG)
def test_attn_split_matches_oracle(pkg, ops, shape, tp, batch, max_seq, tokens, fp8, positions):
    cfg, layer, qg, k, v, position, active, cos, sin = _case(pkg, shape, tp, batch, max_seq, tokens, fp8, positions)
    out, d_k, d_v = _run_split(ops, cfg, layer, qg, k, v, position, active, cos, sin, tokens, fp8)
    if tokens == 1:
        want = layer.decode_core(qg, k, v, cos.unsqueeze(1), sin.unsqueeze(1), position, active)
    else:
        want = layer.verify_core(qg, k, v, cos.reshape(batch, tokens, -1), sin.reshape(batch, tokens, -1), position,
                                 active)
    on = (active > 0.5).repeat_interleave(tokens)
    assert_attention_e5m2_close(out.cpu()[on], want.reshape(batch * tokens, -1)[on], what=f"attention {shape} tp{tp}")
    if fp8:
        d = (e5m2_code(d_k.cpu()) - e5m2_code(layer.k_cache)).abs()  # e4m3 bytes: same sign-magnitude order
        assert d.max().item() <= 1 and (d > 0).float().mean().item() <= 1e-3, "k cache (e4m3 codes)"
    else:
        assert_bf16_close(d_k.cpu(), layer.k_cache, frac=0.001, what="k cache")
    assert torch.equal(d_v.cpu(), layer.v_cache)


def test_attn_split_agrees_with_the_decode_kernel_at_config3_shape(pkg, ops):
    """Config 3's cache (512 positions) at batch 8: the split kernels and the one-CTA-per-row decode kernel
    compute the same arithmetic up to fp32 summation order."""
    positions = [0, 1, 31, 32, 300, 511, 255, 77]
    cfg, layer, qg, k, v, position, active, cos, sin = _case(pkg, "full", 1, 8, 512, 1, False, positions)
    out, d_k, _ = _run_split(ops, cfg, layer, qg, k, v, position, active, cos, sin, 1, False)
    ref_k, ref_v = layer.k_cache.to(DEV), layer.v_cache.to(DEV)
    out2 = torch.empty_like(out)
    ops.attn_decode(torch.cat((qg, k, v), -1).reshape(8, -1).to(DEV), layer.q_norm.to(DEV), layer.k_norm.to(DEV),
                    cos.to(DEV), sin.to(DEV), ref_k, ref_v, position.to(DEV), active.to(DEV), out2, batch=8,
                    num_q_heads=layer.heads, num_kv_heads=layer.kv_heads, head_dim=cfg.head_dim, rot_dim=cfg.rotary_dim,
                    eps=cfg.rms_norm_eps)
    torch.cuda.synchronize()
    on = active > 0.5
    want = out2.cpu()[on].view(torch.float8_e5m2).to(torch.bfloat16)
    assert_attention_e5m2_close(out.cpu()[on], want, what="split vs decode kernel")
    assert torch.equal(d_k, ref_k)


PREFILL = [
    # shape, tp, max_seq, start, tokens, fp8
    ("tiny", 1, 64, 0, 16, True),
    ("tiny", 1, 64, 16, 16, True),
    ("full", 8, 32768, 16384, 64, True),
    ("full", 8, 32768, 30000, 48, False),
    ("full", 1, 32768, 30016, 32, True),
]


@pytest.mark.parametrize("shape,tp,max_seq,start,tokens,fp8", PREFILL)
def test_attn_prefill_long_and_fp8_matches_oracle(pkg, ops, shape, tp, max_seq, start, tokens, fp8):
    """A prefill chunk continuing a row at ~16K and ~30K of a 32K cache (the reference's 2048-key
    softmax blocks, TP = 8 and one-GPU head counts), and the FP8 e4m3 cache: the chunk's keys and values
    are written as cache bytes and read back as the cache's round trip of them (model.py:748-752)."""
    cfg = pkg.config.tiny_config(1) if shape == "tiny" else pkg.config.full_config(1)
    gen = torch.Generator().manual_seed(41 + start + tokens)
    rows, slot = 2, 1
    w = pkg.weights.synthetic_layer(cfg, 3, seed=11, device="cpu", std=0.1)
    layer = om.AttentionLayer(cfg, w, "layers.3", tp, 0, rows, max_seq, torch.bfloat16, FP8_SCALES if fp8 else None)
    for cache, which in ((layer.k_cache, 0), (layer.v_cache, 1)):
        cache.copy_(layer.store(torch.randn(cache.shape, generator=gen).to(torch.bfloat16), which))
    hd, heads, kvh = cfg.head_dim, layer.heads, layer.kv_heads
    qg = torch.randn(1, tokens, heads * 2 * hd, generator=gen).to(torch.bfloat16)
    k = torch.randn(1, tokens, kvh * hd, generator=gen).to(torch.bfloat16)
    v = torch.randn(1, tokens, kvh * hd, generator=gen).to(torch.bfloat16)
    cos, sin = om.rotary(cfg, torch.arange(start, start + tokens), torch.bfloat16)
    d_k, d_v = layer.k_cache.to(DEV), layer.v_cache.to(DEV)
    out = torch.empty(tokens, heads * hd, dtype=torch.uint8, device=DEV)
    ws = torch.empty(ops.attn_prefill_workspace_bytes(tokens, heads, hd), dtype=torch.uint8, device=DEV)
    ops.attn_prefill(torch.cat((qg, k, v), -1).reshape(tokens, -1).to(DEV), layer.q_norm.to(DEV), layer.k_norm.to(DEV),
                     cos.to(DEV), sin.to(DEV), d_k, d_v, out, ws, slot=slot, start=start, num_q_heads=heads,
                     num_kv_heads=kvh, head_dim=hd, rot_dim=cfg.rotary_dim, eps=cfg.rms_norm_eps,
                     kv_scales=FP8_SCALES if fp8 else None)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    slot_t, start_t = torch.tensor([slot], dtype=torch.int32), torch.tensor([start], dtype=torch.int32)
    want = layer.prefill_core(qg, k, v, cos.unsqueeze(0), sin.unsqueeze(0), slot_t, start_t)
    assert_attention_e5m2_close(out.cpu(), want.reshape(tokens, -1), what=f"attention prefill {shape} tp{tp}")
    if fp8:
        d = (e5m2_code(d_k.cpu()) - e5m2_code(layer.k_cache)).abs()
        assert d.max().item() <= 1 and (d > 0).float().mean().item() <= 1e-3, "k cache (e4m3 codes)"
    else:
        assert_bf16_close(d_k.cpu(), layer.k_cache, frac=0.001, what="k cache")
    assert torch.equal(d_v.cpu(), layer.v_cache)
