"""Host-side planning without a GPU: the GEMMs' K-split choices and the bench's per-step byte count."""

import importlib
from types import SimpleNamespace

import pytest


@pytest.fixture(scope="module")
def ops(pkg):
    return importlib.import_module(pkg.__name__ + ".ops")


def test_decode_split_choices_fill_one_wave(ops):
    # 256 rows: 5120-output row-parallel projections get 3 K splits (40 tiles x 3 = 120 CTAs on 148 SMs);
    # the wide column-parallel projections, whose grids already cover the SMs, run unsplit.
    assert ops.choose_splits(256, 5120, 17408) == 3
    assert ops.choose_splits(256, 5120, 6144) == 3
    assert ops.choose_splits(256, 16384, 5120) == 1
    assert ops.choose_splits(256, 14336, 5120) == 1
    # Few rows: the same single wave, with at least 4 K stages per split.
    assert ops.choose_splits(8, 5120, 6144) == 3
    assert ops.choose_splits(8, 5120, 1024) == 2


def test_token_tiles_and_bf16_splits(ops):
    assert ops.token_tile(1) == 128 and ops.token_tile(128) == 128 and ops.token_tile(129) == 256
    # in_proj_b / in_proj_a: 8 splits at 5120 (the split count fixes the fp32 summation order).
    assert ops.bf16_linear_splits(256, 96, 5120) == 8
    assert ops.bf16_linear_splits(256, 96, 128) == 1


def test_decode_step_bytes_counts_weights_state_and_cache():
    bench = importlib.import_module("bench")
    torch = importlib.import_module("torch")
    lin = lambda o, i: SimpleNamespace(out_features=o, in_features=i)  # noqa: E731
    gdn = SimpleNamespace(kind="linear_attention", gate_up=lin(64, 32), down=lin(32, 32),
                          mixer=SimpleNamespace(qkvz=lin(96, 32), out=lin(32, 64), ab=lin(4, 32),
                                                state=torch.zeros(2, 4, 8, 8), conv_state=torch.zeros(2, 10, 3)))
    attn = SimpleNamespace(kind="full_attention", gate_up=lin(64, 32), down=lin(32, 32),
                           mixer=SimpleNamespace(qkv=lin(48, 32), o=lin(32, 32), k_cache=torch.zeros(2, 1, 16, 8)))
    step = SimpleNamespace(layers=[gdn, attn])
    head = SimpleNamespace(lm_head=lin(320, 32))
    positions = torch.tensor([[3, 600], [4, 20]], dtype=torch.int32)  # two steps; 600 counts as MAX_SEQ (512)
    fp8 = lambda o, i: o * i * 33 // 32  # noqa: E731
    want = fp8(320, 32)                                                    # lm_head at its FP8 size
    want += 2 * (fp8(64, 32) + fp8(32, 32))                                # MLPs
    want += fp8(96, 32) + fp8(32, 64) + 4 * 32 * 2                         # GDN projections, BF16 in_proj_b/a
    want += (2 * 4 * 8 * 8 + 2 * 10 * 3) * 2 * 2                           # state and conv state in and out
    kv_positions = (3 + 512 + 4 + 20) / 2                                  # mean over the steps of the rows' sum
    want += fp8(48, 32) + fp8(32, 32) + int(kv_positions * 1 * 8 * 2 * 2)  # attention projections, K and V
    assert bench.MAX_SEQ == 512
    assert bench.decode_step_bytes(step, head, "linear_attention", positions) == want


def test_input_builders_equal_the_oracles_and_check_positions(pkg):
    """The host input builders give the rotary tables the oracle (and the reference, generate.py:25-31) uses,
    the reference's shapes and dtypes, and refuse positions past the cache."""
    import pytest
    import torch

    from oracle import cpu_model as om

    inp = __import__(pkg.__name__ + ".inputs", fromlist=["inputs"])
    cfg = pkg.config.full_config(1)
    pos = torch.tensor([0, 5, 511, 30000, 32766], dtype=torch.int32)
    cos, sin = inp.rotary(cfg, pos)
    ocos, osin = om.rotary(cfg, pos, torch.bfloat16)
    assert torch.equal(cos, ocos) and torch.equal(sin, osin)
    d = inp.decode_inputs(cfg, [3, 9], 512, [True, False])
    assert d["cos"].shape == (2, 1, cfg.rotary_dim) and d["position"].dtype == torch.int32 and d["active"].tolist() == [1.0, 0.0]
    p = inp.prefill_inputs(cfg, 2, 512, 100, 512)
    assert p["cos"].shape == (1, 512, cfg.rotary_dim) and int(p["n_valid"]) == 100
    v = inp.verify_inputs(cfg, [10, 20], 4, 512, [True, True], [0, 3])
    assert v["cos"].shape == (2, 4, cfg.rotary_dim) and v["accepted"].tolist() == [0, 3]
    m = inp.mtp_step_inputs(cfg, [10], 4, 512, [True])
    assert torch.equal(m["cos"][0, 0], inp.rotary(cfg, torch.tensor([11]))[0][0])
    with pytest.raises(ValueError):
        inp.decode_inputs(cfg, [511], 512)
    with pytest.raises(ValueError):
        inp.verify_inputs(cfg, [509], 4, 512, [True], [0])
