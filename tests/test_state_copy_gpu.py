"""Save / restore of a slot's recurrent states (q38_copy_state_rows, B200Step's save_slot / restore_slot).

* The kernel moves exactly one row of every buffer, bit for bit, including rows that are not 16-byte
  aligned, and leaves every other row alone.
* The reference's prefix reuse (tests/test_prefill.py:209-232, scheduler.py:116-135): a prompt's first
  chunk is prefilled into a slot and saved, other steps then change the slot's states, the saved states
  are restored and the prompt's second chunk is prefilled. The result must equal, bit for bit, a step
  that prefilled both chunks in a row, and match the oracle doing the same calls (hidden states within
  2e-2, gated-delta state within 1e-2).
"""

from pathlib import Path

import pytest
import torch
from safetensors import safe_open

from oracle import cpu_model as om
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


def test_copy_state_rows_moves_one_row_of_every_buffer(ops):
    gen = torch.Generator(device=DEV).manual_seed(3)
    shapes = [(6, 48, 128, 128), (6, 10240, 3), (6, 7, 5), (6, 3), (6, 1000, 17)]
    bufs = [torch.randn(s, device=DEV, generator=gen).to(torch.bfloat16) for s in shapes]
    bufs.append(torch.randint(0, 255, (6, 333), device=DEV, dtype=torch.uint8, generator=gen))
    before = [b.clone() for b in bufs]
    rows = ops.StateRows(bufs)
    rows.copy(1, 4)
    rows.copy(5, 5)  # the same row: nothing moves
    torch.cuda.synchronize()
    for b, old in zip(bufs, before):
        want = old.clone()
        want[4] = old[1]
        assert torch.equal(b, want)
    # More buffers than one launch takes.
    many = [torch.randn(4, 64, device=DEV, generator=gen) for _ in range(130)]
    old = [m.clone() for m in many]
    ops.StateRows(many).copy(3, 0)
    torch.cuda.synchronize()
    for m, o in zip(many, old):
        assert torch.equal(m[0], o[3]) and torch.equal(m[1:], o[1:])


def _golden_weights(pkg):
    with safe_open(str(GOLDEN), "pt") as f:
        meta = f.metadata()
    cfg = pkg.config.tiny_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, int(meta["seed"]), "cpu", float(meta["std"]))
    return cfg, w


def test_saved_prefix_then_extension_equals_whole_prompt(pkg, step_mod):
    cfg, w = _golden_weights(pkg)
    batch, max_seq, chunk, slot = 3, 64, 16, 1
    gen = torch.Generator().manual_seed(5)
    chunks = [torch.randn(1, chunk, cfg.hidden_size, generator=gen).to(torch.bfloat16) for _ in range(2)]
    decode_x = [torch.randn(batch, 1, cfg.hidden_size, generator=gen).to(torch.bfloat16) for _ in range(2)]

    def prefill_inputs(start):
        cos, sin = om.rotary(cfg, torch.arange(start, start + chunk), torch.bfloat16)
        return dict(cos=cos.unsqueeze(0), sin=sin.unsqueeze(0), slot=torch.tensor([slot], dtype=torch.int32),
                    start=torch.tensor([start], dtype=torch.int32), n_valid=torch.tensor([chunk], dtype=torch.int32))

    def decode_inputs(s):
        # Row `slot` decodes at positions inside the second chunk's span, which that chunk overwrites.
        position = torch.tensor([3 + s, chunk + s, 9 + s], dtype=torch.int32)
        cos, sin = om.rotary(cfg, position, torch.bfloat16)
        return dict(cos=cos.unsqueeze(1), sin=sin.unsqueeze(1), position=position, active=torch.ones(batch))

    def run(model, reuse: bool):
        model(inputs_embeds=chunks[0], **prefill_inputs(0))
        if reuse:
            model(inputs_embeds=chunks[0], save_slot=torch.tensor([slot], dtype=torch.int32))
            for s in range(2):
                model(inputs_embeds=decode_x[s], **decode_inputs(s))
            model(inputs_embeds=chunks[0], restore_slot=torch.tensor([slot], dtype=torch.int32))
        return model(inputs_embeds=chunks[1], **prefill_inputs(chunk))

    whole = step_mod.B200Step(cfg, w, max_seq, batch, saved_states=True, use_graph=False)
    reused = step_mod.B200Step(cfg, w, max_seq, batch, saved_states=True)
    oracle = om.OracleStep(cfg, w, max_seq, batch, saved_states=True)
    want_gpu = run(whole, reuse=False)
    got = run(reused, reuse=True)
    want = run(oracle, reuse=True)
    assert torch.equal(got, want_gpu), "restored prefix + extension differs from the whole prompt"
    assert_hidden_close(got.reshape(chunk, -1), want.reshape(chunk, -1), what="saved prefix vs oracle")
    for l, lw, (kind, mixer, *_r) in zip(reused.layers, whole.layers, oracle.layers):
        if kind == om.LINEAR:
            assert torch.equal(l.mixer.state[slot], lw.mixer.state[slot])
            assert torch.equal(l.mixer.conv_state[slot], lw.mixer.conv_state[slot])
            d = (l.mixer.state.cpu().float() - mixer.recurrent_state.float()).abs().max().item()
            assert d < 1e-2, f"gated-delta state differs from the oracle by {d}"
            assert torch.equal(l.mixer.conv_state.cpu(), mixer.conv_state)


def test_copy_states_refuses_bad_slots(pkg, step_mod):
    cfg, w = _golden_weights(pkg)
    plain = step_mod.B200Step(cfg, w, 64, 3, use_graph=False)
    with pytest.raises(ValueError):
        plain(inputs_embeds=torch.zeros(1), save_slot=torch.tensor([0], dtype=torch.int32))
    saved = step_mod.B200Step(cfg, w, 64, 3, saved_states=True, use_graph=False)
    with pytest.raises(ValueError):
        saved(inputs_embeds=torch.zeros(1), restore_slot=torch.tensor([3], dtype=torch.int32))
