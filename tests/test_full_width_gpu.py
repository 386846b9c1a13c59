"""BASELINE config 0 at full width through B200Step and B200Head, against the reference's own outputs.

The fixture (tests/golden/full_block.safetensors, made by the reference: one full-width 4-layer block,
batch 8, rows at positions uniform in [0, 512), two greedy steps, the whole 248,320-token vocabulary)
gives every step's inputs, the reference's hidden state, its HeadStep maxima, top-4 groups and
ChipHead tokens. Checks per step:

* The head on the reference's own hidden state (teacher-forced): B200Head's maxima within 2e-4 of the
  row peak of the reference's (the head's input is the bf16 rounding of the normed row, whose fp32 sum of
  squares runs in another order here, so a few inputs can sit one bf16 ulp apart, each moving a logit by
  about 1e-5 of the peak), its best 4 groups the reference's (a swap only between groups whose
  reference maxima are that close), and the recheck on them gives the reference's tokens exactly.
* The hidden state from B200Step, against a bound measured on the same inputs: the oracle run with its
  matmuls in another legitimate summation order (fp32 instead of BF16 accumulation) shows how far the
  reference's own arithmetic moves under reordering (every FP8 linear rounds its input to e5m2, so one
  bf16 ulp upstream can move a whole e5m2 step); B200Step must stay within 3x that spread of the
  reference, and within 2e-2 wherever the spread is smaller.
* B200Head.next_tokens (the recheck on the device) gives the same tokens as the host recheck on the
  same maxima, and the reference's tokens on the reference's hidden state.
* Greedy tokens end to end (B200Step, B200Head.next_tokens): identical to the
  reference's, except where the reference's best two candidates are a near tie under the measured
  spread (their logit gap below 3x the largest move, over the step's rows, of those logits under the
  reordering). Step 1 takes the
  reference's tokens (teacher forcing), so one differing row cannot change the others.
"""

import pytest
import torch

from oracle import cpu_model as om
from tests import full_width as fw

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fixture(pkg):
    tensors, meta = fw.load()
    cfg, w, head = fw.model(pkg, meta)
    return tensors, meta, cfg, w, head


def _rel_l2(a, b):
    a, b = a.float().reshape(b.shape[0], -1), b.float().reshape(b.shape[0], -1)
    return (a - b).norm(dim=-1) / b.norm(dim=-1)


def _logits(cfg, hidden, norm_w, lm_rows, row, tokens):
    norm = om.rms_norm(hidden.float(), norm_w, cfg.rms_norm_eps).reshape(hidden.shape[0], -1)[row]
    return [float(lm_rows[t] @ norm) for t in tokens]


def test_full_width_greedy_tokens_top4_and_hidden_match_reference(pkg, fixture):
    step_mod = __import__(pkg.__name__ + ".step", fromlist=["step"])
    tensors, meta, cfg, w, head = fixture
    batch, max_seq = int(meta["batch"]), int(meta["max_seq"])
    step = step_mod.B200Step(cfg, w, max_seq, batch)
    fw.seed_step(step, cfg, meta)
    bhead = step_mod.B200Head(cfg, head, batch)
    reordered = om.OracleStep(cfg, w, max_seq, batch, linear_fp32=True)
    fw.seed_oracle(reordered, cfg, meta)
    lm_rows = head["lm_head"].dequant()
    norm_w = head["norm_weight"]
    exact, near_ties = 0, []
    for s in range(int(meta["steps"])):
        x, inputs = tensors[f"step{s}.x"], fw.inputs(tensors, s)
        y_ref, want_max = tensors[f"step{s}.y"], tensors[f"step{s}.maxima"]
        want_top4, want_tokens = tensors[f"step{s}.top4"], tensors[f"step{s}.tokens_out"].tolist()

        # The head alone, on the reference's hidden state.
        got_max = bhead.run_graph(y_ref)
        peak = want_max.abs().amax(-1, keepdim=True)
        rel = ((got_max - want_max).abs() / peak).max().item()
        assert rel <= 2e-4, f"step {s}: maxima differ by {rel:.3g} of the row peak"
        top4 = got_max.topk(4, dim=-1).indices
        same_values = (want_max.gather(1, top4) - want_max.gather(1, want_top4)).abs() <= 2e-4 * peak
        assert same_values.all(), f"step {s}: top-4 groups {top4.tolist()} vs the reference's {want_top4.tolist()}"
        assert om.recheck_tokens(cfg, y_ref, norm_w, lm_rows, got_max) == want_tokens, f"step {s}: head tokens"
        assert bhead.next_tokens(y_ref) == want_tokens, f"step {s}: the device recheck's tokens"

        # The hidden state, against the measured reordering spread.
        y_gpu = step(inputs_embeds=x, **inputs)
        y_alt = reordered(inputs_embeds=x, **inputs)
        err, spread = _rel_l2(y_gpu, y_ref), _rel_l2(y_alt, y_ref)
        bound = torch.clamp(3 * spread.max(), min=2e-2)
        assert (err <= bound).all(), f"step {s}: relative L2 per row {err.tolist()}, reordering spread {spread.tolist()}"

        # Greedy tokens end to end.
        got_tokens = bhead.next_tokens(y_gpu)
        assert got_tokens == om.recheck_tokens(cfg, y_gpu, norm_w, lm_rows, bhead.run_graph(y_gpu)), "device vs host recheck"
        # How far the reordering moves the logits of the reference's and the GPU's tokens, over all rows of the
        # step (the same statistic as the hidden-state bound: the spread is a property of the arithmetic).
        moves = []
        for row, (g, want) in enumerate(zip(got_tokens, want_tokens)):
            ref_l = _logits(cfg, y_ref, norm_w, lm_rows, row, (want, g))
            alt_l = _logits(cfg, y_alt, norm_w, lm_rows, row, (want, g))
            moves.append(max(abs(a - b) for a, b in zip(ref_l, alt_l)))
        for row, (g, want) in enumerate(zip(got_tokens, want_tokens)):
            if g == want:
                exact += 1
                continue
            ref_l = _logits(cfg, y_ref, norm_w, lm_rows, row, (want, g))
            gap = ref_l[0] - ref_l[1]
            near_ties.append((s, row, round(gap, 4), round(max(moves), 4)))
            assert gap <= 3 * max(moves), (f"step {s} row {row}: token {g} instead of {want}, logit gap {gap:.4g} against "
                                           f"a reordering move of up to {max(moves):.4g}")
    total = int(meta["steps"]) * batch
    print(f"full-width greedy tokens: {exact} of {total} identical; near ties {near_ties}")
