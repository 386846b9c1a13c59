"""The reference's own serving loops drive the B200 step objects: the drop-in boundary, end to end.

The reference's Scheduler (qwen38_inf2/scheduler.py, imported unmodified from the copy oracle/build_ref.py
makes) runs multi-turn sessions with prefix reuse (copy_states), prefill chunks, and speculative verify
steps of 4 tokens drafted by the MTP layer, once with B200Step / B200MTP / B200Head (the head through the
reference's own ChipHead over B200Head.run_graph, as runner.load would wire it) and once with the oracle
in the same places. Both must emit the same tokens. The reference's batched_greedy_generate (prompts fed
a token per decode step) is checked the same way with B200Head.next_tokens as the head. Tiny test shape,
where greedy choices have no near ties.
"""

import sys

import pytest
import torch

from oracle import cpu_model as om
from oracle import ref_step

pytestmark = pytest.mark.gpu
BATCH, MAX_SEQ, CHUNK, K, SEED, STD = 3, 64, 16, 4, 7, 0.1


def _ref():
    if not ref_step.available():
        pytest.skip("the reference's package is not in oracle/_ref (run oracle/build_ref.py where it is present)")
    if str(ref_step.REF) not in sys.path:
        sys.path.insert(0, str(ref_step.REF))
    import qwen38_inf2.checkpoint as rcheckpoint
    import qwen38_inf2.generate as rgen
    import qwen38_inf2.scheduler as rsched

    return rcheckpoint, rgen, rsched


def _model(pkg):
    cfg = pkg.config.tiny_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, SEED, "cpu", STD)
    head = pkg.weights.synthetic_head(cfg, SEED, "cpu", STD)
    mtp = pkg.weights.synthetic_mtp(cfg, SEED, "cpu", STD)
    table = pkg.weights.embedding_rows(cfg, range(cfg.vocab_size), SEED, STD)
    return cfg, w, head, mtp, table


def _source(rcheckpoint, head, table):
    return rcheckpoint.DictSource({rcheckpoint.FINAL_NORM: head["norm_weight"],
                                   rcheckpoint.LM_HEAD: head["lm_head"].dequant().to(torch.bfloat16),
                                   rcheckpoint.EMBED_TOKENS: table})


# Multi-turn sessions whose next turn extends the last prompt, as an agent's conversation does: the slot's
# saved states at the end of a prompt are restored and only the extension is prefilled (scheduler.py:116-135).
SESSIONS = [[[5, 17, 42, 99, 3, 8, 8, 1], [5, 17, 42, 99, 3, 8, 8, 1, 64, 2, 2, 90]], [[11] * 20 + [7, 3]], [[1, 2, 3]],
            [[100, 50, 25, 12, 6], [100, 50, 25, 12, 6, 31, 30, 29, 28, 27, 26, 25, 24, 23, 22, 21, 20, 19, 18]]]


def test_reference_scheduler_with_mtp_speculation_drives_b200_like_the_oracle(pkg):
    rcheckpoint, rgen, rsched = _ref()
    step_mod = __import__(pkg.__name__ + ".step", fromlist=["step"])
    cfg, w, head, mtp_w, table = _model(pkg)
    source = _source(rcheckpoint, head, table)

    def scheduler(decode, mtp, run_graph):
        chip = rgen.ChipHead(source, cfg.rms_norm_eps, run_graph, BATCH * K)
        return rsched.Scheduler(decode, decode, chip, cfg, BATCH, MAX_SEQ, CHUNK, copy_states=decode, verify=decode,
                                verify_tokens=K, mtp=mtp)

    gpu_step = step_mod.B200Step(cfg, w, MAX_SEQ, BATCH, saved_states=True, verify_tokens=K)
    gpu_mtp = step_mod.B200MTP(cfg, mtp_w, MAX_SEQ, BATCH, tokens=K, max_chunk=CHUNK)
    gpu_head = step_mod.B200Head(cfg, head, BATCH * K)
    got = list(scheduler(gpu_step, gpu_mtp, gpu_head.run_graph).run_sessions(SESSIONS, 10))

    oracle = om.OracleStep(cfg, w, MAX_SEQ, BATCH, saved_states=True, verify_tokens=K)
    oracle_mtp = om.OracleMTP(cfg, mtp_w, MAX_SEQ, BATCH)
    maxima = lambda hidden: om.head_maxima(cfg, hidden, head["norm_weight"], head["lm_head"].q, head["lm_head"].scale)  # noqa: E731
    sched = scheduler(oracle, oracle_mtp, maxima)
    want = list(sched.run_sessions(SESSIONS, 10))
    assert got == want
    assert sched.reused_tokens > 0 and sched.drafted_tokens >= 0


class _DeviceHead:
    """ChipHead's interface over B200Head.next_tokens (the recheck on the device) and the embedding table."""

    def __init__(self, head, table):
        self.head, self.table = head, table

    def embed_batch(self, ids, dtype):
        return self.table[torch.as_tensor(list(ids), dtype=torch.long)].unsqueeze(1).to(dtype)

    def next_tokens(self, hidden, recheck_groups=None):
        return self.head.next_tokens(hidden, recheck_groups)


def test_reference_batched_greedy_generate_drives_b200_like_the_oracle(pkg):
    rcheckpoint, rgen, _ = _ref()
    step_mod = __import__(pkg.__name__ + ".step", fromlist=["step"])
    cfg, w, head, _, table = _model(pkg)
    prompts = [[3, 17, 42, 99, 5], [9, 9, 4], [77, 78, 79, 80, 1, 2], [12, 13]]
    gpu = list(rgen.batched_greedy_generate(step_mod.B200Step(cfg, w, MAX_SEQ, BATCH),
                                            _DeviceHead(step_mod.B200Head(cfg, head, BATCH), table), cfg, prompts, BATCH,
                                            12, MAX_SEQ))
    maxima = lambda hidden: om.head_maxima(cfg, hidden, head["norm_weight"], head["lm_head"].q, head["lm_head"].scale)  # noqa: E731
    chip = rgen.ChipHead(_source(rcheckpoint, head, table), cfg.rms_norm_eps, maxima, BATCH)
    want = list(rgen.batched_greedy_generate(om.OracleStep(cfg, w, MAX_SEQ, BATCH), chip, cfg, prompts, BATCH, 12, MAX_SEQ))
    assert gpu == want
