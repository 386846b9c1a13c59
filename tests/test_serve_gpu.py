"""The prefill-first serving loop (serve.py) over B200Step / B200Head against the same loop over the oracle.

Tiny test shape, 3 slots, 5 prompts of different lengths (two prefill chunks for the longest), 6 greedy
tokens each: the same tokens for every prompt, and the accounting of prompt and generated tokens.
"""

import pytest
import torch

from oracle import cpu_model as om

pytestmark = pytest.mark.gpu
SEED, STD, BATCH, MAX_SEQ, CHUNK = 7, 0.1, 3, 64, 16


class _OracleStep:
    def __init__(self, cfg, w):
        self.cfg, self.batch, self.max_seq = cfg, BATCH, MAX_SEQ
        self.inner = om.OracleStep(cfg, w, MAX_SEQ, BATCH)

    def __call__(self, inputs_embeds, **inputs):
        return self.inner(inputs_embeds=inputs_embeds.cpu(), **inputs)


class _OracleHead:
    def __init__(self, cfg, head):
        self.cfg, self.head, self.rows = cfg, head, head["lm_head"].dequant()

    def next_tokens(self, hidden, recheck_groups=None):
        maxima = om.head_maxima(self.cfg, hidden, self.head["norm_weight"], self.head["lm_head"].q, self.head["lm_head"].scale)
        return om.recheck_tokens(self.cfg, hidden, self.head["norm_weight"], self.rows, maxima)


class _CpuEmbeddings:
    def __init__(self, table):
        self.table = table

    def embed(self, ids):
        return self.table[torch.as_tensor(list(ids), dtype=torch.long)]


def test_serving_loop_matches_the_oracle(pkg):
    serve = __import__(pkg.__name__ + ".serve", fromlist=["serve"])
    step_mod = __import__(pkg.__name__ + ".step", fromlist=["step"])
    cfg = pkg.config.tiny_config(num_blocks=1)
    w = {}
    for i in range(cfg.num_hidden_layers):
        w |= pkg.weights.synthetic_layer(cfg, i, SEED, "cpu", STD)
    head = pkg.weights.synthetic_head(cfg, SEED, "cpu", STD)
    table = pkg.weights.embedding_rows(cfg, range(cfg.vocab_size), SEED, STD)
    prompts = [[3, 17, 42, 99, 5], list(range(1, 21)), [9, 9, 4], [77, 78, 79, 80, 1, 2], [12, 13, 14]]
    got = serve.serve(step_mod.B200Step(cfg, w, MAX_SEQ, BATCH), step_mod.B200Head(cfg, head, BATCH),
                      serve.Embeddings(table.cuda()), prompts, 6, chunk=CHUNK)
    want = serve.serve(_OracleStep(cfg, w), _OracleHead(cfg, head), _CpuEmbeddings(table), prompts, 6, chunk=CHUNK)
    assert got.outputs == want.outputs
    assert got.prompt_tokens == sum(map(len, prompts)) and got.generated_tokens == 6 * len(prompts)
    assert got.prefill_calls == 6 and got.total_tokens_per_s > 0
