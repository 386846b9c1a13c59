"""Prefill-first serving over the drop-in step objects: the "total tokens/s (prefill + decode)" workload.

The reference's Scheduler.run without speculation (qwen38_inf2/scheduler.py:204-267, its _prefill
:110-143): every free slot takes the next waiting prompt, which is prefilled chunk by chunk into that
row (generate.prefill_inputs), its first new token chosen from the last prompt token's hidden state; then
one decode step for every running row (generate.batch_step_inputs), a token each, until a row has
max_new_tokens or reaches the cache's last usable position, and its slot takes the next prompt. The calls
are the reference's: B200Step(**inputs) for prefill and decode, B200Head.next_tokens for the greedy
token (its exact recheck on the GPU). Embeddings are rows of a device table gathered on the GPU.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Sequence

import torch

from . import inputs as I
from . import ops


@dataclass
class ServeStats:
    prompt_tokens: int = 0
    generated_tokens: int = 0
    prefill_calls: int = 0
    decode_steps: int = 0
    prefill_s: float = 0.0
    decode_s: float = 0.0
    wall_s: float = 0.0
    outputs: dict = field(default_factory=dict)

    @property
    def total_tokens_per_s(self) -> float:
        return (self.prompt_tokens + self.generated_tokens) / self.wall_s if self.wall_s else 0.0


class Embeddings:
    """ChipHead.embed_batch (generate.py:183-184) on the device: rows of a bf16 table [vocab, hidden] on the GPU."""

    def __init__(self, table: torch.Tensor):
        self.table = table
        self.device = table.device

    def embed(self, ids: Sequence[int]) -> torch.Tensor:
        """[len(ids), hidden] bf16 on the device."""
        idx = torch.tensor(list(ids), dtype=torch.int32).to(self.device, non_blocking=True)
        out = torch.empty(len(idx), self.table.shape[1], dtype=self.table.dtype, device=self.device)
        return ops.embed_rows(self.table, idx, out)


def serve(step, head, embeddings: Embeddings, prompts: Sequence[Sequence[int]], max_new_tokens: int,
          chunk: int = 512) -> ServeStats:
    """Runs every prompt to max_new_tokens greedy tokens through `step`'s slots; returns the tokens per
    prompt and the time spent. step.max_seq - chunk positions per row are usable, as in the reference."""
    cfg, B, max_seq = step.cfg, step.batch, step.max_seq
    for p in prompts:
        if not p or len(p) >= max_seq - chunk:
            raise ValueError(f"prompts need 1 .. {max_seq - chunk - 1} tokens")
    stats = ServeStats(outputs={i: [] for i in range(len(prompts))})
    waiting = list(range(len(prompts)))[::-1]
    rows: list[dict | None] = [None] * B
    t_start = time.perf_counter()
    while waiting or any(rows):
        for slot in range(B):
            if rows[slot] is not None or not waiting:
                continue
            index = waiting.pop()
            ids = list(prompts[index])
            t0 = time.perf_counter()
            hidden = None
            for start in range(0, len(ids), chunk):
                piece = ids[start:start + chunk]
                emb = embeddings.embed(piece + [0] * (chunk - len(piece))).reshape(1, chunk, -1)
                hidden = step(inputs_embeds=emb, **I.prefill_inputs(cfg, slot, start, len(piece), chunk))
                stats.prefill_calls += 1
            last = (len(ids) - 1) % chunk
            token = head.next_tokens(hidden[:, last:last + 1])[0]
            stats.prefill_s += time.perf_counter() - t0
            stats.prompt_tokens += len(ids)
            stats.generated_tokens += 1
            stats.outputs[index].append(token)
            rows[slot] = {"index": index, "last": token, "position": len(ids), "new": 1}
            if max_new_tokens <= 1:
                rows[slot] = None
        if not any(rows):
            continue
        t0 = time.perf_counter()
        active = [r is not None for r in rows]
        positions = [r["position"] if r else 0 for r in rows]
        emb = embeddings.embed([r["last"] if r else 0 for r in rows]).reshape(B, 1, -1)
        hidden = step(inputs_embeds=emb, **I.decode_inputs(cfg, positions, max_seq, active))
        tokens = head.next_tokens(hidden)
        stats.decode_steps += 1
        stats.decode_s += time.perf_counter() - t0
        for slot, r in enumerate(rows):
            if r is None:
                continue
            r["position"] += 1
            r["new"] += 1
            r["last"] = tokens[slot]
            stats.generated_tokens += 1
            stats.outputs[r["index"]].append(tokens[slot])
            if r["new"] >= max_new_tokens or r["position"] + 1 > max_seq - chunk:
                rows[slot] = None
    stats.wall_s = time.perf_counter() - t_start
    return stats
