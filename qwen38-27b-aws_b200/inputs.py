"""Host-side inputs of the step calls, as the reference's callers build them (qwen38_inf2/generate.py:25-115).

These define the drop-in boundary's arguments: B200Step, B200MTP and B200Head take exactly the tensors
these functions return, so a caller written against the reference (batched_greedy_generate, Scheduler)
and this package's own serving loop (serve.py) feed the same inputs. Positions are int32, activity
float32, cos / sin bf16 of the rotary dimensions (theta = rope_theta, the first rotary_dim dims).
"""

from __future__ import annotations

from typing import Sequence

import torch

from .config import TextConfig

BF16 = torch.bfloat16


def rotary(cfg: TextConfig, positions: torch.Tensor, dtype=BF16) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin [len(positions), rotary_dim]: frequencies 1 / theta^(2i / dim) for the half dims, each repeated
    over both halves (generate.py:25-31; the same fp32 operations in the same order, so the tables match
    the reference's bit for bit)."""
    dim = cfg.rotary_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    angles = positions.to(torch.float32).reshape(-1, 1) * inv
    return angles.cos().repeat(1, 2).to(dtype), angles.sin().repeat(1, 2).to(dtype)


def decode_inputs(cfg: TextConfig, positions: Sequence[int], max_seq_len: int, active: Sequence[bool] | None = None,
                  dtype=BF16) -> dict[str, torch.Tensor]:
    """One token per row, each at its own position (generate.batch_step_inputs, generate.py:38-55). The
    cache's last position takes inactive rows' writes, so active rows must be below it."""
    pos = torch.as_tensor(list(positions), dtype=torch.int32)
    on = torch.ones(len(pos), dtype=torch.bool) if active is None else torch.as_tensor(list(active), dtype=torch.bool)
    if bool((pos[on] >= max_seq_len - 1).any()):
        raise ValueError(f"position {int(pos[on].max())} is past the last usable one of max_seq_len {max_seq_len}")
    cos, sin = rotary(cfg, pos, dtype)
    return {"cos": cos.unsqueeze(1), "sin": sin.unsqueeze(1), "position": pos, "active": on.to(torch.float32)}


def prefill_inputs(cfg: TextConfig, slot: int, start: int, n_valid: int, chunk: int, dtype=BF16) -> dict[str, torch.Tensor]:
    """A chunk of `chunk` tokens of one row from `start`, the first `n_valid` real (generate.py:58-69)."""
    if start < 0 or not 0 < n_valid <= chunk:
        raise ValueError(f"a chunk starts at a position >= 0 and holds 1 to {chunk} tokens")
    cos, sin = rotary(cfg, start + torch.arange(chunk), dtype)
    as1 = lambda v: torch.tensor([v], dtype=torch.int32)  # noqa: E731
    return {"cos": cos.unsqueeze(0), "sin": sin.unsqueeze(0), "slot": as1(slot), "start": as1(start), "n_valid": as1(n_valid)}


def verify_inputs(cfg: TextConfig, positions: Sequence[int], tokens: int, max_seq_len: int, active: Sequence[bool],
                  accepted: Sequence[int], dtype=BF16) -> dict[str, torch.Tensor]:
    """`tokens` tokens per row from each row's position, committing `accepted` of the last verify step's
    (generate.py:72-87)."""
    pos = torch.as_tensor(list(positions), dtype=torch.int32)
    on = torch.as_tensor(list(active), dtype=torch.bool)
    if bool((pos[on] + tokens > max_seq_len - 1).any()):
        raise ValueError(f"{tokens} tokens from position {int(pos[on].max())} pass max_seq_len {max_seq_len}")
    cos, sin = rotary(cfg, (pos.unsqueeze(-1) + torch.arange(tokens)).reshape(-1), dtype)
    return {"cos": cos.reshape(len(pos), tokens, -1), "sin": sin.reshape(len(pos), tokens, -1), "position": pos,
            "active": on.to(torch.float32), "accepted": torch.as_tensor(list(accepted), dtype=torch.int32)}


def mtp_step_inputs(cfg: TextConfig, indices: Sequence[int], tokens: int, max_seq_len: int, active: Sequence[bool],
                    dtype=BF16) -> dict[str, torch.Tensor]:
    """The MTP layer's steps: `tokens` per row from each row's MTP index, rotary at the index plus one
    (generate.py:90-99)."""
    out = verify_inputs(cfg, indices, tokens, max_seq_len, active, [0] * len(indices), dtype)
    del out["accepted"]
    at = (torch.as_tensor(list(indices), dtype=torch.int32).unsqueeze(-1) + 1 + torch.arange(tokens)).reshape(-1)
    cos, sin = rotary(cfg, at, dtype)
    out["cos"], out["sin"] = cos.reshape(len(indices), tokens, -1), sin.reshape(len(indices), tokens, -1)
    return out


def mtp_prefill_inputs(cfg: TextConfig, slot: int, start: int, n_valid: int, chunk: int, dtype=BF16) -> dict[str, torch.Tensor]:
    """The MTP layer's prefill chunk from MTP index `start`, rotary one on (generate.py:102-107)."""
    out = prefill_inputs(cfg, slot, start, n_valid, chunk, dtype)
    cos, sin = rotary(cfg, start + 1 + torch.arange(chunk), dtype)
    out["cos"], out["sin"] = cos.unsqueeze(0), sin.unsqueeze(0)
    return out


def state_copy_inputs(cfg: TextConfig, slot: int, save: bool, dtype=BF16) -> dict[str, torch.Tensor]:
    """Save or restore one row's recurrent states (generate.py:110-115)."""
    return {"inputs_embeds": torch.zeros(1, 1, cfg.hidden_size, dtype=dtype),
            ("save_slot" if save else "restore_slot"): torch.tensor([slot], dtype=torch.int32)}
