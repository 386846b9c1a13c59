"""CPU restatement of the reference's step (test infrastructure: the checker, never the product).

This is the arithmetic of qwen38_inf2/model.py's CPU branches (`device.type == "cpu"`), restated
function by function with the same rounding points, so that its outputs can be compared with the
CUDA path bit for bit where the arithmetic is integer-like and within tolerance where fp32 sums are
reordered. Each function cites the reference lines it follows. One deliberate difference, the one
BASELINE asks for: FP8 linears decode e4m3 weights with per-32 power-of-two scales instead of the
reference's scale-free e5m2 bytes; the reference's own test swaps the codec the same way
(tests/test_model_parity.py:255-257).

State lives in plain dicts of tensors (per layer): conv_state, recurrent_state, k_cache, v_cache,
and for verify the pending_* buffers, shaped as the reference's module buffers.
"""

from __future__ import annotations

import importlib
import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

_pkg = importlib.import_module("qwen38-27b-aws_b200")
LINEAR = _pkg.config.LINEAR
FULL = _pkg.config.FULL

MASKED_SCORE = -1e4  # model.py:32
DELTA_CHUNK = 128  # model.py:34
ATTENTION_BLOCK = 2048  # model.py:36


# ---------------------------------------------------------------------------------------------
# Elementwise pieces (model.py:44-87)
# ---------------------------------------------------------------------------------------------
def silu(x: torch.Tensor) -> torch.Tensor:
    """x * sigmoid(x) in x's dtype (model.py:48-51)."""
    return x * torch.sigmoid(x)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """fp32 RMS norm times (1 + w), back to x's dtype (model.py:54-57)."""
    h = x.float()
    h = h * torch.rsqrt((h * h).mean(-1, keepdim=True) + eps)
    return (h * (1.0 + weight.float())).type_as(x)


def l2_norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """model.py:60-61."""
    return x * torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)


def repeat_heads(x: torch.Tensor, repeats: int, dim: int) -> torch.Tensor:
    """Each head repeated `repeats` times in place, as repeat_interleave (model.py:64-67)."""
    return x.repeat_interleave(repeats, dim=dim)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    """model.py:70-72."""
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rotary(q, k, cos, sin):
    """Partial rotary over the first cos.shape[-1] dims, in the tensors' dtype (model.py:75-82)."""
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    n = cos.shape[-1]
    qr = q[..., :n] * cos + rotate_half(q[..., :n]) * sin
    kr = k[..., :n] * cos + rotate_half(k[..., :n]) * sin
    return torch.cat((qr, q[..., n:]), dim=-1), torch.cat((kr, k[..., n:]), dim=-1)


def fp8_round(x: torch.Tensor) -> torch.Tensor:
    """e5m2 and back (model.py:85-87)."""
    return x.to(torch.float8_e5m2).to(x.dtype)


def rotary(cfg, positions: torch.Tensor, dtype: torch.dtype):
    """cos, sin ``[len(positions), rotary_dim]`` (generate.py:25-31)."""
    dim = cfg.rotary_dim
    inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
    freqs = positions.float().unsqueeze(-1) * inv_freq
    return freqs.cos().repeat(1, 2).to(dtype), freqs.sin().repeat(1, 2).to(dtype)


@dataclass
class Linear:
    """An FP8 linear: e4m3 bytes [out, in] and per-32 scales, applied as the reference's CPU branch
    applies `weight_fp8`: x rounded to e5m2, then a matmul with the dequantised weight cast to x's
    dtype (model.py:221-225)."""

    q: torch.Tensor
    scale: torch.Tensor
    _w: dict = field(default_factory=dict)
    # Accumulate as an fp32 matmul instead of the BF16 one (same values, another summation order):
    # used only to measure how much the model's output moves under a legitimate reordering.
    fp32: bool = False

    def weight(self, dtype) -> torch.Tensor:
        if dtype not in self._w:
            self._w[dtype] = _pkg.codec.dequantize_mx_e4m3(self.q, self.scale).to(dtype)
        return self._w[dtype]

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x = fp8_round(x)
        if self.fp32:
            return F.linear(x.float(), self.weight(torch.float32)).to(x.dtype)
        return F.linear(x, self.weight(x.dtype))


def linear_of(w) -> Linear:
    return Linear(w.q.cpu(), w.scale.cpu())


# ---------------------------------------------------------------------------------------------
# The chunked gated delta rule (model.py:90-155)
# ---------------------------------------------------------------------------------------------
def unit_lower_inverse(lower: torch.Tensor, base: int = 8) -> torch.Tensor:
    """(I - lower)^-1 by blocked forward substitution (model.py:131-155): blocks of `base` by the
    product series, then neighbouring blocks merged with the block-triangular inverse formula."""
    n = lower.shape[-1]
    idx = torch.arange(n)
    same = (idx // base).unsqueeze(-1) == (idx // base)
    local = lower * same
    inv = torch.eye(n) + local
    power = local
    for _ in range(int(math.log2(base)) - 1):
        power = power @ power
        inv = inv + inv @ power
    size = base
    while size < n:
        merged = inv.clone()
        for first in range(0, n, 2 * size):
            top, bot = slice(first, first + size), slice(first + size, first + 2 * size)
            merged[..., bot, top] = inv[..., bot, bot] @ lower[..., bot, top] @ inv[..., top, top]
        inv, size = merged, 2 * size
    return inv


def chunked_gated_delta(query, key, value, log_decay, beta, state, chunk: int = DELTA_CHUNK):
    """The gated delta rule over [heads, tokens, ...] in pieces of `chunk` tokens (model.py:90-128)."""
    heads, tokens, dk = key.shape
    pieces = tokens // chunk
    q = query.reshape(heads, pieces, chunk, dk)
    k = key.reshape(heads, pieces, chunk, dk)
    v = value.reshape(heads, pieces, chunk, -1)
    g = log_decay.reshape(heads, pieces, chunk).cumsum(-1)
    b = beta.reshape(heads, pieces, chunk, 1)
    idx = torch.arange(chunk)
    causal = (idx.unsqueeze(-1) >= idx.unsqueeze(0)).float()
    below = (idx.unsqueeze(-1) > idx.unsqueeze(0)).float()
    decay = ((g.unsqueeze(-1) - g.unsqueeze(-2)) * causal).exp() * causal
    kb = k * b
    inv = unit_lower_inverse(-(kb @ k.transpose(-1, -2)) * decay * below)
    u = inv @ (v * b)
    w = inv @ (kb * g.exp().unsqueeze(-1))
    outs = []
    for i in range(pieces):
        attn = (q[:, i] @ k[:, i].transpose(-1, -2)) * decay[:, i]
        vn = u[:, i] - w[:, i] @ state
        outs.append((q[:, i] * g[:, i].exp().unsqueeze(-1)) @ state + attn @ vn)
        last = g[:, i, -1]
        state = state * last.exp().reshape(heads, 1, 1) + (
            k[:, i] * (last.unsqueeze(-1) - g[:, i]).exp().unsqueeze(-1)
        ).transpose(-1, -2) @ vn
    return torch.cat(outs, dim=1), state


def recurrent_gated_delta(query, key, value, log_decay, beta, state):
    """The rule one token at a time (tests/test_prefill.py:18-26 states it the same way)."""
    outs = []
    for t in range(key.shape[1]):
        state = state * log_decay[:, t].exp().reshape(-1, 1, 1)
        delta = (value[:, t] - (state * key[:, t].unsqueeze(-1)).sum(-2)) * beta[:, t].unsqueeze(-1)
        state = state + key[:, t].unsqueeze(-1) * delta.unsqueeze(-2)
        outs.append((state * query[:, t].unsqueeze(-1)).sum(-2))
    return torch.stack(outs, dim=1), state


def blocked_attention(query, keys, values, visible, block: int = ATTENTION_BLOCK):
    """Online-softmax attention in blocks of positions (model.py:170-191)."""
    best = torch.full((*query.shape[:2], 1), 2 * MASKED_SCORE)
    total = torch.zeros(*query.shape[:2], 1)
    out = torch.zeros(*query.shape[:2], values.shape[-1])
    for first in range(0, keys.shape[1], block):
        s = (query @ keys[:, first : first + block].transpose(-1, -2)).float()
        s = s + torch.where(visible[:, first : first + block], 0.0, MASKED_SCORE)
        nb = torch.maximum(best, s.amax(dim=-1, keepdim=True))
        wts = (s - nb).exp()
        rescale = (best - nb).exp()
        total = total * rescale + wts.sum(dim=-1, keepdim=True)
        out = out * rescale + (wts.to(values.dtype) @ values[:, first : first + block]).float()
        best = nb
    return out / total


# ---------------------------------------------------------------------------------------------
# Layers
# ---------------------------------------------------------------------------------------------
class GDNLayer:
    """GatedDeltaNetStep's CPU branches (model.py:274-521) for one rank's heads."""

    def __init__(self, cfg, w: dict, prefix: str, tp: int, batch: int, dtype, verify_tokens: int = 0,
                 saved_states: bool = False):
        self.cfg, self.dtype = cfg, dtype
        la = f"{prefix}.linear_attn"
        self.qkv = linear_of(w[f"{la}.in_proj_qkv"])
        self.z = linear_of(w[f"{la}.in_proj_z"])
        self.out = linear_of(w[f"{la}.out_proj"])
        self.b = w[f"{la}.in_proj_b"].cpu().to(dtype)
        self.a = w[f"{la}.in_proj_a"].cpu().to(dtype)
        self.conv_w = w[f"{la}.conv_weight"].cpu().to(dtype)
        self.A_log = w[f"{la}.A_log"].cpu().to(dtype)
        self.dt_bias = w[f"{la}.dt_bias"].cpu().to(dtype)
        self.norm_w = w[f"{la}.norm_weight"].cpu().to(dtype)
        self.hk = cfg.linear_num_key_heads // tp
        self.hv = cfg.linear_num_value_heads // tp
        self.kd, self.vd = self.hk * cfg.linear_key_head_dim, self.hv * cfg.linear_value_head_dim
        conv_dim = 2 * self.kd + self.vd
        self.batch = batch
        rows = batch * (2 if saved_states else 1)
        self.conv_state = torch.zeros(rows, conv_dim, cfg.linear_conv_kernel_dim - 1, dtype=dtype)
        sdt = {"float32": torch.float32, "bf16": torch.bfloat16}[cfg.recurrent_state_format]
        self.state_dtype = sdt
        self.recurrent_state = torch.zeros(rows, self.hv, cfg.linear_key_head_dim, cfg.linear_value_head_dim, dtype=sdt)
        if verify_tokens:
            dk, dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
            self.pending_key = torch.zeros(batch, verify_tokens, self.hv, dk)
            self.pending_delta = torch.zeros(batch, verify_tokens, self.hv, dv)
            self.pending_decay = torch.zeros(batch, verify_tokens, self.hv)
            self.pending_input = torch.zeros(batch, verify_tokens, conv_dim, dtype=dtype)

    def split(self, mixed):
        """q, k per value head, v, all fp32 (model.py:322-331)."""
        n = mixed.shape[0]
        dk, dv, rep = self.cfg.linear_key_head_dim, self.cfg.linear_value_head_dim, self.cfg.linear_key_repeat
        q = mixed[:, : self.kd].reshape(n, self.hk, dk)
        k = mixed[:, self.kd : 2 * self.kd].reshape(n, self.hk, dk)
        v = mixed[:, 2 * self.kd :].reshape(n, self.hv, dv)
        q, k = repeat_heads(q, rep, 1), repeat_heads(k, rep, 1)
        return l2_norm(q.float()) / math.sqrt(dk), l2_norm(k.float()), v.float()

    def gates(self, x):
        """beta and log decay [tokens, v_heads] (model.py:333-337)."""
        beta = F.linear(x, self.b).sigmoid().float()
        a = F.linear(x, self.a).float()
        return beta, -self.A_log.float().exp() * F.softplus(a + self.dt_bias.float())

    def finish(self, out, z):
        """Gated RMS norm per head, then out_proj (model.py:339-345)."""
        return self.out(self.gated_norm(out, z).reshape(out.shape[0], 1, self.vd))

    def live(self, buf):
        return buf[: self.batch]

    def decode(self, x, position, active):
        """One token per row (model.py:347-374). x [B, 1, H]."""
        B = x.shape[0]
        qkv = self.qkv(x).reshape(B, -1)
        z = self.z(x).reshape(B, -1)
        xf = x.reshape(B, -1)
        h = self.decode_core(qkv, z, F.linear(xf, self.b), F.linear(xf, self.a), position, active)
        return self.out(h.reshape(B, 1, self.vd))

    def decode_core(self, qkv, z, b_raw, a_raw, position, active):
        """Everything between the input projections and out_proj for one token per row: qkv
        [B, conv_dim], z [B, value_dim], b_raw/a_raw [B, v_heads] (the in_proj_b / in_proj_a outputs).
        Returns out_proj's input [B, value_dim] and updates the states (model.py:350-373, :339-344)."""
        dt, B = qkv.dtype, qkv.shape[0]
        on = active.reshape(B, 1, 1) > 0.5
        keep = torch.where((position == 0) & (active > 0.5), 0.0, 1.0)
        qkv = qkv.unsqueeze(-1)
        cs = self.live(self.conv_state)
        window = torch.cat((cs * keep.reshape(B, 1, 1).to(dt), qkv), dim=-1)
        self.conv_state[:B] = torch.where(on, window[:, :, 1:], cs)
        q, k, v = self.split(silu((window * self.conv_w).sum(dim=-1)))
        z = z.reshape(B, self.hv, -1)
        beta = b_raw.sigmoid().float()
        log_decay = -self.A_log.float().exp() * F.softplus(a_raw.float() + self.dt_bias.float())
        beta = (beta * active.unsqueeze(-1)).unsqueeze(-1)
        log_decay = log_decay * active.unsqueeze(-1)
        s = self.live(self.recurrent_state).float() * keep.reshape(B, 1, 1, 1) * log_decay.exp()[..., None, None]
        delta = (v - (s * k.unsqueeze(-1)).sum(dim=-2)) * beta
        s = s + k.unsqueeze(-1) * delta.unsqueeze(-2)
        self.recurrent_state[:B] = s.to(self.state_dtype)
        out = (s * q.unsqueeze(-1)).sum(dim=-2).to(dt)
        return self.gated_norm(out, z).reshape(B, self.vd)

    def gated_norm(self, out, z):
        """The gated RMS norm of `_finish` without the projection (model.py:339-344)."""
        h = out.float()
        h = h * torch.rsqrt((h * h).mean(-1, keepdim=True) + self.cfg.rms_norm_eps)
        h = self.norm_w * h.to(self.dtype)
        return (h * silu(z.float())).to(self.dtype)

    def prefill(self, x, slot, start, n_valid):
        """A chunk of one row (model.py:476-521, CPU branch). x [1, T, H]."""
        T = x.shape[1]
        h = self.prefill_core(self.qkv(x)[0], self.z(x)[0], F.linear(x[0], self.b), F.linear(x[0], self.a), slot, start,
                              n_valid)
        return self.out(h.reshape(T, 1, self.vd)).reshape(1, T, -1)

    def prefill_core(self, qkv, z, b_raw, a_raw, slot, start, n_valid):
        """Between the projections of `prefill`: qkv [T, conv_dim], z [T, value_dim], b_raw/a_raw [T, v_heads]
        (the in_proj_b / in_proj_a outputs). Returns out_proj's input [T, value_dim] and replaces the
        slot's states (model.py:481-521)."""
        dt, T = qkv.dtype, qkv.shape[0]
        kern = self.cfg.linear_conv_kernel_dim
        s_idx, keep = int(slot.reshape(-1)[0]), (start > 0).to(dt)
        valid = (torch.arange(T) < n_valid).float()
        history = self.conv_state[s_idx] * keep
        window = torch.cat((history.transpose(0, 1), qkv))
        carried = window.index_select(0, n_valid.long().reshape(-1) + torch.arange(kern - 1)).transpose(0, 1)
        self.conv_state[s_idx] = carried
        beta = b_raw.sigmoid().float()
        log_decay = -self.A_log.float().exp() * F.softplus(a_raw.float() + self.dt_bias.float())
        beta, log_decay = beta * valid.unsqueeze(-1), log_decay * valid.unsqueeze(-1)
        state = self.recurrent_state[s_idx].float() * keep.float()
        conv = sum(window.transpose(0, 1)[:, j : j + T] * self.conv_w[:, j : j + 1] for j in range(kern))
        q, k, v = self.split(silu(conv).transpose(0, 1))
        out, state = chunked_gated_delta(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), log_decay.transpose(0, 1),
                                         beta.transpose(0, 1), state, min(DELTA_CHUNK, T))
        self.recurrent_state[s_idx] = state.to(self.state_dtype)
        z = z.reshape(T, self.hv, -1)
        return self.gated_norm(out.transpose(0, 1).to(dt), z).reshape(T, self.vd)

    def verify(self, x, position, active, accepted):
        """K tokens per row (model.py:376-454). x [B, K, H]."""
        B, K = x.shape[:2]
        xf = x.reshape(B * K, -1)
        h = self.verify_core(self.qkv(x), self.z(x), F.linear(xf, self.b).reshape(B, K, -1),
                             F.linear(xf, self.a).reshape(B, K, -1), position, active, accepted)
        return self.out(h.reshape(B * K, 1, self.vd)).reshape(B, K, -1)

    def verify_core(self, qkv, z, b_raw, a_raw, position, active, accepted):
        """Between the projections of `verify`: qkv [B, K, conv_dim], z [B, K, value_dim], b_raw/a_raw
        [B, K, v_heads]. Commits the last verify step's first `accepted` tokens (from the pending buffers),
        runs the K tokens from the committed state as one small chunk, keeps their updates pending, and
        returns out_proj's input [B, K, value_dim] (model.py:383-453, _commit_and_read :262-271)."""
        dt = qkv.dtype
        B, K = qkv.shape[:2]
        kern = self.cfg.linear_conv_kernel_dim
        dk, dv = self.cfg.linear_key_head_dim, self.cfg.linear_value_head_dim
        on = (active > 0.5).reshape(B, 1)
        keep = torch.where((position.reshape(B, 1) == 0) & on, 0.0, 1.0)
        # Commit: decay by the accepted tokens' log decays, plus each one's key x delta decayed by those after it.
        taken = [(accepted.reshape(B, 1) > j).float() for j in range(K)]
        decays = [self.pending_decay[:, j] * taken[j] for j in range(K)]
        remaining = sum(decays)
        scale = torch.where(on, remaining.exp() * keep, 1.0)
        weighted = []
        for j in range(K):
            remaining = remaining - decays[j]
            weighted.append(self.pending_key[:, j] * (remaining.exp() * taken[j] * keep * on).unsqueeze(-1))
        # The conv history: the kern - 1 inputs before the first uncommitted token.
        cs = self.live(self.conv_state)
        window = torch.cat((cs, self.pending_input.transpose(1, 2)), dim=-1)
        at = (accepted.long().reshape(B, 1, 1) + torch.arange(kern - 1)).expand(-1, window.shape[1], -1)
        history = torch.where(on.reshape(B, 1, 1), window.gather(2, at) * keep.reshape(B, 1, 1).to(dt), cs)
        self.conv_state[:B] = history
        window = torch.cat((history, qkv.transpose(1, 2)), dim=-1)
        mixed = torch.stack([(window[:, :, t : t + kern] * self.conv_w).sum(dim=-1) for t in range(K)], dim=1)
        q, k, v = (part.reshape(B, K, *part.shape[1:]) for part in self.split(silu(mixed).reshape(B * K, -1)))
        beta = b_raw.sigmoid().float() * active.reshape(B, 1, 1)
        log_decay = (-self.A_log.float().exp() * F.softplus(a_raw.float() + self.dt_bias.float())) * active.reshape(B, 1, 1)
        # The committed state (rounded to the state's dtype) and the new tokens' keys and queries against it.
        heads = self.hv
        pairs = B * heads
        state = self.live(self.recurrent_state).reshape(pairs, dk, dv)
        w_k = torch.stack(weighted, dim=2).reshape(pairs, -1, dk)
        deltas = self.pending_delta.transpose(1, 2).reshape(pairs, -1, dv)
        committed = (state.float() * scale.reshape(pairs, 1, 1).expand(-1, dk, -1) + w_k.transpose(1, 2) @ deltas).to(state.dtype)
        self.recurrent_state[:B] = committed.reshape(B, heads, dk, dv)
        reads = torch.cat((k, q), dim=1).permute(0, 2, 3, 1).reshape(pairs, dk, 2 * K)
        products = (reads.transpose(1, 2) @ committed.float()).reshape(B, heads, 2 * K, dv).transpose(1, 2)
        k_state, q_state = products[:, :K], products[:, K:]
        # The K tokens as one chunk: a K x K triangular solve for the deltas, then the outputs.
        cum = [log_decay[:, 0]]
        for t in range(1, K):
            cum.append(cum[-1] + log_decay[:, t])
        deltas, outs = [], []
        for t in range(K):
            d = v[:, t] - cum[t].exp().unsqueeze(-1) * k_state[:, t]
            for j in range(t):
                d = d - ((cum[t] - cum[j]).exp() * (k[:, t] * k[:, j]).sum(dim=-1)).unsqueeze(-1) * deltas[j]
            deltas.append(d * beta[:, t].unsqueeze(-1))
            o = cum[t].exp().unsqueeze(-1) * q_state[:, t]
            for j in range(t + 1):
                o = o + ((cum[t] - cum[j]).exp() * (q[:, t] * k[:, j]).sum(dim=-1)).unsqueeze(-1) * deltas[j]
            outs.append(o)
        self.pending_key = k.float().clone()
        self.pending_delta = torch.stack(deltas, dim=1)
        self.pending_decay = log_decay.float().clone()
        self.pending_input = qkv.clone()
        out = torch.stack(outs, dim=1).reshape(B * K, heads, -1).to(dt)
        return self.gated_norm(out, z.reshape(B * K, heads, -1)).reshape(B, K, self.vd)

    def copy_states(self, slot: int, to_saved: bool):
        """model.py:456-464."""
        if self.recurrent_state.shape[0] == self.batch:
            raise ValueError("this layer keeps no saved states")
        src, dst = (slot, slot + self.batch) if to_saved else (slot + self.batch, slot)
        self.recurrent_state[dst] = self.recurrent_state[src]
        self.conv_state[dst] = self.conv_state[src]


FP8_E4M3_MAX = 240.0  # model.py:37-41: the largest e4m3 value the cache's static scales assume


class AttentionLayer:
    """FullAttentionStep's CPU branches (model.py:524-809) for one rank's heads, with a BF16 cache or,
    with `kv_scales` = (k_scale, v_scale) (bf16 scalars), the FP8 e4m3 cache (uint8 bytes of
    value / scale, clamped to +-240; model.py:579-608)."""

    def __init__(self, cfg, w: dict, prefix: str, tp: int, rank: int, batch: int, max_seq: int, dtype, kv_scales=None):
        self.cfg, self.dtype, self.max_seq = cfg, dtype, max_seq
        self.scales = None if kv_scales is None else tuple(torch.as_tensor(s, dtype=dtype).reshape(1) for s in kv_scales)
        sa = f"{prefix}.self_attn"
        self.q = linear_of(w[f"{sa}.q_proj"])
        self.k = linear_of(w[f"{sa}.k_proj"])
        self.v = linear_of(w[f"{sa}.v_proj"])
        self.o = linear_of(w[f"{sa}.o_proj"])
        self.q_norm = w[f"{sa}.q_norm_weight"].cpu().to(dtype)
        self.k_norm = w[f"{sa}.k_norm_weight"].cpu().to(dtype)
        self.heads = cfg.num_attention_heads // tp
        self.kv_heads = cfg.kv_heads_per_rank(tp)
        hd = cfg.head_dim
        cache_dtype = dtype if self.scales is None else torch.uint8
        self.k_cache = torch.zeros(batch, self.kv_heads, max_seq, hd, dtype=cache_dtype)
        self.v_cache = torch.zeros(batch, self.kv_heads, max_seq, hd, dtype=cache_dtype)

    @property
    def groups(self):
        return self.heads // self.kv_heads

    def store(self, t, which: int):
        """What the cache holds for t: itself, or e4m3 bytes of t / scale clamped to +-240 (model.py:579-585)."""
        if self.scales is None:
            return t
        scale = self.scales[which].float()
        return (t.float() / scale).clamp(-FP8_E4M3_MAX, FP8_E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)

    def load(self, t, which: int):
        """Cached values back from `store` (model.py:587-589)."""
        if self.scales is None:
            return t
        return (t.view(torch.float8_e4m3fn).to(self.dtype) * self.scales[which]).to(self.dtype)

    def round_trip(self, t, which: int):
        """A key or value as it reads back from the cache (model.py:591-593)."""
        return self.load(self.store(t, which), which)

    def project(self, x, cos, sin):
        """model.py:565-577."""
        rows, T = x.shape[:2]
        return self.norm_rope(self.q(x), self.k(x), self.v(x), cos, sin)

    def norm_rope(self, qg, k, v, cos, sin):
        """From the raw q_proj/k_proj/v_proj outputs [rows, T, ...]: q/k RMS norms, rotary, the gate
        (model.py:570-577)."""
        hd, eps = self.cfg.head_dim, self.cfg.rms_norm_eps
        rows, T = qg.shape[:2]
        qg = qg.reshape(rows, T, self.heads, hd * 2)
        query, gate = qg[..., :hd], qg[..., hd:]
        query = rms_norm(query, self.q_norm, eps).transpose(1, 2)
        key = rms_norm(k.reshape(rows, T, self.kv_heads, hd), self.k_norm, eps).transpose(1, 2)
        value = v.reshape(rows, T, self.kv_heads, hd).transpose(1, 2)
        query, key = apply_rotary(query, key, cos, sin)
        return query, key, value, gate.reshape(rows, T, self.heads * hd)

    def write(self, key, value, positions):
        """Scatter keys/values [rows, kv, n, hd] at each row's positions [rows, n] (model.py:603-608)."""
        rows, kvh, n, hd = key.shape
        at = positions.reshape(rows, 1, n, 1).expand(-1, kvh, -1, hd)
        self.k_cache.scatter_(2, at, key)
        self.v_cache.scatter_(2, at, value)

    def decode(self, x, cos, sin, position, active):
        """model.py:610-639 (BF16 cache)."""
        return self.o(self.decode_core(self.q(x), self.k(x), self.v(x), cos, sin, position, active))

    def decode_core(self, qg, k, v, cos, sin, position, active):
        """From the raw projections [B, 1, ...] to o_proj's input [B, 1, heads * hd], writing the
        token's key and value to the cache (model.py:613-639 without o_proj)."""
        hd, B = self.cfg.head_dim, qg.shape[0]
        query, key, value, gate = self.norm_rope(qg, k, v, cos, sin)
        grouped = query.reshape(B, self.kv_heads, self.groups, hd)
        where = torch.where(active > 0.5, position.long(), self.max_seq - 1).unsqueeze(-1)
        earlier = torch.arange(self.max_seq) < position.unsqueeze(-1)
        keys, values = self.load(self.k_cache, 0), self.load(self.v_cache, 1)
        cached = torch.matmul(grouped, keys.transpose(2, 3)).float() + torch.where(earlier, 0.0, MASKED_SCORE).reshape(B, 1, 1, -1)
        own = torch.matmul(grouped, self.round_trip(key, 0).transpose(2, 3)).float()
        wts = torch.softmax(torch.cat((cached, own), dim=-1) * hd**-0.5, dim=-1).to(qg.dtype)
        out = torch.matmul(wts[..., :-1], values) + wts[..., -1:] * self.round_trip(value, 1)
        out = out.reshape(B, 1, self.heads * hd)
        self.write(self.store(key, 0), self.store(value, 1), where)
        return out * torch.sigmoid(gate)

    def verify(self, x, cos, sin, position, active):
        """K tokens per row (model.py:641-675, BF16 cache)."""
        return self.o(self.verify_core(self.q(x), self.k(x), self.v(x), cos, sin, position, active))

    def verify_core(self, qg, k, v, cos, sin, position, active):
        """From the raw projections [B, K, ...] to o_proj's input [B, K, heads * hd]: each token against the
        cache before `position` and the step's own tokens up to itself; the tokens' keys and values are
        written from `position` on (inactive rows at the last K positions) (model.py:648-675)."""
        hd = self.cfg.head_dim
        B, K = qg.shape[:2]
        query, key, value, gate = self.norm_rope(qg, k, v, cos, sin)
        steps = torch.arange(K)
        where = torch.where(active.unsqueeze(-1) > 0.5, position.long().unsqueeze(-1) + steps, self.max_seq - K + steps)
        grouped = query.reshape(B, self.kv_heads, self.groups, K, hd)
        earlier = torch.arange(self.max_seq) < position.unsqueeze(-1)
        keys, values = self.load(self.k_cache, 0), self.load(self.v_cache, 1)
        cached = torch.matmul(grouped, keys.unsqueeze(2).transpose(-1, -2)).float()
        cached = cached + torch.where(earlier, 0.0, MASKED_SCORE).reshape(B, 1, 1, 1, -1)
        causal = steps.unsqueeze(0) <= steps.unsqueeze(-1)
        own_key = self.round_trip(key, 0).unsqueeze(2)
        own = torch.matmul(grouped, own_key.transpose(-1, -2)).float() + torch.where(causal, 0.0, MASKED_SCORE)
        wts = torch.softmax(torch.cat((cached, own), dim=-1) * hd**-0.5, dim=-1).to(qg.dtype)
        out = (torch.matmul(wts[..., : self.max_seq], values.unsqueeze(2))
               + torch.matmul(wts[..., self.max_seq :], self.round_trip(value, 1).unsqueeze(2)))
        out = out.permute(0, 3, 1, 2, 4).reshape(B, K, self.heads * hd)
        self.write(self.store(key, 0), self.store(value, 1), where)
        return out * torch.sigmoid(gate)

    def prefill(self, x, cos, sin, slot, start, n_valid):
        """model.py:732-786 (CPU branch, BF16 cache)."""
        return self.o(self.prefill_core(self.q(x), self.k(x), self.v(x), cos, sin, slot, start))

    def prefill_core(self, qg, k, v, cos, sin, slot, start):
        """Between the projections of `prefill`: raw q_proj/k_proj/v_proj outputs [1, T, ...] to o_proj's input
        [1, T, heads * hd], writing the chunk's keys and values to the slot's cache (model.py:735-786)."""
        hd, T = self.cfg.head_dim, qg.shape[1]
        G = self.groups
        s_idx, st = int(slot.reshape(-1)[0]), int(start.reshape(-1)[0])
        query, key, value, gate = self.norm_rope(qg, k, v, cos, sin)
        grouped = (query[0] * hd**-0.5).reshape(self.kv_heads, G * T, hd)
        own_k, own_v = self.round_trip(key[0], 0), self.round_trip(value[0], 1)
        index = torch.arange(G * T) % T
        visible = torch.cat(((torch.arange(self.max_seq) < st).expand(G * T, -1), torch.arange(T).unsqueeze(0) <= index.unsqueeze(-1)), dim=-1)
        keys = torch.cat((self.load(self.k_cache[s_idx], 0), own_k), dim=1)
        values = torch.cat((self.load(self.v_cache[s_idx], 1), own_v), dim=1)
        out = blocked_attention(grouped, keys, values, visible, ATTENTION_BLOCK)
        out = out.to(qg.dtype).reshape(self.heads, T, hd).transpose(0, 1).reshape(1, T, self.heads * hd)
        self.k_cache[s_idx, :, st : st + T] = self.store(key[0], 0)
        self.v_cache[s_idx, :, st : st + T] = self.store(value[0], 1)
        return out * torch.sigmoid(gate)


class MLPLayer:
    """model.py:241-259 (CPU branch)."""

    def __init__(self, w: dict, prefix: str):
        self.gate = linear_of(w[f"{prefix}.mlp.gate_proj"])
        self.up = linear_of(w[f"{prefix}.mlp.up_proj"])
        self.down = linear_of(w[f"{prefix}.mlp.down_proj"])

    def __call__(self, x):
        return self.down(silu(self.gate(x)) * self.up(x))


class OracleStep:
    """Qwen38Step on CPU for one rank (model.py:903-995): same call, same routing by inputs.

    `weights` holds the layers' (possibly TP-sharded) tensors named as weights.synthetic_layer names
    them, with layer indices from 0 within this step's layer list.
    """

    def __init__(self, cfg, weights: dict, max_seq_len: int, batch_size: int = 1, tp_degree: int = 1, rank: int = 0,
                 all_reduce=None, dtype=torch.bfloat16, saved_states: bool = False, linear_fp32: bool = False,
                 verify_tokens: int = 0, kv_scales=None):
        """`kv_scales` {layer index: (k_scale, v_scale)} gives those attention layers the FP8 e4m3 cache."""
        self.cfg, self.dtype = cfg, dtype
        self.all_reduce = all_reduce or (lambda t: t)
        self.layers = []
        for i, kind in enumerate(cfg.layer_types):
            p = f"layers.{i}"
            mixer = (GDNLayer(cfg, weights, p, tp_degree, batch_size, dtype, verify_tokens, saved_states) if kind == LINEAR
                     else AttentionLayer(cfg, weights, p, tp_degree, rank, batch_size, max_seq_len, dtype,
                                         (kv_scales or {}).get(i)))
            self.layers.append((kind, mixer, MLPLayer(weights, p), weights[f"{p}.input_layernorm_weight"].cpu().to(dtype),
                                weights[f"{p}.post_attention_layernorm_weight"].cpu().to(dtype)))
        if linear_fp32:
            for _, mixer, mlp, *_r in self.layers:
                for obj in (mixer, mlp):
                    for v in vars(obj).values():
                        if isinstance(v, Linear):
                            v.fp32 = True

    def __call__(self, inputs_embeds, cos=None, sin=None, position=None, active=None, slot=None, start=None,
                 n_valid=None, save_slot=None, restore_slot=None, accepted=None):
        if save_slot is not None or restore_slot is not None:
            which = save_slot if save_slot is not None else restore_slot
            for kind, mixer, *_ in self.layers:
                if kind == LINEAR:
                    mixer.copy_states(int(which.reshape(-1)[0]), save_slot is not None)
            return inputs_embeds
        x = inputs_embeds.to(self.dtype)
        for i in range(len(self.layers)):
            x = self.layer(i, x, cos, sin, position, active, slot, start, n_valid, accepted)
        return x

    def layer(self, i, x, cos=None, sin=None, position=None, active=None, slot=None, start=None, n_valid=None,
              accepted=None):
        """DecoderLayer.forward (model.py:918-930) for layer i alone."""
        eps = self.cfg.rms_norm_eps
        kind, mixer, mlp, w_in, w_post = self.layers[i]
        h = rms_norm(x, w_in, eps)
        if accepted is not None:
            m = mixer.verify(h, position, active, accepted) if kind == LINEAR else mixer.verify(h, cos, sin, position, active)
        elif slot is not None:
            m = mixer.prefill(h, slot, start, n_valid) if kind == LINEAR else mixer.prefill(h, cos, sin, slot, start, n_valid)
        else:
            m = mixer.decode(h, position, active) if kind == LINEAR else mixer.decode(h, cos, sin, position, active)
        x = x + self.all_reduce(m)
        return x + self.all_reduce(mlp(rms_norm(x, w_post, eps)))


class OracleMTP:
    """MTPStep's CPU branch (model.py:812-860) for one rank: the normed embedding of token t + 1 and the
    twice-normed hidden state at t, joined and projected by fc, then one full-attention decoder layer in
    its verify form over its own KV cache (prefill only writes that cache), the layer's norm divided by
    (1 + the final norm's weight). With TP > 1, rank r takes fc's input columns r * 2H / tp .. (r + 1) *
    2H / tp of the joined row (the reference's rank_gate split is this at tp = 2), summed by all_reduce."""

    def __init__(self, cfg, weights: dict, max_seq_len: int, batch_size: int, tp_degree: int = 1, rank: int = 0,
                 all_reduce=None, dtype=torch.bfloat16, kv_scales=None):
        from dataclasses import replace

        self.cfg, self.tp, self.rank = cfg, tp_degree, rank
        self.all_reduce = all_reduce or (lambda t: t)
        self.fc = linear_of(weights["fc"])
        norm = lambda name: weights[name].cpu().to(dtype)  # noqa: E731
        self.embedding_norm, self.hidden_norm = norm("embedding_norm_weight"), norm("hidden_norm_weight")
        self.norm, self.final_norm = norm("norm_weight"), norm("final_norm_weight")
        layer = {k: v for k, v in weights.items() if k.startswith("layers.")}
        self.step = OracleStep(replace(cfg, layer_types=(FULL,)), layer, max_seq_len, batch_size, tp_degree, rank,
                               self.all_reduce, dtype, kv_scales={0: kv_scales} if kv_scales else None)

    @property
    def attention(self):
        return self.step.layers[0][1]

    def __call__(self, hidden, inputs_embeds, cos, sin, position=None, active=None, slot=None, start=None, n_valid=None):
        eps = self.cfg.rms_norm_eps
        embedded = rms_norm(inputs_embeds, self.embedding_norm, eps)
        state = rms_norm(rms_norm(hidden, self.final_norm, eps), self.hidden_norm, eps)
        joined = torch.cat((embedded, state), dim=-1)
        if self.tp > 1:
            width = joined.shape[-1] // self.tp
            joined = joined[..., self.rank * width:(self.rank + 1) * width]
        x = self.all_reduce(self.fc(joined))
        if slot is not None:
            # cache_chunk (model.py:855-856, :795-800): only the layer's keys and values are kept.
            _, mixer, _, w_in, _ = self.step.layers[0]
            mixer.prefill(rms_norm(x, w_in, eps), cos, sin, slot, start, n_valid)
            return x[:, :1]
        x = self.step.layer(0, x, cos, sin, position, active, accepted=active)
        out = rms_norm(x, self.norm, eps)
        return (out.float() / (1.0 + self.final_norm.float())).to(x.dtype)


# ---------------------------------------------------------------------------------------------
# Head (model.py:863-900, generate.py:186-208)
# ---------------------------------------------------------------------------------------------
def head_maxima(cfg, hidden, norm_weight, lm_head_q, lm_head_scale, group: int = 32) -> torch.Tensor:
    """HeadStep's CPU branch for one vocab slice: fp32 logits of the bf16-normed rows against the
    dequantised lm_head, then the max of each group of `group` tokens (model.py:890-895)."""
    x = rms_norm(hidden, norm_weight, cfg.rms_norm_eps).reshape(hidden.shape[0], -1)
    weight = _pkg.codec.dequantize_mx_e4m3(lm_head_q, lm_head_scale)  # [vocab, hidden]
    logits = x.float() @ weight.T
    return torch.stack([g.amax(dim=-1) for g in logits.split(group, dim=-1)], dim=-1)


def recheck_tokens(cfg, hidden, norm_weight, lm_head_rows_fp32, maxima, group: int = 32, recheck_groups: int = 4):
    """ChipHead.next_tokens's host recheck (generate.py:186-208): the best `recheck_groups` groups of
    each row rescored exactly against the lm_head rows with the fp32-normed hidden state."""
    best = maxima.float().topk(min(recheck_groups, maxima.shape[-1]), dim=-1).indices.tolist()
    norm = rms_norm(hidden.float(), norm_weight, cfg.rms_norm_eps).reshape(hidden.shape[0], -1)
    tokens = []
    for row, groups in enumerate(best):
        best_token, best_logit = -1, -torch.inf
        for g in groups:
            first = g * group
            logit, index = (lm_head_rows_fp32[first : first + group] @ norm[row]).max(dim=0)
            if logit > best_logit:
                best_token, best_logit = first + int(index), logit
        if best_token < 0:
            raise FloatingPointError(f"row {row}'s logits are not finite")
        tokens.append(best_token)
    return tokens
