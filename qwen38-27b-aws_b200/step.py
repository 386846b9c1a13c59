"""The drop-in step objects: `B200Step` and `B200Head`.

`B200Step(**inputs)` has the call of the reference's `NeuronStep.__call__(inputs_embeds, **inputs)`
(qwen38_inf2/neuron.py:273-280) and `SimulatedCoresStep.__call__` (cpu_sim.py:83-85): host tensors
in, the hidden state ``[rows, tokens, hidden]`` back on the host, routed by which inputs are present
exactly as `Qwen38Step.forward` routes them (model.py:983-995):

* decode: inputs_embeds [B, 1, H], cos/sin [B, 1, rot], position int32 [B], active float32 [B];
* prefill: inputs_embeds [1, C, H], cos/sin [1, C, rot], slot/start/n_valid int32 [1]: one row's chunk
  of C tokens, eagerly (the chunk length varies), with buffers sized on first use per C;
* verify: inputs_embeds [B, K, H], cos/sin [B, K, rot], position/active as decode, accepted int32 [B]:
  commit each row's accepted tokens of the last verify step, then run K tokens without changing the
  states (their updates kept pending), eagerly (needs verify_tokens=K at construction);
* save_slot / restore_slot int32 [1]: copy one row's recurrent states, return inputs_embeds.

`B200Head.run_graph(hidden=...)` is the reference's lm_head graph call (generate.py:194):
hidden [B, 1, H] -> group-of-32 maxima [B, V / 32] float32 on the host.

One process drives one GPU. With tp_degree > 1 every rank makes the same calls with the same inputs
(torch.distributed), holds its slice of heads, and the row-parallel outputs are summed across ranks
after o_proj / out_proj / down_proj (model.py:259, :374, :639): by default inside those projections'
GEMM kernels over NVLink peer memory (ops.Communicator, q38_fp8_gemm_allreduce), the residual stream
living in the communicator's shared region; with fused_allreduce=False by a GEMM then an NCCL
all-reduce (the baseline).

The decode step is captured once into a CUDA graph and replayed: ~9 kernels per layer, all on one
stream, with every buffer allocated up front. Nothing here falls back to PyTorch math: the layer
arithmetic is the C-ABI kernels (ops.py) or it fails.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import torch

from . import ops, weights as W
from .config import FULL, LINEAR, TextConfig

BF16 = torch.bfloat16


@dataclass
class _GDN:
    qkvz: ops.DeviceLinear
    ab: ops.DeviceBF16Linear
    conv_w: torch.Tensor
    a_log: torch.Tensor
    dt_bias: torch.Tensor
    norm_w: torch.Tensor
    out: ops.DeviceLinear
    conv_state: torch.Tensor
    state: torch.Tensor
    pending: tuple | None = None  # verify: (key f32, delta f32, log decay f32, conv input bf16) [B, K, ...]


@dataclass
class _Attn:
    qkv: ops.DeviceLinear
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o: ops.DeviceLinear
    k_cache: torch.Tensor
    v_cache: torch.Tensor
    kv_scales: tuple[float, float] | None = None  # the FP8 e4m3 cache's static scales (None: a BF16 cache)


@dataclass
class _Layer:
    kind: str
    ln_in: torch.Tensor
    ln_post: torch.Tensor
    mixer: object
    gate_up: ops.DeviceLinear
    down: ops.DeviceLinear


class _Acts:
    """Activation buffers of one prefill chunk length (attributes set by B200Step._fill_acts)."""


class B200Step:
    """The decoder layers of one rank on one B200, called like the reference's NeuronStep."""

    def __init__(self, cfg: TextConfig, layer_weights, max_seq_len: int, batch_size: int, tp_degree: int = 1,
                 rank: int = 0, device: torch.device | str | None = None, saved_states: bool = False,
                 use_graph: bool = True, process_group=None, verify_tokens: int = 0, fused_allreduce: bool = True,
                 max_chunk: int = 512, kv_cache_format: str = "bf16", kv_scales=None, presharded: bool = False,
                 streamk: bool = False):
        """`layer_weights(i)` returns layer i's unsharded weights (weights.synthetic_layer names), or
        `layer_weights` is a dict holding them all. `kv_cache_format` "fp8" keeps the KV cache as FP8 e4m3
        bytes with static per-layer scales (the reference's kv_cache_format, model.py:556-563): `kv_scales`
        {layer index: (k_scale, v_scale)}, by default weights.synthetic_kv_scales. With `presharded`,
        `layer_weights(i)` already gives this rank's cut (weights.RankShards.layer). At TP = 1 the
        row-parallel projections (out_proj, o_proj, down_proj with the residual add) run as split-K
        clusters, or stream-K (q38_fp8_gemm_streamk) with `streamk=True`."""
        if kv_cache_format not in ("bf16", "fp8"):
            raise ValueError(f"kv_cache_format must be bf16 or fp8, not {kv_cache_format!r}")
        self.kv_fp8 = kv_cache_format == "fp8"
        self.kv_scales = kv_scales
        cfg.validate_tp(tp_degree)
        self.cfg, self.tp, self.rank = cfg, tp_degree, rank
        self.max_seq, self.batch = max_seq_len, batch_size
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        self.group = process_group
        self.use_graph = use_graph
        self.streamk = streamk
        self.saved = saved_states
        self.verify_tokens = verify_tokens
        get = layer_weights if callable(layer_weights) else (lambda i: layer_weights)
        self.comm = None
        with torch.cuda.device(self.device):
            cut = (lambda i: get(i)) if presharded else (lambda i: W.shard_layer(cfg, get(i), i, rank, tp_degree))  # noqa: E731
            self.layers = [self._prepare(i, cut(i)) for i in range(cfg.num_hidden_layers)]
            if tp_degree > 1 and fused_allreduce:
                rows = max(batch_size, batch_size * max(verify_tokens, 1), max_chunk)
                self.comm = ops.Communicator(rank, tp_degree, rows, cfg.hidden_size, self.device, process_group)
            self._alloc_activations()
            self._side = torch.cuda.Stream(device=self.device)
        self._graph = None
        self._graph_key = None
        self._state_rows = None  # every gated-delta layer's state buffers, for copy_states

    # ------------------------------------------------------------------ setup
    def _prepare(self, i: int, w: dict) -> _Layer:
        cfg, dev, p = self.cfg, self.device, f"layers.{i}"
        t = lambda name: w[f"{p}.{name}"].to(dev, BF16).contiguous()  # noqa: E731
        lin = lambda *names: ops.DeviceLinear(W.FP8Weight.cat_rows([w[f"{p}.{n}"] for n in names]), dev)  # noqa: E731
        rows = self.batch * (2 if self.saved else 1)
        if cfg.layer_types[i] == LINEAR:
            hv = cfg.linear_num_value_heads // self.tp
            conv_dim = cfg.linear_conv_dim // self.tp
            mixer = _GDN(
                qkvz=lin("linear_attn.in_proj_qkv", "linear_attn.in_proj_z"),
                ab=ops.DeviceBF16Linear(torch.cat((t("linear_attn.in_proj_b"), t("linear_attn.in_proj_a"))), dev),
                conv_w=t("linear_attn.conv_weight"),
                a_log=t("linear_attn.A_log"),
                dt_bias=t("linear_attn.dt_bias"),
                norm_w=t("linear_attn.norm_weight"),
                out=lin("linear_attn.out_proj"),
                conv_state=torch.zeros(rows, conv_dim, cfg.linear_conv_kernel_dim - 1, dtype=BF16, device=dev),
                state=torch.zeros(rows, hv, cfg.linear_key_head_dim, cfg.linear_value_head_dim, dtype=BF16, device=dev),
            )
            K = self.verify_tokens
            if K:
                f32 = dict(dtype=torch.float32, device=dev)
                mixer.pending = (torch.zeros(self.batch, K, hv, cfg.linear_key_head_dim, **f32),
                                 torch.zeros(self.batch, K, hv, cfg.linear_value_head_dim, **f32),
                                 torch.zeros(self.batch, K, hv, **f32),
                                 torch.zeros(self.batch, K, conv_dim, dtype=BF16, device=dev))
        elif cfg.layer_types[i] == FULL:
            kvh = cfg.kv_heads_per_rank(self.tp)
            scales = None
            if self.kv_fp8:
                held = (f"{p}.self_attn.k_scale", f"{p}.self_attn.v_scale")  # a checkpoint's calibrated scales
                scales = ((self.kv_scales or {}).get(i)
                          or (tuple(float(w[n].reshape(-1)[0]) for n in held) if held[0] in w else None)
                          or W.synthetic_kv_scales(cfg, i))
                scales = tuple(float(torch.tensor(float(v), dtype=BF16)) for v in scales)  # the bf16 parameters
            cache_dtype = torch.uint8 if self.kv_fp8 else BF16
            mixer = _Attn(
                qkv=lin("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"),
                q_norm=t("self_attn.q_norm_weight"),
                k_norm=t("self_attn.k_norm_weight"),
                o=lin("self_attn.o_proj"),
                k_cache=torch.zeros(self.batch, kvh, self.max_seq, cfg.head_dim, dtype=cache_dtype, device=dev),
                v_cache=torch.zeros(self.batch, kvh, self.max_seq, cfg.head_dim, dtype=cache_dtype, device=dev),
                kv_scales=scales,
            )
        else:
            raise ValueError(cfg.layer_types[i])
        # gate_proj and up_proj interleaved in 64-row blocks: the fused GEMM's epilogue finds each gate row's
        # up row in the same 128-row tile and writes SiLU(gate) * up as down_proj's e5m2 input.
        gate_up = ops.DeviceLinear(W.FP8Weight.interleave_rows(w[f"{p}.mlp.gate_proj"], w[f"{p}.mlp.up_proj"]), dev)
        return _Layer(cfg.layer_types[i], t("input_layernorm_weight"), t("post_attention_layernorm_weight"), mixer,
                      gate_up, lin("mlp.down_proj"))

    def _alloc_activations(self):
        self._fill_acts(self, self.batch)
        self.position = torch.zeros(self.batch, dtype=torch.int32, device=self.device)
        self.active = torch.zeros(self.batch, dtype=torch.float32, device=self.device)
        # Attention decode's schedule: rows longest first, recomputed at the start of every decode step
        # (a permutation at all times, so a layer run on its own between steps is still correct).
        self.attn_order = torch.arange(self.batch, dtype=torch.int32, device=self.device)
        self._prefill_acts = {}
        self._verify_acts = None
        cfg = self.cfg
        need = ops.gdn_decode_workspace_bytes(self.batch, cfg.linear_num_key_heads // self.tp, cfg.linear_key_head_dim)
        self.gdn_workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=self.device)
        # Attention split along the cache (long caches, the FP8 cache): one workspace for decode and verify.
        heads, kvh = cfg.num_attention_heads // self.tp, cfg.kv_heads_per_rank(self.tp)
        need = max(ops.attn_split_workspace_bytes(self.batch, heads, kvh, k, self.max_seq, cfg.head_dim)
                   for k in {1, max(self.verify_tokens, 1)})
        self.attn_workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=self.device)

    def _fill_acts(self, a, rows: int) -> None:
        """Activation buffers for `rows` token rows on `a` (the step itself for decode, a _Acts for a
        prefill chunk), with the split-K plan of every GEMM at that row count and one shared workspace."""
        cfg, dev, tp = self.cfg, self.device, self.tp
        H = cfg.hidden_size
        hv = cfg.linear_num_value_heads // tp
        vd = cfg.linear_value_dim // tp
        heads = cfg.num_attention_heads // tp
        inter = cfg.intermediate_size // tp
        z = lambda *s, dt=BF16: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
        # With the fused all-reduce the residual stream is the communicator's (peers write into it).
        a.x = self.comm.x[:rows] if self.comm is not None else z(rows, H)
        a.x_in = z(rows, H)
        a.hb = z(rows, H)
        a.hq = z(rows, H, dt=torch.uint8)
        widths = [l.mixer.qkvz.out_features for l in self.layers if l.kind == LINEAR]
        widths += [l.mixer.qkv.out_features for l in self.layers if l.kind == FULL]
        a.proj = z(rows, max(widths))
        a.ab = z(rows, 2 * hv)
        a.mix_gdn = z(rows, vd, dt=torch.uint8)
        a.mix_attn = z(rows, heads * cfg.head_dim, dt=torch.uint8)
        a.mlp_q = z(rows, inter, dt=torch.uint8)
        a.partial = z(rows, H) if tp > 1 and self.comm is None else None
        a.cos = z(rows, cfg.rotary_dim)
        a.sin = z(rows, cfg.rotary_dim)
        a.splits = {}
        need = 0
        for l in self.layers:
            for lin in (l.mixer.out if l.kind == LINEAR else l.mixer.o, l.down,
                        l.mixer.qkvz if l.kind == LINEAR else l.mixer.qkv):
                sp = ops.choose_splits(rows, lin.out_features, lin.in_features)
                if self.comm is not None and lin is not (l.mixer.qkvz if l.kind == LINEAR else l.mixer.qkv):
                    sp = min(sp, 8)  # the fused all-reduce reduces K splits within one portable cluster
                a.splits[id(lin)] = sp
                need = max(need, ops.gemm_workspace_bytes(rows, lin.out_features, sp))
        hv2 = 2 * cfg.linear_num_value_heads // tp
        a.ab_splits = ops.bf16_linear_splits(rows, hv2, H)
        a.ab_workspace = z(max(ops.gemm_workspace_bytes(rows, hv2, a.ab_splits), 256), dt=torch.uint8)
        a.workspace = z(max(need, 256), dt=torch.uint8)
        a.sk_workspace = None
        if tp == 1 and self.streamk:
            rowpar = [lin for l in self.layers for lin in (l.mixer.out if l.kind == LINEAR else l.mixer.o, l.down)]
            a.sk_workspace = z(max(ops.streamk_workspace_bytes(rows, lin.out_features, lin.in_features) for lin in rowpar),
                               dt=torch.uint8)

    # ------------------------------------------------------------------ kernels of one decode step
    def _gemm(self, a, x_q, lin: ops.DeviceLinear, y, residual=None):
        ops.fp8_gemm(x_q, lin, y, residual=residual, splits=a.splits.get(id(lin), 1), workspace=a.workspace)

    def _row_parallel(self, a, x_q, lin: ops.DeviceLinear):
        """x += all_reduce(bf16(x_q @ W^T)) (the reference's `x + all_reduce(proj(...))`)."""
        if self.tp == 1:
            if a.sk_workspace is not None:
                ops.fp8_gemm_streamk(x_q, lin, a.x, a.sk_workspace, residual=a.x)
            else:
                self._gemm(a, x_q, lin, a.x, residual=a.x)
            return
        if self.comm is not None:
            ops.fp8_gemm_allreduce(x_q, lin, self.comm, splits=a.splits.get(id(lin), 1))
            return
        self._gemm(a, x_q, lin, a.partial)
        torch.distributed.all_reduce(a.partial, group=self.group)
        a.x.add_(a.partial)

    def _decode_layers(self):
        self.x.copy_(self.x_in)
        if self._orders_rows():
            ops.attn_row_order(self.position, self.active, self.max_seq, self.attn_order)
        for l in self.layers:
            self._layer(l, self)

    def _orders_rows(self) -> bool:
        return (any(l.kind == FULL for l in self.layers) and self.batch <= ops.ATTN_ORDER_MAX_ROWS
                and not self._split_attention(0))

    def run_layer(self, i: int) -> None:
        """Layer i alone, eagerly, on self.x and the loaded decode inputs (for layer-by-layer checks)."""
        self._layer(self.layers[i], self)

    def _layer(self, l: _Layer, a, chunk=None, verify: int = 0):
        """DecoderLayer.forward (model.py:918-930) on the activation set `a`: a decode step over all
        rows, with `chunk` = (slot, start, n_valid) one row's prefill chunk of a.x's rows, or with
        `verify` = K the K tokens of every row (a.x row b * K + t)."""
        cfg, eps, tp = self.cfg, self.cfg.rms_norm_eps, self.tp
        m = l.mixer
        if l.kind == LINEAR:
            ops.rmsnorm_quant(a.x, l.ln_in, eps, y_bf16=a.hb, y_e5m2=a.hq)
            # in_proj_b/a (a thin BF16 GEMM on a few SMs, with its own workspace) runs on a side stream
            # beside in_proj_qkvz, whose 2-SM tiles leave SM pairs idle; both join before the mixer.
            main = torch.cuda.current_stream(self.device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                ops.bf16_linear(a.hb, m.ab, a.ab, splits=a.ab_splits, workspace=a.ab_workspace)
            self._gemm(a, a.hq, m.qkvz, a.proj)
            main.wait_stream(self._side)
            heads = dict(num_k_heads=cfg.linear_num_key_heads // tp, num_v_heads=cfg.linear_num_value_heads // tp,
                         head_k=cfg.linear_key_head_dim, head_v=cfg.linear_value_head_dim, eps=eps)
            if verify:
                ops.gdn_verify(a.proj, a.ab, m.conv_state, m.conv_w, m.a_log, m.dt_bias, m.norm_w, m.state, *m.pending,
                               a.position, a.active, a.accepted, a.mix_gdn, batch=self.batch, tokens=verify,
                               workspace=a.gdn_verify_ws, **heads)
            elif chunk is None:
                ops.gdn_decode(a.proj, a.ab, m.conv_state, m.conv_w, m.a_log, m.dt_bias, m.norm_w, m.state,
                               a.position, a.active, a.mix_gdn, batch=self.batch, workspace=self.gdn_workspace, **heads)
            else:
                slot, start, n_valid = chunk
                ops.gdn_prefill(a.proj, a.ab, m.conv_state, m.conv_w, m.a_log, m.dt_bias, m.norm_w, m.state, a.mix_gdn,
                                a.gdn_ws, slot=slot, start=start, n_valid=n_valid, **heads)
            self._row_parallel(a, a.mix_gdn, m.out)
        else:
            ops.rmsnorm_quant(a.x, l.ln_in, eps, y_e5m2=a.hq)
            self._gemm(a, a.hq, m.qkv, a.proj)
            heads = dict(num_q_heads=cfg.num_attention_heads // tp, num_kv_heads=cfg.kv_heads_per_rank(tp),
                         head_dim=cfg.head_dim, rot_dim=cfg.rotary_dim, eps=eps)
            if chunk is None and self._split_attention(verify):
                ops.attn_split(a.proj, m.q_norm, m.k_norm, a.cos, a.sin, m.k_cache, m.v_cache, a.position, a.active,
                               a.mix_attn, batch=self.batch, tokens=max(verify, 1), kv_scales=m.kv_scales,
                               workspace=self.attn_workspace, **heads)
            elif verify:
                ops.attn_verify(a.proj, m.q_norm, m.k_norm, a.cos, a.sin, m.k_cache, m.v_cache, a.position, a.active,
                                a.mix_attn, batch=self.batch, tokens=verify, **heads)
            elif chunk is None:
                ops.attn_decode(a.proj, m.q_norm, m.k_norm, a.cos, a.sin, m.k_cache, m.v_cache, a.position, a.active,
                                a.mix_attn, batch=self.batch, row_order=self.attn_order, **heads)
            else:
                slot, start, _ = chunk
                ops.attn_prefill(a.proj, m.q_norm, m.k_norm, a.cos, a.sin, m.k_cache, m.v_cache, a.mix_attn, a.attn_ws,
                                 slot=slot, start=start, kv_scales=m.kv_scales, **heads)
            self._row_parallel(a, a.mix_attn, m.o)
        ops.rmsnorm_quant(a.x, l.ln_post, eps, y_e5m2=a.hq)
        ops.fp8_gemm_silu(a.hq, l.gate_up, a.mlp_q)
        self._row_parallel(a, a.mlp_q, l.down)

    # Caches up to these lengths fit the one-CTA-per-(row, KV head) decode and verify kernels, which keep
    # every score of the row in shared memory; longer caches and the FP8 cache take the split kernels.
    DECODE_KERNEL_MAX_SEQ = 4096
    VERIFY_KERNEL_MAX_SEQ = 2048

    def _split_attention(self, verify: int) -> bool:
        limit = self.VERIFY_KERNEL_MAX_SEQ if verify else self.DECODE_KERNEL_MAX_SEQ
        return self.kv_fp8 or self.max_seq > limit

    # ------------------------------------------------------------------ prefill
    def _chunk_acts(self, tokens: int):
        a = self._prefill_acts.get(tokens)
        if a is None:
            cfg, tp = self.cfg, self.tp
            a = _Acts()
            with torch.cuda.device(self.device):
                self._fill_acts(a, tokens)
                gdn = ops.gdn_prefill_workspace_bytes(tokens, cfg.linear_num_key_heads // tp,
                                                      cfg.linear_num_value_heads // tp, cfg.linear_key_head_dim,
                                                      cfg.linear_value_head_dim)
                attn = ops.attn_prefill_workspace_bytes(tokens, cfg.num_attention_heads // tp, cfg.head_dim)
                a.gdn_ws = torch.zeros(gdn, dtype=torch.uint8, device=self.device)
                a.attn_ws = torch.zeros(max(attn, 256), dtype=torch.uint8, device=self.device)
            self._prefill_acts[tokens] = a
        return a

    def prefill(self, embeds: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, slot: int, start: int,
                n_valid: int) -> torch.Tensor:
        """One row's chunk (model.py:983-995 with `slot`): embeds [1, C, H] -> hidden [C, H] on the device.
        Tokens from n_valid on are padding: they run through the layers but leave the states alone."""
        tokens = embeds.shape[1]
        if embeds.shape[0] != 1:
            raise ValueError(f"prefill takes [1, chunk, hidden], got {tuple(embeds.shape)}")
        if not 0 <= slot < self.batch:
            raise ValueError(f"slot {slot} outside the {self.batch} rows")
        if not 0 <= n_valid <= tokens or start < 0 or start + tokens > self.max_seq:
            raise ValueError(f"chunk at {start} of {tokens} tokens ({n_valid} valid) does not fit {self.max_seq} positions")
        a = self._load_chunk(embeds, cos, sin)
        for l in self.layers:
            self._layer(l, a, (slot, start, n_valid))
        return a.x

    def _load_chunk(self, embeds, cos, sin):
        tokens = embeds.shape[1]
        a = self._chunk_acts(tokens)
        a.x.copy_(embeds.reshape(tokens, -1), non_blocking=True)
        a.cos.copy_(cos.reshape(tokens, -1), non_blocking=True)
        a.sin.copy_(sin.reshape(tokens, -1), non_blocking=True)
        return a

    def cache_chunk(self, i: int, x: torch.Tensor, cos, sin, slot: int, start: int) -> None:
        """FullAttentionStep.cache_chunk (model.py:795-800) for attention layer i: the chunk's keys and
        values into the slot's cache from the layer input x [C, H] on the device (its norm, qkv projection
        and rotary; the attention output is computed and dropped)."""
        l = self.layers[i]
        if l.kind != FULL:
            raise ValueError(f"layer {i} has no KV cache")
        a = self._load_chunk(x.reshape(1, x.shape[0], -1), cos, sin)
        cfg, m = self.cfg, l.mixer
        ops.rmsnorm_quant(a.x, l.ln_in, cfg.rms_norm_eps, y_e5m2=a.hq)
        self._gemm(a, a.hq, m.qkv, a.proj)
        ops.attn_prefill(a.proj, m.q_norm, m.k_norm, a.cos, a.sin, m.k_cache, m.v_cache, a.mix_attn, a.attn_ws, slot=slot,
                         start=start, num_q_heads=cfg.num_attention_heads // self.tp,
                         num_kv_heads=cfg.kv_heads_per_rank(self.tp), head_dim=cfg.head_dim, rot_dim=cfg.rotary_dim,
                         eps=cfg.rms_norm_eps, kv_scales=m.kv_scales)

    def run_prefill_layer(self, i: int, embeds, cos, sin, slot: int, start: int, n_valid: int) -> torch.Tensor:
        """Layer i alone on a prefill chunk whose input is `embeds` [1, C, H] (for layer-by-layer checks)."""
        a = self._load_chunk(embeds, cos, sin)
        self._layer(self.layers[i], a, (slot, start, n_valid))
        return a.x

    # ------------------------------------------------------------------ verify
    def verify(self, embeds, cos, sin, position, active, accepted) -> torch.Tensor:
        """K tokens per row for speculative decoding (model.py:983-995 with `accepted`): embeds [B, K, H]
        -> hidden [B * K, H] on the device."""
        K = self.verify_tokens
        B = self.batch
        if not K:
            raise ValueError("this step was built without verify_tokens")
        if tuple(embeds.shape[:2]) != (B, K):
            raise ValueError(f"verify takes [{B}, {K}, hidden], got {tuple(embeds.shape)}")
        acc = accepted.reshape(-1)
        if acc.numel() != B or int(acc.min()) < 0 or int(acc.max()) > K:
            raise ValueError(f"accepted must hold {B} counts in 0..{K}")
        a = self._verify_acts
        if a is None:
            a = _Acts()
            with torch.cuda.device(self.device):
                self._fill_acts(a, B * K)
                a.position = torch.zeros(B, dtype=torch.int32, device=self.device)
                a.active = torch.zeros(B, dtype=torch.float32, device=self.device)
                a.accepted = torch.zeros(B, dtype=torch.int32, device=self.device)
                cfg = self.cfg
                need = ops.gdn_verify_workspace_bytes(B, K, cfg.linear_num_key_heads // self.tp, cfg.linear_key_head_dim)
                a.gdn_verify_ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=self.device)
            self._verify_acts = a
        a.x.copy_(embeds.reshape(B * K, -1), non_blocking=True)
        a.cos.copy_(cos.reshape(B * K, -1), non_blocking=True)
        a.sin.copy_(sin.reshape(B * K, -1), non_blocking=True)
        a.position.copy_(position.reshape(-1).to(torch.int32), non_blocking=True)
        a.active.copy_(active.reshape(-1).to(torch.float32), non_blocking=True)
        a.accepted.copy_(acc.to(torch.int32), non_blocking=True)
        for l in self.layers:
            self._layer(l, a, verify=K)
        return a.x

    def kernels_per_decode_step(self) -> int:
        """Launches of this library's kernels in one decode step (for the bench's gpu_launches)."""
        n = 1 if self._orders_rows() else 0  # the attention row order
        attn = 6 if self._split_attention(0) else 4  # rmsnorm, qkv, attention (3 launches when split), o_proj
        for l in self.layers:
            n += (6 if l.kind == LINEAR else attn) + 3  # GDN: rmsnorm, qkvz, ab, q/k prep, decode, out_proj; MLP: 3
        return n

    def decode_device(self):
        """One decode step over the inputs already in the device buffers (x_in, cos, sin, position, active)."""
        if self.use_graph and (self.tp == 1 or self.comm is not None):
            if self._graph is None:
                self._capture()
            self._graph.replay()
        else:
            self._decode_layers()
        return self.x

    def _capture(self):
        # One warm-up pass outside capture (per-device kernel attributes, module loading) with every
        # row inactive: inactive rows keep their recurrent and conv states bit for bit and write their
        # key/value only at the cache's last position, which no sequence reads (model.py:621).
        active = self.active.clone()
        self.active.zero_()
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._decode_layers()
        torch.cuda.current_stream(self.device).wait_stream(side)
        self.active.copy_(active)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph):
            self._decode_layers()

    def close(self) -> None:
        """Releases the CUDA graph and the communicator's peer mappings (call before the process group goes)."""
        self._graph = None
        if self.comm is not None:
            torch.cuda.synchronize(self.device)
            self.comm.close()
            self.comm = None

    # ------------------------------------------------------------------ the reference's call
    def __call__(self, inputs_embeds: torch.Tensor, **inputs: torch.Tensor) -> torch.Tensor:
        if "save_slot" in inputs or "restore_slot" in inputs:
            self.copy_states(inputs)
            return inputs_embeds
        if "accepted" in inputs:
            out = self.verify(inputs_embeds, inputs["cos"], inputs["sin"], inputs["position"], inputs["active"],
                              inputs["accepted"])
            return _to_host(out).reshape(self.batch, self.verify_tokens, -1)
        if "slot" in inputs:
            scalar = lambda name: int(inputs[name].reshape(-1)[0])  # noqa: E731
            out = self.prefill(inputs_embeds, inputs["cos"], inputs["sin"], scalar("slot"), scalar("start"),
                               scalar("n_valid"))
            return _to_host(out).reshape(1, inputs_embeds.shape[1], -1)
        rows = inputs_embeds.shape[0]
        if rows != self.batch or inputs_embeds.shape[1] != 1:
            raise ValueError(f"decode takes [{self.batch}, 1, hidden], got {tuple(inputs_embeds.shape)}")
        self.load_decode_inputs(inputs_embeds, inputs["cos"], inputs["sin"], inputs["position"], inputs["active"])
        out = self.decode_device()
        return _to_host(out).reshape(rows, 1, -1)

    def load_decode_inputs(self, embeds, cos, sin, position, active):
        self.x_in.copy_(embeds.reshape(self.batch, -1), non_blocking=True)
        self.cos.copy_(cos.reshape(self.batch, -1), non_blocking=True)
        self.sin.copy_(sin.reshape(self.batch, -1), non_blocking=True)
        self.position.copy_(position.reshape(-1).to(torch.int32), non_blocking=True)
        self.active.copy_(active.reshape(-1).to(torch.float32), non_blocking=True)

    def copy_states(self, inputs):
        """Save one row's recurrent and conv states to its spare row or restore them (model.py:456-464)."""
        if not self.saved:
            raise ValueError("this step keeps no saved states")
        to_saved = "save_slot" in inputs
        slot = int((inputs["save_slot"] if to_saved else inputs["restore_slot"]).reshape(-1)[0])
        if not 0 <= slot < self.batch:
            raise ValueError(f"slot {slot} outside the {self.batch} rows")
        src, dst = (slot, slot + self.batch) if to_saved else (slot + self.batch, slot)
        if self._state_rows is None:
            bufs = [b for l in self.layers if l.kind == LINEAR for b in (l.mixer.state, l.mixer.conv_state)]
            self._state_rows = ops.StateRows(bufs)
        with torch.cuda.device(self.device):
            self._state_rows.copy(src, dst)


def _to_host(t: torch.Tensor) -> torch.Tensor:
    """A new host tensor holding t, in page-locked memory from torch's caching host allocator (a fresh
    tensor per call costs no allocation once the cache holds a block of its size), copied at full PCIe
    speed; returns once the copy is done. Page-locked outputs also make a caller's copy back to the
    device (the head's input) a true asynchronous copy."""
    out = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    out.copy_(t, non_blocking=True)
    torch.cuda.current_stream(t.device).synchronize()
    return out


class B200Head:
    """Final norm and the lm_head group maxima of one rank's vocab slice (HeadStep, model.py:863-900)."""

    def __init__(self, cfg: TextConfig, head_weights: dict, batch_size: int, tp_degree: int = 1, rank: int = 0,
                 device=None, group_rows: int = 32, process_group=None, presharded: bool = False):
        if group_rows != 32:
            raise ValueError("the lm_head kernel takes groups of 32")
        self.cfg, self.batch, self.tp, self.rank = cfg, batch_size, tp_degree, rank
        self.group = process_group
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        shard = head_weights if presharded else W.shard_head(cfg, head_weights, rank, tp_degree)
        self.norm_w = shard["norm_weight"].to(self.device, BF16).contiguous()
        # The kernel multiplies BF16 by BF16: the e4m3 * 2^s weights are exact in BF16.
        self.lm_head = ops.DeviceBF16Linear(shard["lm_head"].to(self.device).dequant().to(BF16), self.device)
        self.vocab_local = self.lm_head.out_features
        self.hidden = torch.zeros(batch_size, cfg.hidden_size, dtype=BF16, device=self.device)
        self.xb = torch.zeros_like(self.hidden)
        self.maxima = torch.zeros(batch_size, self.vocab_local // 32, dtype=torch.float32, device=self.device)
        self.gathered = (torch.zeros(tp_degree, batch_size, self.vocab_local // 32, dtype=torch.float32, device=self.device)
                         if tp_degree > 1 else None)
        self._tokens = None  # next_tokens' device buffers, made on first use

    def maxima_device(self) -> torch.Tensor:
        ops.rmsnorm_quant(self.hidden, self.norm_w, self.cfg.rms_norm_eps, y_bf16=self.xb)
        ops.lm_head_groupmax(self.xb, self.lm_head, self.maxima)
        if self.tp == 1:
            return self.maxima
        torch.distributed.all_gather_into_tensor(self.gathered, self.maxima, group=self.group)
        return self.gathered.permute(1, 0, 2).reshape(self.batch, -1)

    def next_tokens(self, hidden: torch.Tensor, recheck_groups: int | None = None) -> list[int]:
        """ChipHead.next_tokens (generate.py:186-208) with its exact recheck on the device: hidden [rows, 1, H]
        (rows <= batch, padded like the reference) -> the greedy token of each row. The maxima stay on the
        GPU; only the token ids come back. `recheck_groups` (default 4) is how many of the best groups are
        rescored, as ChipHead's argument of that name."""
        rows = hidden.shape[0]
        if rows > self.batch:
            raise ValueError(f"the head takes at most {self.batch} rows, got {rows}")
        k = recheck_groups or 4
        with torch.cuda.device(self.device):
            if self._tokens is None:
                self._tokens = torch.zeros(self.batch, dtype=torch.int32, device=self.device)
                self._slots = {}
            if k not in self._slots:  # contiguous per-candidate buffers, for the cross-rank max
                self._slots[k] = (torch.zeros(self.batch, k, dtype=torch.float32, device=self.device),
                                  torch.zeros(self.batch, k, dtype=torch.int32, device=self.device))
            self.hidden.zero_()
            self.hidden[:rows].copy_(hidden.reshape(rows, -1), non_blocking=True)
            maxima = self.maxima_device()
            eps = self.cfg.rms_norm_eps
            if self.tp == 1:
                ops.lm_head_recheck(self.hidden, self.norm_w, eps, maxima, self.lm_head, 0, k, tokens=self._tokens)
            else:
                logits, toks = self._slots[k]
                ops.lm_head_recheck(self.hidden, self.norm_w, eps, maxima, self.lm_head, self.rank * self.vocab_local, k,
                                    slot_logits=logits, slot_tokens=toks)
                # Each candidate slot is scored on the one rank holding its group; -inf / -1 elsewhere.
                torch.distributed.all_reduce(logits, op=torch.distributed.ReduceOp.MAX, group=self.group)
                torch.distributed.all_reduce(toks, op=torch.distributed.ReduceOp.MAX, group=self.group)
                ops.lm_head_pick(logits, toks, self._tokens)
            tokens = _to_host(self._tokens[:rows]).tolist()
        for row, t in enumerate(tokens):
            if t < 0:
                raise FloatingPointError(f"row {row}'s logits are not finite, so the graph produced NaN or infinity")
        return tokens

    def run_graph(self, hidden: torch.Tensor) -> torch.Tensor:
        rows = hidden.shape[0]
        if rows != self.batch:
            raise ValueError(f"the head graph takes {self.batch} rows, got {rows}")
        self.hidden.copy_(hidden.reshape(rows, -1), non_blocking=True)
        return _to_host(self.maxima_device())


class B200MTP:
    """The MTP draft layer (MTPStep, qwen38_inf2/model.py:812-860) of one rank, called as the reference's
    MTP graph: `mtp(hidden=..., inputs_embeds=..., **generate.mtp_step_inputs(...))` for K tokens per row
    (Scheduler._mtp_drafts, scheduler.py:160-193), or with `generate.mtp_prefill_inputs` for a prompt
    chunk of one row, which only fills the layer's cache (Scheduler._mtp_prefill, scheduler.py:145-158).
    Host tensors in, host tensors out.

    fc's input [normed embedding | twice-normed hidden state] is cut by columns into tp equal slices:
    rank r multiplies its slice, and the partial products are summed across ranks by the fused GEMM +
    all-reduce (at tp = 2 this is the reference's rank_gate split; it holds for any tp). The decoder layer
    is a one-layer B200Step in its verify form: each token against the layer's cache before its position
    and its step's own tokens up to itself. The output is the layer's norm divided by (1 + the final
    norm's weight), one kernel (q38_rmsnorm_divide)."""

    def __init__(self, cfg: TextConfig, mtp_weights: dict, max_seq_len: int, batch_size: int, tokens: int = 4,
                 tp_degree: int = 1, rank: int = 0, device=None, process_group=None, fused_allreduce: bool = True,
                 max_chunk: int = 512, kv_cache_format: str = "bf16", kv_scales=None, presharded: bool = False):
        self.cfg, self.tp, self.rank, self.batch, self.tokens = cfg, tp_degree, rank, batch_size, tokens
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        self.group = process_group
        layer_w = {k: v for k, v in mtp_weights.items() if k.startswith("layers.")}
        self.layer = B200Step(replace(cfg, layer_types=(FULL,)), layer_w, max_seq_len, batch_size, tp_degree, rank,
                              self.device, use_graph=False, process_group=process_group, verify_tokens=tokens,
                              fused_allreduce=fused_allreduce, max_chunk=max_chunk, kv_cache_format=kv_cache_format,
                              kv_scales={0: kv_scales} if kv_scales else None)
        shard = W.shard_mtp(cfg, mtp_weights, rank, tp_degree)
        H = cfg.hidden_size
        rows = max(batch_size * tokens, max_chunk)
        dev = self.device
        with torch.cuda.device(dev):
            self.fc = ops.DeviceLinear(shard["fc"], dev)
            vec = lambda name: shard[name].to(dev, BF16).contiguous()  # noqa: E731
            self.embedding_norm, self.hidden_norm = vec("embedding_norm_weight"), vec("hidden_norm_weight")
            self.norm, self.final_norm = vec("norm_weight"), vec("final_norm_weight")
            z = lambda *sh, dt=BF16: torch.zeros(*sh, dtype=dt, device=dev)  # noqa: E731
            self.emb, self.hid, self.tmp, self.out = z(rows, H), z(rows, H), z(rows, H), z(rows, H)
            self.x = z(rows, H)
            self.joined = z(rows, 2 * H, dt=torch.uint8)  # e5m2 of [normed embedding | normed hidden]
            self.fc_in = z(rows, 2 * H // tp_degree, dt=torch.uint8) if tp_degree > 1 else None
            self.fc_ws = z(max(256, max(ops.gemm_workspace_bytes(r, H, 8) for r in (batch_size * tokens, max_chunk))),
                           dt=torch.uint8)

    def _project(self, rows: int) -> torch.Tensor:
        """x = all_reduce(fc(e5m2([rms(embedding) | rms(rms(hidden, final), hidden)]))) [rows, H] on the device."""
        cfg, H, eps = self.cfg, self.cfg.hidden_size, self.cfg.rms_norm_eps
        ops.rmsnorm_quant(self.emb[:rows], self.embedding_norm, eps, y_e5m2=self.joined[:rows, :H])
        ops.rmsnorm_quant(self.hid[:rows], self.final_norm, eps, y_bf16=self.tmp[:rows])
        ops.rmsnorm_quant(self.tmp[:rows], self.hidden_norm, eps, y_e5m2=self.joined[:rows, H:])
        splits = ops.choose_splits(rows, H, self.fc.in_features)
        if self.tp == 1:
            ops.fp8_gemm(self.joined[:rows], self.fc, self.x[:rows], splits=splits, workspace=self.fc_ws)
            return self.x[:rows]
        width = 2 * H // self.tp
        self.fc_in[:rows].copy_(self.joined[:rows, self.rank * width:(self.rank + 1) * width])
        comm = self.layer.comm
        if comm is not None:
            comm.x[:rows].zero_()  # the fused projection adds into the residual stream
            ops.fp8_gemm_allreduce(self.fc_in[:rows], self.fc, comm, splits=min(splits, 8))
            return comm.x[:rows]
        ops.fp8_gemm(self.fc_in[:rows], self.fc, self.x[:rows], splits=splits, workspace=self.fc_ws)
        torch.distributed.all_reduce(self.x[:rows], group=self.group)
        return self.x[:rows]

    def __call__(self, hidden: torch.Tensor, inputs_embeds: torch.Tensor, cos, sin, position=None, active=None,
                 slot=None, start=None, n_valid=None) -> torch.Tensor:
        H = self.cfg.hidden_size
        rows = inputs_embeds.shape[0] * inputs_embeds.shape[1]
        with torch.cuda.device(self.device):
            self.emb[:rows].copy_(inputs_embeds.reshape(rows, H), non_blocking=True)
            self.hid[:rows].copy_(hidden.reshape(rows, H), non_blocking=True)
            x = self._project(rows)
            if slot is not None:
                # Prefill only fills the layer's cache; the reference returns the projection's first row.
                scalar = lambda v: int(v.reshape(-1)[0])  # noqa: E731
                self.layer.cache_chunk(0, x, cos, sin, scalar(slot), scalar(start))
                return _to_host(x[:1]).reshape(1, 1, H)
            B, K = inputs_embeds.shape[:2]
            if (B, K) != (self.batch, self.tokens):
                raise ValueError(f"MTP steps take [{self.batch}, {self.tokens}, hidden], got {tuple(inputs_embeds.shape)}")
            y = self.layer.verify(x.reshape(B, K, H), cos, sin, position, active, torch.zeros(B, dtype=torch.int32))
            ops.rmsnorm_divide(y, self.norm, self.final_norm, self.cfg.rms_norm_eps, self.out[:rows])
            return _to_host(self.out[:rows]).reshape(B, K, H)

    def close(self) -> None:
        self.layer.close()
