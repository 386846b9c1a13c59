"""One wrapper per C-ABI call of include/q38.h, taking torch CUDA tensors.

Each launches on the current torch stream and raises `_lib.Q38Error` on a bad status. Shapes and
dtypes are checked here so a wrong call fails on the host with a message, not on the device.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib, codec

BF16 = torch.bfloat16
U8 = torch.uint8


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("all tensors must be on a CUDA device")


class DeviceLinear:
    """An FP8 linear prepared for the GEMM kernel: e4m3 bytes [out, in] in 16 KB swizzled tiles and
    tiled UE8M0 scales."""

    def __init__(self, w, device):
        self.out_features, self.in_features = w.q.shape
        self.q = codec.tile_weight(w.q.to(device=device, dtype=U8))
        self.sf = codec.tile_scales(codec.scale_to_ue8m0(w.scale.to(device))).contiguous()
        lib = _lib.load()
        _need(self.sf.numel() == lib.q38_sf_tile_bytes(self.out_features, self.in_features), "scale tiling mismatch")
        _need(self.q.numel() == lib.q38_weight_tile_bytes(self.out_features, self.in_features), "weight tiling mismatch")

    @property
    def nbytes(self) -> int:
        return self.q.numel() + self.sf.numel()


class DeviceBF16Linear:
    """A BF16 weight [out, in] in the GEMM kernel's swizzled 16 KB tiles (64 values of K per tile row)."""

    def __init__(self, w: torch.Tensor, device):
        self.out_features, self.in_features = w.shape
        self.w = codec.tile_weight(w.to(device=device, dtype=BF16))
        _need(self.w.numel() == _lib.load().q38_weight_tile_bytes(self.out_features, 2 * self.in_features),
              "weight tiling mismatch")


def token_tile(tokens: int) -> int:
    return 256 if tokens > 128 else 128


def choose_splits(tokens: int, features: int, k: int, sms: int = 148) -> int:
    """K splits that bring the grid near one CTA per SM for weight-streaming (few-token) GEMMs."""
    tiles = -(-features // 128) * -(-tokens // token_tile(tokens))
    kc = -(-k // 128)
    if tiles >= sms // 2:
        return 1
    return max(1, min(kc // 4, sms // tiles))


def gemm_workspace_bytes(tokens: int, features: int, splits: int) -> int:
    return _lib.load().q38_fp8_gemm_workspace_bytes(tokens, features, splits)


def fp8_gemm(x_e5m2: torch.Tensor, lin: DeviceLinear, y: torch.Tensor, residual: torch.Tensor | None = None,
             splits: int = 1, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """y[:, :out] = bf16(e5m2(x) @ W^T) (+ residual, in bf16)."""
    _cuda(x_e5m2, y, residual, workspace)
    _need(x_e5m2.dtype == U8 and x_e5m2.dim() == 2 and x_e5m2.stride(1) == 1 and x_e5m2.stride(0) == x_e5m2.shape[1],
          "x must be contiguous uint8 e5m2 [tokens, k]")
    tokens, k = x_e5m2.shape
    _need(k == lin.in_features, f"x has {k} columns, the weight {lin.in_features}")
    _need(y.dtype == BF16 and y.dim() == 2 and y.stride(1) == 1 and y.shape[0] >= tokens, "y must be bf16 [tokens, >= out]")
    epi = 0
    ldr = 0
    if residual is not None:
        _need(residual.dtype == BF16 and residual.stride(1) == 1, "residual must be bf16 with unit column stride")
        epi, ldr = 1, residual.stride(0)
    ws_ptr, ws_bytes = None, 0
    if splits > 1:
        _need(workspace is not None, "split K needs a workspace")
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    _lib.call("q38_fp8_gemm", x_e5m2.data_ptr(), tokens, k, lin.q.data_ptr(), lin.sf.data_ptr(), lin.out_features, epi,
              y.data_ptr(), y.stride(0), residual.data_ptr() if residual is not None else None, ldr, splits, ws_ptr,
              ws_bytes, _stream())
    return y


def streamk_workspace_bytes(tokens: int, features: int, k: int) -> int:
    """Workspace bytes of fp8_gemm_streamk for this shape on the current device."""
    n = _lib.load().q38_fp8_gemm_streamk_workspace_bytes(tokens, features, k)
    _need(n > 0, f"no stream-K plan for {tokens} x {features} x {k} (bad shape or no device)")
    return n


def fp8_gemm_streamk(x_e5m2: torch.Tensor, lin: DeviceLinear, y: torch.Tensor, workspace: torch.Tensor,
                     residual: torch.Tensor | None = None) -> torch.Tensor:
    """y[:, :out] = bf16(e5m2(x) @ W^T) (+ residual, in bf16), the K steps of all tiles divided evenly over
    one CTA (pair) per SM; `workspace` zero-initialised, streamk_workspace_bytes long."""
    _cuda(x_e5m2, y, residual, workspace)
    _need(x_e5m2.dtype == U8 and x_e5m2.dim() == 2 and x_e5m2.stride(1) == 1 and x_e5m2.stride(0) == x_e5m2.shape[1],
          "x must be contiguous uint8 e5m2 [tokens, k]")
    tokens, k = x_e5m2.shape
    _need(k == lin.in_features, f"x has {k} columns, the weight {lin.in_features}")
    _need(y.dtype == BF16 and y.dim() == 2 and y.stride(1) == 1 and y.shape[0] >= tokens, "y must be bf16 [tokens, >= out]")
    epi, ldr = 0, 0
    if residual is not None:
        _need(residual.dtype == BF16 and residual.stride(1) == 1, "residual must be bf16 with unit column stride")
        epi, ldr = 1, residual.stride(0)
    _lib.call("q38_fp8_gemm_streamk", x_e5m2.data_ptr(), tokens, k, lin.q.data_ptr(), lin.sf.data_ptr(),
              lin.out_features, epi, y.data_ptr(), y.stride(0), residual.data_ptr() if residual is not None else None,
              ldr, workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream())
    return y


class _DeviceArray:
    """A raw device allocation seen by torch through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class Communicator:
    """One rank's side of the fused all-reduce: its exchange region, mapped into every peer over NVLink.

    Every rank of `group` constructs it collectively (the IPC handles travel by an all-gather of the
    group). `x` is this rank's residual stream, bf16 [max_tokens, hidden], living in the region: the
    fused projections write their result into every rank's `x`."""

    def __init__(self, rank: int, world: int, max_tokens: int, hidden: int, device, group=None):
        lib = _lib.load()
        handle = ctypes.c_void_p()
        _lib.call("q38_comm_init", rank, world, max_tokens, hidden, ctypes.byref(handle))
        self.handle = handle
        self.group = group
        self.rank, self.world, self.max_tokens, self.hidden = rank, world, max_tokens, hidden
        nb = lib.q38_comm_ipc_handle_bytes()
        buf = (ctypes.c_uint8 * nb)()
        _lib.call("q38_comm_ipc_handle", handle, buf, nb)
        mine = torch.tensor(bytearray(buf), dtype=torch.uint8, device=device)
        every = torch.empty(world * nb, dtype=torch.uint8, device=device)
        torch.distributed.all_gather_into_tensor(every, mine, group=group)
        every = every.cpu().contiguous()
        _lib.call("q38_comm_connect", handle, every.data_ptr())
        ptr = lib.q38_comm_residual(handle)
        self.x = torch.as_tensor(_DeviceArray(ptr, (max_tokens, hidden), "<i2"), device=device).view(BF16)

    def close(self) -> None:
        """Collective: every rank finishes its kernels, then unmaps its peers and frees its region."""
        if self.handle is not None:
            self.x = None
            torch.cuda.synchronize()
            torch.distributed.barrier(group=self.group)
            _lib.call("q38_comm_destroy", self.handle)
            self.handle = None


def fp8_gemm_allreduce(x_e5m2: torch.Tensor, lin: DeviceLinear, comm: Communicator, splits: int = 1) -> None:
    """comm.x[:tokens] += all_reduce(bf16(e5m2(x) @ W^T)) across the communicator's ranks, fused."""
    _cuda(x_e5m2)
    _need(x_e5m2.dtype == U8 and x_e5m2.dim() == 2 and x_e5m2.is_contiguous(), "x must be contiguous uint8 e5m2")
    tokens, k = x_e5m2.shape
    _need(k == lin.in_features and lin.out_features == comm.hidden, "shape mismatch")
    _lib.call("q38_fp8_gemm_allreduce", x_e5m2.data_ptr(), tokens, k, lin.q.data_ptr(), lin.sf.data_ptr(),
              lin.out_features, splits, comm.handle, _stream())


def fp8_gemm_silu(x_e5m2: torch.Tensor, lin: DeviceLinear, y_e5m2: torch.Tensor) -> torch.Tensor:
    """y = e5m2(SiLU(gate) * up) with `lin` the gate/up weight interleaved in 64-row blocks."""
    _cuda(x_e5m2, y_e5m2)
    _need(x_e5m2.dtype == U8 and x_e5m2.is_contiguous(), "x must be contiguous uint8 e5m2 [tokens, k]")
    tokens, k = x_e5m2.shape
    _need(k == lin.in_features, f"x has {k} columns, the weight {lin.in_features}")
    _need(y_e5m2.dtype == U8 and y_e5m2.stride(1) == 1 and y_e5m2.shape[0] >= tokens, "y must be uint8 [tokens, >= out / 2]")
    _lib.call("q38_fp8_gemm_silu", x_e5m2.data_ptr(), tokens, k, lin.q.data_ptr(), lin.sf.data_ptr(), lin.out_features,
              y_e5m2.data_ptr(), y_e5m2.stride(0), _stream())
    return y_e5m2


def rmsnorm_quant(x: torch.Tensor, w: torch.Tensor, eps: float, y_bf16: torch.Tensor | None = None,
                  y_e5m2: torch.Tensor | None = None) -> None:
    _cuda(x, w, y_bf16, y_e5m2)
    rows, n = x.shape
    _need(x.dtype == BF16 and w.dtype == BF16 and w.numel() == n, "rmsnorm_quant: bf16 x [rows, n], w [n]")
    _lib.call("q38_rmsnorm_quant", x.data_ptr(), x.stride(0), w.data_ptr(), rows, n, eps,
              y_bf16.data_ptr() if y_bf16 is not None else None, y_bf16.stride(0) if y_bf16 is not None else 0,
              y_e5m2.data_ptr() if y_e5m2 is not None else None, y_e5m2.stride(0) if y_e5m2 is not None else 0,
              _stream())


def rmsnorm_divide(x: torch.Tensor, w: torch.Tensor, w_div: torch.Tensor, eps: float, y: torch.Tensor) -> None:
    """y = bf16(bf16(rms_norm(x) * (1 + w)) / (1 + w_div)) per row (the MTP layer's output)."""
    _cuda(x, w, w_div, y)
    rows, n = x.shape
    _need(x.dtype == BF16 and y.dtype == BF16 and w.numel() == n and w_div.numel() == n and x.stride(1) == 1
          and y.stride(1) == 1, "rmsnorm_divide: bf16 x, y [rows, n], w, w_div [n]")
    _lib.call("q38_rmsnorm_divide", x.data_ptr(), x.stride(0), w.data_ptr(), w_div.data_ptr(), rows, n, eps, y.data_ptr(),
              y.stride(0), _stream())


def silu_mul_quant(gu: torch.Tensor, n: int, y_e5m2: torch.Tensor) -> None:
    _cuda(gu, y_e5m2)
    rows = gu.shape[0]
    _lib.call("q38_silu_mul_quant", gu.data_ptr(), gu.stride(0), rows, n, y_e5m2.data_ptr(), y_e5m2.stride(0), _stream())


def bf16_linear(x: torch.Tensor, lin: DeviceBF16Linear, y: torch.Tensor, splits: int = 1,
                workspace: torch.Tensor | None = None) -> None:
    """y = bf16(x @ W^T), BF16 in, fp32 accumulate (tcgen05 kind::f16). Split K sums the partials
    through `workspace` when one is given (CTAs in pairs on any free SMs: the form to run beside
    another kernel), else through the shared memory of a cluster of the splits; same bits either way."""
    _cuda(x, y, workspace)
    rows, k = x.shape
    _need(x.dtype == BF16 and x.is_contiguous() and k == lin.in_features, "x must be contiguous bf16 [rows, in]")
    ws_ptr, ws_bytes = None, 0
    if splits > 1 and workspace is not None:
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    _lib.call("q38_bf16_linear", x.data_ptr(), x.stride(0), rows, k, lin.w.data_ptr(), lin.out_features, y.data_ptr(),
              y.stride(0), splits, ws_ptr, ws_bytes, _stream())


def bf16_linear_splits(rows: int, n_out: int, k: int) -> int:
    """K splits for a thin BF16 linear (96 outputs): 8 balance streaming parallelism against the
    reduction of the split partials at 5120 x 96. The partials are summed in split order, so the
    split count fixes the fp32 summation order and with it the last bit of every output."""
    kc = -(-k // 64)
    return max(1, min(kc // 4, 8))


def gdn_decode_workspace_bytes(batch: int, num_k_heads: int, head_k: int) -> int:
    return _lib.load().q38_gdn_decode_workspace_bytes(batch, num_k_heads, head_k)


def gdn_verify_workspace_bytes(batch: int, tokens: int, num_k_heads: int, head_k: int) -> int:
    return _lib.load().q38_gdn_verify_workspace_bytes(batch, tokens, num_k_heads, head_k)


_workspaces: dict = {}
_retired: list = []


def _workspace(device, nbytes: int) -> torch.Tensor:
    """A per-device scratch buffer for callers that pass none. It only grows, and a replaced buffer is
    kept alive, so a CUDA graph that captured an older one stays valid."""
    key = torch.device(device).index
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _retired.append(buf)
        buf = torch.zeros(max(nbytes, 256), dtype=U8, device=device)
        _workspaces[key] = buf
    return buf


def gdn_decode(qkvz, ab, conv_state, conv_weight, a_log, dt_bias, norm_weight, state, position, active, out, *,
               batch: int, num_k_heads: int, num_v_heads: int, head_k: int, head_v: int, eps: float,
               workspace: torch.Tensor | None = None) -> None:
    _cuda(qkvz, ab, conv_state, conv_weight, a_log, dt_bias, norm_weight, state, position, active, out, workspace)
    _need(position.dtype == torch.int32 and active.dtype == torch.float32, "position int32, active float32")
    _need(state.is_contiguous() and conv_state.is_contiguous(), "state buffers must be contiguous")
    need = _lib.load().q38_gdn_decode_workspace_bytes(batch, num_k_heads, head_k)
    ws = workspace if workspace is not None else _workspace(qkvz.device, need)
    _lib.call("q38_gdn_decode", qkvz.data_ptr(), qkvz.stride(0), ab.data_ptr(), ab.stride(0), conv_state.data_ptr(),
              conv_weight.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(), norm_weight.data_ptr(), state.data_ptr(),
              position.data_ptr(), active.data_ptr(), out.data_ptr(), out.stride(0), batch, num_k_heads, num_v_heads,
              head_k, head_v, conv_weight.shape[1], eps, ws.data_ptr(), ws.numel() * ws.element_size(), _stream())


def attn_decode(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, position, active, out, *, batch: int,
                num_q_heads: int, num_kv_heads: int, head_dim: int, rot_dim: int, eps: float,
                row_order: torch.Tensor | None = None) -> None:
    """`row_order` (int32 [batch], from attn_row_order) schedules the rows longest first; same bytes."""
    _cuda(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, position, active, out, row_order)
    _need(cos.is_contiguous() and sin.is_contiguous() and cos.shape[-1] == rot_dim, "cos/sin [batch, rot] contiguous")
    _need(k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous")
    _need(row_order is None or (row_order.dtype == torch.int32 and row_order.numel() == batch), "row_order int32 [batch]")
    _lib.call("q38_attn_decode", qkv.data_ptr(), qkv.stride(0), q_norm_w.data_ptr(), k_norm_w.data_ptr(), cos.data_ptr(),
              sin.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2], position.data_ptr(),
              active.data_ptr(), out.data_ptr(), out.stride(0), batch, num_q_heads, num_kv_heads, head_dim, rot_dim, eps,
              None if row_order is None else row_order.data_ptr(), _stream())


ATTN_ORDER_MAX_ROWS = 4096  # q38_attn_row_order's batch limit


def attn_row_order(position: torch.Tensor, active: torch.Tensor, max_seq: int, row_order: torch.Tensor) -> torch.Tensor:
    """row_order = the rows by decreasing visible cache length (ties by index), for attn_decode."""
    _cuda(position, active, row_order)
    batch = position.numel()
    _need(position.dtype == torch.int32 and active.dtype == torch.float32 and active.numel() == batch,
          "position int32 [batch], active float32 [batch]")
    _need(row_order.dtype == torch.int32 and row_order.numel() == batch and row_order.is_contiguous(),
          "row_order int32 [batch] contiguous")
    _lib.call("q38_attn_row_order", position.data_ptr(), active.data_ptr(), max_seq, batch, row_order.data_ptr(),
              _stream())
    return row_order


def gdn_prefill_workspace_bytes(tokens: int, num_k_heads: int, num_v_heads: int, head_k: int, head_v: int) -> int:
    return _lib.load().q38_gdn_prefill_workspace_bytes(tokens, num_k_heads, num_v_heads, head_k, head_v)


def gdn_prefill(qkvz, ab, conv_state, conv_weight, a_log, dt_bias, norm_weight, state, out, workspace, *, slot: int,
                start: int, n_valid: int, num_k_heads: int, num_v_heads: int, head_k: int, head_v: int,
                eps: float) -> None:
    """One row's prefill chunk through the gated delta rule (qkvz/ab rows are the chunk's tokens)."""
    _cuda(qkvz, ab, conv_state, conv_weight, a_log, dt_bias, norm_weight, state, out, workspace)
    _need(state.is_contiguous() and conv_state.is_contiguous(), "state buffers must be contiguous")
    tokens = qkvz.shape[0]
    _need(ab.shape[0] >= tokens and out.shape[0] >= tokens, "ab and out need a row per token")
    _lib.call("q38_gdn_prefill_chunk", qkvz.data_ptr(), qkvz.stride(0), ab.data_ptr(), ab.stride(0),
              conv_state.data_ptr(), conv_weight.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(),
              norm_weight.data_ptr(), state.data_ptr(), slot, state.shape[0], tokens, start, n_valid, out.data_ptr(),
              out.stride(0), num_k_heads, num_v_heads, head_k, head_v, conv_weight.shape[1], eps, workspace.data_ptr(),
              workspace.numel() * workspace.element_size(), _stream())


def attn_prefill_workspace_bytes(tokens: int, num_q_heads: int, head_dim: int) -> int:
    return _lib.load().q38_attn_prefill_workspace_bytes(tokens, num_q_heads, head_dim)


def attn_prefill(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, out, workspace, *, slot: int, start: int,
                 num_q_heads: int, num_kv_heads: int, head_dim: int, rot_dim: int, eps: float,
                 kv_scales: tuple[float, float] | None = None) -> None:
    """One row's prefill chunk through keys-first gated attention; writes the chunk's K/V to the cache.
    `kv_scales` = (k_scale, v_scale) selects the FP8 e4m3 cache (uint8 k_cache / v_cache)."""
    _cuda(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, out, workspace)
    _need(cos.is_contiguous() and sin.is_contiguous() and cos.shape[-1] == rot_dim, "cos/sin [tokens, rot] contiguous")
    _need(k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous")
    fp8 = kv_scales is not None
    _need(k_cache.dtype == (U8 if fp8 else BF16) and v_cache.dtype == k_cache.dtype,
          "caches: uint8 e4m3 with kv_scales, else bf16")
    tokens = qkv.shape[0]
    head = (qkv.data_ptr(), qkv.stride(0), q_norm_w.data_ptr(), k_norm_w.data_ptr(), cos.data_ptr(), sin.data_ptr(),
            k_cache.data_ptr(), v_cache.data_ptr())
    tail = (slot, k_cache.shape[0], k_cache.shape[2], tokens, start, out.data_ptr(), out.stride(0), num_q_heads,
            num_kv_heads, head_dim, rot_dim, eps, workspace.data_ptr(), workspace.numel() * workspace.element_size(),
            _stream())
    if fp8:
        _lib.call("q38_attn_prefill_e4m3", *head, float(kv_scales[0]), float(kv_scales[1]), *tail)
    else:
        _lib.call("q38_attn_prefill", *head, *tail)


def gdn_verify(qkvz, ab, conv_state, conv_weight, a_log, dt_bias, norm_weight, state, pending_key, pending_delta,
               pending_decay, pending_input, position, active, accepted, out, *, batch: int, tokens: int,
               num_k_heads: int, num_v_heads: int, head_k: int, head_v: int, eps: float,
               workspace: torch.Tensor | None = None) -> None:
    """K verify tokens per row with commit-on-accept (rows b * tokens + t of qkvz/ab/out)."""
    _cuda(qkvz, ab, conv_state, conv_weight, a_log, dt_bias, norm_weight, state, pending_key, pending_delta,
          pending_decay, pending_input, position, active, accepted, out, workspace)
    need = _lib.load().q38_gdn_verify_workspace_bytes(batch, tokens, num_k_heads, head_k)
    ws = workspace if workspace is not None else _workspace(qkvz.device, need)
    _need(position.dtype == torch.int32 and accepted.dtype == torch.int32 and active.dtype == torch.float32,
          "position/accepted int32, active float32")
    _need(pending_key.dtype == torch.float32 and pending_delta.dtype == torch.float32 and
          pending_decay.dtype == torch.float32 and pending_input.dtype == BF16, "pending buffers f32 (input bf16)")
    for t in (state, conv_state, pending_key, pending_delta, pending_decay, pending_input):
        _need(t.is_contiguous(), "state and pending buffers must be contiguous")
    _need(pending_key.shape[:2] == (batch, tokens), "pending buffers [batch, tokens, ...]")
    _lib.call("q38_gdn_verify_commit", qkvz.data_ptr(), qkvz.stride(0), ab.data_ptr(), ab.stride(0),
              conv_state.data_ptr(), conv_weight.data_ptr(), a_log.data_ptr(), dt_bias.data_ptr(),
              norm_weight.data_ptr(), state.data_ptr(), pending_key.data_ptr(), pending_delta.data_ptr(),
              pending_decay.data_ptr(), pending_input.data_ptr(), position.data_ptr(), active.data_ptr(),
              accepted.data_ptr(), out.data_ptr(), out.stride(0), batch, tokens, num_k_heads, num_v_heads, head_k,
              head_v, conv_weight.shape[1], eps, ws.data_ptr(), ws.numel() * ws.element_size(), _stream())


def attn_verify(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, position, active, out, *, batch: int, tokens: int,
                num_q_heads: int, num_kv_heads: int, head_dim: int, rot_dim: int, eps: float) -> None:
    """K verify tokens per row of gated attention (rows b * tokens + t); writes the tokens' K/V."""
    _cuda(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, position, active, out)
    _need(cos.is_contiguous() and sin.is_contiguous() and cos.shape[-1] == rot_dim, "cos/sin [rows, rot] contiguous")
    _need(k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous")
    _lib.call("q38_attn_verify", qkv.data_ptr(), qkv.stride(0), q_norm_w.data_ptr(), k_norm_w.data_ptr(),
              cos.data_ptr(), sin.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2],
              position.data_ptr(), active.data_ptr(), out.data_ptr(), out.stride(0), batch, tokens, num_q_heads,
              num_kv_heads, head_dim, rot_dim, eps, _stream())


def lm_head_groupmax(x: torch.Tensor, lin: DeviceBF16Linear, maxima: torch.Tensor, group: int = 32) -> None:
    _cuda(x, maxima)
    rows, k = x.shape
    _need(x.is_contiguous() and x.dtype == BF16 and k == lin.in_features, "bf16 contiguous x [rows, hidden]")
    _need(maxima.dtype == torch.float32 and maxima.stride(1) == 1, "maxima fp32")
    _lib.call("q38_lm_head_groupmax", x.data_ptr(), rows, k, lin.w.data_ptr(), lin.out_features, group,
              maxima.data_ptr(), maxima.stride(0), _stream())


KV_BF16, KV_E4M3 = 0, 1  # cache formats of attn_split


def attn_split_workspace_bytes(batch: int, num_q_heads: int, num_kv_heads: int, tokens: int, max_seq: int,
                               head_dim: int) -> int:
    return _lib.load().q38_attn_split_workspace_bytes(batch, num_q_heads, num_kv_heads, tokens, max_seq, head_dim)


def attn_split(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, position, active, out, *, batch: int, tokens: int,
               num_q_heads: int, num_kv_heads: int, head_dim: int, rot_dim: int, eps: float,
               kv_scales: tuple[float, float] | None = None, workspace: torch.Tensor | None = None) -> None:
    """Decode (tokens = 1) or verify (tokens = K) attention split along the cache, for caches of any
    length; `kv_scales` = (k_scale, v_scale) selects the FP8 e4m3 cache (uint8 k_cache / v_cache)."""
    _cuda(qkv, q_norm_w, k_norm_w, cos, sin, k_cache, v_cache, position, active, out, workspace)
    fp8 = kv_scales is not None
    _need(k_cache.dtype == (U8 if fp8 else BF16) and v_cache.dtype == k_cache.dtype,
          "caches: uint8 e4m3 with kv_scales, else bf16")
    _need(k_cache.is_contiguous() and v_cache.is_contiguous(), "caches must be contiguous")
    _need(cos.is_contiguous() and sin.is_contiguous() and cos.shape[-1] == rot_dim, "cos/sin [rows, rot] contiguous")
    _need(position.dtype == torch.int32 and active.dtype == torch.float32, "position int32, active float32")
    max_seq = k_cache.shape[2]
    need = attn_split_workspace_bytes(batch, num_q_heads, num_kv_heads, tokens, max_seq, head_dim)
    ws = workspace if workspace is not None else _workspace(qkv.device, need)
    ks, vs = kv_scales if fp8 else (1.0, 1.0)
    _lib.call("q38_attn_split", qkv.data_ptr(), qkv.stride(0), q_norm_w.data_ptr(), k_norm_w.data_ptr(), cos.data_ptr(),
              sin.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), KV_E4M3 if fp8 else KV_BF16, float(ks), float(vs),
              max_seq, position.data_ptr(), active.data_ptr(), out.data_ptr(), out.stride(0), batch, tokens,
              num_q_heads, num_kv_heads, head_dim, rot_dim, eps, ws.data_ptr(), ws.numel() * ws.element_size(),
              _stream())


class StateRows:
    """A fixed list of state buffers whose rows `copy` moves together (q38_copy_state_rows), e.g. every
    gated-delta layer's recurrent and conv state: rows of the same index across all of them."""

    def __init__(self, buffers: list[torch.Tensor]):
        _cuda(*buffers)
        for t in buffers:
            _need(t.is_contiguous() and t.dim() >= 1, "state buffers must be contiguous with rows along dim 0")
        self.buffers = list(buffers)  # keeps the storage alive
        n = len(buffers)
        self._ptrs = (ctypes.c_void_p * n)(*[t.data_ptr() for t in buffers])
        self._row_bytes = (ctypes.c_int64 * n)(*[t[0].numel() * t.element_size() if t.shape[0] else 0 for t in buffers])
        self._rows = (ctypes.c_int64 * n)(*[t.shape[0] for t in buffers])

    def copy(self, src_row: int, dst_row: int) -> None:
        _lib.call("q38_copy_state_rows", self._ptrs, self._row_bytes, self._rows, len(self.buffers), src_row, dst_row,
                  _stream())


def lm_head_recheck(hidden: torch.Tensor, norm_w: torch.Tensor, eps: float, maxima: torch.Tensor, lin: DeviceBF16Linear,
                    vocab_first: int, candidates: int, tokens: torch.Tensor | None = None,
                    slot_logits: torch.Tensor | None = None, slot_tokens: torch.Tensor | None = None) -> None:
    """ChipHead.next_tokens' exact recheck on the device: tokens int32 [rows], and/or per-candidate slots."""
    _cuda(hidden, norm_w, maxima, tokens, slot_logits, slot_tokens)
    rows, h = hidden.shape
    _need(hidden.dtype == BF16 and hidden.stride(1) == 1 and h == lin.in_features, "hidden bf16 [rows, hidden]")
    _need(maxima.dtype == torch.float32 and maxima.stride(1) == 1 and maxima.shape[0] >= rows, "maxima fp32 [rows, groups]")
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.call("q38_lm_head_recheck", hidden.data_ptr(), hidden.stride(0), norm_w.data_ptr(), eps, maxima.data_ptr(),
              maxima.stride(0), maxima.shape[1], lin.w.data_ptr(), vocab_first, lin.out_features, h, 32, candidates, rows,
              ptr(slot_logits), ptr(slot_tokens), ptr(tokens), _stream())


def embed_rows(table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[i] = table[ids[i]] (bf16 rows; ids int32 on the device)."""
    _cuda(table, ids, out)
    _need(table.dtype == BF16 and table.is_contiguous() and out.dtype == BF16 and out.stride(-1) == 1, "bf16 table and out")
    _need(ids.dtype == torch.int32 and ids.is_contiguous(), "ids int32")
    n = ids.numel()
    _lib.call("q38_embed_rows", table.data_ptr(), table.shape[0], table.shape[1], ids.data_ptr(), n, out.data_ptr(),
              out.stride(-2) if out.dim() > 1 else table.shape[1], _stream())
    return out


def lm_head_pick(slot_logits: torch.Tensor, slot_tokens: torch.Tensor, tokens: torch.Tensor) -> None:
    _cuda(slot_logits, slot_tokens, tokens)
    rows, candidates = slot_logits.shape
    _lib.call("q38_lm_head_pick", slot_logits.data_ptr(), slot_tokens.data_ptr(), candidates, rows, tokens.data_ptr(),
              _stream())


def device_status(reset: bool = True) -> int:
    return _lib.load().q38_device_status(1 if reset else 0)
