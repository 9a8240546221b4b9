"""Host-side mirror of Qwen3.5's gated-delta linear-attention mixer.

`GatedDeltaAttention` follows `gated_delta_attention(cx, input, config)`
(crates/rxla-models/src/qwen3_5/layers.rs:114-268, paths inside the rxla
project): parameter names, shapes and errors as the reference's scope
declares them; the arithmetic runs in librxla_b200 (the W8 linears and
rxla_b200_gated_delta) on the tensors' CUDA device.

Where the reference recomputes the whole sequence from a zero state on every
call, a `GatedDeltaState` here carries the conv history and the recurrent
state of each sequence, so a prompt is processed once and decode steps
continue from it; `apply` without a state is the reference's full-sequence
forward.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .nn import InvalidLayerInput, _ptr, _stream, quantized_linear


class GatedDeltaState:
    """Per-sequence state of one gated-delta layer: the last conv_kernel - 1
    mixed rows (bf16 [batch, K-1, 3W]) and the recurrent state f32
    [batch, heads, D, D] (column j of the reference's [Dk, Dv] state at
    [b, h, j, :])."""

    def __init__(self, batch: int, heads: int, head_dim: int, conv_kernel: int, device="cuda"):
        self.batch, self.heads, self.head_dim, self.conv_kernel = batch, heads, head_dim, conv_kernel
        w3 = 3 * heads * head_dim
        self.conv_state = torch.zeros(batch, max(conv_kernel - 1, 1), w3, dtype=torch.bfloat16,
                                      device=device)
        self.state = torch.zeros(batch, heads, head_dim, head_dim, dtype=torch.float32,
                                 device=device)
        self.started = False  # False: the next call starts every sequence from zero

    def reset(self):
        self.started = False


def workspace_size(batch: int, tokens: int, heads: int, head_dim: int) -> int:
    n = ctypes.c_size_t()
    _lib.call("rxla_b200_gated_delta_workspace_size", int(batch), int(tokens), int(heads),
              int(head_dim), ctypes.byref(n))
    return int(n.value)


def gated_delta(mixed, z, b, a, conv_weight, a_log, dt_bias, norm_weight, *,
                state: GatedDeltaState, eps: float = 1e-6, out=None, workspace=None,
                stream=None) -> torch.Tensor:
    """rxla_b200_gated_delta for `rows = batch * tokens` token rows.

    mixed [rows, 3W], z [rows, W], b / a [rows, H]: bf16 2-D views with a unit
    inner stride (e.g. column slices of one fused projection).  Continues
    `state` (or starts it, when state.started is False) and returns the bf16
    out_proj input [rows, W]."""
    H, D, K, B = state.heads, state.head_dim, state.conv_kernel, state.batch
    W = H * D
    rows = mixed.shape[0]
    for t, width, name in ((mixed, 3 * W, "mixed"), (z, W, "z"), (b, H, "b"), (a, H, "a")):
        if t.dtype != torch.bfloat16 or t.dim() != 2 or t.shape != (rows, width) or t.stride(1) != 1:
            raise InvalidLayerInput(f"{name} must be a bf16 [rows, {width}] view with unit inner stride")
    if rows % B:
        raise InvalidLayerInput("rows must be batch * tokens")
    tokens = rows // B
    if tuple(conv_weight.shape[-1:]) != (K,) or conv_weight.numel() != 3 * W * K:
        raise InvalidLayerInput(f"conv1d.weight must be [{3 * W}, 1, {K}]")
    if out is None:
        out = torch.empty(rows, W, dtype=torch.bfloat16, device=mixed.device)
    if workspace is None:
        workspace = torch.empty(workspace_size(B, tokens, H, D), dtype=torch.uint8,
                                device=mixed.device)
    g = _lib.GatedDeltaArgs()
    g.struct_size = ctypes.sizeof(_lib.GatedDeltaArgs)
    g.batch, g.tokens, g.heads, g.head_dim, g.conv_kernel = B, tokens, H, D, K
    g.mixed, g.z, g.beta_logits, g.a = (mixed.data_ptr(), z.data_ptr(), b.data_ptr(),
                                        a.data_ptr())
    g.mixed_row_stride, g.z_row_stride = mixed.stride(0), z.stride(0)
    g.b_row_stride, g.a_row_stride = b.stride(0), a.stride(0)
    g.conv_weight, g.a_log = conv_weight.data_ptr(), a_log.data_ptr()
    g.dt_bias, g.norm_weight = dt_bias.data_ptr(), norm_weight.data_ptr()
    g.eps = eps
    g.has_state = int(state.started)
    g.conv_state, g.state = state.conv_state.data_ptr(), state.state.data_ptr()
    g.out = out.data_ptr()
    g.workspace, g.workspace_bytes = workspace.data_ptr(), workspace.numel()
    _lib.call("rxla_b200_gated_delta", ctypes.byref(g), _stream(stream))
    state.started = True
    return out


class GatedDeltaAttention:
    """qwen3_5 `gated_delta_attention` with W8 projections.

    params: the mixer scope's tensors on one CUDA device, by the reference's
    names — in_proj_qkv / in_proj_z / in_proj_b / in_proj_a / out_proj
    `.weight` (u8 [out, in], value + 128) and `.scale` (f32 [out, in / group]),
    `conv1d.weight` f32 [3W, 1, K], `A_log` and `dt_bias` f32 [H],
    `norm.weight` f32 [D].  The four input projections are fused into one
    weight at construction, so one W8 linear produces mixed | z | b | a.
    """

    NAMES = ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj")

    def __init__(self, params, *, hidden_size: int, linear_heads: int, linear_head_dim: int,
                 conv_kernel: int = 4, quant_group_size: int, epsilon: float = 1e-6):
        H, D, K, G = linear_heads, linear_head_dim, conv_kernel, quant_group_size
        W = H * D
        if min(hidden_size, H, D, K, G) <= 0 or hidden_size % G or W % G:
            raise InvalidLayerInput("positive widths and a group size dividing the input widths")
        want = {"in_proj_qkv": (3 * W, hidden_size), "in_proj_z": (W, hidden_size),
                "in_proj_b": (H, hidden_size), "in_proj_a": (H, hidden_size),
                "out_proj": (hidden_size, W)}
        for name, shape in want.items():
            w, s = params[f"{name}.weight"], params[f"{name}.scale"]
            if tuple(w.shape) != shape or w.dtype != torch.uint8:
                raise InvalidLayerInput(f"{name}.weight must be U8 {list(shape)}")
            if s.dtype != torch.float32 or s.numel() != shape[0] * (shape[1] // G):
                raise InvalidLayerInput(f"{name}.scale must be F32 [{shape[0]}, {shape[1] // G}]")
        cw = params["conv1d.weight"]
        if cw.dtype != torch.float32 or cw.numel() != 3 * W * K:
            raise InvalidLayerInput(f"conv1d.weight must be F32 [{3 * W}, 1, {K}]")
        for name, n in (("A_log", H), ("dt_bias", H), ("norm.weight", D)):
            if params[name].dtype != torch.float32 or params[name].numel() != n:
                raise InvalidLayerInput(f"{name} must be F32 [{n}]")
        self.hidden, self.H, self.D, self.K, self.G, self.eps = hidden_size, H, D, K, G, epsilon
        ins = self.NAMES[:4]
        self.w_in = torch.cat([params[f"{n}.weight"] for n in ins]).contiguous()
        self.s_in = torch.cat([params[f"{n}.scale"].reshape(-1, hidden_size // G)
                               for n in ins]).contiguous()
        self.w_out = params["out_proj.weight"].contiguous()
        self.s_out = params["out_proj.scale"].contiguous()
        self.conv_w = cw.reshape(3 * W, K).contiguous()
        self.a_log = params["A_log"].contiguous()
        self.dt_bias = params["dt_bias"].contiguous()
        self.norm_w = params["norm.weight"].contiguous()

    def new_state(self, batch: int) -> GatedDeltaState:
        return GatedDeltaState(batch, self.H, self.D, self.K, device=self.w_in.device)

    def apply(self, input: torch.Tensor, state: GatedDeltaState | None = None,
              residual: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """input [batch, tokens, hidden] (F32 or bf16, the normalised layer
        input).  Without `residual`: returns the mixer output F32 [batch,
        tokens, hidden] (the bf16 out_proj dot widened).  With `residual` (F32
        [batch, tokens, hidden]): adds bf16(out_proj) into it in place and
        returns it (`hidden.add(mixed)` of qwen3_5/mod.rs:246).  `state`
        continues each sequence (None: a zero state, the reference's
        full-sequence forward)."""
        if input.dim() != 3 or input.shape[-1] != self.hidden:
            raise InvalidLayerInput("input must be [batch, sequence, hidden]")
        B, T, _ = input.shape
        if state is None:
            state = self.new_state(B)
        elif state.batch != B:
            raise InvalidLayerInput("state batch differs from the input's")
        H, D, W = self.H, self.D, self.H * self.D
        proj = quantized_linear(input.reshape(B * T, self.hidden), self.w_in, self.s_in, self.G,
                                out_dtype=torch.bfloat16, stream=stream)
        y = gated_delta(proj[:, :3 * W], proj[:, 3 * W:4 * W], proj[:, 4 * W:4 * W + H],
                        proj[:, 4 * W + H:4 * W + 2 * H], self.conv_w, self.a_log, self.dt_bias,
                        self.norm_w, state=state, eps=self.eps, stream=stream)
        if residual is not None:
            if residual.dtype != torch.float32 or tuple(residual.shape) != (B, T, self.hidden):
                raise InvalidLayerInput("residual must be F32 [batch, sequence, hidden]")
            quantized_linear(y, self.w_out, self.s_out, self.G, epilogue=_lib.EPI_RESIDUAL_ADD,
                             out=residual.view(B * T, self.hidden), stream=stream)
            return residual
        out = quantized_linear(y, self.w_out, self.s_out, self.G, out_dtype=torch.bfloat16,
                               stream=stream)
        return out.float().reshape(B, T, self.hidden)


__all__ = ["GatedDeltaAttention", "GatedDeltaState", "gated_delta", "workspace_size"]
