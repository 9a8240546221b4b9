"""Host-side mirror of Qwen3.5's full-attention layer.

`GatedFullAttention` follows `full_attention(cx, input, angles, mask, config)`
(crates/rxla-models/src/qwen3_5/layers.rs:28-100, paths inside the rxla
project) in its decode form over a paged KV cache: a q_proj whose rows hold,
per head, the query and a sigmoid output gate; zero-centred q / k RMSNorm
(weight + 1, crates/rxla-nn/src/layers.rs:470-491); partial SplitHalf RoPE
over the first `rotary_dim` dimensions (layers.rs:11-26); grouped-query
attention over the cached keys; the gated output through o_proj.  The
arithmetic runs in librxla_b200: one W8 linear for the fused q | gate | k | v
projection, rxla_b200_paged_decode_attention (norms, RoPE, append, GQA),
rxla_b200_sigmoid_gate, and the o_proj W8 linear with the residual add.

The attention kernels take head_dim 64 or 128; Qwen3.5-0.8B's 256 is not
supported.
"""
from __future__ import annotations

import torch

from . import _lib
from .nn import (InvalidLayerInput, PagedKvCache, paged_decode_attention,
                 paged_decode_workspace_size, quantized_linear, rope_inv_freq, sigmoid_gate)


class GatedFullAttention:
    """params: the layer's `self_attn` scope on one CUDA device, by the
    reference's names — q_proj (u8 [2·Hq·D, hidden], per head query rows then
    gate rows), k_proj / v_proj (u8 [Hkv·D, hidden]), o_proj (u8 [hidden,
    Hq·D]) `.weight` with f32 `.scale` [rows, in / group], and the
    zero-centred `q_norm.weight` / `k_norm.weight` f32 [D].  At construction
    the q_proj rows are reordered (all query rows, then all gate rows) and
    fused with k_proj and v_proj, so one W8 linear gives q | gate | k | v."""

    def __init__(self, params, *, hidden_size: int, attention_heads: int, key_value_heads: int,
                 head_dim: int, rotary_dim: int, rope_theta: float, quant_group_size: int,
                 epsilon: float = 1e-6, batch: int = 1, max_context: int = 256):
        Hq, Hkv, D, G = attention_heads, key_value_heads, head_dim, quant_group_size
        if D not in (64, 128):
            raise InvalidLayerInput("the attention kernels take head_dim 64 or 128")
        if Hq % Hkv or rotary_dim <= 0 or rotary_dim > D or rotary_dim % 2 or \
                hidden_size % G or (Hq * D) % G:
            raise InvalidLayerInput("invalid Qwen3.5 attention configuration")
        want = {"q_proj": (2 * Hq * D, hidden_size), "k_proj": (Hkv * D, hidden_size),
                "v_proj": (Hkv * D, hidden_size), "o_proj": (hidden_size, Hq * D)}
        for name, shape in want.items():
            w, sc = params[f"{name}.weight"], params[f"{name}.scale"]
            if tuple(w.shape) != shape or w.dtype != torch.uint8:
                raise InvalidLayerInput(f"{name}.weight must be U8 {list(shape)}")
            if sc.dtype != torch.float32 or sc.numel() != shape[0] * (shape[1] // G):
                raise InvalidLayerInput(f"{name}.scale must be F32 [{shape[0]}, {shape[1] // G}]")
        dev = params["q_proj.weight"].device
        rows = torch.arange(2 * Hq * D, device=dev).reshape(Hq, 2, D)
        order = torch.cat([rows[:, 0].reshape(-1), rows[:, 1].reshape(-1)])  # queries, then gates
        wq = params["q_proj.weight"].index_select(0, order)
        sq = params["q_proj.scale"].reshape(2 * Hq * D, -1).index_select(0, order)
        self.w_in = torch.cat([wq, params["k_proj.weight"], params["v_proj.weight"]]).contiguous()
        self.s_in = torch.cat([sq, params["k_proj.scale"].reshape(Hkv * D, -1),
                               params["v_proj.scale"].reshape(Hkv * D, -1)]).contiguous()
        self.w_out = params["o_proj.weight"].contiguous()
        self.s_out = params["o_proj.scale"].contiguous()
        # zero-centred RMSNorm: the stored weight plus one, in f32
        self.q_norm = (params["q_norm.weight"].float() + 1.0).contiguous()
        self.k_norm = (params["k_norm.weight"].float() + 1.0).contiguous()
        self.inv_freq = torch.from_numpy(rope_inv_freq(rope_theta, rotary_dim)).to(dev)
        self.hidden, self.Hq, self.Hkv, self.D, self.G = hidden_size, Hq, Hkv, D, G
        self.rot, self.eps = rotary_dim, epsilon
        self.cache = PagedKvCache(batch=batch, kv_heads=Hkv, head_dim=D, max_context=max_context,
                                  device=dev)
        self.workspace = torch.zeros(paged_decode_workspace_size(batch, Hq, Hkv, D, max_context),
                                     dtype=torch.uint8, device=dev)

    def step(self, x: torch.Tensor, residual: torch.Tensor | None = None, stream=None):
        """One token per sequence: x [batch, hidden] (F32 or bf16, the
        normalised layer input) at each sequence's next position.  Without
        `residual` returns the layer output F32 [batch, hidden] (the bf16
        o_proj dot widened); with it (F32 [batch, hidden]) adds bf16(o_proj)
        into it in place and returns it."""
        B = self.cache.batch
        if x.dim() != 2 or tuple(x.shape) != (B, self.hidden):
            raise InvalidLayerInput("input must be [batch, hidden]")
        Hq, Hkv, D = self.Hq, self.Hkv, self.D
        qd, kd = Hq * D, Hkv * D
        proj = quantized_linear(x, self.w_in, self.s_in, self.G, out_dtype=torch.bfloat16,
                                stream=stream)
        att = paged_decode_attention(proj[:, :qd], proj[:, 2 * qd:2 * qd + kd],
                                     proj[:, 2 * qd + kd:], self.cache, q_heads=Hq,
                                     q_norm_weight=self.q_norm, k_norm_weight=self.k_norm,
                                     eps=self.eps, inv_freq=self.inv_freq, rotary_dim=self.rot,
                                     advance_ctx=True, workspace=self.workspace, stream=stream)
        y = sigmoid_gate(att, proj[:, qd:2 * qd], out=att, stream=stream)
        if residual is not None:
            if residual.dtype != torch.float32 or tuple(residual.shape) != (B, self.hidden):
                raise InvalidLayerInput("residual must be F32 [batch, hidden]")
            quantized_linear(y, self.w_out, self.s_out, self.G, epilogue=_lib.EPI_RESIDUAL_ADD,
                             out=residual, stream=stream)
            return residual
        return quantized_linear(y, self.w_out, self.s_out, self.G, out_dtype=torch.bfloat16,
                                stream=stream).float()

    def forward(self, x: torch.Tensor, stream=None) -> torch.Tensor:
        """A prompt [batch, T, hidden] token by token from each sequence's
        current position: the rows of the reference's causal full-sequence
        forward (layers.rs:28-100 with the causal mask of qwen3_5/mod.rs:229).
        Returns F32 [batch, T, hidden]."""
        if x.dim() != 3:
            raise InvalidLayerInput("input must be [batch, sequence, hidden]")
        return torch.stack([self.step(x[:, t].contiguous(), stream=stream)
                            for t in range(x.shape[1])], dim=1)


__all__ = ["GatedFullAttention"]
