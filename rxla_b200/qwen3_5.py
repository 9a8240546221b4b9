"""Host-side mirror of Qwen3.5's full-attention layer and of the hybrid model.

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

`Qwen3_5Model` composes the whole text model (`qwen3_5`, mod.rs:199-260):
W8 embedding, zero-centred RMSNorms, gated-delta and full-attention mixers,
SwiGLU MLP, tied W8 head.

The decode attention takes head_dim 64, 128 or 256 (Qwen3.5-0.8B's), with
rotary_dim <= 128 at 256.
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
        if D not in (64, 128, 256):
            raise InvalidLayerInput("the decode attention takes head_dim 64, 128 or 256")
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

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None,
                stream=None) -> torch.Tensor:
        """T tokens per sequence, x [batch, T, hidden] (F32 or bf16, the
        normalised layer input, contiguous) from each sequence's current
        position: the rows of the reference's causal full-sequence forward
        (layers.rs:28-100 with the causal mask of qwen3_5/mod.rs:229).  The
        projections run once over all batch * T rows; the attention runs
        token by token, each call appending its token's K/V and attending
        over the positions before it.  Without `residual` returns F32
        [batch, T, hidden]; with it (F32 [batch, T, hidden], contiguous) adds
        bf16(o_proj) into it in place and returns it."""
        B = self.cache.batch
        if x.dim() != 3 or x.shape[0] != B or x.shape[2] != self.hidden or not x.is_contiguous():
            raise InvalidLayerInput("input must be contiguous [batch, sequence, hidden]")
        T = x.shape[1]
        if residual is not None and (residual.dtype != torch.float32 or
                                     tuple(residual.shape) != (B, T, self.hidden) or
                                     not residual.is_contiguous()):
            raise InvalidLayerInput("residual must be contiguous F32 [batch, sequence, hidden]")
        Hq, Hkv, D = self.Hq, self.Hkv, self.D
        qd, kd = Hq * D, Hkv * D
        proj = quantized_linear(x.view(B * T, self.hidden), self.w_in, self.s_in, self.G,
                                out_dtype=torch.bfloat16, stream=stream)
        pv = proj.view(B, T, -1)
        att = torch.empty(T, B, qd, dtype=torch.bfloat16, device=x.device)
        for t in range(T):
            paged_decode_attention(pv[:, t, :qd], pv[:, t, 2 * qd:2 * qd + kd],
                                   pv[:, t, 2 * qd + kd:], self.cache, q_heads=Hq,
                                   q_norm_weight=self.q_norm, k_norm_weight=self.k_norm,
                                   eps=self.eps, inv_freq=self.inv_freq, rotary_dim=self.rot,
                                   advance_ctx=True, out=att[t], workspace=self.workspace,
                                   stream=stream)
        if B == 1 or T == 1:  # token-major rows are batch-major rows
            y = sigmoid_gate(att.view(T * B, qd), proj[:, qd:2 * qd], out=att.view(T * B, qd),
                             stream=stream)
        else:
            y = torch.empty(B, T, qd, dtype=torch.bfloat16, device=x.device)
            for t in range(T):
                sigmoid_gate(att[t], pv[:, t, qd:2 * qd], out=y[:, t], stream=stream)
            y = y.view(B * T, qd)
        if residual is not None:
            quantized_linear(y, self.w_out, self.s_out, self.G, epilogue=_lib.EPI_RESIDUAL_ADD,
                             out=residual.view(B * T, self.hidden), stream=stream)
            return residual
        return quantized_linear(y, self.w_out, self.s_out, self.G, out_dtype=torch.bfloat16,
                                stream=stream).float().view(B, T, self.hidden)


class Qwen3_5Model:
    """The hybrid Qwen3.5 text model, `qwen3_5(cx, token_ids, config)`
    (crates/rxla-models/src/qwen3_5/mod.rs:199-260), with W8 storage, for a
    batch of sequences whose state — every linear-attention layer's conv
    history and recurrent state, every full-attention layer's paged KV cache —
    is carried from call to call, where the reference recomputes the whole
    sequence.

    params: device tensors by the checkpoint names below "model.language_model."
    (`embed_tokens.weight` u8 [V, H] and `.scale`, `layers.{i}.input_layernorm.weight`,
    `layers.{i}.post_attention_layernorm.weight`, `layers.{i}.linear_attn.*` or
    `layers.{i}.self_attn.*`, `layers.{i}.mlp.{gate,up,down}_proj.{weight,scale}`,
    `norm.weight`).  Every RMSNorm is zero-centred (weight + 1).  `layer_types`:
    "linear" or "full" per layer (mod.rs:8-12).  The tied LM head is the W8
    linear over the embedding with bf16 x and an f32 dot (the reference's is an
    F32 linear over the dequantized embedding)."""

    def __init__(self, params, *, vocabulary: int, hidden_size: int, intermediate_size: int,
                 layer_types, attention_heads: int, key_value_heads: int, head_dim: int,
                 linear_heads: int, linear_head_dim: int, conv_kernel: int, rope_theta: float,
                 rotary_dim: int, epsilon: float, quant_group_size: int, batch: int = 1,
                 max_context: int = 256):
        from .gated_delta import GatedDeltaAttention
        G = quant_group_size
        self.V, self.H, self.G, self.eps, self.B = vocabulary, hidden_size, G, epsilon, batch
        self.types = list(layer_types)
        self.embed_w = params["embed_tokens.weight"]
        self.embed_s = params["embed_tokens.scale"]
        if tuple(self.embed_w.shape) != (vocabulary, hidden_size) or self.embed_w.dtype != torch.uint8:
            raise InvalidLayerInput("embed_tokens.weight must be U8 [vocabulary, hidden]")
        zc = lambda name: (params[name].float() + 1.0).contiguous()  # zero-centred norm weight
        self.norm_in, self.norm_post, self.mixers, self.states = [], [], [], []
        self.mlp_gu, self.mlp_gu_s, self.mlp_d, self.mlp_d_s = [], [], [], []
        for i, kind in enumerate(self.types):
            pre = f"layers.{i}."
            self.norm_in.append(zc(pre + "input_layernorm.weight"))
            self.norm_post.append(zc(pre + "post_attention_layernorm.weight"))
            if kind == "linear":
                sub = {k[len(pre + "linear_attn."):]: v for k, v in params.items()
                       if k.startswith(pre + "linear_attn.")}
                m = GatedDeltaAttention(sub, hidden_size=hidden_size, linear_heads=linear_heads,
                                        linear_head_dim=linear_head_dim, conv_kernel=conv_kernel,
                                        quant_group_size=G, epsilon=epsilon)
                self.mixers.append(m)
                self.states.append(m.new_state(batch))
            elif kind == "full":
                sub = {k[len(pre + "self_attn."):]: v for k, v in params.items()
                       if k.startswith(pre + "self_attn.")}
                self.mixers.append(GatedFullAttention(
                    sub, hidden_size=hidden_size, attention_heads=attention_heads,
                    key_value_heads=key_value_heads, head_dim=head_dim, rotary_dim=rotary_dim,
                    rope_theta=rope_theta, quant_group_size=G, epsilon=epsilon, batch=batch,
                    max_context=max_context))
                self.states.append(None)
            else:
                raise InvalidLayerInput(f"layer type {kind!r}")
            # SwiGLU MLP (layers.rs:270-293): [gate; up] rows for the fused epilogue
            self.mlp_gu.append(torch.cat([params[pre + "mlp.gate_proj.weight"],
                                          params[pre + "mlp.up_proj.weight"]]).contiguous())
            self.mlp_gu_s.append(torch.cat([params[pre + "mlp.gate_proj.scale"],
                                            params[pre + "mlp.up_proj.scale"]]).contiguous())
            self.mlp_d.append(params[pre + "mlp.down_proj.weight"].contiguous())
            self.mlp_d_s.append(params[pre + "mlp.down_proj.scale"].contiguous())
        self.norm_final = zc("norm.weight")

    def forward(self, ids: torch.Tensor, stream=None) -> torch.Tensor:
        """ids int32 [batch, T] on the device: the next T tokens of every
        sequence.  Returns the last position's logits f32 [batch, vocabulary]."""
        from .nn import rms_norm_bf16, w8_embedding
        if ids.dim() != 2 or ids.shape[0] != self.B or ids.dtype != torch.int32:
            raise InvalidLayerInput("ids must be int32 [batch, T]")
        B, T = ids.shape
        h = w8_embedding(ids, self.embed_w, self.embed_s, self.G, stream=stream)  # [B, T, H] f32
        for i, kind in enumerate(self.types):
            xn = rms_norm_bf16(h, self.norm_in[i], self.eps, stream=stream)
            if kind == "linear":
                self.mixers[i].apply(xn, self.states[i], residual=h, stream=stream)
            else:
                self.mixers[i].forward(xn, residual=h, stream=stream)
            xn = rms_norm_bf16(h, self.norm_post[i], self.eps, stream=stream)
            u = quantized_linear(xn.reshape(B * T, self.H), self.mlp_gu[i], self.mlp_gu_s[i],
                                 self.G, epilogue=_lib.EPI_SWIGLU, out_dtype=torch.bfloat16,
                                 stream=stream)
            quantized_linear(u, self.mlp_d[i], self.mlp_d_s[i], self.G,
                             epilogue=_lib.EPI_RESIDUAL_ADD, out=h.view(B * T, self.H),
                             stream=stream)
        hn = rms_norm_bf16(h[:, -1].contiguous(), self.norm_final, self.eps, stream=stream)
        return quantized_linear(hn, self.embed_w, self.embed_s, self.G, out_dtype=torch.float32,
                                stream=stream)


__all__ = ["GatedFullAttention", "Qwen3_5Model"]
