"""CPU oracle of Qwen3.5's full-attention layer — TEST INFRASTRUCTURE ONLY.

A restatement of `full_attention` (crates/rxla-models/src/qwen3_5/layers.rs:
28-100, paths inside the rxla project) over a whole sequence with the causal
mask (qwen3_5/mod.rs:229), built from the C oracle's pieces: the bf16-compute
W8 linear (mode 1), the per-row RMSNorm, SplitHalf RoPE over the first
rotary_dim dimensions, grouped-query attention with an f64 softmax.  As the
decode oracle does, k and v are rounded to bf16 where the paged cache stores
them.  Only `tests/` uses it, as the checker.
"""
from __future__ import annotations

import numpy as np

from . import bf16_round, causal_mask, gqa_attention, rms_norm, rope_inv_freq, rope_split_half, \
    w8_linear


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))


def full_attention(x, params, *, attention_heads, key_value_heads, head_dim, rotary_dim,
                   rope_theta, group_size, eps=1e-6, positions=None, round_attention=False,
                   linear_mode=1, round_keys=True):
    """x [B, T, hidden] F32 (the normalised layer input).  params: q_proj /
    k_proj / v_proj / o_proj `.weight` u8 and `.scale` f32, q_norm.weight and
    k_norm.weight f32 [D] (zero-centred: the norm multiplies by weight + 1).
    Returns the layer output [B, T, hidden] F32 (the bf16 o_proj dot widened).
    round_attention=True rounds the attended values to bf16 before the gate,
    as the paged attention kernel's bf16 output does (the reference keeps
    them F32): the model of that one extra rounding point, used to measure
    its effect.  linear_mode: the C oracle's W8 linear mode (1: the
    reference's rounding points with f64 sums; 4: the same with f32 running
    sums, the accumulation-noise model; 0: F32 compute).  round_keys=False
    keeps the rotated keys F32 instead of rounding them to bf16 as the paged
    cache stores them (the F32 form used to pin the layer's structure)."""
    B, T, hid = x.shape
    Hq, Hkv, D = attention_heads, key_value_heads, head_dim

    def proj(name, inp):
        return w8_linear(inp.reshape(B * T, -1), params[f"{name}.weight"], params[f"{name}.scale"],
                         group_size, mode=linear_mode).reshape(B, T, -1)

    q = proj("q_proj", x).reshape(B, T, Hq, 2 * D)
    query = np.ascontiguousarray(q[..., :D])
    gate = _sigmoid(q[..., D:].reshape(B, T, Hq * D))           # layers.rs:50-55
    key = proj("k_proj", x).reshape(B, T, Hkv, D)
    value = proj("v_proj", x).reshape(B, T, Hkv, D)
    qw = (np.asarray(params["q_norm.weight"], np.float32) + np.float32(1.0)).astype(np.float32)
    kw = (np.asarray(params["k_norm.weight"], np.float32) + np.float32(1.0)).astype(np.float32)
    query = rms_norm(query, qw, eps)                             # layers.rs:56-66
    key = rms_norm(key, kw, eps)                                 # layers.rs:67-77
    pos = np.arange(T, dtype=np.int32) if positions is None else np.asarray(positions, np.int32)
    inv = rope_inv_freq(rope_theta, rotary_dim)
    pos_rows = np.broadcast_to(pos[None, :, None], (B, T, Hq)).reshape(-1)
    query = rope_split_half(query.reshape(-1, D), pos_rows, inv, rotary_dim).reshape(B, T, Hq, D)
    pos_rows = np.broadcast_to(pos[None, :, None], (B, T, Hkv)).reshape(-1)
    key = rope_split_half(key.reshape(-1, D), pos_rows, inv, rotary_dim).reshape(B, T, Hkv, D)
    if round_keys:
        key = bf16_round(key)  # the cache's storage
    mask = causal_mask(pos, pos)[None, None]
    att = gqa_attention(query.transpose(0, 2, 1, 3), key.transpose(0, 2, 1, 3),
                        value.transpose(0, 2, 1, 3), mask)       # [B, Hq, T, D]
    att = att.transpose(0, 2, 1, 3).reshape(B, T, Hq * D)
    if round_attention:
        att = bf16_round(att)
    att = att.astype(np.float64)
    y = (att * gate).astype(np.float32)                          # layers.rs:94-95
    return proj("o_proj", y)


def qwen3_5_forward(ids, params, *, layer_types, vocabulary, hidden_size, attention_heads,
                    key_value_heads, head_dim, linear_heads, linear_head_dim, rope_theta,
                    rotary_dim, epsilon, quant_group_size, gpu_rounding=False,
                    f32_compute=False):
    """`qwen3_5(cx, token_ids, config)` (crates/rxla-models/src/qwen3_5/mod.rs:
    199-260) on the CPU: ids [B, T]; returns logits [B, T, vocabulary].
    params by the names below "model.language_model." (numpy arrays).

    gpu_rounding=True models what the GPU path computes differently — f32
    running sums in every W8 linear (the decoder tests' noise-floor model),
    bf16 attended values before the output gate, and the tied head on bf16 x
    and bf16 dequantized weights with an f32 sum (the reference's head is an
    F32 linear, mod.rs:157-173) — so that their effect can be measured.
    f32_compute=True runs every linear in F32 and keeps keys F32 (no bf16
    rounding point anywhere): the form that pins the composition against an
    F32 implementation of the same model."""
    from . import gated_delta as gdo
    mode = 0 if f32_compute else (4 if gpu_rounding else 1)
    lin_mode = lambda x, w, s, g: w8_linear(x, w, s, g, mode=mode)
    ids = np.asarray(ids)
    B, T = ids.shape
    G = quant_group_size
    emb_w = np.asarray(params["embed_tokens.weight"])
    emb_s = np.asarray(params["embed_tokens.scale"]).reshape(vocabulary, -1)
    col = np.arange(hidden_size) // G
    # quantized_embedding (mod.rs:134-155): take, cast, -128, × group scale (f32)
    h = ((emb_w[ids].astype(np.float32) - np.float32(128.0)) *
         emb_s[ids][..., col]).astype(np.float32)
    zc = lambda name: (np.asarray(params[name], np.float32) + np.float32(1.0)).astype(np.float32)
    for i, kind in enumerate(layer_types):
        pre = f"layers.{i}."
        xn = rms_norm(h, zc(pre + "input_layernorm.weight"), epsilon)
        if kind == "linear":
            sub = {k[len(pre + "linear_attn."):]: v for k, v in params.items()
                   if k.startswith(pre + "linear_attn.")}
            sub["conv1d.weight"] = np.asarray(sub["conv1d.weight"])
            out, _, _ = gdo.gated_delta_attention(xn, sub, heads=linear_heads,
                                                  head_dim=linear_head_dim, group_size=G,
                                                  eps=epsilon, w8_linear=lambda x, w, s, g, mode=1:
                                                  lin_mode(x, w, s, g))
        else:
            sub = {k[len(pre + "self_attn."):]: v for k, v in params.items()
                   if k.startswith(pre + "self_attn.")}
            out = full_attention(xn, sub, attention_heads=attention_heads,
                                 key_value_heads=key_value_heads, head_dim=head_dim,
                                 rotary_dim=rotary_dim, rope_theta=rope_theta, group_size=G,
                                 eps=epsilon, round_attention=gpu_rounding, linear_mode=mode,
                                 round_keys=not f32_compute)
        h = (h + out).astype(np.float32)                               # mod.rs:246
        xn = rms_norm(h, zc(pre + "post_attention_layernorm.weight"), epsilon)

        def lin(name, inp):
            return w8_linear(inp.reshape(B * T, -1), params[pre + f"mlp.{name}.weight"],
                             params[pre + f"mlp.{name}.scale"], G, mode=mode).reshape(B, T, -1)
        gate = lin("gate_proj", xn).astype(np.float64)
        up = lin("up_proj", xn).astype(np.float64)
        y = (gate / (1.0 + np.exp(-gate)) * up).astype(np.float32)   # layers.rs:270-293
        h = (h + lin("down_proj", y)).astype(np.float32)
    hn = rms_norm(h, zc("norm.weight"), epsilon)
    # tied LM head (mod.rs:157-173): F32 hidden · F32 dequantized embedding
    return w8_linear(hn.reshape(B * T, -1), emb_w, emb_s, G,
                     mode=5 if gpu_rounding and not f32_compute else 0).reshape(B, T, vocabulary)
