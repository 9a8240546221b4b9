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
                   rope_theta, group_size, eps=1e-6, positions=None, round_attention=False):
    """x [B, T, hidden] F32 (the normalised layer input).  params: q_proj /
    k_proj / v_proj / o_proj `.weight` u8 and `.scale` f32, q_norm.weight and
    k_norm.weight f32 [D] (zero-centred: the norm multiplies by weight + 1).
    Returns the layer output [B, T, hidden] F32 (the bf16 o_proj dot widened).
    round_attention=True rounds the attended values to bf16 before the gate,
    as the paged attention kernel's bf16 output does (the reference keeps
    them F32): the model of that one extra rounding point, used to measure
    its effect."""
    B, T, hid = x.shape
    Hq, Hkv, D = attention_heads, key_value_heads, head_dim

    def proj(name, inp):
        return w8_linear(inp.reshape(B * T, -1), params[f"{name}.weight"], params[f"{name}.scale"],
                         group_size, mode=1).reshape(B, T, -1)

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
