"""CPU oracle of Qwen3.5's gated-delta linear attention — TEST INFRASTRUCTURE ONLY.

A numpy (float64) restatement of `gated_delta_attention`
(crates/rxla-models/src/qwen3_5/layers.rs:114-268, paths inside the rxla
project): the reference's F32 graph evaluated in f64, with the bf16 rounding
points of its quantized projections (the W8 linears of the C oracle, mode 1).
Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU legs use it,
as the checker; the product library never calls it.

The reference recomputes the whole sequence from a zero state on every call
(layers.rs:198-242); `gated_delta_core` also accepts a carried conv history
and recurrent state, which the full-sequence forward over the concatenated
tokens must reproduce (tested in tests/test_gated_delta_oracle.py).
"""
from __future__ import annotations

import numpy as np


def _sigmoid(x):
    # the reference's logistic (crates/rxla-core/src/ops.rs:332-337)
    return 1.0 / (1.0 + np.exp(-x))


def _softplus(x):
    # max(x, 0) + log1p(exp(-|x|)) (crates/rxla-core/src/ops.rs:256-262 and its
    # StableHLO emission)
    return np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))


def _silu(x):
    # silu = x * sigmoid(x) (ops.rs:340-342)
    return x * _sigmoid(x)


def _l2_norm(x):
    # layers.rs:103-112: x * rsqrt(sum(x^2, last) + 1e-6)
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + 1e-6)


def gated_delta_core(mixed, z, b, a, conv_weight, a_log, dt_bias, norm_weight, *, heads,
                     head_dim, eps=1e-6, conv_state=None, state=None):
    """The mixer between the input projections and out_proj.

    mixed [B, T, 3W], z [B, T, W], b / a [B, T, H] (the projections' F32
    values), conv_weight [3W, K], a_log / dt_bias [H], norm_weight [D].
    conv_state [B, K-1, 3W] (the previous K-1 mixed rows, oldest first) and
    state [B, H, Dk, Dv] continue a sequence; None = zeros (the reference).

    Returns (y [B, T, W] float64 — the F32 value out_proj receives, before its
    bf16 cast —, new conv_state [B, K-1, 3W], new state [B, H, Dk, Dv]).
    """
    mixed = np.asarray(mixed, np.float64)
    B, T, C3 = mixed.shape
    H, D = heads, head_dim
    W = H * D
    assert C3 == 3 * W
    w = np.asarray(conv_weight, np.float64).reshape(C3, -1)
    K = w.shape[1]
    hist = np.zeros((B, K - 1, C3)) if conv_state is None else np.asarray(conv_state, np.float64)
    xp = np.concatenate([hist, mixed], axis=1)  # [B, K-1+T, 3W]
    # causal depthwise conv, padding [[K-1, 0]], cross-correlation
    # (conv2d_oihw with groups = 3W, layers.rs:131-145)
    conv = np.zeros_like(mixed)
    for j in range(K):
        conv += w[:, j][None, None, :] * xp[:, j:j + T, :]
    x = _silu(conv)
    q_scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))  # f32 constant (layers.rs:152)
    q = _l2_norm(x[..., :W].reshape(B, T, H, D)) * q_scale
    k = _l2_norm(x[..., W:2 * W].reshape(B, T, H, D))
    v = x[..., 2 * W:].reshape(B, T, H, D)
    beta = _sigmoid(np.asarray(b, np.float64))  # [B, T, H]  (layers.rs:179-187)
    decay = _softplus(np.asarray(a, np.float64) + np.asarray(dt_bias, np.float64)) * \
        -np.exp(np.asarray(a_log, np.float64))  # (layers.rs:188-197)
    S = np.zeros((B, H, D, D)) if state is None else np.array(state, np.float64)
    out = np.empty((B, T, H, D))
    for t in range(T):  # layers.rs:205-242
        S = S * np.exp(decay[:, t])[:, :, None, None]
        pred = np.einsum("bhkv,bhk->bhv", S, k[:, t])
        delta = (v[:, t] - pred) * beta[:, t][:, :, None]
        S = S + k[:, t][:, :, :, None] * delta[:, :, None, :]
        out[:, t] = np.einsum("bhkv,bhk->bhv", S, q[:, t])
    # gated RMSNorm over Dv (layers.rs:243-259)
    ns = 1.0 / np.sqrt((out * out).mean(-1, keepdims=True) + eps)
    zz = np.asarray(z, np.float64).reshape(B, T, H, D)
    y = out * ns * np.asarray(norm_weight, np.float64) * _silu(zz)
    new_hist = xp[:, T:, :] if K > 1 else hist
    return y.reshape(B, T, W), new_hist, S


def gated_delta_attention(x, params, *, heads, head_dim, group_size, eps=1e-6,
                          conv_state=None, state=None, w8_linear=None):
    """The whole mixer: projections (bf16-compute QuantizedLinear), the core,
    out_proj.  x [B, T, hidden] F32 (the normalised layer input).  params maps
    the reference's names (in_proj_qkv / in_proj_z / in_proj_b / in_proj_a /
    out_proj .weight u8 and .scale f32, conv1d.weight, A_log, dt_bias,
    norm.weight) to arrays.  Returns (mixer output [B, T, hidden] F32 — the
    bf16 dot of out_proj widened —, new conv_state, new state)."""
    if w8_linear is None:
        from . import w8_linear
    B, T, hid = x.shape
    W = heads * head_dim

    def proj(name, inp):
        return w8_linear(inp.reshape(B * T, -1), params[f"{name}.weight"], params[f"{name}.scale"],
                         group_size, mode=1).reshape(B, T, -1)

    mixed = proj("in_proj_qkv", x)
    z = proj("in_proj_z", x)
    b = proj("in_proj_b", x)
    a = proj("in_proj_a", x)
    y, cs, st = gated_delta_core(mixed, z, b, a, params["conv1d.weight"], params["A_log"],
                                 params["dt_bias"], params["norm.weight"], heads=heads,
                                 head_dim=head_dim, eps=eps, conv_state=conv_state, state=state)
    out = proj("out_proj", y.astype(np.float32))
    return out, cs, st
