"""Gated-delta linear attention on the GPU (rxla_b200_gated_delta) against the
CPU oracle's restatement of qwen3_5 `gated_delta_attention`
(crates/rxla-models/src/qwen3_5/layers.rs:114-268).

Tolerances.  The mixer is F32 in the reference; the kernels run it in f32
(the oracle in f64) and round the out_proj input to bf16, so an element
differs by at most one bf16 ulp plus f32-level error:
|Δ| <= 2^-8·|ref| + 1e-4·max|ref|.  The recurrent state (f32 on both
sides of the boundary) is held to rtol 2e-4 / atol 2e-5·max.  The conv
history is a copy of bf16 projection rows: bit-exact.  Whole-layer outputs
(W8 projections + mixer + W8 out_proj, bf16 dots) are held to the linear
tests' bar: max |Δ| <= max|ref| / 64, mean |Δ| <= 1e-3·mean|ref|.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from oracle import gated_delta as gdo
from rxla_b200 import _lib
from rxla_b200.gated_delta import GatedDeltaAttention, GatedDeltaState, gated_delta

pytestmark = pytest.mark.gpu


def _inputs(B, T, H, D, K, seed):
    rng = np.random.default_rng(seed)
    W = H * D
    bf = lambda *s, sc=1.0: oracle.bf16_round((rng.standard_normal(s) * sc).astype(np.float32))
    return dict(mixed=bf(B, T, 3 * W), z=bf(B, T, W), b=bf(B, T, H), a=bf(B, T, H),
                conv_weight=(rng.standard_normal((3 * W, K)) * 0.5).astype(np.float32),
                a_log=np.log(rng.uniform(1, 16, H)).astype(np.float32),
                dt_bias=(rng.standard_normal(H) * 0.5).astype(np.float32),
                norm_weight=(1 + 0.1 * rng.standard_normal(D)).astype(np.float32))


def _gpu_call(c, lo, hi, state, H, D):
    """Run tokens [lo, hi) of every sequence through the GPU op; returns f32 out."""
    B = c["mixed"].shape[0]
    W = H * D
    # one fused projection row: mixed | z | b | a
    row = np.concatenate([c["mixed"][:, lo:hi], c["z"][:, lo:hi], c["b"][:, lo:hi],
                          c["a"][:, lo:hi]], axis=2).reshape(B * (hi - lo), -1)
    proj = torch.from_numpy(row).cuda().bfloat16()
    t = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()
    out = gated_delta(proj[:, :3 * W], proj[:, 3 * W:4 * W], proj[:, 4 * W:4 * W + H],
                      proj[:, 4 * W + H:], t(c["conv_weight"]), t(c["a_log"]), t(c["dt_bias"]),
                      t(c["norm_weight"]), state=state)
    torch.cuda.synchronize()
    return out.float().cpu().numpy().reshape(B, hi - lo, W)


def _check_out(got, ref):
    tol = 2.0 ** -8 * np.abs(ref) + 1e-4 * np.abs(ref).max()
    bad = np.abs(got - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} elements beyond one bf16 ulp; " \
        f"max |d| {np.abs(got - ref).max():.3g}"


def _check_state(state, S_ref, hist_ref, c):
    S = state.state.cpu().numpy().transpose(0, 1, 3, 2)  # [b, h, j, :] holds column j
    np.testing.assert_allclose(S, S_ref, rtol=2e-4, atol=2e-5 * np.abs(S_ref).max())
    K = c["conv_weight"].shape[1]
    if K > 1:
        got = oracle.bf16_bits_to_f32(state.conv_state.view(torch.int16).cpu().numpy().view(np.uint16))
        np.testing.assert_array_equal(got.reshape(hist_ref.shape), hist_ref.astype(np.float32))


@pytest.mark.parametrize("B,T,H,D,K", [(1, 64, 4, 128, 4), (3, 37, 2, 64, 4), (2, 5, 3, 32, 4),
                                       (2, 20, 2, 128, 1), (1, 200, 16, 128, 4)])
def test_full_sequence_matches_oracle(cuda, B, T, H, D, K):
    c = _inputs(B, T, H, D, K, seed=B * 1000 + T + D)
    y_ref, hist, S_ref = gdo.gated_delta_core(**c, heads=H, head_dim=D)
    state = GatedDeltaState(B, H, D, K)
    got = _gpu_call(c, 0, T, state, H, D)
    _check_out(got, y_ref)
    _check_state(state, S_ref, hist, c)


@pytest.mark.parametrize("D,pieces", [(128, [40, 1, 1, 1, 3, 18]), (64, [1, 1, 2, 1, 9])])
def test_prefill_then_decode_continues_the_state(cuda, D, pieces):
    """A prompt in one call, then decode calls of one or a few tokens with the
    carried state, give the full-sequence forward's rows; pieces shorter than
    the conv history (K - 1 = 3) take their older rows from the conv state."""
    B, H, K = 2, 4, 4
    T = sum(pieces)
    c = _inputs(B, T, H, D, K, seed=77 + D)
    y_ref, hist, S_ref = gdo.gated_delta_core(**c, heads=H, head_dim=D)
    state = GatedDeltaState(B, H, D, K)
    lo = 0
    for n in pieces:
        got = _gpu_call(c, lo, lo + n, state, H, D)
        _check_out(got, y_ref[:, lo:lo + n])
        lo += n
    _check_state(state, S_ref, hist, c)


@pytest.mark.parametrize("D,K", [(32, 1), (32, 4), (64, 4), (128, 2)])
def test_single_token_calls_from_zero_state(cuda, D, K):
    """Every call one token per sequence from the first token on (the fused
    single-token kernel for few sequences: conv history shifted in place,
    the state started from zero by the first call), with the runtime conv
    width (K = 1, 2) and the float4 one (K = 4)."""
    B, H, T = 3, 2, 6
    c = _inputs(B, T, H, D, K, seed=500 + D + K)
    y_ref, hist, S_ref = gdo.gated_delta_core(**c, heads=H, head_dim=D)
    state = GatedDeltaState(B, H, D, K)
    for t in range(T):
        _check_out(_gpu_call(c, t, t + 1, state, H, D), y_ref[:, t:t + 1])
    _check_state(state, S_ref, hist, c)


def test_decode_batch_64_continues_the_state(cuda):
    """The decode shape of a serving step: 64 sequences, one token each, after
    a short prompt (the wide-grid recurrence variant)."""
    B, H, D, K, T0 = 64, 16, 128, 4, 6
    c = _inputs(B, T0 + 2, H, D, K, seed=901)
    y_ref, hist, S_ref = gdo.gated_delta_core(**c, heads=H, head_dim=D)
    state = GatedDeltaState(B, H, D, K)
    _gpu_call(c, 0, T0, state, H, D)
    for t in (T0, T0 + 1):
        _check_out(_gpu_call(c, t, t + 1, state, H, D), y_ref[:, t:t + 1])
    _check_state(state, S_ref, hist, c)


def _layer_params(hidden, H, D, K, G, seed):
    rng = np.random.default_rng(seed)
    W = H * D
    p = {}
    for name, (n, k) in {"in_proj_qkv": (3 * W, hidden), "in_proj_z": (W, hidden),
                         "in_proj_b": (H, hidden), "in_proj_a": (H, hidden),
                         "out_proj": (hidden, W)}.items():
        w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
        p[f"{name}.weight"], p[f"{name}.scale"] = oracle.quantize_w8(w, G)
    p["conv1d.weight"] = (rng.standard_normal((3 * W, 1, K)) * 0.5).astype(np.float32)
    p["A_log"] = np.log(rng.uniform(1, 16, H)).astype(np.float32)
    p["dt_bias"] = (rng.standard_normal(H) * 0.5).astype(np.float32)
    p["norm.weight"] = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    return p


def _check_layer(got, ref):
    err = np.abs(got - ref)
    assert err.max() <= np.abs(ref).max() / 64, f"max |d| {err.max():.4g}"
    assert err.mean() <= 1e-3 * np.abs(ref).mean(), f"mean |d| {err.mean():.4g}"


def test_layer_at_qwen3_5_0_8b_widths(cuda):
    """The whole mixer at the Qwen3.5-0.8B linear-attention widths (hidden
    1024, 16 heads of 128, conv 4, group 128): fused W8 input projection,
    the three kernels, W8 out_proj, against the oracle's layer."""
    hidden, H, D, K, G, B, T = 1024, 16, 128, 4, 128, 1, 48
    p = _layer_params(hidden, H, D, K, G, seed=8)
    x = np.random.default_rng(9).standard_normal((B, T, hidden)).astype(np.float32)
    ref, _, _ = gdo.gated_delta_attention(x, p, heads=H, head_dim=D, group_size=G)
    layer = GatedDeltaAttention({k: torch.from_numpy(v).cuda() for k, v in p.items()},
                                hidden_size=hidden, linear_heads=H, linear_head_dim=D,
                                conv_kernel=K, quant_group_size=G)
    got = layer.apply(torch.from_numpy(x).cuda()).cpu().numpy()
    _check_layer(got, ref)


def test_layer_residual_prefill_then_decode(cuda):
    """Batch 4: a 16-token prompt per sequence, then three decode steps, each
    added into the f32 residual stream (hidden.add(mixed), qwen3_5/mod.rs:246),
    against the oracle's full-sequence layer."""
    hidden, H, D, K, G, B, T0, steps = 1024, 16, 128, 4, 128, 4, 16, 3
    p = _layer_params(hidden, H, D, K, G, seed=18)
    rng = np.random.default_rng(19)
    x = rng.standard_normal((B, T0 + steps, hidden)).astype(np.float32)
    res0 = rng.standard_normal((B, T0 + steps, hidden)).astype(np.float32)
    ref, _, _ = gdo.gated_delta_attention(x, p, heads=H, head_dim=D, group_size=G)
    layer = GatedDeltaAttention({k: torch.from_numpy(v).cuda() for k, v in p.items()},
                                hidden_size=hidden, linear_heads=H, linear_head_dim=D,
                                conv_kernel=K, quant_group_size=G)
    state = layer.new_state(B)
    spans = [(0, T0)] + [(T0 + i, T0 + i + 1) for i in range(steps)]
    for lo, hi in spans:
        r = torch.from_numpy(np.ascontiguousarray(res0[:, lo:hi])).cuda()
        layer.apply(torch.from_numpy(np.ascontiguousarray(x[:, lo:hi])).cuda(), state, residual=r)
        _check_layer(r.cpu().numpy() - res0[:, lo:hi], ref[:, lo:hi])


def test_rejects_bad_shapes(cuda):
    c = _inputs(1, 4, 2, 64, 4, seed=1)
    state = GatedDeltaState(1, 2, 64, 4)
    a = _lib.GatedDeltaArgs()
    a.struct_size = 8  # stale struct
    assert _lib.load().rxla_b200_gated_delta(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _gpu_call(dict(c, conv_weight=c["conv_weight"][:, :3]), 0, 4, state, 2, 64)
