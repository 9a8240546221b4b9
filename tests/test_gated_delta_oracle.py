"""The gated-delta oracle (oracle/gated_delta.py), pinned on the CPU.

1. Against an independent implementation of the same published layer:
   transformers' own Qwen3.5 torch functions, run by
   tests/golden/gen_gated_delta.py into gated_delta_transformers.npz.
2. Properties of the reference's full-sequence semantics that the GPU path's
   state relies on: a sequence processed in pieces, carrying the conv history
   and the recurrent state, equals the full forward; a zero decay with beta
   one makes the state exactly the last k ⊗ v (the delta rule overwrites).
"""
from pathlib import Path

import numpy as np

from oracle import gated_delta as gdo

GOLDEN = Path(__file__).resolve().parent / "golden" / "gated_delta_transformers.npz"


def _case(B, T, H, D, K, seed):
    r = np.random.default_rng(seed)
    W = H * D
    f = lambda *s: r.standard_normal(s).astype(np.float32)
    return dict(mixed=f(B, T, 3 * W), z=f(B, T, W), b=f(B, T, H), a=f(B, T, H),
                conv_weight=f(3 * W, K) * 0.5, a_log=np.log(r.uniform(1, 16, H)).astype(np.float32),
                dt_bias=f(H) * 0.5, norm_weight=(1 + 0.1 * f(D)).astype(np.float32))


def test_oracle_matches_transformers_fixture():
    g = np.load(GOLDEN)
    H, D = int(g["heads"]), int(g["head_dim"])
    y, _, S = gdo.gated_delta_core(g["mixed"], g["z"], g["b"], g["a"], g["conv_weight"],
                                   g["a_log"], g["dt_bias"], g["norm_weight"], heads=H,
                                   head_dim=D, eps=float(g["eps"]))
    # transformers evaluates in float32; the oracle in float64
    np.testing.assert_allclose(y, g["y"], rtol=2e-4, atol=2e-5)
    np.testing.assert_allclose(S, g["state"], rtol=2e-4, atol=2e-5)


def test_pieces_with_carried_state_equal_full_forward():
    H, D, K = 2, 8, 4
    c = _case(2, 11, H, D, K, seed=3)
    full, cs_full, st_full = gdo.gated_delta_core(**c, heads=H, head_dim=D)
    cs, st, outs = None, None, []
    for lo, hi in [(0, 2), (2, 3), (3, 9), (9, 10), (10, 11)]:  # pieces shorter than K-1 too
        piece = {k: (v[:, lo:hi] if k in ("mixed", "z", "b", "a") else v) for k, v in c.items()}
        y, cs, st = gdo.gated_delta_core(**piece, heads=H, head_dim=D, conv_state=cs, state=st)
        outs.append(y)
    np.testing.assert_allclose(np.concatenate(outs, axis=1), full, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(cs, cs_full, rtol=0, atol=0)
    np.testing.assert_allclose(st, st_full, rtol=1e-12, atol=1e-12)


def test_delta_rule_overwrites_with_unit_beta_and_no_decay():
    """beta = 1 and decay = 0 (a_log = -inf): S_t = S_{t-1} + k (v - Sᵀk)ᵀ.
    With one token from zero state S = k vᵀ exactly."""
    H, D, K = 1, 8, 1
    c = _case(1, 1, H, D, K, seed=5)
    c["b"][:] = 1e4  # sigmoid -> 1
    c["a_log"][:] = -np.inf  # exp(A_log) = 0 -> no decay
    c["conv_weight"][:] = 1.0
    _, _, S = gdo.gated_delta_core(**c, heads=H, head_dim=D)
    x = c["mixed"][0, 0].astype(np.float64)
    x = x / (1 + np.exp(-x))
    k = x[D:2 * D] / np.sqrt((x[D:2 * D] ** 2).sum() + 1e-6)
    v = x[2 * D:]
    np.testing.assert_allclose(S[0, 0], np.outer(k, v), rtol=1e-12, atol=1e-12)
