"""The Qwen3.5 oracles (oracle/qwen3_5.py: the full-attention layer and the
whole model), pinned on the CPU against an independent implementation of the
same published model: transformers' `Qwen3_5Attention` and
`Qwen3_5ForCausalLM`, run by tests/golden/gen_qwen3_5_attention.py and
gen_qwen3_5_model.py on the dequantized W8 weights into
qwen3_5_attention_transformers.npz and qwen3_5_model_transformers.npz.  The pin covers what a restatement can get
structurally wrong — the per-head [query | gate] split of q_proj, the
zero-centred q/k norms, the partial rotary embedding's half split over the
first rotary_dim dimensions, GQA head sharing, the causal mask and the
sigmoid output gate — at F32 tolerance, with the oracle in its F32-compute
form (W8 linear mode 0, keys not rounded to the cache's bf16)."""
import json
from pathlib import Path

import numpy as np

from oracle import qwen3_5 as q35

GOLDEN = Path(__file__).resolve().parent / "golden" / "qwen3_5_attention_transformers.npz"
GOLDEN_MODEL = Path(__file__).resolve().parent / "golden" / "qwen3_5_model_transformers.npz"


def _load():
    g = np.load(GOLDEN)
    params = {k.replace("__", "."): g[k] for k in g.files if "__" in k}
    kw = dict(attention_heads=int(g["heads"]), key_value_heads=int(g["kv_heads"]),
              head_dim=int(g["head_dim"]), rotary_dim=int(g["rotary_dim"]),
              rope_theta=float(g["rope_theta"]), group_size=int(g["group_size"]),
              eps=float(g["eps"]))
    return g["x"], g["y"], params, kw


def test_full_attention_matches_transformers_fixture():
    x, y, params, kw = _load()
    got = q35.full_attention(x, params, linear_mode=0, round_keys=False, **kw)
    np.testing.assert_allclose(got, y, rtol=2e-5, atol=2e-6 * np.abs(y).max())


def test_reference_rounding_points_stay_within_bf16_of_the_f32_layer():
    """The reference-semantics oracle (bf16 compute, keys as the cache stores
    them) differs from the F32 layer by bf16-level rounding only."""
    x, y, params, kw = _load()
    got = q35.full_attention(x, params, **kw)
    err = np.abs(got - y)
    assert err.max() <= 0.01 * np.abs(y).max()
    assert err.mean() <= 0.01 * np.abs(y).mean()


def test_swapped_query_and_gate_halves_are_caught():
    """A planted mistake in the oracle's input — q_proj's [query | gate] rows
    exchanged per head — moves the output far beyond the pin's tolerance."""
    x, y, params, kw = _load()
    H, D = kw["attention_heads"], kw["head_dim"]
    p = dict(params)
    for name in ("q_proj.weight", "q_proj.scale"):
        a = p[name].reshape(H, 2, D, -1)
        p[name] = np.ascontiguousarray(a[:, ::-1]).reshape(params[name].shape)
    got = q35.full_attention(x, p, linear_mode=0, round_keys=False, **kw)
    assert np.abs(got - y).max() > 0.1 * np.abs(y).max()


def _load_model():
    g = np.load(GOLDEN_MODEL)
    params = {k.replace("__", "."): g[k] for k in g.files if "__" in k}
    cfg = json.loads(str(g["config"]))
    kw = {k: v for k, v in cfg.items() if k not in ("intermediate_size", "conv_kernel")}
    return g["ids"], g["logits"], params, kw


def test_model_matches_transformers_fixture():
    """The 4-layer hybrid (linear, full, linear, full) in the oracle's F32 form
    — W8 embedding, zero-centred norms, both mixers, SwiGLU, residual adds,
    tied head — against transformers' causal forward: every position's
    logits at F32 tolerance (measured 7e-5 of an 18 maximum)."""
    ids, y, params, kw = _load_model()
    got = q35.qwen3_5_forward(ids, params, f32_compute=True, **kw)
    np.testing.assert_allclose(got, y, rtol=1e-4, atol=1e-5 * np.abs(y).max())


def test_model_reference_rounding_keeps_the_greedy_tokens():
    """The reference-semantics forward (bf16 compute) against the F32 model:
    the same greedy token at every position, logits within a few percent."""
    ids, y, params, kw = _load_model()
    got = q35.qwen3_5_forward(ids, params, **kw)
    assert (got.argmax(-1) == y.argmax(-1)).all()
    assert np.abs(got - y).mean() <= 0.05 * np.abs(y).mean()


def test_model_pin_catches_a_plain_rmsnorm():
    """A planted mistake in the oracle's input — every layer norm weight
    shifted by -1, i.e. the norms applied as plain (not zero-centred)
    RMSNorms — moves the logits far beyond the pin's tolerance."""
    ids, y, params, kw = _load_model()
    p = {k: (v - np.float32(1.0) if k.endswith("layernorm.weight") else v)
         for k, v in params.items()}
    got = q35.qwen3_5_forward(ids, p, f32_compute=True, **kw)
    assert np.abs(got - y).max() > 0.1 * np.abs(y).max()
