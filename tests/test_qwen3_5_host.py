"""Host-side logic of the Qwen3.5 mirrors (rxla_b200/qwen3_5.py,
rxla_b200/gated_delta.py) on the CPU: the weight layouts built at load — the
q_proj rows reordered into [all queries; all gates] and fused with k / v, the
gated-delta in-projections fused as qkv | z | b | a — and the argument checks
that refuse bad shapes before any device call.  The layers are constructed on
CPU tensors; nothing here launches a kernel."""
import numpy as np
import pytest
import torch

import oracle
from rxla_b200.gated_delta import GatedDeltaAttention
from rxla_b200.nn import InvalidLayerInput
from rxla_b200.qwen3_5 import GatedFullAttention, Qwen3_5Model


def _w8(rng, n, k, G):
    q, s = oracle.quantize_w8(rng.standard_normal((n, k)).astype(np.float32), G)
    return torch.from_numpy(q), torch.from_numpy(s)


def _attn_params(hidden, Hq, Hkv, D, G, seed=0):
    rng = np.random.default_rng(seed)
    p = {}
    for name, (n, k) in {"q_proj": (2 * Hq * D, hidden), "k_proj": (Hkv * D, hidden),
                         "v_proj": (Hkv * D, hidden), "o_proj": (hidden, Hq * D)}.items():
        p[f"{name}.weight"], p[f"{name}.scale"] = _w8(rng, n, k, G)
    p["q_norm.weight"] = torch.from_numpy((0.1 * rng.standard_normal(D)).astype(np.float32))
    p["k_norm.weight"] = torch.from_numpy((0.1 * rng.standard_normal(D)).astype(np.float32))
    return p


ATTN = dict(hidden_size=128, attention_heads=4, key_value_heads=2, head_dim=64, rotary_dim=32,
            rope_theta=1e7, quant_group_size=64)


def _attn(p=None, **kw):
    a = dict(ATTN, **kw)
    p = p or _attn_params(a["hidden_size"], a["attention_heads"], a["key_value_heads"],
                          a["head_dim"], a["quant_group_size"])
    return GatedFullAttention(p, batch=2, max_context=32, **a), p


def test_q_proj_rows_reordered_into_queries_then_gates():
    """q_proj stores per head [query rows | gate rows] (layers.rs:50-55); the
    fused weight holds every head's query rows, then every gate row, then
    k_proj and v_proj, with the scales moved alongside."""
    layer, p = _attn()
    Hq, Hkv, D = 4, 2, 64
    wq = p["q_proj.weight"].reshape(Hq, 2, D, -1)
    sq = p["q_proj.scale"].reshape(Hq, 2, D, -1)
    want_w = torch.cat([wq[:, 0].reshape(Hq * D, -1), wq[:, 1].reshape(Hq * D, -1),
                        p["k_proj.weight"], p["v_proj.weight"]])
    want_s = torch.cat([sq[:, 0].reshape(Hq * D, -1), sq[:, 1].reshape(Hq * D, -1),
                        p["k_proj.scale"].reshape(Hkv * D, -1),
                        p["v_proj.scale"].reshape(Hkv * D, -1)])
    assert torch.equal(layer.w_in, want_w)
    assert torch.equal(layer.s_in, want_s)
    # zero-centred norms: the kernels get weight + 1
    assert torch.equal(layer.q_norm, p["q_norm.weight"] + 1.0)
    assert torch.equal(layer.k_norm, p["k_norm.weight"] + 1.0)


@pytest.mark.parametrize("kw,msg", [(dict(head_dim=96), "head_dim"),
                                    (dict(key_value_heads=3), "configuration"),
                                    (dict(rotary_dim=33), "configuration"),
                                    (dict(rotary_dim=128), "configuration")])
def test_attention_configuration_checks(kw, msg):
    a = dict(ATTN, **kw)
    p = _attn_params(a["hidden_size"], a["attention_heads"], a["key_value_heads"],
                     a["head_dim"] if a["head_dim"] != 96 else 64, a["quant_group_size"])
    with pytest.raises(InvalidLayerInput, match=msg):
        GatedFullAttention(p, batch=2, max_context=32, **a)


def test_attention_weight_shape_checks():
    p = _attn_params(128, 4, 2, 64, 64)
    p["k_proj.weight"] = p["k_proj.weight"][:-1]
    with pytest.raises(InvalidLayerInput, match="k_proj.weight"):
        _attn(p)
    p = _attn_params(128, 4, 2, 64, 64)
    p["o_proj.scale"] = p["o_proj.scale"].double()
    with pytest.raises(InvalidLayerInput, match="o_proj.scale"):
        _attn(p)


def test_attention_forward_argument_checks():
    layer, _ = _attn()
    x = torch.zeros(2, 3, 128)
    with pytest.raises(InvalidLayerInput, match="contiguous"):
        layer.forward(x.transpose(0, 1).contiguous().transpose(0, 1))
    with pytest.raises(InvalidLayerInput):
        layer.forward(torch.zeros(3, 3, 128))  # batch differs from the cache's
    with pytest.raises(InvalidLayerInput):
        layer.forward(torch.zeros(2, 3, 64))
    with pytest.raises(InvalidLayerInput, match="residual"):
        layer.forward(x, residual=torch.zeros(2, 3, 128, dtype=torch.float64))
    with pytest.raises(InvalidLayerInput, match="residual"):
        layer.forward(x, residual=torch.zeros(2, 4, 128))
    with pytest.raises(InvalidLayerInput):
        layer.step(torch.zeros(3, 128))


def _gdn_params(hidden, H, D, K, G, seed=1):
    rng = np.random.default_rng(seed)
    W = H * D
    p = {}
    for name, (n, k) in {"in_proj_qkv": (3 * W, hidden), "in_proj_z": (W, hidden),
                         "in_proj_b": (H, hidden), "in_proj_a": (H, hidden),
                         "out_proj": (hidden, W)}.items():
        p[f"{name}.weight"], p[f"{name}.scale"] = _w8(rng, n, k, G)
    p["conv1d.weight"] = torch.from_numpy(rng.standard_normal((3 * W, 1, K)).astype(np.float32))
    p["A_log"] = torch.zeros(H)
    p["dt_bias"] = torch.zeros(H)
    p["norm.weight"] = torch.ones(D)
    return p


def test_gated_delta_in_projections_fused_in_order():
    """One W8 linear makes mixed | z | b | a: the fused weight is the four
    projections' rows in that order, with their scales."""
    p = _gdn_params(128, 2, 32, 4, 64)
    m = GatedDeltaAttention(p, hidden_size=128, linear_heads=2, linear_head_dim=32,
                            conv_kernel=4, quant_group_size=64)
    names = ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a")
    assert torch.equal(m.w_in, torch.cat([p[f"{n}.weight"] for n in names]))
    assert torch.equal(m.s_in, torch.cat([p[f"{n}.scale"].reshape(-1, 2) for n in names]))
    assert tuple(m.conv_w.shape) == (3 * 64, 4)


@pytest.mark.parametrize("break_", ["conv", "alog", "norm", "z", "group"])
def test_gated_delta_checks(break_):
    p = _gdn_params(128, 2, 32, 4, 64)
    kw = dict(hidden_size=128, linear_heads=2, linear_head_dim=32, conv_kernel=4,
              quant_group_size=64)
    if break_ == "conv":
        p["conv1d.weight"] = p["conv1d.weight"][..., :3]
    elif break_ == "alog":
        p["A_log"] = torch.zeros(3)
    elif break_ == "norm":
        p["norm.weight"] = torch.ones(32, dtype=torch.float64)
    elif break_ == "z":
        p["in_proj_z.weight"] = p["in_proj_z.weight"][:, :64]
    else:
        kw["quant_group_size"] = 48
    with pytest.raises(InvalidLayerInput):
        GatedDeltaAttention(p, **kw)


def test_model_rejects_unknown_layer_types_and_bad_ids():
    rng = np.random.default_rng(2)
    H, V, I, G = 128, 256, 128, 64
    p = {}
    p["embed_tokens.weight"], p["embed_tokens.scale"] = _w8(rng, V, H, G)
    pre = "layers.0."
    p[pre + "input_layernorm.weight"] = torch.zeros(H)
    p[pre + "post_attention_layernorm.weight"] = torch.zeros(H)
    for name, (n, k) in {"gate_proj": (I, H), "up_proj": (I, H), "down_proj": (H, I)}.items():
        p[pre + f"mlp.{name}.weight"], p[pre + f"mlp.{name}.scale"] = _w8(rng, n, k, G)
    p["norm.weight"] = torch.zeros(H)
    cfg = dict(vocabulary=V, hidden_size=H, intermediate_size=I, attention_heads=2,
               key_value_heads=1, head_dim=64, linear_heads=2, linear_head_dim=64,
               conv_kernel=4, rope_theta=1e7, rotary_dim=32, epsilon=1e-6, quant_group_size=G)
    with pytest.raises(InvalidLayerInput, match="layer type"):
        Qwen3_5Model(p, layer_types=["sliding"], **cfg)
    bad = dict(p, **{"embed_tokens.weight": p["embed_tokens.weight"][:, :64]})
    with pytest.raises(InvalidLayerInput, match="embed_tokens"):
        Qwen3_5Model(bad, layer_types=["sliding"], **cfg)
    p.update({pre + "self_attn." + k: v for k, v in _attn_params(H, 2, 1, 64, G).items()})
    model = Qwen3_5Model(p, layer_types=["full"], batch=2, max_context=16, **cfg)
    with pytest.raises(InvalidLayerInput, match="int32"):
        model.forward(torch.zeros(2, 3, dtype=torch.int64))
    with pytest.raises(InvalidLayerInput, match="int32"):
        model.forward(torch.zeros(3, 3, dtype=torch.int32))
