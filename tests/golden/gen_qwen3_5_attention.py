"""Generate tests/golden/qwen3_5_attention_transformers.npz, an independent pin
of the Qwen3.5 full-attention oracle (oracle/qwen3_5.py `full_attention`).

rxla's full-attention layer (crates/rxla-models/src/qwen3_5/layers.rs:28-100)
cannot run here (Rust + a PJRT plugin).  Hugging Face transformers ships a
separate PyTorch implementation of the same published layer: `Qwen3_5Attention`
(q_proj rows as per-head [query | gate] pairs, zero-centred q/k RMSNorm,
partial rotary embedding over the first `partial_rotary_factor · head_dim`
dimensions, grouped-query attention, the sigmoid output gate, o_proj).  This
script quantizes seeded weights to W8 with the oracle's quantizer (itself
pinned to the reference's encoder), hands transformers the dequantized F32
weights, runs its eager causal forward, and stores the W8 parameters, the
input and the output.  tests/test_qwen3_5_oracle.py checks the oracle in its
F32-compute form against them.

    python tests/golden/gen_qwen3_5_attention.py        # from the repository root
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from transformers.models.qwen3_5 import modeling_qwen3_5 as hf  # noqa: E402
from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig  # noqa: E402

OUT = Path(__file__).resolve().parent / "qwen3_5_attention_transformers.npz"


def main() -> None:
    B, T, hidden, Hq, Hkv, D, rot, G = 2, 9, 64, 4, 2, 32, 16, 32
    theta, eps = 1e7, 1e-6
    rng = np.random.default_rng(20261203)
    params = {}
    dense = {}
    for name, (n, k) in {"q_proj": (2 * Hq * D, hidden), "k_proj": (Hkv * D, hidden),
                         "v_proj": (Hkv * D, hidden), "o_proj": (hidden, Hq * D)}.items():
        w = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)
        q, s = oracle.quantize_w8(w, G)
        params[f"{name}.weight"], params[f"{name}.scale"] = q, s
        dense[name] = ((q.astype(np.float32) - np.float32(128.0)) *
                       np.repeat(s.reshape(n, k // G), G, axis=1)).astype(np.float32)
    params["q_norm.weight"] = (0.1 * rng.standard_normal(D)).astype(np.float32)
    params["k_norm.weight"] = (0.1 * rng.standard_normal(D)).astype(np.float32)
    x = rng.standard_normal((B, T, hidden)).astype(np.float32)

    cfg = Qwen3_5TextConfig(vocab_size=128, hidden_size=hidden, intermediate_size=128,
                            num_hidden_layers=1, num_attention_heads=Hq, num_key_value_heads=Hkv,
                            head_dim=D, rms_norm_eps=eps, layer_types=["full_attention"],
                            rope_parameters={"rope_type": "default", "rope_theta": theta,
                                             "partial_rotary_factor": rot / D})
    cfg._attn_implementation = "eager"
    att = hf.Qwen3_5Attention(cfg, 0).eval()
    with torch.no_grad():
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            getattr(att, name).weight.copy_(torch.from_numpy(dense[name]))
        att.q_norm.weight.copy_(torch.from_numpy(params["q_norm.weight"]))
        att.k_norm.weight.copy_(torch.from_numpy(params["k_norm.weight"]))
        xt = torch.from_numpy(x)
        pos = torch.arange(T)[None].expand(B, -1)
        cos, sin = hf.Qwen3_5TextRotaryEmbedding(cfg)(xt, pos)
        mask = torch.full((T, T), torch.finfo(torch.float32).min).triu(1)[None, None]
        y, _ = att(xt, (cos, sin), mask.expand(B, 1, T, T))
    np.savez_compressed(OUT, x=x, y=y.numpy(), heads=np.int32(Hq), kv_heads=np.int32(Hkv),
                        head_dim=np.int32(D), rotary_dim=np.int32(rot), group_size=np.int32(G),
                        rope_theta=np.float64(theta), eps=np.float32(eps),
                        **{k.replace(".", "__"): v for k, v in params.items()})
    print(OUT)


if __name__ == "__main__":
    main()
