"""Generate tests/golden/qwen3_5_model_transformers.npz, an independent pin of
the Qwen3.5 model oracle (oracle/qwen3_5.py `qwen3_5_forward`).

rxla's Qwen3.5 text model (crates/rxla-models/src/qwen3_5/mod.rs:199-260)
cannot run here (Rust + a PJRT plugin).  Hugging Face transformers ships a
separate PyTorch implementation of the same published model,
`Qwen3_5ForCausalLM`: token embedding, per layer a zero-centred RMSNorm, the
gated-delta or the gated full-attention mixer by `layer_types`, the residual
add, a second norm, the SwiGLU MLP and its residual add; the final norm and
the tied LM head.  This script quantizes seeded weights of a 4-layer model
(linear, full, linear, full) to W8 with the oracle's quantizer, hands
transformers the dequantized F32 weights (its torch fallbacks for the conv
and the delta rule), runs its causal forward over seeded token ids, and stores
the W8 parameters, the ids and the logits.  tests/test_qwen3_5_oracle.py checks
the oracle in its F32-compute form against them.

    python tests/golden/gen_qwen3_5_model.py        # from the repository root
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from transformers.models.qwen3_5 import modeling_qwen3_5 as hf  # noqa: E402
from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig  # noqa: E402

OUT = Path(__file__).resolve().parent / "qwen3_5_model_transformers.npz"

CFG = dict(vocabulary=128, hidden_size=64, intermediate_size=96,
           layer_types=["linear", "full", "linear", "full"], attention_heads=4,
           key_value_heads=2, head_dim=32, linear_heads=2, linear_head_dim=32, conv_kernel=4,
           rope_theta=1e7, rotary_dim=16, epsilon=1e-6, quant_group_size=32)


def main() -> None:
    c = CFG
    V, H, I, G = c["vocabulary"], c["hidden_size"], c["intermediate_size"], c["quant_group_size"]
    Hq, Hkv, D = c["attention_heads"], c["key_value_heads"], c["head_dim"]
    Hl, Dl, K = c["linear_heads"], c["linear_head_dim"], c["conv_kernel"]
    Wl = Hl * Dl
    rng = np.random.default_rng(20261204)
    params, dense = {}, {}

    def w8(name, n, k, sc):
        q, s = oracle.quantize_w8((rng.standard_normal((n, k)) * sc).astype(np.float32), G)
        params[name + ".weight"], params[name + ".scale"] = q, s
        dense[name + ".weight"] = ((q.astype(np.float32) - np.float32(128.0)) *
                                   np.repeat(s.reshape(n, k // G), G, axis=1)).astype(np.float32)

    def vec(name, arr):
        params[name] = dense[name] = np.asarray(arr, np.float32)

    w8("embed_tokens", V, H, 0.5)
    for i, kind in enumerate(c["layer_types"]):
        pre = f"layers.{i}."
        vec(pre + "input_layernorm.weight", 0.1 * rng.standard_normal(H))
        vec(pre + "post_attention_layernorm.weight", 0.1 * rng.standard_normal(H))
        if kind == "linear":
            la = pre + "linear_attn."
            w8(la + "in_proj_qkv", 3 * Wl, H, H ** -0.5)
            w8(la + "in_proj_z", Wl, H, H ** -0.5)
            w8(la + "in_proj_b", Hl, H, H ** -0.5)
            w8(la + "in_proj_a", Hl, H, H ** -0.5)
            w8(la + "out_proj", H, Wl, Wl ** -0.5)
            vec(la + "conv1d.weight", 0.5 * rng.standard_normal((3 * Wl, 1, K)))
            vec(la + "A_log", np.log(rng.uniform(1, 16, Hl)))
            vec(la + "dt_bias", 0.5 * rng.standard_normal(Hl))
            vec(la + "norm.weight", 1 + 0.1 * rng.standard_normal(Dl))
        else:
            sa = pre + "self_attn."
            w8(sa + "q_proj", 2 * Hq * D, H, H ** -0.5)
            w8(sa + "k_proj", Hkv * D, H, H ** -0.5)
            w8(sa + "v_proj", Hkv * D, H, H ** -0.5)
            w8(sa + "o_proj", H, Hq * D, (Hq * D) ** -0.5)
            vec(sa + "q_norm.weight", 0.1 * rng.standard_normal(D))
            vec(sa + "k_norm.weight", 0.1 * rng.standard_normal(D))
        w8(pre + "mlp.gate_proj", I, H, H ** -0.5)
        w8(pre + "mlp.up_proj", I, H, H ** -0.5)
        w8(pre + "mlp.down_proj", H, I, I ** -0.5)
    vec("norm.weight", 0.1 * rng.standard_normal(H))
    ids = rng.integers(0, V, (2, 11)).astype(np.int32)

    cfg = Qwen3_5TextConfig(
        vocab_size=V, hidden_size=H, intermediate_size=I, num_hidden_layers=len(c["layer_types"]),
        num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D, rms_norm_eps=c["epsilon"],
        rope_parameters={"rope_type": "default", "rope_theta": c["rope_theta"],
                         "partial_rotary_factor": c["rotary_dim"] / D},
        layer_types=[{"linear": "linear_attention", "full": "full_attention"}[t]
                     for t in c["layer_types"]],
        linear_num_key_heads=Hl, linear_num_value_heads=Hl, linear_key_head_dim=Dl,
        linear_value_head_dim=Dl, linear_conv_kernel_dim=K, tie_word_embeddings=True)
    cfg._attn_implementation = "eager"
    model = hf.Qwen3_5ForCausalLM(cfg).eval()
    sd = {"model." + k: torch.from_numpy(v) for k, v in dense.items()}
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    with torch.no_grad():
        logits = model(input_ids=torch.from_numpy(ids).long(), use_cache=False).logits
    np.savez_compressed(OUT, ids=ids, logits=logits.numpy(), config=np.array(json.dumps(CFG)),
                        **{k.replace(".", "__"): v for k, v in params.items()})
    print(OUT)


if __name__ == "__main__":
    main()
