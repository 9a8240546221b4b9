"""Generate tests/golden/gated_delta_transformers.npz, an independent pin of the
gated-delta oracle (oracle/gated_delta.py).

rxla's gated-delta mixer (crates/rxla-models/src/qwen3_5/layers.rs:114-268)
cannot run here (Rust + a PJRT plugin).  Hugging Face transformers ships a
separate PyTorch implementation of the same published layer (Qwen3.5's
Gated DeltaNet: causal depthwise conv + SiLU, L2-normalised q/k, the gated
delta rule, the gated RMSNorm).  This script runs transformers' own torch
functions — `torch_recurrent_gated_delta_rule` (with its in-kernel q/k L2
norm) and `Qwen3_5RMSNormGated`, plus the causal `F.conv1d` its
`Qwen3_5GatedDeltaNet.forward` uses without the fused kernels — on seeded
inputs, and stores inputs and outputs.  tests/test_gated_delta_oracle.py
checks the oracle against them.  transformers computes in float32, so the
comparison is at float32 tolerance.

    python tests/golden/gen_gated_delta.py        # from the repository root
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F
from transformers.models.qwen3_5 import modeling_qwen3_5 as hf

OUT = Path(__file__).resolve().parent / "gated_delta_transformers.npz"


def main() -> None:
    g = torch.Generator().manual_seed(20261202)
    B, T, H, D, K = 2, 13, 3, 16, 4
    W = H * D
    C3 = 3 * W

    def rnd(*shape, scale=1.0):
        # bf16-representable values, as the projections deliver them
        return (torch.randn(*shape, generator=g) * scale).bfloat16().float()

    mixed = rnd(B, T, C3)
    z = rnd(B, T, W)
    b = rnd(B, T, H)
    a = rnd(B, T, H)
    conv_w = torch.randn(C3, K, generator=g) * 0.5
    a_log = torch.log(torch.rand(H, generator=g) * 15 + 1)
    dt_bias = torch.randn(H, generator=g) * 0.5
    norm_w = 1.0 + torch.randn(D, generator=g) * 0.1
    eps = 1e-6

    x = F.silu(F.conv1d(mixed.transpose(1, 2), conv_w.unsqueeze(1), padding=K - 1,
                        groups=C3)[..., :T]).transpose(1, 2)
    q, k, v = torch.split(x, [W, W, W], dim=-1)
    q = q.reshape(B, T, H, D)
    k = k.reshape(B, T, H, D)
    v = v.reshape(B, T, H, D)
    beta = b.sigmoid()
    gdec = -a_log.exp() * F.softplus(a + dt_bias)
    core, state = hf.torch_recurrent_gated_delta_rule(
        q, k, v, g=gdec, beta=beta, initial_state=None, output_final_state=True,
        use_qk_l2norm_in_kernel=True)
    norm = hf.Qwen3_5RMSNormGated(D, eps=eps)
    with torch.no_grad():
        norm.weight.copy_(norm_w)
        y = norm(core.reshape(-1, D), z.reshape(-1, D)).reshape(B, T, W)
    np.savez_compressed(
        OUT, mixed=mixed.numpy(), z=z.numpy(), b=b.numpy(), a=a.numpy(),
        conv_weight=conv_w.numpy(), a_log=a_log.numpy(), dt_bias=dt_bias.numpy(),
        norm_weight=norm_w.numpy(), eps=np.float32(eps), heads=np.int32(H), head_dim=np.int32(D),
        y=y.detach().numpy(), state=state.numpy())
    print(OUT)


if __name__ == "__main__":
    main()
