"""Paged GQA decode attention parity on the GPU (rxla_b200_paged_decode_attention).

Inputs are seeded bf16 values; the reference is the CPU oracle's restatement
of the same contract (q/k RMSNorm, SplitHalf RoPE at position ctx_len, KV
append with clamp / checked semantics, f64 softmax over the bf16 cache).
Tolerance: the kernel keeps q and the softmax weights at f32 accuracy
(bf16 hi + lo splits) and rounds the output to bf16, so the difference is one
bf16 ulp of the output plus f32-level error: |Δ| <= 2^-7·|ref| + 2^-14·max|v|.
"""
import numpy as np
import pytest
import torch

import oracle
from rxla_b200 import _lib, nn

pytestmark = pytest.mark.gpu


def _setup(batch, hq, hkv, d, ctx, max_context, seed, rot=None, norms=True, num_pages=None,
           pages_per_seq=None):
    max_pages = (max_context + 15) // 16
    num_pages = num_pages or batch * max_pages + 3
    rng = np.random.default_rng(seed)
    pt = rng.permutation(num_pages)[: batch * max_pages].reshape(batch, max_pages).astype(np.int32)
    kp = oracle.f32_to_bf16_bits(oracle.normal(num_pages * hkv * 16 * d, seed + 1)).reshape(num_pages, hkv, 16, d)
    vp = oracle.f32_to_bf16_bits(oracle.normal(num_pages * hkv * 16 * d, seed + 2)).reshape(num_pages, hkv, 16, d)
    q = oracle.bf16_round(oracle.normal(batch * hq * d, seed + 3).reshape(batch, hq * d))
    kn = oracle.bf16_round(oracle.normal(batch * hkv * d, seed + 4).reshape(batch, hkv * d))
    vn = oracle.bf16_round(oracle.normal(batch * hkv * d, seed + 5).reshape(batch, hkv * d))
    qw = oracle.bf16_round(oracle.normal(d, seed + 6, 1.0, 0.1)) if norms else None
    kw = oracle.bf16_round(oracle.normal(d, seed + 7, 1.0, 0.1)) if norms else None
    rot = d if rot is None else rot
    inv = oracle.rope_inv_freq(1e6, rot) if rot else None
    return dict(batch=batch, hq=hq, hkv=hkv, d=d, pt=pt, kp=kp, vp=vp, q=q, kn=kn, vn=vn, qw=qw,
                kw=kw, inv=inv, rot=rot, ctx=np.array(ctx, np.int32), max_context=max_context,
                num_pages=num_pages, pps=pages_per_seq)


def _run_gpu(c, kv_update=_lib.KV_CLAMP, advance=True, workspace=None, repeat=1):
    dev = "cuda"
    cache = nn.PagedKvCache(batch=c["batch"], kv_heads=c["hkv"], head_dim=c["d"],
                            max_context=c["max_context"], num_pages=c["num_pages"])
    cache.k.copy_(torch.from_numpy(c["kp"].view(np.int16)).view(torch.bfloat16))
    cache.v.copy_(torch.from_numpy(c["vp"].view(np.int16)).view(torch.bfloat16))
    cache.page_table = torch.from_numpy(c["pt"]).to(dev)
    cache.ctx_lens = torch.from_numpy(c["ctx"].copy()).to(dev)
    if c["pps"] is not None:
        cache.pages_per_seq = torch.from_numpy(np.array(c["pps"], np.int32)).to(dev)
    # one fused qkv row per sequence: q | k | v
    qkv = torch.from_numpy(np.concatenate([c["q"], c["kn"], c["vn"]], axis=1)).to(dev).bfloat16()
    qd, kd = c["hq"] * c["d"], c["hkv"] * c["d"]
    q, k, v = qkv[:, :qd], qkv[:, qd:qd + kd], qkv[:, qd + kd:]
    t = lambda a: None if a is None else torch.from_numpy(a).to(dev)
    acc = torch.full((c["batch"],), -7, dtype=torch.int32, device=dev)
    outs = []
    for _ in range(repeat):
        out = nn.paged_decode_attention(q, k, v, cache, q_heads=c["hq"], q_norm_weight=t(c["qw"]),
                                        k_norm_weight=t(c["kw"]), eps=1e-6, inv_freq=t(c["inv"]),
                                        rotary_dim=c["rot"], kv_update=kv_update,
                                        advance_ctx=advance, accepted=acc, workspace=workspace)
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy())
    kp = cache.k.cpu().view(torch.int16).numpy().view(np.uint16)
    vp = cache.v.cpu().view(torch.int16).numpy().view(np.uint16)
    return outs, kp, vp, cache.ctx_lens.cpu().numpy(), acc.cpu().numpy()


def _run_oracle(c, kv_update=0, advance=True):
    kp, vp, ctx = c["kp"].copy(), c["vp"].copy(), c["ctx"].copy()
    out, acc = oracle.paged_decode_attention(
        q=c["q"], k_new=c["kn"], v_new=c["vn"], k_pages=kp, v_pages=vp, page_table=c["pt"],
        ctx_lens=ctx, hq=c["hq"], hkv=c["hkv"], d=c["d"], q_norm_w=c["qw"], k_norm_w=c["kw"],
        eps=1e-6, inv_freq=c["inv"], rotary_dim=c["rot"] if c["inv"] is not None else 0,
        kv_update=kv_update, advance_ctx=advance, pages_per_seq=c["pps"])
    return out, kp, vp, ctx, acc


def _abs_weighted_v(c, kp_after, vp_after):
    """Σ_t p_t |v_t| per output element, from the oracle's cache state (f64)."""
    batch, hq, hkv, d = c["batch"], c["hq"], c["hkv"], c["d"]
    G = hq // hkv
    res = np.zeros((batch, hq * d))
    for b in range(batch):
        pos = int(c["ctx"][b])
        cap = (c["pps"][b] if c["pps"] is not None else c["pt"].shape[1]) * 16
        n = 0 if pos < 0 else min(pos + 1, cap)
        if n == 0:
            continue
        slots = np.arange(n)
        pages = c["pt"][b][slots // 16]
        V = oracle.bf16_bits_to_f32(vp_after[pages, :, slots % 16]).astype(np.float64)  # [n, hkv, d]
        # uniform-weight bound is enough here: Σ p|v| <= max_t |v_t|
        res[b] = np.repeat(np.abs(V).max(axis=0), G, axis=0).reshape(-1)
    return res


def _check_close(got, ref, bound):
    tol = 2.0 ** -7 * np.abs(ref) + 2.0 ** -14 * bound + 1e-6
    excess = np.abs(got - ref) - tol
    assert excess.max() <= 0, f"excess {excess.max()} at {np.unravel_index(excess.argmax(), excess.shape)}"


@pytest.mark.parametrize("ctx", [[0, 1, 15, 16], [17, 31, 32, 33], [100, 255, 256, 511]])
def test_edge_lengths_single_split(cuda, ctx):
    c = _setup(4, 8, 2, 64, ctx, max_context=1024, seed=sum(ctx))
    (out,), kp, vp, ctx_a, acc = _run_gpu(c)
    ref, kpo, vpo, ctx_o, acc_o = _run_oracle(c)
    _check_close(out, ref, _abs_weighted_v(c, kpo, vpo))
    np.testing.assert_array_equal(ctx_a, ctx_o)
    np.testing.assert_array_equal(acc, acc_o)
    np.testing.assert_array_equal(vp, vpo)  # v appended exactly
    dk = np.abs(oracle.bf16_bits_to_f32(kp) - oracle.bf16_bits_to_f32(kpo))
    assert dk.max() <= 2.0 ** -7 * np.abs(oracle.bf16_bits_to_f32(kpo)).max()


def test_config3_shape_split_k(cuda):
    """BASELINE config 3 shape (Hq 32, Hkv 8, D 128), batch 8, L ~ U[512, 8192], split-K."""
    ctx = list(oracle.randint(6, 33, 512, 8193)) + [8191, 4096]
    c = _setup(8, 32, 8, 128, ctx, max_context=8192, seed=33)
    (out,), kp, vp, ctx_a, acc = _run_gpu(c)
    ref, kpo, vpo, ctx_o, acc_o = _run_oracle(c)
    _check_close(out, ref, _abs_weighted_v(c, kpo, vpo))
    np.testing.assert_array_equal(ctx_a, ctx_o)
    np.testing.assert_array_equal(vp, vpo)


def test_batch64_many_splits(cuda):
    ctx = list(oracle.randint(64, 44, 1, 2048))
    c = _setup(64, 16, 4, 128, ctx, max_context=2048, seed=44, rot=64)
    (out,), kp, vp, ctx_a, acc = _run_gpu(c)
    ref, kpo, vpo, ctx_o, acc_o = _run_oracle(c)
    _check_close(out, ref, _abs_weighted_v(c, kpo, vpo))


@pytest.mark.parametrize("batch,hq,hkv,ctx_hi", [(2, 8, 2, 1024), (16, 4, 1, 600)])
def test_head_dim_256(cuda, batch, hq, hkv, ctx_hi):
    """head_dim 256 (Qwen3.5-0.8B's full-attention heads) with partial RoPE
    over 64 dims and q/k norms: the small-batch and the many-sequence
    variants of the decode kernel."""
    ctx = list(oracle.randint(batch, 256 + batch, 1, ctx_hi - 1))
    c = _setup(batch, hq, hkv, 256, ctx, max_context=ctx_hi, seed=256 + batch, rot=64)
    (out,), kp, vp, ctx_a, acc = _run_gpu(c)
    ref, kpo, vpo, ctx_o, acc_o = _run_oracle(c)
    _check_close(out, ref, _abs_weighted_v(c, kpo, vpo))
    np.testing.assert_array_equal(ctx_a, ctx_o)
    np.testing.assert_array_equal(vp, vpo)
    dk = np.abs(oracle.bf16_bits_to_f32(kp) - oracle.bf16_bits_to_f32(kpo))
    assert dk.max() <= 2.0 ** -7 * np.abs(oracle.bf16_bits_to_f32(kpo)).max()


def test_single_sequence_long_pps1(cuda):
    c = _setup(1, 32, 8, 128, [3000], max_context=4096, seed=55)
    (out,), kp, vp, ctx_a, acc = _run_gpu(c)
    ref, kpo, vpo, ctx_o, _ = _run_oracle(c)
    _check_close(out, ref, _abs_weighted_v(c, kpo, vpo))


@pytest.mark.parametrize("mode", [_lib.KV_CLAMP, _lib.KV_CHECKED])
def test_out_of_range_positions(cuda, mode):
    """update_at clamps, update_at_checked rejects (kv_cache.rs:43-112)."""
    c = _setup(3, 8, 2, 64, [64, 63, 70], max_context=64, seed=66, pages_per_seq=[4, 4, 4])
    (out,), kp, vp, ctx_a, acc = _run_gpu(c, kv_update=mode)
    ref, kpo, vpo, ctx_o, acc_o = _run_oracle(c, kv_update=mode)
    np.testing.assert_array_equal(acc, acc_o)
    np.testing.assert_array_equal(ctx_a, ctx_o)
    np.testing.assert_array_equal(vp, vpo)
    _check_close(out, ref, _abs_weighted_v(c, kpo, vpo))


def test_no_norm_no_rope_and_deterministic(cuda):
    c = _setup(5, 12, 3, 128, [5, 77, 300, 1000, 1500], max_context=2048, seed=77, rot=0, norms=False)
    ws = torch.zeros(nn.paged_decode_workspace_size(5, 12, 3, 128, 2048), dtype=torch.uint8, device="cuda")
    outs, kp, vp, ctx_a, acc = _run_gpu(c, advance=False, workspace=ws, repeat=2)
    ref, kpo, vpo, ctx_o, _ = _run_oracle(c, advance=False)
    _check_close(outs[0], ref, _abs_weighted_v(c, kpo, vpo))
    np.testing.assert_array_equal(outs[0], outs[1])
    assert int(ws[:4 * (5 * 3 + 1)].view(torch.int32).abs().sum()) == 0  # counters reset
    assert nn.device_status() == 0


def test_invalid_arguments(cuda):
    c = _setup(1, 8, 3, 64, [3], max_context=64, seed=1)
    with pytest.raises(_lib.RxlaError) as e:
        _run_gpu(c)
    assert e.value.code == _lib.INVALID_ARGUMENT
