"""The allocation-free decode attention (rxla_b200_paged_decode_attention_noalloc).

It is for callers that may not call cudaMalloc (code inside another runtime's
execute callback, whose runtime owns device memory; latency-critical loops
where an allocation can synchronise the device).  It runs the same kernel as
rxla_b200_paged_decode_attention with the split-K scratch taken from a fixed
array inside the library.  This file runs last (pytest collects it after the
other test files) and also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from rxla_b200 import _lib, nn

pytestmark = pytest.mark.gpu


def _case(batch, hq, hkv, d, ctx, max_context, seed):
    max_pages = (max_context + 15) // 16
    num_pages = batch * max_pages
    rng = np.random.default_rng(seed)
    pt = rng.permutation(num_pages).reshape(batch, max_pages).astype(np.int32)
    kp = oracle.f32_to_bf16_bits(oracle.normal(num_pages * hkv * 16 * d, seed + 1)).reshape(num_pages, hkv, 16, d)
    vp = oracle.f32_to_bf16_bits(oracle.normal(num_pages * hkv * 16 * d, seed + 2)).reshape(num_pages, hkv, 16, d)
    qkv = oracle.bf16_round(oracle.normal(batch * (hq + 2 * hkv) * d, seed + 3)).reshape(batch, -1)
    return dict(batch=batch, hq=hq, hkv=hkv, d=d, pt=pt, kp=kp, vp=vp, qkv=qkv,
                ctx=np.array(ctx, np.int32), max_context=max_context, num_pages=num_pages)


def _args(c, cache, qkv, out, qn, kn, inv, workspace=None):
    d, hq, hkv = c["d"], c["hq"], c["hkv"]
    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(a)
    a.batch, a.q_heads, a.kv_heads, a.head_dim = c["batch"], hq, hkv, d
    a.q = qkv.data_ptr()
    a.k_new = qkv.data_ptr() + hq * d * 2
    a.v_new = qkv.data_ptr() + (hq + hkv) * d * 2
    a.q_row_stride = a.kv_row_stride = qkv.stride(0)
    a.q_norm_weight, a.k_norm_weight, a.norm_eps = qn.data_ptr(), kn.data_ptr(), 1e-6
    a.inv_freq, a.rotary_dim = inv.data_ptr(), d
    a.k_pages, a.v_pages = cache.k.data_ptr(), cache.v.data_ptr()
    a.num_pages, a.page_size = c["num_pages"], 16
    a.max_pages_per_seq = cache.page_table.shape[1]
    a.page_table, a.ctx_lens = cache.page_table.data_ptr(), cache.ctx_lens.data_ptr()
    a.kv_update, a.advance_ctx = _lib.KV_CLAMP, 0
    a.out = out.data_ptr()
    if workspace is not None:
        a.workspace, a.workspace_bytes = workspace.data_ptr(), workspace.numel()
    a.max_context = c["max_context"]
    return a


def _fresh_cache(c):
    cache = nn.PagedKvCache(batch=c["batch"], kv_heads=c["hkv"], head_dim=c["d"],
                            max_context=c["max_context"], num_pages=c["num_pages"])
    cache.k.copy_(torch.from_numpy(c["kp"].view(np.int16)).view(torch.bfloat16))
    cache.v.copy_(torch.from_numpy(c["vp"].view(np.int16)).view(torch.bfloat16))
    cache.page_table = torch.from_numpy(c["pt"]).cuda()
    cache.ctx_lens = torch.from_numpy(c["ctx"].copy()).cuda()
    return cache


@pytest.mark.parametrize("shape", [
    (6, 32, 8, 128, [1, 40, 700, 1500, 2047, 333], 2048),  # many splits per sequence
    (2, 8, 2, 64, [17, 255], 256),
])
def test_noalloc_matches_workspace_entry_point_twice(shape):
    batch, hq, hkv, d, ctx, max_context = shape
    c = _case(batch, hq, hkv, d, ctx, max_context, seed=batch + d)
    dev = torch.device("cuda:0")
    qkv = torch.from_numpy(c["qkv"]).to(dev).bfloat16()
    qn = torch.from_numpy(oracle.bf16_round(oracle.normal(d, 9, 1.0, 0.1))).to(dev)
    kn = torch.from_numpy(oracle.bf16_round(oracle.normal(d, 10, 1.0, 0.1))).to(dev)
    inv = torch.from_numpy(oracle.rope_inv_freq(1e6, d)).to(dev)
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    # the existing entry point with a caller-provided workspace
    cache = _fresh_cache(c)
    ws = torch.zeros(nn.paged_decode_workspace_size(batch, hq, hkv, d, max_context),
                     dtype=torch.uint8, device=dev)
    ref = torch.empty(batch, hq * d, dtype=torch.bfloat16, device=dev)
    a = _args(c, cache, qkv, ref, qn, kn, inv, workspace=ws)
    assert lib.rxla_b200_paged_decode_attention(ctypes.byref(a), stream) == 0
    torch.cuda.synchronize()
    ref_np = ref.float().cpu().numpy()
    k_after = cache.k.clone()

    # the allocation-free entry point, two calls in a row on fresh copies of the cache
    for _ in range(2):
        cache = _fresh_cache(c)
        out = torch.empty(batch, hq * d, dtype=torch.bfloat16, device=dev)
        a = _args(c, cache, qkv, out, qn, kn, inv)
        st = lib.rxla_b200_paged_decode_attention_noalloc(ctypes.byref(a), stream)
        assert st == 0, lib.rxla_b200_last_error_message()
        torch.cuda.synchronize()
        got = out.float().cpu().numpy()
        tol = 2.0 ** -7 * np.abs(ref_np) + 1e-6  # the attention tests' bf16-ulp tolerance
        assert (np.abs(got - ref_np) <= tol).all()
        assert torch.equal(cache.k, k_after)  # the same append
    assert lib.rxla_b200_device_status(0) == 0
    # and both against the CPU oracle's restatement of the attention step,
    # at the attention tests' tolerance
    qkv_np = c["qkv"]
    ora, _ = oracle.paged_decode_attention(
        q=qkv_np[:, :hq * d], k_new=qkv_np[:, hq * d:(hq + hkv) * d],
        v_new=qkv_np[:, (hq + hkv) * d:], k_pages=c["kp"].copy(), v_pages=c["vp"].copy(),
        page_table=c["pt"], ctx_lens=c["ctx"].copy(), hq=hq, hkv=hkv, d=d,
        q_norm_w=qn.cpu().numpy(), k_norm_w=kn.cpu().numpy(), eps=1e-6,
        inv_freq=inv.cpu().numpy(), rotary_dim=d)
    vmax = np.abs(oracle.bf16_bits_to_f32(c["vp"])).max()
    assert (np.abs(got - ora) <= 2.0 ** -7 * np.abs(ora) + 2.0 ** -14 * vmax + 1e-6).all()


def test_noalloc_rejects_shapes_beyond_its_scratch():
    c = _case(1, 8, 2, 64, [3], 64, seed=1)
    dev = torch.device("cuda:0")
    cache = _fresh_cache(c)
    qkv = torch.from_numpy(c["qkv"]).to(dev).bfloat16()
    out = torch.empty(1, 8 * 64, dtype=torch.bfloat16, device=dev)
    one = torch.ones(64, device=dev)
    a = _args(c, cache, qkv, out, one, one, torch.ones(32, device=dev))
    a.batch = 16384  # split partials of 16384 sequences: far above the built-in scratch
    lib = _lib.load()
    need = nn.paged_decode_workspace_size(16384, 8, 2, 64, a.max_context)
    assert need > _lib.NOALLOC_SCRATCH_BYTES
    st = lib.rxla_b200_paged_decode_attention_noalloc(ctypes.byref(a), None)
    assert st == _lib.OUT_OF_RANGE
    assert b"scratch" in lib.rxla_b200_last_error_message()
