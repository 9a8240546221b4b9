"""The XLA custom-call adapters on the GPU, called the way XLA calls a legacy
GPU custom call: a stream, a host array of device pointers (operands, then
results) and the backend_config bytes.  Against the CPU oracle on the same
seeded inputs, with the tolerances of the direct entry points' tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from rxla_b200 import _lib, nn
from tests.test_attention_gpu import _abs_weighted_v, _check_close, _run_oracle, _setup
from tests.test_w8_linear_gpu import _case, _check

pytestmark = pytest.mark.gpu


def _buffers(*tensors):
    return (ctypes.c_void_p * len(tensors))(*[t.data_ptr() for t in tensors])


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _call(name, cfg, *tensors):
    lib = _lib.load()
    bufs = _buffers(*tensors)
    args = [_stream(), bufs, ctypes.cast(ctypes.byref(cfg), ctypes.c_void_p), ctypes.sizeof(cfg)]
    if name.endswith("_status"):
        args.append(None)  # XlaCustomCallStatus*: unused on success
    getattr(lib, name)(*args)
    torch.cuda.synchronize()
    assert lib.rxla_b200_device_status(0) == 0


def _linear_cfg(m, n, k, group, x_dtype=_lib.BF16, y_dtype=_lib.BF16, epilogue=_lib.EPI_STORE,
                fused_norm=0, eps=1e-6):
    c = _lib.XlaLinearConfig()
    c.magic, c.version = _lib.XLA_LINEAR_MAGIC, 1
    c.m, c.n, c.k, c.group_size = m, n, k, group
    c.x_dtype, c.y_dtype, c.epilogue, c.fused_norm, c.eps = x_dtype, y_dtype, epilogue, fused_norm, eps
    assert _lib.load().rxla_b200_xla_check_config(b"rxla_b200_xla_w8a16_linear_status",
                                                  ctypes.byref(c), ctypes.sizeof(c)) == 0
    return c


@pytest.mark.parametrize("m,n,k,group", [(1, 4096, 4096, 4096), (5, 384, 1024, 128),
                                         (40, 640, 2048, 2048)])
def test_xla_linear_matches_oracle(cuda, m, n, k, group):
    """Operands [x, weight, scale], result [y]: the reference-rounding linear."""
    x, w, s = _case(m, n, k, group, seed=900 + m)
    xt = torch.from_numpy(x).cuda().bfloat16()
    wt, st = torch.from_numpy(w).cuda(), torch.from_numpy(np.ascontiguousarray(s)).cuda()
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _call("rxla_b200_xla_w8a16_linear_status", _linear_cfg(m, n, k, group), xt, wt, st, y)
    _check(y.float().cpu().numpy(), x, w, s, group)


@pytest.mark.parametrize("aliased", [True, False])
def test_xla_fused_norm_residual(cuda, aliased):
    """Operands [h, norm_weight, weight, scale, residual], result [y]: y is
    residual + bf16(linear(rms_norm(h))), whether y aliases the residual
    operand (a donated buffer) or not (then the residual is copied first and
    stays unchanged)."""
    m, n, k = 3, 512, 4096
    h = oracle.normal(m * k, 910, 0.0, 2.0).reshape(m, k)
    nw = oracle.bf16_round(oracle.normal(k, 911, 1.0, 0.02))
    w = (oracle.randint(n * k, 912, -127, 128).reshape(n, k) + 128).astype(np.uint8)
    s = oracle.uniform(n, 913, 1e-3, 1e-2).reshape(n, 1)
    r0 = oracle.normal(m * n, 914).reshape(m, n)
    ht, nwt = torch.from_numpy(h).cuda(), torch.from_numpy(nw).cuda()
    wt, st = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda()
    r = torch.from_numpy(r0).cuda()
    y = r if aliased else torch.empty_like(r)
    cfg = _linear_cfg(m, n, k, k, x_dtype=_lib.F32, y_dtype=_lib.F32,
                      epilogue=_lib.EPI_RESIDUAL_ADD, fused_norm=1)
    _call("rxla_b200_xla_w8a16_linear", cfg, ht, nwt, wt, st, r, y)
    # the bf16 dot of the same fused-norm kernel, and the oracle for it
    dot = nn.quantized_norm_linear(ht, nwt, 1e-6, wt, st, k).float().cpu().numpy()
    _check(dot, oracle.bf16_round(oracle.rms_norm(h, nw, 1e-6)), w, s, k)
    np.testing.assert_array_equal(y.cpu().numpy(), (r0 + dot).astype(np.float32))
    if not aliased:
        np.testing.assert_array_equal(r.cpu().numpy(), r0)


@pytest.mark.parametrize("aliased", [True, False])
def test_xla_paged_decode_attention_matches_oracle(cuda, aliased):
    """Operands [q, k_new, v_new, q_norm_w, k_norm_w, inv_freq, page_table,
    ctx_lens, k_pages, v_pages], results [out, ctx_lens, k_pages, v_pages]:
    the allocation-free decode attention with the KV cache as (donated or
    copied) state, against the oracle; the lengths advance by one."""
    c = _setup(3, 32, 8, 128, [5, 300, 1000], max_context=1024, seed=920)
    dev = "cuda"
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    q = t(c["q"]).bfloat16()
    kn, vn = t(c["kn"]).bfloat16(), t(c["vn"]).bfloat16()
    kp = t(c["kp"].view(np.int16)).view(torch.bfloat16)
    vp = t(c["vp"].view(np.int16)).view(torch.bfloat16)
    pt, ctx = t(c["pt"]), t(c["ctx"])
    qw, kw, inv = t(c["qw"]), t(c["kw"]), t(c["inv"])
    out = torch.empty(3, 32 * 128, dtype=torch.bfloat16, device=dev)
    if aliased:
        ctx_o, kp_o, vp_o = ctx, kp, vp
    else:
        ctx_o, kp_o, vp_o = torch.empty_like(ctx), torch.empty_like(kp), torch.empty_like(vp)
    a = _lib.XlaAttentionConfig()
    a.magic, a.version = _lib.XLA_ATTENTION_MAGIC, 1
    a.batch, a.q_heads, a.kv_heads, a.head_dim = 3, 32, 8, 128
    a.page_size, a.max_pages_per_seq, a.num_pages = 16, c["pt"].shape[1], c["num_pages"]
    a.max_context, a.has_qk_norm, a.rotary_dim = 1024, 1, c["rot"]
    a.kv_update, a.norm_eps, a.scale = _lib.KV_CLAMP, 1e-6, 0.0
    _call("rxla_b200_xla_paged_decode_attention_status", a, q, kn, vn, qw, kw, inv, pt, ctx, kp,
          vp, out, ctx_o, kp_o, vp_o)
    ref, kpo, vpo, ctx_ref, _ = _run_oracle(c, advance=True)
    _check_close(out.float().cpu().numpy(), ref, _abs_weighted_v(c, kpo, vpo))
    np.testing.assert_array_equal(ctx_o.cpu().numpy(), ctx_ref)
    np.testing.assert_array_equal(vp_o.cpu().view(torch.int16).numpy().view(np.uint16), vpo)
    if not aliased:  # the operands are untouched
        np.testing.assert_array_equal(ctx.cpu().numpy(), c["ctx"])
        np.testing.assert_array_equal(vp.cpu().view(torch.int16).numpy().view(np.uint16), c["vp"])
