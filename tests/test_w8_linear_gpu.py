"""W8A16 linear parity on the GPU, through the C ABI (rxla_b200_w8a16_linear).

Checked against the CPU oracle on the same seeded inputs, at the reference's
own rounding points (oracle mode 1: bf16(x) · bf16(f32(q)·s), f64 sum, bf16
output).  The kernel forms the same exact products and sums them in fp32, so
the only difference is the fp32 accumulation: at most one bf16 ulp of the
output plus that error — |Δ| <= 2^-7·|ref| + 2^-20·Σ|x·q·s|.
"""
import numpy as np
import pytest
import torch

import oracle
from rxla_b200 import _lib, nn

pytestmark = pytest.mark.gpu


def _bound(x, w, s, group):
    k = x.shape[1]
    q = np.abs(w.astype(np.float64) - 128.0)
    xa = np.abs(oracle.bf16_round(x).astype(np.float64))
    sg = np.repeat(s.astype(np.float64), group, axis=1) if s.shape[1] > 1 else s.astype(np.float64)
    return xa @ (q * sg).T if s.shape[1] > 1 else (xa @ q.T) * s.reshape(1, -1)


def _case(m, n, k, group, seed):
    x = oracle.bf16_round(oracle.normal(m * k, seed).reshape(m, k))
    w = (oracle.randint(n * k, seed + 1, -127, 128).reshape(n, k) + 128).astype(np.uint8)
    s = oracle.uniform(n * (k // group), seed + 2, 1e-3, 1e-2).reshape(n, k // group)
    return x, w, s


def _run(x, w, s, group, x_dtype=torch.bfloat16, out_dtype=torch.bfloat16, dev="cuda"):
    xt = torch.from_numpy(x).to(dev).to(x_dtype)
    wt = torch.from_numpy(w).to(dev)
    st = torch.from_numpy(np.ascontiguousarray(s)).to(dev)
    y = nn.quantized_linear(xt, wt, st, group, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def _check(y, x, w, s, group, bf16_out=True):
    ref = oracle.w8_linear(x, w, s, group, mode=1 if bf16_out else 0).astype(np.float64)
    if not bf16_out:  # unrounded fp32 output: the f64 dot of the same bf16 operands
        xb = oracle.bf16_round(x).astype(np.float64)
        groups = s.shape[1]
        sg = np.repeat(s, w.shape[1] // groups, axis=1)
        wd = oracle.bf16_round(((w.astype(np.float32) - 128.0) * sg).astype(np.float32))
        ref = xb @ wd.astype(np.float64).T
    bound = _bound(x, w, s, group)
    rel = 2.0 ** -7 if bf16_out else 2.0 ** -22
    excess = np.abs(y - ref) - (rel * np.abs(ref) + 2.0 ** -20 * bound)
    assert excess.max() <= 0, f"reference-rounding excess {excess.max()}"
    if bf16_out:  # most outputs are bit-identical to the reference
        assert np.mean(y == ref) > 0.97, f"only {np.mean(y == ref):.3f} identical"


@pytest.mark.parametrize("m", [1, 2, 7, 8, 9, 16, 17, 32, 33, 70])
def test_sweep_shapes_small(cuda, m):
    x, w, s = _case(m, 200, 1024, 1024, seed=10 + m)
    _check(_run(x, w, s, 1024), x, w, s, 1024)


@pytest.mark.parametrize("n,k", [(4096, 4096), (6144, 4096), (4096, 12288), (12288, 4096)])
@pytest.mark.parametrize("m", [1, 8, 32, 128])
def test_config2_shapes(cuda, n, k, m):
    """(N,K) sweep, per-channel scales, M in {1,8,32,128}
    (M > 8 runs on the tcgen05 GEMM)."""
    x, w, s = oracle.linear_sweep_case(m, n, k, seed=n + k + m)
    _check(_run(x, w, s, k), x, w, s, k)


@pytest.mark.parametrize("n,k", [(4096, 4096), (12288, 4096), (4096, 12288), (6144, 4096)])
@pytest.mark.parametrize("m", [512, 2048])
def test_config2_prefill_shapes(cuda, m, n, k):
    """Config 2's tensor-bound rows (M = 512, 2048) on the tcgen05 GEMM: all
    eight (N,K) x M combinations."""
    x, w, s = oracle.linear_sweep_case(m, n, k, seed=n + k + m)
    _check(_run(x, w, s, k), x, w, s, k)


@pytest.mark.parametrize("m,group", [(24, 1024), (130, 64), (9, 128)])
def test_gemm_dequant_bit_exact(cuda, m, group):
    """The tcgen05 GEMM's dequantization is the reference's, bit for bit: one-hot
    x rows read single weights through the unrounded f32 output (partial tiles
    in M and N, per-channel and grouped scales)."""
    n, k = 300, 1024
    rng = np.random.default_rng(m)
    cols = rng.choice(k, size=m, replace=m > k)
    x = np.zeros((m, k), np.float32)
    x[np.arange(m), cols] = 1.0
    w = ((np.arange(n)[:, None] * 7 + np.arange(k)[None, :] * 13) % 256).astype(np.uint8)
    expo = oracle.uniform(n * (k // group), 77, -30.0, 2.0).reshape(n, k // group)
    s = (10.0 ** expo).astype(np.float32)
    s[::5] *= -1.0
    y = _run(x, w, s, group, out_dtype=torch.float32)
    sg = np.repeat(s, group, axis=1)
    wd = oracle.bf16_round(((w.astype(np.float32) - np.float32(128.0)) * sg).astype(np.float32))
    expect = wd[:, cols].T.astype(np.float32) + np.float32(0.0)
    np.testing.assert_array_equal((y + np.float32(0.0)).view(np.uint32), expect.view(np.uint32))


def test_gemm_residual_and_grouped(cuda):
    """Residual epilogue and grouped scales on the GEMM path (M > 8)."""
    x, w, s = _case(40, 384, 1024, 128, seed=41)
    _check(_run(x, w, s, 128), x, w, s, 128)
    h = oracle.normal(40 * 384, 42).reshape(40, 384)
    ht = torch.from_numpy(h).cuda()
    nn.quantized_linear(torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda(),
                        torch.from_numpy(s).cuda(), 128, epilogue=_lib.EPI_RESIDUAL_ADD, out=ht)
    y = _run(x, w, s, 128)
    np.testing.assert_array_equal(ht.cpu().numpy(), (h + y).astype(np.float32))


@pytest.mark.parametrize("group", [64, 128, 512])
def test_grouped_scales(cuda, group):
    x, w, s = _case(5, 300, 1024, group, seed=group)
    _check(_run(x, w, s, group), x, w, s, group)


@pytest.mark.parametrize("lo,hi", [(0.02, 0.2), (1e-30, 1e-20), (0.5, 40.0)])
def test_scale_ranges(cuda, lo, hi):
    """Scales at and beyond the kernel's fast dequant range (s >= 2^-5 takes the
    power-of-two fixup path) and tiny scales stay bit-faithful to the reference."""
    x, w, _ = _case(3, 256, 1024, 1024, seed=int(lo * 1000) + 5)
    s = oracle.uniform(256 * 2, 8, lo, hi).reshape(256, 2)
    _check(_run(x, w, s, 512), x, w, s, 512)
    s1 = s[:, :1].copy()
    _check(_run(x, w, s1, 1024), x, w, s1, 1024)


@pytest.mark.parametrize("group", [1024, 64])
def test_dequant_bit_exact(cuda, group):
    """One-hot x rows read single dequantized weights through the unrounded f32
    output: y[t, n] = bf16(f32(q - 128) · s) exactly, for every byte value and
    scales from 1e-36 to 1e3, negative and zero (the kernel's packed
    denormal-FMA dequantization against the reference's convert / subtract /
    multiply / convert chain).  Zeros compare without their sign: a dot
    product's sum of zero terms is +0."""
    m, n, k = 8, 512, 1024
    cols = np.array([0, 65, 130, 300, 511, 640, 900, 1023])
    x = np.zeros((m, k), np.float32)
    x[np.arange(m), cols] = 1.0
    rows = np.arange(n)
    w = np.zeros((n, k), np.uint8)
    for t, c in enumerate(cols):
        w[:, c] = (rows + 37 * t) % 256  # every byte value twice per column
    groups = k // group
    expo = oracle.uniform(n * groups, 31, -36.0, 3.0).reshape(n, groups)
    s = (10.0 ** expo).astype(np.float32)
    s[::7] *= -1.0
    s[5::11] = 0.0
    s[3::13] = 2.0 ** np.round(expo[3::13] * 3.3)  # exact powers of two
    y = _run(x, w, s, group, out_dtype=torch.float32)
    sg = np.repeat(s, group, axis=1)
    wd = oracle.bf16_round(((w.astype(np.float32) - np.float32(128.0)) * sg).astype(np.float32))
    expect = wd[:, cols].T.astype(np.float32) + np.float32(0.0)  # -0 -> +0
    np.testing.assert_array_equal((y + np.float32(0.0)).view(np.uint32), expect.view(np.uint32))


@pytest.mark.parametrize("n,k,group", [(37, 48, 16), (5, 64, 32), (1, 64, 64), (3, 1000, 8)])
def test_odd_shapes_generic_path(cuda, n, k, group):
    """Shapes off the fast path (K % 64 != 0, small groups) use the generic kernel."""
    x, w, s = _case(3, n, k, group, seed=n * k)
    _check(_run(x, w, s, group), x, w, s, group)


def test_f32_input_and_output(cuda):
    x, w, s = _case(4, 256, 512, 512, seed=5)
    x32 = oracle.normal(4 * 512, 99).reshape(4, 512)  # f32, rounded to bf16 by the kernel
    y = _run(x32, w, s, 512, x_dtype=torch.float32, out_dtype=torch.float32)
    _check(y, x32, w, s, 512, bf16_out=False)


def test_residual_epilogue(cuda):
    x, w, s = _case(3, 512, 1024, 1024, seed=21)
    h = oracle.normal(3 * 512, 22).reshape(3, 512)
    ht = torch.from_numpy(h).cuda()
    nn.quantized_linear(torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda(),
                        torch.from_numpy(s).cuda(), 1024, epilogue=_lib.EPI_RESIDUAL_ADD, out=ht)
    y = _run(x, w, s, 1024)  # bf16 dot
    expect = (h + y).astype(np.float32)
    np.testing.assert_array_equal(ht.cpu().numpy(), expect)


@pytest.mark.parametrize("m,n,k,group", [(1, 1536, 512, 512), (8, 3000, 1024, 128), (20, 700, 2048, 2048),
                                         (64, 1024, 1024, 1024),
                                         # x fragments held in registers (per-channel
                                         # scales, K a multiple of 1024 up to 4096): the
                                         # gate/up instance of the 8B decode step
                                         (1, 12288, 4096, 4096), (8, 6144, 4096, 4096),
                                         (3, 2000, 3072, 3072), (5, 777, 1024, 1024)])
def test_swiglu_epilogue(cuda, m, n, k, group):
    x, w, s = _case(m, 2 * n, k, group, seed=m + n)
    xt = torch.from_numpy(x).cuda().bfloat16()
    y = nn.quantized_linear(xt, torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda(), group,
                            epilogue=_lib.EPI_SWIGLU).float().cpu().numpy()
    _check_swiglu(y, x, w, s, group, n)


def _check_swiglu(y, x, w, s, group, n):
    """silu(bf16(gate)) * bf16(up) within one bf16 ulp of each half plus the
    fp32 accumulation error, propagated through silu and the product."""
    ref = oracle.w8_linear(x, w, s, group, mode=1).astype(np.float64)
    bound = _bound(x, w, s, group)
    g_ex, u_ex = ref[:, :n], ref[:, n:]
    # each of gate / up: at most one bf16 ulp + fp32 accumulation error
    dg = 2.0 ** -7 * np.abs(g_ex) + 2.0 ** -20 * bound[:, :n]
    du = 2.0 ** -7 * np.abs(u_ex) + 2.0 ** -20 * bound[:, n:]
    gate = g_ex
    sig = 1.0 / (1.0 + np.exp(-gate))
    expect = gate * sig * u_ex
    dsilu = np.abs(sig * (1.0 + gate * (1.0 - sig)))  # |d silu / d g|
    tol = dsilu * dg * (np.abs(u_ex) + du) + np.abs(gate * sig) * du + 2.0 ** -7 * np.abs(expect)
    excess = np.abs(y - expect) - 1.01 * tol
    assert excess.max() <= 1e-7, f"swiglu excess {excess.max()}"


def test_deterministic(cuda):
    x, w, s = _case(8, 4096, 4096, 4096, seed=77)
    a = _run(x, w, s, 4096)
    b = _run(x, w, s, 4096)
    np.testing.assert_array_equal(a, b)


def test_quantized_linear_layer_mirror(cuda):
    """QuantizedLinear.apply: F32 in, F32 out (the bf16 dot widened), reference errors."""
    x, w, s = _case(6, 64, 256, 32, seed=3)
    params = {"proj.weight": torch.from_numpy(w).cuda(), "proj.scale": torch.from_numpy(s).cuda()}
    y = nn.QuantizedLinear(64, 32).apply(params, "proj", torch.from_numpy(x).cuda())
    assert y.dtype == torch.float32 and tuple(y.shape) == (6, 64)
    _check(y.cpu().numpy(), x, w, s, 32)
    with pytest.raises(nn.InvalidLayerInput):
        nn.QuantizedLinear(64, 48).apply(params, "proj", torch.from_numpy(x).cuda())
    with pytest.raises(nn.InvalidLayerInput):
        nn.QuantizedLinear(64, 32).apply(params, "proj", torch.from_numpy(x).cuda().bfloat16())


def test_invalid_sizes_rejected_without_launch(cuda):
    x = torch.zeros(2, 64, device="cuda", dtype=torch.bfloat16)
    w = torch.zeros(8, 64, device="cuda", dtype=torch.uint8)
    s = torch.ones(8, 1, device="cuda")
    y = torch.empty(2, 8, device="cuda", dtype=torch.bfloat16)
    lib = _lib.load()
    st = lib.rxla_b200_w8a16_linear(x.data_ptr(), _lib.BF16, w.data_ptr(), s.data_ptr(), 48, 2, 8,
                                    64, y.data_ptr(), _lib.BF16, 0, None)
    assert st == _lib.INVALID_ARGUMENT
    assert b"group_size" in lib.rxla_b200_last_error_message()
    assert lib.rxla_b200_w8a16_linear(None, _lib.BF16, None, None, 64, 0, 8, 64, None, _lib.BF16,
                                      0, None) == _lib.OK  # m == 0 is a no-op
    assert nn.device_status() == 0


@pytest.mark.parametrize("m,n,k,epi", [(1, 6144, 4096, "store"), (1, 12288, 4096, "swiglu"),
                                       (8, 4096, 4096, "swiglu"), (3, 151936, 4096, "f32"),
                                       (2, 10240, 5120, "store"), (5, 512, 2048, "residual"),
                                       (1, 300, 12288, "store")])
def test_fused_norm_linear(cuda, m, n, k, epi):
    """rxla_b200_w8a16_norm_linear: the RMSNorm of the f32 residual fused into
    the linear's prologue, the instances a decode step runs (qkv, gate/up with
    SwiGLU, the tied head's f32 logits at K = 4096 with x in registers; K = 5120
    and 12288 through shared memory).  Against the oracle's rms_norm, the bf16
    cast and the reference-rounding linear."""
    rows = 2 * n if epi == "swiglu" else n
    h = oracle.normal(m * k, 300 + m + k, 0.0, 3.0).reshape(m, k)
    nw = oracle.bf16_round(oracle.normal(k, 301 + k, 1.0, 0.02))
    w = (oracle.randint(rows * k, 302 + n, -127, 128).reshape(rows, k) + 128).astype(np.uint8)
    s = oracle.uniform(rows, 303 + n, 1e-3, 1e-2).reshape(rows, 1)
    x = oracle.bf16_round(oracle.rms_norm(h, nw, 1e-6))
    ht, nwt = torch.from_numpy(h).cuda(), torch.from_numpy(nw).cuda()
    wt, st = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda()
    if epi == "store":
        y = nn.quantized_norm_linear(ht, nwt, 1e-6, wt, st, k).float().cpu().numpy()
        _check(y, x, w, s, k)
    elif epi == "f32":
        y = nn.quantized_norm_linear(ht, nwt, 1e-6, wt, st, k, out_dtype=torch.float32).cpu().numpy()
        _check(y, x, w, s, k, bf16_out=False)
    elif epi == "residual":
        r0 = oracle.normal(m * n, 304, 0.0, 1.0).reshape(m, n)
        rt = torch.from_numpy(r0).cuda()
        nn.quantized_norm_linear(ht, nwt, 1e-6, wt, st, k, epilogue=_lib.EPI_RESIDUAL_ADD, out=rt)
        yb = nn.quantized_norm_linear(ht, nwt, 1e-6, wt, st, k).float().cpu().numpy()
        _check(yb, x, w, s, k)
        np.testing.assert_array_equal(rt.cpu().numpy(), (r0 + yb).astype(np.float32))
    else:
        y = nn.quantized_norm_linear(ht, nwt, 1e-6, wt, st, k, epilogue=_lib.EPI_SWIGLU)
        _check_swiglu(y.float().cpu().numpy(), x, w, s, k, n)
    assert nn.device_status() == 0


@pytest.mark.parametrize("m,n,k,group,epi", [(32, 4096, 4096, 4096, _lib.EPI_STORE),
                                             (64, 6144, 4096, 128, _lib.EPI_STORE),
                                             (100, 4096, 12288, 12288, _lib.EPI_RESIDUAL_ADD),
                                             (64, 1024, 4096, 4096, _lib.EPI_SWIGLU),
                                             (9, 768, 2048, 2048, _lib.EPI_STORE)])
def test_linear_with_split_k_workspace(cuda, m, n, k, group, epi):
    """rxla_b200_w8a16_linear_ws: the GEMM splits K over the caller's
    workspace (sized by rxla_b200_w8a16_linear_workspace_size); same results
    as the oracle, the workspace's counters left zero, and a second call on
    the same workspace gives the same bits."""
    rows = 2 * n if epi == _lib.EPI_SWIGLU else n
    x, w, s = _case(m, rows, k, group, seed=700 + m)
    xt = torch.from_numpy(x).cuda().bfloat16()
    wt, st = torch.from_numpy(w).cuda(), torch.from_numpy(np.ascontiguousarray(s)).cuda()
    size = nn.linear_workspace_size(m, n, k, group, epi)
    ws = torch.zeros(max(size, 16), dtype=torch.uint8, device="cuda")
    if epi == _lib.EPI_RESIDUAL_ADD:
        # into a zero residual: y = 0 + bf16(dot) = the bf16 dot exactly
        outs = []
        for _ in range(2):
            y = torch.zeros(m, n, device="cuda")
            nn.quantized_linear(xt, wt, st, group, epilogue=epi, out=y, workspace=ws)
            outs.append(y)
        _check(outs[0].cpu().numpy(), x, w, s, group)
    else:
        outs = [nn.quantized_linear(xt, wt, st, group, epilogue=epi, workspace=ws)
                for _ in range(2)]
        y = outs[0].float().cpu().numpy()
        if epi == _lib.EPI_SWIGLU:
            _check_swiglu(y, x, w, s, group, n)
        else:
            _check(y, x, w, s, group)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    if size > 0:  # the split counters are zero again after every call
        assert int(ws[:1 << 20].count_nonzero()) == 0
    assert _lib.load().rxla_b200_device_status(0) == 0


def test_linear_workspace_too_small_is_rejected(cuda):
    m, n, k = 64, 4096, 4096
    size = nn.linear_workspace_size(m, n, k)
    if size == 0:
        pytest.skip("this shape does not split on this device")
    x, w, s = _case(m, n, k, k, seed=760)
    ws = torch.zeros(size // 2, dtype=torch.uint8, device="cuda")
    with pytest.raises(Exception, match="workspace"):
        nn.quantized_linear(torch.from_numpy(x).cuda().bfloat16(), torch.from_numpy(w).cuda(),
                            torch.from_numpy(s).cuda(), k, workspace=ws)
