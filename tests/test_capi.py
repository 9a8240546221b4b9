"""C-ABI boundary checks that need no GPU.

* every function declared in include/rxla_b200.h is exported by
  librxla_b200.so and bound in rxla_b200._lib.SIGNATURES;
* argument validation returns the documented status (negated absl class, as
  crates/rxla-pjrt/src/runtime.rs:49-107 maps them) before touching CUDA.
"""
import ctypes
import re
import subprocess

import pytest

from rxla_b200 import _lib
from tests.conftest import ROOT

HEADER = ROOT / "include" / "rxla_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rxla_b200_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for expected in ("rxla_b200_w8a16_linear", "rxla_b200_paged_decode_attention",
                     "rxla_b200_decoder_step", "rxla_b200_allreduce"):
        assert expected in names


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (rxla_b200_\w+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    extra = sorted(exported - set(declared_functions()))
    assert not extra, f"exported but not declared: {extra}"


def test_python_binding_covers_every_symbol():
    assert set(declared_functions()) <= set(_lib.SIGNATURES)
    lib = _lib.load()
    for n in declared_functions():
        assert getattr(lib, n) is not None


def test_abi_version_and_error_message():
    lib = _lib.load()
    assert lib.rxla_b200_abi_version() == 1
    assert isinstance(lib.rxla_b200_last_error_message(), bytes)


def test_linear_validation_without_cuda():
    lib = _lib.load()
    # group size that does not divide k (crates/rxla-nn/src/layers.rs:266-275)
    st = lib.rxla_b200_w8a16_linear(None, _lib.BF16, None, None, 48, 2, 8, 64, None, _lib.BF16,
                                    _lib.EPI_STORE, None)
    assert st == _lib.INVALID_ARGUMENT
    assert b"group_size" in lib.rxla_b200_last_error_message()
    # residual epilogue needs an f32 output
    st = lib.rxla_b200_w8a16_linear(None, _lib.BF16, None, None, 64, 2, 8, 64, None, _lib.BF16,
                                    _lib.EPI_RESIDUAL_ADD, None)
    assert st == _lib.INVALID_ARGUMENT
    # m == 0 is a no-op that succeeds
    st = lib.rxla_b200_w8a16_linear(None, _lib.BF16, None, None, 64, 0, 8, 64, None, _lib.BF16,
                                    _lib.EPI_STORE, None)
    assert st == _lib.OK


def test_attention_validation_without_cuda():
    lib = _lib.load()
    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(a)
    a.batch, a.q_heads, a.kv_heads, a.head_dim = 1, 8, 3, 64  # 8 % 3 != 0 (attention.rs:99-112)
    assert lib.rxla_b200_paged_decode_attention(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT
    a.kv_heads, a.head_dim = 2, 96
    assert lib.rxla_b200_paged_decode_attention(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT
    a.struct_size = 8  # older / foreign struct
    assert lib.rxla_b200_paged_decode_attention(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT


def test_workspace_size_is_deterministic():
    lib = _lib.load()
    n1, n2 = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.rxla_b200_paged_decode_workspace_size(64, 32, 8, 128, 8192, ctypes.byref(n1)) == 0
    assert lib.rxla_b200_paged_decode_workspace_size(64, 32, 8, 128, 8192, ctypes.byref(n2)) == 0
    assert n1.value == n2.value and n1.value > 64 * 8 * 4
    assert lib.rxla_b200_paged_decode_workspace_size(1, 32, 8, 128, 0, ctypes.byref(n1)) == 0


def test_decoder_config_validation_without_cuda():
    lib = _lib.load()
    cfg = _lib.DecoderConfig()
    cfg.struct_size = ctypes.sizeof(cfg)
    cfg.layers, cfg.hidden, cfg.q_heads, cfg.kv_heads, cfg.head_dim = 1, 64, 6, 4, 16
    cfg.intermediate, cfg.vocab, cfg.rms_eps, cfg.rope_theta = 96, 128, 1e-6, 1e6
    cfg.embedding_dtype, cfg.max_batch, cfg.max_context, cfg.tp_size = _lib.U8, 1, 16, 1
    h = ctypes.c_void_p()
    assert lib.rxla_b200_decoder_create(ctypes.byref(cfg), 0, None, ctypes.byref(h)) == \
        _lib.INVALID_ARGUMENT  # 6 % 4 != 0
    cfg.kv_heads, cfg.rms_eps = 2, 0.0
    assert lib.rxla_b200_decoder_create(ctypes.byref(cfg), 0, None, ctypes.byref(h)) == \
        _lib.INVALID_ARGUMENT
    assert lib.rxla_b200_decoder_destroy(None) == _lib.OK


def test_context_lengths_and_peer_allreduce_validation_without_cuda():
    """The entry points added for external prefill and the one-shot peer
    all-reduce reject bad arguments before any CUDA call."""
    lib = _lib.load()
    lens = (ctypes.c_int32 * 2)(5, 7)
    assert lib.rxla_b200_decoder_set_context_lengths(None, lens, 2, None) == _lib.INVALID_ARGUMENT
    assert lib.rxla_b200_comm_p2p_enable(None, 1024) == _lib.INVALID_ARGUMENT
    assert lib.rxla_b200_p2p_allreduce_f32(None, None, None, 16, None) == _lib.INVALID_ARGUMENT
    msg = lib.rxla_b200_last_error_message().decode()
    assert "p2p allreduce" in msg


def test_prefill_validation_without_cuda():
    """The prefill entry rejects a missing decoder or prompt before any CUDA call."""
    lib = _lib.load()
    toks = (ctypes.c_int32 * 4)(1, 2, 3, 4)
    assert lib.rxla_b200_decoder_prefill(None, 0, toks, 4, None, None, None) == _lib.INVALID_ARGUMENT
    assert "decoder_prefill" in lib.rxla_b200_last_error_message().decode()


def test_python_constants_match_header_enums():
    """The dtype and status codes the Python binding uses are the header's."""
    text = (ROOT / "include" / "rxla_b200.h").read_text()
    enums = {m.group(1): int(m.group(2)) for m in re.finditer(r"RXLA_B200_(\w+)\s*=\s*(-?\d+)", text)}
    for name in ("F32", "BF16", "U8", "I32", "F16", "OK", "INVALID_ARGUMENT", "NOT_FOUND"):
        assert getattr(_lib, name) == enums[name], name


def test_python_noalloc_limit_matches_header():
    """The allocation-free attention's scratch limit the binding and its tests
    use is the header's RXLA_B200_NOALLOC_SCRATCH_BYTES."""
    text = HEADER.read_text()
    m = re.search(r"#define\s+RXLA_B200_NOALLOC_SCRATCH_BYTES\s+\(([^)]*)\)", text)
    assert m, "RXLA_B200_NOALLOC_SCRATCH_BYTES not found"
    expr = re.sub(r"(\d+)u\b", r"\1", m.group(1))
    assert re.fullmatch(r"[\d\s*+()]+", expr), expr
    assert eval(expr) == _lib.NOALLOC_SCRATCH_BYTES
    m = re.search(r"#define\s+RXLA_B200_COMM_ID_BYTES\s+(\d+)", text)
    assert m and int(m.group(1)) == _lib.COMM_ID_BYTES


def test_wait_timeout_range_is_checked_without_cuda():
    """rxla_b200_set_wait_timeout refuses budgets outside [1 ms, 60 s] before
    any CUDA call."""
    lib = _lib.load()
    assert lib.rxla_b200_set_wait_timeout(999_999) == _lib.INVALID_ARGUMENT
    assert lib.rxla_b200_set_wait_timeout(60_000_000_001) == _lib.INVALID_ARGUMENT
    assert "[1 ms, 60 s]" in lib.rxla_b200_last_error_message().decode()
    assert lib.rxla_b200_get_wait_timeout(None) == _lib.INVALID_ARGUMENT


def test_bounded_wait_check_validates_without_cuda():
    """rxla_b200_bounded_wait_check refuses an unknown kind and a flag wait
    without an aligned flag before any CUDA call."""
    lib = _lib.load()
    assert lib.rxla_b200_bounded_wait_check(2, None, 0, None) == _lib.INVALID_ARGUMENT
    assert lib.rxla_b200_bounded_wait_check(1, None, 1, None) == _lib.INVALID_ARGUMENT
    assert lib.rxla_b200_bounded_wait_check(1, 0x1004, 1, None) == _lib.INVALID_ARGUMENT
    assert "8-byte aligned" in lib.rxla_b200_last_error_message().decode()


def _linear_cfg(**kw):
    c = _lib.XlaLinearConfig()
    c.magic, c.version = _lib.XLA_LINEAR_MAGIC, 1
    c.m, c.n, c.k, c.group_size = 4, 64, 128, 128
    c.x_dtype, c.y_dtype, c.epilogue, c.fused_norm, c.eps = _lib.BF16, _lib.BF16, 0, 0, 1e-6
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def _attn_cfg(**kw):
    c = _lib.XlaAttentionConfig()
    c.magic, c.version = _lib.XLA_ATTENTION_MAGIC, 1
    c.batch, c.q_heads, c.kv_heads, c.head_dim = 2, 8, 2, 64
    c.page_size, c.max_pages_per_seq, c.num_pages, c.max_context = 16, 4, 8, 64
    c.has_qk_norm, c.rotary_dim, c.kv_update, c.norm_eps, c.scale = 1, 64, 0, 1e-6, 0.0
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_xla_config_layout_matches_header():
    """The backend_config structs are a wire format: 64 bytes each, the
    header's field order (checked against the C++ static_asserts' offsets)."""
    assert ctypes.sizeof(_lib.XlaLinearConfig) == 64
    assert ctypes.sizeof(_lib.XlaAttentionConfig) == 64
    assert _lib.XlaLinearConfig.m.offset == 8 and _lib.XlaLinearConfig.x_dtype.offset == 40
    assert _lib.XlaLinearConfig.eps.offset == 56
    assert _lib.XlaAttentionConfig.num_pages.offset == 32
    assert _lib.XlaAttentionConfig.max_context.offset == 40
    assert _lib.XlaAttentionConfig.scale.offset == 60
    text = HEADER.read_text()
    for name, value in (("RXLA_B200_XLA_LINEAR_MAGIC", _lib.XLA_LINEAR_MAGIC),
                        ("RXLA_B200_XLA_ATTENTION_MAGIC", _lib.XLA_ATTENTION_MAGIC)):
        m = re.search(rf"#define\s+{name}\s+0x([0-9A-Fa-f]+)u", text)
        assert m and int(m.group(1), 16) == value


def test_xla_check_config_without_cuda():
    """rxla_b200_xla_check_config: the lowering's compile-time validation of
    the backend_config bytes (size, magic, version, shape), no CUDA call."""
    lib = _lib.load()
    lin, att = b"rxla_b200_xla_w8a16_linear_status", b"rxla_b200_xla_paged_decode_attention"
    c = _linear_cfg()
    assert lib.rxla_b200_xla_check_config(lin, ctypes.byref(c), ctypes.sizeof(c)) == _lib.OK
    assert lib.rxla_b200_xla_check_config(lin, ctypes.byref(c), 56) == _lib.INVALID_ARGUMENT
    assert "expected 64" in lib.rxla_b200_last_error_message().decode()
    bad = _linear_cfg(magic=1)
    assert lib.rxla_b200_xla_check_config(lin, ctypes.byref(bad), 64) == _lib.INVALID_ARGUMENT
    newer = _linear_cfg(version=2)
    assert lib.rxla_b200_xla_check_config(lin, ctypes.byref(newer), 64) == _lib.UNIMPLEMENTED
    for kw in ({"group_size": 48}, {"epilogue": 9}, {"epilogue": _lib.EPI_RESIDUAL_ADD},
               {"fused_norm": 1}, {"y_dtype": _lib.U8}):
        c = _linear_cfg(**kw)
        assert lib.rxla_b200_xla_check_config(lin, ctypes.byref(c), 64) == _lib.INVALID_ARGUMENT, kw
    c = _linear_cfg(fused_norm=1, x_dtype=_lib.F32)
    assert lib.rxla_b200_xla_check_config(lin, ctypes.byref(c), 64) == _lib.OK
    a = _attn_cfg()
    assert lib.rxla_b200_xla_check_config(att, ctypes.byref(a), 64) == _lib.OK
    for kw in ({"q_heads": 7}, {"page_size": 32}, {"max_context": 65}, {"rotary_dim": 128},
               {"kv_update": 5}):
        a = _attn_cfg(**kw)
        assert lib.rxla_b200_xla_check_config(att, ctypes.byref(a), 64) == _lib.INVALID_ARGUMENT, kw
    assert lib.rxla_b200_xla_check_config(b"other_target", ctypes.byref(a), 64) == _lib.NOT_FOUND


def test_xla_handler_reports_a_bad_config_without_cuda():
    """A handler given a bad backend_config launches nothing and leaves the
    reason as the thread's error message (the status form would also pass it
    to XlaCustomCallStatusSetFailure when XLA is in the process)."""
    lib = _lib.load()
    c = _linear_cfg(magic=7)
    lib.rxla_b200_xla_w8a16_linear_status(None, None, ctypes.cast(ctypes.byref(c), ctypes.c_void_p),
                                          64, None)
    assert "magic" in lib.rxla_b200_last_error_message().decode()
    a = _attn_cfg(version=3)
    lib.rxla_b200_xla_paged_decode_attention(None, None, ctypes.cast(ctypes.byref(a), ctypes.c_void_p),
                                             64)
    assert "version 3" in lib.rxla_b200_last_error_message().decode()


def test_gated_delta_validation_without_cuda():
    """rxla_b200_gated_delta checks its shape before any CUDA call; an empty
    call (no tokens) succeeds without launching."""
    lib = _lib.load()
    a = _lib.GatedDeltaArgs()
    a.struct_size = ctypes.sizeof(a)
    a.batch, a.tokens, a.heads, a.head_dim, a.conv_kernel, a.eps = 1, 4, 2, 96, 4, 1e-6
    assert lib.rxla_b200_gated_delta(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT
    assert "head_dim" in lib.rxla_b200_last_error_message().decode()
    a.head_dim, a.conv_kernel = 64, 9
    assert lib.rxla_b200_gated_delta(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT
    a.conv_kernel, a.eps = 4, 0.0
    assert lib.rxla_b200_gated_delta(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT
    a.eps, a.tokens = 1e-6, 0
    assert lib.rxla_b200_gated_delta(ctypes.byref(a), None) == _lib.OK
    a.tokens = 4  # null pointers
    assert lib.rxla_b200_gated_delta(ctypes.byref(a), None) == _lib.INVALID_ARGUMENT
    n = ctypes.c_size_t()
    assert lib.rxla_b200_gated_delta_workspace_size(2, 3, 4, 64, ctypes.byref(n)) == _lib.OK
    W = 4 * 64
    al = lambda v: (v + 255) // 256 * 256
    assert n.value == al(6 * 3 * W * 4) + al(6 * 4 * 8) + al(6 * W * 4)


def test_sigmoid_gate_validation_without_cuda():
    lib = _lib.load()
    assert lib.rxla_b200_sigmoid_gate(None, 8, None, 8, -1, 8, None, 8, None) == _lib.INVALID_ARGUMENT
    assert lib.rxla_b200_sigmoid_gate(None, 8, None, 8, 0, 8, None, 8, None) == _lib.OK
    assert lib.rxla_b200_sigmoid_gate(None, 4, None, 8, 2, 8, None, 8, None) == _lib.INVALID_ARGUMENT
