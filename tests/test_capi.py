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
