"""ctypes binding of librxla_b200.so (the C ABI in include/rxla_b200.h).

The library is loaded from this package directory only; there is no fallback:
if the .so is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "librxla_b200.so"

OK = 0
INVALID_ARGUMENT = -3
DEADLINE_EXCEEDED = -4
NOT_FOUND = -5
RESOURCE_EXHAUSTED = -8
FAILED_PRECONDITION = -9
OUT_OF_RANGE = -11
UNIMPLEMENTED = -12
INTERNAL = -13
UNAVAILABLE = -14

F32, BF16, U8, I32, F16 = 0, 1, 2, 3, 4
EPI_STORE, EPI_RESIDUAL_ADD, EPI_SWIGLU = 0, 1, 2
KV_CLAMP, KV_CHECKED = 0, 1
NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024  # RXLA_B200_NOALLOC_SCRATCH_BYTES
COMM_ID_BYTES = 128  # RXLA_B200_COMM_ID_BYTES

_STATUS_NAMES = {v: k for k, v in list(globals().items()) if k.isupper() and isinstance(v, int)
                 and v <= 0 and k not in ("F32",)}


class RxlaError(RuntimeError):
    """A failing status from librxla_b200 (code = negated absl status class)."""

    def __init__(self, code: int, message: str):
        self.code = code
        name = {
            INVALID_ARGUMENT: "INVALID_ARGUMENT", DEADLINE_EXCEEDED: "DEADLINE_EXCEEDED",
            NOT_FOUND: "NOT_FOUND", RESOURCE_EXHAUSTED: "RESOURCE_EXHAUSTED",
            FAILED_PRECONDITION: "FAILED_PRECONDITION", OUT_OF_RANGE: "OUT_OF_RANGE",
            UNIMPLEMENTED: "UNIMPLEMENTED", INTERNAL: "INTERNAL", UNAVAILABLE: "UNAVAILABLE",
        }.get(code, str(code))
        super().__init__(f"{name}: {message}")


class PagedDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_uint32),
        ("batch", ctypes.c_int32), ("q_heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("k_new", ctypes.c_void_p), ("v_new", ctypes.c_void_p),
        ("q_row_stride", ctypes.c_int64), ("kv_row_stride", ctypes.c_int64),
        ("q_norm_weight", ctypes.c_void_p), ("k_norm_weight", ctypes.c_void_p),
        ("norm_eps", ctypes.c_float),
        ("inv_freq", ctypes.c_void_p), ("rotary_dim", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("k_pages", ctypes.c_void_p), ("v_pages", ctypes.c_void_p),
        ("num_pages", ctypes.c_int64), ("page_size", ctypes.c_int32),
        ("max_pages_per_seq", ctypes.c_int32),
        ("page_table", ctypes.c_void_p), ("pages_per_seq", ctypes.c_void_p),
        ("ctx_lens", ctypes.c_void_p),
        ("kv_update", ctypes.c_int32), ("advance_ctx", ctypes.c_int32),
        ("accepted", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("max_context", ctypes.c_int32),
    ]


class DecoderConfig(ctypes.Structure):
    _fields_ = [("struct_size", ctypes.c_uint32)] + \
        [(n, ctypes.c_int32) for n in ("layers", "hidden", "q_heads", "kv_heads", "head_dim",
                                       "intermediate", "vocab")] + \
        [("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)] + \
        [(n, ctypes.c_int32) for n in ("embedding_dtype", "group_size", "max_batch",
                                       "max_context", "tp_rank", "tp_size")]


class GatedDeltaArgs(ctypes.Structure):
    """rxla_b200_gated_delta_args."""
    _fields_ = [("struct_size", ctypes.c_uint32)] + \
        [(n, ctypes.c_int32) for n in ("batch", "tokens", "heads", "head_dim", "conv_kernel")] + \
        [(n, ctypes.c_void_p) for n in ("mixed", "z", "beta_logits", "a")] + \
        [(n, ctypes.c_int64) for n in ("mixed_row_stride", "z_row_stride", "b_row_stride",
                                       "a_row_stride")] + \
        [(n, ctypes.c_void_p) for n in ("conv_weight", "a_log", "dt_bias", "norm_weight")] + \
        [("eps", ctypes.c_float), ("has_state", ctypes.c_int32)] + \
        [(n, ctypes.c_void_p) for n in ("conv_state", "state", "out", "workspace")] + \
        [("workspace_bytes", ctypes.c_size_t)]


XLA_LINEAR_MAGIC = 0x4E4C3852  # RXLA_B200_XLA_LINEAR_MAGIC
XLA_ATTENTION_MAGIC = 0x54413852  # RXLA_B200_XLA_ATTENTION_MAGIC


class XlaLinearConfig(ctypes.Structure):
    """rxla_b200_xla_linear_config: the custom call's backend_config bytes."""
    _fields_ = [("magic", ctypes.c_uint32), ("version", ctypes.c_uint32)] + \
        [(n, ctypes.c_int64) for n in ("m", "n", "k", "group_size")] + \
        [(n, ctypes.c_int32) for n in ("x_dtype", "y_dtype", "epilogue", "fused_norm")] + \
        [("eps", ctypes.c_float), ("reserved", ctypes.c_int32)]


class XlaAttentionConfig(ctypes.Structure):
    """rxla_b200_xla_attention_config: the custom call's backend_config bytes."""
    _fields_ = [("magic", ctypes.c_uint32), ("version", ctypes.c_uint32)] + \
        [(n, ctypes.c_int32) for n in ("batch", "q_heads", "kv_heads", "head_dim", "page_size",
                                       "max_pages_per_seq")] + \
        [("num_pages", ctypes.c_int64)] + \
        [(n, ctypes.c_int32) for n in ("max_context", "has_qk_norm", "rotary_dim", "kv_update")] + \
        [("norm_eps", ctypes.c_float), ("scale", ctypes.c_float)]


# name -> (restype, argtypes); every symbol declared in include/rxla_b200.h
_vp, _i32, _i64, _u64, _f32, _sz = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64,
                                    ctypes.c_uint64, ctypes.c_float, ctypes.c_size_t)
SIGNATURES = {
    "rxla_b200_abi_version": (_i32, []),
    "rxla_b200_last_error_message": (ctypes.c_char_p, []),
    "rxla_b200_device_info": (_i32, [_i32, _vp, _vp, _vp]),
    "rxla_b200_device_status": (_i32, [_i32]),
    "rxla_b200_set_wait_timeout": (_i32, [_i64]),
    "rxla_b200_get_wait_timeout": (_i32, [ctypes.POINTER(_i64)]),
    "rxla_b200_bounded_wait_check": (_i32, [_i32, _vp, _u64, _vp]),
    "rxla_b200_w8a16_linear": (_i32, [_vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i32,
                                      _i32, _vp]),
    "rxla_b200_w8a16_linear_workspace_size": (_i32, [_i64, _i64, _i64, _i64, _i32,
                                                     ctypes.POINTER(ctypes.c_size_t)]),
    "rxla_b200_w8a16_linear_ws": (_i32, [_vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i32,
                                         _i32, _vp, _sz, _vp]),
    "rxla_b200_w8a16_norm_linear": (_i32, [_vp, _vp, _f32, _vp, _vp, _i64, _i64, _i64, _i64, _vp,
                                           _i32, _i32, _vp]),
    "rxla_b200_bf16_linear": (_i32, [_vp, _i32, _vp, _i64, _i64, _i64, _vp, _i32, _i32, _vp]),
    "rxla_b200_paged_decode_workspace_size": (_i32, [_i32, _i32, _i32, _i32, _i32,
                                                     ctypes.POINTER(_sz)]),
    "rxla_b200_paged_decode_attention": (_i32, [ctypes.POINTER(PagedDecodeArgs), _vp]),
    "rxla_b200_paged_decode_attention_noalloc": (_i32, [ctypes.POINTER(PagedDecodeArgs), _vp]),
    "rxla_b200_rms_norm_bf16": (_i32, [_vp, _vp, _i64, _i64, _f32, _vp, _vp]),
    "rxla_b200_argmax": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "rxla_b200_w8_embedding": (_i32, [_vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "rxla_b200_sigmoid_gate": (_i32, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _vp]),
    "rxla_b200_gated_delta_workspace_size": (_i32, [_i32, _i32, _i32, _i32, ctypes.POINTER(_sz)]),
    "rxla_b200_gated_delta": (_i32, [ctypes.POINTER(GatedDeltaArgs), _vp]),
    "rxla_b200_decoder_create": (_i32, [ctypes.POINTER(DecoderConfig), _i32, _vp,
                                        ctypes.POINTER(_vp)]),
    "rxla_b200_decoder_destroy": (_i32, [_vp]),
    "rxla_b200_decoder_parameter": (_i32, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp),
                                           ctypes.POINTER(_i64), ctypes.POINTER(_i32)]),
    "rxla_b200_decoder_init_synthetic": (_i32, [_vp, _u64]),
    "rxla_b200_decoder_set_parameter": (_i32, [_vp, ctypes.c_char_p, _vp, _i64]),
    "rxla_b200_decoder_io": (_i32, [_vp, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                    ctypes.POINTER(_vp)]),
    "rxla_b200_decoder_reset": (_i32, [_vp, _vp]),
    "rxla_b200_decoder_step": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp]),
    "rxla_b200_decoder_step_host": (_i32, [_vp, _vp, _i32, _vp, _vp]),
    "rxla_b200_decoder_prefill": (_i32, [_vp, _i32, _vp, _i32, _vp, _vp, _vp]),
    "rxla_b200_safetensors_open": (_i32, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "rxla_b200_safetensors_close": (_i32, [_vp]),
    "rxla_b200_safetensors_count": (_i32, [_vp, ctypes.POINTER(_i32)]),
    "rxla_b200_safetensors_info": (_i32, [_vp, _i32, ctypes.POINTER(ctypes.c_char_p),
                                          ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                                          ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]),
    "rxla_b200_safetensors_find": (_i32, [_vp, ctypes.c_char_p, ctypes.POINTER(_i32)]),
    "rxla_b200_safetensors_metadata": (_i32, [_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p)]),
    "rxla_b200_safetensors_read": (_i32, [_vp, _i32, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_int64, _vp, ctypes.c_int64]),
    "rxla_b200_decoder_load_safetensors": (_i32, [_vp, ctypes.c_char_p, ctypes.c_char_p,
                                                  ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "rxla_b200_decoder_context_lengths": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "rxla_b200_decoder_set_context_lengths": (_i32, [_vp, _vp, _i32, _vp]),
    "rxla_b200_decoder_kv_cache": (_i32, [_vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                          ctypes.POINTER(_i64)]),
    "rxla_b200_xla_w8a16_linear": (None, [_vp, _vp, _vp, _sz]),
    "rxla_b200_xla_w8a16_linear_status": (None, [_vp, _vp, _vp, _sz, _vp]),
    "rxla_b200_xla_paged_decode_attention": (None, [_vp, _vp, _vp, _sz]),
    "rxla_b200_xla_paged_decode_attention_status": (None, [_vp, _vp, _vp, _sz, _vp]),
    "rxla_b200_xla_check_config": (_i32, [ctypes.c_char_p, _vp, _sz]),
    "rxla_b200_comm_unique_id": (_i32, [_vp]),
    "rxla_b200_comm_init": (_i32, [_vp, _i32, _i32, _i32, ctypes.POINTER(_vp)]),
    "rxla_b200_comm_destroy": (_i32, [_vp]),
    "rxla_b200_allreduce": (_i32, [_vp, _vp, _i64, _i32, _vp]),
    "rxla_b200_comm_p2p_enable": (_i32, [_vp, _i64]),
    "rxla_b200_p2p_allreduce_f32": (_i32, [_vp, _vp, _vp, _i64, _vp]),
}

_lib = None


def load() -> ctypes.CDLL:
    """Load librxla_b200.so from the package directory (raises if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RxlaError(FAILED_PRECONDITION,
                        f"{LIB_PATH} is missing: build it with `python -m rxla_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH), mode=ctypes.RTLD_GLOBAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue  # symbol checks live in tests/test_capi.py
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    if status != OK:
        msg = load().rxla_b200_last_error_message()
        raise RxlaError(status, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
