"""Host-side mirror of rxla's operator surface for the W8 decode hot path.

Names, argument meaning and error behaviour follow the reference (paths inside
the rxla project); the arithmetic runs in librxla_b200 on the tensors' CUDA
device, with torch used only for device memory and streams.

  QuantizedLinear / quantized_linear   crates/rxla-nn/src/layers.rs:231-298,784-793
  linear (bf16 weight)                 crates/rxla-core/src/nn.rs:286-310
  rms_norm                             crates/rxla-core/src/ops.rs:929-945
  PagedKvCache / decode_attention      crates/rxla-core/src/kv_cache.rs:7-112,
                                       crates/rxla-core/src/attention.rs:83-252,
                                       crates/rxla-core/src/rotary.rs:17-74
  rope_inv_freq                        crates/rxla-models/src/qwen3_5/mod.rs:211-228
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import torch

from . import _lib
from ._lib import RxlaError


class InvalidLayerInput(ValueError):
    """Mirror of rxla_nn::Error::InvalidLayerInput (crates/rxla-nn/src/layers.rs:258-275)."""


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}


def quantized_linear(x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor,
                     group_size: int | None = None, *, out_dtype=torch.bfloat16,
                     epilogue: int = _lib.EPI_STORE, out: torch.Tensor | None = None,
                     workspace: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """W8A16 linear through rxla_b200_w8a16_linear.

    x [..., K] bf16/f32, weight u8 [N, K] (value + 128; [2N, K] = [gate; up] for
    EPI_SWIGLU), scale f32 [N_rows, K / group].  Returns y [..., N] in out_dtype
    (bf16: the bf16 dot; f32: the unrounded fp32 dot), or accumulates into the
    f32 `out` for EPI_RESIDUAL_ADD.  With `workspace` (a zero-filled u8 device
    tensor of at least linear_workspace_size bytes) the call goes through
    rxla_b200_w8a16_linear_ws, whose tensor-core GEMM may split K.
    """
    if x.dtype not in _DT or weight.dtype != torch.uint8 or scale.dtype != torch.float32:
        raise InvalidLayerInput("QuantizedLinear needs bf16/f32 x, u8 weight, f32 scale")
    if x.dim() == 0:
        raise InvalidLayerInput("QuantizedLinear needs an input with rank at least one")
    k = x.shape[-1]
    rows = weight.shape[0]
    if weight.dim() != 2 or weight.shape[1] != k:
        raise InvalidLayerInput("weight must be [out_features, in_features]")
    group = k if group_size is None else int(group_size)
    if group <= 0 or k % group != 0:
        raise InvalidLayerInput("positive widths and a group size dividing the input width")
    if scale.numel() != rows * (k // group):
        raise InvalidLayerInput("scale must be [out_features, in_features / group_size]")
    n = rows // 2 if epilogue == _lib.EPI_SWIGLU else rows
    lead = x.shape[:-1]
    m = int(np.prod(lead)) if len(lead) else 1
    x2 = x.reshape(m, k)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    if out is None:
        if epilogue == _lib.EPI_RESIDUAL_ADD:
            raise InvalidLayerInput("the residual epilogue needs `out` (f32) to add into")
        out = torch.empty(*lead, n, dtype=out_dtype, device=x.device)
    if workspace is not None:
        _lib.call("rxla_b200_w8a16_linear_ws", _ptr(x2), _DT[x.dtype], _ptr(weight),
                  _ptr(scale), group, m, n, k, _ptr(out), _DT[out.dtype], epilogue,
                  _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(stream))
        return out
    _lib.call("rxla_b200_w8a16_linear", _ptr(x2), _DT[x.dtype], _ptr(weight),
              _ptr(scale), group, m, n, k, _ptr(out), _DT[out.dtype], epilogue, _stream(stream))
    return out


def linear_workspace_size(m: int, n: int, k: int, group_size: int | None = None,
                          epilogue: int = _lib.EPI_STORE) -> int:
    """Bytes of the split-K workspace of quantized_linear for an [m, k] x
    [n, k] call on the current device (rxla_b200_w8a16_linear_workspace_size;
    0: this shape does not split)."""
    size = ctypes.c_size_t(0)
    _lib.call("rxla_b200_w8a16_linear_workspace_size", int(m), int(n), int(k),
              int(k if group_size is None else group_size), int(epilogue), ctypes.byref(size))
    return int(size.value)


def quantized_norm_linear(h: torch.Tensor, norm_weight: torch.Tensor, epsilon: float,
                          weight: torch.Tensor, scale: torch.Tensor,
                          group_size: int | None = None, *, out_dtype=torch.bfloat16,
                          epilogue: int = _lib.EPI_STORE, out: torch.Tensor | None = None,
                          stream=None) -> torch.Tensor:
    """QuantizedLinear of bf16(rms_norm(h) * norm_weight), the norm fused into
    the linear's prologue (rxla_b200_w8a16_norm_linear): h f32 [..., K], the
    other arguments as for quantized_linear."""
    if h.dtype != torch.float32 or norm_weight.dtype != torch.float32:
        raise InvalidLayerInput("the fused norm needs an F32 h and norm weight")
    if not (epsilon > 0 and math.isfinite(epsilon)):
        raise InvalidLayerInput("RMSNorm requires a finite positive epsilon")
    k = h.shape[-1]
    rows = weight.shape[0]
    if weight.dim() != 2 or weight.shape[1] != k or norm_weight.numel() != k:
        raise InvalidLayerInput("weight must be [out_features, in_features], norm [in_features]")
    group = k if group_size is None else int(group_size)
    if group <= 0 or k % group != 0 or scale.numel() != rows * (k // group):
        raise InvalidLayerInput("scale must be [out_features, in_features / group_size]")
    n = rows // 2 if epilogue == _lib.EPI_SWIGLU else rows
    lead = h.shape[:-1]
    m = int(np.prod(lead)) if len(lead) else 1
    h2 = h.reshape(m, k).contiguous()
    if out is None:
        if epilogue == _lib.EPI_RESIDUAL_ADD:
            raise InvalidLayerInput("the residual epilogue needs `out` (f32) to add into")
        out = torch.empty(*lead, n, dtype=out_dtype, device=h.device)
    _lib.call("rxla_b200_w8a16_norm_linear", _ptr(h2), _ptr(norm_weight), ctypes.c_float(epsilon),
              _ptr(weight), _ptr(scale), group, m, n, k, _ptr(out), _DT[out.dtype], epilogue,
              _stream(stream))
    return out


class QuantizedLinear:
    """rxla_nn::QuantizedLinear::new(out_features, group_size) (layers.rs:231-256).

    `apply(params, name, input)` reads `{name}.weight` (u8 [out, in]) and
    `{name}.scale` (f32 [out, in/group]) from `params` and returns the F32
    boundary value of the bf16-compute layer, as apply_quantized_linear does
    with layer compute dtype BF16 (layers.rs:289-297).
    """

    def __init__(self, out_features: int, group_size: int):
        self.out_features = int(out_features)
        self.group_size = int(group_size)

    def apply(self, params, name: str, input: torch.Tensor) -> torch.Tensor:
        if input.dtype != torch.float32 or input.dim() == 0:
            raise InvalidLayerInput("an F32 input with rank at least one")
        k = input.shape[-1]
        if (self.out_features <= 0 or self.group_size <= 0 or k <= 0
                or k % self.group_size != 0):
            raise InvalidLayerInput("positive widths and a group size dividing the input width")
        w = params[f"{name}.weight"]
        s = params[f"{name}.scale"]
        if tuple(w.shape) != (self.out_features, k) or w.dtype != torch.uint8:
            raise InvalidLayerInput(f"{name}.weight must be U8 [{self.out_features}, {k}]")
        y = quantized_linear(input, w, s, self.group_size, out_dtype=torch.bfloat16)
        return y.float()


def bf16_linear(x: torch.Tensor, weight: torch.Tensor, *, out_dtype=torch.float32,
                epilogue: int = _lib.EPI_STORE, out=None, stream=None) -> torch.Tensor:
    """y = bf16(x) · weightᵀ with a bf16 weight [N, K] (rxla_b200_bf16_linear)."""
    k = x.shape[-1]
    n = weight.shape[0]
    lead = x.shape[:-1]
    m = int(np.prod(lead)) if len(lead) else 1
    x2 = x.reshape(m, k).contiguous()
    if out is None:
        out = torch.empty(*lead, n, dtype=out_dtype, device=x.device)
    _lib.call("rxla_b200_bf16_linear", _ptr(x2), _DT[x.dtype], _ptr(weight), m, n, k,
              _ptr(out), _DT[out.dtype], epilogue, _stream(stream))
    return out


def rms_norm_bf16(x: torch.Tensor, weight: torch.Tensor, epsilon: float,
                  out=None, stream=None) -> torch.Tensor:
    """bf16(x * rsqrt(mean(x²) + eps) * w) over the last axis (ops.rs:929-945)."""
    if not (epsilon > 0 and math.isfinite(epsilon)):
        raise InvalidLayerInput("RMSNorm requires a finite positive epsilon")
    width = x.shape[-1]
    rows = x.numel() // width
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.call("rxla_b200_rms_norm_bf16", _ptr(x), _ptr(weight), rows, width,
              ctypes.c_float(epsilon), _ptr(out), _stream(stream))
    return out


def argmax(logits: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    v = logits.shape[-1]
    rows = logits.numel() // v
    if out is None:
        out = torch.empty(logits.shape[:-1], dtype=torch.int32, device=logits.device)
    _lib.call("rxla_b200_argmax", _ptr(logits), rows, v, _ptr(out), _stream(stream))
    return out


def rope_inv_freq(theta: float, rotary_dim: int) -> np.ndarray:
    """θ^(-2i/rotary_dim) in f32, as qwen3_5/mod.rs:213-222 computes it on the host."""
    i = np.arange(rotary_dim // 2, dtype=np.float32)
    return np.power(np.float32(theta), (np.float32(-2.0) * i) / np.float32(rotary_dim),
                    dtype=np.float32)


class PagedKvCache:
    """Paged bf16 K/V cache on the device: [num_pages, kv_heads, 16, head_dim] each.

    The device-side counterpart of rxla_core::KvCache (crates/rxla-core/src/kv_cache.rs:7-112)
    for decode: `page_table[b, i]` is the i-th page of sequence b, `ctx_lens[b]` the
    number of cached tokens, i.e. the position of the next token.
    """

    PAGE = 16

    def __init__(self, *, batch: int, kv_heads: int, head_dim: int, max_context: int,
                 num_pages: int | None = None, device="cuda"):
        self.batch, self.kv_heads, self.head_dim = batch, kv_heads, head_dim
        self.max_context = max_context
        self.max_pages = (max_context + self.PAGE - 1) // self.PAGE
        self.num_pages = num_pages or batch * self.max_pages
        shape = (self.num_pages, kv_heads, self.PAGE, head_dim)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.page_table = torch.arange(batch * self.max_pages, dtype=torch.int32,
                                       device=device).reshape(batch, self.max_pages) % self.num_pages
        self.ctx_lens = torch.zeros(batch, dtype=torch.int32, device=device)
        self.pages_per_seq = None


def paged_decode_workspace_size(batch, q_heads, kv_heads, head_dim, max_context) -> int:
    n = ctypes.c_size_t()
    _lib.call("rxla_b200_paged_decode_workspace_size", batch, q_heads, kv_heads, head_dim,
              max_context, ctypes.byref(n))
    return int(n.value)


def paged_decode_attention(q, k_new, v_new, cache: PagedKvCache, *, q_heads: int,
                           q_norm_weight=None, k_norm_weight=None, eps: float = 1e-6,
                           inv_freq=None, rotary_dim: int = 0, scale: float = 0.0,
                           kv_update: int = _lib.KV_CLAMP, advance_ctx: bool = False,
                           accepted=None, out=None, workspace=None, stream=None):
    """One decode step of GQA over the paged cache (rxla_b200_paged_decode_attention).

    q [batch, q_heads*D], k_new / v_new [batch, kv_heads*D] (bf16 views with a row
    stride, e.g. slices of a fused QKV output).  Returns out [batch, q_heads*D] bf16.
    """
    batch, hkv, d = cache.batch, cache.kv_heads, cache.head_dim
    if out is None:
        out = torch.empty(batch, q_heads * d, dtype=torch.bfloat16, device=q.device)
    if workspace is None:
        workspace = torch.zeros(paged_decode_workspace_size(batch, q_heads, hkv, d,
                                                            cache.max_context),
                                dtype=torch.uint8, device=q.device)
    a = _lib.PagedDecodeArgs()
    a.struct_size = ctypes.sizeof(_lib.PagedDecodeArgs)
    a.batch, a.q_heads, a.kv_heads, a.head_dim = batch, q_heads, hkv, d
    a.q, a.k_new, a.v_new = q.data_ptr(), k_new.data_ptr(), v_new.data_ptr()
    a.q_row_stride = q.stride(0)
    a.kv_row_stride = k_new.stride(0)
    if k_new.stride(0) != v_new.stride(0):
        raise InvalidLayerInput("k_new and v_new must share a row stride")
    a.q_norm_weight = 0 if q_norm_weight is None else q_norm_weight.data_ptr()
    a.k_norm_weight = 0 if k_norm_weight is None else k_norm_weight.data_ptr()
    a.norm_eps = eps
    a.inv_freq = 0 if inv_freq is None else inv_freq.data_ptr()
    a.rotary_dim = rotary_dim
    a.scale = scale
    a.k_pages, a.v_pages = cache.k.data_ptr(), cache.v.data_ptr()
    a.num_pages = cache.num_pages
    a.page_size = PagedKvCache.PAGE
    a.max_pages_per_seq = cache.page_table.shape[1]
    a.page_table = cache.page_table.data_ptr()
    a.pages_per_seq = 0 if cache.pages_per_seq is None else cache.pages_per_seq.data_ptr()
    a.ctx_lens = cache.ctx_lens.data_ptr()
    a.kv_update = kv_update
    a.advance_ctx = int(advance_ctx)
    a.accepted = 0 if accepted is None else accepted.data_ptr()
    a.out = out.data_ptr()
    a.workspace = workspace.data_ptr()
    a.workspace_bytes = workspace.numel()
    a.max_context = cache.max_context
    _lib.call("rxla_b200_paged_decode_attention", ctypes.byref(a), _stream(stream))
    return out


def w8_embedding(ids: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor, group_size: int,
                 stream=None) -> torch.Tensor:
    """The W8 token embedding (qwen3_5/mod.rs:134-155) through
    rxla_b200_w8_embedding: ids int32 [...] on the device, weight u8 [vocab,
    hidden], scale f32 [vocab, hidden / group_size]; returns f32 [..., hidden]."""
    if ids.dtype != torch.int32 or weight.dtype != torch.uint8 or scale.dtype != torch.float32:
        raise InvalidLayerInput("embedding needs int32 ids, u8 weight, f32 scale")
    vocab, hidden = weight.shape
    if hidden % group_size or scale.numel() != vocab * (hidden // group_size):
        raise InvalidLayerInput("scale must be [vocab, hidden / group_size]")
    ids_c = ids.contiguous()
    out = torch.empty(*ids.shape, hidden, dtype=torch.float32, device=weight.device)
    _lib.call("rxla_b200_w8_embedding", _ptr(ids_c), ids_c.numel(), _ptr(weight), _ptr(scale),
              vocab, hidden, group_size, _ptr(out), _stream(stream))
    return out


def sigmoid_gate(x: torch.Tensor, gate: torch.Tensor, out: torch.Tensor | None = None,
                 stream=None) -> torch.Tensor:
    """bf16(x · sigmoid(gate)) through rxla_b200_sigmoid_gate: Qwen3.5's
    attention output gate (crates/rxla-models/src/qwen3_5/layers.rs:50-55,
    94-95).  x, gate: bf16 [rows, width] views with unit inner stride."""
    if x.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16 or x.shape != gate.shape \
            or x.dim() != 2 or x.stride(1) != 1 or gate.stride(1) != 1:
        raise InvalidLayerInput("sigmoid_gate needs bf16 [rows, width] x and gate")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.call("rxla_b200_sigmoid_gate", _ptr(x), x.stride(0), _ptr(gate), gate.stride(0),
              x.shape[0], x.shape[1], _ptr(out), out.stride(0), _stream(stream))
    return out


def device_status(reset: bool = False) -> int:
    return int(_lib.load().rxla_b200_device_status(int(reset)))


__all__ = ["QuantizedLinear", "quantized_linear", "bf16_linear", "rms_norm_bf16", "argmax",
           "rope_inv_freq", "device_status", "InvalidLayerInput", "RxlaError", "PagedKvCache",
           "paged_decode_attention", "paged_decode_workspace_size", "sigmoid_gate",
           "w8_embedding"]
