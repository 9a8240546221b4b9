"""CPU oracle for the W8 decode hot path — TEST INFRASTRUCTURE ONLY.

A C restatement (``rxla_oracle.c``) of rxla's reference semantics, loaded here
through ctypes with numpy conveniences.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
may import this package, and only as the checker or the timed CPU baseline;
the product library never routes through it.

Reference functions restated (paths inside the rxla project):
  quantize_w8      benchmarks/quantize_qwen3_5_w8.py:33-44
  w8_linear        crates/rxla-nn/src/layers.rs:257-298
  rms_norm         crates/rxla-core/src/ops.rs:929-945
  rope_*           crates/rxla-core/src/rotary.rs:17-74, qwen3_5/mod.rs:211-228
  gqa_attention    crates/rxla-core/src/attention.rs:83-252
  causal_mask      crates/rxla-core/src/attention.rs:14-32
  kv_update        crates/rxla-core/src/kv_cache.rs:53-112
  Decoder          crates/rxla-models/src/qwen3_5/{mod.rs,layers.rs} (Qwen3 form)
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "librxla_oracle.so"
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


def build() -> Path:
    """Compile the oracle with gcc (oracle/build_oracle.sh)."""
    subprocess.run(["bash", str(_HERE / "build_oracle.sh")], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    L = ctypes.CDLL(str(_LIB_PATH))
    sig = {
        "oracle_bf16_round": (_f32, [_f32]),
        "oracle_f32_to_bf16": (ctypes.c_uint16, [_f32]),
        "oracle_splitmix64": (ctypes.c_uint64, [ctypes.c_uint64]),
        "oracle_fill_normal": (None, [_f32p, _i64, ctypes.c_uint64, _f32, _f32]),
        "oracle_fill_uniform": (None, [_f32p, _i64, ctypes.c_uint64, _f32, _f32]),
        "oracle_fill_randint": (None, [_i32p, _i64, ctypes.c_uint64, _i32, _i32]),
        "oracle_quantize_w8": (None, [_f32p, _i64, _i64, _i64, _u8p, _f32p]),
        "oracle_w8_linear": (None, [_f32p, _i64, _i64, _u8p, _f32p, _i64, _i64, _i32, _f32p]),
        "oracle_linear": (None, [_f32p, _i64, _i64, _f32p, _i64, _i32, _f32p]),
        "oracle_rms_norm": (None, [_f32p, _i64, _i64, _f32p, _f32, _f32p]),
        "oracle_rope_inv_freq": (None, [_f32, _i32, _f32p]),
        "oracle_rope_split_half": (None, [_f32p, _i64, _i64, _i32, _i32p, _f32p]),
        "oracle_rope_cos_sin": (None, [_f32p, _i64, _i64, _f32p, _f32p, _i32, _f32p]),
        "oracle_gqa_attention": (None, [_f32p, _f32p, _f32p, _vp, _i64, _i64, _i64, _i64,
                                        _i64, _i64, _i64, _i64, _i64, _f32, _f32p]),
        "oracle_causal_mask": (None, [_i32p, _i64, _i32p, _i64, _f32p]),
        "oracle_kv_update": (_i32, [_f32p, _f32p, _i64p, _f32p, _f32p, _i64p, _i32, _i32p,
                                    _i32]),
        "oracle_paged_decode_attention": (None, [
            _i32, _i32, _i32, _i32, _f32p, _f32p, _f32p, _i64, _i64, _vp, _vp, _f32, _vp,
            _i32, _f32, _u16p, _u16p, _i32, _i32, _i32p, _vp, _i32p, _i32, _i32, _vp, _f32p]),
        "oracle_decoder_create": (_vp, [_vp]),
        "oracle_decoder_destroy": (None, [_vp]),
        "oracle_decoder_parameter": (_i64, [_vp, ctypes.c_char_p, ctypes.POINTER(_vp),
                                            ctypes.POINTER(_i32)]),
        "oracle_decoder_init_synthetic": (None, [_vp, ctypes.c_uint64]),
        "oracle_decoder_reset": (None, [_vp]),
        "oracle_decoder_step": (None, [_vp, _i32p, _i32, _f32p, _i32p]),
        "oracle_decoder_forward": (None, [_vp, _i32p, _i32, _f32p, _i32p]),
        "oracle_decoder_context": (_i32, [_vp, _i32]),
        "oracle_decoder_kv": (None, [_vp, _i32, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
        "oracle_decoder_prefill": (_i32, [_vp, _i32, _i32p, _i32, _f32p, _i32p]),
        "oracle_decoder_set_context": (_i32, [_vp, _i32, _i32]),
        "oracle_set_num_threads": (None, [_i32]),
        "oracle_num_threads": (_i32, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- numerics

def bf16_round(x) -> np.ndarray:
    """Round f32 values to the nearest-even bfloat16 (returned as f32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, (u >> 16) | 0x40, r)
    return (r.astype(np.uint32) << 16).view(np.float32).reshape(x.shape)


def f32_to_bf16_bits(x) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- data

def normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(int(n), np.float32)
    lib().oracle_fill_normal(out, int(n), seed, mean, std)
    return out


def uniform(n: int, seed: int, lo: float, hi: float) -> np.ndarray:
    out = np.empty(int(n), np.float32)
    lib().oracle_fill_uniform(out, int(n), seed, lo, hi)
    return out


def randint(n: int, seed: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(int(n), np.int32)
    lib().oracle_fill_randint(out, int(n), seed, lo, hi)
    return out


def linear_sweep_case(m: int, n: int, k: int, seed: int):
    """Config 2 inputs: x ~ bf16 N(0,1) [m,k]; q ~ U{-127..127} stored +128; scale ~ U[1e-3,1e-2]."""
    x = bf16_round(normal(m * k, seed * 4 + 0).reshape(m, k))
    q = randint(n * k, seed * 4 + 1, -127, 128).reshape(n, k)
    w = (q + 128).astype(np.uint8)
    scale = uniform(n, seed * 4 + 2, 1e-3, 1e-2).reshape(n, 1)
    return x, w, scale


# ---------------------------------------------------------------- ops

def quantize_w8(w: np.ndarray, group: int):
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.uint8)
    s = np.empty((n, k // group), np.float32)
    lib().oracle_quantize_w8(w, n, k, group, q, s)
    return q, s


def w8_linear(x, w, scale, group: int | None = None, mode: int = 1) -> np.ndarray:
    """QuantizedLinear; mode 0 F32 compute, 1 BF16 compute (reference), 2 exact factored."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    scale = np.ascontiguousarray(scale, np.float32)
    lead = x.shape[:-1]
    k = x.shape[-1]
    m = int(np.prod(lead)) if lead else 1
    n = w.shape[0]
    group = k if group is None else group
    y = np.empty((m, n), np.float32)
    lib().oracle_w8_linear(x.reshape(m, k), m, k, w, scale.reshape(-1), n, group, mode, y)
    return y.reshape(*lead, n)


def linear(x, w, bf16: bool = False) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    lead = x.shape[:-1]
    k = x.shape[-1]
    m = int(np.prod(lead)) if lead else 1
    y = np.empty((m, w.shape[0]), np.float32)
    lib().oracle_linear(x.reshape(m, k), m, k, w, w.shape[0], int(bf16), y)
    return y.reshape(*lead, w.shape[0])


def rms_norm(x, w, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    rows = x.size // x.shape[-1]
    y = np.empty_like(x)
    lib().oracle_rms_norm(x, rows, x.shape[-1], w, eps, y)
    return y


def rope_inv_freq(theta: float, rotary_dim: int) -> np.ndarray:
    out = np.empty(rotary_dim // 2, np.float32)
    lib().oracle_rope_inv_freq(theta, rotary_dim, out)
    return out


def rope_split_half(x, positions, inv_freq, rotary_dim: int | None = None) -> np.ndarray:
    x = np.array(x, np.float32, copy=True, order="C")
    width = x.shape[-1]
    rows = x.size // width
    pos = np.ascontiguousarray(np.broadcast_to(np.asarray(positions, np.int32), (rows,)))
    lib().oracle_rope_split_half(x, rows, width, rotary_dim or width, pos,
                                 np.ascontiguousarray(inv_freq, np.float32))
    return x


def rope_cos_sin(x, cos_t, sin_t, layout: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    width = x.shape[-1]
    rows = x.size // width
    c = np.ascontiguousarray(np.broadcast_to(cos_t, (rows, width // 2)), np.float32)
    s = np.ascontiguousarray(np.broadcast_to(sin_t, (rows, width // 2)), np.float32)
    y = np.empty_like(x)
    lib().oracle_rope_cos_sin(x, rows, width, c, s, layout, y)
    return y


def causal_mask(qpos, kpos) -> np.ndarray:
    qpos = np.ascontiguousarray(qpos, np.int32)
    kpos = np.ascontiguousarray(kpos, np.int32)
    m = np.empty((qpos.size, kpos.size), np.float32)
    lib().oracle_causal_mask(qpos, qpos.size, kpos, kpos.size, m)
    return m


def gqa_attention(q, k, v, mask=None, scale: float | None = None) -> np.ndarray:
    """q [B,Hq,T,D], k [B,Hkv,S,D], v [B,Hkv,S,Dv]; mask broadcastable to [B,Hq,T,S]."""
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    B, hq, T, D = q.shape
    hkv, S, Dv = k.shape[1], k.shape[2], v.shape[3]
    scale = float(1.0 / np.sqrt(np.float32(D))) if scale is None else scale
    mptr, mb, mh = None, 0, 0
    if mask is not None:
        full = np.ascontiguousarray(np.broadcast_to(mask, (B, hq, T, S)), np.float32)
        mask = full
        mptr, mb, mh = _ptr(full), hq * T * S, T * S
    out = np.empty((B, hq, T, Dv), np.float32)
    lib().oracle_gqa_attention(q, k, v, mptr, mb, mh, B, hq, hkv, T, S, D, Dv,
                               np.float32(scale), out)
    return out


def kv_update(k_cache, v_cache, k_upd, v_upd, starts, checked: bool = False) -> int:
    """In-place paired dynamic_update_slice; returns accepted (1/0)."""
    shape = np.asarray(k_cache.shape, np.int64)
    ushape = np.asarray(k_upd.shape, np.int64)
    return lib().oracle_kv_update(k_cache, v_cache, shape, np.ascontiguousarray(k_upd, np.float32),
                                  np.ascontiguousarray(v_upd, np.float32), ushape,
                                  len(k_cache.shape), np.asarray(starts, np.int32), int(checked))


def paged_decode_attention(*, q, k_new, v_new, k_pages, v_pages, page_table, ctx_lens,
                           hq, hkv, d, q_norm_w=None, k_norm_w=None, eps=1e-6,
                           inv_freq=None, rotary_dim=0, scale=0.0, pages_per_seq=None,
                           kv_update=0, advance_ctx=False, page_size=16):
    """Restated contract of rxla_b200_paged_decode_attention; mutates pages / ctx_lens."""
    batch = ctx_lens.shape[0]
    q = np.ascontiguousarray(q, np.float32).reshape(batch, -1)
    k_new = np.ascontiguousarray(k_new, np.float32).reshape(batch, -1)
    v_new = np.ascontiguousarray(v_new, np.float32).reshape(batch, -1)
    out = np.zeros((batch, hq * d), np.float32)
    accepted = np.zeros(batch, np.int32)
    qn = None if q_norm_w is None else np.ascontiguousarray(q_norm_w, np.float32)
    kn = None if k_norm_w is None else np.ascontiguousarray(k_norm_w, np.float32)
    inv = None if inv_freq is None else np.ascontiguousarray(inv_freq, np.float32)
    pps = None if pages_per_seq is None else np.ascontiguousarray(pages_per_seq, np.int32)
    lib().oracle_paged_decode_attention(
        batch, hq, hkv, d, q, k_new, v_new, q.shape[1], k_new.shape[1], _ptr(qn), _ptr(kn),
        eps, _ptr(inv), rotary_dim if inv is not None else 0, scale, k_pages, v_pages,
        page_size, page_table.shape[1], page_table, _ptr(pps), ctx_lens, kv_update,
        int(advance_ctx), _ptr(accepted), out)
    return out, accepted


class _DecCfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("layers", "hidden", "q_heads", "kv_heads", "head_dim", "intermediate", "vocab")] + \
               [("rms_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)] + \
               [(n, ctypes.c_int32) for n in
                ("embedding_bf16", "group_size", "max_batch", "max_context", "linear_mode")]


class Decoder:
    """The Qwen3-style W8 decoder restated on the CPU (greedy, dense bf16 cache)."""

    def __init__(self, *, layers, hidden, q_heads, kv_heads, head_dim, intermediate, vocab,
                 rms_eps=1e-6, rope_theta=1e6, embedding_bf16=False, group_size=0,
                 max_batch=1, max_context=256, linear_mode=1):
        """linear_mode 1: the reference's QuantizedLinear rounding (bf16(W_deq)),
        f64 sums, and the reference's F32 tied head (f32 hidden · f32 W_deq);
        3: exact q with the scale on the fp32 dot;
        4: the noise-floor model of a bf16-activation, fp32-accumulation
        implementation: mode 1's rounding points with fp32 running sums, and
        the tied head on bf16 operands with an fp32 sum."""
        self.cfg = _DecCfg(layers, hidden, q_heads, kv_heads, head_dim, intermediate, vocab,
                           rms_eps, rope_theta, int(embedding_bf16), group_size, max_batch,
                           max_context, linear_mode)
        self.vocab = vocab
        self._h = lib().oracle_decoder_create(ctypes.byref(self.cfg))

    def close(self):
        if self._h:
            lib().oracle_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def parameter(self, name: str) -> np.ndarray:
        ptr = ctypes.c_void_p()
        dt = ctypes.c_int32()
        nbytes = lib().oracle_decoder_parameter(self._h, name.encode(), ctypes.byref(ptr),
                                                ctypes.byref(dt))
        if nbytes < 0:
            raise KeyError(name)
        np_dt = {0: np.float32, 1: np.uint16, 2: np.uint8}[dt.value]
        count = nbytes // np.dtype(np_dt).itemsize
        buf = (ctypes.c_char * nbytes).from_address(ptr.value)
        return np.frombuffer(buf, dtype=np_dt, count=count)

    def init_synthetic(self, seed: int):
        lib().oracle_decoder_init_synthetic(self._h, seed)

    def kv_cache(self, layer: int):
        """Dense bf16 K/V of one layer: [max_batch, kv_heads, max_context, head_dim] each."""
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        lib().oracle_decoder_kv(self._h, layer, ctypes.byref(k), ctypes.byref(v))
        c = self.cfg
        n = c.max_batch * c.kv_heads * c.max_context * c.head_dim
        shape = (c.max_batch, c.kv_heads, c.max_context, c.head_dim)
        kk = np.frombuffer((ctypes.c_uint16 * n).from_address(k.value), np.uint16).reshape(shape)
        vv = np.frombuffer((ctypes.c_uint16 * n).from_address(v.value), np.uint16).reshape(shape)
        return kk, vv

    def reset(self):
        lib().oracle_decoder_reset(self._h)

    def forward(self, prompt):
        """Full-sequence causal forward of one prompt from position 0 (the
        reference's prompt path, qwen3_5/mod.rs:199-260): the last row's
        logits [vocab] and greedy token.  The decoder's state is untouched."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        logits = np.empty(self.vocab, np.float32)
        nxt = np.empty(1, np.int32)
        lib().oracle_decoder_forward(self._h, prompt, prompt.shape[0], logits, nxt)
        return logits, int(nxt[0])

    def prefill(self, seq: int, prompt):
        """The full-sequence forward of `prompt` for the empty sequence `seq`
        that also stores the prompt rows' K/V and sets its context to the
        prompt length (decode steps then continue after the prompt; the same
        state as stepping the prompt token by token).  Returns the last row's
        logits [vocab] and greedy token."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        logits = np.empty(self.vocab, np.float32)
        nxt = np.empty(1, np.int32)
        if lib().oracle_decoder_prefill(self._h, seq, prompt, prompt.shape[0], logits, nxt) != 0:
            raise ValueError("oracle prefill: sequence not empty or prompt longer than max_context")
        return logits, int(nxt[0])

    def set_context(self, seq: int, ctx: int):
        """Set sequence `seq`'s context length directly (cached values stay as
        they are), e.g. to time a step at a long context."""
        if lib().oracle_decoder_set_context(self._h, seq, ctx) != 0:
            raise ValueError("oracle set_context: out of range")

    def step(self, tokens):
        tokens = np.ascontiguousarray(tokens, np.int32)
        b = tokens.shape[0]
        logits = np.empty((b, self.vocab), np.float32)
        nxt = np.empty(b, np.int32)
        lib().oracle_decoder_step(self._h, tokens, b, logits, nxt)
        return logits, nxt


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    """OpenMP threads of the oracle from now on (overrides OMP_NUM_THREADS,
    which torchrun sets to 1)."""
    lib().oracle_set_num_threads(int(n))


def library_path() -> str:
    return str(_LIB_PATH)


__all__ = [n for n in dir() if not n.startswith("_")]
os.environ.setdefault("OMP_PROC_BIND", "false")
