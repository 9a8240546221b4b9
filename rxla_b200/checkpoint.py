"""safetensors checkpoints: the C-ABI reader (rxla_b200_safetensors_*) and a
writer for the same format.

Mirrors crates/rxla-safetensors/src/lib.rs (SafeTensors::open / names / info /
metadata / read_u8 / read_f32) for the W8 checkpoint format that
benchmarks/quantize_qwen3_5_w8.py writes ("rxla-qwen3.5-w8-v1": U8 weights,
F32 "<name>.scale" [rows, cols / G], metadata "format" and "group_size")."""
from __future__ import annotations

import ctypes
import json
import struct

import numpy as np

from . import _lib

_DTYPES = {_lib.F32: np.float32, _lib.BF16: np.uint16, _lib.U8: np.uint8, _lib.I32: np.int32,
           _lib.F16: np.float16}
_NAMES = {np.dtype(np.float32): "F32", np.dtype(np.uint8): "U8", np.dtype(np.int32): "I32",
          np.dtype(np.float16): "F16", np.dtype(np.float64): "F64", np.dtype(np.int64): "I64",
          np.dtype(np.uint16): "U16"}


class SafeTensors:
    """A validated .safetensors file, read through librxla_b200."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _lib.call("rxla_b200_safetensors_open", str(path).encode(), ctypes.byref(h))
        self._h = h

    def close(self):
        if self._h:
            _lib.load().rxla_b200_safetensors_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> list[str]:
        n = ctypes.c_int32()
        _lib.call("rxla_b200_safetensors_count", self._h, ctypes.byref(n))
        return [self._info(i)[0] for i in range(n.value)]

    def _info(self, index: int):
        name, dt, nd = ctypes.c_char_p(), ctypes.c_int32(), ctypes.c_int32()
        shape, nbytes = (ctypes.c_int64 * 8)(), ctypes.c_int64()
        _lib.call("rxla_b200_safetensors_info", self._h, index, ctypes.byref(name),
                  ctypes.byref(dt), ctypes.byref(nd), shape, ctypes.byref(nbytes))
        return name.value.decode(), dt.value, tuple(shape[:nd.value]), nbytes.value

    def _index(self, name: str) -> int:
        i = ctypes.c_int32()
        _lib.call("rxla_b200_safetensors_find", self._h, name.encode(), ctypes.byref(i))
        return i.value

    def info(self, name: str):
        """(dtype code, shape, bytes) of a tensor (dtype -1: no code at the boundary)."""
        return self._info(self._index(name))[1:]

    def metadata(self, key: str) -> str | None:
        v = ctypes.c_char_p()
        rc = _lib.load().rxla_b200_safetensors_metadata(self._h, key.encode(), ctypes.byref(v))
        return v.value.decode() if rc == 0 else None

    def read(self, name: str, rows=None, cols=None) -> np.ndarray:
        """The tensor's exact payload (bf16 as uint16), or the block
        rows=(r0, n) × cols=(c0, n) of it seen as a matrix."""
        i = self._index(name)
        _, dt, shape, nbytes = self._info(i)
        if dt not in _DTYPES:
            raise ValueError(f"{name}: dtype without a boundary code")
        R = shape[0] if len(shape) >= 2 else 1
        C = int(np.prod(shape[1:] if len(shape) >= 2 else shape, dtype=np.int64))
        r0, nr = rows if rows is not None else (0, R)
        c0, nc = cols if cols is not None else (0, C)
        out = np.empty((nr, nc), _DTYPES[dt])
        _lib.call("rxla_b200_safetensors_read", self._h, i, r0, nr, c0, nc,
                  out.ctypes.data_as(ctypes.c_void_p), out.nbytes)
        if rows is None and cols is None:
            return out.reshape(shape)
        return out


def save_file(path: str, tensors: dict, metadata: dict | None = None, bf16: set | None = None):
    """Write a .safetensors file: 8-byte little-endian header length, JSON
    header (dtype, shape, data_offsets per tensor; string "__metadata__"),
    payloads in insertion order.  uint16 arrays named in `bf16` are stored as
    BF16."""
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        dt = "BF16" if bf16 and name in bf16 else _NAMES[a.dtype]
        b = a.tobytes()
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
