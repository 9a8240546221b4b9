"""safetensors reader (rxla_b200_safetensors_*): CPU-only.

The cases restate crates/rxla-safetensors/tests/checkpoint.rs: exact U8 and
integer payload bits, float formats, scalars and empty tensors, metadata, and
the malformed files that SafeTensors::new rejects (lib.rs:147-177)."""
import json
import struct

import numpy as np
import pytest

from rxla_b200 import _lib
from rxla_b200.checkpoint import SafeTensors, save_file


def _raw(path, header: str, payload: bytes, hlen=None):
    h = header.encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h) if hlen is None else hlen))
        f.write(h)
        f.write(payload)


def test_u8_and_integer_payloads_keep_their_bits(tmp_path):
    w = np.array([[0, 1, 127], [128, 254, 255]], np.uint8)
    idx = np.array([[-2**31, -16777217, -1], [0, 16777217, 2**31 - 1]], np.int32)
    p = tmp_path / "a.safetensors"
    save_file(p, {"weight": w, "indices": idx, "count": np.array(16777217, np.int32),
                  "empty": np.zeros((0, 2), np.int32), "i64": np.array(1, np.int64)})
    with SafeTensors(p) as f:
        assert f.names() == ["weight", "indices", "count", "empty", "i64"]
        assert f.info("weight") == (_lib.U8, (2, 3), 6)
        np.testing.assert_array_equal(f.read("weight"), w)
        np.testing.assert_array_equal(f.read("indices"), idx)
        assert f.read("count").item() == 16777217
        assert f.read("empty").shape == (0, 2)
        assert f.info("i64")[0] == -1  # no boundary code: listed, not read
        with pytest.raises(Exception):
            f.read("i64")
        with pytest.raises(Exception):
            f.read("missing")


def test_float_formats_scalars_blocks_and_metadata(tmp_path):
    vals = np.array([-2.0, 0.0, 1.5, np.inf, np.nan], np.float32)
    bf = (vals.view(np.uint32) >> 16).astype(np.uint16)
    scale = np.arange(12, dtype=np.float32).reshape(6, 2)
    p = tmp_path / "b.safetensors"
    save_file(p, {"f32": vals, "f16": vals.astype(np.float16), "bf16": bf,
                  "scalar": np.array(42.0, np.float32), "w.scale": scale},
              metadata={"format": "rxla-qwen3.5-w8-v1", "group_size": 128}, bf16={"bf16"})
    with SafeTensors(p) as f:
        assert f.metadata("format") == "rxla-qwen3.5-w8-v1"
        assert f.metadata("group_size") == "128"
        assert f.metadata("absent") is None
        np.testing.assert_array_equal(f.read("f32")[:4], vals[:4])
        assert np.isnan(f.read("f32")[4])
        assert f.info("f16")[0] == _lib.F16
        np.testing.assert_array_equal(f.read("f16").astype(np.float32)[:4], vals[:4])
        assert f.info("bf16")[0] == _lib.BF16
        np.testing.assert_array_equal(f.read("bf16"), bf)
        assert f.read("scalar").item() == 42.0
        # a block of rows and columns (what a tensor-parallel rank reads)
        np.testing.assert_array_equal(f.read("w.scale", rows=(2, 3), cols=(1, 1)), scale[2:5, 1:2])
        np.testing.assert_array_equal(f.read("w.scale", rows=(1, 4)), scale[1:5])
        with pytest.raises(Exception):
            f.read("w.scale", rows=(4, 3))  # past the last row


@pytest.mark.parametrize("data", [b"", b"\0" * 4, struct.pack("<Q", 2**64 - 1),
                                  struct.pack("<Q", 8) + b"{}"])
def test_malformed_prefix_is_rejected(tmp_path, data):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(data)
    with pytest.raises(Exception):
        SafeTensors(p)


@pytest.mark.parametrize("header,payload", [
    ('{"x":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', 4),   # bytes != shape
    ('{"x":{"dtype":"F32","shape":[1],"data_offsets":[1,5]}}', 5),   # gap before the first
    ('{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', 3),   # payload too short
    ('{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4]}}', 5),   # payload too long
    ('{"x":{"dtype":"F32","shape":[1],"data_offsets":[0,4]},'
     '"y":{"dtype":"F32","shape":[1],"data_offsets":[2,6]}}', 6),    # overlap
    ('{"x":{"dtype":"Q7","shape":[1],"data_offsets":[0,1]}}', 1),    # unknown dtype
    ('{"x":{"dtype":"U8","shape":[1],"data_offsets":[0,1]},'
     '"x":{"dtype":"U8","shape":[1],"data_offsets":[1,2]}}', 2),     # duplicate name
    ('{"x":{"dtype":"U8","shape":[1]}}', 1),                         # no data_offsets
    ('{"__metadata__":{"a":1}}', 0),                                 # non-string metadata
    ('["x"]', 0),                                                    # not an object
])
def test_malformed_header_is_rejected(tmp_path, header, payload):
    p = tmp_path / "bad.safetensors"
    _raw(p, header, b"\0" * payload)
    with pytest.raises(Exception):
        SafeTensors(p)


def test_header_padding_and_escapes(tmp_path):
    hdr = json.dumps({"__metadata__": {"note": "tab\tquote\" é"},
                      "a/b.c": {"dtype": "U8", "shape": [2], "data_offsets": [0, 2]}})
    p = tmp_path / "c.safetensors"
    _raw(p, hdr + "    ", b"\x07\x09")
    with SafeTensors(p) as f:
        assert f.names() == ["a/b.c"]
        assert f.metadata("note") == "tab\tquote\" é"
        np.testing.assert_array_equal(f.read("a/b.c"), [7, 9])


def test_loader_validation_without_cuda(tmp_path):
    lib = _lib.load()
    assert lib.rxla_b200_decoder_load_safetensors(None, b"x", b"", None, None) == _lib.INVALID_ARGUMENT
    import ctypes
    h = ctypes.c_void_p()
    assert lib.rxla_b200_safetensors_open(str(tmp_path / "none").encode(), ctypes.byref(h)) == \
        _lib.NOT_FOUND
