"""The safetensors loader (ModelWeights, objeta-parser lib.rs:97-330) on CPU:
files written here by hand, single file and shard directory, metadata
skipping, dtypes and the F16 / BF16 widening rules, malformed headers."""
import json
import struct

import numpy as np
import pytest

from objeta_b200._lib import CudaError
from objeta_b200.weights import ModelWeights


def _write(path, tensors, metadata=None, pad=0):
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (dtype, shape, data) in tensors.items():
        b = np.ascontiguousarray(data).tobytes()
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode() + b" " * pad
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def test_single_file_and_dtypes(tmp_path):
    f32 = np.arange(6, dtype=np.float32).reshape(2, 3)
    bf = np.array([0x3F80, 0x4000, 0xC040, 0x0000], np.uint16)                 # 1, 2, -3, 0
    f16 = np.array([0x3C00, 0x0001, 0x83FF, 0x7C00, 0xFC00], np.uint16)         # 1, 2^-24, -(1023 * 2^-24), inf, -inf
    e8 = np.array([127, 0, 255], np.uint8)
    p = tmp_path / "m.safetensors"
    _write(p, {"w.f32": ("F32", (2, 3), f32), "w.bf16": ("BF16", (4,), bf), "w.f16": ("F16", (5,), f16),
               "w.scale": ("F8_E8M0", (3,), e8), "ids": ("I64", (2,), np.array([7, -1], np.int64))},
           metadata={"format": "pt", "note": 'a "quoted" {brace} [x]'})
    w = ModelWeights.open(p)
    assert len(w) == 5 and sorted(w.keys()) == sorted(["w.f32", "w.bf16", "w.f16", "w.scale", "ids"])
    assert w.contains("w.f32") and not w.contains("__metadata__") and not w.contains("nope")
    info = w.info("w.f32")
    assert info.dtype == "F32" and info.shape == [2, 3] and info.nbytes == 24 and info.nelem == 6
    assert np.array_equal(w.get_matrix("w.f32")[2].reshape(2, 3), f32)
    assert w.get_f32("w.bf16").tolist() == [1.0, 2.0, -3.0, 0.0]
    h = w.get_f32("w.f16")
    assert h[0] == 1.0 and h[1] == np.float32(2.0 ** -24) and h[2] == np.float32(-1023 * 2.0 ** -24)
    assert np.isposinf(h[3]) and np.isneginf(h[4])
    assert w.get_array("w.scale").tolist() == [127, 0, 255]
    assert w.get_array("ids").tolist() == [7, -1]
    with pytest.raises(CudaError) as e:
        w.get_f32("w.scale")
    assert "cannot convert" in e.value.source_message
    with pytest.raises(CudaError) as e:
        w.get_raw("missing.tensor")
    assert "missing tensor: missing.tensor" in e.value.source_message


def test_shard_directory(tmp_path):
    _write(tmp_path / "model-00002-of-00002.safetensors", {"b": ("U8", (3,), np.array([4, 5, 6], np.uint8))})
    _write(tmp_path / "model-00001-of-00002.safetensors", {"a": ("U8", (2,), np.array([1, 2], np.uint8))})
    (tmp_path / "config.json").write_text("{}")
    w = ModelWeights(tmp_path)
    assert sorted(w.keys()) == ["a", "b"]
    assert w.get_raw("a").tolist() == [1, 2] and w.get_raw("b").tolist() == [4, 5, 6]


def test_malformed_files(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(CudaError) as e:
        ModelWeights(p)
    assert "header length exceeds file size" in e.value.source_message
    _write(p, {"x": ("Q7", (1,), np.zeros(1, np.uint8))})
    with pytest.raises(CudaError) as e:
        ModelWeights(p)
    assert "Unknown dtype: Q7" in e.value.source_message
    p.write_bytes(struct.pack("<Q", 9) + b'{"x": 12}')
    with pytest.raises(CudaError) as e:
        ModelWeights(p)
    assert "invalid tensor entry" in e.value.source_message
    hdr = json.dumps({"x": {"dtype": "U8", "shape": [8], "data_offsets": [0, 8]}}).encode()
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"abc")
    with pytest.raises(CudaError) as e:
        ModelWeights(p)
    assert "outside the file" in e.value.source_message
    with pytest.raises(CudaError) as e:
        ModelWeights(tmp_path / "does-not-exist.safetensors")
    assert e.value.kind == "Io"
