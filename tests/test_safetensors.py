"""The safetensors reader (w4format.SafeTensors / load_model_tensors) on the CPU: tensors
written by save_safetensors come back bit for bit, BF16 widens to the float32 whose top
half it is, a model directory of several files merges, and a header whose byte ranges do
not match the file is refused."""
import json
import struct

import numpy as np
import pytest

import w4format


def test_roundtrip_f32_f16(tmp_path):
    g = np.random.default_rng(0)
    t = {"a": g.standard_normal((3, 5)).astype(np.float32),
         "b": g.standard_normal(7).astype(np.float16),
         "c": np.zeros((0, 4), np.float32)}
    w4format.save_safetensors(tmp_path / "m.safetensors", t)
    st = w4format.SafeTensors(tmp_path / "m.safetensors")
    assert sorted(st.keys()) == ["a", "b", "c"]
    for k, v in t.items():
        got = st.get(k)
        assert got.dtype == v.dtype and got.shape == v.shape
        assert np.array_equal(got.view(np.uint8), v.view(np.uint8))


def _write_raw(path, header: dict, data: bytes):
    raw = json.dumps(header).encode()
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(raw)))
        fh.write(raw)
        fh.write(data)


def test_bf16_widens_and_metadata_is_skipped(tmp_path):
    x = np.array([1.5, -2.25, 3.0e-3, 65504.0], np.float32)
    top = (x.view(np.uint32) >> 16).astype(np.uint16)          # exact bf16 for these
    _write_raw(tmp_path / "b.safetensors",
               {"__metadata__": {"format": "pt"},
                "w": {"dtype": "BF16", "shape": [2, 2], "data_offsets": [0, 8]}},
               top.tobytes())
    st = w4format.SafeTensors(tmp_path / "b.safetensors")
    assert st.keys() == ["w"]
    got = st.get("w")
    assert got.dtype == np.float32 and got.shape == (2, 2)
    assert np.array_equal(got.reshape(-1).view(np.uint32), top.astype(np.uint32) << 16)


def test_model_directory_merges_files(tmp_path):
    w4format.save_safetensors(tmp_path / "model-00001.safetensors",
                              {"x": np.ones(3, np.float32)})
    w4format.save_safetensors(tmp_path / "model-00002.safetensors",
                              {"y": np.full(2, 2.0, np.float16)})
    t = w4format.load_model_tensors(tmp_path)
    assert sorted(t) == ["x", "y"] and t["y"].dtype == np.float16
    with pytest.raises(FileNotFoundError):
        w4format.load_model_tensors(tmp_path / "empty")


@pytest.mark.parametrize("entry", [
    {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]},     # range shorter than shape
    {"dtype": "F32", "shape": [8], "data_offsets": [0, 32]},     # past the end of the file
    {"dtype": "Q4", "shape": [4], "data_offsets": [0, 16]},      # unknown dtype
])
def test_bad_header_is_refused(tmp_path, entry):
    _write_raw(tmp_path / "bad.safetensors", {"t": entry}, bytes(16))
    with pytest.raises(ValueError):
        w4format.SafeTensors(tmp_path / "bad.safetensors")
