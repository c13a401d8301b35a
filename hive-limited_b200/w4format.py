"""The per-32 int4 weight contract, the safetensors reader and the model geometry.

Host-side only (numpy): nothing here touches the GPU, so the synthetic-model generator
and the tests can import it on a machine without the native library.

The quantisation rule and its packing are the reference's numeric contract and have to
be identical bit for bit (engine/limited.py:24-58 in HIVE Limited):

    per 32-element block along K:  s = max|w| / 7      (s == 0 -> 1.0)
                                   q = clip(round_half_even(w / s), -7, +7)
    packing, 8 values per uint32:  word i, byte b = q[8i+b] (low nibble)
                                                  | q[8i+4+b] (high nibble)
    scales: float32 [N, K/32]

The low nibbles of one word line up with four consecutive int8 activations, and the
high nibbles with the next four: that is what lets the GPU feed a whole 32-bit word
to one dp4a after a single mask.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

F32 = np.float32
BLOCK = 32


def quantize_w4(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Dense [N, K] float weights -> (packed uint32 [N, K/8], scales float32 [N, K/32]).

    Same contract and errors as engine/limited.py:40-58.
    """
    if w.ndim != 2:
        raise ValueError(f"expected a 2-D weight matrix, got shape {w.shape}")
    n, k = w.shape
    if k % BLOCK:
        raise ValueError(f"K={k} is not a multiple of {BLOCK}")
    blocks = w.astype(F32, copy=False).reshape(n, k // BLOCK, BLOCK)
    scale = (np.abs(blocks).max(2) / F32(7.0)).astype(F32)
    scale[scale == 0] = F32(1.0)
    q = np.clip(np.rint(blocks / scale[:, :, None]), -7, 7).astype(np.int8)
    nib = (q.view(np.uint8) & 15).astype(np.uint32).reshape(n, k // 8, 2, 4)
    # nib[:, i, 0, b] = q[8i+b] -> bits 8b..8b+3 ; nib[:, i, 1, b] = q[8i+4+b] -> bits 8b+4..
    shifts = (np.arange(4, dtype=np.uint32) * 8)
    packed = ((nib[:, :, 0, :] << shifts) | (nib[:, :, 1, :] << (shifts + 4))).sum(
        axis=2, dtype=np.uint32)
    return np.ascontiguousarray(packed, dtype=np.uint32), np.ascontiguousarray(scale)


def dequantize_w4(packed: np.ndarray, scale: np.ndarray, k: int) -> np.ndarray:
    """Inverse of quantize_w4 (engine/limited.py:61-75): float32 [N, K]."""
    q = unpack_w4(packed, k).astype(F32)
    n = packed.shape[0]
    return (q.reshape(n, k // BLOCK, BLOCK) * scale[:, :, None]).reshape(n, k).astype(F32)


def unpack_w4(packed: np.ndarray, k: int) -> np.ndarray:
    """packed uint32 [N, K/8] -> the signed int4 values as int8 [N, K]."""
    n = packed.shape[0]
    by = packed.view(np.uint8).reshape(n, k // 8, 4)
    lo = (by & 15).astype(np.int8)
    hi = (by >> 4).astype(np.int8)
    out = np.empty((n, k // 8, 2, 4), np.int8)
    out[:, :, 0, :] = np.where(lo >= 8, lo - 16, lo)
    out[:, :, 1, :] = np.where(hi >= 8, hi - 16, hi)
    return out.reshape(n, k)


# ---------------------------------------------------------------------------
# safetensors reader (the public file format: an 8-byte little-endian header size, a
# JSON header mapping each tensor name to {dtype, shape, data_offsets}, then the raw
# tensor bytes). The module keeps the reference engine's names (SafeTensors with keys()
# and get(), load_model_tensors) because limited.Engine and its callers import them.
# ---------------------------------------------------------------------------

# numpy element type of each safetensors dtype tag; BF16 is read as its 16 raw bits and
# widened to float32 (bf16 is the top half of an f32)
_NP_OF_TAG = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "BF16": np.uint16,
              "I64": np.int64, "I32": np.int32, "I16": np.int16, "I8": np.int8,
              "U8": np.uint8, "BOOL": np.bool_}


def _read_index(path: Path) -> tuple[dict, int]:
    """The header's tensor entries and the file offset where tensor data begins; every
    entry's byte range is checked against its dtype and shape and against the file."""
    size = path.stat().st_size
    with open(path, "rb") as fh:
        prefix = fh.read(8)
        if len(prefix) != 8:
            raise ValueError(f"{path}: not a safetensors file (no header size)")
        hlen = int.from_bytes(prefix, "little")
        if hlen <= 0 or 8 + hlen > size:
            raise ValueError(f"{path}: header size {hlen} does not fit the file")
        header = json.loads(fh.read(hlen))
    base = 8 + hlen
    index = {}
    for name, entry in header.items():
        if name == "__metadata__":
            continue
        tag, shape, (lo, hi) = entry["dtype"], list(entry["shape"]), entry["data_offsets"]
        if tag not in _NP_OF_TAG:
            raise ValueError(f"{name}: unsupported dtype {tag}")
        count = int(np.prod(shape, dtype=np.int64)) if shape else 1
        if hi - lo != count * np.dtype(_NP_OF_TAG[tag]).itemsize or base + hi > size:
            raise ValueError(f"{name}: data range {lo}..{hi} does not match {tag}{shape}")
        index[name] = (tag, tuple(shape), lo)
    return index, base


class SafeTensors:
    """Tensors of one .safetensors file, mapped read-only (no copy until a tensor is
    widened or written to)."""

    def __init__(self, path):
        self.path = Path(path)
        self._index, self._base = _read_index(self.path)
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")

    def keys(self) -> list[str]:
        return list(self._index)

    def get(self, name: str) -> np.ndarray:
        tag, shape, lo = self._index[name]
        dt = np.dtype(_NP_OF_TAG[tag])
        count = int(np.prod(shape, dtype=np.int64)) if shape else 1
        start = self._base + lo
        arr = self._map[start:start + count * dt.itemsize].view(dt).reshape(shape)
        if tag == "BF16":
            return (arr.astype(np.uint32) << 16).view(np.float32)
        return arr


def load_model_tensors(model_dir) -> dict[str, np.ndarray]:
    """Every tensor of every .safetensors file in a model directory (files in name
    order; a name that appears twice keeps its last file's tensor)."""
    files = sorted(Path(model_dir).glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {model_dir}")
    out: dict[str, np.ndarray] = {}
    for f in files:
        st = SafeTensors(f)
        out.update((name, st.get(name)) for name in st.keys())
    return out


def save_safetensors(path, tensors: dict[str, np.ndarray]) -> None:
    """Write float32/float16 tensors as one .safetensors file (used to hand synthetic
    models to code that reads a model directory)."""
    names = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16"}
    header, off, blobs = {}, 0, []
    for k, v in tensors.items():
        v = np.ascontiguousarray(v)
        header[k] = {"dtype": names[v.dtype], "shape": list(v.shape),
                     "data_offsets": [off, off + v.nbytes]}
        off += v.nbytes
        blobs.append(v)
    raw = json.dumps(header).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(raw)))
        fh.write(raw)
        for v in blobs:
            fh.write(v.tobytes())


# ---------------------------------------------------------------------------
# geometry (engine/limited.py:138-164)
# ---------------------------------------------------------------------------

class Config:
    """Geometry read from the model's own config.json.

    `max_context` defaults to the reference's 4096 and can be raised: the 8B decode
    workload (4096-token prompt + 256 generated) needs 4352 positions.
    """

    def __init__(self, cfg: dict, max_context: int = 4096):
        self.raw = dict(cfg)
        self.n_layer = cfg["num_hidden_layers"]
        self.hidden = cfg["hidden_size"]
        self.ffn = cfg["intermediate_size"]
        self.n_head = cfg["num_attention_heads"]
        self.n_kv = cfg["num_key_value_heads"]
        self.head_dim = cfg.get("head_dim", self.hidden // self.n_head)
        self.vocab = cfg["vocab_size"]
        self.rms_eps = cfg.get("rms_norm_eps", 1e-6)
        self.rope_theta = cfg.get("rope_theta", 1000000.0)
        self.tied = bool(cfg.get("tie_word_embeddings", False))
        self.eos = cfg.get("eos_token_id", None)
        self.max_context = int(cfg.get("max_context", max_context))

    @property
    def group(self) -> int:
        return self.n_head // self.n_kv

    @classmethod
    def load(cls, model_dir) -> "Config":
        with open(Path(model_dir) / "config.json", "r", encoding="utf-8") as fh:
            return cls(json.load(fh))
