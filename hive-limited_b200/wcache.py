"""On-disk cache of an engine's device-ready weights.

The reference re-quantises every weight from the checkpoint on every load
(engine/limited.py:257-297); for the 8B geometry that is tens of seconds of host and
device work before the first token. An entry of this cache holds exactly the bytes the
engine uploads, in the layout the kernels read:

  * every projection in the tile-interleaved int4 layout (what hv_w4_prepack leaves on
    the device: nibbles, then scales), with its K, rows and gate/up pairing;
  * the f16 embedding and the f32 norm gains.

An entry is one directory <root>/<key>/ holding manifest.json and weights.bin; every
blob starts on a 256-byte boundary of weights.bin. The key hashes the layout version,
the model geometry, the shard (world, rank) and the identity of the source -- the names,
sizes and modification times of a model directory's files, or a tag the caller gives
for a synthetic model -- so a changed checkpoint or shard plan is a miss, never a stale
hit. An entry is written into a temporary directory and renamed into place, so readers
see a complete entry or none; a manifest that does not parse, or a weights.bin whose
size is not the manifest's, reads as a miss.

Host-side only (numpy), no GPU calls.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import tempfile
from pathlib import Path

import numpy as np

LAYOUT_VERSION = 1
ALIGN = 256
GEOMETRY = ("n_layer", "hidden", "ffn", "n_head", "n_kv", "head_dim", "vocab", "tied")


def entry_key(cfg, world: int, rank: int, model_dir=None, tag=None,
              w4_layout: str = "pp") -> tuple[str, dict]:
    """(key, identity) of the cache entry for this model source and shard. Exactly one
    of `model_dir` (a checkpoint directory) or `tag` (a caller-chosen name, e.g. for a
    seeded synthetic model) identifies the source. `w4_layout` is the arrangement of the
    prepacked tiles ("pp" or "dq"), which the cached bytes are in."""
    if (model_dir is None) == (tag is None):
        raise ValueError("a weight-cache key needs exactly one of model_dir or tag")
    if w4_layout not in ("pp", "dq"):
        raise ValueError(f"w4_layout={w4_layout!r}")
    ident = {"layout": LAYOUT_VERSION, "world": int(world), "rank": int(rank),
             "geometry": {k: getattr(cfg, k) for k in GEOMETRY}}
    if w4_layout != "pp":
        ident["w4_layout"] = w4_layout
    if model_dir is not None:
        files = sorted(p for p in Path(model_dir).iterdir()
                       if p.is_file() and (p.suffix == ".safetensors" or p.name == "config.json"))
        ident["files"] = [[p.name, p.stat().st_size, p.stat().st_mtime_ns] for p in files]
    else:
        ident["tag"] = str(tag)
    key = hashlib.sha256(json.dumps(ident, sort_keys=True).encode()).hexdigest()[:32]
    return key, ident


class EntryWriter:
    """Builds one entry in a temporary directory under `root`; commit() renames it into
    place (if another writer committed the same key first, theirs is kept)."""

    def __init__(self, root, key: str, ident: dict):
        self.root = Path(root)
        self.root.mkdir(parents=True, exist_ok=True)
        self.final = self.root / key
        self.tmp = Path(tempfile.mkdtemp(prefix=f".{key}.", dir=self.root))
        self.ident = ident
        self.items: dict[str, dict] = {}
        self.off = 0
        self.fh = open(self.tmp / "weights.bin", "wb")

    def _blob(self, arr: np.ndarray) -> dict:
        arr = np.ascontiguousarray(arr)
        pad = (-self.off) % ALIGN
        if pad:
            self.fh.write(b"\0" * pad)
            self.off += pad
        meta = {"offset": self.off, "nbytes": int(arr.nbytes), "dtype": arr.dtype.str,
                "shape": list(arr.shape)}
        arr.tofile(self.fh)
        self.off += arr.nbytes
        return meta

    def add_array(self, name: str, arr: np.ndarray) -> None:
        self.items[name] = {"kind": "array", "data": self._blob(arr)}

    def add_w4(self, name: str, nib: np.ndarray, scale: np.ndarray, k: int, rows: int,
               pair: int) -> None:
        """A projection in the tile-interleaved layout: nibble bytes and scale bytes as
        hv_w4_prepack wrote them for (rows, K, pair_ffn)."""
        self.items[name] = {"kind": "w4", "k": int(k), "rows": int(rows), "pair": int(pair),
                            "nib": self._blob(nib), "scale": self._blob(scale)}

    def commit(self) -> Path:
        self.fh.close()
        man = {"layout": LAYOUT_VERSION, "ident": self.ident, "size": self.off,
               "items": self.items}
        (self.tmp / "manifest.json").write_text(json.dumps(man))
        try:
            os.rename(self.tmp, self.final)
        except OSError:                       # the same entry was committed meanwhile
            shutil.rmtree(self.tmp, ignore_errors=True)
        return self.final

    def abort(self) -> None:
        try:
            self.fh.close()
        finally:
            shutil.rmtree(self.tmp, ignore_errors=True)


class Entry:
    """A committed entry, read through a memory map of weights.bin."""

    def __init__(self, path):
        self.path = Path(path)
        man = json.loads((self.path / "manifest.json").read_text())
        if man.get("layout") != LAYOUT_VERSION:
            raise ValueError(f"{self.path}: layout {man.get('layout')} != {LAYOUT_VERSION}")
        size = (self.path / "weights.bin").stat().st_size
        if size != man["size"]:
            raise ValueError(f"{self.path}: weights.bin holds {size} bytes, the manifest "
                             f"{man['size']}")
        self.ident, self.items = man["ident"], man["items"]
        self._mm = (np.memmap(self.path / "weights.bin", dtype=np.uint8, mode="r") if size
                    else np.zeros(0, np.uint8))

    def _view(self, meta: dict) -> np.ndarray:
        o, n = meta["offset"], meta["nbytes"]
        if o < 0 or o + n > self._mm.size:
            raise ValueError(f"{self.path}: blob [{o}, {o + n}) outside weights.bin")
        return self._mm[o:o + n].view(np.dtype(meta["dtype"])).reshape(meta["shape"])

    def array(self, name: str) -> np.ndarray:
        it = self.items[name]
        if it["kind"] != "array":
            raise ValueError(f"{name} is a {it['kind']} item")
        return self._view(it["data"])

    def w4(self, name: str) -> tuple[np.ndarray, np.ndarray, int, int, int]:
        """(nibble bytes, scale bytes, K, rows, pair_ffn) of a projection."""
        it = self.items[name]
        if it["kind"] != "w4":
            raise ValueError(f"{name} is a {it['kind']} item")
        return self._view(it["nib"]), self._view(it["scale"]), it["k"], it["rows"], it["pair"]


def open_entry(root, key: str):
    """The committed entry for `key` under `root`, or None (absent, or unreadable)."""
    try:
        return Entry(Path(root) / key)
    except (OSError, ValueError, KeyError, TypeError):
        return None
