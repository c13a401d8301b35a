"""The on-disk weight cache (wcache.py), host side: entries round-trip byte for byte,
blobs are 256-byte aligned, the key changes with everything that changes the uploaded
bytes (geometry, shard, source files, tag), incomplete entries read as misses, and a
second writer of the same key keeps the first entry."""
import os
import time

import numpy as np
import pytest

import limited
import synth
import wcache
from w4format import Config, save_safetensors


def _cfg(**kw):
    return Config(synth.tiny_arch(**kw))


def _write(root, key, ident, seed=0):
    g = np.random.default_rng(seed)
    arrays = {"emb16": g.standard_normal((64, 32)).astype(np.float16),
              "0.an": g.standard_normal(32).astype(np.float32)}
    w4 = {"0.qkv": (g.integers(0, 255, 1280 * 3, dtype=np.uint8),
                    g.integers(0, 255, 320 * 3, dtype=np.uint8), 256, 24, 0)}
    w = wcache.EntryWriter(root, key, ident)
    for n, a in arrays.items():
        w.add_array(n, a)
    for n, (nib, sc, k, rows, pair) in w4.items():
        w.add_w4(n, nib, sc, k, rows, pair)
    return w.commit(), arrays, w4


def test_round_trip_and_alignment(tmp_path):
    key, ident = wcache.entry_key(_cfg(), 1, 0, tag="synthetic:tiny:7")
    path, arrays, w4 = _write(tmp_path, key, ident)
    assert path == tmp_path / key
    e = wcache.open_entry(tmp_path, key)
    assert e is not None and e.ident == ident
    for n, a in arrays.items():
        got = e.array(n)
        assert got.dtype == a.dtype and np.array_equal(got, a)
    nib, sc, k, rows, pair = e.w4("0.qkv")
    assert (k, rows, pair) == (256, 24, 0)
    assert np.array_equal(nib, w4["0.qkv"][0]) and np.array_equal(sc, w4["0.qkv"][1])
    for it in e.items.values():
        for blob in ([it["data"]] if it["kind"] == "array" else [it["nib"], it["scale"]]):
            assert blob["offset"] % wcache.ALIGN == 0
    with pytest.raises(ValueError):
        e.w4("0.an")
    assert not [p for p in tmp_path.iterdir() if p.name.startswith(".")]  # no temp left


def test_key_follows_geometry_shard_and_source(tmp_path):
    base = wcache.entry_key(_cfg(), 1, 0, tag="a")[0]
    assert wcache.entry_key(_cfg(), 1, 0, tag="a")[0] == base
    assert wcache.entry_key(_cfg(hidden=512), 1, 0, tag="a")[0] != base
    assert wcache.entry_key(_cfg(), 2, 0, tag="a")[0] != base
    assert wcache.entry_key(_cfg(), 2, 1, tag="a")[0] != wcache.entry_key(_cfg(), 2, 0, tag="a")[0]
    assert wcache.entry_key(_cfg(), 1, 0, tag="b")[0] != base
    assert wcache.entry_key(_cfg(), 1, 0, tag="a", w4_layout="dq")[0] != base
    assert wcache.entry_key(_cfg(), 1, 0, tag="a", w4_layout="pp")[0] == base
    with pytest.raises(ValueError):
        wcache.entry_key(_cfg(), 1, 0)
    with pytest.raises(ValueError):
        wcache.entry_key(_cfg(), 1, 0, model_dir=tmp_path, tag="a")
    # a model directory: its files' names, sizes and modification times
    (tmp_path / "config.json").write_text("{}")
    save_safetensors(tmp_path / "model.safetensors", {"x": np.zeros(4, np.float32)})
    k1 = wcache.entry_key(_cfg(), 1, 0, model_dir=tmp_path)[0]
    assert wcache.entry_key(_cfg(), 1, 0, model_dir=tmp_path)[0] == k1
    t = time.time() + 5
    os.utime(tmp_path / "model.safetensors", (t, t))
    assert wcache.entry_key(_cfg(), 1, 0, model_dir=tmp_path)[0] != k1


def test_incomplete_entries_are_misses(tmp_path):
    key, ident = wcache.entry_key(_cfg(), 1, 0, tag="t")
    assert wcache.open_entry(tmp_path, key) is None            # absent
    path, _, _ = _write(tmp_path, key, ident)
    with open(path / "weights.bin", "r+b") as fh:             # truncated
        fh.truncate(100)
    assert wcache.open_entry(tmp_path, key) is None
    key2, ident2 = wcache.entry_key(_cfg(), 1, 0, tag="u")
    path2, _, _ = _write(tmp_path, key2, ident2)
    (path2 / "manifest.json").write_text("{not json")             # unreadable manifest
    assert wcache.open_entry(tmp_path, key2) is None
    w = wcache.EntryWriter(tmp_path, "k3", {})                   # aborted write
    w.add_array("x", np.zeros(8, np.float32))
    w.abort()
    assert wcache.open_entry(tmp_path, "k3") is None
    assert not [p for p in tmp_path.iterdir() if p.name.startswith(".")]


def test_second_writer_keeps_the_first_entry(tmp_path):
    key, ident = wcache.entry_key(_cfg(), 1, 0, tag="race")
    _write(tmp_path, key, ident, seed=1)
    _write(tmp_path, key, ident, seed=2)
    e = wcache.open_entry(tmp_path, key)
    want = np.random.default_rng(1).standard_normal((64, 32)).astype(np.float16)
    assert np.array_equal(e.array("emb16"), want)
    assert not [p for p in tmp_path.iterdir() if p.name.startswith(".")]


def test_engine_checks_cache_arguments_before_device_work(tmp_path):
    cfg = _cfg()
    with pytest.raises(ValueError, match="exactly one"):
        limited.Engine(config=cfg, tensors={}, weight_cache=tmp_path)   # no identity
