"""CPU-side checks of the native library and the host logic (no GPU calls)."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "hive_b200.h"


def header_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bint\s+(hv_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    import build
    path = build.build()
    return ctypes.CDLL(str(path))


def test_library_exports_every_header_symbol(lib):
    syms = header_symbols()
    assert len(syms) > 40
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_covers_header():
    import hvdrv
    assert set(header_symbols()) == set(hvdrv.exported_symbols())


def header_arities() -> dict:
    """Parameter count of every hv_* declaration in the header ((void) counts 0)."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    out = {}
    for name, params in re.findall(r"\bint\s+(hv_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_binding_arities_match_header():
    """Every ctypes signature in hvdrv has the header's parameter count."""
    import hvdrv
    ar = header_arities()
    assert set(ar) == set(hvdrv._SIGS)
    bad = {n: (len(hvdrv._SIGS[n]), ar[n]) for n in ar if len(hvdrv._SIGS[n]) != ar[n]}
    assert not bad, bad


def test_library_version_and_kernels(lib):
    import hvdrv
    hvdrv.load()
    assert hvdrv.load().hv_version() == hvdrv.ABI_VERSION
    ks = hvdrv.kernel_list()
    for k in ("k_a4gv", "k_qa8s", "k_rmsnorm", "k_attn_sc", "k_attn_cx", "k_step", "k_argmax_p"):
        assert k in ks


def test_errors_are_reported_not_fatal(lib):
    """Argument checks fail with a status and a message; nothing aborts the process."""
    import hvdrv
    with pytest.raises(hvdrv.CudaError) as e:
        hvdrv.a4gv(0, 0, 0, 0, 0, 8, 16)
    assert "bad arguments" in str(e.value)
    with pytest.raises(hvdrv.CudaError) as e:
        hvdrv.rmsnorm(0, 0, 0, 1, 128)
    assert e.value.code == 1001


def test_manifest_matches_library():
    import hashlib
    import json

    import build
    build.build()
    man = json.loads(build.MANIFEST.read_text())
    assert man["sha256"] == hashlib.sha256(build.LIB.read_bytes()).hexdigest()
    assert man["arch"] == "sm_100a"


def test_step_desc_layout_matches_header(tmp_path):
    """The ctypes mirror of hv_step_desc / hv_layer_w / hv_step_peers has the C layout:
    every field's offset and each struct's size as the C compiler lays out the header."""
    import shutil
    import subprocess
    import limited
    assert ctypes.sizeof(limited._LayerW) == 14 * 8
    # 8 ints + 2 floats + 2 ints = 48 bytes, then 24 pointers, world, rank, peers, kv_dtype,
    # w4_layout, kv_base, kv_rows
    assert limited._StepDesc.layers.offset == 48
    assert limited._StepDesc.world.offset == 48 + 24 * 8
    assert limited._StepDesc.peers.offset == 48 + 24 * 8 + 8
    assert limited._StepDesc.kv_dtype.offset == 48 + 24 * 8 + 16
    assert limited._StepDesc.w4_layout.offset == 48 + 24 * 8 + 20
    assert limited._StepDesc.kv_base.offset == 48 + 24 * 8 + 24
    assert limited._StepDesc.kv_rows.offset == 48 + 24 * 8 + 32
    assert ctypes.sizeof(limited._StepDesc) == 48 + 24 * 8 + 40
    assert ctypes.sizeof(limited._StepPeers) == 5 * 8 * 8
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler for the header's own layout")
    structs = [("hv_step_desc", limited._StepDesc), ("hv_layer_w", limited._LayerW),
               ("hv_step_peers", limited._StepPeers)]
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "hive_b200.h"',
             'int main(void) {']
    for cname, py in structs:
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ['  return 0;', '}']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for ln in subprocess.run([str(exe)], capture_output=True, text=True,
                             check=True).stdout.splitlines():
        cname, field, val = ln.split()
        got[(cname, field)] = int(val)
    for cname, py in structs:
        assert got[(cname, "sizeof")] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[(cname, f)] == getattr(py, f).offset, (cname, f)


def test_gpu_only_paths_fail_loudly_without_gpu():
    """No CPU fallback: constructing an engine needs the GPU."""
    import hvdrv
    try:
        n = hvdrv.device_count()
    except hvdrv.CudaError:
        n = 0
    if n:
        pytest.skip("a GPU is visible")
    import limited
    import synth
    with pytest.raises((hvdrv.CudaError, RuntimeError)):
        limited.Engine(config=synth.tiny_arch(), tensors={})


def test_host_quantizer_matches_oracle():
    import hv_oracle
    import w4format
    w = (np.random.default_rng(0).standard_normal((33, 96)) * 0.02).astype(np.float32)
    a = w4format.quantize_w4(w)
    b = hv_oracle.quantize_w4(w)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    back = w4format.dequantize_w4(a[0], a[1], 96)
    assert np.abs(back - w).max() <= np.abs(w).max() / 7 / 2 * 1.0001


def test_big_tensors_are_drawn_in_row_blocks(monkeypatch):
    """Above BIG_DRAW elements a tensor is BIG_BLOCKS row blocks, block b from stream
    (seed, index, b); below it, one stream (seed, index). Either way the draw does not
    depend on how many threads draw."""
    import synth
    monkeypatch.setattr(synth, "BIG_DRAW", 1000)
    x = synth.draw(3, 7, (40, 64), "w")
    edges = [40 * b // synth.BIG_BLOCKS for b in range(synth.BIG_BLOCKS + 1)]
    for b in range(synth.BIG_BLOCKS):
        want = synth.rng_for(3, 7, b).standard_normal((edges[b + 1] - edges[b], 64),
                                                       dtype=np.float32) * np.float32(0.02)
        assert np.array_equal(x[edges[b]:edges[b + 1]], want)
    small = synth.draw(3, 7, (10, 64), "w")
    assert np.array_equal(small, synth.rng_for(3, 7).standard_normal((10, 64),
                                                                      dtype=np.float32)
                          * np.float32(0.02))
    import w4format
    cfg = w4format.Config(synth.tiny_arch())
    a = dict(synth.iter_tensors(cfg, 5, threads=1))
    b = dict(synth.iter_tensors(cfg, 5, threads=6))
    for k in a:
        assert np.array_equal(a[k], b[k])


def test_synthetic_draw_is_deterministic_and_thread_independent():
    import synth
    import w4format
    cfg = w4format.Config(synth.tiny_arch())
    a = dict(synth.iter_tensors(cfg, 5, threads=1))
    b = dict(synth.iter_tensors(cfg, 5, threads=4))
    assert list(a) == [n for n, _, _ in synth.tensor_plan(cfg)]
    for k in a:
        assert np.array_equal(a[k], b[k])
