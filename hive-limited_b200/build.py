"""Build libhive_b200.so (the C-ABI kernel library) in-tree with nvcc for sm_100a.

    python hive-limited_b200/build.py            # build if sources changed
    python hive-limited_b200/build.py --force    # rebuild

Each .cu under csrc/ compiles to an object in _build/ (parallel), then one shared
library is linked with the CUDA runtime static and NCCL dynamic. A MANIFEST.json next to
the library records its sha256 and ABI version; the engine checks it at load, as the
reference checks its PTX manifest (engine/limited.py:218-235).
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libhive_b200.so"
MANIFEST = HERE / "MANIFEST.json"
INCLUDE = HERE.parent / "include"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2",
         "-Xptxas", "-warn-spills", f"-I{INCLUDE}", "--expt-relaxed-constexpr"]
LIBS = ["-lnccl"]


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _deps():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
                  + list(INCLUDE.glob("*.h")) + [Path(__file__)])


def _stamp() -> str:
    h = hashlib.sha256()
    for p in _deps():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(ARCH + FLAGS + LIBS).encode())
    return h.hexdigest()


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose or r.stderr.strip():
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    stamp = _stamp()
    if not force and LIB.exists() and MANIFEST.exists():
        try:
            if json.loads(MANIFEST.read_text()).get("source_stamp") == stamp:
                return LIB
        except (ValueError, OSError):
            pass
    BUILD.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp),
           *map(str, objs), *LIBS]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    digest = hashlib.sha256(LIB.read_bytes()).hexdigest()
    MANIFEST.write_text(json.dumps({
        "library": LIB.name, "sha256": digest, "abi_version": 1,
        "arch": "sm_100a", "source_stamp": stamp}, indent=1) + "\n")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
