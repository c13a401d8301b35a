"""ctypes binding to libhive_b200.so — the replacement for HIVE Limited's engine/cudrv.py.

Same surface as the reference's driver binding (init, device, device_name,
driver_version, device_attribute, compute_capability, retain_primary_context,
set_current, synchronize, mem_info, alloc, free, upload, download, memset8,
stream_create, stream_synchronize, capture_begin, capture_end, graph_instantiate,
graph_launch, graph_destroy, CudaError), plus one function per kernel. Device pointers
are Python ints; every native call returns a status and a failure raises CudaError
carrying the library's message.

There is no CPU fallback: if the library cannot be loaded or no GPU is present, the
first call raises.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_NAME = "libhive_b200.so"
ABI_VERSION = 3

_L = None
_lib_path = None


class CudaError(RuntimeError):
    """A library call failed. Carries the call name, the status and the message."""

    def __init__(self, fn: str, code: int, msg: str = ""):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.fn, self.code, self.msg = fn, code, msg


_VP, _I, _SZ, _F = C.c_void_p, C.c_int, C.c_size_t, C.c_float
_PI = C.POINTER(C.c_int)

# name -> argtypes (all functions return int)
_SIGS = {
    "hv_version": [],
    "hv_kernel_list": [C.c_char_p, _SZ],
    "hv_last_error": [C.c_char_p, _SZ],
    "hv_init": [],
    "hv_device_count": [_PI],
    "hv_set_device": [_I],
    "hv_get_device": [_PI],
    "hv_device_name": [_I, C.c_char_p, _I],
    "hv_compute_capability": [_I, _PI, _PI],
    "hv_device_attribute": [_I, _I, _PI],
    "hv_driver_version": [_PI],
    "hv_mem_info": [C.POINTER(_SZ), C.POINTER(_SZ)],
    "hv_synchronize": [],
    "hv_alloc": [C.POINTER(_VP), _SZ],
    "hv_free": [_VP],
    "hv_upload": [_VP, _VP, _SZ],
    "hv_download": [_VP, _VP, _SZ],
    "hv_memset": [_VP, _I, _SZ],
    "hv_host_alloc": [C.POINTER(_VP), _SZ],
    "hv_host_free": [_VP],
    "hv_upload_async": [_VP, _VP, _SZ, _VP],
    "hv_download_async": [_VP, _VP, _SZ, _VP],
    "hv_copy_async": [_VP, _VP, _SZ, _VP],
    "hv_comm_init": [_I, C.POINTER(_I), C.POINTER(_VP)],
    "hv_comm_unique_id": [_VP],
    "hv_comm_init_rank": [_I, _I, _VP, _I, C.POINTER(_VP)],
    "hv_allgather": [_VP, C.POINTER(_VP), C.POINTER(_VP), _SZ, C.POINTER(_VP)],
    "hv_comm_size": [_VP, C.POINTER(_I), C.POINTER(_I)],
    "hv_comm_destroy": [_VP],
    "hv_stream_create": [C.POINTER(_VP)],
    "hv_stream_destroy": [_VP],
    "hv_stream_synchronize": [_VP],
    "hv_capture_begin": [_VP],
    "hv_capture_end": [_VP, C.POINTER(_VP)],
    "hv_graph_instantiate": [_VP, C.POINTER(_VP)],
    "hv_graph_launch": [_VP, _VP],
    "hv_graph_destroy": [_VP, _VP],
    "hv_event_create": [C.POINTER(_VP)],
    "hv_event_destroy": [_VP],
    "hv_event_record": [_VP, _VP],
    "hv_event_elapsed_ms": [_VP, _VP, C.POINTER(_F)],
    "hv_qa8s": [_VP, _VP, _VP, _I, _VP],
    "hv_a4gv": [_VP, _VP, _VP, _VP, _VP, _I, _I, _VP],
    "hv_a4gv_idot": [_VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _VP],
    "hv_rmsnorm": [_VP, _VP, _VP, _I, _I, _F, _VP],
    "hv_rope": [_VP, _VP, _VP, _VP, _I, _I, _VP],
    "hv_kv_append": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _VP],
    "hv_attn_decode": [_VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP],
    "hv_kv_append_f16": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _VP],
    "hv_attn_decode_f16": [_VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP],
    "hv_attn_reserve": [_I, _I, _I],
    "hv_attn_decode_noalloc": [_VP, _VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP],
    "hv_silu_mul": [_VP, _VP, _VP, _I, _VP],
    "hv_vadd": [_VP, _VP, _VP, _I, _VP],
    "hv_gather_emb": [_VP, _VP, _VP, _I, _VP],
    "hv_argmax_partial": [_VP, _VP, _VP, _I, _I, _VP],
    "hv_argmax_final": [_VP, _VP, _VP, _VP, _VP, _VP, _I, _VP],
    "hv_argmax_key": [_VP, _I, _I, _VP, _VP],
    "hv_argmax_key_final": [_VP, _I, _VP, _VP, _VP, _VP, _VP],
    "hv_quantize_w4": [_VP, _VP, _VP, _I, _I, _VP],
    "hv_wait_probe": [_VP, C.c_uint32, C.c_uint32, C.c_longlong, _VP, _VP],
    "hv_w4_prepacked_size": [_I, _I, _I, C.POINTER(_SZ), C.POINTER(_SZ)],
    "hv_w4_prepack": [_VP, _VP, _I, _I, _I, _VP, _VP, _VP],
    "hv_a4gv_pp": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _VP],
    "hv_w4_prepack_dq": [_VP, _VP, _I, _I, _I, _VP, _VP, _VP],
    "hv_a4gv_dq": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _VP],
    "hv_gemv_set_split": [_I],
    "hv_a4gemm_pp": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP],
    "hv_a4gemm_dq": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _VP],
    "hv_gather_rows": [_VP, _VP, _VP, _I, _I, _VP],
    "hv_qa8s_rows": [_VP, _VP, _VP, _I, _I, _VP],
    "hv_qk_rows": [_VP, _VP, _VP, _VP, _VP, _I, _VP, _VP, _VP, _I, _I, _I, _I, _F, _I, _VP],
    "hv_qk_rows_f16": [_VP, _VP, _VP, _VP, _VP, _I, _VP, _VP, _VP, _I, _I, _I, _I, _F, _I, _VP],
    "hv_attn_rows_scratch": [_I, _I, _I, _I, C.POINTER(_SZ), C.POINTER(_SZ)],
    "hv_attn_rows": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _VP, _VP, _VP],
    "hv_attn_rows_f16": [_VP, _VP, _VP, _VP, _VP, _I, _I, _I, _I, _I, _I, _VP, _VP, _VP],
    "hv_silu_rows": [_VP, _VP, _I, _I, _VP],
    "hv_step_config": [_I, _I, _I, _PI, _PI, C.POINTER(_SZ), _PI, C.POINTER(_SZ)],
    "hv_step_launch": [_VP, _I, _VP],
    "hv_step_set_option": [_I, _I],
    "hv_ipc_handle": [_VP, _VP],
    "hv_ipc_open": [_VP, C.POINTER(_VP)],
    "hv_ipc_close": [_VP],
    "hv_step_plans_bytes": [C.POINTER(_SZ)],
    "hv_step_plans": [_I, _I, _I, _VP, _SZ],
}


def library_path(kernels_dir=None) -> Path:
    d = Path(kernels_dir) if kernels_dir else Path(os.environ.get("HIVE_B200_LIB_DIR", HERE))
    return d / LIB_NAME


def load(kernels_dir=None, verify: bool = True):
    """Load the library once. With `verify`, its sha256 must match MANIFEST.json (the
    equivalent of the reference's PTX manifest check, engine/limited.py:218-235) and its
    ABI version must be the one this binding speaks."""
    global _L, _lib_path
    if _L is not None and kernels_dir is None:
        return _L                     # the per-call fast path: no filesystem access
    path = library_path(kernels_dir)
    if _L is not None:
        if path.resolve() != _lib_path.resolve():
            raise RuntimeError(f"{LIB_NAME} already loaded from {_lib_path}")
        return _L
    if not path.exists():
        raise RuntimeError(
            f"{path} not found: build it with `python hive-limited_b200/build.py` "
            "(there is no CPU fallback)")
    if verify:
        man = path.parent / "MANIFEST.json"
        if man.exists():
            want = json.loads(man.read_text()).get("sha256")
            got = hashlib.sha256(path.read_bytes()).hexdigest()
            if want != got:
                raise RuntimeError(f"{path.name}: sha256 mismatch.\n  manifest {want}\n"
                                   f"  on disk  {got}\nRefusing to run a library that is "
                                   "not the one built.")
    lib = C.CDLL(str(path))
    for name, args in _SIGS.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = C.c_int
    if lib.hv_version() != ABI_VERSION:
        raise RuntimeError(f"{path.name}: ABI version {lib.hv_version()} != {ABI_VERSION}")
    _L, _lib_path = lib, path
    return lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load().hv_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def _call(name: str, *args) -> None:
    rc = getattr(_L if _L is not None else load(), name)(*args)
    if rc != 0:
        raise CudaError(name, rc, last_error())


def kernel_list() -> list[str]:
    buf = C.create_string_buffer(1024)
    _call("hv_kernel_list", buf, len(buf))
    return buf.value.decode().split(",")


# ---- context (engine/cudrv.py:73-143) ---------------------------------------

def init() -> None:
    _call("hv_init")


def device_count() -> int:
    n = C.c_int()
    _call("hv_device_count", C.byref(n))
    return n.value


def device(index: int = 0) -> int:
    return int(index)


def device_name(dev: int) -> str:
    buf = C.create_string_buffer(128)
    _call("hv_device_name", dev, buf, 128)
    return buf.value.decode(errors="replace")


def driver_version() -> str:
    v = C.c_int()
    _call("hv_driver_version", C.byref(v))
    return f"{v.value // 1000}.{(v.value % 1000) // 10}"


def device_attribute(dev: int, attr: int) -> int:
    v = C.c_int()
    _call("hv_device_attribute", dev, attr, C.byref(v))
    return v.value


def compute_capability(dev: int) -> tuple[int, int]:
    a, b = C.c_int(), C.c_int()
    _call("hv_compute_capability", dev, C.byref(a), C.byref(b))
    return a.value, b.value


def retain_primary_context(dev: int) -> int:
    """Binds the device's primary context to this thread; the returned handle is what
    set_current() takes."""
    _call("hv_set_device", dev)
    return int(dev)


def set_current(ctx: int) -> None:
    _call("hv_set_device", int(ctx))


def synchronize() -> None:
    _call("hv_synchronize")


def mem_info() -> tuple[int, int]:
    f, t = C.c_size_t(), C.c_size_t()
    _call("hv_mem_info", C.byref(f), C.byref(t))
    return f.value, t.value


# ---- memory -------------------------------------------------------------------

def alloc(nbytes: int) -> int:
    p = C.c_void_p()
    _call("hv_alloc", C.byref(p), int(nbytes))
    return p.value or 0


def free(ptr: int) -> None:
    _call("hv_free", C.c_void_p(ptr))


def upload(dst: int, host_ptr: int, nbytes: int) -> None:
    _call("hv_upload", C.c_void_p(dst), C.c_void_p(host_ptr), int(nbytes))


def download(host_ptr: int, src: int, nbytes: int) -> None:
    _call("hv_download", C.c_void_p(host_ptr), C.c_void_p(src), int(nbytes))


def memset8(ptr: int, value: int, nbytes: int) -> None:
    _call("hv_memset", C.c_void_p(ptr), int(value), int(nbytes))


def host_alloc(nbytes: int) -> int:
    p = C.c_void_p()
    _call("hv_host_alloc", C.byref(p), int(nbytes))
    return p.value or 0


def host_free(ptr: int) -> None:
    _call("hv_host_free", C.c_void_p(ptr))


def upload_async(dst, host_ptr, nbytes, stream=0):
    _call("hv_upload_async", C.c_void_p(dst), C.c_void_p(host_ptr), int(nbytes),
          C.c_void_p(stream))


def download_async(host_ptr, src, nbytes, stream=0):
    _call("hv_download_async", C.c_void_p(host_ptr), C.c_void_p(src), int(nbytes),
          C.c_void_p(stream))


def copy_async(dst, src, nbytes, stream=0):
    _call("hv_copy_async", C.c_void_p(dst), C.c_void_p(src), int(nbytes), C.c_void_p(stream))


# ---- streams, graphs, events ------------------------------------------------------

def stream_create() -> int:
    s = C.c_void_p()
    _call("hv_stream_create", C.byref(s))
    return s.value or 0


def stream_destroy(stream: int) -> None:
    _call("hv_stream_destroy", C.c_void_p(stream))


def stream_synchronize(stream: int) -> None:
    _call("hv_stream_synchronize", C.c_void_p(stream))


def capture_begin(stream: int) -> None:
    _call("hv_capture_begin", C.c_void_p(stream))


def capture_end(stream: int) -> int:
    g = C.c_void_p()
    _call("hv_capture_end", C.c_void_p(stream), C.byref(g))
    return g.value or 0


def graph_instantiate(graph: int) -> int:
    e = C.c_void_p()
    _call("hv_graph_instantiate", C.c_void_p(graph), C.byref(e))
    return e.value or 0


def graph_launch(exec_: int, stream: int) -> None:
    _call("hv_graph_launch", C.c_void_p(exec_), C.c_void_p(stream))


def graph_destroy(graph: int, exec_: int) -> None:
    try:
        _call("hv_graph_destroy", C.c_void_p(graph), C.c_void_p(exec_))
    except CudaError:
        pass


def event_create() -> int:
    e = C.c_void_p()
    _call("hv_event_create", C.byref(e))
    return e.value or 0


def event_destroy(e: int) -> None:
    _call("hv_event_destroy", C.c_void_p(e))


def event_record(e: int, stream: int = 0) -> None:
    _call("hv_event_record", C.c_void_p(e), C.c_void_p(stream))


def event_elapsed_ms(e0: int, e1: int) -> float:
    ms = C.c_float()
    _call("hv_event_elapsed_ms", C.c_void_p(e0), C.c_void_p(e1), C.byref(ms))
    return ms.value


# ---- kernels ------------------------------------------------------------------------

def _p(x):
    return C.c_void_p(int(x))


def qa8s(src, a8, sa, nb, stream=0):
    _call("hv_qa8s", _p(src), _p(a8), _p(sa), nb, _p(stream))


def a4gv(a8, sa, b4, sw, dst, k8, n, stream=0):
    _call("hv_a4gv", _p(a8), _p(sa), _p(b4), _p(sw), _p(dst), k8, n, _p(stream))


def a4gv_idot(a8, sa, b4, sw, dst, idot, k8, n, stream=0):
    _call("hv_a4gv_idot", _p(a8), _p(sa), _p(b4), _p(sw), _p(dst), _p(idot), k8, n, _p(stream))


def rmsnorm(src, dst, w, rows, cols, eps=1e-5, stream=0):
    _call("hv_rmsnorm", _p(src), _p(dst), _p(w), rows, cols, C.c_float(eps), _p(stream))


def rope(vec, cos_t, sin_t, pos, heads, half, stream=0):
    _call("hv_rope", _p(vec), _p(cos_t), _p(sin_t), _p(pos), heads, half, _p(stream))


def kv_append(k, v, kc, vc, pos, nkv, hd, cap, stream=0, f16=False):
    """f16=True: kc/vc are binary16 caches (hv_kv_append_f16, the compressed-KV lane)."""
    _call("hv_kv_append_f16" if f16 else "hv_kv_append", _p(k), _p(v), _p(kc), _p(vc), _p(pos),
          nkv, hd, cap, _p(stream))


def attn_decode(q, kc, vc, ctx, scale, pos, nq, hd, group, kvstride, stream=0, f16=False):
    """f16=True: kc/vc are binary16 caches (hv_attn_decode_f16)."""
    _call("hv_attn_decode_f16" if f16 else "hv_attn_decode", _p(q), _p(kc), _p(vc), _p(ctx),
          _p(scale), _p(pos), nq, hd, group, kvstride, _p(stream))


def attn_reserve(nkv, group, cap):
    _call("hv_attn_reserve", nkv, group, cap)


IPC_HANDLE_BYTES = 64


def ipc_handle(ptr) -> bytes:
    """64-byte CUDA IPC handle of a device allocation made by this process."""
    buf = C.create_string_buffer(IPC_HANDLE_BYTES)
    _call("hv_ipc_handle", _p(ptr), buf)
    return buf.raw


COMM_ID_BYTES = 128


class Comm:
    """The C ABI's all-gather communicator (hv_comm_*): Comm(devs=[0, 1]) drives several
    GPUs from this process; Comm(nranks=, rank=, uid=, dev=) is one rank of a
    one-process-per-GPU job (uid from comm_unique_id() on one rank, passed to all)."""

    def __init__(self, devs=None, nranks=None, rank=None, uid=None, dev=None):
        self.ptr = _VP()
        if devs is not None:
            arr = (_I * len(devs))(*devs)
            _call("hv_comm_init", len(devs), arr, C.byref(self.ptr))
            self.ndev = len(devs)
        else:
            _call("hv_comm_init_rank", nranks, rank,
                  C.create_string_buffer(uid, COMM_ID_BYTES), dev, C.byref(self.ptr))
            self.ndev = 1

    def size(self):
        n, d = _I(), _I()
        _call("hv_comm_size", self.ptr, C.byref(n), C.byref(d))
        return n.value, d.value

    def allgather(self, send, recv, nbytes, streams=None):
        """recv[i] <- every rank's nbytes of send, rank after rank (device i of this
        process); asynchronous on streams[i] (default stream when None)."""
        n = self.ndev
        s = (_VP * n)(*[int(x) for x in send])
        r = (_VP * n)(*[int(x) for x in recv])
        st = (_VP * n)(*[int(x) for x in streams]) if streams else None
        _call("hv_allgather", self.ptr, s, r, nbytes, st)

    def destroy(self):
        if self.ptr:
            _call("hv_comm_destroy", self.ptr)
            self.ptr = _VP()


def comm_unique_id() -> bytes:
    buf = C.create_string_buffer(COMM_ID_BYTES)
    _call("hv_comm_unique_id", buf)
    return buf.raw


def ipc_open(handle: bytes) -> int:
    """Map another process's allocation (its ipc_handle) into this process."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("an IPC handle is 64 bytes")
    out = _VP()
    _call("hv_ipc_open", C.create_string_buffer(handle, IPC_HANDLE_BYTES), C.byref(out))
    return int(out.value)


def ipc_close(ptr):
    _call("hv_ipc_close", _p(ptr))


STEP_OPT_INFLIGHT = 1
STEP_OPT_EVICT_FIRST = 2
STEP_OPT_LOCAL_QKV_BARRIER = 3
STEP_OPT_REF_BLAS_RUNS = 5


def step_set_option(option, value):
    """Tuning of the fused step (bulk copies in flight per SM, L2 evict-first streaming);
    results do not change."""
    _call("hv_step_set_option", int(option), int(value))


def attn_decode_noalloc(q, kc, vc, ctx, scale, pos, nq, hd, group, kvstride, stream=0):
    """attn_decode over the library's fixed static scratch: never allocates (see
    hv_attn_decode_noalloc in include/hive_b200.h for its limits)."""
    _call("hv_attn_decode_noalloc", _p(q), _p(kc), _p(vc), _p(ctx), _p(scale), _p(pos), nq,
          hd, group, kvstride, _p(stream))


def silu_mul(gate, up, act, n, stream=0):
    _call("hv_silu_mul", _p(gate), _p(up), _p(act), n, _p(stream))


def vadd(a, b, out, n, stream=0):
    _call("hv_vadd", _p(a), _p(b), _p(out), n, _p(stream))


def gather_emb(emb16, tok, h, hid, stream=0):
    _call("hv_gather_emb", _p(emb16), _p(tok), _p(h), hid, _p(stream))


def argmax_partial(logits, pv, pi, n, parts, stream=0):
    _call("hv_argmax_partial", _p(logits), _p(pv), _p(pi), n, parts, _p(stream))


def argmax_final(pv, pi, tok, gen, step, pos, parts, stream=0):
    _call("hv_argmax_final", _p(pv), _p(pi), _p(tok), _p(gen), _p(step), _p(pos), parts,
          _p(stream))


def argmax_key(logits, n, base, key, stream=0):
    """Fold one vocabulary shard (global ids base..base+n-1) into its 64-bit argmax key."""
    _call("hv_argmax_key", _p(logits), n, base, _p(key), _p(stream))


def argmax_key_final(keys, nkeys, tok, gen, step, pos, stream=0):
    """Token = the best of `nkeys` shard keys; advances tok/gen/step/pos like argmax_f and
    clears the keys."""
    _call("hv_argmax_key_final", _p(keys), nkeys, _p(tok), _p(gen), _p(step), _p(pos),
          _p(stream))


def token_of_key(key: int) -> int:
    """Global token id carried by a 64-bit argmax key (-1 for the empty key 0)."""
    return (~key) & 0xFFFFFFFF if key else -1


def w4_prepacked_size(rows, k, pair_ffn=0):
    a, b = C.c_size_t(), C.c_size_t()
    _call("hv_w4_prepacked_size", rows, k, pair_ffn, C.byref(a), C.byref(b))
    return a.value, b.value


def w4_prepack(b4, sw, rows, k, pair_ffn, pb4, psw, stream=0):
    _call("hv_w4_prepack", _p(b4), _p(sw), rows, k, pair_ffn, _p(pb4), _p(psw), _p(stream))


def a4gv_pp(a8, sa, pb4, psw, dst, k8, rows, pair_ffn=0, stream=0):
    _call("hv_a4gv_pp", _p(a8), _p(sa), _p(pb4), _p(psw), _p(dst), k8, rows, pair_ffn,
          _p(stream))


def w4_prepack_dq(b4, sw, rows, k, pair_ffn, pb4, psw, stream=0):
    """The dq arrangement of the tiles (sizes as w4_prepacked_size) for a4gv_dq."""
    _call("hv_w4_prepack_dq", _p(b4), _p(sw), rows, k, pair_ffn, _p(pb4), _p(psw), _p(stream))


def a4gv_dq(a8, sa, pb4, psw, dst, k8, rows, pair_ffn=0, stream=0):
    """a4gv_pp with dp4a block dots over the dq arrangement (bit-identical results)."""
    _call("hv_a4gv_dq", _p(a8), _p(sa), _p(pb4), _p(psw), _p(dst), k8, rows, pair_ffn,
          _p(stream))


def wait_probe(word, mask, want, limit_ns, status, stream=0):
    """The fused step's bounded wait on a caller's device word (see hv_wait_probe):
    *status becomes HV_E_TIMEOUT (1004) if (*word & mask) != want for limit_ns."""
    _call("hv_wait_probe", _p(word), int(mask), int(want), int(limit_ns), _p(status),
          _p(stream))


def a4gemm_pp(a8, sa, pb4, psw, dst, k8, rows, pair_ffn, ntok, stream=0):
    """a4gv_pp for ntok tokens at once (prompt prefill); rows of dst are tokens."""
    _call("hv_a4gemm_pp", _p(a8), _p(sa), _p(pb4), _p(psw), _p(dst), k8, rows, pair_ffn,
          ntok, _p(stream))


def a4gemm_dq(a8, sa, pb4, psw, dst, k8, rows, pair_ffn, ntok, stream=0):
    """a4gemm_pp over weights in the dq arrangement (same results)."""
    _call("hv_a4gemm_dq", _p(a8), _p(sa), _p(pb4), _p(psw), _p(dst), k8, rows, pair_ffn,
          ntok, _p(stream))


def gather_rows(emb16, tok, h, hid, ntok, stream=0):
    _call("hv_gather_rows", _p(emb16), _p(tok), _p(h), hid, ntok, _p(stream))


def qa8s_rows(src, a8, sa, nb, ntok, stream=0):
    _call("hv_qa8s_rows", _p(src), _p(a8), _p(sa), nb, ntok, _p(stream))


def qk_rows(qkv, qn, kn, cos_t, sin_t, pos0, q_out, kc, vc, nq, nkv, hd, cap, eps, ntok,
            stream=0, f16=False):
    _call("hv_qk_rows_f16" if f16 else "hv_qk_rows", _p(qkv), _p(qn), _p(kn), _p(cos_t),
          _p(sin_t), int(pos0), _p(q_out), _p(kc), _p(vc), nq, nkv, hd, cap, C.c_float(eps),
          ntok, _p(stream))


def attn_rows_scratch(nq, group, cap, ntok) -> tuple[int, int]:
    a, b = C.c_size_t(), C.c_size_t()
    _call("hv_attn_rows_scratch", nq, group, cap, ntok, C.byref(a), C.byref(b))
    return a.value, b.value


def attn_rows(q, kc, vc, ctx, scale, pos0, nq, hd, group, kvstride, ntok, part, ticket,
              stream=0, f16=False):
    _call("hv_attn_rows_f16" if f16 else "hv_attn_rows", _p(q), _p(kc), _p(vc), _p(ctx),
          _p(scale), int(pos0), nq, hd, group, kvstride, ntok, _p(part), _p(ticket),
          _p(stream))


def silu_rows(gu, act, ffn, ntok, stream=0):
    _call("hv_silu_rows", _p(gu), _p(act), ffn, ntok, _p(stream))


def gemv_set_split(enable: bool) -> None:
    """Whether hv_a4gv_pp may run small matrices on the iteration-split kernel (default
    on; the results are identical either way)."""
    _call("hv_gemv_set_split", 1 if enable else 0)


def quantize_w4(w, packed, scale, n, k, stream=0):
    _call("hv_quantize_w4", _p(w), _p(packed), _p(scale), n, k, _p(stream))


class Scalar:
    """Kept for source compatibility with engine/cudrv.py:272-278."""

    __slots__ = ("value",)

    def __init__(self, value: int):
        self.value = int(value)
