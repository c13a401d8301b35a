"""ORACLE — test infrastructure only. Never imported by the product path.

A CPU restatement, in numpy, of the numeric contract of HIVE Limited's batch-1 decode
step (engine/reference.py and the weight format of engine/limited.py). Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use it, to check and time
the product against.

Pinning: every function below is checked against golden vectors produced by running
the reference's own engine/reference.py where its checkout is present
(tests/golden/make_golden.py writes them, tests/test_oracle.py checks them):

* bit-exact: quantize_w4, quantize_act, the int32 block dots, gemv_w4's fp32 output
  (numpy's pairwise summation order restated in `pairwise_sum`), rmsnorm, rope, the
  residual add, the embedding gather and argmax;
* exp-based ops (silu_mul, attention): the reference calls np.exp and OpenBLAS's gemv
  (`keys @ q`), whose results depend on how numpy and OpenBLAS were built and on the
  host's thread count. The oracle restates both (`np_exp`: numpy's float32 SIMD exp;
  `blas_rowdots`: the order OpenBLAS forms each row dot, BLAS_THREADS runs for long
  row counts) in oracle/hv_oracle_c.c, pinned bit for bit against np.exp and `keys @ q`
  of the host that made the golden vectors (tests/test_oracle_c.py). The rest of the
  attention (max, the pairwise w.sum(), the division, the sequential axis-0 sum of
  w * v) is numpy's own, which does not depend on the host.

The compressed-KV lane (kv_round, OracleModel(kv_dtype="f16")) has no counterpart in the
reference: it is the reference's step with each appended k/v row rounded to binary16.
Its rounding is numpy's float32 -> float16 conversion, checked against Python's own
IEEE binary16 packing (struct format 'e') in tests/test_kv16.py.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent))

F32 = np.float32
BLOCK = 32
RMS_EPS = F32(1e-5)          # engine/reference.py:34 (the shipped kernel's epsilon)
PW_BLOCK = 128               # numpy's pairwise-summation leaf size
# OpenBLAS threads on the host that produced the golden vectors (8 cores): gemv calls of
# 128 * rows >= 460800 are split into this many runs of rows, which changes the order of
# the row dots near each run's end (hvo_blas_row_kind).
BLAS_THREADS = 8


# ---------------------------------------------------------------------------
# weight format (engine/limited.py:40-75)
# ---------------------------------------------------------------------------

def quantize_w4(w: np.ndarray):
    """engine/limited.py:40-58: per-32 s=max|w|/7 (0->1), q=clip(round(w/s),-7,7),
    byte-sliced nibble packing. Returns (packed u32 [N,K/8], scale f32 [N,K/32])."""
    n, k = w.shape
    assert k % BLOCK == 0
    blocks = w.astype(F32).reshape(n, k // BLOCK, BLOCK)
    scale = (np.abs(blocks).max(2) / F32(7.0)).astype(F32)
    scale[scale == 0] = F32(1.0)
    q = np.clip(np.round(blocks / scale[:, :, None]), -7, 7).astype(np.int8).reshape(n, k)
    g = (q.view(np.uint8) & 15).astype(np.uint32).reshape(n, k // 8, 8)
    packed = (g[:, :, 0] | (g[:, :, 1] << 8) | (g[:, :, 2] << 16) | (g[:, :, 3] << 24)
              | (g[:, :, 4] << 4) | (g[:, :, 5] << 12) | (g[:, :, 6] << 20)
              | (g[:, :, 7] << 28))
    return np.ascontiguousarray(packed, np.uint32), np.ascontiguousarray(scale)


def unpack_w4(packed: np.ndarray, k: int) -> np.ndarray:
    """engine/reference.py:75-84: the signed int4 values as int8 [N, K]."""
    n = packed.shape[0]
    out = np.zeros((n, k), np.int8)
    for b in range(4):
        lo = ((packed >> (8 * b)) & 0xF).astype(np.int16)
        hi = ((packed >> (8 * b + 4)) & 0xF).astype(np.int16)
        out[:, b::8] = np.where(lo >= 8, lo - 16, lo)
        out[:, 4 + b::8] = np.where(hi >= 8, hi - 16, hi)
    return out


# ---------------------------------------------------------------------------
# numpy's pairwise summation, restated (numpy 2.x float32 add.reduce)
# ---------------------------------------------------------------------------

def pairwise_plan(n: int) -> list[tuple[int, int]]:
    """Leaves (start, length) of numpy's pairwise recursion over n contiguous values:
    n <= 128 is one leaf; otherwise split at n2 = n//2 rounded down to a multiple of 8."""
    if n <= PW_BLOCK:
        return [(0, n)]
    n2 = n // 2
    n2 -= n2 % 8
    return pairwise_plan(n2) + [(s + n2, m) for s, m in pairwise_plan(n - n2)]


def _leaf(x: np.ndarray) -> np.ndarray:
    """One leaf over the last axis: < 8 values -> sequential from +0; otherwise eight
    strided accumulators, the fixed tree ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the
    n % 8 tail added in order."""
    n = x.shape[-1]
    if n < 8:
        res = np.zeros(x.shape[:-1], F32)
        for i in range(n):
            res = (res + x[..., i]).astype(F32)
        return res
    r = x[..., 0:8].astype(F32).copy()
    i = 8
    while i < n - (n % 8):
        r = (r + x[..., i:i + 8]).astype(F32)
        i += 8
    res = (((r[..., 0] + r[..., 1]) + (r[..., 2] + r[..., 3]))
           + ((r[..., 4] + r[..., 5]) + (r[..., 6] + r[..., 7]))).astype(F32)
    while i < n:
        res = (res + x[..., i]).astype(F32)
        i += 1
    return res


def _pairwise(x: np.ndarray) -> np.ndarray:
    n = x.shape[-1]
    if n <= PW_BLOCK:
        return _leaf(x)
    n2 = n // 2
    n2 -= n2 % 8
    return (_pairwise(x[..., :n2]) + _pairwise(x[..., n2:])).astype(F32)


def pairwise_sum(x: np.ndarray) -> np.ndarray:
    """float32 sum over the last axis in numpy's order: (+0) + pairwise(row)."""
    x = np.asarray(x, F32)
    return (F32(0.0) + _pairwise(x)).astype(F32)


# ---------------------------------------------------------------------------
# the ops (engine/reference.py:37-118)
# ---------------------------------------------------------------------------

def rmsnorm(x: np.ndarray, w: np.ndarray, eps=RMS_EPS) -> np.ndarray:
    """engine/reference.py:37-41: y = w * (x / sqrt(mean(x^2) + eps)), row-wise.
    mean = pairwise_sum(x*x) / n in float32; every op separately rounded."""
    x = np.asarray(x, F32)
    n = x.shape[-1]
    ms = (pairwise_sum(x * x) / F32(n)).astype(F32)[..., None]
    return (np.asarray(w, F32) * (x / np.sqrt((ms + F32(eps)).astype(F32)))).astype(F32)


def quantize_act(a: np.ndarray):
    """engine/reference.py:44-59 (= quant_a8s): per-32 s = max|a|/127 (0 -> 1),
    q = trunc(f32(a/s) +- 0.5) clipped to +-127, block sums.
    Returns (q int8 [K], s f32 [K/32], bsum int32 [K/32])."""
    a = np.asarray(a, F32).reshape(-1)
    nb = a.size // BLOCK
    blocks = a.reshape(nb, BLOCK)
    s = (np.abs(blocks).max(1) / F32(127.0)).astype(F32)
    s[s == 0] = F32(1.0)
    half = np.where(blocks < 0, F32(-0.5), F32(0.5)).astype(F32)
    q = np.trunc((blocks / s[:, None]).astype(F32) + half).astype(np.int32)
    q = np.clip(q, -127, 127)
    return q.astype(np.int8).reshape(-1), s, q.sum(1).astype(np.int32)


def block_dots(qw: np.ndarray, qa: np.ndarray) -> np.ndarray:
    """Exact int32 dot of every 32-block: idot[n, b] = sum_j qw[n, 32b+j] * qa[32b+j].
    |idot| <= 7*127*32, so a float32 product-sum of these integers is exact too."""
    n, k = qw.shape
    nb = k // BLOCK
    out = np.empty((n, nb), np.int32)
    qa_b = qa.reshape(nb, BLOCK).astype(F32)
    step = max(1, (1 << 24) // k)
    for r0 in range(0, n, step):
        w = qw[r0:r0 + step].reshape(-1, nb, BLOCK).astype(F32)
        out[r0:r0 + step] = np.einsum("nbk,bk->nb", w, qa_b).astype(np.int32)
    return out


def combine(idot: np.ndarray, sw: np.ndarray, sa: np.ndarray) -> np.ndarray:
    """engine/reference.py:70-72: c = f32(f32(s_w * s_a) * f32(idot)), y = sum over
    blocks in numpy's pairwise order."""
    c = ((sw.astype(F32) * sa[None, :].astype(F32)).astype(F32)
         * idot.astype(F32)).astype(F32)
    return pairwise_sum(c)


def gemv_q(qa, sa, packed, scale, k, qw=None):
    """GEMV from an already-quantised activation. Returns (idot, y)."""
    if qw is None:
        qw = unpack_w4(packed, k)
    idot = block_dots(qw, qa)
    return idot, combine(idot, scale, sa)


def gemv_w4(a, packed, scale, k, qw=None) -> np.ndarray:
    """engine/reference.py:62-72: quantise a, exact int32 block dots, fp32 combine."""
    qa, sa, _ = quantize_act(a)
    return gemv_q(qa, sa, packed, scale, k, qw)[1]


def rope_tables(cap: int, head_dim: int, theta: float):
    """engine/limited.py:330-335 / engine/reference.py:160-164: f32(cos/sin(f64))."""
    half = head_dim // 2
    pos = np.arange(cap, dtype=np.float64)[:, None]
    inv = 1.0 / (theta ** (np.arange(half, dtype=np.float64) * 2.0 / head_dim))
    ang = pos * inv[None, :]
    return np.cos(ang).astype(F32), np.sin(ang).astype(F32)


def rope(vec: np.ndarray, pos: int, cos_t, sin_t) -> np.ndarray:
    """engine/reference.py:87-93: rotate-half [lo*c - hi*s, hi*c + lo*s]."""
    half = vec.shape[1] // 2
    c, s = cos_t[pos].astype(F32), sin_t[pos].astype(F32)
    lo, hi = vec[:, :half].astype(F32), vec[:, half:].astype(F32)
    return np.concatenate([(lo * c).astype(F32) - (hi * s).astype(F32),
                           (hi * c).astype(F32) + (lo * s).astype(F32)], 1).astype(F32)


def silu_mul(gate, up) -> np.ndarray:
    """engine/reference.py:96-101: g * sigma(g) * u, sigma by the sign-split exp form."""
    g = np.asarray(gate, F32)
    sgn = np.where(g < 0, F32(-1.0), F32(1.0)).astype(F32)
    e = np_exp(-(sgn * g))
    sig = (F32(0.5) * (F32(1.0) + sgn * ((F32(1.0) - e) / (F32(1.0) + e)))).astype(F32)
    return (g * sig * np.asarray(up, F32)).astype(F32)


def attention(q, kc, vc, pos: int, group: int, scale: float) -> np.ndarray:
    """engine/reference.py:104-118: causal softmax attention over positions 0..pos,
    kv head = h // group."""
    n_head, dim = q.shape
    out = np.zeros_like(q, dtype=F32)
    for h in range(n_head):
        kvh = h // group
        keys = kc[kvh, : pos + 1].astype(F32)
        vals = vc[kvh, : pos + 1].astype(F32)
        logits = blas_rowdots(keys, q[h]) * F32(scale)
        logits -= logits.max()
        w = np_exp(logits)
        w /= w.sum()
        out[h] = (w[:, None] * vals).sum(0)
    return out


def np_exp(x) -> np.ndarray:
    """np.exp on float32 as numpy's x86-64 SIMD kernel computes it (hvo_np_expf)."""
    x = np.ascontiguousarray(x, F32)
    y = np.empty_like(x)
    _clib().hvo_np_exp_arr(x.ctypes.data, y.ctypes.data, x.size)
    return y


def blas_rowdots(keys, x, threads: int = None) -> np.ndarray:
    """`keys @ x` for keys [T, 128] as OpenBLAS's gemv forms each row dot
    (hvo_blas_rowdots); `threads`: the reference host's OpenBLAS thread count."""
    keys = np.ascontiguousarray(keys, F32)
    x = np.ascontiguousarray(x, F32)
    assert keys.ndim == 2 and keys.shape[1] == 128 and x.shape == (128,)
    out = np.empty(keys.shape[0], F32)
    _clib().hvo_blas_rowdots(keys.ctypes.data, 128, x.ctypes.data, out.ctypes.data,
                             keys.shape[0], BLAS_THREADS if threads is None else threads)
    return out


def argmax(logits) -> int:
    """engine/reference.py:219: first maximal index (ties -> lowest id)."""
    return int(np.argmax(logits))


# ---------------------------------------------------------------------------
# the model step (engine/reference.py:121-225)
# ---------------------------------------------------------------------------

def kv_round(x: np.ndarray, kv_dtype: str) -> np.ndarray:
    """A k or v row as the cache holds it: unchanged for "f32"; for "f16" rounded to
    binary16 (round to nearest, ties to even; overflow to infinity) and widened back."""
    if kv_dtype == "f16":
        return x.astype(np.float16).astype(F32)
    return x


class OracleModel:
    """CPU forward of the whole decode step over already-quantised weights.

    `w` maps: "emb16" f16 [V, hid]; per layer l: f"{l}.an|fn|qn|kn" f32 gains and
    f"{l}.qkv|o|gu|down" -> (packed, scale, K); "onorm"; "head" -> (packed, scale, K).
    qkv rows are [q | k | v] and gu rows are [gate | up], as the reference fuses them.

    kv_dtype "f16" is the compressed-KV lane, which the reference does not have: each k
    and v row is rounded to IEEE binary16 (nearest, ties to even: numpy's astype) when it
    is appended, and attention (engine/reference.py:104-118, unchanged) reads the widened
    values. The caches stay float32 arrays holding those values.
    """

    def __init__(self, cfg, w: dict, max_context: int, eps=RMS_EPS, kv_dtype="f32"):
        if kv_dtype not in ("f32", "f16"):
            raise ValueError(f"kv_dtype={kv_dtype!r}")
        self.kv_dtype = kv_dtype
        self.cfg, self.w, self.cap, self.eps = cfg, w, max_context, F32(eps)
        self.cos, self.sin = rope_tables(max_context, cfg.head_dim, cfg.rope_theta)
        self._qw = {}
        self.reset()

    def reset(self):
        c = self.cfg
        self.KC = np.zeros((c.n_layer, c.n_kv, self.cap, c.head_dim), F32)
        self.VC = np.zeros((c.n_layer, c.n_kv, self.cap, c.head_dim), F32)

    def _gemv(self, name, x):
        packed, scale, k = self.w[name]
        if name not in self._qw:
            self._qw[name] = unpack_w4(packed, k)
        return gemv_w4(x, packed, scale, k, self._qw[name])

    def step(self, token: int, pos: int, head: bool = True):
        c = self.cfg
        qd, nq, nkv = c.head_dim, c.n_head, c.n_kv
        h = self.w["emb16"][token].astype(F32)
        for l in range(c.n_layer):
            hn = rmsnorm(h, self.w[f"{l}.an"], self.eps)
            qkv = self._gemv(f"{l}.qkv", hn)
            q = qkv[: nq * qd].reshape(nq, qd)
            kk = qkv[nq * qd: (nq + nkv) * qd].reshape(nkv, qd)
            v = qkv[(nq + nkv) * qd:].reshape(nkv, qd)
            q = rmsnorm(q, self.w[f"{l}.qn"], self.eps)
            kk = rmsnorm(kk, self.w[f"{l}.kn"], self.eps)
            q = rope(q, pos, self.cos, self.sin)
            kk = rope(kk, pos, self.cos, self.sin)
            self.KC[l][:, pos, :] = kv_round(kk, self.kv_dtype)
            self.VC[l][:, pos, :] = kv_round(v, self.kv_dtype)
            ctx = attention(q, self.KC[l], self.VC[l], pos, c.group,
                            1.0 / np.sqrt(qd)).reshape(-1)
            h = (h + self._gemv(f"{l}.o", ctx)).astype(F32)
            hn = rmsnorm(h, self.w[f"{l}.fn"], self.eps)
            gu = self._gemv(f"{l}.gu", hn)
            act = silu_mul(gu[: c.ffn], gu[c.ffn:])
            h = (h + self._gemv(f"{l}.down", act)).astype(F32)
        self.h_final = h
        if not head:
            return None
        hn = rmsnorm(h, self.w["onorm"], self.eps)
        return self._gemv("head", hn)

    def generate(self, prompt_ids, max_new: int):
        """Greedy, engine/reference.py:211-225. Returns (tokens, list of logits)."""
        self.reset()
        logits = None
        for i, tok in enumerate(prompt_ids):
            logits = self.step(int(tok), i, head=(i == len(prompt_ids) - 1))
        out, all_logits, pos = [], [logits], len(prompt_ids)
        for _ in range(max_new):
            nxt = argmax(logits)
            out.append(nxt)
            logits = self.step(nxt, pos)
            all_logits.append(logits)
            pos += 1
        return out, all_logits


def quantize_model(cfg, tensors: dict) -> dict:
    """Fuse and quantise a name->array model the way the reference does
    (engine/reference.py:133-158). A tied LM head comes from the f16 embedding."""
    c = cfg
    w = {}
    emb = tensors["model.embed_tokens.weight"]
    w["emb16"] = emb.astype(np.float16)
    for l in range(c.n_layer):
        p = f"model.layers.{l}."
        t = lambda n: tensors[p + n].astype(F32)  # noqa: E731
        wqkv = np.concatenate([t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"),
                               t("self_attn.v_proj.weight")], 0)
        wgu = np.concatenate([t("mlp.gate_proj.weight"), t("mlp.up_proj.weight")], 0)
        w[f"{l}.an"] = t("input_layernorm.weight")
        w[f"{l}.fn"] = t("post_attention_layernorm.weight")
        w[f"{l}.qn"] = t("self_attn.q_norm.weight")
        w[f"{l}.kn"] = t("self_attn.k_norm.weight")
        w[f"{l}.qkv"] = quantize_w4(wqkv) + (wqkv.shape[1],)
        w[f"{l}.o"] = quantize_w4(t("self_attn.o_proj.weight")) + (c.n_head * c.head_dim,)
        w[f"{l}.gu"] = quantize_w4(wgu) + (wgu.shape[1],)
        w[f"{l}.down"] = quantize_w4(t("mlp.down_proj.weight")) + (c.ffn,)
    w["onorm"] = tensors["model.norm.weight"].astype(F32)
    head = w["emb16"].astype(F32) if c.tied else tensors["lm_head.weight"].astype(F32)
    w["head"] = quantize_w4(head) + (head.shape[1],)
    return w


# ---------------------------------------------------------------------------
# the C restatement of gemv_q (oracle/hv_oracle_c.c), for the large model sizes
# ---------------------------------------------------------------------------

_CLIB = None


def _clib():
    global _CLIB
    if _CLIB is None:
        import ctypes
        import build_oracle
        lib = ctypes.CDLL(str(build_oracle.build()))
        vp, lg = ctypes.c_void_p, ctypes.c_long
        lib.hvo_gemv.argtypes = [vp, vp, vp, vp, lg, lg, vp, vp]
        lib.hvo_gemv.restype = None
        lib.hvo_pairwise_sum.argtypes = [vp, lg]
        lib.hvo_pairwise_sum.restype = ctypes.c_float
        lib.hvo_quantize_w4.argtypes = [vp, lg, lg, vp, vp]
        lib.hvo_quantize_w4.restype = None
        lib.hvo_np_exp_arr.argtypes = [vp, vp, lg]
        lib.hvo_np_exp_arr.restype = None
        lib.hvo_np_expf.argtypes = [ctypes.c_float]
        lib.hvo_np_expf.restype = ctypes.c_float
        lib.hvo_blas_rowdots.argtypes = [vp, lg, vp, vp, ctypes.c_int, ctypes.c_int]
        lib.hvo_blas_rowdots.restype = None
        lib.hvo_blas_row_kind.argtypes = [ctypes.c_int] * 3
        lib.hvo_blas_row_kind.restype = ctypes.c_int
        _CLIB = lib
    return _CLIB


def gemv_q_c(qa, sa, packed, scale, k, want_idot=False):
    """Same contract as gemv_q, computed by the C oracle (OpenMP over rows)."""
    qa = np.ascontiguousarray(qa, np.int8)
    sa = np.ascontiguousarray(sa, F32)
    packed = np.ascontiguousarray(packed, np.uint32)
    scale = np.ascontiguousarray(scale, F32)
    n = packed.shape[0]
    y = np.empty(n, F32)
    idot = np.empty((n, k // BLOCK), np.int32) if want_idot else None
    _clib().hvo_gemv(qa.ctypes.data, sa.ctypes.data, packed.ctypes.data, scale.ctypes.data,
                     n, k, y.ctypes.data, idot.ctypes.data if want_idot else None)
    return idot, y


def quantize_w4_c(w: np.ndarray):
    """quantize_w4 by the C restatement (OpenMP over rows); bit-identical."""
    w = np.ascontiguousarray(w, F32)
    n, k = w.shape
    packed = np.empty((n, k // 8), np.uint32)
    scale = np.empty((n, k // BLOCK), F32)
    _clib().hvo_quantize_w4(w.ctypes.data, n, k, packed.ctypes.data, scale.ctypes.data)
    return packed, scale


def quantize_model_c(cfg, tensors) -> dict:
    """quantize_model over a name -> array source (dict or iterator of pairs), with the C
    quantiser; keeps only the quantised model on the host."""
    c = cfg
    src = dict(tensors) if isinstance(tensors, dict) else None
    it = None if src is not None else iter(tensors)
    pend = {} if src is None else src

    def take(name):
        while name not in pend:
            k, v = next(it)
            pend[k] = v
        return pend.pop(name)

    w = {}
    emb = take("model.embed_tokens.weight")
    w["emb16"] = emb.astype(np.float16)
    del emb
    if c.tied:
        w["head"] = quantize_w4_c(w["emb16"].astype(F32)) + (c.hidden,)
    for l in range(c.n_layer):
        p = f"model.layers.{l}."
        t = lambda n: take(p + n)  # noqa: E731
        wqkv = np.concatenate([t("self_attn.q_proj.weight"), t("self_attn.k_proj.weight"),
                               t("self_attn.v_proj.weight")], 0)
        w[f"{l}.qkv"] = quantize_w4_c(wqkv) + (c.hidden,)
        del wqkv
        w[f"{l}.o"] = quantize_w4_c(t("self_attn.o_proj.weight")) + (c.n_head * c.head_dim,)
        wgu = np.concatenate([t("mlp.gate_proj.weight"), t("mlp.up_proj.weight")], 0)
        w[f"{l}.gu"] = quantize_w4_c(wgu) + (c.hidden,)
        del wgu
        w[f"{l}.down"] = quantize_w4_c(t("mlp.down_proj.weight")) + (c.ffn,)
        w[f"{l}.an"] = t("input_layernorm.weight").astype(F32)
        w[f"{l}.fn"] = t("post_attention_layernorm.weight").astype(F32)
        w[f"{l}.qn"] = t("self_attn.q_norm.weight").astype(F32)
        w[f"{l}.kn"] = t("self_attn.k_norm.weight").astype(F32)
    w["onorm"] = take("model.norm.weight").astype(F32)
    if not c.tied:
        w["head"] = quantize_w4_c(take("lm_head.weight")) + (c.hidden,)
    return w


def gemv_w4_c(a, packed, scale, k):
    qa, sa, _ = quantize_act(a)
    return gemv_q_c(qa, sa, packed, scale, k)[1]


class FastOracleModel(OracleModel):
    """OracleModel with the GEMVs done by the C restatement (bit-identical)."""

    def _gemv(self, name, x):
        packed, scale, k = self.w[name]
        return gemv_w4_c(x, packed, scale, k)
