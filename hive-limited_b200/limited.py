"""HIVE Limited's batch-1 decode engine, B200-native.

Same public API as engine/limited.py of the reference (Engine, generate, stream,
logits, verify_graph, bits_per_weight, weight_bytes, bind_thread, free, cfg,
device_name, kv_bytes, _graph_ok; quantize_w4 / dequantize_w4 / Config / SafeTensors /
load_model_tensors / BLOCK), with the driver layer replaced: kernels come from
libhive_b200.so (hand-written CUDA for sm_100a) through ctypes (hvdrv.py). No PyTorch,
no CPU fallback.

Two step implementations, both bit-identical by construction:
  * the eager step issues the reference's sequence of kernels one by one
    (engine/limited.py:374-419), each a standalone hv_* entry point;
  * the fused step (default) runs the whole token -- every layer, the LM head and the
    greedy argmax -- as ONE persistent kernel launch (hv_step_launch).
"""
from __future__ import annotations

import ctypes as C
import time

import numpy as np

import hvdrv
import wcache
from w4format import (BLOCK, Config, SafeTensors, dequantize_w4, load_model_tensors,  # noqa: F401
                      quantize_w4)

F32 = np.float32
RMS_EPS = 1e-5          # the shipped rmsnorm kernel's epsilon (engine/reference.py:34)
GVBD = 256              # kept for source compatibility (engine/limited.py:183)
ARGMAX_PARTS = 128      # argmax_p partial count (engine/limited.py:423-425)


class _LayerW(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "qkv_b4", "qkv_sw", "o_b4", "o_sw", "gu_b4", "gu_sw", "dn_b4", "dn_sw",
        "an", "fn", "qn", "kn", "kc", "vc")]


class _StepDesc(C.Structure):
    _fields_ = ([(n, C.c_int) for n in ("n_layer", "hidden", "ffn", "n_head", "n_kv",
                                          "head_dim", "head_rows", "cap")]
                + [("eps", C.c_float), ("attn_scale", C.c_float),
                   ("attn_chunks", C.c_int), ("vocab", C.c_int)]
                + [(n, C.c_void_p) for n in (
                    "layers", "emb16", "onorm", "head_b4", "head_sw", "cos_t", "sin_t",
                    "tok", "pos", "step", "gen", "h", "qkv", "ctx", "act", "logits",
                    "part", "ticket", "amax_v", "amax_i", "barrier", "status", "trace",
                    "plans")]
                + [("world", C.c_int), ("rank", C.c_int), ("peers", C.c_void_p),
                   ("kv_dtype", C.c_int), ("w4_layout", C.c_int),
                   ("kv_base", C.c_void_p), ("kv_rows", C.c_longlong)])


MAX_WORLD = 8


class _StepPeers(C.Structure):
    _fields_ = [(n, C.c_void_p * MAX_WORLD) for n in ("h", "ctx", "act", "barrier", "xchg")]


STEP_HEAD = 1
STEP_ARGMAX = 2


def shard_plan(cfg, world: int, rank: int) -> dict:
    """Rows of every projection held by `rank` of `world` (column-parallel sharding: each
    output element is computed whole on one GPU, so results match one GPU bit for bit).
    -> {"q": (r0, r1) q-proj rows, "kv": (r0, r1) rows of k-proj and of v-proj,
        "hid": (r0, r1) rows of o-proj and down-proj, "ffn": (r0, r1) rows of gate and of
        up, "vocab": (r0, r1) LM-head rows, "n_head", "n_kv", "ffn_n", "vocab_n"}"""
    if not 1 <= world <= MAX_WORLD or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world} (1..{MAX_WORLD} ranks)")
    qd = cfg.head_dim
    for name, n, unit in (("n_head", cfg.n_head, 1), ("n_kv", cfg.n_kv, 1),
                          ("hidden", cfg.hidden, 8), ("ffn", cfg.ffn, 32),
                          ("vocab", cfg.vocab, 1)):
        if n % (world * unit):
            raise ValueError(f"{name} = {n} does not split into {world} shards of whole "
                             f"{unit}-row units")
    nh, nk = cfg.n_head // world, cfg.n_kv // world
    hs, fs, vs = cfg.hidden // world, cfg.ffn // world, cfg.vocab // world
    return {"q": (rank * nh * qd, (rank + 1) * nh * qd),
            "kv": (rank * nk * qd, (rank + 1) * nk * qd),
            "hid": (rank * hs, (rank + 1) * hs), "ffn": (rank * fs, (rank + 1) * fs),
            "vocab": (rank * vs, (rank + 1) * vs),
            "n_head": nh, "n_kv": nk, "ffn_n": fs, "vocab_n": vs}


class _TensorSource:
    """name -> float array, from a dict or from an iterator of (name, array) pairs drawn
    lazily (so a streamed synthetic model is never fully resident on the host)."""

    def __init__(self, src):
        if isinstance(src, dict):
            self._d, self._it = dict(src), None
        else:
            self._d, self._it = {}, iter(src)

    def take(self, name) -> np.ndarray:
        while name not in self._d:
            if self._it is None:
                raise KeyError(f"missing tensor {name!r} -- is this a Qwen3 model?")
            try:
                k, v = next(self._it)
            except StopIteration:
                self._it = None
                continue
            self._d[k] = v
        return self._d.pop(name)


class Engine:
    """Batch-1 resident decode (engine/limited.py:186-659).

    Extra keyword arguments beyond the reference's:
      config / tensors  -- build from a geometry dict and a name -> array source instead
                           of a model directory (synthetic workloads);
      max_context       -- KV capacity (the reference fixes 4096);
      device            -- CUDA device index;
      fused             -- use the one-launch fused step (default) or the eager sequence;
      quantize_on       -- "device" (hv_quantize_w4, bit-identical) or "host" (numpy);
      world / rank / exchange
                        -- column-parallel sharding over `world` GPUs, one process per GPU:
                           this engine holds rank `rank`'s rows of every projection and its
                           heads; `exchange(bytes) -> list[bytes]` is an all-gather over the
                           ranks (any transport) used once, to swap the CUDA IPC handles of
                           the buffers the fused step writes into on every rank;
      prefill           -- "steps" (default): the prompt runs through the decode step one
                           token at a time, as the reference does; "batched": runs of
                           PREFILL_BATCH tokens go through each layer at once (GEMMs over
                           the prepacked weights, hv_*_rows kernels), with results
                           bit-identical to the eager token-by-token prefill (one GPU);
      weight_cache / cache_tag
                        -- a directory of device-ready weights (wcache.py): on a hit the
                           engine uploads the cached prepacked int4 weights, embedding and
                           norms and reads no checkpoint; on a miss it loads as usual and
                           then writes the entry. The entry is keyed by the model
                           directory's files, or by `cache_tag` for `tensors=` sources.
                           `cache_hit` tells which happened (None without a cache).
      gemv_layout       -- "pp" (default): weight tiles for tensor-pipe block dots
                           (hv_w4_prepack); "dq": the same tiles arranged for dp4a block
                           dots (hv_w4_prepack_dq, hv_a4gv_dq, hv_a4gemm_dq). Results are
                           bit-identical; only the speed differs.
      kv_dtype          -- "f32" (default): the reference's fp32 KV cache; "f16": the
                           compressed-KV lane, an IEEE binary16 cache (half the KV bytes
                           per step). Each k/v row is rounded to nearest-even binary16 when
                           appended and attention reads the widened values; the results
                           then follow the oracle run with that rounding, not the
                           reference's fp32 cache.
    """

    def __init__(self, model_dir=None, kernels_dir=None, verify_kernels=True, quiet=False, *,
                 config=None, tensors=None, max_context=None, device=0, fused=True,
                 quantize_on="device", world=1, rank=0, exchange=None, weight_cache=None,
                 cache_tag=None, prefill="steps", kv_dtype="f32", gemv_layout="pp"):
        if config is None:
            self.cfg = Config.load(model_dir)
        else:
            self.cfg = config if isinstance(config, Config) else Config(config)
        if max_context is not None:
            self.cfg.max_context = int(max_context)
        self.quiet = quiet
        self.fused = bool(fused)
        self._buffers: list[int] = []
        self._opened: list[int] = []
        self.world, self.rank = int(world), int(rank)
        if prefill not in ("steps", "batched"):
            raise ValueError(f"prefill={prefill!r}: 'steps' or 'batched'")
        if prefill == "batched" and self.world > 1:
            raise ValueError("the batched prefill runs on one GPU (world = 1)")
        self.prefill_mode = prefill
        if kv_dtype not in ("f32", "f16"):
            raise ValueError(f"kv_dtype={kv_dtype!r}: 'f32' or 'f16'")
        self.kv_dtype = kv_dtype
        self.kv_f16 = kv_dtype == "f16"
        if gemv_layout not in ("pp", "dq"):
            raise ValueError(f"gemv_layout={gemv_layout!r}: 'pp' or 'dq'")
        self.gemv_layout = gemv_layout
        self._pf = None
        self.shard = shard_plan(self.cfg, self.world, self.rank)
        if self.world > 1 and (not self.fused or exchange is None):
            raise ValueError("a sharded engine runs the fused step and needs `exchange`")
        self._exchange = exchange
        self.d_peers = None
        self.cache_hit = None
        key = ident = None
        if weight_cache is not None:          # argument errors before any device work
            key, ident = wcache.entry_key(self.cfg, self.world, self.rank,
                                          model_dir=None if cache_tag is not None else model_dir,
                                          tag=cache_tag, w4_layout=gemv_layout)
        hvdrv.load(kernels_dir, verify=verify_kernels)
        hvdrv.init()
        self.dev = hvdrv.device(device)
        major, minor = hvdrv.compute_capability(self.dev)
        if (major, minor) != (10, 0):
            raise RuntimeError(f"libhive_b200 is built for sm_100a (B200); this device is "
                               f"{major}.{minor}")
        self.ctx = hvdrv.retain_primary_context(self.dev)
        self.device_name = hvdrv.device_name(self.dev)
        self._graph = self._graph_exec = 0
        self._graph_ok = None
        self._stream = 0
        self._stream_cur = 0
        try:
            entry = wcache.open_entry(weight_cache, key) if weight_cache is not None else None
            if entry is not None:
                self._upload_cached(entry)
                self.cache_hit = True
            else:
                src = _TensorSource(tensors if tensors is not None
                                    else load_model_tensors(model_dir))
                self._upload_weights(src, quantize_on)
                del src
                if weight_cache is not None:
                    self._save_cache(weight_cache, key, ident)
                    self.cache_hit = False
            self._alloc_state()
        except BaseException:
            # the caller gets no engine to free(): release what was allocated so far
            self.free()
            raise

    # -- setup ----------------------------------------------------------------------

    def _log(self, msg):
        if not self.quiet:
            print(msg, flush=True)

    def _alloc(self, nbytes: int) -> int:
        p = hvdrv.alloc(max(int(nbytes), 16))
        self._buffers.append(p)
        return p

    def _up(self, arr: np.ndarray) -> int:
        arr = np.ascontiguousarray(arr)
        p = self._alloc(arr.nbytes)
        hvdrv.upload(p, arr.ctypes.data, arr.nbytes)
        return p

    def _up_w4(self, parts: list[np.ndarray], pair_ffn: int = 0):
        """Quantise rows [part0 | part1 | ...] to the per-32 int4 form, upload, and reorder
        into the GEMV's tile-interleaved layout (hv_w4_prepack; pair_ffn > 0 pairs gate
        and up rows). -> (pb4, psw, K, N, pair_ffn)"""
        k = parts[0].shape[1]
        n = sum(p.shape[0] for p in parts)
        tmp = []                          # the reference-layout copy, freed below
        try:
            if self._quantize_on == "host":
                w = np.concatenate([p.astype(F32, copy=False) for p in parts], 0)
                packed, scale = quantize_w4(w)
                b4 = hvdrv.alloc(packed.nbytes)
                tmp.append(b4)
                sw = hvdrv.alloc(scale.nbytes)
                tmp.append(sw)
                hvdrv.upload(b4, packed.ctypes.data, packed.nbytes)
                hvdrv.upload(sw, scale.ctypes.data, scale.nbytes)
            else:
                b4 = hvdrv.alloc(n * k // 2)
                tmp.append(b4)
                sw = hvdrv.alloc(n * k // BLOCK * 4)
                tmp.append(sw)
                off = 0
                for p in parts:
                    p = np.ascontiguousarray(p, dtype=F32)
                    hvdrv.upload(self._stage + off, p.ctypes.data, p.nbytes)
                    off += p.nbytes
                hvdrv.quantize_w4(self._stage, b4, sw, n, k)
            nib_bytes, sc_bytes = hvdrv.w4_prepacked_size(n, k, pair_ffn)
            pb4, psw = self._alloc(nib_bytes), self._alloc(sc_bytes)
            prepack = hvdrv.w4_prepack_dq if self.gemv_layout == "dq" else hvdrv.w4_prepack
            prepack(b4, sw, n, k, pair_ffn, pb4, psw)
            hvdrv.synchronize()
        finally:
            for q in tmp:
                hvdrv.free(q)
        return pb4, psw, k, n, pair_ffn

    def _upload_weights(self, src: _TensorSource, quantize_on: str):
        c = self.cfg
        qd, nq, nkv = c.head_dim, c.n_head, c.n_kv
        self._quantize_on = quantize_on
        self._stage = 0
        if quantize_on == "device":
            elems = max((nq + 2 * nkv) * qd * c.hidden, 2 * c.ffn * c.hidden,
                        c.hidden * nq * qd, c.hidden * c.ffn, c.vocab * c.hidden)
            self._stage = hvdrv.alloc(elems * 4)
        try:
            self._log(f"quantizing {c.n_layer} layers to per-32 int4 ...")
            emb = src.take("model.embed_tokens.weight")
            emb16 = emb.astype(np.float16)
            del emb
            self.d_emb16 = self._up(emb16)
            sh = self.shard
            v0, v1 = sh["vocab"]
            if c.tied:                        # the reference quantises the f16 copy
                self.head = self._up_w4([emb16[v0:v1].astype(F32)])
            del emb16
            self.layers = []
            for l in range(c.n_layer):
                p = f"model.layers.{l}."
                t = lambda n: src.take(p + n)  # noqa: E731
                (q0, q1), (k0, k1) = sh["q"], sh["kv"]
                (h0, h1), (f0, f1) = sh["hid"], sh["ffn"]
                qkv = self._up_w4([t("self_attn.q_proj.weight")[q0:q1],
                                   t("self_attn.k_proj.weight")[k0:k1],
                                   t("self_attn.v_proj.weight")[k0:k1]])
                o = self._up_w4([t("self_attn.o_proj.weight")[h0:h1]])
                gu = self._up_w4([t("mlp.gate_proj.weight")[f0:f1],
                                  t("mlp.up_proj.weight")[f0:f1]], pair_ffn=f1 - f0)
                down = self._up_w4([t("mlp.down_proj.weight")[h0:h1]])
                self.layers.append({
                    "an": self._up(t("input_layernorm.weight").astype(F32)),
                    "fn": self._up(t("post_attention_layernorm.weight").astype(F32)),
                    "qn": self._up(t("self_attn.q_norm.weight").astype(F32)),
                    "kn": self._up(t("self_attn.k_norm.weight").astype(F32)),
                    "qkv": qkv, "o": o, "gu": gu, "down": down,
                })
                if (l + 1) % 7 == 0:
                    self._log(f"  {l + 1}/{c.n_layer}")
            self.d_onorm = self._up(src.take("model.norm.weight").astype(F32))
            if not c.tied:
                self.head = self._up_w4([src.take("lm_head.weight")[v0:v1]])
            self.n_head_rows = self.head[3]
        finally:
            if self._stage:
                hvdrv.free(self._stage)
                self._stage = 0

    # -- the weight cache (wcache.py) -------------------------------------------------

    def _download(self, ptr: int, shape, dtype) -> np.ndarray:
        out = np.empty(shape, dtype)
        hvdrv.download(out.ctypes.data, ptr, out.nbytes)
        return out

    def _cache_items(self):
        """(name, kind, device object, shape, dtype) of every uploaded weight."""
        c = self.cfg
        yield "emb16", "array", self.d_emb16, (c.vocab, c.hidden), np.float16
        for l, L in enumerate(self.layers):
            for nm, n in (("an", c.hidden), ("fn", c.hidden), ("qn", c.head_dim),
                          ("kn", c.head_dim)):
                yield f"{l}.{nm}", "array", L[nm], (n,), F32
            for nm in ("qkv", "o", "gu", "down"):
                yield f"{l}.{nm}", "w4", L[nm], None, None
        yield "onorm", "array", self.d_onorm, (c.hidden,), F32
        yield "head", "w4", self.head, None, None

    def _save_cache(self, root, key: str, ident: dict):
        w = wcache.EntryWriter(root, key, ident)
        try:
            for name, kind, obj, shape, dtype in self._cache_items():
                if kind == "array":
                    w.add_array(name, self._download(obj, shape, dtype))
                else:
                    pb4, psw, k, n, pair = obj
                    nib, scb = hvdrv.w4_prepacked_size(n, k, pair)
                    w.add_w4(name, self._download(pb4, (nib,), np.uint8),
                             self._download(psw, (scb,), np.uint8), k, n, pair)
            path = w.commit()
        except BaseException:
            w.abort()
            raise
        self._log(f"weight cache written: {path}")

    def _upload_cached(self, e):
        """Upload a cache entry (the bytes _save_cache downloaded, unchanged)."""
        c = self.cfg
        sh = self.shard
        qd = c.head_dim
        want_rows = {"qkv": (sh["n_head"] + 2 * sh["n_kv"]) * qd,
                     "o": sh["hid"][1] - sh["hid"][0], "gu": 2 * sh["ffn_n"],
                     "down": sh["hid"][1] - sh["hid"][0]}
        want_k = {"qkv": c.hidden, "o": c.n_head * qd, "gu": c.hidden, "down": c.ffn}

        def up_w4(name, rows=None, k=None):
            nib, sc, kk, n, pair = e.w4(name)
            if (rows is not None and n != rows) or (k is not None and kk != k):
                raise ValueError(f"weight cache {e.path}: {name} is {n}x{kk}, "
                                 f"expected {rows}x{k}")
            if (nib.nbytes, sc.nbytes) != hvdrv.w4_prepacked_size(n, kk, pair):
                raise ValueError(f"weight cache {e.path}: {name} has the wrong byte count")
            return self._up(nib), self._up(sc), kk, n, pair

        self._quantize_on = "cache"
        self._log(f"loading device-ready weights from {e.path} ...")
        self.d_emb16 = self._up(e.array("emb16"))
        self.layers = []
        for l in range(c.n_layer):
            d = {nm: self._up(e.array(f"{l}.{nm}")) for nm in ("an", "fn", "qn", "kn")}
            for nm in ("qkv", "o", "gu", "down"):
                d[nm] = up_w4(f"{l}.{nm}", want_rows[nm], want_k[nm])
            self.layers.append(d)
        self.d_onorm = self._up(e.array("onorm"))
        self.head = up_w4("head", sh["vocab_n"], c.hidden)
        self.n_head_rows = self.head[3]
        hvdrv.synchronize()

    def _alloc_state(self):
        c = self.cfg
        hid, ffn, qd = c.hidden, c.ffn, c.head_dim
        nq, cap = c.n_head, c.max_context
        nkv = self.shard["n_kv"]                     # this rank's kv heads (all, unsharded)
        qkv_rows = (self.shard["n_head"] + 2 * nkv) * qd
        wide = max(hid, ffn, nq * qd)
        self.d_h = self._alloc(hid * 4)
        self.d_hn = self._alloc(hid * 4)
        self.d_qkv = self._alloc(qkv_rows * 4)
        self.d_ctx = self._alloc(nq * qd * 4)
        self.d_o = self._alloc(hid * 4)
        self.d_gu = self._alloc(2 * ffn * 4)
        self.d_act = self._alloc(ffn * 4)
        self.d_logits = self._alloc(self.n_head_rows * 4)
        self.d_a8 = self._alloc(wide)
        self.d_sa = self._alloc(2 * (wide // BLOCK) * 4)
        # KV cache: f32 (or binary16), one allocation, [layer][k|v][n_kv][cap][hd]
        esz = 2 if self.kv_f16 else 4
        self.kv_bytes = 2 * c.n_layer * nkv * cap * qd * esz
        self.d_kv = self._alloc(self.kv_bytes)
        per = nkv * cap * qd * esz
        self.KC = [self.d_kv + (2 * l) * per for l in range(c.n_layer)]
        self.VC = [self.d_kv + (2 * l + 1) * per for l in range(c.n_layer)]
        hvdrv.memset8(self.d_kv, 0, self.kv_bytes)
        half = qd // 2
        pos = np.arange(cap, dtype=np.float64)[:, None]
        inv = 1.0 / (c.rope_theta ** (np.arange(half, dtype=np.float64) * 2.0 / qd))
        ang = pos * inv[None, :]
        self.d_cos = self._up(np.cos(ang).astype(F32))
        self.d_sin = self._up(np.sin(ang).astype(F32))
        self.attn_scale = F32(1.0 / np.sqrt(qd))
        self.d_scale = self._up(np.array([self.attn_scale], F32))
        self.d_tok = self._alloc(4)
        self.d_pos = self._alloc(4)
        self.d_step = self._alloc(4)
        self.d_pv = self._alloc(ARGMAX_PARTS * 4)
        self.d_pi = self._alloc(ARGMAX_PARTS * 4)
        self.d_gen = self._alloc((cap + 1) * 4)
        hvdrv.attn_reserve(nkv, c.group, cap)
        self._build_desc()

    def _build_desc(self):
        """The fused step's descriptor and its scratch (engine/limited.py has no
        equivalent: the reference issues each kernel separately)."""
        c = self.cfg
        sh = self.shard
        grid, threads = C.c_int(), C.c_int()
        smem, chunks, part = C.c_size_t(), C.c_int(), C.c_size_t()
        hvdrv._call("hv_step_config", sh["n_kv"], c.group, c.max_context, C.byref(grid),
                    C.byref(threads), C.byref(smem), C.byref(chunks), C.byref(part))
        self.step_grid = grid.value
        lw = (_LayerW * c.n_layer)()
        for l, w in enumerate(self.layers):
            lw[l] = _LayerW(w["qkv"][0], w["qkv"][1], w["o"][0], w["o"][1], w["gu"][0],
                            w["gu"][1], w["down"][0], w["down"][1], w["an"], w["fn"],
                            w["qn"], w["kn"], self.KC[l], self.VC[l])
        self.d_layers = self._alloc(C.sizeof(lw))
        hvdrv.upload(self.d_layers, C.addressof(lw), C.sizeof(lw))
        self.d_part = self._alloc(part.value * 4)
        self.d_ticket = self._alloc((2 * sh["n_kv"] + 1) * 4)
        hvdrv.memset8(self.d_ticket, 0, (2 * sh["n_kv"] + 1) * 4)
        self.d_amax_v = self._alloc(grid.value * 4)
        self.d_amax_i = self._alloc(grid.value * 4)
        self.d_barrier = self._alloc(16)
        self.d_status = self._alloc(4)
        hvdrv.memset8(self.d_barrier, 0, 16)
        hvdrv.memset8(self.d_status, 0, 4)
        nbytes = C.c_size_t()
        hvdrv._call("hv_step_plans_bytes", C.byref(nbytes))
        plans = C.create_string_buffer(nbytes.value)
        hvdrv._call("hv_step_plans", c.hidden, c.n_head * c.head_dim, c.ffn, plans,
                    nbytes.value)
        self.d_plans = self._alloc(nbytes.value)
        hvdrv.upload(self.d_plans, C.addressof(plans), nbytes.value)
        hb4, hsw, _, hn, _ = self.head
        if self.world > 1:
            self._connect_peers()
        self._desc = _StepDesc(
            c.n_layer, c.hidden, sh["ffn_n"], sh["n_head"], sh["n_kv"], c.head_dim, hn,
            c.max_context,
            RMS_EPS, float(self.attn_scale), chunks.value, c.vocab,
            self.d_layers, self.d_emb16, self.d_onorm, hb4, hsw, self.d_cos, self.d_sin,
            self.d_tok, self.d_pos, self.d_step, self.d_gen, self.d_h, self.d_qkv,
            self.d_ctx, self.d_act, self.d_logits, self.d_part, self.d_ticket,
            self.d_amax_v, self.d_amax_i, self.d_barrier, self.d_status, None, self.d_plans,
            self.world, self.rank, self.d_peers, 1 if self.kv_f16 else 0,
            1 if self.gemv_layout == "dq" else 0,
            self.d_kv, 2 * c.n_layer * sh["n_kv"] * c.max_context)

    def _connect_peers(self):
        """Swap CUDA IPC handles of the buffers every rank's step writes into (residual,
        quantised attention output and SiLU output, barrier word, argmax exchange) and
        upload the peer table. The barrier and exchange words are zeroed before the swap,
        so no rank's first launch can meet a stale word."""
        self.d_xchg = self._alloc((MAX_WORLD + 1) * 4 * 4)
        hvdrv.memset8(self.d_xchg, 0, (MAX_WORLD + 1) * 4 * 4)
        hvdrv.synchronize()
        mine = [self.d_h, self.d_ctx, self.d_act, self.d_barrier, self.d_xchg]
        blob = b"".join(hvdrv.ipc_handle(p) for p in mine)
        blobs = self._exchange(blob)
        if len(blobs) != self.world:
            raise RuntimeError(f"exchange returned {len(blobs)} entries for {self.world} ranks")
        peers = _StepPeers()
        n = hvdrv.IPC_HANDLE_BYTES
        for k, b in enumerate(blobs):
            for j, name in enumerate(("h", "ctx", "act", "barrier", "xchg")):
                if k == self.rank:
                    ptr = mine[j]
                else:
                    ptr = hvdrv.ipc_open(bytes(b[j * n:(j + 1) * n]))
                    self._opened.append(ptr)
                getattr(peers, name)[k] = ptr
        self.d_peers = self._alloc(C.sizeof(peers))
        hvdrv.upload(self.d_peers, C.addressof(peers), C.sizeof(peers))

    def _set_i32(self, ptr: int, value: int):
        hvdrv.upload(ptr, np.array([value], np.int32).ctypes.data, 4)

    def _get_i32(self, ptr: int) -> int:
        out = np.zeros(1, np.int32)
        hvdrv.download(out.ctypes.data, ptr, 4)
        return int(out[0])

    # -- the decode step ------------------------------------------------------------------

    def _gemv(self, src, w4, dst):
        """quantize activations to per-32 int8, then the exact-int32 int4 GEMV."""
        pb4, psw, k, n, pair = w4
        s = self._stream_cur
        hvdrv.qa8s(src, self.d_a8, self.d_sa, k // BLOCK, s)
        gemv = hvdrv.a4gv_dq if self.gemv_layout == "dq" else hvdrv.a4gv_pp
        gemv(self.d_a8, self.d_sa, pb4, psw, dst, k // 8, n, pair, s)

    def _step_eager(self):
        """One transformer step at d_pos, kernel by kernel (engine/limited.py:374-419)."""
        c = self.cfg
        hid, ffn, qd = c.hidden, c.ffn, c.head_dim
        nq, nkv, cap = c.n_head, c.n_kv, c.max_context
        s = self._stream_cur
        dq = self.d_qkv
        dk = self.d_qkv + nq * qd * 4
        dv = self.d_qkv + (nq + nkv) * qd * 4
        hvdrv.gather_emb(self.d_emb16, self.d_tok, self.d_h, hid, s)
        for l, w in enumerate(self.layers):
            hvdrv.rmsnorm(self.d_h, self.d_hn, w["an"], 1, hid, RMS_EPS, s)
            self._gemv(self.d_hn, w["qkv"], self.d_qkv)
            hvdrv.rmsnorm(dq, dq, w["qn"], nq, qd, RMS_EPS, s)
            hvdrv.rmsnorm(dk, dk, w["kn"], nkv, qd, RMS_EPS, s)
            hvdrv.rope(dq, self.d_cos, self.d_sin, self.d_pos, nq, qd // 2, s)
            hvdrv.rope(dk, self.d_cos, self.d_sin, self.d_pos, nkv, qd // 2, s)
            hvdrv.kv_append(dk, dv, self.KC[l], self.VC[l], self.d_pos, nkv, qd, cap, s,
                            f16=self.kv_f16)
            hvdrv.attn_decode(dq, self.KC[l], self.VC[l], self.d_ctx, self.d_scale,
                              self.d_pos, nq, qd, c.group, cap * qd, s, f16=self.kv_f16)
            self._gemv(self.d_ctx, w["o"], self.d_o)
            hvdrv.vadd(self.d_h, self.d_o, self.d_h, hid, s)
            hvdrv.rmsnorm(self.d_h, self.d_hn, w["fn"], 1, hid, RMS_EPS, s)
            self._gemv(self.d_hn, w["gu"], self.d_gu)
            hvdrv.silu_mul(self.d_gu, self.d_gu + ffn * 4, self.d_act, ffn, s)
            self._gemv(self.d_act, w["down"], self.d_o)
            hvdrv.vadd(self.d_h, self.d_o, self.d_h, hid, s)
        hvdrv.rmsnorm(self.d_h, self.d_hn, self.d_onorm, 1, hid, RMS_EPS, s)
        self._gemv(self.d_hn, self.head, self.d_logits)

    def _argmax_into_next(self):
        """Pick the next token and advance tok/pos/step on device (limited.py:421-428)."""
        s = self._stream_cur
        hvdrv.argmax_partial(self.d_logits, self.d_pv, self.d_pi, self.n_head_rows,
                             ARGMAX_PARTS, s)
        hvdrv.argmax_final(self.d_pv, self.d_pi, self.d_tok, self.d_gen, self.d_step,
                           self.d_pos, ARGMAX_PARTS, s)

    def _step_fused(self, flags: int):
        hvdrv._call("hv_step_launch", C.byref(self._desc), int(flags),
                    C.c_void_p(self._stream_cur))

    TRACE_PHASES = ("qkv_prologue", "qkv_gemv", "barrier1", "attention", "barrier2",
                    "o_prologue", "o_gemv", "barrier3", "gu_prologue", "gu_gemv", "barrier4",
                    "down_prologue", "down_gemv", "barrier5")
    TRACE_WAITS = ("wait_attn_scores", "wait_attn_values", "wait_qkv_gemv", "wait_gu_gemv",
                   "attn_scores_busy_kcycles")
    TRACE_ATTN = ("attn_heads", "attn_scores", "attn_scores_out", "attn_ctx_wait",
                  "attn_ctx_sum", "attn_ctx_chain")

    def profile_step(self, flags: int = STEP_HEAD | STEP_ARGMAX) -> dict:
        """Run one fused step at the current tok/pos with the per-phase trace on.

        Returns {"total_us", "phases": {name: {"median_us", "max_us"}}, "raw": ns array
        [grid, stride]} where each phase's duration is taken per CTA and summed over the
        layers (median and max over CTAs)."""
        c = self.cfg
        stride = 10 + 28 * c.n_layer
        n = self.step_grid * stride
        buf = hvdrv.alloc(n * 8)
        try:
            hvdrv.memset8(buf, 0, n * 8)
            self._desc.trace = buf
            self._step_fused(flags)
            hvdrv.synchronize()
            self._check_status()
            raw = np.zeros((self.step_grid, stride), np.uint64)
            hvdrv.download(raw.ctypes.data, buf, raw.nbytes)
        finally:
            self._desc.trace = None
            hvdrv.free(buf)
        t = raw.astype(np.int64)
        t = t - t[:, :1]
        out = {}
        def prev_mark(l, k):      # the mark that ends the phase before (layer l, mark k)
            if k > 0:
                return 2 + 28 * l + k - 1
            return 1 if l == 0 else 2 + 28 * (l - 1) + 13

        for k, name in enumerate(self.TRACE_PHASES):
            idx = np.array([2 + 28 * l + k for l in range(c.n_layer)])
            pidx = np.array([prev_mark(l, k) for l in range(c.n_layer)])
            d = t[:, idx] - t[:, pidx]
            out[name] = {"median_us": float(np.median(d, axis=0).sum() / 1e3),
                         "max_us": float(d.max(axis=0).sum() / 1e3)}
        # inside the attention, CTAs that had a work item (the marks stay 0 otherwise)
        prev = 2
        for k, name in zip(range(14, 20), self.TRACE_ATTN):
            busy = raw[:, 2 + k] != 0       # phase B marks: only the CTAs of a ctx item
            idx = np.array([2 + 28 * l + k for l in range(c.n_layer)])
            d = (t[:, idx] - t[:, idx - k + prev])[busy]
            prev = k
            if d.size:
                out[name] = {"median_us": float(np.median(d, axis=0).sum() / 1e3),
                             "max_us": float(d.max(axis=0).sum() / 1e3)}
        for k, name in zip(range(21, 26), self.TRACE_WAITS):
            idx = np.array([2 + 28 * l + k for l in range(c.n_layer)])
            d = raw[:, idx].astype(np.int64)
            out[name] = {"median_us": float(np.median(d, axis=0).sum() / 1e3),
                         "max_us": float(d.max(axis=0).sum() / 1e3)}
        for name, k0, k1 in (("qkv_pro_load", None, 26), ("qkv_pro_sumsq", 26, 27),
                             ("qkv_pro_quant", 27, 0)):
            idx1 = np.array([2 + 28 * l + k1 for l in range(c.n_layer)])
            idx0 = (np.array([prev_mark(l, 0) for l in range(c.n_layer)]) if k0 is None
                    else np.array([2 + 28 * l + k0 for l in range(c.n_layer)]))
            d = t[:, idx1] - t[:, idx0]
            out[name] = {"median_us": float(np.median(d, axis=0).sum() / 1e3),
                         "max_us": float(d.max(axis=0).sum() / 1e3)}
        th = 2 + 28 * c.n_layer
        for k, name in enumerate(("head_prologue", "head_gemv", "argmax")):
            d = t[:, th + k] - t[:, th + k - 1 if k else prev_mark(c.n_layer, 0)]
            out[name] = {"median_us": float(np.median(d) / 1e3), "max_us": float(d.max() / 1e3)}
        out["setup"] = {"median_us": float(np.median(t[:, 1]) / 1e3),
                        "max_us": float(t[:, 1].max() / 1e3)}
        for k, name in zip(range(3, 8), ("producer_wait_slot_us", "producer_wait_flight_us",
                                          "producer_slots", "ctx_wait_slots_us",
                                          "ctx_sum_us")):
            v = raw[:, th + k].astype(np.float64) / (1.0 if k == 5 else 1e3)
            out[name] = {"median_us": float(np.median(v)), "max_us": float(v.max())}
        last = flags & STEP_ARGMAX and th + 2 or (flags & STEP_HEAD and th + 1 or th - 1)
        return {"total_us": float(t[:, last].max() / 1e3), "phases": out, "raw": raw}

    def step_status(self) -> int:
        """Nonzero if a bounded wait inside the fused step ran out (HV_E_TIMEOUT)."""
        return self._get_i32(self.d_status)

    def reset_step_state(self):
        """Clear the fused step's barrier/ticket/status words after a failed launch."""
        hvdrv.synchronize()
        hvdrv.memset8(self.d_barrier, 0, 16)
        hvdrv.memset8(self.d_status, 0, 4)
        hvdrv.memset8(self.d_ticket, 0, (2 * self.shard["n_kv"] + 1) * 4)

    def _check_status(self):
        st = self.step_status()
        if st:
            self.reset_step_state()
            raise hvdrv.CudaError("hv_step_launch", st,
                                  "a bounded device-side wait ran out; state was reset")

    def _prefill_token(self, tok: int, pos: int, last_flags):
        """Step one prompt token. `last_flags` is None for every prompt token but the last;
        for the last it is the fused step's flags (the eager step always runs the head)."""
        self._set_i32(self.d_tok, int(tok))
        self._set_i32(self.d_pos, pos)
        if self.fused:
            self._step_fused(0 if last_flags is None else last_flags)
        else:
            self._step_eager()

    def _decode_one(self):
        """One decode iteration (engine/limited.py:479-484).

        Eager: argmax of the current logits -> tok/gen/step/pos, then the step at the new
        position. Fused: the same work in the other order inside one launch -- the step
        at the current tok/pos, its LM head, then argmax -> tok/gen/step/pos -- because
        the fused prefill's last launch already took the first argmax. Either way an
        iteration is one full step, and token i sits in gen[i] once iteration i is done.
        """
        if self.fused:
            self._step_fused(STEP_HEAD | STEP_ARGMAX)
        else:
            self._argmax_into_next()
            self._step_eager()

    def bind_thread(self):
        """Bind this engine's device to the calling thread (engine/limited.py:430-436)."""
        hvdrv.set_current(self.ctx)

    # -- public API -------------------------------------------------------------------

    def _check_len(self, prompt_ids, max_new):
        c = self.cfg
        if not prompt_ids:
            raise ValueError("prompt_ids is empty")
        if len(prompt_ids) + max_new > c.max_context:
            raise ValueError(
                f"{len(prompt_ids)} prompt + {max_new} new exceeds the {c.max_context}-token "
                "context of this engine")

    def _prefill(self, prompt_ids, last_flags=STEP_HEAD | STEP_ARGMAX):
        if self.prefill_mode == "batched":
            self._prefill_batched(prompt_ids, argmax=bool(last_flags & STEP_ARGMAX))
            return
        self._set_i32(self.d_step, 0)
        hvdrv.memset8(self.d_gen, 0, (self.cfg.max_context + 1) * 4)
        n = len(prompt_ids)
        for i, tok in enumerate(prompt_ids):
            self._prefill_token(tok, i, last_flags if i == n - 1 else None)

    # ---- batched prefill --------------------------------------------------------------

    PREFILL_BATCH = 256      # prompt tokens that go through a layer together

    def _prefill_buffers(self) -> dict:
        """Device buffers of one run of PREFILL_BATCH tokens (allocated on first use)."""
        if self._pf is not None:
            return self._pf
        c = self.cfg
        b, hid, ffn, qd, nq, nkv = (self.PREFILL_BATCH, c.hidden, c.ffn, c.head_dim, c.n_head,
                                    c.n_kv)
        wide = max(hid, ffn, nq * qd)
        part_b, ticket_b = hvdrv.attn_rows_scratch(nq, c.group, c.max_context, b)
        pf = {"n": b, "tok": self._alloc(b * 4), "h": self._alloc(b * hid * 4),
              "hn": self._alloc(b * hid * 4), "a8": self._alloc(b * wide),
              "sa": self._alloc(b * 2 * (wide // BLOCK) * 4),
              "qkv": self._alloc(b * (nq + 2 * nkv) * qd * 4), "q": self._alloc(b * nq * qd * 4),
              "ctx": self._alloc(b * nq * qd * 4), "o": self._alloc(b * hid * 4),
              "gu": self._alloc(b * 2 * ffn * 4), "act": self._alloc(b * ffn * 4),
              "part": self._alloc(part_b), "ticket": self._alloc(ticket_b)}
        hvdrv.memset8(pf["ticket"], 0, ticket_b)
        self._pf = pf
        return pf

    def _gemm(self, src, w4, dst, m: int):
        """quant_a8s per row, then the W4A8 GEMM of m tokens (rows of src and dst)."""
        pb4, psw, k, n, pair = w4
        s, pf = self._stream_cur, self._pf
        hvdrv.qa8s_rows(src, pf["a8"], pf["sa"], k // BLOCK, m, s)
        gemm = hvdrv.a4gemm_dq if self.gemv_layout == "dq" else hvdrv.a4gemm_pp
        gemm(pf["a8"], pf["sa"], pb4, psw, dst, k // 8, n, pair, m, s)

    def _prefill_batched(self, prompt_ids, argmax: bool):
        """The prompt through every layer PREFILL_BATCH tokens at a time: per token the
        arithmetic of the eager step (engine/limited.py:374-419), so the KV cache and the
        last token's logits equal the token-by-token prefill's bit for bit. Leaves the
        state the token-by-token prefill leaves: logits of the last prompt token, tok and
        pos at it, step 0 -- then, with `argmax`, the first greedy token taken as the
        fused step's last prompt launch does (gen[0], step 1, pos = prompt length)."""
        c = self.cfg
        hid, ffn, qd, nq, nkv, cap = (c.hidden, c.ffn, c.head_dim, c.n_head, c.n_kv,
                                      c.max_context)
        toks = np.ascontiguousarray(prompt_ids, np.int32)
        n = toks.size
        if n == 0 or n > cap:
            raise ValueError(f"{n} prompt tokens for a {cap}-token context")
        pf = self._prefill_buffers()
        s = self._stream_cur
        self._set_i32(self.d_step, 0)
        hvdrv.memset8(self.d_gen, 0, (cap + 1) * 4)
        m = 0
        for b0 in range(0, n, pf["n"]):
            m = min(pf["n"], n - b0)
            hvdrv.synchronize()                 # the host copy below reuses pf["tok"]
            hvdrv.upload(pf["tok"], toks[b0:b0 + m].ctypes.data, 4 * m)
            hvdrv.gather_rows(self.d_emb16, pf["tok"], pf["h"], hid, m, s)
            for l, w in enumerate(self.layers):
                hvdrv.rmsnorm(pf["h"], pf["hn"], w["an"], m, hid, RMS_EPS, s)
                self._gemm(pf["hn"], w["qkv"], pf["qkv"], m)
                hvdrv.qk_rows(pf["qkv"], w["qn"], w["kn"], self.d_cos, self.d_sin, b0, pf["q"],
                              self.KC[l], self.VC[l], nq, nkv, qd, cap, RMS_EPS, m, s,
                              f16=self.kv_f16)
                hvdrv.attn_rows(pf["q"], self.KC[l], self.VC[l], pf["ctx"], self.d_scale, b0,
                                nq, qd, c.group, cap * qd, m, pf["part"], pf["ticket"], s,
                                f16=self.kv_f16)
                self._gemm(pf["ctx"], w["o"], pf["o"], m)
                hvdrv.vadd(pf["h"], pf["o"], pf["h"], m * hid, s)
                hvdrv.rmsnorm(pf["h"], pf["hn"], w["fn"], m, hid, RMS_EPS, s)
                self._gemm(pf["hn"], w["gu"], pf["gu"], m)
                hvdrv.silu_rows(pf["gu"], pf["act"], ffn, m, s)
                self._gemm(pf["act"], w["down"], pf["o"], m)
                hvdrv.vadd(pf["h"], pf["o"], pf["h"], m * hid, s)
        # the last prompt token: final norm and LM head, as the eager step ends
        hvdrv.copy_async(self.d_h, pf["h"] + (m - 1) * hid * 4, hid * 4, s)
        hvdrv.rmsnorm(self.d_h, self.d_hn, self.d_onorm, 1, hid, RMS_EPS, s)
        self._gemv(self.d_hn, self.head, self.d_logits)
        self._set_i32(self.d_tok, int(toks[-1]))
        self._set_i32(self.d_pos, n - 1)
        if argmax and self.fused:
            self._argmax_into_next()

    def _token(self, i: int) -> int:
        """Token i of the current generation, once decode iteration i has run."""
        return self._get_i32(self.d_gen + 4 * i)

    def generate(self, prompt_ids, max_new=64, stop_on_eos=True, use_graph=None):
        """Greedy generation. Returns (tokens, prefill_seconds, decode_seconds)."""
        c = self.cfg
        self._check_len(prompt_ids, max_new)
        hvdrv.synchronize()
        t0 = time.perf_counter()
        self._prefill(prompt_ids)
        hvdrv.synchronize()
        t1 = time.perf_counter()
        graph = self._graph_ok if use_graph is None else use_graph
        if graph:
            try:
                self._build_graph()
            except Exception:
                graph = False
        out = []
        for i in range(max_new):
            if graph:
                self._step_graph()
            else:
                self._decode_one()
            if stop_on_eos:
                hvdrv.synchronize()
                tok = self._token(i)
                out.append(tok)
                if c.eos is not None and tok == c.eos:
                    break
            else:
                out.append(None)
        hvdrv.synchronize()
        t2 = time.perf_counter()
        if self.fused:
            self._check_status()
        if out and out[0] is None:
            got = np.zeros(c.max_context + 1, np.int32)
            hvdrv.download(got.ctypes.data, self.d_gen, got.nbytes)
            out = [int(x) for x in got[:len(out)]]
        return out, t1 - t0, t2 - t1

    # ---- graph-replayed decode (engine/limited.py:502-539) ------------------------------

    def _build_graph(self):
        if self._graph_exec:
            return
        if not self._stream:
            self._stream = hvdrv.stream_create()
        hvdrv.synchronize()
        hvdrv.capture_begin(self._stream)
        self._stream_cur = self._stream
        try:
            self._decode_one()
            graph = hvdrv.capture_end(self._stream)
        except Exception:
            try:
                hvdrv.capture_end(self._stream)
            except Exception:
                pass
            raise
        finally:
            self._stream_cur = 0
        self._graph = graph
        self._graph_exec = hvdrv.graph_instantiate(graph)

    def _step_graph(self):
        hvdrv.graph_launch(self._graph_exec, self._stream)

    def verify_graph(self, prompt_ids, n=24) -> bool:
        """The graph must produce the same tokens as issuing the launches directly."""
        eager, _, _ = self.generate(prompt_ids, max_new=n, use_graph=False)
        fast, _, _ = self.generate(prompt_ids, max_new=n, use_graph=True)
        return eager == fast

    def stream(self, prompt_ids, max_new=64, stop_evt=None, host_tokens=False):
        """Yields ("prefill", seconds) once, then ("tok", id, seconds_since_first_token).

        With host_tokens (fused step only), every decode step is driven from the host:
        the token and position are copied host->device from pinned memory, the step is
        launched, and the token it produces is copied back device->host before the next
        step -- the loop a host-side sampler or detokeniser would run."""
        c = self.cfg
        self._check_len(prompt_ids, max_new)
        if host_tokens and not self.fused:
            raise ValueError("host_tokens needs the fused step")
        hvdrv.synchronize()
        t0 = time.perf_counter()
        self._prefill(prompt_ids)
        hvdrv.synchronize()
        yield ("prefill", time.perf_counter() - t0)
        if host_tokens:
            yield from self._stream_host_fed(len(prompt_ids), max_new, stop_evt)
            return
        graph = bool(self._graph_ok)
        if graph:
            try:
                self._build_graph()
            except Exception:
                graph = False
        first = None
        for i in range(max_new):
            if stop_evt is not None and stop_evt.is_set():
                return
            if graph:
                self._step_graph()
            else:
                self._decode_one()
            hvdrv.synchronize()
            now = time.perf_counter()
            if first is None:
                first = now
            tok = self._token(i)
            yield ("tok", tok, now - first)
            if c.eos is not None and tok == c.eos:
                return

    def _stream_host_fed(self, n_prompt, max_new, stop_evt):
        c = self.cfg
        pin = hvdrv.host_alloc(16)
        buf = (C.c_int32 * 4).from_address(pin)
        try:
            tok = self._get_i32(self.d_tok)        # token 0, from the prefill's argmax
            first = None
            for i in range(max_new):
                if stop_evt is not None and stop_evt.is_set():
                    return
                buf[0], buf[1] = tok, n_prompt + i
                hvdrv.upload_async(self.d_tok, pin, 4)
                hvdrv.upload_async(self.d_pos, pin + 4, 4)
                self._step_fused(STEP_HEAD | STEP_ARGMAX)
                hvdrv.download_async(pin + 8, self.d_tok, 4)
                hvdrv.synchronize()
                now = time.perf_counter()
                if first is None:
                    first = now
                yield ("tok", tok, now - first)
                if c.eos is not None and tok == c.eos:
                    return
                tok = int(buf[2])
        finally:
            hvdrv.host_free(pin)

    def logits(self, prompt_ids) -> np.ndarray:
        """Run the prompt and return the final f32 logits."""
        n = len(prompt_ids)
        if self.prefill_mode == "batched":
            self._prefill_batched(prompt_ids, argmax=False)
        else:
            for i, tok in enumerate(prompt_ids):
                self._prefill_token(tok, i, STEP_HEAD if i == n - 1 else None)
        hvdrv.synchronize()
        if self.fused:
            self._check_status()
        return self.download_logits()

    def download_logits(self) -> np.ndarray:
        out = np.zeros(self.n_head_rows, F32)
        hvdrv.download(out.ctypes.data, self.d_logits, out.nbytes)
        return out

    def _weight_bits(self) -> tuple[int, int]:
        bits = elems = 0
        mats = [w[key] for w in self.layers for key in ("qkv", "o", "gu", "down")]
        for b4, sw, k, n, _ in mats + [self.head]:
            bits += n * (k // 8) * 32 + n * (k // BLOCK) * 32
            elems += n * k
        return bits, elems

    def bits_per_weight(self) -> float:
        bits, elems = self._weight_bits()
        return bits / elems

    def weight_bytes(self) -> int:
        """Weight bytes a batch-1 step reads per token (packed int4 + f32 scales)."""
        bits, _ = self._weight_bits()
        return bits // 8

    def free(self):
        if getattr(self, "_graph_exec", 0) or getattr(self, "_graph", 0):
            hvdrv.graph_destroy(self._graph, self._graph_exec)
            self._graph = self._graph_exec = 0
        if getattr(self, "_stream", 0):
            try:
                hvdrv.stream_destroy(self._stream)
            except Exception:
                pass
            self._stream = 0
        for p in getattr(self, "_opened", []):
            try:
                hvdrv.ipc_close(p)
            except Exception:
                pass
        self._opened = []
        for p in self._buffers:
            try:
                hvdrv.free(p)
            except Exception:
                pass
        self._buffers.clear()
