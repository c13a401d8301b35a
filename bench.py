"""Batch-1 W4A8 Qwen3 decode throughput on B200 (tok/s), with its HBM roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload qwen3-8b-p4096-g256]

Workload (random-init, seeded; there is no network for checkpoints): Qwen3-8B geometry
(hidden 4096, ffn 12288, 36 layers, 32/8 heads of 128, vocab 151936, untied head),
per-32 int4 weights with f32 scales (5.00 bits/weight), a 4096-token random prompt
prefilled into an fp32 KV cache, then greedy decode at batch 1. A step is one decode
token: the whole forward, the LM head and the greedy argmax -- one fused kernel launch.
Decode positions run 4096..4351 (the workload's 256 generated tokens); a longer timed
run rewinds the position to 4096 every 256 steps so every step has the same shape.

value    : decode tok/s, device-timed (CUDA events, inputs resident), max over ranks.
e2e      : the same through the public API (Engine.stream with host_tokens): every step
           copies its token + position host->device from pinned memory and the produced
           token device->host.
roofline : algorithmic bytes per step (int4 weights + f32 scales of every GEMV and the
           LM head, plus the fp32 KV read) / average step time, against the measured HBM
           copy bandwidth in MEASURED_PEAKS.json.
cpu_baseline : the oracle (a C + numpy restatement of the reference's engine/reference.py)
           on the host cores, a bounded sample of decode steps at the same context.

--gpus N > 1 (under torchrun): by default (--mode sharded) the N GPUs decode ONE stream
together, every projection column-sharded across them with the all-gathers done inside
the fused step as NVLink peer stores (strong scaling; value = that stream's tok/s, the
roofline against N x the HBM peak); --mode replicas runs N independent streams (weak
scaling; value = total tok/s).
--impl reference: the reference's CPU algorithm (oracle port, all host threads) on rank 0.
--kv-dtype f16: the compressed-KV lane (binary16 cache, half the KV bytes; results follow
its own oracle, not the reference's fp32 cache). The default f32 is the headline.
"""
from __future__ import annotations

import argparse
import json
import os
import struct
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "hive-limited_b200"))
sys.path.insert(0, str(REPO / "oracle"))

import synth  # noqa: E402
import w4format  # noqa: E402

F32 = np.float32
METRIC = "batch-1 decode tok/s (Qwen3-8B W4A8); GEMV HBM GB/s vs B200 peak"
UNIT = "tok/s"


# ---------------------------------------------------------------------------
# distributed plumbing (host-side barrier, max and all-gather over TCP, stdlib only)
# ---------------------------------------------------------------------------

def _recv_exact(sock, n: int) -> bytes:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            raise ConnectionError("a rank closed its connection")
        buf += chunk
    return bytes(buf)


def _send_msg(sock, payload: bytes):
    sock.sendall(struct.pack("<Q", len(payload)) + payload)


def _recv_msg(sock) -> bytes:
    return _recv_exact(sock, struct.unpack("<Q", _recv_exact(sock, 8))[0])


class Dist:
    """The ranks of one `torchrun` job on one node, with the standard library only: rank 0
    serves a TCP socket on MASTER_ADDR, port HV_BENCH_PORT or else MASTER_PORT + 1
    (torchrun's own store holds MASTER_PORT), and every collective is an all-gather of one
    bytes object per rank through it. A rank that leaves closes its socket, so the others'
    next collective raises instead of waiting; so does a silent rank after `timeout_s`."""

    def __init__(self, timeout_s: float = 600.0):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.timeout = timeout_s
        self.peers = []           # rank 0: the sockets of ranks 1 .. world - 1, in order
        self.sock = None          # other ranks: the socket to rank 0
        if self.world > 1:
            self._connect()

    def _connect(self):
        import socket
        addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
        port = int(os.environ.get("HV_BENCH_PORT")
                   or int(os.environ.get("MASTER_PORT", "29500")) + 1)
        deadline = time.monotonic() + self.timeout
        if self.rank == 0:
            srv = socket.create_server((addr, port))
            srv.settimeout(self.timeout)
            got = {}
            try:
                while len(got) < self.world - 1:
                    c, _ = srv.accept()
                    c.settimeout(self.timeout)
                    got[struct.unpack("<i", _recv_exact(c, 4))[0]] = c
            except BaseException:
                for c in got.values():
                    c.close()
                raise
            finally:
                srv.close()
            self.peers = [got[r] for r in range(1, self.world)]
            return
        while True:
            try:
                s = socket.create_connection((addr, port), timeout=5.0)
                break
            except OSError:
                if time.monotonic() > deadline:
                    raise TimeoutError(f"rank {self.rank}: no rank 0 at {addr}:{port}")
                time.sleep(0.2)
        s.settimeout(self.timeout)
        s.sendall(struct.pack("<i", self.rank))
        self.sock = s

    def allgather_bytes(self, blob: bytes) -> list[bytes]:
        """One bytes object per rank, in rank order, on every rank (also the sharded
        engine's one swap of CUDA IPC handles)."""
        if self.world == 1:
            return [blob]
        try:
            if self.rank == 0:
                parts = [blob] + [_recv_msg(c) for c in self.peers]
                out = struct.pack("<i", len(parts)) + b"".join(
                    struct.pack("<Q", len(p)) + p for p in parts)
                for c in self.peers:
                    _send_msg(c, out)
                return parts
            _send_msg(self.sock, blob)
            out = _recv_msg(self.sock)
        except BaseException:
            self.close()              # the other ranks' next collective fails too
            raise
        n, off, parts = struct.unpack_from("<i", out)[0], 4, []
        for _ in range(n):
            ln = struct.unpack_from("<Q", out, off)[0]
            parts.append(out[off + 8:off + 8 + ln])
            off += 8 + ln
        return parts

    def barrier(self):
        self.allgather_bytes(b"")

    def max(self, x: float) -> float:
        return max(struct.unpack("<d", b)[0] for b in self.allgather_bytes(struct.pack("<d", x)))

    def sum(self, x: float) -> float:
        return sum(struct.unpack("<d", b)[0] for b in self.allgather_bytes(struct.pack("<d", x)))

    def close(self):
        for c in self.peers + ([self.sock] if self.sock else []):
            try:
                c.close()
            except OSError:
                pass
        self.peers, self.sock = [], None


# ---------------------------------------------------------------------------
# measurement helpers
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.rows, self.proc = gpu, [], None
        self.t_on = self.t_off = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self._th = threading.Thread(target=self._read, daemon=True)
        self._th.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.perf_counter(), line.strip()))

    def mark(self, on: bool):
        if on:
            self.t_on = time.perf_counter()
        else:
            self.t_off = time.perf_counter()

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        lo, hi = (self.t_on or 0) - 0.06, (self.t_off or time.perf_counter()) + 0.06
        sel = [r for t, r in self.rows if lo <= t <= hi] or [r for _, r in self.rows]
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in sel:
            f = [x.strip() for x in r.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic(bytes_per_step: float):
    """DRAM bytes per launch of the fused step: the ratio of ncu's DRAM bytes to the
    algorithmic bytes, measured on a small case of the same kernel
    (profiles/k_step_traffic.json), applied to this workload's algorithmic bytes."""
    p = REPO / "profiles" / "k_step_traffic.json"
    try:
        ratio = float(json.loads(p.read_text())["traffic_over_algorithmic"])
    except (OSError, ValueError, KeyError):
        return None
    return ratio * bytes_per_step


def step_bytes(cfg, head_rows: int, pos: int, kv_elem: int = 4) -> int:
    """Algorithmic HBM bytes of one decode step at position `pos`: int4 weights + f32
    scales of every GEMV (0.625 B per weight) plus the K and V rows 0..pos read (fp32,
    or kv_elem = 2 for the binary16 cache)."""
    c = cfg
    qd = c.head_dim
    per_layer = ((c.n_head + 2 * c.n_kv) * qd * c.hidden + c.hidden * c.n_head * qd
                 + 2 * c.ffn * c.hidden + c.hidden * c.ffn)
    w = c.n_layer * per_layer + head_rows * c.hidden
    kv = 2 * c.n_layer * c.n_kv * qd * kv_elem * (pos + 1)
    return int(w * 5 // 8 + kv)


# ---------------------------------------------------------------------------
# CPU side: the oracle port of the reference's decode step
# ---------------------------------------------------------------------------

def cpu_decode_sample(cfg, seed, n_prompt, n_steps, budget_s=25.0):
    """Time greedy decode steps of the oracle at positions n_prompt.. (bounded). The KV
    rows 0..n_prompt-1 are filled with seeded N(0,1) values instead of running the
    prompt (a 4096-token CPU prefill would take days); a step's cost does not depend on
    the values. Returns (tok/s, steps, seconds, threads)."""
    import hv_oracle as O
    t0 = time.perf_counter()
    w = O.quantize_model_c(cfg, synth.iter_tensors(cfg, seed))
    cap = n_prompt + n_steps + 1
    m = O.FastOracleModel(cfg, w, cap)
    g = np.random.default_rng(seed)
    for l in range(cfg.n_layer):
        m.KC[l][:, :n_prompt] = g.standard_normal((cfg.n_kv, n_prompt, cfg.head_dim), F32)
        m.VC[l][:, :n_prompt] = g.standard_normal((cfg.n_kv, n_prompt, cfg.head_dim), F32)
    setup = time.perf_counter() - t0
    tok = synth.prompt_ids(cfg, seed, 1)[0]
    done, t1 = 0, time.perf_counter()
    for i in range(n_steps):
        logits = m.step(tok, n_prompt + i)
        tok = O.argmax(logits)
        done += 1
        if time.perf_counter() - t1 > budget_s:
            break
    dt = time.perf_counter() - t1
    threads = int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1))
    return done / dt, done, dt, threads, setup


# ---------------------------------------------------------------------------
# the arms
# ---------------------------------------------------------------------------

def run_reference(args, dist: Dist):
    if dist.rank != 0:
        return 0
    arch, seed, n_prompt, n_new = synth.WORKLOADS[args.workload]
    cfg = w4format.Config(synth.ARCH[arch])
    rate, done, dt, threads, setup = cpu_decode_sample(cfg, seed, n_prompt,
                                                       max(args.warmup + args.steps, 2),
                                                       budget_s=args.cpu_budget)
    value = done / dt
    sample = (f"{done} oracle decode steps of {arch} at positions {n_prompt}..; "
              f"KV rows of the prompt filled with seeded values; setup {setup:.0f} s")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": dist.world, "steps": done, "warmup": 0, "ms_per_step": 1e3 * dt / done,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded random-init weights and prompt)",
        "config": {"workload": args.workload, "batch": 1, "prompt": n_prompt,
                   "generated": n_new, "kv": "f32", "weights": "int4 + f32 scale per 32"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


STEP_OPTS = {"inflight": 1, "evict_first": 2, "local_qkv_barrier": 3}
STEP_OPT_DEFAULTS = {"inflight": 6, "evict_first": 1, "local_qkv_barrier": 0}
# A/B-only names that are not step options: layout_dq=1 times a second engine of the same
# model whose weight tiles are in the dq arrangement (gemv_layout="dq")
AB_ENGINE_OPTS = ("layout_dq",)


def parse_opts(text: str) -> dict:
    """'a=1,b=0' -> {'a': 1, 'b': 0} over STEP_OPTS names ('' -> {})."""
    out = {}
    for item in filter(None, (x.strip() for x in text.split(","))):
        name, _, value = item.partition("=")
        out[name] = int(value)
    return out


def run_ab(args, dist, eng, decode, pin, n_prompt, window, done, hvdrv, make_alt=None):
    """Fused-step option sets against the baseline in this process (one load, one
    prefill): `--ab-rounds` rounds, each timing every set for --steps steps in turn
    (CUDA events, max over ranks), and each set's logits of one step at the first decode
    position compared bit for bit with the baseline's. A set with layout_dq=1 runs on a
    second engine (make_alt() -> (engine, decode), built once, prefilled the same way).
    -> list of per-set results."""
    sets = [{}] + [parse_opts(x) for x in args.ab]
    base = dict(STEP_OPT_DEFAULTS, **parse_opts(",".join(args.step_opt)))
    alt = []

    def apply(opts):
        for name, value in dict(base, **opts).items():
            if name not in AB_ENGINE_OPTS:
                hvdrv.step_set_option(STEP_OPTS[name], value)

    def engine_of(opts):
        if not opts.get("layout_dq"):
            return eng, decode
        if not alt:
            alt.append(make_alt())
        return alt[0]

    def one_step_logits(e):
        hvdrv.upload_async(e.d_pos, pin, 4)                # position n_prompt, step 0
        hvdrv.upload_async(e.d_step, pin + 4, 4)
        hvdrv.upload_async(e.d_tok, pin + 8, 4)
        e._decode_one()
        hvdrv.synchronize()
        e._check_status()
        return e.download_logits()

    pbuf = np.ctypeslib.as_array((np.ctypeslib.ctypes.c_int32 * 4).from_address(pin))
    pbuf[2] = 17                                           # a fixed input token
    ref = None
    times = [[] for _ in sets]
    same = [True for _ in sets]
    e0, e1 = hvdrv.event_create(), hvdrv.event_create()
    for _ in range(args.ab_rounds):
        for i, opts in enumerate(sets):
            apply(opts)
            e, dec = engine_of(opts)
            lg = one_step_logits(e)
            if ref is None:
                ref = lg
            same[i] = same[i] and bool(np.array_equal(lg.view(np.uint32), ref.view(np.uint32)))
            done[0] = 0
            hvdrv.upload_async(e.d_pos, pin, 4)
            hvdrv.upload_async(e.d_step, pin + 4, 4)
            dec(3)
            dist.barrier()
            hvdrv.synchronize()
            hvdrv.event_record(e0, 0)
            dec(args.steps)
            hvdrv.event_record(e1, 0)
            hvdrv.synchronize()
            times[i].append(dist.max(hvdrv.event_elapsed_ms(e0, e1)) / args.steps)
    apply({})
    for e, _ in alt:
        e.free()
    out = []
    for opts, t, ok in zip(sets, times, same):
        ms = float(np.median(t))
        out.append({"options": opts or "baseline", "ms_per_step": ms, "tok_s": 1e3 / ms,
                    "runs_ms": [round(x, 4) for x in t], "logits_identical": ok})
    return out


def run_ours(args, dist: Dist):
    import hvdrv
    import limited
    for opt in args.step_opt:
        name, _, value = opt.partition("=")
        hvdrv.step_set_option(STEP_OPTS[name], int(value))
    arch, seed, n_prompt, n_new = synth.WORKLOADS[args.workload]
    cfg = w4format.Config(synth.ARCH[arch])
    cap = n_prompt + n_new
    t0 = time.perf_counter()
    sharded = dist.world > 1 and args.mode == "sharded"

    def make_engine(gemv_layout):
        return limited.Engine(
            config=cfg, tensors=synth.iter_tensors(cfg, seed), quiet=True, max_context=cap,
            device=dist.local, fused=not args.eager, world=dist.world if sharded else 1,
            rank=dist.rank if sharded else 0,
            exchange=dist.allgather_bytes if sharded else None,
            weight_cache=args.weight_cache, prefill=args.prefill,
            cache_tag=f"synthetic:{arch}:seed{seed}" if args.weight_cache else None,
            kv_dtype=args.kv_dtype, gemv_layout=gemv_layout)

    eng = make_engine(args.gemv_layout)
    t_load = time.perf_counter() - t0
    prompt = synth.prompt_ids(cfg, seed, n_prompt)
    window = cap - n_prompt              # decode positions available before a rewind

    # prefill (the last prompt token's launch takes the first argmax)
    t0 = time.perf_counter()
    eng._prefill(prompt)
    hvdrv.synchronize()
    eng._check_status()
    t_prefill = time.perf_counter() - t0

    pin = hvdrv.host_alloc(16)
    pbuf = np.ctypeslib.as_array((np.ctypeslib.ctypes.c_int32 * 4).from_address(pin))
    pbuf[:] = [n_prompt, 0, 0, 0]
    done = [0]

    def decoder(e):
        def decode(k):
            for _ in range(k):
                if done[0] and done[0] % window == 0:      # rewind to the first position
                    hvdrv.upload_async(e.d_pos, pin, 4)
                    hvdrv.upload_async(e.d_step, pin + 4, 4)
                e._decode_one()
                done[0] += 1
        return decode

    decode = decoder(eng)

    def make_alt():
        """The same model with dq weight tiles, prefilled like the first engine."""
        e = make_engine("dq")
        e._prefill(prompt)
        hvdrv.synchronize()
        e._check_status()
        return e, decoder(e)

    decode(args.warmup)
    hvdrv.synchronize()
    clocks = ClockSampler(dist.local)
    clocks.start()
    time.sleep(0.3)
    e0, e1 = hvdrv.event_create(), hvdrv.event_create()
    dist.barrier()
    hvdrv.synchronize()
    clocks.mark(True)
    hvdrv.event_record(e0, 0)
    first_step = done[0]
    decode(args.steps)
    hvdrv.event_record(e1, 0)
    hvdrv.synchronize()
    clocks.mark(False)
    dist.barrier()
    ms = hvdrv.event_elapsed_ms(e0, e1)
    clk = clocks.stop()
    eng._check_status()
    ms_max = dist.max(ms)
    ms_per_step = ms_max / args.steps
    # replicas: every GPU decodes its own stream (weak scaling, tokens add up); sharded:
    # the GPUs decode ONE stream together (strong scaling)
    value = (1 if sharded else dist.world) * args.steps / (ms_max / 1e3)

    # algorithmic bytes over the timed steps (position of each step)
    positions = [n_prompt + ((first_step + i) % window) for i in range(args.steps)]
    head_rows = eng.n_head_rows * (dist.world if sharded else 1)
    n_peak = dist.world if sharded else 1        # the HBM of every GPU the stream uses
    kv_elem = 2 if args.kv_dtype == "f16" else 4
    bytes_mean = float(np.mean([step_bytes(cfg, head_rows, p, kv_elem) for p in positions]))
    peak, peak_kind = measured_peak()
    achieved = bytes_mean / (ms_per_step / 1e3) / 1e9
    # the committed ncu capture is of the one-GPU f32-cache step over pp tiles
    traffic = (None if sharded or args.kv_dtype != "f32" or args.eager or args.gemv_layout != "pp"
               else profiled_traffic(bytes_mean))

    if args.profile and dist.rank == 0:
        # one extra step with the per-phase device trace, at the next decode position
        # (after the timed region, so it perturbs nothing that is measured)
        if done[0] and done[0] % window == 0:      # at the cache's end: rewind first
            hvdrv.upload_async(eng.d_pos, pin, 4)
            hvdrv.upload_async(eng.d_step, pin + 4, 4)
        prof = eng.profile_step()
        print(f"per-phase trace of one step at position {n_prompt + done[0] % window} "
              f"(us, summed over {cfg.n_layer} layers; median and max over CTAs):",
              file=sys.stderr)
        for name, v in prof["phases"].items():
            print(f"  {name:26s} {v['median_us']:10.1f} {v['max_us']:10.1f}", file=sys.stderr)
        print(f"  total {prof['total_us']:.1f} us", file=sys.stderr, flush=True)
        eng._check_status()

    ab = None
    if args.ab:
        ab = run_ab(args, dist, eng, decode, pin, n_prompt, window, done, hvdrv, make_alt)

    # end to end through the public API: Engine.stream with host-fed tokens
    n_e2e = min(args.e2e_steps, window)
    ev = list(eng.stream(prompt, max_new=n_e2e, host_tokens=True)) if n_e2e > 0 else []
    times = [e[2] for e in ev if e[0] == "tok"]
    e2e = (len(times) - 1) / (times[-1] - times[0]) if len(times) > 1 else None
    e2e_all = dist.sum(e2e or 0.0) if dist.world > 1 and not sharded else e2e

    line = None
    if dist.rank == 0:
        cpu = None
        if dist.world == 1 and not args.no_cpu:
            rate, n_cpu, dt, threads, setup = cpu_decode_sample(
                cfg, seed, n_prompt, 64, budget_s=args.cpu_budget)
            cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"{n_cpu} oracle decode steps of {arch} at positions "
                             f"{n_prompt}.. in {dt:.1f} s (KV rows of the prompt filled "
                             f"with seeded values)"}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong" if sharded else "weak",
            "vs_baseline": None,
            "dtype": "int8", "data": "synthetic (seeded random-init weights and prompt)",
            "config": {"workload": args.workload, "model": arch, "batch": 1,
                       "prompt": n_prompt, "generated": n_new, "kv": args.kv_dtype,
                       "weights": "int4 + f32 scale per 32 (5.00 bits/weight)",
                       "gemv_layout": args.gemv_layout,
                       "step": "eager kernel sequence" if args.eager else "fused (one launch)",
                       "parallelism": (f"column-sharded x{dist.world} (NVLink peer stores "
                                       "inside the fused step)" if sharded else
                                       "replicas" if dist.world > 1 else "single"),
                       "l2": f"inputs larger than L2 ({bytes_mean / 1e9:.1f} GB read per step)",
                       "positions": f"{min(positions)}..{max(positions)}"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak * n_peak,
                         "unit": "GB/s", "frac": achieved / (peak * n_peak), "traffic": traffic,
                         "peak_kind": peak_kind,
                         "kernel": "eager sequence" if args.eager else "k_step",
                         "bytes_per_step": bytes_mean},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_all, "unit": UNIT, "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4},
            # the fused step is one launch; the eager sequence is the reference's 19 per
            # layer plus the embedding gather, final norm, head (2) and argmax (2)
            "gpu_launches": args.steps * (19 * cfg.n_layer + 6 if args.eager else 1),
            "clocks": clk,
            "load_s": round(t_load, 1), "prefill_s": round(t_prefill, 2),
            "prefill": args.prefill, "step_options": args.step_opt,
            **({"ab": ab} if ab is not None else {}),
            "weight_cache": {None: None, True: "hit", False: "miss"}[eng.cache_hit],
        }
        print(json.dumps(line), flush=True)
    hvdrv.host_free(pin)
    eng.free()
    return 0


def run_gemv_sweep(args, dist: Dist):
    """The isolated W4A8 GEMV sweep (batch 1): the six sweep shapes (weights N(0,0.02)
    from seed 1, activation N(0,1)) and the 151936 x 5120 LM head (seed 4), through the
    C ABI: hv_a4gv_pp over the engine's tile-interleaved layout and hv_a4gv over the
    reference's row-major layout. One JSON line per (shape, kernel): device time per
    launch (CUDA events over `--gemv-reps` launches) and achieved GB/s of the algorithmic
    0.625 B per weight. Weight copies rotate so every launch reads bytes that are not in
    L2 (126 MB): at least `--gemv-rotate-mb` MB of copies per shape, or one copy with
    `--gemv-rotate-mb 0`."""
    if dist.rank != 0:
        return 0
    import hvdrv
    hvdrv.init()
    peak, peak_kind = measured_peak()
    e0, e1 = hvdrv.event_create(), hvdrv.event_create()
    cases = [(j, n, k) for j, (n, k) in enumerate(synth.GEMV_SHAPES)] + [(None, *synth.HEAD_SHAPE)]
    if args.gemv_max_rows:
        cases = [c for c in cases if c[1] <= args.gemv_max_rows]
    if getattr(args, "gemv_shape", None):
        want = {tuple(int(x) for x in sh.lower().split("x")) for sh in args.gemv_shape}
        cases = [c for c in cases if (c[1], c[2]) in want]
    for j, n, k in cases:
        if j is None:
            w, h = synth.head_case(1)
            a = h[0]
        else:
            w, a = synth.gemv_case(j, n, k)
        nb = k // 32
        alg = n * k * 5 // 8
        bufs = []

        def dev(nbytes):
            p = hvdrv.alloc(nbytes)
            bufs.append(p)
            return p

        wd = hvdrv.alloc(w.nbytes)
        hvdrv.upload(wd, w.ctypes.data, w.nbytes)
        b4, sw = dev(n * k // 2), dev(n * nb * 4)
        hvdrv.quantize_w4(wd, b4, sw, n, k)
        hvdrv.synchronize()
        hvdrv.free(wd)
        del w
        nib, scb = hvdrv.w4_prepacked_size(n, k, 0)
        pb4, psw = dev(nib), dev(scb)
        hvdrv.w4_prepack(b4, sw, n, k, 0, pb4, psw)
        qb4, qsw = dev(nib), dev(scb)
        hvdrv.w4_prepack_dq(b4, sw, n, k, 0, qb4, qsw)
        ad, a8, sa, y = dev(k * 4), dev(k), dev(nb * 8), dev(n * 4)
        hvdrv.upload(ad, a.ctypes.data, a.nbytes)
        hvdrv.qa8s(ad, a8, sa, nb)
        copies = max(1, -(-(args.gemv_rotate_mb << 20) // alg)) if args.gemv_rotate_mb else 1
        rot_pp, rot_ref, rot_dq = [(pb4, psw)], [(b4, sw)], [(qb4, qsw)]
        for _ in range(copies - 1):
            p, s = dev(nib), dev(scb)
            hvdrv.copy_async(p, pb4, nib)
            hvdrv.copy_async(s, psw, scb)
            rot_pp.append((p, s))
            p, s = dev(nib), dev(scb)
            hvdrv.copy_async(p, qb4, nib)
            hvdrv.copy_async(s, qsw, scb)
            rot_dq.append((p, s))
            p, s = dev(n * k // 2), dev(n * nb * 4)
            hvdrv.copy_async(p, b4, n * k // 2)
            hvdrv.copy_async(s, sw, n * nb * 4)
            rot_ref.append((p, s))
        hvdrv.synchronize()

        def pp(c):
            hvdrv.a4gv_pp(a8, sa, rot_pp[c][0], rot_pp[c][1], y, k // 8, n, 0)

        def ref(c):
            hvdrv.a4gv(a8, sa, rot_ref[c][0], rot_ref[c][1], y, k // 8, n)

        def dq(c):
            hvdrv.a4gv_dq(a8, sa, rot_dq[c][0], rot_dq[c][1], y, k // 8, n, 0)

        # the dp4a kernel's output against the tensor-pipe kernel's, bit for bit
        y_pp, y_dq = np.empty(n, np.float32), np.empty(n, np.float32)
        pp(0)
        hvdrv.synchronize()
        hvdrv.download(y_pp.ctypes.data, y, y_pp.nbytes)
        dq(0)
        hvdrv.synchronize()
        hvdrv.download(y_dq.ctypes.data, y, y_dq.nbytes)
        same = bool(np.array_equal(y_pp.view(np.uint32), y_dq.view(np.uint32)))

        for kernel, layout, launch in (("k_a4gv_pp", "tile-interleaved (engine)", pp),
                                       ("k_a4gv_dq", "dq tiles, dp4a block dots", dq),
                                       ("k_a4gv_mma", "row-major (reference)", ref)):
            for i in range(max(3, copies)):
                launch(i % copies)
            hvdrv.synchronize()
            hvdrv.event_record(e0, 0)
            for i in range(args.gemv_reps):
                launch(i % copies)
            hvdrv.event_record(e1, 0)
            hvdrv.synchronize()
            us = hvdrv.event_elapsed_ms(e0, e1) * 1e3 / args.gemv_reps
            gbs = alg / (us * 1e-6) / 1e9
            print(json.dumps({
                "metric": "W4A8 GEMV HBM GB/s (batch 1)", "workload": "gemv-sweep",
                "shape": [n, k], "kernel": kernel, "layout": layout, "value": gbs,
                "unit": "GB/s", "us_per_launch": us, "bytes_per_launch": alg,
                "frac": gbs / peak, "peak": peak, "peak_kind": peak_kind,
                "launches": args.gemv_reps,
                **({"bit_identical_to_pp": same} if kernel == "k_a4gv_dq" else {}),
                "l2": f"{copies} rotating weight copies ({copies * alg / 2**20:.0f} MB)"}),
                flush=True)
        for p in bufs:
            hvdrv.free(p)
    return 0


def run_head_argmax(args, dist: Dist):
    """The LM-head GEMV + greedy argmax workload (151936 x 5120 int4 weights from seed 4,
    N(0,1) hidden states quantised per 32), vocabulary-sharded over the ranks: rank r holds
    rows [r V/N, (r+1) V/N) in the engine's tile layout and, for every hidden state, runs
    the GEMV of its shard and folds its logits into that state's 64-bit argmax key
    (hv_a4gv_pp + hv_argmax_key). Device time over `--head-states` states (CUDA events, max
    over ranks); weight copies rotate so the shard is read from HBM, not L2. After the
    timed region the keys are all-gathered on the host (8 bytes per state and rank) and
    the tokens formed. Their parity with np.argmax is tests/test_gpu_head_argmax.py's."""
    import hvdrv
    hvdrv.init()
    hvdrv.retain_primary_context(hvdrv.device(dist.local))
    n_all, k = synth.HEAD_SHAPE
    world, rank = dist.world, dist.rank
    if n_all % world:
        raise SystemExit(f"{n_all} vocabulary rows do not split over {world} ranks")
    rows = n_all // world
    r0 = rank * rows
    ns = args.head_states
    w, h = synth.head_case(ns)
    nb = k // 32
    bufs = []

    def dev(nbytes):
        p = hvdrv.alloc(nbytes)
        bufs.append(p)
        return p

    ws = np.ascontiguousarray(w[r0:r0 + rows])
    wd = hvdrv.alloc(ws.nbytes)
    hvdrv.upload(wd, ws.ctypes.data, ws.nbytes)
    b4, sw = dev(rows * k // 2), dev(rows * nb * 4)
    hvdrv.quantize_w4(wd, b4, sw, rows, k)
    hvdrv.synchronize()
    hvdrv.free(wd)
    nib, scb = hvdrv.w4_prepacked_size(rows, k, 0)
    alg = rows * k * 5 // 8
    copies = max(1, -(-(args.gemv_rotate_mb << 20) // alg)) if args.gemv_rotate_mb else 1
    rot = []
    for _ in range(copies):
        p, q = dev(nib), dev(scb)
        hvdrv.w4_prepack(b4, sw, rows, k, 0, p, q)
        rot.append((p, q))
    hd = dev(ns * k * 4)
    hvdrv.upload(hd, np.ascontiguousarray(h).ctypes.data, ns * k * 4)
    a8, sa = dev(ns * k), dev(ns * nb * 8)
    hvdrv.qa8s_rows(hd, a8, sa, nb, ns)
    logits, keys = dev(rows * 4), dev(ns * 8)

    def run(i0, i1):
        for i in range(i0, i1):
            pb, ps = rot[i % copies]
            hvdrv.a4gv_pp(a8 + i * k, sa + i * nb * 8, pb, ps, logits, k // 8, rows, 0)
            hvdrv.argmax_key(logits, rows, r0, keys + 8 * i)

    warm = min(args.warmup, ns)
    hvdrv.memset8(keys, 0, ns * 8)
    run(0, warm)
    hvdrv.synchronize()
    hvdrv.memset8(keys, 0, ns * 8)
    e0, e1 = hvdrv.event_create(), hvdrv.event_create()
    dist.barrier()
    hvdrv.synchronize()
    hvdrv.event_record(e0, 0)
    run(0, ns)
    hvdrv.event_record(e1, 0)
    hvdrv.synchronize()
    ms = dist.max(hvdrv.event_elapsed_ms(e0, e1))
    mine = np.zeros(ns, np.uint64)
    hvdrv.download(mine.ctypes.data, keys, ns * 8)
    blobs = dist.allgather_bytes(mine.tobytes())
    best = np.max(np.stack([np.frombuffer(b, np.uint64) for b in blobs]), axis=0)
    toks = [hvdrv.token_of_key(int(x)) for x in best]
    line = None
    if rank == 0:
        peak, peak_kind = measured_peak()
        per_state_s = ms / 1e3 / ns
        achieved = alg / per_state_s / 1e9              # GB/s on each GPU
        line = {
            "metric": "LM-head GEMV + greedy argmax (151936x5120 W4A8, vocabulary-sharded)",
            "value": ns / (ms / 1e3), "unit": "hidden states/s", "n_gpus": world,
            "steps": ns, "warmup": warm, "ms_per_step": ms / ns, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seed 4 head weights, N(0,1) hidden states)",
            "config": {"workload": "lm-head-argmax", "shape": [n_all, k], "shards": world,
                       "rows_per_shard": rows, "states": ns,
                       "l2": f"{copies} rotating weight copies per rank",
                       "exchange": "8-byte key per state and rank, all-gathered on the "
                                   "host after the timed region"},
            "roofline": {"bound": "hbm", "achieved": achieved * world,
                         "peak": peak * world, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": None, "peak_kind": peak_kind,
                         "kernel": "k_a4gv_pp + k_argmax_key",
                         "bytes_per_state_per_gpu": alg},
            "tokens": {"first": toks[:8], "all_valid": all(0 <= t < n_all for t in toks)},
            "gpu_launches": 2 * ns,
        }
        print(json.dumps(line), flush=True)
    for p in bufs:
        hvdrv.free(p)
    return 0 if line is None or line["tokens"]["all_valid"] else 1


def run_prefill_sweep(args, dist: Dist):
    """The prefill GEMM (hv_a4gemm_pp) on the 8B layer shapes for a run of
    `--prefill-tokens` tokens: device time per GEMM (CUDA events over `--gemv-reps`
    launches), prompt tokens per second through that matrix, the int8 MMA rate it
    sustains (2 * N * K * T ops per launch) and the weight bytes it reads per token.
    One JSON line per shape."""
    if dist.rank != 0:
        return 0
    import hvdrv
    hvdrv.init()
    e0, e1 = hvdrv.event_create(), hvdrv.event_create()
    ntok = args.prefill_tokens
    cfg = w4format.Config(synth.ARCH["qwen3-8b"])
    hid, ffn, qd = cfg.hidden, cfg.ffn, cfg.head_dim
    shapes = [("qkv", (cfg.n_head + 2 * cfg.n_kv) * qd, hid, 0),
              ("o", hid, cfg.n_head * qd, 0), ("gate_up", 2 * ffn, hid, ffn),
              ("down", hid, ffn, 0)]
    g = np.random.default_rng(9)
    for name, n, k, pair in shapes:
        bufs = []

        def dev(nbytes):
            ptr = hvdrv.alloc(nbytes)
            bufs.append(ptr)
            return ptr

        packed = g.integers(0, 2**32, (n, k // 8), dtype=np.uint32)
        scale = (g.random((n, k // 32), dtype=np.float32) * 0.01 + 1e-3).astype(F32)
        b4, sw = dev(packed.nbytes), dev(scale.nbytes)
        hvdrv.upload(b4, packed.ctypes.data, packed.nbytes)
        hvdrv.upload(sw, scale.ctypes.data, scale.nbytes)
        nib, scb = hvdrv.w4_prepacked_size(n, k, pair)
        pb4, psw = dev(nib), dev(scb)
        hvdrv.w4_prepack(b4, sw, n, k, pair, pb4, psw)
        x = g.standard_normal((ntok, k), dtype=np.float32)
        xd, a8, sa, y = dev(x.nbytes), dev(ntok * k), dev(ntok * (k // 32) * 8), dev(ntok * n * 4)
        hvdrv.upload(xd, x.ctypes.data, x.nbytes)
        hvdrv.qa8s_rows(xd, a8, sa, k // 32, ntok)
        for _ in range(3):
            hvdrv.a4gemm_pp(a8, sa, pb4, psw, y, k // 8, n, pair, ntok)
        hvdrv.synchronize()
        hvdrv.event_record(e0, 0)
        for _ in range(args.gemv_reps):
            hvdrv.a4gemm_pp(a8, sa, pb4, psw, y, k // 8, n, pair, ntok)
        hvdrv.event_record(e1, 0)
        hvdrv.synchronize()
        us = hvdrv.event_elapsed_ms(e0, e1) * 1e3 / args.gemv_reps
        print(json.dumps({
            "metric": "W4A8 prefill GEMM", "workload": "prefill-gemm",
            "matrix": name, "shape": [n, k], "tokens": ntok, "kernel": "k_a4gemm_pp",
            "us_per_launch": us, "tokens_per_s": ntok / (us * 1e-6),
            "int8_tops": 2.0 * n * k * ntok / (us * 1e-6) / 1e12,
            "weight_bytes_per_token": n * k * 5 / 8 / ntok, "launches": args.gemv_reps}),
            flush=True)
        for ptr in bufs:
            hvdrv.free(ptr)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen3-8b-p4096-g256", choices=list(synth.WORKLOADS))
    ap.add_argument("--e2e-steps", type=int, default=128,
                    help="tokens of the end-to-end run (0 skips it, and its second prefill)")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="also print the fused step's per-phase device trace (stderr)")
    ap.add_argument("--mode", default="sharded", choices=["sharded", "replicas"],
                    help="with more than one GPU: shard one stream across them (column "
                         "parallel) or run one independent stream per GPU")
    ap.add_argument("--ab", action="append", default=[], metavar="NAME=VALUE[,...]",
                    help="also time this fused-step option set against the baseline in "
                         "the same process (repeatable); results under 'ab'")
    ap.add_argument("--ab-rounds", type=int, default=3)
    ap.add_argument("--step-opt", action="append", default=[], metavar="NAME=VALUE",
                    help="fused-step tuning option (results unchanged): "
                         + ", ".join(STEP_OPTS))
    ap.add_argument("--prefill", default="steps", choices=["steps", "batched"],
                    help="how the prompt is prefilled before the timed decode: through the "
                         "decode step token by token (as the reference), or in batches")
    ap.add_argument("--kv-dtype", default="f32", choices=["f32", "f16"],
                    help="KV cache element type: f32 (the reference's cache) or f16 (the "
                         "compressed-KV lane)")
    ap.add_argument("--eager", action="store_true",
                    help="time the reference's kernel-by-kernel sequence (19 launches per "
                         "layer) instead of the fused step, e.g. for a per-kernel ncu list")
    ap.add_argument("--gemv-layout", default="pp", choices=["pp", "dq"],
                    help="weight tiles for tensor-pipe block dots (pp) or dp4a block dots "
                         "(dq); results are bit-identical")
    ap.add_argument("--weight-cache", default=None, metavar="DIR",
                    help="load device-ready weights from DIR when present, else quantise "
                         "and write them there (the timed steps are the same either way)")
    ap.add_argument("--gemv-sweep", action="store_true",
                    help="instead of the decode step: the isolated GEMV sweep, one JSON line "
                         "per shape and kernel")
    ap.add_argument("--prefill-sweep", action="store_true",
                    help="instead of the decode step: the prefill GEMM on the 8B layer "
                         "shapes, one JSON line per matrix")
    ap.add_argument("--prefill-tokens", type=int, default=256)
    ap.add_argument("--head-argmax", action="store_true",
                    help="instead of the decode step: the vocabulary-sharded LM head + "
                         "greedy argmax workload (151936 x 5120), one JSON line")
    ap.add_argument("--head-states", type=int, default=2000)
    ap.add_argument("--gemv-reps", type=int, default=300)
    ap.add_argument("--gemv-max-rows", type=int, default=0,
                    help="sweep only the shapes with at most this many rows (0: all)")
    ap.add_argument("--gemv-rotate-mb", type=int, default=320)
    ap.add_argument("--gemv-shape", action="append", default=[], metavar="NxK",
                    help="sweep only these shapes (repeatable), e.g. 151936x4096")
    args = ap.parse_args(argv)
    for opt in args.step_opt:
        if opt.partition("=")[0] not in STEP_OPTS or not opt.partition("=")[2].isdigit():
            ap.error(f"option {opt!r}: NAME=VALUE with NAME in {', '.join(STEP_OPTS)}")
    ab_names = list(STEP_OPTS) + list(AB_ENGINE_OPTS)
    for opt in [x for a in args.ab for x in a.split(",") if x.strip()]:
        if opt.partition("=")[0] not in ab_names or not opt.partition("=")[2].isdigit():
            ap.error(f"--ab option {opt!r}: NAME=VALUE with NAME in {', '.join(ab_names)}")
    if any(parse_opts(a).get("layout_dq") for a in args.ab) and args.gemv_layout != "pp":
        ap.error("--ab layout_dq=1 compares a dq engine against the pp engine")
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.eager and (args.ab or (int(os.environ.get("WORLD_SIZE", "1")) > 1
                                   and args.mode == "sharded")):
        ap.error("--eager runs one GPU per stream (no --ab, no sharded mode)")
    dist = Dist()
    try:
        if args.gemv_sweep:
            return run_gemv_sweep(args, dist)
        if args.prefill_sweep:
            return run_prefill_sweep(args, dist)
        if args.head_argmax:
            return run_head_argmax(args, dist)
        if args.impl == "reference":
            return run_reference(args, dist)
        return run_ours(args, dist)
    finally:
        dist.close()


if __name__ == "__main__":
    raise SystemExit(main())
