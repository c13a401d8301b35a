"""bench.py's decode line, produced on the CPU against a fake driver and a fake engine:
one JSON line on stdout carrying every key the measurement contract names (metric,
value, unit, n_gpus, steps, warmup, ms_per_step, higher_is_better, scaling,
vs_baseline, dtype, data, config, roofline, cpu_baseline, e2e, gpu_launches, clocks),
with the numbers derived from the device timing as documented: value = steps / time,
roofline achieved = algorithmic bytes / step time. Only the host logic is under test;
the numbers come from the B200 runs."""
import ctypes
import json
import os
import sys
import types

import numpy as np
import pytest

import bench

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TESTS = os.path.dirname(os.path.abspath(__file__))


class FakeDriver(types.ModuleType):
    def __init__(self, ms):
        super().__init__("hvdrv")
        self.ms = ms
        self.bufs = []

    def host_alloc(self, n):
        b = ctypes.create_string_buffer(int(n))
        self.bufs.append(b)
        return ctypes.addressof(b)

    def event_elapsed_ms(self, a, b):
        return self.ms

    def w4_prepacked_size(self, n, k, pair=0):
        return n * k // 2, n * k // 32 * 4

    def __getattr__(self, name):        # every other call: accepted, no effect
        if name.startswith("__"):       # module introspection (importers, torch) sees none
            raise AttributeError(name)
        return lambda *a, **k: 1


class FakeEngine:
    launched = 0

    last_kw = {}

    def __init__(self, *a, **kw):
        self.kw = kw
        FakeEngine.last_kw = kw
        self.d_pos, self.d_step, self.d_tok = 8, 16, 24
        self.n_head_rows = 151936
        self.cache_hit = None

    def _prefill(self, prompt):
        assert len(prompt) == 4096

    def _decode_one(self):
        FakeEngine.launched += 1

    def _check_status(self):
        pass

    def free(self):
        pass


@pytest.mark.parametrize("extra", [[], ["--kv-dtype", "f16"], ["--gemv-layout", "dq"],
                                   ["--eager"]])
def test_decode_line_carries_the_contract(monkeypatch, capsys, extra):
    import limited
    drv = FakeDriver(ms=320.0)                              # 100 steps in 320 ms
    monkeypatch.setitem(sys.modules, "hvdrv", drv)
    monkeypatch.setattr(limited, "Engine", FakeEngine)
    monkeypatch.setattr(bench.synth, "iter_tensors", lambda cfg, seed: iter(()))
    assert bench.main(["--steps", "100", "--warmup", "3", "--no-cpu", "--e2e-steps", "0",
                       *extra]) == 0
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    ln = lines[0]
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "roofline", "cpu_baseline", "e2e", "gpu_launches", "clocks"):
        assert key in ln, key
    assert ln["n_gpus"] == 1 and ln["steps"] == 100 and ln["warmup"] == 3
    assert ln["ms_per_step"] == pytest.approx(3.2)
    assert ln["value"] == pytest.approx(100 / 0.32)
    assert ln["higher_is_better"] is True and ln["scaling"] == "weak"
    assert ln["config"]["workload"] == "qwen3-8b-p4096-g256"
    rf = ln["roofline"]
    for key in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert key in rf, key
    assert rf["bound"] == "hbm" and rf["unit"] == "GB/s"
    assert rf["achieved"] == pytest.approx(rf["bytes_per_step"] / 3.2e-3 / 1e9)
    assert rf["frac"] == pytest.approx(rf["achieved"] / rf["peak"])
    kv = dict(zip(extra[::2], extra[1::2])).get("--kv-dtype", "f32") if len(extra) != 1 \
        else "f32"
    assert ln["config"]["kv"] == kv
    if kv == "f16":                      # half the KV bytes, and no f32 ncu traffic figure
        assert rf["traffic"] is None
    assert set(ln["e2e"]) >= {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"}
    eager = "--eager" in extra
    assert ln["gpu_launches"] == 100 * (19 * 36 + 6 if eager else 1)
    assert (ln["roofline"]["kernel"] == "eager sequence") == eager
    assert FakeEngine.last_kw["fused"] is (not eager)
    assert set(ln["clocks"]) >= {"sm_mhz", "sm_max_mhz", "reasons"}


def test_step_bytes_counts_the_kv_element_size():
    import w4format
    cfg = w4format.Config(bench.synth.ARCH["qwen3-8b"])
    b32 = bench.step_bytes(cfg, 151936, 4224)
    b16 = bench.step_bytes(cfg, 151936, 4224, kv_elem=2)
    kv32 = 2 * cfg.n_layer * cfg.n_kv * 128 * 4 * 4225
    assert b32 - b16 == kv32 // 2
    assert b32 == pytest.approx(5.976e9, rel=2e-3)          # weights + scales + fp32 KV


def test_reference_line_carries_the_contract(monkeypatch, capsys):
    """--impl reference: the CPU restatement's timing on rank 0, with impl, cpu_baseline
    and an e2e block of zero copies; the CPU sample itself is stubbed here."""
    monkeypatch.setattr(bench, "cpu_decode_sample",
                        lambda cfg, seed, n_prompt, n_steps, budget_s: (0.5, 8, 16.0, 32, 4.0))
    assert bench.main(["--impl", "reference", "--steps", "5", "--warmup", "3"]) == 0
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    ln = lines[0]
    assert ln["impl"] == "reference"
    assert ln["value"] == pytest.approx(0.5) and ln["unit"] == bench.UNIT
    assert ln["metric"] == bench.METRIC and ln["higher_is_better"] is True
    cb = ln["cpu_baseline"]
    assert cb["value"] == ln["value"] and cb["cores"] == 32 and cb["kind"] in ("port",
                                                                              "reference")
    assert ln["e2e"] == {"value": ln["value"], "unit": ln["unit"], "h2d_bytes_per_step": 0,
                         "d2h_bytes_per_step": 0}
    assert ln["config"]["workload"] == "qwen3-8b-p4096-g256"


def _rank_bench(rank, world, port, mode, result):
    """One rank of `bench.py --gpus 2` on the CPU: TCP plumbing, fake driver and engine
    (each rank's device time differs, so the max over ranks is visible)."""
    import contextlib
    import io
    sys.path[:0] = [p for p in (os.path.join(REPO, "hive-limited_b200"),
                                os.path.join(REPO, "oracle"), REPO, TESTS) if p not in sys.path]
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), HV_BENCH_PORT=str(port))
    try:
        import bench as b
        import limited
        sys.modules["hvdrv"] = FakeDriver(ms=300.0 + 20.0 * rank)
        limited.Engine = FakeEngine
        b.synth.iter_tensors = lambda cfg, seed: iter(())
        out = io.StringIO()
        with contextlib.redirect_stdout(out):
            rc = b.main(["--gpus", str(world), "--steps", "100", "--warmup", "3", "--no-cpu",
                         "--e2e-steps", "0", "--mode", mode])
        result.put((rank, rc, out.getvalue()))
    except BaseException as e:                  # report, do not hang the parent
        result.put((rank, -1, repr(e)))
    finally:
        result.close()
        result.join_thread()


@pytest.mark.parametrize("mode", ["sharded", "replicas"])
def test_two_rank_line(mode):
    """Rank 0 alone prints; ms_per_step is the slower rank's; sharded: one stream's
    tok/s (strong scaling, roofline peak x 2); replicas: the sum over streams (weak)."""
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_bench, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (rc, out)) for r, rc, out in (q.get(timeout=240) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    assert got[0][0] == 0 and got[1][0] == 0, got
    assert not [x for x in got[1][1].splitlines() if x.startswith("{")]
    lines = [json.loads(x) for x in got[0][1].splitlines() if x.startswith("{")]
    assert len(lines) == 1
    ln = lines[0]
    assert ln["n_gpus"] == 2 and ln["ms_per_step"] == pytest.approx(3.2)
    if mode == "sharded":
        assert ln["scaling"] == "strong" and ln["value"] == pytest.approx(100 / 0.32)
        assert ln["roofline"]["frac"] == pytest.approx(ln["roofline"]["achieved"]
                                                       / ln["roofline"]["peak"])
    else:
        assert ln["scaling"] == "weak" and ln["value"] == pytest.approx(2 * 100 / 0.32)


def test_head_argmax_line(monkeypatch, capsys):
    """--head-argmax: one line in hidden states/s with its roofline, on a shrunken head
    (the fake driver's keys all carry token 5)."""
    n_all, k = 64, 256
    monkeypatch.setattr(bench.synth, "HEAD_SHAPE", (n_all, k))
    monkeypatch.setattr(bench.synth, "head_case", lambda ns: (
        np.zeros((n_all, k), np.float32), np.zeros((ns, k), np.float32)))
    drv = FakeDriver(ms=10.0)
    key = np.uint64((1 << 32) | ((~5) & 0xFFFFFFFF))

    def download(host_ptr, src, n):
        arr = np.full(n // 8, key, np.uint64)
        ctypes.memmove(host_ptr, arr.ctypes.data, n)
    drv.download = download
    import hvdrv
    drv.token_of_key = hvdrv.token_of_key        # the real key -> token rule (pure)
    monkeypatch.setitem(sys.modules, "hvdrv", drv)
    assert bench.main(["--head-argmax", "--head-states", "100", "--warmup", "3"]) == 0
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    ln = lines[0]
    assert ln["unit"] == "hidden states/s" and ln["value"] == pytest.approx(100 / 0.01)
    assert ln["config"]["shards"] == 1 and ln["config"]["rows_per_shard"] == n_all
    rf = ln["roofline"]
    assert rf["achieved"] == pytest.approx(n_all * k * 5 // 8 / 1e-4 / 1e9)
    assert rf["frac"] == pytest.approx(rf["achieved"] / rf["peak"])
    assert ln["tokens"] == {"first": [5] * 8, "all_valid": True}
    assert ln["gpu_launches"] == 200
