"""bench.py's measurement modes, run on the CPU against a fake driver module (every call
succeeds, every event pair reads 1 ms): the GEMV sweep and the prefill sweep print one
well-formed JSON line per shape, and the in-process A/B loop times every option set,
applies and restores the options, and checks logits identity. Only the host control
flow is under test here; the numbers come from the B200 runs."""
import json
import sys
import types

import numpy as np
import pytest

import bench


class FakeDriver(types.ModuleType):
    def __init__(self):
        super().__init__("hvdrv")
        self.top = 1 << 20
        self.options = {}
        self.logits_calls = 0

    def alloc(self, n):
        self.top += (int(n) + 4095) // 4096 * 4096
        return self.top

    def w4_prepacked_size(self, n, k, pair=0):
        return n * k // 2, n * k // 32 * 4

    def event_create(self):
        return 1

    def event_elapsed_ms(self, a, b):
        return 1.0

    def step_set_option(self, option, value):
        self.options[option] = value

    def __getattr__(self, name):        # every other call: accepted, no effect
        return lambda *a, **k: None


class FakeDist:
    world, rank, local = 1, 0, 0

    def barrier(self):
        pass

    def max(self, x):
        return x


def run_lines(capsys, fn, *args):
    assert fn(*args) == 0
    return [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]


def test_gemv_sweep_lines(monkeypatch, capsys):
    monkeypatch.setitem(sys.modules, "hvdrv", FakeDriver())
    ns = types.SimpleNamespace(gemv_reps=4, gemv_rotate_mb=8, gemv_max_rows=2048)
    lines = run_lines(capsys, bench.run_gemv_sweep, ns, FakeDist())
    assert len(lines) == 6                  # 2048x2048, 2048x6144; three kernels each
    assert [ln["kernel"] for ln in lines[:3]] == ["k_a4gv_pp", "k_a4gv_dq", "k_a4gv_mma"]
    assert "bit_identical_to_pp" in lines[1] and "bit_identical_to_pp" not in lines[0]
    for ln in lines:
        assert ln["unit"] == "GB/s" and ln["us_per_launch"] == pytest.approx(250.0)
        assert ln["bytes_per_launch"] == ln["shape"][0] * ln["shape"][1] * 5 // 8


def test_prefill_sweep_lines(monkeypatch, capsys):
    monkeypatch.setitem(sys.modules, "hvdrv", FakeDriver())
    ns = types.SimpleNamespace(gemv_reps=4, prefill_tokens=8)
    lines = run_lines(capsys, bench.run_prefill_sweep, ns, FakeDist())
    assert [ln["matrix"] for ln in lines] == ["qkv", "o", "gate_up", "down"]
    assert all(ln["tokens"] == 8 and ln["kernel"] == "k_a4gemm_pp" for ln in lines)


class FakeEngine:
    d_pos, d_step, d_tok = 10, 20, 30

    def __init__(self, drv):
        self.drv = drv

    def _decode_one(self):
        pass

    def _check_status(self):
        pass

    def download_logits(self):
        # identical logits unless inflight is 3 (to see the check work)
        return np.full(16, 2.0 if self.drv.options.get(1) == 3 else 1.0, np.float32)


def test_ab_loop_times_every_set_and_restores_options(monkeypatch):
    drv = FakeDriver()
    pin = (np.ctypeslib.ctypes.c_int32 * 4)()
    addr = np.ctypeslib.ctypes.addressof(pin)
    ns = types.SimpleNamespace(ab=["inflight=3", "local_qkv_barrier=1,inflight=8"],
                               ab_rounds=2, steps=5, step_opt=["evict_first=0"])
    done = [0]
    calls = []
    out = bench.run_ab(ns, FakeDist(), FakeEngine(drv), lambda k: calls.append(k), addr, 4096,
                       256, done, drv)
    assert [o["options"] for o in out] == ["baseline", {"inflight": 3},
                                           {"local_qkv_barrier": 1, "inflight": 8}]
    assert all(o["ms_per_step"] == pytest.approx(0.2) and len(o["runs_ms"]) == 2 for o in out)
    assert [o["logits_identical"] for o in out] == [True, False, True]
    assert calls.count(5) == 2 * 3                     # every set timed in every round
    # the options end as --step-opt left them: defaults plus evict_first=0
    assert drv.options == {1: 6, 2: 0, 3: 0}


def test_ab_layout_set_runs_on_a_second_engine(monkeypatch):
    """layout_dq=1 times a second engine (built once, freed at the end) with its own
    decode loop; the step options are applied around it as for every set, and logits
    identity is checked against the baseline engine's."""
    drv = FakeDriver()
    pin = (np.ctypeslib.ctypes.c_int32 * 4)()
    addr = np.ctypeslib.ctypes.addressof(pin)
    ns = types.SimpleNamespace(ab=["layout_dq=1"], ab_rounds=3, steps=4, step_opt=[])
    base_calls, alt_calls, made, freed = [], [], [], []

    class AltEngine(FakeEngine):
        def free(self):
            freed.append(1)

    def make_alt():
        made.append(1)
        return AltEngine(drv), lambda k: alt_calls.append(k)

    out = bench.run_ab(ns, FakeDist(), FakeEngine(drv), lambda k: base_calls.append(k), addr,
                       4096, 256, [0], drv, make_alt)
    assert [o["options"] for o in out] == ["baseline", {"layout_dq": 1}]
    assert made == [1] and freed == [1]
    assert base_calls.count(4) == 3 and alt_calls.count(4) == 3
    assert all(o["logits_identical"] for o in out)
    assert 5 not in drv.options                 # layout_dq is not passed as a step option


def test_ab_option_names_are_checked():
    with pytest.raises(SystemExit):
        bench.main(["--ab", "layout_dq=1", "--gemv-layout", "dq"])
    with pytest.raises(SystemExit):
        bench.main(["--ab", "no_such_option=1"])
    with pytest.raises(SystemExit):
        bench.main(["--step-opt", "layout_dq=1"])
