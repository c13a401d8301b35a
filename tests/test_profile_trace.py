"""Engine.profile_step's reading of the fused step's trace, on the CPU: a synthetic trace
with known phase durations per CTA goes through the same download path (a fake driver),
and every reported phase is the per-layer duration, medianed (or maxed) over CTAs and
summed over layers, in microseconds. Next to the B200 numbers this is what makes the
per-phase tables trustworthy."""
import ctypes
import types

import numpy as np
import pytest

import limited
import synth

GRID, NL = 3, 2
TL = 28                                          # trace entries per layer


def synthetic_trace():
    th = 2 + TL * NL
    raw = np.zeros((GRID, 10 + TL * NL), np.uint64)
    for b in range(GRID):
        clock = 1000 * b
        raw[b, 0] = clock
        clock += 50
        raw[b, 1] = clock
        for l in range(NL):
            base = 2 + TL * l

            def mark(k, dur):
                nonlocal clock
                clock += dur
                raw[b, base + k] = clock
            mark(26, 30 + b)                     # prologue: vector loaded and squared
            mark(27, 20)                         # sum of squares
            mark(0, 40)                          # quantised: qkv prologue ends
            mark(1, 100 + l)                     # qkv GEMV
            mark(2, 10)                          # barrier 1
            for k, dur in zip(range(14, 17), (5, 15, 7)):
                mark(k, dur)                     # attention scores (every CTA has a chunk)
            if b != 1:                           # the context items: CTAs 0 and 2 only
                for k, dur in zip(range(17, 20), (9, 3, 50 if b == 0 else 1)):
                    mark(k, dur)
            mark(3, 2)
            for k in range(4, 14):
                mark(k, 10 * k + b)
            raw[b, base + 21:base + 26] = [11, 12, 13, 14 + b, 1000]   # waits, busy cycles
        clock += 60
        raw[b, th] = clock
        clock += 200
        raw[b, th + 1] = clock
        clock += 5
        raw[b, th + 2] = clock
        raw[b, th + 3:th + 6] = [1000 + b, 0, 77]
    return raw


class FakeDriver(types.ModuleType):
    def __init__(self, raw):
        super().__init__("hvdrv")
        self.raw = raw

    def download(self, host_ptr, src, n):
        assert n == self.raw.nbytes
        ctypes.memmove(host_ptr, self.raw.ctypes.data, n)

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return lambda *a, **k: 1


def test_profile_step_phases(monkeypatch):
    raw = synthetic_trace()
    monkeypatch.setattr(limited, "hvdrv", FakeDriver(raw))
    eng = object.__new__(limited.Engine)
    eng.cfg = limited.Config(synth.tiny_arch(n_layer=NL))
    eng.step_grid = GRID
    eng._desc = limited._StepDesc()
    eng._stream_cur = 0
    eng._check_status = lambda: None
    out = eng.profile_step()
    ph = out["phases"]

    def us(per_cta_per_layer, how):            # [layer][cta] ns -> summed over layers
        return sum(how(np.array(v, float)) for v in per_cta_per_layer) / 1e3

    ctas = range(GRID)
    assert ph["qkv_prologue"]["median_us"] == pytest.approx(
        us([[90 + b for b in ctas]] * NL, np.median))
    assert ph["qkv_prologue"]["max_us"] == pytest.approx(us([[90 + b for b in ctas]] * NL, np.max))
    assert ph["qkv_gemv"]["median_us"] == pytest.approx((100 + 101) / 1e3)
    assert ph["barrier1"]["max_us"] == pytest.approx(2 * 10 / 1e3)
    # attention = its parts + 2 ns; the context chain takes 50 ns on CTA 0, 1 ns on CTA 2,
    # CTA 1 has no context item
    att = [[5 + 15 + 7 + (0 if b == 1 else 9 + 3 + (50 if b == 0 else 1)) + 2 for b in ctas]] * NL
    assert ph["attention"]["median_us"] == pytest.approx(us(att, np.median))
    assert ph["attention"]["max_us"] == pytest.approx(us(att, np.max))
    assert ph["attn_ctx_chain"]["max_us"] == pytest.approx(2 * 50 / 1e3)
    assert ph["attn_ctx_chain"]["median_us"] == pytest.approx(2 * 25.5 / 1e3)
    assert ph["attn_scores"]["median_us"] == pytest.approx(2 * 15 / 1e3)
    assert ph["down_gemv"]["median_us"] == pytest.approx(2 * (120 + 1) / 1e3)
    assert ph["barrier5"]["max_us"] == pytest.approx(2 * (130 + 2) / 1e3)
    assert ph["qkv_pro_load"]["median_us"] == pytest.approx(2 * 31 / 1e3)
    assert ph["qkv_pro_sumsq"]["median_us"] == pytest.approx(2 * 20 / 1e3)
    assert ph["qkv_pro_quant"]["median_us"] == pytest.approx(2 * 40 / 1e3)
    assert ph["wait_gu_gemv"]["median_us"] == pytest.approx(2 * 15 / 1e3)
    assert ph["attn_scores_busy_kcycles"]["median_us"] == pytest.approx(2 * 1000 / 1e3)
    assert ph["head_prologue"]["median_us"] == pytest.approx(60 / 1e3)
    assert ph["head_gemv"]["median_us"] == pytest.approx(200 / 1e3)
    assert ph["argmax"]["max_us"] == pytest.approx(5 / 1e3)
    assert ph["setup"]["median_us"] == pytest.approx(50 / 1e3)
    assert ph["producer_slots"]["median_us"] == 77
    assert ph["producer_wait_slot_us"]["max_us"] == pytest.approx(1002 / 1e3)
    # the slowest CTA's end of argmax, from its own start
    ends = raw[:, 2 + TL * NL + 2].astype(float) - raw[:, 0]
    assert out["total_us"] == pytest.approx(ends.max() / 1e3)
