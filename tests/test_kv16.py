"""The compressed-KV lane (binary16 cache) on the CPU: its rounding rule, its oracle, its
accuracy against the reference's fp32-cache decode, and the host plumbing that selects
the _f16 entry points. The kernels themselves are checked on the GPU
(test_gpu_kv16.py)."""
import struct

import numpy as np
import pytest

import hv_oracle as O
import synth
import w4format

F32 = np.float32
LN2 = 0.6931471805599453


def ieee_half_bits(x: float) -> int:
    """binary16 bits of x by Python's own IEEE packing (round to nearest, ties to even)."""
    return struct.unpack("<H", struct.pack("<e", x))[0]


def test_f16_rounding_matches_ieee_packing():
    """numpy's float32 -> float16 (the oracle's kv_round) is IEEE round-to-nearest-even:
    random values over the whole finite range, exact midpoints between neighbouring
    halves (ties), the subnormal range and the top of the range."""
    g = np.random.default_rng(0)
    xs = [(g.standard_normal(20000) * np.exp2(g.integers(-30, 16, 20000))).astype(F32)]
    # midpoints of adjacent binary16 values (exact in float32): ties go to the even one
    h = np.arange(0, 0x7BFF, 7, dtype=np.uint16).view(np.float16).astype(F32)
    h1 = (np.arange(0, 0x7BFF, 7, dtype=np.uint16) + 1).view(np.float16).astype(F32)
    mid = ((h.astype(np.float64) + h1) / 2).astype(F32)
    assert np.array_equal(mid.astype(np.float64), (h.astype(np.float64) + h1) / 2)
    xs += [mid, -mid, np.nextafter(mid, np.inf).astype(F32), np.nextafter(mid, -np.inf).astype(F32)]
    xs.append(np.array([0.0, -0.0, 5.9604645e-08, 2.9802322e-08, 2.9802326e-08, 6.1035156e-05,
                        65504.0, 65519.996, -65519.996, 1e-10, -1e-10], F32))
    x = np.concatenate(xs)
    x = x[np.abs(x) < F32(65520.0)]          # overflow: test_f16_overflow_and_nan
    assert x.size > 30000
    got = x.astype(np.float16).view(np.uint16)
    want = np.array([ieee_half_bits(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, want)


def test_f16_overflow_and_nan():
    """Beyond the largest half the rounding goes to infinity (65520 is the first value that
    rounds up past 65504); NaN stays NaN. CUDA's __float2half_rn follows the same IEEE
    rule; the GPU test checks the device conversion on these values."""
    x = np.array([65520.0, -65520.0, 1e6, np.inf, -np.inf, np.nan, 65519.996], F32)
    with np.errstate(over="ignore"):
        h = x.astype(np.float16)
    assert np.isposinf(h[0]) and np.isneginf(h[1]) and np.isposinf(h[2])
    assert np.isposinf(h[3]) and np.isneginf(h[4]) and np.isnan(h[5])
    assert h[6] == np.float16(65504.0)


CASES = [("decode_tiny.npz", synth.tiny_arch(), 7),
         ("decode_tiny_tied.npz", synth.tiny_arch(n_layer=3, hidden=512, ffn=1024, n_head=8,
                                                  n_kv=2, vocab=2048, tied=True), 8),
         ("decode_tiny_long.npz", synth.tiny_arch(), 9)]


@pytest.mark.parametrize("name,arch,seed", CASES)
def test_oracle_kv16_lane_against_reference(golden, name, arch, seed):
    """The lane's oracle against the reference's own fp32-cache decode: the cache holds
    only binary16 values; logits up to the first token fork stay within 2.5e-2 of the
    logit scale (measured: at most 1.46e-2 on these models, the size of the model's
    sensitivity to last-bit changes in exp); tokens agree or fork at a near-tie (top-2
    margin below ln 2 in the reference's logits, the acceptance rule of the reference's
    verify.py:57-81)."""
    g = golden(name)
    cfg = w4format.Config(arch)
    w = O.quantize_model(cfg, synth.model_tensors(cfg, seed))
    ids, want = g["prompt"].tolist(), g["tokens"].tolist()
    m = O.OracleModel(cfg, w, len(ids) + len(want) + 2, kv_dtype="f16")
    toks, logits = m.generate(ids, len(want))
    used = len(ids) + len(want) - 1            # positions written
    for C in (m.KC, m.VC):
        held = C[:, :, :used]
        assert np.array_equal(held, held.astype(np.float16).astype(F32))
    first = next((i for i, (a, b) in enumerate(zip(toks, want)) if a != b), None)
    ref = g["logits"]
    upto = len(want) if first is None else first
    for i in range(upto + 1):
        err = np.abs(logits[i].astype(np.float64) - ref[i]).max() / np.abs(ref[i]).max()
        assert err < 2.5e-2, (i, err)
    if first is not None:
        top = np.sort(ref[first])[::-1]
        assert top[0] - top[1] < LN2, (first, top[0] - top[1])


def test_oracle_f32_lane_is_unchanged(golden):
    """kv_dtype="f32" (the default) is the reference's step, bit for bit."""
    g = golden("decode_tiny.npz")
    cfg = w4format.Config(synth.tiny_arch())
    w = O.quantize_model(cfg, synth.model_tensors(cfg, 7))
    ids = g["prompt"].tolist()
    m = O.OracleModel(cfg, w, 20, kv_dtype="f32")
    toks, logits = m.generate(ids, int(g["n_new"]))
    assert toks == g["tokens"].tolist()
    assert np.array_equal(np.stack(logits).view(np.uint32), g["logits"].view(np.uint32))
    with pytest.raises(ValueError):
        O.OracleModel(cfg, w, 20, kv_dtype="bf16")


def test_driver_routes_f16_calls(monkeypatch):
    """hvdrv's f16=True selects the _f16 entry points, with the same arguments."""
    import hvdrv
    seen = []
    monkeypatch.setattr(hvdrv, "_call", lambda name, *a: seen.append((name, len(a))))
    for f16 in (False, True):
        hvdrv.kv_append(1, 2, 3, 4, 5, 2, 128, 64, f16=f16)
        hvdrv.attn_decode(1, 2, 3, 4, 5, 6, 8, 128, 4, 64 * 128, f16=f16)
        hvdrv.qk_rows(1, 2, 3, 4, 5, 0, 7, 8, 9, 8, 2, 128, 64, 1e-5, 3, f16=f16)
        hvdrv.attn_rows(1, 2, 3, 4, 5, 0, 8, 128, 4, 64 * 128, 3, 6, 7, f16=f16)
    names = [n for n, _ in seen]
    assert names == ["hv_kv_append", "hv_attn_decode", "hv_qk_rows", "hv_attn_rows",
                     "hv_kv_append_f16", "hv_attn_decode_f16", "hv_qk_rows_f16",
                     "hv_attn_rows_f16"]
    assert [k for _, k in seen[:4]] == [k for _, k in seen[4:]]
    for name in names:
        assert name in hvdrv._SIGS
    assert [len(hvdrv._SIGS[n]) for n in names[:4]] == [len(hvdrv._SIGS[n]) for n in names[4:]]


def test_engine_rejects_unknown_kv_dtype():
    import limited
    with pytest.raises(ValueError, match="kv_dtype"):
        limited.Engine(config=synth.tiny_arch(), tensors={}, kv_dtype="bf16")


def test_engine_rejects_bad_gemv_layout():
    """Checked before any device work."""
    import limited
    with pytest.raises(ValueError, match="gemv_layout"):
        limited.Engine(config=synth.tiny_arch(), tensors={}, gemv_layout="rowmajor")
