"""Pin the C restatement of the GEMV to the numpy oracle and the reference's goldens."""
import numpy as np
import pytest

import hv_oracle as O

F32 = np.float32


@pytest.mark.parametrize("i", range(5))
def test_c_gemv_matches_reference_golden(golden, i):
    g = golden("ops.npz")
    a, p, sc = g[f"gv{i}_a"], g[f"gv{i}_packed"], g[f"gv{i}_scale"]
    qa, sa, _ = O.quantize_act(a)
    idot, y = O.gemv_q_c(qa, sa, p, sc, a.size, want_idot=True)
    assert np.array_equal(idot, g[f"gv{i}_idot"])
    assert np.array_equal(y.view(np.uint32), g[f"gv{i}_y"].view(np.uint32))


@pytest.mark.parametrize("n,k", [(37, 32), (5, 224), (16, 2048), (9, 5120), (4, 12288),
                                 (3, 25600), (7, 32 * 1000)])
def test_c_gemv_matches_numpy_oracle(n, k):
    g = np.random.default_rng(n * 7 + k)
    p, sc = O.quantize_w4((g.standard_normal((n, k)) * 0.02).astype(F32))
    a = g.standard_normal(k).astype(F32) * F32(3.0)
    qa, sa, _ = O.quantize_act(a)
    i1, y1 = O.gemv_q(qa, sa, p, sc, k)
    i2, y2 = O.gemv_q_c(qa, sa, p, sc, k, want_idot=True)
    assert np.array_equal(i1, i2)
    assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))


def test_c_pairwise_sum_is_numpys():
    lib = O._clib()
    for n in (1, 7, 8, 100, 129, 800, 4096, 5120, 25600):
        x = (np.random.default_rng(n).standard_normal(n) * 10).astype(F32)
        got = lib.hvo_pairwise_sum(x.ctypes.data, n)
        assert np.float32(got).view(np.uint32) == x.sum().view(np.uint32)


def test_fast_oracle_model_matches_reference_decode(golden):
    import synth
    import w4format
    g = golden("decode_tiny.npz")
    cfg = w4format.Config(synth.tiny_arch())
    w = O.quantize_model(cfg, synth.model_tensors(cfg, 7))
    m = O.FastOracleModel(cfg, w, 5 + 12 + 2)
    toks, logits = m.generate(g["prompt"].tolist(), 12)
    assert toks == g["tokens"].tolist()
    assert np.array_equal(np.stack(logits).view(np.uint32), g["logits"].view(np.uint32))


def test_c_quantizer_matches_reference(golden):
    g = golden("ops.npz")
    p, s = O.quantize_w4_c(g["qw_in"])
    assert np.array_equal(p, g["qw_packed"])
    assert np.array_equal(s.view(np.uint32), g["qw_scale"].view(np.uint32))
    w = (np.random.default_rng(9).standard_normal((70, 4096)) * 0.02).astype(F32)
    p1, s1 = O.quantize_w4(w)
    p2, s2 = O.quantize_w4_c(w)
    assert np.array_equal(p1, p2) and np.array_equal(s1.view(np.uint32), s2.view(np.uint32))


def test_quantize_model_c_matches_numpy():
    import synth
    import w4format
    for arch in (synth.tiny_arch(), synth.tiny_arch(tied=True)):
        cfg = w4format.Config(arch)
        a = O.quantize_model(cfg, synth.model_tensors(cfg, 3))
        b = O.quantize_model_c(cfg, synth.iter_tensors(cfg, 3))
        assert sorted(a) == sorted(b)
        for key in a:
            if isinstance(a[key], tuple):
                assert all(np.array_equal(x, y) for x, y in zip(a[key], b[key])), key
            else:
                assert np.array_equal(a[key], b[key]), key


@pytest.mark.skipif(not __import__("os").environ.get("HV_SLOW_TESTS"),
                    reason="set HV_SLOW_TESTS=1 (the 1.7B and 8B models drawn and quantised)")
@pytest.mark.parametrize("name,workload,n_new", [
    ("decode_qwen3_1p7b.npz", "qwen3-1.7b-p32-g64", 64),
    ("decode_qwen3_8b_p4.npz", "qwen3-8b-p4096-g256", 2)])
def test_fast_oracle_matches_reference_at_real_shapes(golden, name, workload, n_new):
    """The oracle at the 1.7B and 8B geometries against the reference's own decode of the
    same seeded model (tests/golden, make_golden.py c1 / c3): the greedy tokens, and every
    step's logits bit for bit (sha256), on the host that made the fixtures (1.7B: all 64
    generated tokens)."""
    import hashlib

    import synth
    import w4format
    try:
        g = golden(name)
    except FileNotFoundError:
        pytest.skip(f"{name} not generated")
    arch, seed = synth.WORKLOADS[workload][:2]
    cfg = w4format.Config(synth.ARCH[arch])
    prompt = g["prompt"].tolist()
    assert prompt == synth.prompt_ids(cfg, seed, len(prompt))
    w = O.quantize_model_c(cfg, synth.iter_tensors(cfg, seed))
    m = O.FastOracleModel(cfg, w, len(prompt) + n_new + 2)
    toks, logits = m.generate(prompt, n_new)
    assert toks == g["tokens"].tolist()[:n_new]
    for i, lg in enumerate(logits):
        assert hashlib.sha256(np.ascontiguousarray(lg).tobytes()).hexdigest() == \
            str(g["logits_sha"][i]), i


def _numerics_inputs():
    import importlib.util
    from conftest import GOLDEN
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN / "make_golden.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    return mg.numerics_inputs()


def test_np_exp_restatement_matches_reference_host(golden):
    """hvo_np_expf == the reference host's np.exp on 327,680 float32 samples of exp's
    whole finite range (tests/golden/numerics.npz)."""
    g = golden("numerics.npz")
    got = O.np_exp(g["exp_x"])
    assert np.array_equal(got.view(np.uint32), g["exp_y"].view(np.uint32))


def test_blas_rowdots_restatement_matches_reference_host(golden):
    """hvo_blas_rowdots == the reference host's `keys @ q` (OpenBLAS gemv) for every row
    of 97 row counts: every remainder mod 4, the single-run limit and the split runs
    above it (tests/golden/numerics.npz)."""
    g = golden("numerics.npz")
    _, q, keys = _numerics_inputs()
    assert int(g["host_cpus"]) == O.BLAS_THREADS
    for T in g["dot_T"].tolist():
        got = O.blas_rowdots(keys[:T], q)
        assert np.array_equal(got.view(np.uint32), g[f"dot_{T}"].view(np.uint32)), T


def _host_like_reference():
    try:
        from numpy._core._multiarray_umath import __cpu_features__ as f
    except ImportError:
        return False
    return bool(f.get("AVX512F")) and bool(f.get("FMA3"))


@pytest.mark.skipif(not _host_like_reference(), reason="numpy without its AVX-512 exp kernel")
def test_np_exp_restatement_matches_live_numpy():
    """On a host whose numpy runs the same SIMD kernel: every 61st float32 of [-104, 0]."""
    b = np.arange(0x80000000, 0xC2D00001, 61, dtype=np.uint32)
    x = b.view(F32)
    assert np.array_equal(O.np_exp(x).view(np.uint32), np.exp(x).view(np.uint32))


@pytest.mark.skipif(not _host_like_reference(), reason="numpy without its AVX-512 kernels")
def test_blas_row_kinds_match_live_numpy_below_the_split():
    """Row counts below OpenBLAS's single-run limit do not depend on the host's thread
    count: there the restatement must equal this host's `keys @ q` too."""
    rng = np.random.default_rng(3)
    q = rng.standard_normal(128, dtype=F32)
    for T in list(range(2, 90)) + [513, 1022, 2047, 3599]:
        keys = rng.standard_normal((T, 128), dtype=F32)
        got = O.blas_rowdots(keys, q)
        assert np.array_equal(got.view(np.uint32), (keys @ q).view(np.uint32)), T
