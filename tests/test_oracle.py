"""Pin the numpy oracle to golden vectors produced by the reference's engine/reference.py.

CPU only. Every bit-exact claim the GPU tests rely on is first checked here: the oracle
reproduces the reference on the reference's own outputs.
"""
import hashlib

import numpy as np
import pytest

import hv_oracle as O
import synth
import w4format

F32 = np.float32


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == F32 else np.uint8)


def test_quantize_w4_matches_reference(golden):
    g = golden("ops.npz")
    p, s = O.quantize_w4(g["qw_in"])
    assert np.array_equal(p, g["qw_packed"])
    assert np.array_equal(bits(s), bits(g["qw_scale"]))
    # the product's host quantiser is an independent implementation of the same rule
    p2, s2 = w4format.quantize_w4(g["qw_in"])
    assert np.array_equal(p2, g["qw_packed"]) and np.array_equal(bits(s2), bits(s))


def test_unpack_roundtrip(golden):
    g = golden("ops.npz")
    q = O.unpack_w4(g["qw_packed"], g["qw_in"].shape[1])
    assert q.min() >= -7 and q.max() <= 7
    assert np.array_equal(q, w4format.unpack_w4(g["qw_packed"], g["qw_in"].shape[1]))


@pytest.mark.parametrize("i", [0, 1])
def test_quantize_act_matches_reference(golden, i):
    g = golden("ops.npz")
    q, s, bs = O.quantize_act(g[f"qa{i}_in"])
    assert np.array_equal(q.astype(np.int32), g[f"qa{i}_q"].reshape(-1))
    assert np.array_equal(bits(s), bits(g[f"qa{i}_s"]))
    assert np.array_equal(bs, g[f"qa{i}_bsum"])


@pytest.mark.parametrize("i", range(5))
def test_gemv_matches_reference_bit_exact(golden, i):
    g = golden("ops.npz")
    a, p, sc, y = g[f"gv{i}_a"], g[f"gv{i}_packed"], g[f"gv{i}_scale"], g[f"gv{i}_y"]
    k = a.size
    qa, sa, _ = O.quantize_act(a)
    idot, y2 = O.gemv_q(qa, sa, p, sc, k)
    assert np.array_equal(idot, g[f"gv{i}_idot"])
    assert np.array_equal(bits(y2), bits(y))


def test_pairwise_plan_shapes():
    assert O.pairwise_plan(128) == [(0, 128)]
    assert O.pairwise_plan(160) == [(0, 80), (80, 80)]
    assert [m for _, m in O.pairwise_plan(800)] == [96, 104] * 4
    assert [m for _, m in O.pairwise_plan(384)] == [96] * 4


@pytest.mark.parametrize("n", [1, 5, 8, 13, 64, 100, 128, 129, 160, 384, 800, 4096, 5120])
def test_pairwise_sum_is_numpys(n):
    x = (np.random.default_rng(n).standard_normal((3, n)) * 100).astype(F32)
    assert np.array_equal(bits(O.pairwise_sum(x)), bits(x.sum(1)))


@pytest.mark.parametrize("i", range(8))
def test_rmsnorm_matches_reference(golden, i):
    g = golden("ops.npz")
    y = O.rmsnorm(g[f"rn{i}_x"], g[f"rn{i}_w"])
    assert np.array_equal(bits(y), bits(g[f"rn{i}_y"]))


@pytest.mark.parametrize("i", range(4))
def test_rope_matches_reference(golden, i):
    g = golden("ops.npz")
    p = int(g[f"rp{i}_pos"])
    cos_t, sin_t = O.rope_tables(4400, 128, 1e6)
    assert np.array_equal(bits(cos_t[p]), bits(g[f"rp{i}_cos"]))
    assert np.array_equal(bits(sin_t[p]), bits(g[f"rp{i}_sin"]))
    y = O.rope(g[f"rp{i}_v"], p, cos_t, sin_t)
    assert np.array_equal(bits(y), bits(g[f"rp{i}_y"]))


def test_silu_matches_reference(golden):
    g = golden("ops.npz")
    y = O.silu_mul(g["silu_g"], g["silu_u"])
    assert np.array_equal(bits(y), bits(g["silu_y"]))


@pytest.mark.parametrize("i", range(3))
def test_attention_matches_reference(golden, i):
    g = golden("ops.npz")
    q = g[f"at{i}_q"]
    nkv = g[f"at{i}_kc"].shape[0]
    y = O.attention(q, g[f"at{i}_kc"], g[f"at{i}_vc"], int(g[f"at{i}_pos"]),
                    q.shape[0] // nkv, 1.0 / np.sqrt(128))
    np.testing.assert_allclose(y, g[f"at{i}_y"], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("name,arch,seed,n_prompt", [
    ("decode_tiny.npz", synth.tiny_arch(), 7, 5),
    ("decode_tiny_tied.npz", synth.tiny_arch(n_layer=3, hidden=512, ffn=1024, n_head=8,
                                             n_kv=2, vocab=2048, tied=True), 8, 9),
    ("decode_tiny_long.npz", synth.tiny_arch(), 9, 300),
    ("decode_tiny_2k.npz", synth.tiny_arch(), 10, 2000),
])
def test_oracle_model_matches_reference_decode(golden, name, arch, seed, n_prompt):
    g = golden(name)
    cfg = w4format.Config(arch)
    w = O.quantize_model(cfg, synth.model_tensors(cfg, seed))
    ids = synth.prompt_ids(cfg, seed, n_prompt)
    assert ids == g["prompt"].tolist()
    n_new = int(g["n_new"])
    m = O.OracleModel(cfg, w, n_prompt + n_new + 2)
    toks, logits = m.generate(ids, n_new)
    assert toks == g["tokens"].tolist()
    got = np.stack(logits)
    # same host, same numpy: the oracle reproduces the reference bit for bit
    assert np.array_equal(bits(got), bits(g["logits"]))


def test_gemv_sweep_digests(golden):
    """The sweep's reference outputs, re-derived from the seeds (small shapes only here;
    the GPU tests cover every shape)."""
    try:
        g = golden("gemv_sweep.npz")
    except FileNotFoundError:
        pytest.skip("gemv_sweep.npz not generated yet")
    for j, (n, k) in enumerate(synth.GEMV_SHAPES[:3]):
        w, a = synth.gemv_case(j, n, k)
        p, sc = O.quantize_w4(w)
        assert hashlib.sha256(p.tobytes()).hexdigest() == str(g[f"s{j}_packed_sha"])
        assert hashlib.sha256(sc.tobytes()).hexdigest() == str(g[f"s{j}_scale_sha"])
        y = O.gemv_w4(a, p, sc, k)
        assert hashlib.sha256(y.tobytes()).hexdigest() == str(g[f"s{j}_y_sha"])
