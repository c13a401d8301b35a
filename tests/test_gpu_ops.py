"""Per-kernel parity on a B200, through the C ABI, against the reference's golden vectors
and the oracle. Every op is bit-exact: integer and byte work, and every float op, the
exp-based SiLU and softmax attention included (numpy's exp and OpenBLAS's row-dot order
are restated by the kernels)."""
import numpy as np
import pytest

import hv_oracle as O
from gpu_util import Dev, bits, quantize_on_device

pytestmark = pytest.mark.gpu
F32 = np.float32


@pytest.mark.parametrize("i", [0, 1])
def test_qa8s_bit_exact(hv, golden, i):
    g = golden("ops.npz")
    a = g[f"qa{i}_in"]
    a8, sa = quantize_on_device(a)
    nb = a.size // 32
    q = a8.get(np.int8)
    s = sa.get(F32)
    assert np.array_equal(q.astype(np.int32), g[f"qa{i}_q"].reshape(-1))
    assert np.array_equal(bits(s[:nb]), bits(g[f"qa{i}_s"]))
    assert np.array_equal(s[nb:].view(np.int32), g[f"qa{i}_bsum"])


@pytest.mark.parametrize("i", range(5))
def test_a4gv_bit_exact_on_reference_goldens(hv, golden, i):
    g = golden("ops.npz")
    a, p, sc = g[f"gv{i}_a"], g[f"gv{i}_packed"], g[f"gv{i}_scale"]
    n, k = p.shape[0], a.size
    a8, sa = quantize_on_device(a)
    b4, sw = Dev(p), Dev(sc)
    y, idot = Dev(nbytes=n * 4), Dev(nbytes=n * (k // 32) * 4)
    hv.a4gv_idot(a8, sa, b4, sw, y, idot, k // 8, n)
    assert np.array_equal(idot.get(np.int32, (n, k // 32)), g[f"gv{i}_idot"])
    assert np.array_equal(bits(y.get(F32)), bits(g[f"gv{i}_y"]))
    y2 = Dev(nbytes=n * 4)
    hv.a4gv(a8, sa, b4, sw, y2, k // 8, n)
    assert np.array_equal(bits(y2.get(F32)), bits(g[f"gv{i}_y"]))


@pytest.mark.parametrize("n,k", [(1, 32), (3, 96), (5, 256), (13, 416), (4097, 2048),
                                 (777, 4096), (130, 5120), (64, 8192), (33, 12288),
                                 (21, 25600), (2, 32 * 1000), (6, 32 * 4096)])
def test_a4gv_bit_exact_vs_oracle(hv, n, k):
    g = np.random.default_rng(n + k)
    p, sc = O.quantize_w4((g.standard_normal((n, k)) * 0.02).astype(F32))
    a = (g.standard_normal(k) * g.uniform(0.1, 5)).astype(F32)
    a[:32] = 0.0                                       # an all-zero activation block
    qa, sa_h, _ = O.quantize_act(a)
    want_idot, want_y = O.gemv_q_c(qa, sa_h, p, sc, k, want_idot=True)
    a8, sa = quantize_on_device(a)
    y, idot = Dev(nbytes=n * 4), Dev(nbytes=n * (k // 32) * 4)
    hv.a4gv_idot(a8, sa, Dev(p), Dev(sc), y, idot, k // 8, n)
    assert np.array_equal(idot.get(np.int32, (n, k // 32)), want_idot)
    assert np.array_equal(bits(y.get(F32)), bits(want_y))


def test_a4gv_rejects_bad_shapes(hv):
    with pytest.raises(hv.CudaError):
        hv.a4gv(16, 16, 16, 16, 16, 3, 4)     # K = 24 is not a multiple of 32


def test_quantize_w4_device_bit_exact(hv, golden):
    g = golden("ops.npz")
    w = g["qw_in"]
    n, k = w.shape
    p, s = Dev(nbytes=n * k // 2), Dev(nbytes=n * k // 32 * 4)
    hv.quantize_w4(Dev(w), p, s, n, k)
    assert np.array_equal(p.get(np.uint32, (n, k // 8)), g["qw_packed"])
    assert np.array_equal(bits(s.get(F32, (n, k // 32))), bits(g["qw_scale"]))
    w2 = (np.random.default_rng(3).standard_normal((300, 4096)) * 0.02).astype(F32)
    p2, s2 = Dev(nbytes=300 * 2048), Dev(nbytes=300 * 128 * 4)
    hv.quantize_w4(Dev(w2), p2, s2, 300, 4096)
    wp, ws = O.quantize_w4(w2)
    assert np.array_equal(p2.get(np.uint32, wp.shape), wp)
    assert np.array_equal(bits(s2.get(F32, ws.shape)), bits(ws))


@pytest.mark.parametrize("i", range(8))
def test_rmsnorm_bit_exact(hv, golden, i):
    g = golden("ops.npz")
    x, w, want = g[f"rn{i}_x"], g[f"rn{i}_w"], g[f"rn{i}_y"]
    rows, cols = (1, x.size) if x.ndim == 1 else x.shape
    out = Dev(nbytes=x.nbytes)
    hv.rmsnorm(Dev(x), out, Dev(w), rows, cols, 1e-5)
    assert np.array_equal(bits(out.get(F32, x.shape)), bits(want))
    inplace = Dev(x)
    hv.rmsnorm(inplace, inplace, Dev(w), rows, cols, 1e-5)
    assert np.array_equal(bits(inplace.get(F32, x.shape)), bits(want))


@pytest.mark.parametrize("i", range(4))
def test_rope_bit_exact(hv, golden, i):
    g = golden("ops.npz")
    v, p = g[f"rp{i}_v"], int(g[f"rp{i}_pos"])
    cos_t, sin_t = O.rope_tables(4400, 128, 1e6)
    vec = Dev(v)
    hv.rope(vec, Dev(cos_t), Dev(sin_t), Dev(np.array([p], np.int32)), v.shape[0], 64)
    assert np.array_equal(bits(vec.get(F32, v.shape)), bits(g[f"rp{i}_y"]))


def test_silu_within_exp_rounding(hv, golden):
    """np.exp and CUDA's expf differ in the last bit now and then. In the reference's
    sign-split form sigma = 0.5 (1 + (1 - e) / (1 + e)), one ulp of e moves sigma by at
    most ~2^-24 absolute (1 - e cancels near g = 0, so ulps of the output are the wrong
    yardstick). Bound: |got - want| <= 2^-21 |g u| + 1e-37."""
    g = golden("ops.npz")
    gt, up, want = g["silu_g"], g["silu_u"], g["silu_y"]
    out = Dev(nbytes=gt.nbytes)
    hv.silu_mul(Dev(gt), Dev(up), out, gt.size)
    got = out.get(F32)
    scale = np.abs(gt.astype(np.float64) * up)
    err = np.abs(got.astype(np.float64) - want)
    worst = float((err / np.maximum(scale, 1e-30)).max())
    print(f"silu: max |diff| / |g u| = {worst:.2e}; exact in "
          f"{np.mean(got.view(np.uint32) == want.view(np.uint32)):.1%} of values")
    assert np.all(err <= 2.0 ** -21 * scale + 1e-37)


def test_vadd_gather_kvapp_exact(hv):
    g = np.random.default_rng(1)
    a, b = g.standard_normal(4096).astype(F32), g.standard_normal(4096).astype(F32)
    out = Dev(nbytes=a.nbytes)
    hv.vadd(Dev(a), Dev(b), out, a.size)
    assert np.array_equal(bits(out.get(F32)), bits((a + b).astype(F32)))
    emb = (g.standard_normal((50, 256)) * 0.02).astype(np.float16)
    h = Dev(nbytes=256 * 4)
    hv.gather_emb(Dev(emb), Dev(np.array([37], np.int32)), h, 256)
    assert np.array_equal(h.get(F32), emb[37].astype(F32))
    nkv, cap, hd = 3, 20, 128
    kc, vc = Dev(nbytes=nkv * cap * hd * 4), Dev(nbytes=nkv * cap * hd * 4)
    k, v = g.standard_normal((nkv, hd)).astype(F32), g.standard_normal((nkv, hd)).astype(F32)
    hv.kv_append(Dev(k), Dev(v), kc, vc, Dev(np.array([11], np.int32)), nkv, hd, cap)
    KC, VC = kc.get(F32, (nkv, cap, hd)), vc.get(F32, (nkv, cap, hd))
    assert np.array_equal(KC[:, 11], k) and np.array_equal(VC[:, 11], v)
    assert not KC[:, :11].any() and not KC[:, 12:].any()


@pytest.mark.parametrize("i", range(3))
def test_attention_matches_reference(hv, golden, i):
    g = golden("ops.npz")
    q, kc, vc, pos = g[f"at{i}_q"], g[f"at{i}_kc"], g[f"at{i}_vc"], int(g[f"at{i}_pos"])
    nq, nkv, cap = q.shape[0], kc.shape[0], kc.shape[1]
    ctx = Dev(nbytes=q.nbytes)
    scale = Dev(np.array([1.0 / np.sqrt(128)], F32))
    hv.attn_decode(Dev(q), Dev(kc), Dev(vc), ctx, scale, Dev(np.array([pos], np.int32)), nq,
                   128, nq // nkv, cap * 128)
    assert np.array_equal(bits(ctx.get(F32, q.shape)), bits(g[f"at{i}_y"]))


@pytest.mark.parametrize("nq,nkv,pos,cap", [(32, 8, 4224, 4352), (64, 8, 2300, 2304),
                                             (16, 8, 0, 64), (8, 8, 5000, 8192)])
def test_attention_long_context_vs_oracle(hv, nq, nkv, pos, cap):
    g = np.random.default_rng(pos)
    q = g.standard_normal((nq, 128)).astype(F32)
    kc = g.standard_normal((nkv, cap, 128)).astype(F32)
    vc = g.standard_normal((nkv, cap, 128)).astype(F32)
    want = O.attention(q, kc, vc, pos, nq // nkv, 1.0 / np.sqrt(128))
    ctx = Dev(nbytes=q.nbytes)
    scale = Dev(np.array([1.0 / np.sqrt(128)], F32))
    hv.attn_decode(Dev(q), Dev(kc), Dev(vc), ctx, scale, Dev(np.array([pos], np.int32)), nq,
                   128, nq // nkv, cap * 128)
    assert np.array_equal(bits(ctx.get(F32, q.shape)), bits(want))


def test_argmax_ties_lowest_and_device_state(hv):
    g = np.random.default_rng(5)
    n = 151936
    logits = g.standard_normal(n).astype(F32)
    logits[[500, 90000, 151935]] = 9.0              # a three-way tie at the max
    pv, pi = Dev(nbytes=128 * 4), Dev(nbytes=128 * 4)
    tok, step, pos = Dev(np.array([0], np.int32)), Dev(np.array([3], np.int32)), \
        Dev(np.array([41], np.int32))
    gen = Dev(nbytes=16 * 4)
    hv.argmax_partial(Dev(logits), pv, pi, n, 128)
    hv.argmax_final(pv, pi, tok, gen, step, pos, 128)
    assert tok.get(np.int32)[0] == 500 == O.argmax(logits)
    assert gen.get(np.int32)[3] == 500
    assert step.get(np.int32)[0] == 4 and pos.get(np.int32)[0] == 42


@pytest.mark.parametrize("n,k,pair", [(5, 32, 0), (13, 416, 0), (777, 4096, 0), (64, 12288, 0),
                                      (21, 25600, 0), (26, 2048, 13), (24576, 4096, 12288),
                                      (10, 160, 5)])
def test_prepack_roundtrip_and_gemv_pp_bit_exact(hv, n, k, pair):
    """hv_w4_prepack only reorders (download + inverse gives the reference layout back);
    the GEMV over the reordered layout is bit-exact with the oracle, rows in reference
    order (for a paired [gate | up] matrix too)."""
    from gpu_util import unprepack
    g = np.random.default_rng(n * 31 + k)
    p, sc = O.quantize_w4((g.standard_normal((n, k)) * 0.02).astype(F32))
    nib, scb = hv.w4_prepacked_size(n, k, pair)
    pb4, psw = Dev(nbytes=nib), Dev(nbytes=scb)
    hv.w4_prepack(Dev(p), Dev(sc), n, k, pair, pb4, psw)
    p2, s2 = unprepack(pb4.get(np.uint32), psw.get(F32), n, k, pair)
    assert np.array_equal(p2, p) and np.array_equal(bits(s2), bits(sc))
    a = (g.standard_normal(k) * 2).astype(F32)
    qa, sa_h, _ = O.quantize_act(a)
    _, want = O.gemv_q_c(qa, sa_h, p, sc, k)
    a8, sa = quantize_on_device(a)
    y = Dev(nbytes=n * 4)
    hv.a4gv_pp(a8, sa, pb4, psw, y, k // 8, n, pair)
    assert np.array_equal(bits(y.get(F32)), bits(want))


@pytest.mark.parametrize("n,k,pair", [(8, 256, 0), (40, 16384, 0), (100, 12288, 0),
                                      (2048, 6144, 0), (24, 2048, 12), (3000, 4096, 0),
                                      (8, 4096, 0), (24, 4096, 12)])
def test_gemv_split_kernel_bit_identical(hv, n, k, pair):
    """hv_a4gv_pp on the iteration-split kernel (few tiles and K >= 4096, the default)
    and on the one-warp-per-tile kernel give the same bits, and both the oracle's
    (multi-leaf plans, gate/up pairs and the 64-iteration limit included)."""
    g = np.random.default_rng(n + 7 * k)
    p, sc = O.quantize_w4((g.standard_normal((n, k)) * 0.02).astype(F32))
    nib, scb = hv.w4_prepacked_size(n, k, pair)
    pb4, psw = Dev(nbytes=nib), Dev(nbytes=scb)
    hv.w4_prepack(Dev(p), Dev(sc), n, k, pair, pb4, psw)
    a = (g.standard_normal(k) * 2).astype(F32)
    qa, sa_h, _ = O.quantize_act(a)
    _, want = O.gemv_q_c(qa, sa_h, p, sc, k)
    a8, sa = quantize_on_device(a)
    out = []
    try:
        for split in (True, False):
            hv.gemv_set_split(split)
            y = Dev(nbytes=n * 4)
            hv.a4gv_pp(a8, sa, pb4, psw, y, k // 8, n, pair)
            out.append(y.get(F32))
    finally:
        hv.gemv_set_split(True)
    assert np.array_equal(bits(out[0]), bits(out[1]))
    assert np.array_equal(bits(out[0]), bits(want))
