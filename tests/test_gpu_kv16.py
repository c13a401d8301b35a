"""The compressed-KV lane (binary16 cache) on a B200.

* hv_kv_append_f16 stores numpy's astype(float16) of each value, bit for bit (ties,
  subnormals, overflow to infinity included);
* hv_attn_decode_f16 and hv_attn_rows_f16 are bit-identical to their f32 counterparts
  run over an f32 cache that holds the same values widened, and hv_qk_rows_f16 stores
  hv_qk_rows' rows rounded: the lane changes only what the cache holds;
* the engine with kv_dtype="f16": fused step bit-identical to the eager kernel sequence
  and to the batched prefill, tokens and logits identical to the lane's oracle, half the
  KV bytes.
"""
import numpy as np
import pytest

import hv_oracle as O
import synth
import w4format
from gpu_util import Dev, bits

pytestmark = pytest.mark.gpu
F32 = np.float32
F16 = np.float16


def test_kv_append_f16_rounds_like_numpy(hv):
    nkv, cap, hd, pos = 3, 24, 128, 17
    g = np.random.default_rng(3)
    k = (g.standard_normal((nkv, hd)) * np.exp2(g.integers(-26, 17, (nkv, hd)))).astype(F32)
    v = g.standard_normal((nkv, hd)).astype(F32)
    # ties between neighbouring halves, the overflow edge, subnormals, signed zero
    h = np.arange(0x3C00, 0x3C00 + 64, dtype=np.uint16).view(F16).astype(np.float64)
    k[0, :63] = ((h[:-1] + h[1:]) / 2).astype(F32)
    k[1, :8] = np.array([65519.996, 65520.0, -65520.0, 1e6, 2.9802322e-08, 2.9802326e-08,
                         -0.0, 5.9604645e-08], F32)
    kc, vc = Dev(nbytes=nkv * cap * hd * 2), Dev(nbytes=nkv * cap * hd * 2)
    hv.kv_append(Dev(k), Dev(v), kc, vc, Dev(np.array([pos], np.int32)), nkv, hd, cap,
                 f16=True)
    KC, VC = kc.get(np.uint16, (nkv, cap, hd)), vc.get(np.uint16, (nkv, cap, hd))
    with np.errstate(over="ignore"):
        assert np.array_equal(KC[:, pos], k.astype(F16).view(np.uint16))
        assert np.array_equal(VC[:, pos], v.astype(F16).view(np.uint16))
    assert not KC[:, :pos].any() and not KC[:, pos + 1:].any()


@pytest.mark.parametrize("nq,nkv,pos,cap", [(32, 8, 4224, 4352), (16, 8, 0, 64),
                                             (8, 2, 2000, 2048), (8, 8, 700, 1024)])
def test_attn_decode_f16_equals_f32_on_widened_cache(hv, nq, nkv, pos, cap):
    g = np.random.default_rng(pos + nq)
    q = g.standard_normal((nq, 128)).astype(F32)
    k16 = g.standard_normal((nkv, cap, 128)).astype(F16)
    v16 = g.standard_normal((nkv, cap, 128)).astype(F16)
    scale = Dev(np.array([1.0 / np.sqrt(128)], F32))
    dpos = Dev(np.array([pos], np.int32))
    a, b = Dev(nbytes=q.nbytes), Dev(nbytes=q.nbytes)
    dq = Dev(q)
    hv.attn_decode(dq, Dev(k16), Dev(v16), a, scale, dpos, nq, 128, nq // nkv, cap * 128,
                   f16=True)
    hv.attn_decode(dq, Dev(k16.astype(F32)), Dev(v16.astype(F32)), b, scale, dpos, nq, 128,
                   nq // nkv, cap * 128)
    assert np.array_equal(bits(a.get(F32)), bits(b.get(F32)))
    want = O.attention(q, k16.astype(F32), v16.astype(F32), pos, nq // nkv, 1.0 / np.sqrt(128))
    assert np.array_equal(bits(a.get(F32, q.shape)), bits(want))


def test_prefill_rows_f16_equal_f32_rows(hv):
    nq, nkv, hd, cap, pos0, ntok, eps = 8, 2, 128, 320, 37, 40, 1e-5
    g = np.random.default_rng(9)
    qkv = g.standard_normal((ntok, (nq + 2 * nkv) * hd)).astype(F32)
    qn = (1 + 0.01 * g.standard_normal(hd)).astype(F32)
    kn = (1 + 0.01 * g.standard_normal(hd)).astype(F32)
    cos_t, sin_t = O.rope_tables(cap, hd, 1e6)
    hist = g.standard_normal((nkv, cap, hd)).astype(F16)       # positions before pos0
    hist[:, pos0:] = 0
    d = {n: Dev(x) for n, x in (("qkv", qkv), ("qn", qn), ("kn", kn),
                                ("cos", cos_t.astype(F32)), ("sin", sin_t.astype(F32)))}
    out = {}
    for f16 in (False, True):
        kc = Dev(hist if f16 else hist.astype(F32))
        vc = Dev(hist if f16 else hist.astype(F32))
        qo = Dev(nbytes=ntok * nq * hd * 4)
        hv.qk_rows(d["qkv"], d["qn"], d["kn"], d["cos"], d["sin"], pos0, qo, kc, vc, nq, nkv,
                   hd, cap, eps, ntok, f16=f16)
        dt = F16 if f16 else F32
        out[f16] = (qo.get(F32), kc.get(dt, (nkv, cap, hd)), vc.get(dt, (nkv, cap, hd)), kc, vc)
    q32, k32, v32, _, _ = out[False]
    q16, k16, v16, kc16, vc16 = out[True]
    assert np.array_equal(bits(q32), bits(q16))
    assert np.array_equal(k16.view(np.uint16), k32.astype(F16).view(np.uint16))
    assert np.array_equal(v16.view(np.uint16), v32.astype(F16).view(np.uint16))
    # attention over the two caches: f16 rows vs f32 rows holding the same values
    scale = Dev(np.array([1.0 / np.sqrt(hd)], F32))
    pb, tb = hv.attn_rows_scratch(nq, nq // nkv, cap, ntok)
    res = []
    for f16, kc, vc in ((True, kc16, vc16),
                        (False, Dev(k16.astype(F32)), Dev(v16.astype(F32)))):
        part, ticket, ctx = Dev(nbytes=pb), Dev(nbytes=tb), Dev(nbytes=ntok * nq * hd * 4)
        hv.attn_rows(Dev(q16), kc, vc, ctx, scale, pos0, nq, hd, nq // nkv, cap * hd, ntok,
                     part, ticket, f16=f16)
        res.append(ctx.get(F32))
    assert np.array_equal(bits(res[0]), bits(res[1]))


def make_engine(arch, seed, cap, **kw):
    import limited
    cfg = w4format.Config(arch)
    return limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, seed), quiet=True,
                          max_context=cap, **kw)


def rel_err(got, want):
    return float(np.abs(got.astype(np.float64) - want).max() / np.abs(want).max())


@pytest.mark.parametrize("name,seed", [("decode_tiny.npz", 7), ("decode_tiny_long.npz", 9)])
def test_engine_f16_lane_matches_its_oracle(hv, golden, name, seed):
    """Fused f16 engine: tokens equal to the lane's oracle (OracleModel kv_dtype="f16"),
    every step's logits bit-identical to it; eager and batched-prefill engines
    bit-identical to it; KV bytes half the f32 engine's."""
    g = golden(name)
    arch = synth.tiny_arch()
    cfg = w4format.Config(arch)
    prompt, n_new = g["prompt"].tolist(), int(g["n_new"])
    cap = len(prompt) + n_new + 2
    m = O.OracleModel(cfg, O.quantize_model(cfg, synth.model_tensors(cfg, seed)), cap,
                      kv_dtype="f16")
    want_toks, want_logits = m.generate(prompt, n_new)
    fused = make_engine(arch, seed, cap, kv_dtype="f16")
    eager = make_engine(arch, seed, cap, kv_dtype="f16", fused=False)
    batched = make_engine(arch, seed, cap, kv_dtype="f16", prefill="batched")
    f32 = make_engine(arch, seed, cap)
    try:
        assert fused.kv_bytes * 2 == f32.kv_bytes
        toks, _, _ = fused.generate(prompt, n_new, stop_on_eos=False)
        assert toks == want_toks
        errs = []
        for i in range(n_new + 1):
            ids = prompt + toks[:i]
            lf = fused.logits(ids)
            errs.append(rel_err(lf, want_logits[i]))
            assert np.array_equal(bits(lf), bits(want_logits[i])), (i, errs[-1])
            if i in (0, n_new):
                assert np.array_equal(bits(lf), bits(eager.logits(ids))), i
                assert np.array_equal(bits(lf), bits(batched.logits(ids))), i
        print(f"{name} f16 lane: logits rel err max {max(errs):.2e}")
        assert batched.generate(prompt, n_new)[0] == want_toks
    finally:
        for e in (fused, eager, batched, f32):
            e.free()


def test_engine_f16_lane_8b_shape_fused_equals_eager(hv):
    """The 8B geometry (GQA group 4, 36 layers): the fused f16 step and the eager f16
    kernel sequence give bit-identical logits after a short prompt."""
    arch = synth.ARCH["qwen3-8b"]
    a = make_engine(arch, 2, 32, kv_dtype="f16")
    try:
        prompt = synth.prompt_ids(a.cfg, 2, 6)
        la = a.logits(prompt)
        a.fused = False
        lb = a.logits(prompt)
        assert np.array_equal(bits(la), bits(lb))
    finally:
        a.free()
