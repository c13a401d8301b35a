"""The dp4a GEMV over the dq tile layout on a B200 (hv_w4_prepack_dq + hv_a4gv_dq):
bit-identical to hv_a4gv_pp (one warp per tile, tensor-pipe block dots) and to the
oracle, for plain and gate/up-paired matrices, tails (nb % 8 != 0), multi-leaf K and the
vocabulary-sized shapes of the GEMV sweep; the dq arrays are a rearrangement of the
tile-interleaved ones (the lane-level CPU model checks the arithmetic,
tests/test_gemv_dq_model.py). An engine with dq tiles (fused step and eager sequence)
gives the pp engine's logits bit for bit."""
import numpy as np
import pytest

import hv_oracle as O
from gpu_util import Dev, bits, quantize_on_device

pytestmark = pytest.mark.gpu
F32 = np.float32


@pytest.mark.parametrize("n,k,pair", [(5, 32, 0), (13, 416, 0), (777, 4096, 0), (64, 12288, 0),
                                      (21, 25600, 0), (26, 2048, 13), (24576, 4096, 12288),
                                      (10, 160, 5), (20, 800, 0), (12288, 4096, 0)])
def test_gemv_dq_equals_pp_and_oracle(hv, n, k, pair):
    g = np.random.default_rng(n * 13 + k)
    p, sc = O.quantize_w4((g.standard_normal((n, k)) * 0.02).astype(F32))
    nib, scb = hv.w4_prepacked_size(n, k, pair)
    b4, sw = Dev(p), Dev(sc)
    pp = (Dev(nbytes=nib), Dev(nbytes=scb))
    dq = (Dev(nbytes=nib), Dev(nbytes=scb))
    hv.w4_prepack(b4, sw, n, k, pair, *pp)
    hv.w4_prepack_dq(b4, sw, n, k, pair, *dq)
    # the same words per (tile, iteration), the same scales
    per = 256
    wp, wd = pp[0].get(np.uint32).reshape(-1, per), dq[0].get(np.uint32).reshape(-1, per)
    assert np.array_equal(np.sort(wp, axis=1), np.sort(wd, axis=1))
    assert np.array_equal(bits(pp[1].get(F32)), bits(dq[1].get(F32)))
    a = (g.standard_normal(k) * 2).astype(F32)
    a[:32] = 0.0                                       # an all-zero activation block
    qa, sa_h, _ = O.quantize_act(a)
    _, want = O.gemv_q_c(qa, sa_h, p, sc, k)
    a8, sa = quantize_on_device(a)
    y_pp, y_dq = Dev(nbytes=n * 4), Dev(nbytes=n * 4)
    hv.a4gv_pp(a8, sa, *pp, y_pp, k // 8, n, pair)
    hv.a4gv_dq(a8, sa, *dq, y_dq, k // 8, n, pair)
    assert np.array_equal(bits(y_dq.get(F32)), bits(y_pp.get(F32)))
    assert np.array_equal(bits(y_dq.get(F32)), bits(want))


def test_gemv_dq_rejects_bad_arguments(hv):
    with pytest.raises(hv.CudaError):
        hv.a4gv_dq(16, 16, 16, 16, 16, 3, 8)           # K = 24: not a multiple of 32
    with pytest.raises(hv.CudaError):
        hv.w4_prepack_dq(16, 16, 10, 64, 4, 16, 16)    # a pair needs rows == 2 * pair


def _engine(arch, seed, cap, **kw):
    import limited
    import synth
    import w4format
    cfg = w4format.Config(arch)
    return limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, seed), quiet=True,
                          max_context=cap, **kw)


@pytest.mark.parametrize("fused", [True, False])
def test_engine_dq_tiles_bit_identical_to_pp(hv, fused):
    """The fused step (k_step over dq slots) and the eager sequence (hv_a4gv_dq) give the
    pp engine's logits bit for bit, and the same greedy tokens."""
    import synth
    arch = synth.tiny_arch(n_layer=3, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096)
    a = _engine(arch, 21, 64, fused=fused)
    b = _engine(arch, 21, 64, fused=fused, gemv_layout="dq")
    try:
        prompt = synth.prompt_ids(a.cfg, 21, 9)
        for n in (1, 5, 9):
            assert np.array_equal(bits(a.logits(prompt[:n])), bits(b.logits(prompt[:n]))), n
        assert a.generate(prompt, 12)[0] == b.generate(prompt, 12)[0]
    finally:
        a.free()
        b.free()


def test_engine_dq_tiles_8b_shape(hv):
    """The 8B geometry (K = 4096 and 12288: one and four pairwise leaves per row)."""
    import synth
    arch = synth.ARCH["qwen3-8b"]
    a = _engine(arch, 2, 16)
    try:
        prompt = synth.prompt_ids(a.cfg, 2, 4)
        la = a.logits(prompt)
    finally:
        a.free()
    b = _engine(arch, 2, 16, gemv_layout="dq")
    try:
        assert np.array_equal(bits(la), bits(b.logits(prompt)))
    finally:
        b.free()


@pytest.mark.parametrize("rows,k,pair,ntok", [(24, 512, 0, 11), (2048, 6144, 0, 37),
                                              (2 * 1536, 4096, 1536, 40)])
def test_prefill_gemm_dq_equals_pp(hv, rows, k, pair, ntok):
    """hv_a4gemm_dq over dq tiles gives hv_a4gemm_pp's rows bit for bit."""
    g = np.random.default_rng(rows + k + ntok)
    p, sc = O.quantize_w4((g.standard_normal((rows, k)) * 0.02).astype(F32))
    nib, scb = hv.w4_prepacked_size(rows, k, pair)
    b4, sw = Dev(p), Dev(sc)
    pp = (Dev(nbytes=nib), Dev(nbytes=scb))
    dq = (Dev(nbytes=nib), Dev(nbytes=scb))
    hv.w4_prepack(b4, sw, rows, k, pair, *pp)
    hv.w4_prepack_dq(b4, sw, rows, k, pair, *dq)
    x = (g.standard_normal((ntok, k)) * 2).astype(F32)
    nb = k // 32
    xd = Dev(x)
    a8, sa = Dev(nbytes=ntok * k), Dev(nbytes=ntok * nb * 8)
    hv.qa8s_rows(xd, a8, sa, nb, ntok)
    y_pp, y_dq = Dev(nbytes=ntok * rows * 4), Dev(nbytes=ntok * rows * 4)
    hv.a4gemm_pp(a8, sa, *pp, y_pp, k // 8, rows, pair, ntok)
    hv.a4gemm_dq(a8, sa, *dq, y_dq, k // 8, rows, pair, ntok)
    assert np.array_equal(bits(y_dq.get(F32)), bits(y_pp.get(F32)))


def test_engine_dq_batched_prefill_equals_pp(hv):
    """A 300-token prompt through the batched prefill (two 256-token runs) on dq tiles
    leaves the pp engine's KV cache and logits bit for bit."""
    import synth
    arch = synth.tiny_arch(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096)
    out = []
    for layout in ("pp", "dq"):
        e = _engine(arch, 11, 320, prefill="batched", gemv_layout=layout)
        try:
            prompt = synth.prompt_ids(e.cfg, 11, 300)
            lg = e.logits(prompt)
            kv = np.empty(e.kv_bytes // 4, F32)
            hv.download(kv.ctypes.data, e.d_kv, kv.nbytes)
            out.append((lg, kv))
        finally:
            e.free()
    assert np.array_equal(bits(out[0][0]), bits(out[1][0]))
    assert np.array_equal(bits(out[0][1]), bits(out[1][1]))


def test_engine_dq_tiles_with_binary16_cache(hv):
    """dq tiles with the binary16 KV cache (k_step<GS, false, __half, true>): the pp
    engine's logits with that cache, bit for bit."""
    import synth
    arch = synth.tiny_arch(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096)
    a = _engine(arch, 23, 64, kv_dtype="f16")
    b = _engine(arch, 23, 64, kv_dtype="f16", gemv_layout="dq")
    try:
        prompt = synth.prompt_ids(a.cfg, 23, 12)
        assert np.array_equal(bits(a.logits(prompt)), bits(b.logits(prompt)))
    finally:
        a.free()
        b.free()
