"""The prefill GEMM (hv_a4gemm_pp) on a B200: every token's output row is bit-identical to
hv_a4gv_pp on that token alone, and to the oracle's gemv_w4, for plain and gate/up-paired
matrices, partial token groups and multi-leaf K."""
import numpy as np
import pytest

import hv_oracle as O
from gpu_util import Dev, bits

pytestmark = pytest.mark.gpu
F32 = np.float32


def quantize_rows(hv, x):
    """quant_a8s per token: a8 [T][K], sa [T][2 K/32] (scales, then block sums)."""
    t, k = x.shape
    nb = k // 32
    xd = Dev(x)
    a8, sa = Dev(nbytes=t * k), Dev(nbytes=t * nb * 8)
    for n in range(t):
        hv.qa8s(xd.ptr + 4 * n * k, a8.ptr + n * k, sa.ptr + 8 * n * nb, nb)
    return a8, sa


@pytest.mark.parametrize("rows,k,pair,ntok", [(24, 512, 0, 11), (24, 256, 12, 8),
                                              (2048, 6144, 0, 37), (6144, 4096, 0, 64),
                                              (2 * 1536, 4096, 1536, 40), (100, 12288, 0, 5)])
def test_prefill_gemm_rows_equal_per_token_gemv(hv, rows, k, pair, ntok):
    g = np.random.default_rng(rows + k + ntok)
    packed, scale = O.quantize_w4((g.standard_normal((rows, k)) * 0.02).astype(F32))
    nib, scb = hv.w4_prepacked_size(rows, k, pair)
    pb4, psw = Dev(nbytes=nib), Dev(nbytes=scb)
    hv.w4_prepack(Dev(packed), Dev(scale), rows, k, pair, pb4, psw)
    x = (g.standard_normal((ntok, k)) * 2).astype(F32)
    a8, sa = quantize_rows(hv, x)
    y = Dev(nbytes=ntok * rows * 4)
    hv.a4gemm_pp(a8, sa, pb4, psw, y, k // 8, rows, pair, ntok)
    got = y.get(F32, (ntok, rows))
    one = Dev(nbytes=rows * 4)
    nb = k // 32
    for n in range(ntok):
        hv.a4gv_pp(a8.ptr + n * k, sa.ptr + 8 * n * nb, pb4, psw, one, k // 8, rows, pair)
        assert np.array_equal(bits(got[n]), bits(one.get(F32))), n
    for n in (0, ntok - 1):
        q, s, _ = O.quantize_act(x[n])
        _, want = O.gemv_q_c(q, s, packed, scale, k)
        assert np.array_equal(bits(got[n]), bits(want)), n


TINY = dict(n_layer=2, hidden=512, ffn=1024, n_head=8, n_kv=2, vocab=4096)


@pytest.mark.parametrize("fused", [False, True])
def test_batched_prefill_equals_token_by_token(hv, fused):
    """A 300-token prompt (two runs of the 256-token batch) prefilled in batches leaves the
    same KV cache and last-token logits as the token-by-token prefill, and greedy decoding
    from it gives the same tokens."""
    import limited
    import synth
    from w4format import Config
    cfg = Config(synth.tiny_arch(**TINY))
    prompt = synth.prompt_ids(cfg, 11, 300)
    out = {}
    for mode in ("steps", "batched"):
        eng = limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, 11), quiet=True,
                             max_context=512, fused=fused, prefill=mode)
        try:
            lg = eng.logits(prompt)
            kv = np.empty(eng.kv_bytes // 4, F32)
            hv.download(kv.ctypes.data, eng.d_kv, kv.nbytes)
            toks, _, _ = eng.generate(prompt, max_new=8)
            out[mode] = (lg, kv[kv != 0].copy(), toks)
        finally:
            eng.free()
    (lg0, kv0, t0), (lg1, kv1, t1) = out["steps"], out["batched"]
    assert np.array_equal(bits(kv0), bits(kv1))
    assert np.array_equal(bits(lg0), bits(lg1))
    assert t0 == t1


GOLDEN_TINY = [("decode_tiny.npz", dict(), 7),
               ("decode_tiny_tied.npz", dict(n_layer=3, hidden=512, ffn=1024, n_head=8, n_kv=2,
                                             vocab=2048, tied=True), 8),
               # several prefill batches, and decode attention over many positions per chunk
               ("decode_tiny_long.npz", dict(), 9),
               ("decode_tiny_2k.npz", dict(), 10)]


@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("name,arch,seed", GOLDEN_TINY)
def test_batched_prefill_matches_reference_decode(hv, golden, name, arch, seed, fused):
    """The reference's own greedy decode of the tiny models (tests/golden, made by
    engine/reference.py): with the batched prefill the tokens are the same and the
    step-0 logits bit-identical."""
    import limited
    import synth
    from w4format import Config
    g = golden(name)
    prompt, want = g["prompt"].tolist(), g["tokens"].tolist()
    cfg = Config(synth.tiny_arch(**arch))
    eng = limited.Engine(config=cfg, tensors=synth.iter_tensors(cfg, seed), quiet=True,
                         max_context=len(prompt) + len(want) + 2, fused=fused,
                         prefill="batched")
    try:
        toks, _, _ = eng.generate(prompt, max_new=len(want))
        assert toks == want
        lg = eng.logits(prompt)
        ref = g["logits"][0]
        err = float(np.abs(lg.astype(np.float64) - ref).max() / np.abs(ref).max())
        assert np.array_equal(lg.view(np.uint32), ref.astype(np.float32).view(np.uint32)), err
    finally:
        eng.free()
