"""LM-head GEMV + greedy argmax over a vocabulary split into shards: the 151936 x 5120
head workload (int4 weights with an f32 scale per 32, drawn N(0,0.02) from seed 4) and
10,000 N(0,1) hidden states quantised per 32 by quant_a8s.

The reference samples with np.argmax over the full logits (engine/reference.py:219, the
first maximal id). Here the vocabulary is split into G = 1, 2, 4, 8 shards of 151936/G
rows, the split the sharded engine gives the LM head across G GPUs: each shard's GEMV
writes its rows, hv_argmax_key folds them into that shard's key, and hv_argmax_key_final
reduces the G keys (what the ranks exchange) into the token.

Checks:
* the logits are bit-identical to the C oracle's gemv_w4 on a sample of states (the
  GEMV's bits are pinned to the reference on the sweep shapes), and identical for every
  shard count;
* every one of the 10,000 tokens, for every G, equals np.argmax of the logits;
* equal maxima in different shards go to the lowest id; -0 equals +0; NaN wins first.
"""
import numpy as np
import pytest

import hv_oracle as O
import synth
from gpu_util import Dev, bits

pytestmark = pytest.mark.gpu
F32 = np.float32
N_STATES = 10_000
SHARDS = (1, 2, 4, 8)
N_ORACLE = 48          # states whose logits the C oracle recomputes
N_KEEP = 64            # states whose logits are kept for every shard count


def plant_cases():
    """(name, logits) vectors with planted ties, signed zeros and NaNs."""
    n = synth.HEAD_SHAPE[0]
    g = np.random.default_rng(17)
    cases = []
    v = g.standard_normal(n).astype(F32)
    v[[100000, 37984, 151935, 18992 * 5 + 3]] = 9.0       # equal maxima in four shards
    cases.append(("tie_across_shards", v))
    v = -np.abs(g.standard_normal(n).astype(F32)) - 1.0
    v[5000], v[3000] = -0.0, 0.0                           # -0 == +0: the lower id wins
    cases.append(("signed_zero_a", v))
    v = v.copy()
    v[5000], v[3000] = 0.0, -0.0
    cases.append(("signed_zero_b", v))
    v = g.standard_normal(n).astype(F32)
    v[[140000, 70000]] = np.nan                            # np.argmax: the first NaN
    v[10] = np.inf
    cases.append(("nan_first", v))
    v = np.full(n, -np.inf, F32)
    v[n - 1] = -3.0e38
    cases.append(("all_but_one_minus_inf", v))
    return cases


def sharded_argmax(hv, logits_ptr, n, shards, keys, tok, gen, step, pos):
    rows = n // shards
    for s in range(shards):
        hv.argmax_key(logits_ptr + 4 * s * rows, rows, s * rows, keys.ptr + 8 * s)
    hv.argmax_key_final(keys, shards, tok, gen, step, pos)


@pytest.mark.parametrize("shards", SHARDS)
def test_planted_ties_zeros_and_nans(hv, shards):
    n = synth.HEAD_SHAPE[0]
    keys = Dev(nbytes=8 * shards)
    tok, step, pos = (Dev(np.zeros(1, np.int32)) for _ in range(3))
    cases = plant_cases()
    gen = Dev(nbytes=4 * len(cases))
    bufs = [Dev(v) for _, v in cases]           # alive until the kernels have run
    for d in bufs:
        sharded_argmax(hv, d.ptr, n, shards, keys, tok, gen, step, pos)
    got = gen.get(np.int32)
    for (name, v), t in zip(cases, got):
        assert t == int(np.argmax(v)), (name, shards, t, int(np.argmax(v)))
    assert step.get(np.int32)[0] == len(cases) and pos.get(np.int32)[0] == len(cases)
    assert not keys.get(np.uint64).any()             # the final reduce leaves keys at 0


@pytest.fixture(scope="module")
def head(hv):
    n, k = synth.HEAD_SHAPE
    nb = k // 32
    w, h = synth.head_case(N_STATES)
    b4, sw = Dev(nbytes=n * k // 2), Dev(nbytes=n * nb * 4)
    wd = Dev(w)
    hv.quantize_w4(wd, b4, sw, n, k)
    wd.free()
    del w
    nib, scb = hv.w4_prepacked_size(n, k, 0)
    pb4, psw = Dev(nbytes=nib), Dev(nbytes=scb)
    hv.w4_prepack(b4, sw, n, k, 0, pb4, psw)
    hd = Dev(h)
    a8, sa = Dev(nbytes=N_STATES * k), Dev(nbytes=N_STATES * nb * 8)
    for s in range(N_STATES):          # quant_a8s per state: [scale | block sum] per state
        hv.qa8s(hd.ptr + 4 * s * k, a8.ptr + s * k, sa.ptr + 8 * s * nb, nb)
    hd.free()
    hv.synchronize()
    H = dict(n=n, k=k, nb=nb, h=h, b4=b4, sw=sw, pb4=pb4, psw=psw, a8=a8, sa=sa,
             tile=hv.w4_prepacked_size(8, k, 0))
    yield H
    for d in (b4, sw, pb4, psw, a8, sa):
        d.free()


def decode_all(hv, H, shards, keep):
    """Tokens of all states with the vocabulary in `shards` shards; the logits of the
    first N_KEEP states are written into `keep` [N_KEEP, n] (or [N_STATES, n])."""
    n, k, nb = H["n"], H["k"], H["nb"]
    rows = n // shards
    nib_t, scb_t = H["tile"]
    keys = Dev(nbytes=8 * shards)
    tok, step, pos = (Dev(np.zeros(1, np.int32)) for _ in range(3))
    gen = Dev(nbytes=4 * N_STATES)
    scratch = Dev(nbytes=4 * n)
    keep_rows = keep.nbytes // (4 * n)
    for s in range(N_STATES):
        a8s, sas = H["a8"].ptr + s * k, H["sa"].ptr + 8 * s * nb
        dst = keep.ptr + 4 * s * n if s < keep_rows else scratch.ptr
        for g in range(shards):
            r0 = g * rows
            t0 = r0 // 8
            hv.a4gv_pp(a8s, sas, H["pb4"].ptr + t0 * nib_t, H["psw"].ptr + t0 * scb_t,
                       dst + 4 * r0, k // 8, rows, 0)
            hv.argmax_key(dst + 4 * r0, rows, r0, keys.ptr + 8 * g)
        hv.argmax_key_final(keys, shards, tok, gen, step, pos)
    toks = gen.get(np.int32)
    assert step.get(np.int32)[0] == N_STATES
    return toks


def test_head_argmax_10k_states_every_shard_count(hv, head):
    H = head
    n, k = H["n"], H["k"]
    # one shard: every state's logits kept for the np.argmax check (6 GB on the device)
    full = Dev(nbytes=4 * n * N_STATES)
    toks1 = decode_all(hv, H, 1, full)
    want = np.empty(N_STATES, np.int64)
    chunk = 500
    for c0 in range(0, N_STATES, chunk):
        lg = np.empty((chunk, n), F32)
        hv.synchronize()
        hv.download(lg.ctypes.data, full.ptr + 4 * c0 * n, lg.nbytes)
        want[c0:c0 + chunk] = np.argmax(lg, axis=1)
    assert np.array_equal(toks1, want), np.flatnonzero(toks1 != want)[:10]

    # the logits are the reference's gemv_w4 bit for bit (C oracle on sampled states)
    packed = H["b4"].get(np.uint32, (n, k // 8))
    scale = H["sw"].get(F32, (n, k // 32))
    a8_all = H["a8"].get(np.int8, (N_STATES, k))
    for s in np.linspace(0, N_STATES - 1, N_ORACLE).astype(int):
        qa, sa, _ = O.quantize_act(H["h"][s])
        assert np.array_equal(a8_all[s], qa)
        _, y = O.gemv_q_c(qa, sa, packed, scale, k)
        lg = np.empty(n, F32)
        hv.download(lg.ctypes.data, full.ptr + 4 * int(s) * n, lg.nbytes)
        assert np.array_equal(bits(lg), bits(y)), s
        assert toks1[s] == O.argmax(y)
    keep1 = np.empty((N_KEEP, n), F32)
    hv.download(keep1.ctypes.data, full.ptr, keep1.nbytes)
    full.free()

    # every shard count: the same logits bits and the same 10,000 tokens
    for shards in SHARDS[1:]:
        keep = Dev(nbytes=4 * n * N_KEEP)
        toks = decode_all(hv, H, shards, keep)
        assert np.array_equal(bits(keep.get(F32, (N_KEEP, n))), bits(keep1)), shards
        assert np.array_equal(toks, toks1), (shards, np.flatnonzero(toks != toks1)[:10])
        keep.free()
    print(f"head argmax: {N_STATES} states, shards {SHARDS}: tokens identical to np.argmax; "
          f"{len(set(toks1.tolist()))} distinct tokens")
