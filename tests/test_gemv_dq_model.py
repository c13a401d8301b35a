"""A lane-level model of the dp4a GEMV over the dq tile layout (hv_w4_prepack_dq and
k_a4gv_dq / gemv_tile8_dq in gemv_mma.cuh), run on the CPU.

The dq arrays are built by a host restatement of k_w4_prepack_dq. Each lane then reads them
with the kernel's own index expressions: words of block 2t at 4L, of block 2t+1 at
128 + 4L, scales at 2L, activations as 32-byte blocks. It forms each block dot the way
block_dot does (byte lanes of lop3 and dp4a.u32.s32: (q + 8) nibbles times signed
activations, high nibbles scaled by 16, minus 8 x the block sum). The combine,
accumulators, quad fold, tail and postfix stack follow gemv_tile8_dq. Every output must
equal the oracle's gemv_w4 bit for bit, and every block dot the oracle's exact int32 dot.
The GPU test then compares the kernel itself with hv_a4gv_pp."""
import numpy as np
import pytest

import hv_oracle as O
from test_prefill_gemm_model import plan_of, pp_row, prepack

F32 = np.float32
NIB_WORDS, SCALES = 256, 64


def ntiles(rows, pair):
    return (pair + 3) // 4 if pair else (rows + 7) // 8


def prepack_dq(packed, scale, rows, k, pair):
    """k_w4_prepack_dq: per tile and 8-block iteration, lane L = 4g + t stores words 0..3 of
    block 2t of row g at 4L and of block 2t+1 at 128 + 4L, their scales at 2L, 2L + 1;
    blocks past nb are zero."""
    nb = k // 32
    niter, ntile = (nb + 7) // 8, ntiles(rows, pair)
    pb = np.zeros((ntile, niter, NIB_WORDS), np.uint32)
    ps = np.zeros((ntile, niter, SCALES), F32)
    w = packed.reshape(rows, nb, 4)
    for tile in range(ntile):
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            row, ok = pp_row(tile, g, rows, pair)
            if not ok:
                continue
            for it in range(niter):
                for h in (0, 1):
                    b = it * 8 + 2 * t + h
                    if b < nb:
                        pb[tile, it, h * 128 + 4 * lane:h * 128 + 4 * lane + 4] = w[row, b]
                        ps[tile, it, 2 * lane + h] = scale[row, b]
    return pb, ps


def dp4a_us(a_words, b_words):
    """dp4a.u32.s32 summed: per 32-bit word, unsigned bytes of a times signed bytes of b."""
    ua = a_words.astype(np.uint32).view(np.uint8).astype(np.int64)
    sb = b_words.astype(np.uint32).view(np.int8).astype(np.int64)
    return ua.reshape(-1, 4).__mul__(sb.reshape(-1, 4)).sum(1)


def block_dot(words, acts, bsum):
    """block_dot(nib, a0, a1, bsum) of hv_common.cuh for one block: words [4] u32 in the
    reference packing, acts [32] int8, bsum their sum."""
    w = words.astype(np.uint32)
    a = np.ascontiguousarray(acts, np.int8).view(np.uint32)     # a0.x .. a1.w
    lo_w = (w & np.uint32(0x0F0F0F0F)) ^ np.uint32(0x08080808)  # lop_lo
    hi_w = (w & np.uint32(0xF0F0F0F0)) ^ np.uint32(0x80808080)  # lop_hi
    lo = int(dp4a_us(lo_w, a[0::2]).sum())     # word i low nibbles x activation word 2i
    hi = int(dp4a_us(hi_w, a[1::2]).sum())     # word i high nibbles x activation word 2i+1
    assert hi % 16 == 0
    return lo + (hi >> 4) - 8 * bsum


def gemv_dq_model(pb, ps, q8, s_a, bsum, rows, k, pair, idot_out=None):
    """gemv_tile8_dq for every tile and lane; returns y [rows] (reference row order)."""
    nb = k // 32
    nfull, ntail = nb // 8, nb % 8
    it_end, pops = plan_of(nb)
    nleaf = len(it_end)
    y = np.zeros(rows, F32)
    acts = q8.reshape(nb, 32)

    def terms(tile, lane, it, nvalid):
        t = lane & 3
        out = []
        for h in (0, 1):
            b = it * 8 + 2 * t + h
            if 2 * t + h >= nvalid:
                out.append(F32(0.0))
                continue
            words = pb[tile, it, h * 128 + 4 * lane:h * 128 + 4 * lane + 4]
            s_w = ps[tile, it, 2 * lane + h]
            d = block_dot(words, acts[b], int(bsum[b]))
            if idot_out is not None:
                idot_out[(tile, lane >> 2, b)] = d
            out.append(F32(F32(s_w * s_a[b]) * F32(d)))
        return out

    for tile in range(ntiles(rows, pair)):
        # per lane: accumulators of blocks 2t (e) and 2t+1 (o), leaf by leaf
        acc = np.zeros((32, 2), F32)
        stacks = [[] for _ in range(32)]
        leaf, leaf_begin = 0, 0

        def fold_quad():
            v = (acc[:, 0] + acc[:, 1]).astype(F32)
            v = (v + v[np.arange(32) ^ 1]).astype(F32)
            v = (v + v[np.arange(32) ^ 2]).astype(F32)
            return v

        def push(v, leaf):
            for lane in range(32):
                stacks[lane].append(F32(v[lane]))
                for _ in range(pops[leaf]):
                    b_, a_ = stacks[lane].pop(), stacks[lane].pop()
                    stacks[lane].append(F32(a_ + b_))

        for it in range(nfull):
            for lane in range(32):
                ce, co = terms(tile, lane, it, 8)
                if it == leaf_begin:
                    acc[lane] = (ce, co)
                else:
                    acc[lane] = (F32(acc[lane, 0] + ce), F32(acc[lane, 1] + co))
            if it + 1 == it_end[leaf] and leaf + 1 < nleaf:
                push(fold_quad(), leaf)
                leaf += 1
                leaf_begin = it_end[leaf - 1]
        v = fold_quad() if nfull > leaf_begin else np.zeros(32, F32)
        if ntail:
            c = [terms(tile, lane, nfull, ntail) for lane in range(32)]
            for lane in range(32):
                q = lane & ~3
                for j in range(ntail):
                    v[lane] = F32(v[lane] + c[q | (j >> 1)][j & 1])
        push(v, nleaf - 1)
        for lane in range(0, 32, 4):                        # lane t == 0 stores row g
            row, ok = pp_row(tile, lane >> 2, rows, pair)
            if ok:
                y[row] = F32(F32(0.0) + stacks[lane][0])
    return y


CASES = [(24, 512, 0), (20, 800, 0), (24, 256, 12), (16, 5120, 0), (8, 12288, 0),
         (13, 2080, 0)]


@pytest.mark.parametrize("rows,k,pair", CASES)
def test_dq_model_matches_oracle(rows, k, pair):
    """K = 800 and 2080 have tail blocks (nb % 8 = 1, 1); 5120 and 12288 several leaves;
    pair > 0 is a gate/up matrix."""
    g = np.random.default_rng(rows * 7 + k)
    packed, scale = O.quantize_w4((g.standard_normal((rows, k)) * 0.02).astype(F32))
    x = (g.standard_normal(k) * 2).astype(F32)
    q8, s_a, bsum = O.quantize_act(x)
    pb, ps = prepack_dq(packed, scale, rows, k, pair)
    idots = {}
    got = gemv_dq_model(pb, ps, q8, s_a, bsum, rows, k, pair, idots)
    idot_ref, want = O.gemv_q(q8, s_a, packed, scale, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    n_real = 0
    for (tile, gq, b), d in idots.items():
        row, ok = pp_row(tile, gq, rows, pair)
        if ok:
            assert d == idot_ref[row, b], (tile, gq, b)
            n_real += 1
        else:                                 # a padding row of the last tile: zero words
            assert d == 0, (tile, gq, b)
    assert n_real == rows * (k // 32)         # every block of every row, once


@pytest.mark.parametrize("rows,k,pair", [(24, 512, 0), (24, 256, 12), (16, 2048, 0)])
def test_dq_is_a_rearrangement_of_pp(rows, k, pair):
    """The dq arrays hold exactly the pp arrays' words per (tile, iteration), rearranged,
    and the same scales in the same places."""
    g = np.random.default_rng(k + pair)
    packed, scale = O.quantize_w4((g.standard_normal((rows, k)) * 0.02).astype(F32))
    pb_dq, ps_dq = prepack_dq(packed, scale, rows, k, pair)
    pb_pp, ps_pp = prepack(packed, scale, rows, k, pair)
    pb_pp = pb_pp.reshape(pb_dq.shape)
    assert np.array_equal(ps_dq.reshape(-1), ps_pp)
    assert np.array_equal(np.sort(pb_dq, axis=2), np.sort(pb_pp, axis=2))
    # and the addressing itself: pp word t of block j at (j >= 4) * 128 + 4L + (j & 3)
    # for lane L = 4g + t; dq word w of block j at (j & 1) * 128 + 4 (4g + j // 2) + w
    for gq in range(8):
        for j in range(8):
            for w in range(4):
                pp_off = (j >= 4) * 128 + 4 * (4 * gq + w) + (j & 3)
                dq_off = (j & 1) * 128 + 4 * (4 * gq + j // 2) + w
                assert np.array_equal(pb_pp[:, :, pp_off], pb_dq[:, :, dq_off])
