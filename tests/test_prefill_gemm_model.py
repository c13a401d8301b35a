"""A lane-level model of k_a4gemm_pp (the prefill GEMM in k_prefill.cu), run on the CPU.

Every lane's loads use the kernel's own index expressions: into the tile-interleaved
weights (built here by a host restatement of hv_w4_prepack's reordering), the per-token
int8 activations and their (scale, block sum) rows. The mma.sync m16n8k32 fragments are
assembled per the PTX fragment layout for 8-bit operands:
  A: a0 = row g, k 4t..4t+3; a1 = row g+8, same k; a2 = row g, k 16+4t..; a3 = row g+8;
  B: b0 = k 4t..4t+3 of column g; b1 = k 16+4t..16+4t+3 of column g;
  D: d0 = (g, 2t), d1 = (g, 2t+1), d2 = (g+8, 2t), d3 = (g+8, 2t+1).
The combine, the per-leaf accumulators, the fold and the postfix stack follow the kernel.
Every token's output must equal the oracle's gemv_w4 bit for bit, so the kernel's
indexing is checked without a GPU; the GPU test compares the kernel itself."""
import numpy as np
import pytest

import hv_oracle as O

F32 = np.float32
NIB_WORDS, SCALES = 256, 64


def plan_of(nb):
    """numpy's pairwise recursion as (it_end, pops) per leaf (gv_make_plan's contract),
    restated from the oracle's leaf plan."""
    leaves = O.pairwise_plan(nb)            # [(start, size)] in order
    it_end = [(s + m) // 8 for s, m in leaves]
    # pops: after leaf i, the number of '+' that close (postfix): recompute from the tree
    pops = [0] * len(leaves)

    def rec(s, m):
        if m <= 128:
            return [(s, m)]
        m2 = m // 2
        m2 -= m2 % 8
        left, right = rec(s, m2), rec(s + m2, m - m2)
        return left + right + ["+"]
    seq, n = rec(0, nb), 0
    for x in seq:
        if x == "+":
            pops[n - 1] += 1
        else:
            n += 1
    assert [(s, m) for s, m in (x for x in seq if x != "+")] == leaves
    return it_end, pops


def pp_row(tile, g, rows, pair):
    if pair > 0:
        p = tile * 4 + (g & 3)
        return (p if g < 4 else pair + p), p < pair
    row = tile * 8 + g
    return row, row < rows


def prepack(packed, scale, rows, k, pair):
    """hv_w4_prepack's layout: per tile and 8-block iteration, lane L = 4g + t stores word
    t of blocks 0..3 at 4L, of blocks 4..7 at 128 + 4L, and row g's scales of blocks 2t,
    2t+1 at 2L."""
    nb = k // 32
    niter = (nb + 7) // 8
    ntile = (pair + 3) // 4 if pair else (rows + 7) // 8
    pb4 = np.zeros((ntile, niter, NIB_WORDS), np.uint32)
    psw = np.zeros((ntile, niter, SCALES), F32)
    w = packed.reshape(rows, nb, 4)
    for tile in range(ntile):
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            row, ok = pp_row(tile, g, rows, pair)
            if not ok:
                continue
            for it in range(niter):
                for j in range(8):
                    off = 4 * lane + j if j < 4 else 128 + 4 * lane + j - 4
                    pb4[tile, it, off] = w[row, it * 8 + j, t]
                psw[tile, it, 2 * lane] = scale[row, it * 8 + 2 * t]
                psw[tile, it, 2 * lane + 1] = scale[row, it * 8 + 2 * t + 1]
    return pb4.reshape(-1), psw.reshape(-1)


def nib(w, hi):
    w = (w >> 4) if hi else w
    return ((w & 0x0F0F0F0F) ^ 0x08080808).astype(np.uint32)


def bytes_u8(words):          # [..] u32 -> [.., 4] u8 (little endian)
    return np.ascontiguousarray(words, np.uint32).view(np.uint8).reshape(*np.shape(words), 4)


def bytes_s8(words):
    return np.ascontiguousarray(words, np.uint32).view(np.int8).reshape(*np.shape(words), 4)


def model_gemm(a8, sa, pb4, psw, rows, k, pair, ntok, layout="pp"):
    """What k_a4gemm_pp computes, lane by lane: y [ntok, rows]. layout "dq": the weights
    are in the dq arrangement and each lane loads word t of block j of row g from
    (j & 1) * 128 + 4 (4 g + j // 2) + t (k_a4gemm_pp<true>)."""
    nb, niter = k // 32, k // 256
    it_end, pops = plan_of(nb)
    ntile = (pair + 3) // 4 if pair else (rows + 7) // 8
    y = np.full((ntok, rows), np.nan, F32)
    a8w = a8.reshape(-1).view(np.uint8)
    lanes = np.arange(32)
    g, t = lanes >> 2, lanes & 3
    for bx in range((ntile + 3) // 4):
        for by in range((ntok + 31) // 32):
            for warp in range(8):
                tile_a = 2 * (bx * 2 + (warp & 1))
                tq = by * 4 + (warp >> 1)
                if tile_a >= ntile or tq * 8 >= ntok:
                    continue
                has_b = tile_a + 1 < ntile
                tile_b = tile_a + 1 if has_b else tile_a
                tok_col = np.minimum(tq * 8 + g, ntok - 1)
                n0, n1 = tq * 8 + 2 * t, tq * 8 + 2 * t + 1
                sa0 = np.minimum(n0, ntok - 1) * 2 * nb
                sa1 = np.minimum(n1, ntok - 1) * 2 * nb
                lane_off = 4 * lanes if layout == "pp" else 16 * g + t
                wa = tile_a * niter * NIB_WORDS + lane_off
                wb = tile_b * niter * NIB_WORDS + lane_off
                if layout == "pp":
                    woff = [j if j < 4 else 128 + j - 4 for j in range(8)]
                else:
                    woff = [(j & 1) * 128 + 4 * (j >> 1) for j in range(8)]
                sca = tile_a * niter * SCALES + 8 * g
                scb = tile_b * niter * SCALES + 8 * g
                act = tok_col * k + 8 * t
                r = np.zeros((4, 8, 32), F32)
                st, leaf, leaf_begin = [], 0, 0
                for it in range(niter):
                    wo, so = it * NIB_WORDS, it * SCALES
                    wA = np.stack([pb4[wa + wo + woff[j]] for j in range(8)])
                    wB = np.stack([pb4[wb + wo + woff[j]] for j in range(8)])
                    swA = np.stack([psw[sca + so + j] for j in range(8)])
                    swB = np.stack([psw[scb + so + j] for j in range(8)])
                    s0 = np.stack([sa[sa0 + 8 * it + j] for j in range(8)])
                    s1 = np.stack([sa[sa1 + 8 * it + j] for j in range(8)])
                    q0 = np.stack([sa[sa0 + nb + 8 * it + j] for j in range(8)]).view(np.int32)
                    q1 = np.stack([sa[sa1 + nb + 8 * it + j] for j in range(8)]).view(np.int32)
                    first = it == leaf_begin
                    for j in range(8):
                        base = act + (it * 8 + j) * 32
                        bw = np.stack([a8w[base + i] for i in range(8)], 1)     # [32 lanes, 8]
                        A = np.zeros((16, 32), np.int64)
                        B = np.zeros((32, 8), np.int64)
                        lo_a, hi_a = bytes_u8(nib(wA[j], 0)), bytes_u8(nib(wA[j], 1))
                        lo_b, hi_b = bytes_u8(nib(wB[j], 0)), bytes_u8(nib(wB[j], 1))
                        bs = bw.view(np.int8)
                        for L in range(32):
                            gg, tt = L >> 2, L & 3
                            A[gg, 4 * tt:4 * tt + 4] = lo_a[L]          # a0
                            A[gg + 8, 4 * tt:4 * tt + 4] = lo_b[L]      # a1
                            A[gg, 16 + 4 * tt:20 + 4 * tt] = hi_a[L]    # a2
                            A[gg + 8, 16 + 4 * tt:20 + 4 * tt] = hi_b[L]  # a3
                            B[4 * tt:4 * tt + 4, gg] = bs[L, 0:4]      # b0
                            B[16 + 4 * tt:20 + 4 * tt, gg] = bs[L, 4:8]  # b1
                        D = A @ B
                        d = np.stack([D[g, 2 * t], D[g, 2 * t + 1], D[g + 8, 2 * t],
                                      D[g + 8, 2 * t + 1]])
                        sw = np.stack([swA[j], swA[j], swB[j], swB[j]])
                        sx = np.stack([s0[j], s1[j], s0[j], s1[j]])
                        qx = np.stack([q0[j], q1[j], q0[j], q1[j]])
                        c = (sw * sx).astype(F32) * (d - 8 * qx).astype(F32)
                        r[:, j] = c if first else (r[:, j] + c).astype(F32)
                    if it + 1 == it_end[leaf]:
                        v = (((r[:, 0] + r[:, 1]) + (r[:, 2] + r[:, 3]))
                             + ((r[:, 4] + r[:, 5]) + (r[:, 6] + r[:, 7])))
                        st.append(v.astype(F32))
                        for _ in range(pops[leaf]):
                            b_ = st.pop()
                            st[-1] = (st[-1] + b_).astype(F32)
                        leaf += 1
                        leaf_begin = it + 1
                out = (F32(0.0) + st[0]).astype(F32)                  # [4, 32]
                for L in range(32):
                    gg = L >> 2
                    row_a, ok_a = pp_row(tile_a, gg, rows, pair)
                    row_b, ok_b = pp_row(tile_b, gg, rows, pair)
                    ok_b = ok_b and has_b
                    for p, (row, ok, n) in enumerate([(row_a, ok_a, n0[L]), (row_a, ok_a, n1[L]),
                                                      (row_b, ok_b, n0[L]),
                                                      (row_b, ok_b, n1[L])]):
                        if ok and n < ntok:
                            y[n, row] = out[p, L]
    return y


@pytest.mark.parametrize("layout", ["pp", "dq"])
@pytest.mark.parametrize("rows,k,pair,ntok", [(24, 512, 0, 11), (24, 256, 12, 8),
                                              (16, 6144, 0, 3), (40, 1024, 20, 33)])
def test_model_of_prefill_gemm_matches_oracle_per_token(rows, k, pair, ntok, layout):
    g = np.random.default_rng(rows * 7 + k + ntok)
    packed, scale = O.quantize_w4((g.standard_normal((rows, k)) * 0.02).astype(F32))
    if layout == "pp":
        pb4, psw = prepack(packed, scale, rows, k, pair)
    else:
        from test_gemv_dq_model import prepack_dq
        pb4, psw = (x.reshape(-1) for x in prepack_dq(packed, scale, rows, k, pair))
    x = (g.standard_normal((ntok, k)) * 2).astype(F32)
    a8 = np.zeros((ntok, k), np.int8)
    sa = np.zeros((ntok, 2 * (k // 32)), F32)
    for n in range(ntok):
        q, s, b = O.quantize_act(x[n])
        a8[n], sa[n, :k // 32], sa[n, k // 32:] = q, s, b.view(F32)
    y = model_gemm(a8, sa.reshape(-1), pb4, psw, rows, k, pair, ntok, layout)
    for n in range(ntok):
        q, s, _ = O.quantize_act(x[n])
        _, want = O.gemv_q(q, s, packed, scale, k)
        assert np.array_equal(y[n].view(np.uint32), want.view(np.uint32)), n
