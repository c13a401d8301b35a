// W4A8 GEMV on the tensor pipe: exact int32 block dots by mma.sync (u8 x s8 -> s32),
// fp32 combine in numpy's pairwise order. Shared by the standalone GEMV kernel and the
// fused step.
//
// Why not dp4a: on sm_100 dp4a (and I2F) issue to the XU pipe, which saturated at ~3.4
// TB/s of weights (ncu: XU 79% busy, issue 27%). One m16n8k32 MMA computes 16 exact
// block dots, so the dot products cost ~16x fewer issue slots and leave XU idle;
// int -> float uses the exact 2^23 magic-number trick instead of I2F.
//
// Fragment mapping (lane = 4 g + t, g = lane / 4, t = lane % 4), 8 weight rows per tile:
//   * k is permuted identically in A and B (an MMA's sum over k does not depend on the
//     order): mma-k 4t+i holds logical element 8t+i and mma-k 16+4t+i holds 8t+4+i. Lane
//     t's A registers are then the low and high nibbles of packed word t of a block
//     (reference layout, unchanged): (w & 0x0F0F0F0F) ^ 0x08080808 = q + 8 per byte.
//   * A rows 0..7 are the tile's 8 weight rows at block 8i + j, A rows 8..15 the SAME
//     rows at block 8i + j + 4, for MMA j = 0..3 of iteration i.
//   * B (32 x 8, s8): column n = activation block 8i + n; lane (g, t) holds activation
//     words 2t and 2t+1 of block 8i + g (one 64-bit shared load).
//   * MMA j leaves row g's dot for block 8i+j in column j and for block 8i+j+4 in column
//     j+4. Lane (g, t) keeps blocks 8i+2t and 8i+2t+1 of row g: it owns numpy's pairwise
//     accumulators 2t and 2t+1, walks them in order, and the leaf fold
//     ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) is an in-lane add and two xor-shuffles over t
//     -- numpy's tree, bit for bit.
//   * D = sum (q+8) a = idot + 8 * bsum; the block sum quant_a8s stores removes the bias.
#pragma once

#include "gemv_w4a8.cuh"

namespace hv {

HV_DEV void mma_u8s8(unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0,
                     unsigned b1, int& d0, int& d1, int& d2, int& d3) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

HV_DEV unsigned nib_lo(unsigned w) { return lop_lo(w); }
HV_DEV unsigned nib_hi(unsigned w) { return lop_lo(w >> 4); }

// exact float of an integer |x| < 2^22 without I2F
HV_DEV float i2f_exact(int x) {
  return __fsub_rn(__int_as_float(0x4B400000 + x), 12582912.0f);
}

HV_DEV unsigned ldg_u32(const uint32_t* p) {
  unsigned v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
HV_DEV float ldg_f1(const float* p) {
  float v;
  asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// One iteration's loads for a lane: word t of the 8 blocks of its row, and the row's
// scales of blocks 2t, 2t+1.
struct MmaLoads {
  unsigned w[8];
  float2 s;
};

// Reference layout (row-major packed words and scales): 8 scattered 4-byte loads.
HV_DEV void mma_load(MmaLoads& L, const uint32_t* r, const float* sr, int it, int t) {
#pragma unroll
  for (int j = 0; j < 8; ++j) L.w[j] = ldg_u32(r + (it * 8 + j) * 4 + t);
  // two scalar loads: a row's scales start at row * nb floats, only 4-byte aligned
  L.s = make_float2(ldg_f1(sr + it * 8 + 2 * t), ldg_f1(sr + it * 8 + 2 * t + 1));
}

HV_DEV uint4 ldg_stream128(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
HV_DEV float2 ldg_stream_f2(const float* p) {
  float2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "l"(p));
  return v;
}

// Tile-interleaved layout (hv_w4_prepack): per 8-row tile and 8-block iteration, 256
// words of nibbles where lane L = 4g + t finds word t of blocks 0..3 at 4L and of blocks
// 4..7 at 128 + 4L, then 64 floats of scales with lane L's pair at 2L. Every warp-wide
// load reads 512 (or 256) contiguous bytes.
constexpr int kPpNibWords = 256;   // per tile and iteration
constexpr int kPpScales = 64;

HV_DEV void mma_load_pp(MmaLoads& L, const uint32_t* tn, const float* ts, int it, int lane) {
  const uint4 a = ldg_stream128(tn + (size_t)it * kPpNibWords + 4 * lane);
  const uint4 b = ldg_stream128(tn + (size_t)it * kPpNibWords + 128 + 4 * lane);
  L.w[0] = a.x; L.w[1] = a.y; L.w[2] = a.z; L.w[3] = a.w;
  L.w[4] = b.x; L.w[5] = b.y; L.w[6] = b.z; L.w[7] = b.w;
  L.s = ldg_stream_f2(ts + (size_t)it * kPpScales + 2 * lane);
}

// Fold lane t's two accumulators with the other three lanes of its quad:
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)).
HV_DEV float quad_fold(float r_even, float r_odd) {
  float v = __fadd_rn(r_even, r_odd);
  v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
  v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
  return v;
}

// The 4 MMAs of one iteration: returns row g's dots (+ 8 bsum) for blocks 8i+2t (e) and
// 8i+2t+1 (o). nvalid < 8 masks blocks >= nvalid (their weights count as zero).
HV_DEV void mma_iter(const unsigned (&w)[8], uint2 bw, int t, int nvalid, int& e, int& o) {
  e = 0;
  o = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const unsigned w0 = (j < nvalid) ? w[j] : 0x88888888u;
    const unsigned w4 = (j + 4 < nvalid) ? w[j + 4] : 0x88888888u;
    int d0, d1, d2, d3;
    mma_u8s8(nib_lo(w0), nib_lo(w4), nib_hi(w0), nib_hi(w4), bw.x, bw.y, d0, d1, d2, d3);
    // column 2t holds block 2t's dot (rows 0..7, j = 2t) or block 2t's (rows 8..15, j+4 = 2t)
    if (t < 2) {
      if (j == 2 * t) e = d0;
      if (j == 2 * t + 1) o = d1;
    } else {
      if (j + 4 == 2 * t) e = d2;
      if (j + 4 == 2 * t + 1) o = d3;
    }
  }
}

// 8 rows of a GEMV. Reference layout (kPP false): lane (g, t) passes the pointers of its
// row g (r, sr); rows that do not exist point at a valid row and are not stored.
// Tile-interleaved layout (kPP true): r and sr are the tile's nibble and scale bases. Computes the leaves
// [leaf_lo, leaf_hi) of the block sum. kFold: the range is every leaf and *y (all four
// lanes of the quad) becomes (+0) + pairwise. Otherwise each finished leaf value goes to
// leafv[leaf] (lane t == 0 writes). act_w: int8 activations as words; sb: (scale, bsum).
template <int U, bool kFold, bool kPP = false>
HV_DEV void gemv_tile8(const uint32_t* __restrict__ r, const float* __restrict__ sr,
                       const unsigned* __restrict__ act_w, const int2* __restrict__ sb,
                       const GvPlan& P, int leaf_lo, int leaf_hi, float* y, float* leafv) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int it_lo = leaf_lo == 0 ? 0 : P.it_end[leaf_lo - 1];
  const int it_hi = P.it_end[leaf_hi - 1];
  const bool has_tail = (leaf_hi == P.nleaf) && P.ntail > 0;

  MmaLoads L[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (it_lo + u < it_hi) {
      if constexpr (kPP) mma_load_pp(L[u], r, sr, it_lo + u, lane);
      else mma_load(L[u], r, sr, it_lo + u, t);
    }
  }

  float st[8];               // fold stack (postfix '+' of numpy's recursion)
  int sp = 0;
  int leaf = leaf_lo;
  int leaf_begin = it_lo;
  int leaf_end = P.it_end[leaf_lo];
  float acc_e = 0.f, acc_o = 0.f;   // accumulators 2t, 2t+1

  for (int it0 = it_lo; it0 < it_hi; it0 += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = it0 + u;
      if (it < it_hi) {
        const uint2 bw = reinterpret_cast<const uint2*>(act_w)[(it * 8 + g) * 4 + t];
        int e, o;
        mma_iter(L[u].w, bw, t, 8, e, o);
        const int4 sbb = reinterpret_cast<const int4*>(sb)[it * 4 + t];   // blocks 2t, 2t+1
        const float ce = __fmul_rn(__fmul_rn(L[u].s.x, __int_as_float(sbb.x)),
                                   i2f_exact(e - 8 * sbb.y));
        const float co = __fmul_rn(__fmul_rn(L[u].s.y, __int_as_float(sbb.z)),
                                   i2f_exact(o - 8 * sbb.w));
        if (it == leaf_begin) {
          acc_e = ce;
          acc_o = co;
        } else {
          acc_e = __fadd_rn(acc_e, ce);
          acc_o = __fadd_rn(acc_o, co);
        }
        const int itn = it + U;
        if (itn < it_hi) {
          if constexpr (kPP) mma_load_pp(L[u], r, sr, itn, lane);
          else mma_load(L[u], r, sr, itn, t);
        }
        if (it + 1 == leaf_end && leaf + 1 < leaf_hi) {
          const float v = quad_fold(acc_e, acc_o);     // a leaf that is not the last
          if constexpr (kFold) {
            st[sp++] = v;
            for (int k = 0; k < P.pops[leaf]; ++k) {
              --sp;
              st[sp - 1] = __fadd_rn(st[sp - 1], st[sp]);
            }
          } else if (t == 0) {
            leafv[leaf] = v;
          }
          ++leaf;
          leaf_begin = leaf_end;
          leaf_end = P.it_end[leaf];
        }
      }
    }
  }

  // the range's last leaf: its 8-accumulator tree (if it has full iterations), then the
  // n % 8 tail blocks in order (only ever in the row's last leaf)
  float v = (it_hi > leaf_begin) ? quad_fold(acc_e, acc_o) : 0.f;
  if (has_tail) {
    const int it = P.nfull, nt = P.ntail;
    MmaLoads T;
    if constexpr (kPP) {
      mma_load_pp(T, r, sr, it, lane);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) T.w[j] = (j < nt) ? ldg_u32(r + (it * 8 + j) * 4 + t) : 0u;
      T.s = make_float2(0.f, 0.f);
    }
    const uint2 bw = (g < nt) ? reinterpret_cast<const uint2*>(act_w)[(it * 8 + g) * 4 + t]
                              : make_uint2(0u, 0u);
    int e, o;
    mma_iter(T.w, bw, t, nt, e, o);
    float ce = 0.f, co = 0.f;
    if (2 * t < nt) {
      const int b = it * 8 + 2 * t;
      const float s = kPP ? T.s.x : __ldg(sr + b);
      ce = __fmul_rn(__fmul_rn(s, __int_as_float(sb[b].x)), i2f_exact(e - 8 * sb[b].y));
    }
    if (2 * t + 1 < nt) {
      const int b = it * 8 + 2 * t + 1;
      const float s = kPP ? T.s.y : __ldg(sr + b);
      co = __fmul_rn(__fmul_rn(s, __int_as_float(sb[b].x)), i2f_exact(o - 8 * sb[b].y));
    }
    // tail block j sits in lane (g, j / 2): even j in ce, odd in co; add in order
    for (int j = 0; j < nt; ++j) {
      const float x = __shfl_sync(0xFFFFFFFFu, (j & 1) ? co : ce, (lane & ~3) | (j >> 1));
      v = __fadd_rn(v, x);
    }
  }
  if constexpr (kFold) {
    st[sp++] = v;
    for (int k = 0; k < P.pops[leaf_hi - 1]; ++k) {
      --sp;
      st[sp - 1] = __fadd_rn(st[sp - 1], st[sp]);
    }
    *y = __fadd_rn(0.0f, st[0]);
  } else if (t == 0) {
    leafv[leaf_hi - 1] = v;
  }
}

// ---- the dp4a form over the "dq" tile layout -------------------------------------------
//
// The same 8-row tiles and 8-block iterations as the tile-interleaved layout, with the
// words of each iteration arranged so that lane L = 4g + t holds ALL four words of its own
// two blocks: words 0..3 of block 2t of row g at 4L, of block 2t+1 at 128 + 4L (scales as
// before: the pair at 2L). A lane then forms its two exact int32 block dots with dp4a
// (block_dot), no tensor-pipe MMA and no selection among MMA outputs; the accumulators,
// their order and the combine are those of gemv_tile8, so the fp32 results are
// bit-identical to the tile-interleaved kernels.
constexpr int kDqNibWords = kPpNibWords;   // per tile and iteration
constexpr int kDqScales = kPpScales;

struct DqLoads {
  uint4 e, o;    // words 0..3 of blocks 2t and 2t+1
  float2 s;      // their scales
};

HV_DEV void dq_load(DqLoads& L, const uint32_t* tn, const float* ts, int it, int lane) {
  L.e = ldg_stream128(tn + (size_t)it * kDqNibWords + 4 * lane);
  L.o = ldg_stream128(tn + (size_t)it * kDqNibWords + 128 + 4 * lane);
  L.s = ldg_stream_f2(ts + (size_t)it * kDqScales + 2 * lane);
}

// Block terms of iteration `it` for lane (g, t): blocks 2t (x) and 2t+1 (y); blocks at or
// beyond nvalid count zero. q: int8 activations, 2 x uint4 per block; sb: (scale bits,
// block sum) per block.
HV_DEV float2 dq_terms(const DqLoads& L, const uint4* __restrict__ q,
                       const int2* __restrict__ sb, int it, int t, int nvalid) {
  const int be = it * 8 + 2 * t;
  float ce = 0.f, co = 0.f;
  if (2 * t < nvalid) {
    const int2 s2 = sb[be];
    const int d = block_dot(L.e, q[2 * be], q[2 * be + 1], s2.y);
    ce = __fmul_rn(__fmul_rn(L.s.x, __int_as_float(s2.x)), i2f_exact(d));
  }
  if (2 * t + 1 < nvalid) {
    const int2 s2 = sb[be + 1];
    const int d = block_dot(L.o, q[2 * be + 2], q[2 * be + 3], s2.y);
    co = __fmul_rn(__fmul_rn(L.s.y, __int_as_float(s2.x)), i2f_exact(d));
  }
  return make_float2(ce, co);
}

// gemv_tile8<U, true, true> over the dq layout: the 8 rows of one tile, every leaf, the
// quad's y = (+0) + pairwise over all blocks.
template <int U>
HV_DEV float gemv_tile8_dq(const uint32_t* __restrict__ tn, const float* __restrict__ ts,
                           const uint4* __restrict__ q, const int2* __restrict__ sb,
                           const GvPlan& P) {
  const int lane = threadIdx.x & 31;
  const int t = lane & 3;
  const int it_hi = P.nfull;
  DqLoads L[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (u < it_hi) dq_load(L[u], tn, ts, u, lane);

  float st[8];               // fold stack (postfix '+' of numpy's recursion)
  int sp = 0;
  int leaf = 0;
  int leaf_begin = 0;
  int leaf_end = P.it_end[0];
  float acc_e = 0.f, acc_o = 0.f;   // accumulators 2t, 2t+1

  for (int it0 = 0; it0 < it_hi; it0 += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = it0 + u;
      if (it < it_hi) {
        const float2 c = dq_terms(L[u], q, sb, it, t, 8);
        if (it == leaf_begin) {
          acc_e = c.x;
          acc_o = c.y;
        } else {
          acc_e = __fadd_rn(acc_e, c.x);
          acc_o = __fadd_rn(acc_o, c.y);
        }
        const int itn = it + U;
        if (itn < it_hi) dq_load(L[u], tn, ts, itn, lane);
        if (it + 1 == leaf_end && leaf + 1 < P.nleaf) {
          st[sp++] = quad_fold(acc_e, acc_o);        // a leaf that is not the last
          for (int k = 0; k < P.pops[leaf]; ++k) {
            --sp;
            st[sp - 1] = __fadd_rn(st[sp - 1], st[sp]);
          }
          ++leaf;
          leaf_begin = leaf_end;
          leaf_end = P.it_end[leaf];
        }
      }
    }
  }
  float v = (it_hi > leaf_begin) ? quad_fold(acc_e, acc_o) : 0.f;
  if (P.ntail > 0) {                 // the n % 8 tail blocks, in order (last leaf only)
    DqLoads T;
    dq_load(T, tn, ts, P.nfull, lane);
    const float2 c = dq_terms(T, q, sb, P.nfull, t, P.ntail);
    for (int j = 0; j < P.ntail; ++j) {
      const float x = __shfl_sync(0xFFFFFFFFu, (j & 1) ? c.y : c.x, (lane & ~3) | (j >> 1));
      v = __fadd_rn(v, x);
    }
  }
  st[sp++] = v;
  for (int k = 0; k < P.pops[P.nleaf - 1]; ++k) {
    --sp;
    st[sp - 1] = __fadd_rn(st[sp - 1], st[sp]);
  }
  return __fadd_rn(0.0f, st[0]);
}

// Folds a row's leaf values leafv[0 .. nleaf) with the plan's postfix '+'.
HV_DEV float fold_leaves(const GvPlan& P, const float* leafv) {
  float st[8];
  int sp = 0;
  for (int i = 0; i < P.nleaf; ++i) {
    st[sp++] = leafv[i];
    for (int k = 0; k < P.pops[i]; ++k) {
      --sp;
      st[sp - 1] = __fadd_rn(st[sp - 1], st[sp]);
    }
  }
  return __fadd_rn(0.0f, st[0]);
}

// Sizes of a matrix of `rows` rows (or gate/up pairs when pair_ffn > 0) in the
// tile-interleaved layout.
HV_HD int pp_tiles(int rows, int pair_ffn) {
  return pair_ffn > 0 ? (pair_ffn + 3) / 4 : (rows + 7) / 8;
}
HV_HD int pp_iters(int nb) { return (nb + 7) / 8; }

// Row of the reference matrix behind quad g of `tile`: plain 8-row tiles, or (pair_ffn
// > 0) 4 gate rows p and their 4 up rows ffn + p of a [gate | up] matrix.
HV_DEV int pp_row(int tile, int g, int rows, int pair_ffn, bool* ok) {
  if (pair_ffn > 0) {
    const int p = tile * 4 + (g & 3);
    *ok = p < pair_ffn;
    return (g < 4) ? p : pair_ffn + p;
  }
  const int row = tile * 8 + g;
  *ok = row < rows;
  return row;
}

}  // namespace hv
