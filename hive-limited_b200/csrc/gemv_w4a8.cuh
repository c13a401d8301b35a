// W4A8 GEMV row routine shared by the standalone k_a4gv kernel and the fused step.
//
// y[n] = sum over 32-blocks b of f32(f32(sw[n,b] * sa[b]) * f32(idot[n,b])), summed in
// numpy's pairwise order (engine/reference.py:62-72 and numpy's float32 add.reduce).
//
// Mapping: one warp computes four rows at once; the 8 lanes of lane group r own row r.
// numpy's pairwise leaf keeps eight strided accumulators r[j] += c[8i + j], so lane j of
// the group IS accumulator j: it walks blocks j, j+8, j+16, ... of its row, in order,
// and the three xor-shuffles of the fold reproduce ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))
// exactly. Leaves end where numpy's recursion splits; their values are folded with the
// recursion's '+' in postfix order.
//
// Loads: every block is 16 bytes of nibbles (one 128-bit load) plus one 4-byte scale.
// The 8 lanes of a group read 128 consecutive bytes of one row, so each warp-wide load
// touches four full 128-byte lines. Loads run U iterations ahead of the arithmetic.
#pragma once

#include "hv_common.cuh"

namespace hv {

constexpr int kGvMaxLeaf = 64;   // leaves of the block-sum recursion (nb <= 4096)

struct GvPlan {
  int nb;            // 32-blocks per row
  int nfull;         // full 8-block iterations (nb - nb % 8) / 8
  int ntail;         // nb % 8 blocks left over (only ever in the last leaf)
  int nleaf;
  int it_end[kGvMaxLeaf];           // iteration index (exclusive) where leaf L ends
  unsigned char pops[kGvMaxLeaf];   // '+' of the recursion closing after leaf L
};

// numpy's pairwise recursion over nb block terms, as iteration boundaries. Runs on the
// host so kernels receive a finished plan.
HV_HD bool gv_make_plan(int nb, GvPlan* g) {
  int sk[64], ss[64], sm[64];
  int sp = 1, nl = 0;
  sk[0] = 0; ss[0] = 0; sm[0] = nb;
  while (sp > 0) {
    --sp;
    const int k = sk[sp], s = ss[sp], m = sm[sp];
    if (k == 1) {
      g->pops[nl - 1]++;
    } else if (m <= kPwLeaf) {
      if (nl >= kGvMaxLeaf) return false;
      g->it_end[nl] = (s + m - ((s + m == nb) ? nb % 8 : 0)) / 8;
      g->pops[nl] = 0;
      ++nl;
    } else {
      if (sp + 3 > 64) return false;
      int m2 = m / 2; m2 -= m2 % 8;
      sk[sp] = 1; ss[sp] = 0; sm[sp] = 0; ++sp;
      sk[sp] = 0; ss[sp] = s + m2; sm[sp] = m - m2; ++sp;
      sk[sp] = 0; ss[sp] = s; sm[sp] = m2; ++sp;
    }
  }
  g->nb = nb;
  g->nfull = nb / 8;
  g->ntail = nb % 8;
  g->nleaf = nl;
  return true;
}

// Quantised activation resident in shared memory.
struct ActView {
  const uint4* q;    // int8 activations, 2 x uint4 per block
  const int2* sb;    // (scale bits, block sum) per block
};

// Computes rows row0 + (lane / 8) of a row-major packed matrix (b4 [N][nb*4] u32,
// sw [N][nb] f32). Returns y for the lane's row in all 8 lanes of its group.
// Rows >= n are computed from row 0's data (so the shuffles stay converged) and must
// not be stored by the caller. When kIdot, also stores the int32 block dots.
template <int U, bool kIdot>
HV_DEV float gemv_rows4(const uint32_t* __restrict__ b4, const float* __restrict__ sw,
                        int row, bool row_ok, const ActView act, const GvPlan& P,
                        int32_t* __restrict__ idot_out) {
  const int lane = threadIdx.x & 31;
  const int sub = lane & 7;
  const unsigned gmask = 0xFFu << (lane & ~7);
  const int nb = P.nb;
  const int nfull = P.nfull;
  const int lrow = row_ok ? row : 0;
  const uint4* __restrict__ wrow = reinterpret_cast<const uint4*>(b4) + (size_t)lrow * nb;
  const float* __restrict__ srow = sw + (size_t)lrow * nb;

  uint4 rn[U];
  float rs[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (u < nfull) {
      rn[u] = ldg_stream4(wrow + u * 8 + sub);
      rs[u] = ldg_stream1(srow + u * 8 + sub);
    }
  }

  float st[8];          // fold stack (postfix '+' of numpy's recursion)
  int sp = 0;
  int leaf = 0;
  int leaf_begin = 0;
  int leaf_end = P.it_end[0];
  float chain = 0.0f;

  for (int it0 = 0; it0 < nfull; it0 += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = it0 + u;
      if (it < nfull) {
        const int b = it * 8 + sub;
        const uint4 a0 = act.q[2 * b];
        const uint4 a1 = act.q[2 * b + 1];
        const int2 sb = act.sb[b];
        const int d = block_dot(rn[u], a0, a1, sb.y);
        const float c = block_term(rs[u], __int_as_float(sb.x), d);
        chain = (it == leaf_begin) ? c : __fadd_rn(chain, c);
        if (kIdot && row_ok) idot_out[(size_t)row * nb + b] = d;
        const int itn = it + U;
        if (itn < nfull) {
          rn[u] = ldg_stream4(wrow + itn * 8 + sub);
          rs[u] = ldg_stream1(srow + itn * 8 + sub);
        }
        if (it + 1 == leaf_end && leaf + 1 < P.nleaf) {
          // a leaf that is not the last: fold its 8 accumulators and push it
          float v = __fadd_rn(chain, __shfl_xor_sync(gmask, chain, 1, 8));
          v = __fadd_rn(v, __shfl_xor_sync(gmask, v, 2, 8));
          v = __fadd_rn(v, __shfl_xor_sync(gmask, v, 4, 8));
          st[sp++] = v;
          for (int k = 0; k < P.pops[leaf]; ++k) {
            const float bb = st[--sp];
            const float aa = st[--sp];
            st[sp++] = __fadd_rn(aa, bb);
          }
          ++leaf;
          leaf_begin = leaf_end;
          leaf_end = P.it_end[leaf];
        }
      }
    }
  }

  // the last leaf: its 8-accumulator fold (if it had full iterations), then the tail
  float v;
  if (nfull > 0) {
    v = __fadd_rn(chain, __shfl_xor_sync(gmask, chain, 1, 8));
    v = __fadd_rn(v, __shfl_xor_sync(gmask, v, 2, 8));
    v = __fadd_rn(v, __shfl_xor_sync(gmask, v, 4, 8));
  } else {
    v = 0.0f;
  }
  if (P.ntail > 0) {
    float ct = 0.0f;
    if (sub < P.ntail) {
      const int b = nfull * 8 + sub;
      const uint4 nib = ldg_stream4(wrow + b);
      const float s = ldg_stream1(srow + b);
      const int2 sb = act.sb[b];
      const int d = block_dot(nib, act.q[2 * b], act.q[2 * b + 1], sb.y);
      ct = block_term(s, __int_as_float(sb.x), d);
      if (kIdot && row_ok) idot_out[(size_t)row * nb + b] = d;
    }
    for (int t = 0; t < P.ntail; ++t) v = __fadd_rn(v, __shfl_sync(gmask, ct, t, 8));
  }
  st[sp++] = v;
  for (int k = 0; k < P.pops[P.nleaf - 1]; ++k) {
    const float bb = st[--sp];
    const float aa = st[--sp];
    st[sp++] = __fadd_rn(aa, bb);
  }
  return __fadd_rn(0.0f, st[0]);
}

// Copies a quantised activation (a8 int8 [nb*32], sa f32 [2*nb] = scales then block sums
// as int32 bits, the quant_a8s layout) into shared memory. Block-cooperative.
HV_DEV void load_act_smem(const int8_t* __restrict__ a8, const float* __restrict__ sa, int nb,
                          uint4* q_s, int2* sb_s) {
  const uint4* src = reinterpret_cast<const uint4*>(a8);
  for (int i = threadIdx.x; i < nb * 2; i += blockDim.x) q_s[i] = src[i];
  for (int b = threadIdx.x; b < nb; b += blockDim.x)
    sb_s[b] = make_int2(__float_as_int(sa[b]), __float_as_int(sa[nb + b]));
}

}  // namespace hv
