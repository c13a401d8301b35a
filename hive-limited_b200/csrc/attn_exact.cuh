// Decode attention in the reference's own order of operations, bit for bit.
//
// engine/reference.py:104-118 computes, per query head h over the T = pos + 1 cached
// positions:
//   logits = (keys @ q) * scale      keys @ q: OpenBLAS sgemv, one row dot per position
//   logits -= logits.max()
//   w = np.exp(logits)               numpy's float32 SIMD exp
//   w /= w.sum()                     numpy's pairwise sum, then one division per element
//   out = (w[:, None] * vals).sum(0) rounded products, summed over positions IN ORDER
// Every step is restated here: np_expf is numpy's exp algorithm, rowdots_blas the order
// OpenBLAS's gemv forms each row dot on the reference host (three row kinds, chosen by
// the row's place in the host's run split), PwTree numpy's pairwise recursion, and the
// weighted V sum a sequential chain per output element. So the context vector equals the
// reference's exactly, and the whole decode is bit-identical.
//
// Work split (used by the eager kernels, the batched prefill and the fused step alike):
//  * scores: per (kv head, chunk of positions), every position's dot with the GS query
//    heads of the kv head; 8 lanes per position (lane j owns OpenBLAS's accumulator j),
//    four positions per warp instruction. Scores go to a [head][cap] buffer, each chunk's
//    maximum to a [head][chunk] buffer.
//  * context: per (kv head, 32-dim slice of the head): the maximum, the pairwise sum of
//    the exps (leaves in parallel, the recursion's '+' level by level), then one warp per
//    query head runs the chain over the positions, lane d owning output dim 32 j + d.
//    The chain is T dependent adds: it is the latency floor of this attention.
#pragma once

#include "attn_decode.cuh"

namespace hv {

constexpr int kTreeMaxLeaf = 256;     // pairwise leaves of one softmax sum: n <= 16384
constexpr int kExactMaxCap = 16384;   // longest cache the exact attention takes
constexpr int kRefRuns = 8;           // OpenBLAS threads of the host the reference ran on
constexpr int kSlices = kHd / 32;     // 32-dim slices of a head (one chain warp each)
constexpr int kChainChunk = 256;      // positions whose weights a chain warp stages at once

// ---------------------------------------------------------------------------
// OpenBLAS's sgemv ("T" form, rows of 128 contiguous floats) forms each row dot in one of
// three ways, by the row's place in its run of rows:
//   kind 0, rows in whole groups of 4: 8 accumulators, accumulator j takes elements
//     j, j+8, ... by fused multiply-add from +0; then s_k = a_k + a_{k+4} and
//     (s0 + s1) + (s2 + s3);
//   kind 1, the next two rows when a run has 2 or 3 left over: 4 accumulators,
//     accumulator j adds the rounded products of elements j, j+4, ...; then
//     (a0 + a1) + (a2 + a3);
//   kind 2, the last row when a run has 1 or 3 left over: kind 0 with every product
//     rounded before its add.
// A gemv of T rows is one run, or -- when 128 T >= 460800 -- `runs` runs of
// ceil(rows left / runs left) rows (at least 4), one per host thread.
// ---------------------------------------------------------------------------
HV_HD int blas_row_kind(int T, int t, int runs) {
  const int nrun = (128L * T >= 460800L && runs > 1) ? runs : 1;
  int r0 = 0, left = T;
  for (int k = 0; k < nrun && left > 0; ++k) {
    int w = (left + (nrun - k) - 1) / (nrun - k);
    if (w < 4) w = 4;
    if (w > left) w = left;
    if (t < r0 + w) {
      const int off = t - r0, full = w & ~3;
      if (off < full) return 0;
      if ((w & 2) && off < full + 2) return 1;
      return 2;
    }
    r0 += w;
    left -= w;
  }
  return 0;
}

// The same split, worked out once for a gemv of T rows: the rows whose dots are not of
// kind 0 are the last 1-3 of each run; at most kMaxRuns runs.
constexpr int kMaxRuns = 32;
struct BlasRuns {
  int n;                       // runs
  int odd0[kMaxRuns];          // first row of the run's leftover (not kind 0)
  int end[kMaxRuns];           // one past the run's last row
  int k1end[kMaxRuns];         // rows [odd0, k1end) are kind 1, [k1end, end) kind 2
};

HV_HD void blas_runs(int T, int runs, BlasRuns* b) {
  int nrun = (128L * T >= 460800L && runs > 1) ? runs : 1;
  if (nrun > kMaxRuns) nrun = kMaxRuns;
  int r0 = 0, left = T, n = 0;
  for (int k = 0; k < nrun && left > 0; ++k) {
    int w = (left + (nrun - k) - 1) / (nrun - k);
    if (w < 4) w = 4;
    if (w > left) w = left;
    const int full = w & ~3;
    b->odd0[n] = r0 + full;
    b->end[n] = r0 + w;
    b->k1end[n] = r0 + full + ((w & 2) ? 2 : 0);
    ++n;
    r0 += w;
    left -= w;
  }
  b->n = n;
}

HV_HD int blas_kind_of(const BlasRuns& b, int t) {
  for (int k = 0; k < b.n; ++k)
    if (t < b.end[k]) return t < b.odd0[k] ? 0 : (t < b.k1end[k] ? 1 : 2);
  return 0;
}

// The row kinds of a block of rows starting at r0, looked up once per block: the run
// holding r0 and the next one (a block of up to 20 rows never spans more than two runs:
// when there are several runs each holds at least 112 rows).
struct RunWin {
  int enda, odd0a, k1a, odd0b, k1b;
};
HV_DEV RunWin run_window(const BlasRuns& b, int r0) {
  int k = 0;
  while (k + 1 < b.n && r0 >= b.end[k]) ++k;
  RunWin w;
  w.enda = b.end[k];
  w.odd0a = b.odd0[k];
  w.k1a = b.k1end[k];
  w.odd0b = k + 1 < b.n ? b.odd0[k + 1] : 0x7FFFFFFF;
  w.k1b = k + 1 < b.n ? b.k1end[k + 1] : 0x7FFFFFFF;
  return w;
}
HV_DEV int kind_in(const RunWin& w, int t) {
  if (t < w.enda) return t < w.odd0a ? 0 : (t < w.k1a ? 1 : 2);
  return t < w.odd0b ? 0 : (t < w.k1b ? 1 : 2);
}

// Query elements an 8-lane group's lane j keeps for kind-0/2 dots: q[h][j + 8 i].
template <int HP>
HV_DEV void load_qregs(const float* q_s, int j, float (&qr)[HP][16]) {
#pragma unroll
  for (int h = 0; h < HP; ++h)
#pragma unroll
    for (int i = 0; i < 16; ++i) qr[h][i] = q_s[h * kHd + j + 8 * i];
}

// Dots of one cache row with HP query heads, in the order OpenBLAS forms the row's dot.
// Called by all 32 lanes; each aligned 8-lane group handles one row (lane j = lane & 7),
// `kind` is its row kind. row(e) returns element e of the group's row as a float; qr the
// lane's query elements; q_s the HP query rows (kind 1 reads them there). Every lane of
// the group gets the HP dots.
template <int HP, class Row>
HV_DEV void rowdots_blas(const Row& row, int kind, const float (&qr)[HP][16],
                         const float* q_s, int j, float (&d)[HP]) {
#pragma unroll
  for (int h = 0; h < HP; ++h) d[h] = 0.0f;
  if (kind == 0) {
    float k[16];                                   // every load before the first FMA
#pragma unroll
    for (int i = 0; i < 16; ++i) k[i] = row(j + 8 * i);
#pragma unroll
    for (int i = 0; i < 16; ++i)
#pragma unroll
      for (int h = 0; h < HP; ++h) d[h] = __fmaf_rn(k[i], qr[h][i], d[h]);
  } else if (kind == 2) {
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const float k = row(j + 8 * i);
#pragma unroll
      for (int h = 0; h < HP; ++h) d[h] = __fadd_rn(d[h], __fmul_rn(k, qr[h][i]));
    }
  } else {
    const int m = j & 3;
#pragma unroll 4
    for (int i = 0; i < 32; ++i) {
      const float k = row(m + 4 * i);
#pragma unroll
      for (int h = 0; h < HP; ++h) d[h] = __fadd_rn(d[h], __fmul_rn(k, q_s[h * kHd + m + 4 * i]));
    }
  }
#pragma unroll
  for (int h = 0; h < HP; ++h) {
    float v = d[h];
    const float v4 = __shfl_xor_sync(0xFFFFFFFFu, v, 4);
    if (kind != 1) v = __fadd_rn(v, v4);
    v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
    v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
    d[h] = v;
  }
}

// ---------------------------------------------------------------------------
// numpy's pairwise recursion as a tree, built and evaluated level by level by one warp.
// pairwise(x[0:n]): n <= 128 is a leaf; otherwise split at n2 = n/2 rounded down to a
// multiple of 8 and add pairwise(left) + pairwise(right). Level d holds the nodes at depth
// d in left-to-right order ([lev[d], lev[d+1]) of the node arrays); an internal node's
// children are nodes child and child + 1 of the next level. Every node gets a value slot
// (its id): leaves are summed in place, internal nodes folded from the deepest level up.
// ---------------------------------------------------------------------------
constexpr int kTreeMaxNode = 2 * kTreeMaxLeaf;
constexpr int kTreeMaxLev = 20;

struct PwTree {
  int n, nnode, nlev, nleaf;
  unsigned short lev[kTreeMaxLev + 1];
  unsigned short start[kTreeMaxNode], size[kTreeMaxNode];
  short child[kTreeMaxNode];               // left child's id, -1 for a leaf
  unsigned short leaf[kTreeMaxLeaf];       // ids of the leaves
};

// Upper bound on the nodes of numpy's recursion over n values.
HV_HD int pw_tree_nodes_max(int n) { return n <= kPwLeaf ? 1 : 4 * ((n + kPwLeaf - 1) / kPwLeaf) + 1; }

// Builds the tree for n values (one warp, every lane gets the result). False if it does
// not fit.
HV_DEV bool pw_tree_build_warp(int n, PwTree* t) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  if (lane == 0) {
    t->start[0] = 0;
    t->size[0] = (unsigned short)(n < 65535 ? n : 65535);
    t->lev[0] = 0;
    t->lev[1] = 1;
  }
  __syncwarp();
  if (n < 1 || n > kExactMaxCap) return false;
  int nl = 0, d = 0;
  for (;; ++d) {
    const int a = t->lev[d], b = t->lev[d + 1];
    if (a == b) break;
    if (d + 2 > kTreeMaxLev) return false;
    int next = b;
    for (int base = a; base < b; base += 32) {
      const int i = base + lane;
      const bool live = i < b;
      const int m = live ? t->size[i] : 0;
      const bool inner = live && m > kPwLeaf;
      const unsigned bi = __ballot_sync(0xFFFFFFFFu, inner);
      const unsigned bl = __ballot_sync(0xFFFFFFFFu, live && !inner);
      const int c = next + 2 * __popc(bi & lt);
      const int k = nl + __popc(bl & lt);
      if (next + 2 * __popc(bi) > kTreeMaxNode || nl + __popc(bl) > kTreeMaxLeaf) return false;
      if (inner) {
        int m2 = m / 2;
        m2 -= m2 % 8;
        t->start[c] = t->start[i];
        t->size[c] = (unsigned short)m2;
        t->start[c + 1] = (unsigned short)(t->start[i] + m2);
        t->size[c + 1] = (unsigned short)(m - m2);
        t->child[i] = (short)c;
      } else if (live) {
        t->child[i] = -1;
        t->leaf[k] = (unsigned short)i;
      }
      next += 2 * __popc(bi);
      nl += __popc(bl);
    }
    if (lane == 0) t->lev[d + 2] = (unsigned short)next;
    __syncwarp();
  }
  if (lane == 0) {
    t->n = n;
    t->nnode = t->lev[d];
    t->nlev = d;
    t->nleaf = nl;
  }
  __syncwarp();
  return true;
}

// ---------------------------------------------------------------------------
// The top of numpy's recursion over T values, cut at depth `depth`: the nodes at that
// depth (or leaves, <= 128 values, above it) in left-to-right order are the chunks of the
// fused step's attention, so each chunk's pairwise sum is an exact subtree of the whole
// sum and only the nodes above the chunks remain to be added. pops[c]: how many '+' of
// the recursion close right after chunk c (postfix order).
// ---------------------------------------------------------------------------
constexpr int kMaxFront = 128;

struct PwFront {
  int n;                                   // chunks
  int cb[kMaxFront + 1];                   // chunk c = values [cb[c], cb[c + 1])
  unsigned char pops[kMaxFront];
};

HV_HD bool pw_front_build(int T, int depth, PwFront* f) {
  int ss[64], sm[64], sk[64], sd[64];      // DFS stack: start, count, kind (0 node, 1 '+')
  int sp = 0, nc = 0;
  ss[0] = 0; sm[0] = T; sk[0] = 0; sd[0] = 0; sp = 1;
  while (sp > 0) {
    --sp;
    const int s = ss[sp], m = sm[sp], k = sk[sp], d = sd[sp];
    if (k == 1) {
      if (nc == 0) return false;
      f->pops[nc - 1]++;
    } else if (m <= kPwLeaf || d >= depth) {
      if (nc >= kMaxFront) return false;
      f->cb[nc] = s;
      f->pops[nc] = 0;
      ++nc;
    } else {
      if (sp + 3 > 64) return false;
      int m2 = m / 2;
      m2 -= m2 % 8;
      ss[sp] = 0; sm[sp] = 0; sk[sp] = 1; sd[sp] = d; ++sp;
      ss[sp] = s + m2; sm[sp] = m - m2; sk[sp] = 0; sd[sp] = d + 1; ++sp;
      ss[sp] = s; sm[sp] = m2; sk[sp] = 0; sd[sp] = d + 1; ++sp;
    }
  }
  f->cb[nc] = T;
  f->n = nc;
  return true;
}

// (+0) + the recursion's '+' over the chunks' sums val[0 .. n) (one thread).
HV_DEV float pw_front_fold(const PwFront& f, const float* val) {
  float st[24];
  int sp = 0;
  for (int c = 0; c < f.n; ++c) {
    st[sp++] = val[c];
    for (int k = 0; k < f.pops[c]; ++k) {
      const float b = st[--sp];
      const float a = st[--sp];
      st[sp++] = __fadd_rn(a, b);
    }
  }
  return __fadd_rn(0.0f, st[0]);
}

// Largest chunk of the recursion cut at a depth with nch = 2^depth chunks: a split leaves
// at most half + 8 values on either side, so after d splits a node holds fewer than
// T / 2^d + 16; leaves above the cut hold at most 128.
HV_HD int front_chunk_max(int cap, int nch) {
  const int a = (cap + nch - 1) / nch + 16;
  return a > kPwLeaf ? a : kPwLeaf;
}

// Depth of the fused step's chunking for n_kv kv heads on `grid` CTAs: every (kv head,
// chunk) work item gets a CTA of its own (n_kv 2^depth <= grid), at most kMaxFront chunks.
HV_HD int front_depth(int n_kv, int grid) {
  int d = 0;
  while (d < 7 && (n_kv << (d + 1)) <= grid) ++d;
  return d;
}

// One leaf [s, s + len) of a head's softmax sum: e_t = np_expf(lg[t] - M) for its
// positions (stored into e[t] when e is set), summed by the 8 lanes of an aligned group
// (sub = lane & 7) in numpy's leaf order: < 8 values sequentially from +0; else eight
// strided accumulators, ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then the len % 8 tail in
// order. Every lane of the group returns the sum. All of a lane's scores are loaded
// before the first exp, so a leaf costs one load latency.
struct LeafRaw {
  float x[16], tl[7];
};

// The scores of the lane's share of leaf [s, s + len) (loads only, all issued at once).
HV_DEV void leaf_load(const float* lg, int s, int len, int sub, LeafRaw& L) {
  const int full = len >= 8 ? len - (len % 8) : 0;
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int i = sub + 8 * m;
    L.x[m] = i < full ? __ldcg(lg + s + i) : 0.0f;
  }
#pragma unroll
  for (int m = 0; m < 7; ++m) L.tl[m] = full + m < len ? __ldcg(lg + s + full + m) : 0.0f;
}

// The exps and the leaf's sum from leaf_load's scores.
HV_DEV float leaf_finish(LeafRaw& L, float M, float* e, int s, int len, int sub) {
  const unsigned gmask = 0xFFu << ((threadIdx.x & 31) & ~7);
  const int full = len >= 8 ? len - (len % 8) : 0;
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int i = sub + 8 * m;
    if (i < full) {
      L.x[m] = np_expf(__fsub_rn(L.x[m], M));
      if (e) e[s + i] = L.x[m];
    }
  }
#pragma unroll
  for (int m = 0; m < 7; ++m) {
    if (full + m < len) {
      L.tl[m] = np_expf(__fsub_rn(L.tl[m], M));
      if (e && sub == 0) e[s + full + m] = L.tl[m];
    }
  }
  float r;
  if (len >= 8) {
    r = L.x[0];
#pragma unroll
    for (int m = 1; m < 16; ++m)
      if (sub + 8 * m < full) r = __fadd_rn(r, L.x[m]);
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 1, 8));
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 2, 8));
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 4, 8));
  } else {
    r = 0.0f;
  }
#pragma unroll
  for (int m = 0; m < 7; ++m)
    if (full + m < len) r = __fadd_rn(r, L.tl[m]);
  return r;
}

HV_DEV float leaf_exp_sum(const float* lg, float M, float* e, int s, int len, int sub) {
  LeafRaw L;
  leaf_load(lg, s, len, sub, L);
  return leaf_finish(L, M, e, s, len, sub);
}

// Sum of leaf [s, s + len) of values x[t * stride] (shared memory) by the 8 lanes of an
// aligned group, numpy's leaf order (as leaf_finish); every lane of the group returns it.
HV_DEV float leaf_sum_strided(const float* x, int stride, int s, int len, int sub) {
  const unsigned gmask = 0xFFu << ((threadIdx.x & 31) & ~7);
  const int full = len >= 8 ? len - (len % 8) : 0;
  float v[16], tl[7];
#pragma unroll
  for (int m = 0; m < 16; ++m) {
    const int i = sub + 8 * m;
    v[m] = i < full ? x[(size_t)(s + i) * stride] : 0.0f;
  }
#pragma unroll
  for (int m = 0; m < 7; ++m) tl[m] = full + m < len ? x[(size_t)(s + full + m) * stride] : 0.0f;
  float r;
  if (len >= 8) {
    r = v[0];
#pragma unroll
    for (int m = 1; m < 16; ++m)
      if (sub + 8 * m < full) r = __fadd_rn(r, v[m]);
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 1, 8));
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 2, 8));
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 4, 8));
  } else {
    r = 0.0f;
  }
#pragma unroll
  for (int m = 0; m < 7; ++m)
    if (full + m < len) r = __fadd_rn(r, tl[m]);
  return r;
}

// pw_tree_fold without the final (+0) +: the value of the tree's root (a subtree of a
// larger sum).
HV_DEV float pw_tree_fold_raw(const PwTree* t, float* vals) {
  const int lane = threadIdx.x & 31;
  for (int d = t->nlev - 1; d >= 0; --d) {
    for (int i = t->lev[d] + lane; i < t->lev[d + 1]; i += 32) {
      const int c = t->child[i];
      if (c >= 0) vals[i] = __fadd_rn(vals[c], vals[c + 1]);
    }
    __syncwarp();
  }
  return vals[0];
}

// One warp: the internal nodes of `t` from the deepest level up, over vals[] (leaf sums
// already at their node ids); returns (+0) + root to every lane.
HV_DEV float pw_tree_fold(const PwTree* t, float* vals) {
  const int lane = threadIdx.x & 31;
  for (int d = t->nlev - 1; d >= 0; --d) {
    for (int i = t->lev[d] + lane; i < t->lev[d + 1]; i += 32) {
      const int c = t->child[i];
      if (c >= 0) vals[i] = __fadd_rn(vals[c], vals[c + 1]);
    }
    __syncwarp();
  }
  return __fadd_rn(0.0f, vals[0]);
}

// ---------------------------------------------------------------------------
// Scores of one 4-position group per warp: positions tb + (lane >> 3) for HP heads.
// ---------------------------------------------------------------------------

// One cache element as a float (binary16 widens exactly).
HV_DEV float kv_elem(const float* p) { return __ldg(p); }
HV_DEV float kv_elem(const __half* p) { return __half2float(__ldg(p)); }

// K element source: a global cache row (float or binary16), converted to float.
template <class KT>
struct GlobalRow {
  const KT* p;
  HV_DEV float operator()(int e) const;
};
template <>
HV_DEV float GlobalRow<float>::operator()(int e) const { return __ldg(p + e); }
template <>
HV_DEV float GlobalRow<__half>::operator()(int e) const { return __half2float(__ldg(p + e)); }

// The weights w_t = np_expf(lg[t] - M) / S of positions [c0, c0 + kChainChunk) into a
// warp's buffer (zero past T).
HV_DEV void chain_weights(const float* lgh, int c0, int T, float M, float S, float* wbuf) {
  const int lane = threadIdx.x & 31;
#pragma unroll 2
  for (int u = 0; u < kChainChunk / 32; ++u) {
    const int t = c0 + 32 * u + lane;
    float w = 0.0f;
    if (t < T) w = __fdiv_rn(np_expf(__fsub_rn(__ldcg(lgh + t), M)), S);
    wbuf[32 * u + lane] = w;
  }
  __syncwarp();
}


// ---------------------------------------------------------------------------
// The standalone (eager) kernels. Grid y = token: a run of query tokens at consecutive
// positions (the batched prefill) or one token (decode). Token y sits at position
// pos = (pos_p ? *pos_p : pos0) + y and attends over T = pos + 1 cache rows (its own row
// already appended). Per-token scratch (`scr`, scr_tok floats apart): scores
// [nq][cap], then the chunk maxima [nq][nch].
// ---------------------------------------------------------------------------
constexpr int kAttnExThreads = 256;

HV_DEV int exact_pos(const int32_t* pos_p, int pos0) {
  return (pos_p ? *pos_p : pos0) + (int)blockIdx.y;
}

// Scores of work item (kv head g, chunk c): grid (nkv * nch, ntok), 256 threads;
// dynamic shared memory: GS * 128 + ceil(cap / nch) * GS floats.
template <int GS, class KT>
__global__ void __launch_bounds__(kAttnExThreads)
k_attn_sc(const float* __restrict__ q, size_t q_tok, const KT* __restrict__ kc,
          const float* __restrict__ scale_p, const int32_t* __restrict__ pos_p, int pos0,
          int cap, int nch, int runs, int nq, float* __restrict__ scr, size_t scr_tok) {
  extern __shared__ __align__(16) float fsm[];
  float* q_s = fsm;
  float* lg_s = q_s + GS * kHd;
  const int g = blockIdx.x / nch, c = blockIdx.x % nch;
  const int pos = exact_pos(pos_p, pos0);
  if (pos < 0 || pos >= cap) return;             // k_attn_cx reports it
  const int T = pos + 1;
  int t0, t1;
  chunk_bounds(T, nch, c, &t0, &t1);
  const float* qg = q + (size_t)blockIdx.y * q_tok + (size_t)g * GS * kHd;
  for (int e = threadIdx.x; e < GS * kHd; e += blockDim.x) q_s[e] = qg[e];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7, r = lane >> 3;
  const float scale = *scale_p;
  const KT* kh = kc + (size_t)g * cap * kHd;
  __shared__ BlasRuns br;
  if (threadIdx.x == 0) blas_runs(T, runs, &br);
  __syncthreads();
  constexpr int HP = GS < 4 ? GS : 4;
#pragma unroll 1
  for (int p0 = 0; p0 < GS; p0 += HP) {
    float qr[HP][16];
    load_qregs<HP>(q_s + p0 * kHd, j, qr);
    for (int tb = t0 + 4 * warp; tb < t1; tb += 4 * (kAttnExThreads / 32)) {
      const int t = tb + r;
      const bool ok = t < t1;
      const int kind = ok ? blas_kind_of(br, t) : 0;
      float d[HP];
      rowdots_blas<HP>(GlobalRow<KT>{kh + (size_t)(ok ? t : t0) * kHd}, kind, qr, q_s + p0 * kHd,
                       j, d);
      float v = d[0];
#pragma unroll
      for (int h = 1; h < HP; ++h) v = (j == h) ? d[h] : v;
      if (ok && j < HP) lg_s[(t - t0) * GS + p0 + j] = __fmul_rn(v, scale);
    }
  }
  __syncthreads();
  float* lg = scr + (size_t)blockIdx.y * scr_tok;
  float* cm = lg + (size_t)nq * cap;
  const int n = t1 - t0;
  for (int i = warp; i < GS; i += kAttnExThreads / 32) {
    const int h = g * GS + i;
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) {
      const float s = lg_s[t * GS + i];
      m = fmaxf(m, s);
      lg[(size_t)h * cap + t0 + t] = s;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) cm[(size_t)h * nch + c] = m;
  }
}

// Shared memory of k_attn_cx (bytes).
template <int GS>
constexpr size_t attn_cx_smem() {
  return ((sizeof(PwTree) + 15) / 16) * 16 +
         sizeof(float) * ((size_t)GS * kTreeMaxNode + (size_t)(kAttnExThreads / 32) * kChainChunk +
                          2 * GS);
}

// Context of work item (kv head g, 32-dim slice jsl) for its GS query heads: grid
// (nkv * 4, ntok), 256 threads. The maximum, the pairwise sum of the exps (head i's leaves
// over the warps w = i mod GS), the fold and the chain (warp i, lane d -> dim 32 jsl + d).
// An out-of-range position leaves NaN in ctx.
template <int GS, class KT>
__global__ void __launch_bounds__(kAttnExThreads)
k_attn_cx(const KT* __restrict__ vc, float* __restrict__ ctx, size_t ctx_tok,
          const int32_t* __restrict__ pos_p, int pos0, int cap, int nch, int nq,
          const float* __restrict__ scr, size_t scr_tok) {
  extern __shared__ __align__(16) unsigned char csm[];
  PwTree& tree = *reinterpret_cast<PwTree*>(csm);
  float* vals = reinterpret_cast<float*>(csm + ((sizeof(PwTree) + 15) / 16) * 16);
  float* wbuf = vals + GS * kTreeMaxNode;
  float* ms = wbuf + (kAttnExThreads / 32) * kChainChunk;   // M, S per head
  __shared__ int ok_s;
  const int g = blockIdx.x / kSlices, jsl = blockIdx.x % kSlices;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = exact_pos(pos_p, pos0);
  float* cx = ctx + (size_t)blockIdx.y * ctx_tok + (size_t)g * GS * kHd + jsl * 32;
  if (warp == 0) {
    const bool built = pos >= 0 && pos < cap && pw_tree_build_warp(pos + 1, &tree);
    if (lane == 0) ok_s = built;
  }
  __syncthreads();
  if (!ok_s) {
    if (warp < GS) cx[warp * kHd + lane] = __int_as_float(0x7fc00000);
    return;
  }
  const int T = pos + 1;
  const float* lg = scr + (size_t)blockIdx.y * scr_tok;
  const float* cm = lg + (size_t)nq * cap;
  for (int i = warp; i < GS; i += kAttnExThreads / 32) {
    float m = -INFINITY;
    for (int c = lane; c < nch; c += 32) m = fmaxf(m, __ldcg(cm + (size_t)(g * GS + i) * nch + c));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (lane == 0) ms[2 * i] = m;
  }
  __syncthreads();
  {
    // leaves: head i's 8-lane groups are those of the warps w = i (mod GS)
    const int i = warp % GS;
    const int gi = (warp / GS) * 4 + (lane >> 3), ng = (kAttnExThreads / 32 / GS) * 4;
    const float* lgh = lg + (size_t)(g * GS + i) * cap;
    const float M = ms[2 * i];
    for (int l0 = 0; l0 < tree.nleaf; l0 += ng) {
      const int l = l0 + gi;
      const bool live = l < tree.nleaf;
      const int id = live ? (int)tree.leaf[l] : 0;
      const float v = leaf_exp_sum(lgh, M, nullptr, live ? (int)tree.start[id] : 0,
                                   live ? (int)tree.size[id] : 1, lane & 7);
      if (live && (lane & 7) == 0) vals[(size_t)i * kTreeMaxNode + id] = v;
    }
  }
  __syncthreads();
  if (warp >= GS) return;
  const int i = warp;
  const float S = pw_tree_fold(&tree, vals + (size_t)i * kTreeMaxNode);
  const float M = ms[2 * i];
  const float* lgh = lg + (size_t)(g * GS + i) * cap;
  const KT* vh = vc + (size_t)g * cap * kHd + jsl * 32 + lane;
  float* wb = wbuf + warp * kChainChunk;
  float acc = 0.0f;
  for (int c0 = 0; c0 < T; c0 += kChainChunk) {
    chain_weights(lgh, c0, T, M, S, wb);
    const int n = min(kChainChunk, T - c0);
    for (int k = 0; k < n; k += 32) {
      float v[32];
#pragma unroll
      for (int r = 0; r < 32; ++r) {
        const int t = c0 + k + r;
        v[r] = t < T ? kv_elem(vh + (size_t)t * kHd) : 0.0f;
      }
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (k + r < n) acc = __fadd_rn(acc, __fmul_rn(wb[k + r], v[r]));
    }
    __syncwarp();
  }
  cx[i * kHd + lane] = acc;
}

}  // namespace hv
