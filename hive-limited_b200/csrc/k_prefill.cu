// Prompt prefill: the W4A8 projections of many tokens at once.
//
// The reference prefills a prompt by running its decode step once per token
// (engine/limited.py:455-462), so every weight byte is read once per prompt token. Here
// the projections of T tokens are one GEMM over the engine's tile-interleaved weights.
// Each token's output is bit-identical to hv_a4gv_pp on that token alone: the same exact
// int32 block dots, the same f32 combine f32(f32(sw * sa) * f32(idot)), the same numpy
// pairwise order (eight strided accumulators per leaf, the ((r0+r1)+(r2+r3))+((r4+r5)+
// (r6+r7)) fold, the recursion's postfix '+', then (+0) + ...).
//
// Mapping onto mma.sync.m16n8k32 (u8 x s8 -> s32), lane = 4 g + t:
//   * A (16 x 32): rows 0..7 are the 8 rows of weight tile 2p at block b, rows 8..15 the
//     8 rows of tile 2p + 1 at the same block. k is permuted as in the decode GEMV, so
//     lane (g, t)'s A registers are the low / high nibbles of packed word t of block b of
//     row g of each tile -- exactly the words the tile-interleaved layout gives lane L.
//   * B (32 x 8): column n is token 8 q + n's int8 activation block b (lane (g, t) holds
//     bytes 8t .. 8t+7 of token 8 q + g's block).
//   * D: lane (g, t) gets the dots of rows g of both tiles with tokens 8 q + 2t and
//     8 q + 2t + 1 -- four (row, token) pairs, whose eight pairwise accumulators per leaf
//     it keeps in registers, so a leaf folds without shuffles.
// Every block's dot is its own MMA (a block's idot must stay separate for the per-block
// scale), so the f32 combine, not the MMA, is the cost: 4 combines per lane per MMA.
//
// A CTA is 8 warps: 2 tile pairs (32 weight rows) x 4 token groups (32 tokens). No CTA
// barrier: warps of the same tile pair share the weights through L1.
#include <cuda_fp16.h>

#include "attn_decode.cuh"
#include "gemv_mma.cuh"
#include "hv_internal.h"

namespace hv {
namespace {

constexpr int kPfMaxBlocks = 1024;   // K <= 32768

HV_DEV float pf_fold8(const float (&r)[8]) {
  return __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                   __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
}

HV_DEV float pf_term(float sw, float sa, int d, int bsum) {
  return __fmul_rn(__fmul_rn(sw, sa), i2f_exact(d - 8 * bsum));
}

// kDq: the weights are in the dq arrangement (hv_w4_prepack_dq): lane (g, t) loads word t
// of each block j of row g from where that arrangement keeps it, as single words.
template <bool kDq>
__global__ void __launch_bounds__(256) k_a4gemm_pp(const int8_t* __restrict__ a8,
                                                   const float* __restrict__ sa,
                                                   const uint32_t* __restrict__ pb4,
                                                   const float* __restrict__ psw,
                                                   float* __restrict__ dst, int ntok,
                                                   int rows, int pair_ffn,
                                                   const __grid_constant__ GvPlan plan) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const int nb = plan.nb, niter = plan.nfull, k = nb * kBlock;
  const int ntile = pp_tiles(rows, pair_ffn);
  const int tile_a = 2 * (blockIdx.x * 2 + (warp & 1));
  const int tq = blockIdx.y * 4 + (warp >> 1);          // tokens 8 tq .. 8 tq + 7
  if (tile_a >= ntile || tq * 8 >= ntok) return;      // whole warps; no CTA barrier below
  const bool has_b = tile_a + 1 < ntile;
  const int tile_b = has_b ? tile_a + 1 : tile_a;       // a missing tile is computed, not stored
  const int tok_col = min(tq * 8 + g, ntok - 1);         // B column of this lane
  const int n0 = tq * 8 + 2 * t, n1 = n0 + 1;           // D columns of this lane
  const int8_t* act = a8 + (size_t)tok_col * k + 8 * t;
  const float* sa0 = sa + (size_t)min(n0, ntok - 1) * 2 * nb;
  const float* sa1 = sa + (size_t)min(n1, ntok - 1) * 2 * nb;
  const uint32_t* wa = pb4 + (size_t)tile_a * niter * kPpNibWords + (kDq ? 16 * g + t : 4 * lane);
  const uint32_t* wb = pb4 + (size_t)tile_b * niter * kPpNibWords + (kDq ? 16 * g + t : 4 * lane);
  const float* sca = psw + (size_t)tile_a * niter * kPpScales + 8 * g;
  const float* scb = psw + (size_t)tile_b * niter * kPpScales + 8 * g;

  float r[4][8];        // accumulators of (row A, n0), (A, n1), (B, n0), (B, n1)
  float st[4][8];       // fold stacks (postfix '+' of numpy's recursion)
  int sp = 0, leaf = 0, leaf_begin = 0;
  for (int it = 0; it < niter; ++it) {
    const size_t wo = (size_t)it * kPpNibWords, so = (size_t)it * kPpScales;
    unsigned wA[8], wB[8];
    if constexpr (kDq) {
      // word t of block j at (j & 1) * 128 + 4 (4 g + j / 2) + t
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        wA[j] = __ldg(wa + wo + (j & 1) * 128 + 4 * (j >> 1));
        wB[j] = __ldg(wb + wo + (j & 1) * 128 + 4 * (j >> 1));
      }
    } else {
      const uint4 a_lo = __ldg(reinterpret_cast<const uint4*>(wa + wo));
      const uint4 a_hi = __ldg(reinterpret_cast<const uint4*>(wa + wo + 128));
      const uint4 b_lo = __ldg(reinterpret_cast<const uint4*>(wb + wo));
      const uint4 b_hi = __ldg(reinterpret_cast<const uint4*>(wb + wo + 128));
      wA[0] = a_lo.x; wA[1] = a_lo.y; wA[2] = a_lo.z; wA[3] = a_lo.w;
      wA[4] = a_hi.x; wA[5] = a_hi.y; wA[6] = a_hi.z; wA[7] = a_hi.w;
      wB[0] = b_lo.x; wB[1] = b_lo.y; wB[2] = b_lo.z; wB[3] = b_lo.w;
      wB[4] = b_hi.x; wB[5] = b_hi.y; wB[6] = b_hi.z; wB[7] = b_hi.w;
    }
    const float4 sA0 = __ldg(reinterpret_cast<const float4*>(sca + so));
    const float4 sA1 = __ldg(reinterpret_cast<const float4*>(sca + so + 4));
    const float4 sB0 = __ldg(reinterpret_cast<const float4*>(scb + so));
    const float4 sB1 = __ldg(reinterpret_cast<const float4*>(scb + so + 4));
    const float swA[8] = {sA0.x, sA0.y, sA0.z, sA0.w, sA1.x, sA1.y, sA1.z, sA1.w};
    const float swB[8] = {sB0.x, sB0.y, sB0.z, sB0.w, sB1.x, sB1.y, sB1.z, sB1.w};
    const float4 x00 = __ldg(reinterpret_cast<const float4*>(sa0 + 8 * it));
    const float4 x01 = __ldg(reinterpret_cast<const float4*>(sa0 + 8 * it + 4));
    const int4 y00 = __ldg(reinterpret_cast<const int4*>(sa0 + nb + 8 * it));
    const int4 y01 = __ldg(reinterpret_cast<const int4*>(sa0 + nb + 8 * it + 4));
    const float4 x10 = __ldg(reinterpret_cast<const float4*>(sa1 + 8 * it));
    const float4 x11 = __ldg(reinterpret_cast<const float4*>(sa1 + 8 * it + 4));
    const int4 y10 = __ldg(reinterpret_cast<const int4*>(sa1 + nb + 8 * it));
    const int4 y11 = __ldg(reinterpret_cast<const int4*>(sa1 + nb + 8 * it + 4));
    const float s0[8] = {x00.x, x00.y, x00.z, x00.w, x01.x, x01.y, x01.z, x01.w};
    const int q0[8] = {y00.x, y00.y, y00.z, y00.w, y01.x, y01.y, y01.z, y01.w};
    const float s1[8] = {x10.x, x10.y, x10.z, x10.w, x11.x, x11.y, x11.z, x11.w};
    const int q1[8] = {y10.x, y10.y, y10.z, y10.w, y11.x, y11.y, y11.z, y11.w};
    uint2 bw[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      bw[j] = __ldg(reinterpret_cast<const uint2*>(act + (size_t)(it * 8 + j) * kBlock));
    const bool first = it == leaf_begin;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int d0, d1, d2, d3;
      mma_u8s8(nib_lo(wA[j]), nib_lo(wB[j]), nib_hi(wA[j]), nib_hi(wB[j]), bw[j].x, bw[j].y,
               d0, d1, d2, d3);
      const float c[4] = {pf_term(swA[j], s0[j], d0, q0[j]), pf_term(swA[j], s1[j], d1, q1[j]),
                          pf_term(swB[j], s0[j], d2, q0[j]), pf_term(swB[j], s1[j], d3, q1[j])};
#pragma unroll
      for (int p = 0; p < 4; ++p) r[p][j] = first ? c[p] : __fadd_rn(r[p][j], c[p]);
    }
    if (it + 1 == plan.it_end[leaf]) {                // a leaf ends: fold, push, close
#pragma unroll
      for (int p = 0; p < 4; ++p) st[p][sp] = pf_fold8(r[p]);
      ++sp;
      for (int c = 0; c < plan.pops[leaf]; ++c) {
        --sp;
#pragma unroll
        for (int p = 0; p < 4; ++p) st[p][sp - 1] = __fadd_rn(st[p][sp - 1], st[p][sp]);
      }
      ++leaf;
      leaf_begin = it + 1;
    }
  }
  bool ok_a, ok_b;
  const int row_a = pp_row(tile_a, g, rows, pair_ffn, &ok_a);
  const int row_b = pp_row(tile_b, g, rows, pair_ffn, &ok_b);
  ok_b = ok_b && has_b;
  if (n0 < ntok) {
    if (ok_a) dst[(size_t)n0 * rows + row_a] = __fadd_rn(0.0f, st[0][0]);
    if (ok_b) dst[(size_t)n0 * rows + row_b] = __fadd_rn(0.0f, st[2][0]);
  }
  if (n1 < ntok) {
    if (ok_a) dst[(size_t)n1 * rows + row_a] = __fadd_rn(0.0f, st[1][0]);
    if (ok_b) dst[(size_t)n1 * rows + row_b] = __fadd_rn(0.0f, st[3][0]);
  }
}

// ---- the per-token steps around the GEMMs, for a run of prompt tokens ----------------
//
// Each kernel applies to every row (token) exactly the arithmetic of the one-token kernel
// the eager step uses, so a batched prefill reproduces the eager per-token prefill bit
// for bit.

// h[t] = f32(emb16[tok[t]]) (gather_emb per token).
__global__ void k_gather_rows(const __half* __restrict__ emb, const int32_t* __restrict__ tok,
                              float* __restrict__ h, int hid) {
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < hid) h[(size_t)t * hid + i] = __half2float(emb[(size_t)tok[t] * hid + i]);
}

// quant_a8s per row: one warp per (row, 32-block); row t's scales and block sums go to
// sa[t][0 .. nb) and sa[t][nb .. 2 nb).
__global__ void __launch_bounds__(256) k_qa8s_rows(const float* __restrict__ src,
                                                   int8_t* __restrict__ a8,
                                                   float* __restrict__ sa, int nb, int ntok) {
  const long long wi = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (wi >= (long long)ntok * nb) return;                 // whole warps
  const int t = (int)(wi / nb), b = (int)(wi % nb);
  const size_t e = ((size_t)t * nb + b) * kBlock + lane;
  int8_t q;
  float s;
  int bs;
  quant_block_warp(src[e], lane, &q, &s, &bs);
  a8[e] = q;
  if (lane == 0) {
    sa[(size_t)t * 2 * nb + b] = s;
    sa[(size_t)t * 2 * nb + nb + b] = __int_as_float(bs);
  }
}

// q/k RMSNorm and RoPE at position pos0 + t, K and V rows appended to the cache: one warp
// per (token, head) over the nq query heads and the nkv key heads (whose warp also
// copies the head's V row). qkv rows are [q | k | v] as the qkv projection writes them.
// KT: the cache's element type (float; __half for the compressed-KV lane, whose rows are
// rounded as hv_kv_append_f16 rounds them).
template <class KT>
__global__ void __launch_bounds__(256) k_qk_rows(const float* __restrict__ qkv,
                                                 const float* __restrict__ qn,
                                                 const float* __restrict__ kn,
                                                 const float* __restrict__ cos_t,
                                                 const float* __restrict__ sin_t, int pos0,
                                                 float* __restrict__ q_out, KT* kc,
                                                 KT* vc, int nq, int nkv, int cap,
                                                 float eps, int ntok) {
  __shared__ __align__(16) float tmp[8][kHd];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = nq + nkv;
  const long long wi = (long long)blockIdx.x * 8 + warp;
  if (wi >= (long long)ntok * heads) return;              // whole warps
  const int t = (int)(wi / heads), h = (int)(wi % heads);
  const int pos = pos0 + t;
  const float* row = qkv + (size_t)t * (nq + 2 * nkv) * kHd;
  const float* cs = cos_t + (size_t)pos * (kHd / 2);
  const float* sn = sin_t + (size_t)pos * (kHd / 2);
  if (h < nq) {
    warp_norm_rope(row + (size_t)h * kHd, qn, cs, sn, eps, tmp[warp],
                   q_out + ((size_t)t * nq + h) * kHd);
  } else if constexpr (!kKvHalf<KT>) {
    const int g = h - nq;
    warp_norm_rope(row + (size_t)(nq + g) * kHd, kn, cs, sn, eps, tmp[warp],
                   kc + ((size_t)g * cap + pos) * kHd);
    reinterpret_cast<float4*>(vc + ((size_t)g * cap + pos) * kHd)[lane] =
        reinterpret_cast<const float4*>(row + (size_t)(nq + nkv + g) * kHd)[lane];
  } else {
    __shared__ __align__(16) float krow[8][kHd];
    const int g = h - nq;
    warp_norm_rope(row + (size_t)(nq + g) * kHd, kn, cs, sn, eps, tmp[warp], krow[warp]);
    const float4 k4 = reinterpret_cast<const float4*>(krow[warp])[lane];
    const float4 v4 = reinterpret_cast<const float4*>(row + (size_t)(nq + nkv + g) * kHd)[lane];
    const size_t at = ((size_t)g * cap + pos) * kHd + 4 * lane;
    reinterpret_cast<__half2*>(kc + at)[0] = __floats2half2_rn(k4.x, k4.y);
    reinterpret_cast<__half2*>(kc + at)[1] = __floats2half2_rn(k4.z, k4.w);
    reinterpret_cast<__half2*>(vc + at)[0] = __floats2half2_rn(v4.x, v4.y);
    reinterpret_cast<__half2*>(vc + at)[1] = __floats2half2_rn(v4.z, v4.w);
  }
}

// act[t] = silu(gate[t]) * up[t] for rows [gate | up] of 2 ffn values (gpu_silu_mul).
__global__ void k_silu_rows(const float* __restrict__ gu, float* __restrict__ act, int ffn) {
  const int t = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < ffn)
    act[(size_t)t * ffn + i] = silu_mul1(gu[(size_t)t * 2 * ffn + i],
                                         gu[(size_t)t * 2 * ffn + ffn + i]);
}

// hv_qk_rows and hv_qk_rows_f16.
template <class KT>
int qk_rows_any(const char* name, const float* qkv, const float* qn, const float* kn,
                const float* cos_t, const float* sin_t, int pos0, float* q_out, KT* kc, KT* vc,
                int nq, int nkv, int hd, int cap, float eps, int ntok, void* stream) {
  HV_REQUIRE(qkv && qn && kn && cos_t && sin_t && q_out && kc && vc && nq > 0 && nkv > 0 &&
                 ntok > 0 && pos0 >= 0,
             HV_E_INVALID, "%s: bad arguments", name);
  HV_REQUIRE(hd == kHd, HV_E_UNSUPPORTED, "%s: head_dim %d (only 128)", name, hd);
  HV_REQUIRE((long long)pos0 + ntok <= cap, HV_E_INVALID,
             "%s: positions %d .. %d outside the cache of %d", name, pos0, pos0 + ntok - 1, cap);
  HV_REQUIRE(((uintptr_t)qkv & 15) == 0 && ((uintptr_t)kc & 15) == 0 &&
                 ((uintptr_t)vc & 15) == 0,
             HV_E_INVALID, "%s: unaligned pointer", name);
  const long long warps = (long long)(nq + nkv) * ntok;
  k_qk_rows<KT><<<(unsigned)((warps + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      qkv, qn, kn, cos_t, sin_t, pos0, q_out, kc, vc, nq, nkv, cap, eps, ntok);
  HV_LAUNCHED("k_qk_rows");
}

// hv_attn_rows and hv_attn_rows_f16: the reference-order attention of hv_attn_decode,
// one query token per grid row, each at its own position pos0 + t.
int attn_rows_any(const char* name, bool kv_half, const float* q, const void* kc,
                  const void* vc, float* ctx, const float* scale, int pos0, int nq, int hd,
                  int group, int kvstride, int ntok, float* part, void* stream) {
  HV_REQUIRE(q && kc && vc && ctx && scale && part && nq > 0 && group > 0 && ntok > 0 &&
                 ntok <= 65535 && pos0 >= 0,
             HV_E_INVALID, "%s: bad arguments", name);
  HV_REQUIRE(hd == kHd, HV_E_UNSUPPORTED, "%s: head_dim %d (only 128)", name, hd);
  HV_REQUIRE(nq % group == 0 && kvstride % hd == 0, HV_E_INVALID,
             "%s: nq %% group or kvstride %% hd is not zero", name);
  HV_REQUIRE(group == 1 || group == 2 || group == 4 || group == 8, HV_E_UNSUPPORTED,
             "%s: group size %d (1, 2, 4 or 8)", name, group);
  const int cap = kvstride / hd;
  HV_REQUIRE((long long)pos0 + ntok <= cap, HV_E_INVALID,
             "%s: positions %d .. %d outside the cache of %d", name, pos0, pos0 + ntok - 1, cap);
  int nch = 0;
  const int rc = attn_exact_chunks(nq / group, cap, &nch);
  if (rc) return rc;
  return attn_exact_launch(group, kv_half, q, (size_t)nq * kHd, kc, vc, ctx, (size_t)nq * kHd,
                           scale, nullptr, pos0, nq, cap, nch, ntok, part,
                           attn_exact_scratch_floats(nq, cap, nch), (cudaStream_t)stream);
}

}  // namespace
}  // namespace hv

using namespace hv;

extern "C" int hv_gather_rows(const uint16_t* emb16, const int32_t* tok, float* h, int hid,
                              int ntok, void* stream) {
  HV_REQUIRE(emb16 && tok && h && hid > 0 && ntok > 0 && ntok <= 65535, HV_E_INVALID,
             "hv_gather_rows: bad arguments");
  k_gather_rows<<<dim3((unsigned)((hid + 255) / 256), (unsigned)ntok), 256, 0,
                  (cudaStream_t)stream>>>(reinterpret_cast<const __half*>(emb16), tok, h, hid);
  HV_LAUNCHED("k_gather_rows");
}

extern "C" int hv_qa8s_rows(const float* src, int8_t* a8, float* sa, int nb, int ntok,
                            void* stream) {
  HV_REQUIRE(src && a8 && sa && nb > 0 && ntok > 0, HV_E_INVALID, "hv_qa8s_rows: bad arguments");
  const long long warps = (long long)nb * ntok;
  HV_REQUIRE((warps + 7) / 8 <= 0x7FFFFFFFll, HV_E_UNSUPPORTED, "hv_qa8s_rows: too many rows");
  k_qa8s_rows<<<(unsigned)((warps + 7) / 8), 256, 0, (cudaStream_t)stream>>>(src, a8, sa, nb,
                                                                              ntok);
  HV_LAUNCHED("k_qa8s_rows");
}

extern "C" int hv_qk_rows(const float* qkv, const float* qn, const float* kn,
                          const float* cos_t, const float* sin_t, int pos0, float* q_out,
                          float* kc, float* vc, int nq, int nkv, int hd, int cap, float eps,
                          int ntok, void* stream) {
  return qk_rows_any("hv_qk_rows", qkv, qn, kn, cos_t, sin_t, pos0, q_out, kc, vc, nq, nkv, hd,
                     cap, eps, ntok, stream);
}

extern "C" int hv_qk_rows_f16(const float* qkv, const float* qn, const float* kn,
                              const float* cos_t, const float* sin_t, int pos0, float* q_out,
                              uint16_t* kc, uint16_t* vc, int nq, int nkv, int hd, int cap,
                              float eps, int ntok, void* stream) {
  return qk_rows_any("hv_qk_rows_f16", qkv, qn, kn, cos_t, sin_t, pos0, q_out,
                     reinterpret_cast<__half*>(kc), reinterpret_cast<__half*>(vc), nq, nkv, hd,
                     cap, eps, ntok, stream);
}

extern "C" int hv_attn_rows_scratch(int nq, int group, int cap, int ntok, size_t* part_bytes,
                                    size_t* ticket_bytes) {
  HV_REQUIRE(nq > 0 && group > 0 && nq % group == 0 && cap > 0 && ntok > 0 && part_bytes &&
                 ticket_bytes,
             HV_E_INVALID, "hv_attn_rows_scratch: bad arguments");
  int nch = 0;
  const int rc = attn_exact_chunks(nq / group, cap, &nch);
  if (rc) return rc;
  *part_bytes = (size_t)ntok * attn_exact_scratch_floats(nq, cap, nch) * sizeof(float);
  *ticket_bytes = sizeof(int);   // not used any more; kept for the entry point's signature
  return HV_OK;
}

extern "C" int hv_attn_rows(const float* q, const float* kc, const float* vc, float* ctx,
                            const float* scale, int pos0, int nq, int hd, int group,
                            int kvstride, int ntok, float* part, int32_t* ticket,
                            void* stream) {
  (void)ticket;
  return attn_rows_any("hv_attn_rows", false, q, kc, vc, ctx, scale, pos0, nq, hd, group,
                       kvstride, ntok, part, stream);
}

extern "C" int hv_attn_rows_f16(const float* q, const uint16_t* kc, const uint16_t* vc,
                                float* ctx, const float* scale, int pos0, int nq, int hd,
                                int group, int kvstride, int ntok, float* part,
                                int32_t* ticket, void* stream) {
  (void)ticket;
  return attn_rows_any("hv_attn_rows_f16", true, q, kc, vc, ctx, scale, pos0, nq, hd, group,
                       kvstride, ntok, part, stream);
}

extern "C" int hv_silu_rows(const float* gu, float* act, int ffn, int ntok, void* stream) {
  HV_REQUIRE(gu && act && ffn > 0 && ntok > 0 && ntok <= 65535, HV_E_INVALID,
             "hv_silu_rows: bad arguments");
  k_silu_rows<<<dim3((unsigned)((ffn + 255) / 256), (unsigned)ntok), 256, 0,
                (cudaStream_t)stream>>>(gu, act, ffn);
  HV_LAUNCHED("k_silu_rows");
}

template <bool kDq>
int a4gemm_any(const char* name, const int8_t* a8, const float* sa, const uint32_t* pb4,
               const float* psw, float* dst, int k8, int rows, int pair_ffn, int ntok,
               void* stream) {
  HV_REQUIRE(a8 && sa && pb4 && psw && dst && k8 > 0 && rows > 0 && ntok > 0, HV_E_INVALID,
             "%s: bad arguments", name);
  HV_REQUIRE(pair_ffn == 0 || rows == 2 * pair_ffn, HV_E_INVALID,
             "%s: a paired matrix has 2 * pair_ffn rows", name);
  HV_REQUIRE(k8 % 32 == 0, HV_E_UNSUPPORTED,
             "%s: K = %d is not a multiple of 256 (whole 8-block iterations)", name, k8 * 8);
  const int nb = k8 / 4;
  HV_REQUIRE(nb <= kPfMaxBlocks, HV_E_UNSUPPORTED, "%s: K = %d exceeds %d", name, k8 * 8,
             kPfMaxBlocks * kBlock);
  HV_REQUIRE(((uintptr_t)a8 & 15) == 0 && ((uintptr_t)sa & 15) == 0 &&
                 ((uintptr_t)pb4 & 15) == 0 && ((uintptr_t)psw & 15) == 0,
             HV_E_INVALID, "%s: unaligned pointer", name);
  GvPlan plan;
  HV_REQUIRE(gv_make_plan(nb, &plan) && plan.ntail == 0, HV_E_UNSUPPORTED,
             "%s: no reduction plan for K", name);
  int depth = 0, maxd = 0;
  for (int l = 0; l < plan.nleaf; ++l) {
    ++depth;
    maxd = depth > maxd ? depth : maxd;
    depth -= plan.pops[l];
  }
  HV_REQUIRE(maxd <= 8, HV_E_UNSUPPORTED, "%s: reduction stack deeper than 8", name);
  const int ntile = pp_tiles(rows, pair_ffn);
  const dim3 grid((unsigned)((ntile + 3) / 4), (unsigned)((ntok + 31) / 32));
  HV_REQUIRE(grid.y <= 65535u, HV_E_UNSUPPORTED, "%s: %d tokens at once", name, ntok);
  k_a4gemm_pp<kDq><<<grid, 256, 0, (cudaStream_t)stream>>>(a8, sa, pb4, psw, dst, ntok, rows,
                                                           pair_ffn, plan);
  HV_LAUNCHED("k_a4gemm_pp");
}

extern "C" int hv_a4gemm_pp(const int8_t* a8, const float* sa, const uint32_t* pb4,
                            const float* psw, float* dst, int k8, int rows, int pair_ffn,
                            int ntok, void* stream) {
  return a4gemm_any<false>("hv_a4gemm_pp", a8, sa, pb4, psw, dst, k8, rows, pair_ffn, ntok,
                           stream);
}

extern "C" int hv_a4gemm_dq(const int8_t* a8, const float* sa, const uint32_t* pb4,
                            const float* psw, float* dst, int k8, int rows, int pair_ffn,
                            int ntok, void* stream) {
  return a4gemm_any<true>("hv_a4gemm_dq", a8, sa, pb4, psw, dst, k8, rows, pair_ffn, ntok,
                          stream);
}
