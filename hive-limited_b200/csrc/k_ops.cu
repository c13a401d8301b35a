// Standalone kernels: one per HIVE Limited PTX entry point (engine/limited.py:173-181),
// with the reference's argument meaning. The decode engine's fast path fuses these into
// one persistent kernel (k_step.cu); these serve the eager path, the C ABI and the
// parity tests.
#include <mutex>

#include <cuda_fp16.h>

#include "attn_exact.cuh"
#include "gemv_mma.cuh"
#include "hv_internal.h"
#include "hv_wait.cuh"

namespace hv {

// hv_a4gv_pp sends matrices of few tiles to the iteration-split kernel (k_a4gv_pps);
// hv_gemv_set_split(0) keeps every matrix on k_a4gv_pp. Results are identical.
static int g_gemv_split = 1;

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device, size).
static std::mutex g_attr_mu;
static int smem_attr(const void* fn, size_t bytes) {
  static const void* fns[64];
  static size_t done[64][16];
  int dev = 0;
  HV_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_attr_mu);
  int slot = -1;
  for (int i = 0; i < 64; ++i) {
    if (fns[i] == fn) { slot = i; break; }
    if (!fns[i]) { fns[i] = fn; slot = i; break; }
  }
  if (slot < 0 || dev >= 16 || done[slot][dev] < bytes) {
    HV_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    if (slot >= 0 && dev < 16) done[slot][dev] = bytes;
  }
  return HV_OK;
}

// ---------------------------------------------------------------------------
// quant_a8s: one warp per 32-block
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_qa8s(const float* __restrict__ src,
                                              int8_t* __restrict__ a8,
                                              float* __restrict__ sa, int nb) {
  const int b = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= nb) return;
  int8_t q;
  float s;
  int bs;
  quant_block_warp(src[b * kBlock + lane], lane, &q, &s, &bs);
  a8[b * kBlock + lane] = q;
  if (lane == 0) {
    sa[b] = s;
    sa[nb + b] = __int_as_float(bs);
  }
}

// ---------------------------------------------------------------------------
// gemv_wpo_a4: a grid of warps, four rows per warp per pass
// ---------------------------------------------------------------------------
template <bool kIdot>
__global__ void __launch_bounds__(256) k_a4gv(const int8_t* __restrict__ a8,
                                              const float* __restrict__ sa,
                                              const uint32_t* __restrict__ b4,
                                              const float* __restrict__ sw,
                                              float* __restrict__ dst,
                                              int32_t* __restrict__ idot, int n,
                                              const __grid_constant__ GvPlan plan) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nb = plan.nb;
  uint4* q_s = reinterpret_cast<uint4*>(smem);
  int2* sb_s = reinterpret_cast<int2*>(smem + (size_t)nb * 32);
  load_act_smem(a8, sa, nb, q_s, sb_s);
  __syncthreads();
  const ActView act{q_s, sb_s};
  const int lane = threadIdx.x & 31;
  const int nquads = (n + 3) / 4;
  const int wpb = blockDim.x >> 5;
  for (int q = blockIdx.x * wpb + (threadIdx.x >> 5); q < nquads; q += gridDim.x * wpb) {
    const int row = q * 4 + (lane >> 3);
    const bool ok = row < n;
    const float y = gemv_rows4<8, kIdot>(b4, sw, row, ok, act, plan, idot);
    if (ok && (lane & 7) == 0) dst[row] = y;
  }
}

// gemv_wpo_a4 on the tensor pipe: one warp per 8-row tile
__global__ void __launch_bounds__(256) k_a4gv_mma(const int8_t* __restrict__ a8,
                                                  const float* __restrict__ sa,
                                                  const uint32_t* __restrict__ b4,
                                                  const float* __restrict__ sw,
                                                  float* __restrict__ dst, int n,
                                                  const __grid_constant__ GvPlan plan) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nb = plan.nb;
  uint4* q_s = reinterpret_cast<uint4*>(smem);
  int2* sb_s = reinterpret_cast<int2*>(smem + (size_t)nb * 32);
  load_act_smem(a8, sa, nb, q_s, sb_s);
  __syncthreads();
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int ntile = (n + 7) / 8;
  const int wpb = blockDim.x >> 5;
  for (int tile = blockIdx.x * wpb + (threadIdx.x >> 5); tile < ntile; tile += gridDim.x * wpb) {
    const int row = tile * 8 + g;
    const bool ok = row < n;
    const int lr = ok ? row : 0;
    float y;
    gemv_tile8<6, true>(b4 + (size_t)lr * nb * 4, sw + (size_t)lr * nb,
                        reinterpret_cast<const unsigned*>(q_s), sb_s, plan, 0, plan.nleaf, &y,
                        nullptr);
    if (t == 0 && ok) dst[row] = y;
  }
}

// ---------------------------------------------------------------------------
// tile-interleaved weight layout (see gemv_mma.cuh) and the GEMV over it
// ---------------------------------------------------------------------------


// one thread per (tile, iteration, lane): 8 nibble words and 2 scales
__global__ void k_w4_prepack(const uint32_t* __restrict__ b4, const float* __restrict__ sw,
                             int rows, int nb, int pair_ffn, int ntile, int niter,
                             uint32_t* __restrict__ pb4, float* __restrict__ psw) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)ntile * niter * 32) return;
  const int lane = (int)(idx & 31);
  const long long rest = idx >> 5;
  const int it = (int)(rest % niter), tile = (int)(rest / niter);
  const int g = lane >> 2, t = lane & 3;
  bool ok;
  const int row = pp_row(tile, g, rows, pair_ffn, &ok);
  uint32_t w[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int blk = it * 8 + j;
    w[j] = (ok && blk < nb) ? b4[((size_t)row * nb + blk) * 4 + t] : 0u;
  }
  uint32_t* dn = pb4 + ((size_t)tile * niter + it) * kPpNibWords;
  reinterpret_cast<uint4*>(dn)[lane] = make_uint4(w[0], w[1], w[2], w[3]);
  reinterpret_cast<uint4*>(dn + 128)[lane] = make_uint4(w[4], w[5], w[6], w[7]);
  const int b0 = it * 8 + 2 * t;
  float* ds = psw + ((size_t)tile * niter + it) * kPpScales;
  ds[2 * lane] = (ok && b0 < nb) ? sw[(size_t)row * nb + b0] : 0.f;
  ds[2 * lane + 1] = (ok && b0 + 1 < nb) ? sw[(size_t)row * nb + b0 + 1] : 0.f;
}

// The dq arrangement of the same tiles (gemv_tile8_dq): lane L = 4g + t of iteration `it`
// gets words 0..3 of blocks 8 it + 2t (at 4L) and 8 it + 2t + 1 (at 128 + 4L) of row g;
// the scales as in k_w4_prepack. Blocks past nb are zero.
__global__ void k_w4_prepack_dq(const uint32_t* __restrict__ b4, const float* __restrict__ sw,
                                int rows, int nb, int pair_ffn, int ntile, int niter,
                                uint32_t* __restrict__ pb4, float* __restrict__ psw) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)ntile * niter * 32) return;
  const int lane = (int)(idx & 31);
  const long long rest = idx >> 5;
  const int it = (int)(rest % niter), tile = (int)(rest / niter);
  const int g = lane >> 2, t = lane & 3;
  bool ok;
  const int row = pp_row(tile, g, rows, pair_ffn, &ok);
  const int be = it * 8 + 2 * t;
  const uint4* src = reinterpret_cast<const uint4*>(b4) + (size_t)row * nb;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  const uint4 e = (ok && be < nb) ? src[be] : zero;
  const uint4 o = (ok && be + 1 < nb) ? src[be + 1] : zero;
  uint32_t* dn = pb4 + ((size_t)tile * niter + it) * kDqNibWords;
  reinterpret_cast<uint4*>(dn)[lane] = e;
  reinterpret_cast<uint4*>(dn + 128)[lane] = o;
  float* ds = psw + ((size_t)tile * niter + it) * kDqScales;
  ds[2 * lane] = (ok && be < nb) ? sw[(size_t)row * nb + be] : 0.f;
  ds[2 * lane + 1] = (ok && be + 1 < nb) ? sw[(size_t)row * nb + be + 1] : 0.f;
}

// GEMV over the dq layout with dp4a block dots, one warp per tile (k_a4gv_pp's schedule);
// results bit-identical to k_a4gv_pp on the same matrix.
__global__ void __launch_bounds__(256) k_a4gv_dq(const int8_t* __restrict__ a8,
                                                 const float* __restrict__ sa,
                                                 const uint32_t* __restrict__ pb4,
                                                 const float* __restrict__ psw,
                                                 float* __restrict__ dst, int rows, int pair_ffn,
                                                 const __grid_constant__ GvPlan plan) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nb = plan.nb;
  uint4* q_s = reinterpret_cast<uint4*>(smem);
  int2* sb_s = reinterpret_cast<int2*>(smem + (size_t)nb * 32);
  load_act_smem(a8, sa, nb, q_s, sb_s);
  __syncthreads();
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int ntile = pp_tiles(rows, pair_ffn), niter = pp_iters(nb);
  const int wpb = blockDim.x >> 5;
  for (int tile = blockIdx.x * wpb + (threadIdx.x >> 5); tile < ntile; tile += gridDim.x * wpb) {
    bool ok;
    const int row = pp_row(tile, g, rows, pair_ffn, &ok);
    const float y = gemv_tile8_dq<8>(pb4 + (size_t)tile * niter * kDqNibWords,
                                     psw + (size_t)tile * niter * kDqScales, q_s, sb_s, plan);
    if (t == 0 && ok) dst[row] = y;
  }
}

// GEMV over the tile-interleaved layout, one warp per tile; with pair_ffn > 0 the output
// keeps the reference order [gate | up].
__global__ void __launch_bounds__(256) k_a4gv_pp(const int8_t* __restrict__ a8,
                                                 const float* __restrict__ sa,
                                                 const uint32_t* __restrict__ pb4,
                                                 const float* __restrict__ psw,
                                                 float* __restrict__ dst, int rows, int pair_ffn,
                                                 const __grid_constant__ GvPlan plan) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nb = plan.nb;
  uint4* q_s = reinterpret_cast<uint4*>(smem);
  int2* sb_s = reinterpret_cast<int2*>(smem + (size_t)nb * 32);
  load_act_smem(a8, sa, nb, q_s, sb_s);
  __syncthreads();
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int ntile = pp_tiles(rows, pair_ffn), niter = pp_iters(nb);
  const int wpb = blockDim.x >> 5;
  for (int tile = blockIdx.x * wpb + (threadIdx.x >> 5); tile < ntile; tile += gridDim.x * wpb) {
    bool ok;
    const int row = pp_row(tile, g, rows, pair_ffn, &ok);
    float y;
    gemv_tile8<8, true, true>(pb4 + (size_t)tile * niter * kPpNibWords,
                              psw + (size_t)tile * niter * kPpScales,
                              reinterpret_cast<const unsigned*>(q_s), sb_s, plan, 0, plan.nleaf,
                              &y, nullptr);
    if (t == 0 && ok) dst[row] = y;
  }
}

// GEMV over the tile-interleaved layout for matrices of few tiles (the small sweep
// shapes, the eager path's layer GEMVs): one CTA per 8-row tile, whose eight warps split
// the tile's iterations (warp w takes iterations w, w + 8, ...), so a 2048-row matrix
// keeps 2048 warps busy instead of 256. Each warp leaves its lanes' two block terms of
// every iteration it owns in shared memory; warp 0 then walks the terms in iteration
// order: the same sequential chains, leaf folds and postfix '+' as gemv_tile8, so the
// result is bit-identical to k_a4gv_pp. Plans with a tail (nb % 8 != 0) use k_a4gv_pp.
constexpr int kSplitMaxIters = 64;    // terms in shared memory: iterations x 256 B
// K = 2048 (8 iterations) measured faster on k_a4gv_pp: 7.6 vs 9.3 us at 2048 x 2048
constexpr int kSplitMinIters = 16;
constexpr int kSplitAhead = 4;        // iterations a warp has in flight

__global__ void __launch_bounds__(256) k_a4gv_pps(const int8_t* __restrict__ a8,
                                                  const float* __restrict__ sa,
                                                  const uint32_t* __restrict__ pb4,
                                                  const float* __restrict__ psw,
                                                  float* __restrict__ dst, int rows,
                                                  int pair_ffn,
                                                  const __grid_constant__ GvPlan plan) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nb = plan.nb, niter = plan.nfull;
  uint4* q_s = reinterpret_cast<uint4*>(smem);
  int2* sb_s = reinterpret_cast<int2*>(smem + (size_t)nb * 32);
  float2* term_s = reinterpret_cast<float2*>(smem + (size_t)nb * 40);   // [niter][32]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const int nw = blockDim.x >> 5;
  const int tile = blockIdx.x;
  const uint32_t* tn = pb4 + (size_t)tile * niter * kPpNibWords;
  const float* ts = psw + (size_t)tile * niter * kPpScales;
  // this warp's weight loads go out before the activation is staged
  MmaLoads L[kSplitAhead];
#pragma unroll
  for (int u = 0; u < kSplitAhead; ++u)
    if (warp + u * nw < niter) mma_load_pp(L[u], tn, ts, warp + u * nw, lane);
  load_act_smem(a8, sa, nb, q_s, sb_s);
  __syncthreads();
  const unsigned* act_w = reinterpret_cast<const unsigned*>(q_s);
  for (int i0 = warp; i0 < niter; i0 += kSplitAhead * nw) {
#pragma unroll
    for (int u = 0; u < kSplitAhead; ++u) {
      const int it = i0 + u * nw;
      if (it < niter) {
        const uint2 bw = reinterpret_cast<const uint2*>(act_w)[(it * 8 + g) * 4 + t];
        int e, o;
        mma_iter(L[u].w, bw, t, 8, e, o);
        const int4 sbb = reinterpret_cast<const int4*>(sb_s)[it * 4 + t];   // blocks 2t, 2t+1
        const float ce = __fmul_rn(__fmul_rn(L[u].s.x, __int_as_float(sbb.x)),
                                   i2f_exact(e - 8 * sbb.y));
        const float co = __fmul_rn(__fmul_rn(L[u].s.y, __int_as_float(sbb.z)),
                                   i2f_exact(o - 8 * sbb.w));
        term_s[it * 32 + lane] = make_float2(ce, co);
        const int itn = it + kSplitAhead * nw;
        if (itn < niter) mma_load_pp(L[u], tn, ts, itn, lane);
      }
    }
  }
  __syncthreads();
  if (warp != 0) return;
  float st[8];                 // fold stack (postfix '+' of numpy's recursion)
  int sp = 0;
  int leaf_begin = 0;
  for (int leaf = 0; leaf < plan.nleaf; ++leaf) {
    const int leaf_end = plan.it_end[leaf];
    float acc_e = 0.f, acc_o = 0.f;             // accumulators 2t, 2t+1 of row g
    for (int it = leaf_begin; it < leaf_end; ++it) {
      const float2 c = term_s[it * 32 + lane];
      if (it == leaf_begin) {
        acc_e = c.x;
        acc_o = c.y;
      } else {
        acc_e = __fadd_rn(acc_e, c.x);
        acc_o = __fadd_rn(acc_o, c.y);
      }
    }
    st[sp++] = (leaf_end > leaf_begin) ? quad_fold(acc_e, acc_o) : 0.f;
    for (int k = 0; k < plan.pops[leaf]; ++k) {
      --sp;
      st[sp - 1] = __fadd_rn(st[sp - 1], st[sp]);
    }
    leaf_begin = leaf_end;
  }
  bool ok;
  const int row = pp_row(tile, g, rows, pair_ffn, &ok);
  if (t == 0 && ok) dst[row] = __fadd_rn(0.0f, st[0]);
}

// ---------------------------------------------------------------------------
// rmsnorm_bp: one CTA per row
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ src,
                                                 float* __restrict__ dst,
                                                 const float* __restrict__ w, int cols,
                                                 float eps, const __grid_constant__ PwPlan plan) {
  extern __shared__ __align__(16) unsigned char smem[];
  float* leafval = reinterpret_cast<float*>(smem);
  float* red = leafval + kPwMaxLeaf;
  float* x = red + 4;
  float* sq = x + cols;
  const float* row = src + (size_t)blockIdx.x * cols;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) {
    const float v = row[i];
    x[i] = v;
    sq[i] = __fmul_rn(v, v);
  }
  __syncthreads();
  const float ss = block_pw_sum(sq, &plan, leafval, red);
  const float ms = __fdiv_rn(ss, (float)cols);
  const float d = __fsqrt_rn(__fadd_rn(ms, eps));
  float* out = dst + (size_t)blockIdx.x * cols;
  for (int i = threadIdx.x; i < cols; i += blockDim.x)
    out[i] = __fmul_rn(w[i], __fdiv_rn(x[i], d));
}

// ---------------------------------------------------------------------------
// rope_pos / kvapp_pos / gpu_silu_mul / vec_add / gather_emb
// ---------------------------------------------------------------------------
__global__ void k_rope(float* __restrict__ vec, const float* __restrict__ cos_t,
                       const float* __restrict__ sin_t, const int32_t* __restrict__ pos,
                       int half) {
  const int p = *pos;
  float* v = vec + (size_t)blockIdx.x * 2 * half;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float c = cos_t[(size_t)p * half + i], s = sin_t[(size_t)p * half + i];
    const float lo = v[i], hi = v[half + i];
    v[i] = __fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s));
    v[half + i] = __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s));
  }
}

__global__ void k_kvapp(const float* __restrict__ k, const float* __restrict__ v,
                        float* __restrict__ kc, float* __restrict__ vc,
                        const int32_t* __restrict__ pos, int hd, int cap) {
  const int p = *pos;
  const int h = blockIdx.x;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    kc[((size_t)h * cap + p) * hd + d] = k[h * hd + d];
    vc[((size_t)h * cap + p) * hd + d] = v[h * hd + d];
  }
}

// The compressed-KV lane's append: each value rounded to the nearest binary16 (ties to
// even, overflow to infinity), the conversion numpy's astype(float16) performs.
__global__ void k_kvapp16(const float* __restrict__ k, const float* __restrict__ v,
                          __half* __restrict__ kc, __half* __restrict__ vc,
                          const int32_t* __restrict__ pos, int hd, int cap) {
  const int p = *pos;
  const int h = blockIdx.x;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    kc[((size_t)h * cap + p) * hd + d] = __float2half_rn(k[h * hd + d]);
    vc[((size_t)h * cap + p) * hd + d] = __float2half_rn(v[h * hd + d]);
  }
}

__global__ void k_silu(const float* __restrict__ g, const float* __restrict__ u,
                       float* __restrict__ act, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) act[i] = silu_mul1(g[i], u[i]);
}

__global__ void k_vadd(const float* __restrict__ a, const float* __restrict__ b,
                       float* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = __fadd_rn(a[i], b[i]);
}

__global__ void k_gather(const __half* __restrict__ emb, const int32_t* __restrict__ tok,
                         float* __restrict__ h, int hid) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < hid) h[i] = __half2float(emb[(size_t)(*tok) * hid + i]);
}

// ---------------------------------------------------------------------------
// argmax_p / argmax_f: first maximal index
// ---------------------------------------------------------------------------
HV_DEV bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

HV_DEV void block_argmax(float* v, int* i, float* sv, int* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xFFFFFFFFu, *v, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, *i, o);
    if (better(ov, oi, *v, *i)) { *v = ov; *i = oi; }
  }
  if (lane == 0) { sv[warp] = *v; si[warp] = *i; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (better(sv[w], si[w], sv[0], si[0])) { sv[0] = sv[w]; si[0] = si[w]; }
  }
  __syncthreads();
  *v = sv[0];
  *i = si[0];
}

__global__ void __launch_bounds__(256) k_argmax_p(const float* __restrict__ logits,
                                                  float* __restrict__ pv,
                                                  int32_t* __restrict__ pi, int n, int parts) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const int lo = (int)(((long long)blockIdx.x * n) / parts);
  const int hi = (int)(((long long)(blockIdx.x + 1) * n) / parts);
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int j = lo + threadIdx.x; j < hi; j += blockDim.x) {
    const float v = logits[j];
    if (better(v, j, bv, bi)) { bv = v; bi = j; }
  }
  block_argmax(&bv, &bi, sv, si);
  if (threadIdx.x == 0) { pv[blockIdx.x] = bv; pi[blockIdx.x] = bi; }
}

__global__ void __launch_bounds__(128) k_argmax_f(const float* __restrict__ pv,
                                                  const int32_t* __restrict__ pi,
                                                  int32_t* tok, int32_t* gen, int32_t* step,
                                                  int32_t* pos, int parts) {
  __shared__ float sv[32];
  __shared__ int si[32];
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int j = threadIdx.x; j < parts; j += blockDim.x)
    if (better(pv[j], pi[j], bv, bi)) { bv = pv[j]; bi = pi[j]; }
  block_argmax(&bv, &bi, sv, si);
  if (threadIdx.x == 0) {
    *tok = bi;
    gen[*step] = bi;
    *step += 1;
    *pos += 1;
  }
}

// ---------------------------------------------------------------------------
// Vocabulary-sharded argmax. Each candidate becomes a 64-bit key whose unsigned order
// is np.argmax's order: high word = the f32 bits mapped to an unsigned total order,
// low word = ~(global id), so equal values rank the lower id higher. -0 counts as +0
// (np compares them equal) and every NaN ranks above +inf (np.argmax returns the first
// NaN). A real key is never 0 (that would need the mapped NaN 0xFFFFFFFF), so 0 is the
// empty key and the cross-shard reduce is a plain unsigned max.
// ---------------------------------------------------------------------------
HV_DEV unsigned long long argmax_key(float v, int id) {
  unsigned u = __float_as_uint(v);
  if (v != v) u = 0x7FC00000u;
  else if (v == 0.f) u = 0u;
  const unsigned ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(~(unsigned)id);
}

HV_DEV unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

__global__ void __launch_bounds__(256) k_argmax_key(const float* __restrict__ logits, int n,
                                                    int base, unsigned long long* key) {
  __shared__ unsigned long long s[8];
  unsigned long long best = 0;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
    best = umax64(best, argmax_key(logits[j], base + j));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
  if ((threadIdx.x & 31) == 0) s[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = umax64(best, s[w]);
    atomicMax(key, best);
  }
}

// One warp: max over the shards' keys, then the device generation state advances as in
// k_argmax_f; the keys are cleared for the next token (each lane clears what it read).
__global__ void __launch_bounds__(32) k_argmax_keyf(unsigned long long* keys, int nkeys,
                                                    int32_t* tok, int32_t* gen,
                                                    int32_t* step, int32_t* pos) {
  unsigned long long best = 0;
  for (int j = threadIdx.x; j < nkeys; j += 32) best = umax64(best, keys[j]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) best = umax64(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
  for (int j = threadIdx.x; j < nkeys; j += 32) keys[j] = 0ull;
  if (threadIdx.x == 0) {
    const int t = best ? (int)(~(unsigned)(best & 0xFFFFFFFFull)) : -1;
    *tok = t;
    gen[*step] = t;
    *step += 1;
    *pos += 1;
  }
}

// One thread: the bounded poll every wait of the fused step uses, on a caller's word.
__global__ void k_wait_probe(const unsigned* word, unsigned mask, unsigned want,
                             unsigned long long limit_ns, int* status) {
  if (threadIdx.x == 0 && blockIdx.x == 0)
    poll_word_until<false>(word, mask, want, status, limit_ns);
}

// ---------------------------------------------------------------------------
// quantize_w4 on the device: one thread per 32-block
// ---------------------------------------------------------------------------
__global__ void k_quantize_w4(const float* __restrict__ w, uint32_t* __restrict__ packed,
                              float* __restrict__ scale, long long nblocks) {
  const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float4* src = reinterpret_cast<const float4*>(w + b * kBlock);
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 t = src[i];
    v[4 * i] = t.x; v[4 * i + 1] = t.y; v[4 * i + 2] = t.z; v[4 * i + 3] = t.w;
  }
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) mx = fmaxf(mx, fabsf(v[i]));
  float s = __fdiv_rn(mx, 7.0f);
  if (s == 0.0f) s = 1.0f;
  uint32_t words[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float r = rintf(__fdiv_rn(v[i], s));
    r = fminf(fmaxf(r, -7.0f), 7.0f);
    const uint32_t nib = (uint32_t)((int)r) & 15u;
    const int word = i / 8, j = i % 8;
    const int shift = (j < 4) ? (8 * j) : (8 * (j - 4) + 4);
    words[word] |= nib << shift;
  }
  reinterpret_cast<uint4*>(packed)[b] = make_uint4(words[0], words[1], words[2], words[3]);
  scale[b] = s;
}

// ---------------------------------------------------------------------------
// decode attention in the reference's order (attn_exact.cuh): a scores kernel over
// (kv head, chunk) items, then a context kernel over (kv head, 32-dim slice) items
// ---------------------------------------------------------------------------

// OpenBLAS threads of the host whose reference results the attention reproduces (the
// row kinds of `keys @ q` depend on it); hv_step_set_option(HV_OPT_REF_BLAS_RUNS).
static int g_ref_runs = kRefRuns;
int ref_blas_runs() { return g_ref_runs; }
int set_ref_blas_runs(int v) {
  HV_REQUIRE(v >= 1 && v <= kMaxRuns, HV_E_INVALID, "reference BLAS runs %d outside [1, %d]",
             v, kMaxRuns);
  g_ref_runs = v;
  return HV_OK;
}

int attn_exact_chunks(int nkv, int cap, int* out) {
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  int nch = (sms + nkv - 1) / nkv;
  const int need = (cap + kAttnChunkMax - 1) / kAttnChunkMax;
  *out = nch > need ? nch : need;
  return HV_OK;
}

size_t attn_exact_scratch_floats(int nq, int cap, int nch) {
  return (size_t)nq * ((size_t)cap + (size_t)nch);
}

template <int GS, class KT>
static int launch_exact(const float* q, size_t q_tok, const KT* kc, const KT* vc, float* ctx,
                        size_t ctx_tok, const float* scale, const int32_t* pos_p, int pos0,
                        int nq, int cap, int nch, int ntok, float* scr, size_t scr_tok,
                        cudaStream_t st) {
  const int nkv = nq / GS;
  const size_t sm1 = sizeof(float) * ((size_t)GS * kHd + (size_t)((cap + nch - 1) / nch) * GS);
  int rc = smem_attr((const void*)k_attn_sc<GS, KT>, sm1);
  if (rc) return rc;
  const size_t sm2 = attn_cx_smem<GS>();
  rc = smem_attr((const void*)k_attn_cx<GS, KT>, sm2);
  if (rc) return rc;
  k_attn_sc<GS, KT><<<dim3(nkv * nch, ntok), kAttnExThreads, sm1, st>>>(
      q, q_tok, kc, scale, pos_p, pos0, cap, nch, g_ref_runs, nq, scr, scr_tok);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail("k_attn_sc", e);
  k_attn_cx<GS, KT><<<dim3(nkv * kSlices, ntok), kAttnExThreads, sm2, st>>>(
      vc, ctx, ctx_tok, pos_p, pos0, cap, nch, nq, scr, scr_tok);
  HV_LAUNCHED("k_attn_cx");
}

int attn_exact_launch(int group, bool kv_half, const float* q, size_t q_tok, const void* kc,
                      const void* vc, float* ctx, size_t ctx_tok, const float* scale,
                      const int32_t* pos_p, int pos0, int nq, int cap, int nch, int ntok,
                      float* scr, size_t scr_tok, cudaStream_t st) {
  HV_REQUIRE(cap <= kExactMaxCap, HV_E_UNSUPPORTED,
             "attention: cache of %d positions (at most %d)", cap, kExactMaxCap);
#define HV_EXACT(G)                                                                          \
  return kv_half ? launch_exact<G>(q, q_tok, static_cast<const __half*>(kc),                 \
                                   static_cast<const __half*>(vc), ctx, ctx_tok, scale,      \
                                   pos_p, pos0, nq, cap, nch, ntok, scr, scr_tok, st)        \
                 : launch_exact<G>(q, q_tok, static_cast<const float*>(kc),                  \
                                   static_cast<const float*>(vc), ctx, ctx_tok, scale,       \
                                   pos_p, pos0, nq, cap, nch, ntok, scr, scr_tok, st)
  switch (group) {
    case 1: HV_EXACT(1);
    case 2: HV_EXACT(2);
    case 4: HV_EXACT(4);
    default: HV_EXACT(8);
  }
#undef HV_EXACT
}

// per-device attention scratch, grown on demand
struct AttnScratch {
  float* buf = nullptr;
  size_t floats = 0;
};
static std::mutex g_attn_mu;
static AttnScratch g_attn[64];

static int attn_scratch(int nq, int cap, int nch, void* stream, AttnScratch** out) {
  int dev = 0;
  HV_CUDA(cudaGetDevice(&dev));
  HV_REQUIRE(dev >= 0 && dev < 64, HV_E_UNSUPPORTED, "device index %d out of range", dev);
  const size_t need = attn_exact_scratch_floats(nq, cap, nch);
  std::lock_guard<std::mutex> lk(g_attn_mu);
  AttnScratch& s = g_attn[dev];
  if (s.floats < need) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (stream) HV_CUDA(cudaStreamIsCapturing((cudaStream_t)stream, &cs));
    HV_REQUIRE(cs == cudaStreamCaptureStatusNone, HV_E_CAPTURE,
               "attention scratch must grow during stream capture; call hv_attn_reserve first");
    if (s.buf) cudaFree(s.buf);
    s.buf = nullptr;
    s.floats = 0;
    HV_CUDA(cudaMalloc(&s.buf, need * sizeof(float)));
    s.floats = need;
  }
  *out = &s;
  return HV_OK;
}

// hv_attn_decode and hv_attn_decode_f16: checks, scratch, chunk count, launch.
static int attn_decode_any(const char* name, bool kv_half, const float* q, const void* kc,
                           const void* vc, float* ctx, const float* scale, const int32_t* pos,
                           int nq, int hd, int group, int kvstride, void* stream) {
  HV_REQUIRE(q && kc && vc && ctx && scale && pos && nq > 0 && group > 0, HV_E_INVALID,
             "%s: bad arguments", name);
  HV_REQUIRE(hd == kHd, HV_E_UNSUPPORTED, "%s: head_dim %d (only 128)", name, hd);
  HV_REQUIRE(nq % group == 0 && kvstride % hd == 0, HV_E_INVALID,
             "%s: nq %% group or kvstride %% hd is not zero", name);
  HV_REQUIRE(group == 1 || group == 2 || group == 4 || group == 8, HV_E_UNSUPPORTED,
             "%s: group size %d (1, 2, 4 or 8)", name, group);
  const int nkv = nq / group, cap = kvstride / hd;
  int nch = 0;
  int rc = attn_exact_chunks(nkv, cap, &nch);
  if (rc) return rc;
  AttnScratch* s = nullptr;
  rc = attn_scratch(nq, cap, nch, stream, &s);
  if (rc) return rc;
  return attn_exact_launch(group, kv_half, q, 0, kc, vc, ctx, 0, scale, pos, 0, nq, cap, nch,
                           1, s->buf, 0, (cudaStream_t)stream);
}

}  // namespace hv

using namespace hv;

extern "C" {

int hv_kernel_list(char* buf, size_t len) {
  static const char* names =
      "k_qa8s,k_a4gv,k_a4gv_mma,k_a4gv_pp,k_a4gv_pps,k_a4gv_dq,k_w4_prepack,k_w4_prepack_dq,k_rmsnorm,k_rope,k_kvapp,k_kvapp16,k_attn_sc,k_attn_cx,k_silu,k_vadd,k_gather,"
      "k_argmax_p,k_argmax_f,k_argmax_key,k_argmax_keyf,k_quantize_w4,k_step,k_wait_probe,k_a4gemm_pp,k_gather_rows,k_qa8s_rows,k_qk_rows,k_silu_rows";
  HV_REQUIRE(buf && len > 0, HV_E_INVALID, "hv_kernel_list: bad buffer");
  strncpy(buf, names, len - 1);
  buf[len - 1] = 0;
  return HV_OK;
}

int hv_qa8s(const float* src, int8_t* a8, float* sa, int nb, void* stream) {
  HV_REQUIRE(src && a8 && sa && nb > 0, HV_E_INVALID, "hv_qa8s: bad arguments");
  k_qa8s<<<(nb + 7) / 8, 256, 0, (cudaStream_t)stream>>>(src, a8, sa, nb);
  HV_LAUNCHED("k_qa8s");
}

static int a4gv_launch(const int8_t* a8, const float* sa, const uint32_t* b4, const float* sw,
                       float* dst, int32_t* idot, int k8, int n, void* stream) {
  HV_REQUIRE(a8 && sa && b4 && sw && dst && k8 > 0 && n > 0, HV_E_INVALID,
             "hv_a4gv: bad arguments");
  HV_REQUIRE(k8 % 4 == 0, HV_E_INVALID, "hv_a4gv: K = %d is not a multiple of 32", k8 * 8);
  HV_REQUIRE(((uintptr_t)a8 & 15) == 0 && ((uintptr_t)b4 & 15) == 0, HV_E_INVALID,
             "hv_a4gv: a8 and b4 must be 16-byte aligned");
  const int nb = k8 / 4;
  HV_REQUIRE(nb <= 4096, HV_E_UNSUPPORTED, "hv_a4gv: K = %d exceeds 131072", k8 * 8);
  const size_t smem = (size_t)nb * 40;
  GvPlan plan;
  HV_REQUIRE(gv_make_plan(nb, &plan), HV_E_UNSUPPORTED, "hv_a4gv: no reduction plan for K");
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  const int nquads = (n + 3) / 4;
  int grid = (nquads + 7) / 8;
  if (grid > sms * 8) grid = sms * 8;
  cudaStream_t st = (cudaStream_t)stream;
  if (idot) {
    rc = smem_attr((const void*)k_a4gv<true>, smem);
    if (rc) return rc;
    k_a4gv<true><<<grid, 256, smem, st>>>(a8, sa, b4, sw, dst, idot, n, plan);
  } else {
    const int ntile = (n + 7) / 8;
    int grid8 = (ntile + 7) / 8;
    if (grid8 > sms * 4) grid8 = sms * 4;
    rc = smem_attr((const void*)k_a4gv_mma, smem);
    if (rc) return rc;
    k_a4gv_mma<<<grid8, 256, smem, st>>>(a8, sa, b4, sw, dst, n, plan);
  }
  HV_LAUNCHED("k_a4gv");
}

int hv_a4gv(const int8_t* a8, const float* sa, const uint32_t* b4, const float* sw,
            float* dst, int k8, int n, void* stream) {
  return a4gv_launch(a8, sa, b4, sw, dst, nullptr, k8, n, stream);
}

int hv_a4gv_idot(const int8_t* a8, const float* sa, const uint32_t* b4, const float* sw,
                 float* dst, int32_t* idot, int k8, int n, void* stream) {
  HV_REQUIRE(idot, HV_E_INVALID, "hv_a4gv_idot: null idot");
  return a4gv_launch(a8, sa, b4, sw, dst, idot, k8, n, stream);
}

int hv_w4_prepacked_size(int rows, int k, int pair_ffn, size_t* nib_bytes, size_t* scale_bytes) {
  HV_REQUIRE(rows > 0 && k > 0 && k % kBlock == 0 && nib_bytes && scale_bytes, HV_E_INVALID,
             "hv_w4_prepacked_size: bad arguments");
  HV_REQUIRE(pair_ffn == 0 || rows == 2 * pair_ffn, HV_E_INVALID,
             "hv_w4_prepacked_size: a paired matrix has 2 * pair_ffn rows");
  const size_t tiles = (size_t)pp_tiles(rows, pair_ffn), iters = (size_t)pp_iters(k / kBlock);
  *nib_bytes = tiles * iters * kPpNibWords * 4;
  *scale_bytes = tiles * iters * kPpScales * 4;
  return HV_OK;
}

int hv_w4_prepack(const uint32_t* b4, const float* sw, int rows, int k, int pair_ffn,
                  uint32_t* pb4, float* psw, void* stream) {
  HV_REQUIRE(b4 && sw && pb4 && psw && rows > 0 && k > 0 && k % kBlock == 0, HV_E_INVALID,
             "hv_w4_prepack: bad arguments");
  HV_REQUIRE(pair_ffn == 0 || rows == 2 * pair_ffn, HV_E_INVALID,
             "hv_w4_prepack: a paired matrix has 2 * pair_ffn rows");
  HV_REQUIRE(((uintptr_t)pb4 & 15) == 0 && ((uintptr_t)psw & 15) == 0, HV_E_INVALID,
             "hv_w4_prepack: outputs must be 16-byte aligned");
  const int nb = k / kBlock;
  const int ntile = pp_tiles(rows, pair_ffn), niter = pp_iters(nb);
  const long long threads = (long long)ntile * niter * 32;
  k_w4_prepack<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      b4, sw, rows, nb, pair_ffn, ntile, niter, pb4, psw);
  HV_LAUNCHED("k_w4_prepack");
}

int hv_a4gv_pp(const int8_t* a8, const float* sa, const uint32_t* pb4, const float* psw,
               float* dst, int k8, int rows, int pair_ffn, void* stream) {
  HV_REQUIRE(a8 && sa && pb4 && psw && dst && k8 > 0 && rows > 0, HV_E_INVALID,
             "hv_a4gv_pp: bad arguments");
  HV_REQUIRE(k8 % 4 == 0, HV_E_INVALID, "hv_a4gv_pp: K = %d is not a multiple of 32", k8 * 8);
  HV_REQUIRE(pair_ffn == 0 || rows == 2 * pair_ffn, HV_E_INVALID,
             "hv_a4gv_pp: a paired matrix has 2 * pair_ffn rows");
  HV_REQUIRE(((uintptr_t)a8 & 15) == 0 && ((uintptr_t)pb4 & 15) == 0 &&
                 ((uintptr_t)psw & 15) == 0, HV_E_INVALID, "hv_a4gv_pp: unaligned pointer");
  const int nb = k8 / 4;
  HV_REQUIRE(nb <= 4096, HV_E_UNSUPPORTED, "hv_a4gv_pp: K = %d exceeds 131072", k8 * 8);
  GvPlan plan;
  HV_REQUIRE(gv_make_plan(nb, &plan), HV_E_UNSUPPORTED, "hv_a4gv_pp: no reduction plan for K");
  const size_t smem = (size_t)nb * 40;
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  const int ntile = pp_tiles(rows, pair_ffn);
  if (g_gemv_split && plan.ntail == 0 && plan.nfull >= kSplitMinIters &&
      plan.nfull <= kSplitMaxIters && ntile < 16 * sms) {
    const size_t smem_s = smem + (size_t)plan.nfull * 32 * sizeof(float2);
    rc = smem_attr((const void*)k_a4gv_pps, smem_s);
    if (rc) return rc;
    k_a4gv_pps<<<ntile, 256, smem_s, (cudaStream_t)stream>>>(a8, sa, pb4, psw, dst, rows,
                                                             pair_ffn, plan);
    HV_LAUNCHED("k_a4gv_pps");
  }
  int grid = (ntile + 7) / 8;
  if (grid > sms * 4) grid = sms * 4;
  rc = smem_attr((const void*)k_a4gv_pp, smem);
  if (rc) return rc;
  k_a4gv_pp<<<grid, 256, smem, (cudaStream_t)stream>>>(a8, sa, pb4, psw, dst, rows, pair_ffn,
                                                       plan);
  HV_LAUNCHED("k_a4gv_pp");
}

int hv_w4_prepack_dq(const uint32_t* b4, const float* sw, int rows, int k, int pair_ffn,
                     uint32_t* pb4, float* psw, void* stream) {
  HV_REQUIRE(b4 && sw && pb4 && psw && rows > 0 && k > 0 && k % kBlock == 0, HV_E_INVALID,
             "hv_w4_prepack_dq: bad arguments");
  HV_REQUIRE(pair_ffn == 0 || rows == 2 * pair_ffn, HV_E_INVALID,
             "hv_w4_prepack_dq: a paired matrix has 2 * pair_ffn rows");
  HV_REQUIRE(((uintptr_t)b4 & 15) == 0 && ((uintptr_t)pb4 & 15) == 0 &&
                 ((uintptr_t)psw & 15) == 0,
             HV_E_INVALID, "hv_w4_prepack_dq: pointers must be 16-byte aligned");
  const int nb = k / kBlock;
  const int ntile = pp_tiles(rows, pair_ffn), niter = pp_iters(nb);
  const long long threads = (long long)ntile * niter * 32;
  k_w4_prepack_dq<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      b4, sw, rows, nb, pair_ffn, ntile, niter, pb4, psw);
  HV_LAUNCHED("k_w4_prepack_dq");
}

int hv_a4gv_dq(const int8_t* a8, const float* sa, const uint32_t* pb4, const float* psw,
               float* dst, int k8, int rows, int pair_ffn, void* stream) {
  HV_REQUIRE(a8 && sa && pb4 && psw && dst && k8 > 0 && rows > 0, HV_E_INVALID,
             "hv_a4gv_dq: bad arguments");
  HV_REQUIRE(k8 % 4 == 0, HV_E_INVALID, "hv_a4gv_dq: K = %d is not a multiple of 32", k8 * 8);
  HV_REQUIRE(pair_ffn == 0 || rows == 2 * pair_ffn, HV_E_INVALID,
             "hv_a4gv_dq: a paired matrix has 2 * pair_ffn rows");
  HV_REQUIRE(((uintptr_t)a8 & 15) == 0 && ((uintptr_t)pb4 & 15) == 0 &&
                 ((uintptr_t)psw & 15) == 0, HV_E_INVALID, "hv_a4gv_dq: unaligned pointer");
  const int nb = k8 / 4;
  HV_REQUIRE(nb <= 4096, HV_E_UNSUPPORTED, "hv_a4gv_dq: K = %d exceeds 131072", k8 * 8);
  GvPlan plan;
  HV_REQUIRE(gv_make_plan(nb, &plan), HV_E_UNSUPPORTED, "hv_a4gv_dq: no reduction plan for K");
  const size_t smem = (size_t)nb * 40;
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  const int ntile = pp_tiles(rows, pair_ffn);
  int grid = (ntile + 7) / 8;
  if (grid > sms * 4) grid = sms * 4;
  rc = smem_attr((const void*)k_a4gv_dq, smem);
  if (rc) return rc;
  k_a4gv_dq<<<grid, 256, smem, (cudaStream_t)stream>>>(a8, sa, pb4, psw, dst, rows, pair_ffn,
                                                       plan);
  HV_LAUNCHED("k_a4gv_dq");
}

int hv_gemv_set_split(int enable) {
  g_gemv_split = enable ? 1 : 0;
  return HV_OK;
}

int hv_rmsnorm(const float* src, float* dst, const float* w, int rows, int cols, float eps,
               void* stream) {
  HV_REQUIRE(src && dst && w && rows > 0 && cols > 0, HV_E_INVALID, "hv_rmsnorm: bad arguments");
  // +8 floats: the idle lane groups of the leaf pass read x[0..8) even when cols < 8
  const size_t smem = sizeof(float) * (kPwMaxLeaf + 4 + 2 * (size_t)cols + 8);
  HV_REQUIRE(smem <= 220 * 1024, HV_E_UNSUPPORTED, "hv_rmsnorm: %d columns is too wide", cols);
  PwPlan plan;
  HV_REQUIRE(pw_make_plan(cols, &plan), HV_E_UNSUPPORTED, "hv_rmsnorm: no plan for %d", cols);
  int rc = smem_attr((const void*)k_rmsnorm, smem);
  if (rc) return rc;
  k_rmsnorm<<<rows, 256, smem, (cudaStream_t)stream>>>(src, dst, w, cols, eps, plan);
  HV_LAUNCHED("k_rmsnorm");
}

int hv_rope(float* vec, const float* cos_t, const float* sin_t, const int32_t* pos, int heads,
            int half, void* stream) {
  HV_REQUIRE(vec && cos_t && sin_t && pos && heads > 0 && half > 0, HV_E_INVALID,
             "hv_rope: bad arguments");
  k_rope<<<heads, 64, 0, (cudaStream_t)stream>>>(vec, cos_t, sin_t, pos, half);
  HV_LAUNCHED("k_rope");
}

int hv_kv_append(const float* k, const float* v, float* kc, float* vc, const int32_t* pos,
                 int nkv, int hd, int cap, void* stream) {
  HV_REQUIRE(k && v && kc && vc && pos && nkv > 0 && hd > 0 && cap > 0, HV_E_INVALID,
             "hv_kv_append: bad arguments");
  k_kvapp<<<nkv, 128, 0, (cudaStream_t)stream>>>(k, v, kc, vc, pos, hd, cap);
  HV_LAUNCHED("k_kvapp");
}

int hv_kv_append_f16(const float* k, const float* v, uint16_t* kc, uint16_t* vc,
                     const int32_t* pos, int nkv, int hd, int cap, void* stream) {
  HV_REQUIRE(k && v && kc && vc && pos && nkv > 0 && hd > 0 && cap > 0, HV_E_INVALID,
             "hv_kv_append_f16: bad arguments");
  k_kvapp16<<<nkv, 128, 0, (cudaStream_t)stream>>>(k, v, reinterpret_cast<__half*>(kc),
                                                   reinterpret_cast<__half*>(vc), pos, hd, cap);
  HV_LAUNCHED("k_kvapp16");
}

int hv_attn_reserve(int nkv, int group, int cap) {
  HV_REQUIRE(nkv > 0 && group > 0 && cap > 0, HV_E_INVALID, "hv_attn_reserve: bad arguments");
  int nch = 0;
  int rc = attn_exact_chunks(nkv, cap, &nch);
  if (rc) return rc;
  AttnScratch* s = nullptr;
  return attn_scratch(nkv * group, cap, nch, nullptr, &s);
}

int hv_attn_decode(const float* q, const float* kc, const float* vc, float* ctx,
                   const float* scale, const int32_t* pos, int nq, int hd, int group,
                   int kvstride, void* stream) {
  return attn_decode_any("hv_attn_decode", false, q, kc, vc, ctx, scale, pos, nq, hd, group,
                         kvstride, stream);
}

int hv_attn_decode_f16(const float* q, const uint16_t* kc, const uint16_t* vc, float* ctx,
                       const float* scale, const int32_t* pos, int nq, int hd, int group,
                       int kvstride, void* stream) {
  return attn_decode_any("hv_attn_decode_f16", true, q, kc, vc, ctx, scale, pos, nq, hd,
                         group, kvstride, stream);
}

int hv_silu_mul(const float* gate, const float* up, float* act, int n, void* stream) {
  HV_REQUIRE(gate && up && act && n > 0, HV_E_INVALID, "hv_silu_mul: bad arguments");
  k_silu<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(gate, up, act, n);
  HV_LAUNCHED("k_silu");
}

int hv_vadd(const float* a, const float* b, float* out, int n, void* stream) {
  HV_REQUIRE(a && b && out && n > 0, HV_E_INVALID, "hv_vadd: bad arguments");
  k_vadd<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(a, b, out, n);
  HV_LAUNCHED("k_vadd");
}

int hv_gather_emb(const uint16_t* emb16, const int32_t* tok, float* h, int hid, void* stream) {
  HV_REQUIRE(emb16 && tok && h && hid > 0, HV_E_INVALID, "hv_gather_emb: bad arguments");
  k_gather<<<(hid + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const __half*>(emb16), tok, h, hid);
  HV_LAUNCHED("k_gather");
}

int hv_argmax_partial(const float* logits, float* pv, int32_t* pi, int n, int parts,
                      void* stream) {
  HV_REQUIRE(logits && pv && pi && n > 0 && parts > 0, HV_E_INVALID,
             "hv_argmax_partial: bad arguments");
  k_argmax_p<<<parts, 256, 0, (cudaStream_t)stream>>>(logits, pv, pi, n, parts);
  HV_LAUNCHED("k_argmax_p");
}

int hv_argmax_final(const float* pv, const int32_t* pi, int32_t* tok, int32_t* gen,
                    int32_t* step, int32_t* pos, int parts, void* stream) {
  HV_REQUIRE(pv && pi && tok && gen && step && pos && parts > 0, HV_E_INVALID,
             "hv_argmax_final: bad arguments");
  k_argmax_f<<<1, 128, 0, (cudaStream_t)stream>>>(pv, pi, tok, gen, step, pos, parts);
  HV_LAUNCHED("k_argmax_f");
}

int hv_argmax_key(const float* logits, int n, int base, uint64_t* key, void* stream) {
  HV_REQUIRE(logits && key && n > 0 && base >= 0 && (long long)base + n <= 0x7FFFFFFFll,
             HV_E_INVALID, "hv_argmax_key: bad arguments");
  HV_REQUIRE(((uintptr_t)key & 7) == 0, HV_E_INVALID, "hv_argmax_key: key not 8-byte aligned");
  int grid = (n + 1023) / 1024;
  if (grid > 512) grid = 512;
  k_argmax_key<<<grid, 256, 0, (cudaStream_t)stream>>>(
      logits, n, base, reinterpret_cast<unsigned long long*>(key));
  HV_LAUNCHED("k_argmax_key");
}

int hv_argmax_key_final(uint64_t* keys, int nkeys, int32_t* tok, int32_t* gen, int32_t* step,
                        int32_t* pos, void* stream) {
  HV_REQUIRE(keys && tok && gen && step && pos && nkeys > 0, HV_E_INVALID,
             "hv_argmax_key_final: bad arguments");
  HV_REQUIRE(((uintptr_t)keys & 7) == 0, HV_E_INVALID,
             "hv_argmax_key_final: keys not 8-byte aligned");
  k_argmax_keyf<<<1, 32, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<unsigned long long*>(keys), nkeys, tok, gen, step, pos);
  HV_LAUNCHED("k_argmax_keyf");
}

int hv_wait_probe(const uint32_t* word, uint32_t mask, uint32_t want, long long limit_ns,
                  int32_t* status, void* stream) {
  HV_REQUIRE(word && status && ((uintptr_t)word & 3) == 0 && ((uintptr_t)status & 3) == 0,
             HV_E_INVALID, "hv_wait_probe: bad arguments");
  HV_REQUIRE(limit_ns > 0 && limit_ns <= 10000000000ll, HV_E_INVALID,
             "hv_wait_probe: limit %lld ns outside (0, 10 s]", limit_ns);
  k_wait_probe<<<1, 32, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<const unsigned*>(word), mask, want, (unsigned long long)limit_ns,
      reinterpret_cast<int*>(status));
  HV_LAUNCHED("k_wait_probe");
}

int hv_quantize_w4(const float* w, uint32_t* packed, float* scale, int n, int k,
                   void* stream) {
  HV_REQUIRE(w && packed && scale && n > 0 && k > 0, HV_E_INVALID,
             "hv_quantize_w4: bad arguments");
  HV_REQUIRE(k % kBlock == 0, HV_E_INVALID, "hv_quantize_w4: K=%d is not a multiple of 32", k);
  HV_REQUIRE(((uintptr_t)w & 15) == 0 && ((uintptr_t)packed & 15) == 0, HV_E_INVALID,
             "hv_quantize_w4: w and packed must be 16-byte aligned");
  const long long nblocks = (long long)n * (k / kBlock);
  k_quantize_w4<<<(unsigned)((nblocks + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      w, packed, scale, nblocks);
  HV_LAUNCHED("k_quantize_w4");
}

}  // extern "C"
