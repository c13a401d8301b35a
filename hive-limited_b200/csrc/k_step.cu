// The fused decode step: HIVE Limited's Engine._step() + LM head + greedy argmax
// (engine/limited.py:374-428) as ONE persistent cooperative kernel.
//
// Why one kernel: at batch 1 the step is ~20 dependent launches per layer (the
// reference issues 538 for 28 layers). Each launch boundary drains the GPU; here the
// dependencies become grid barriers inside one launch, and every CTA recomputes the
// small vector work it needs (RMSNorm + per-32 quantisation of a 4-20 KB vector, the
// q/k norms and RoPE of its own heads) instead of waiting on a separate kernel.
//
// Per layer, five phases separated by grid barriers:
//   P1 qkv  : act <- quant(rmsnorm(h, an)); rows of W_qkv        -> qkv
//   P2 attn : per (kv head, chunk): q/k norm + RoPE, KV append at pos, split softmax;
//             last CTA of each kv head merges                     -> ctx
//   P3 o    : act <- quant(ctx);   rows of W_o, h[row] += y        -> h
//   P4 gu   : act <- quant(rmsnorm(h, fn)); gate/up row pairs, SiLU -> act
//   P5 down : act <- quant(act);   rows of W_down, h[row] += y     -> h
// then the head: act <- quant(rmsnorm(h, onorm)); rows of the LM head -> logits and a
// per-CTA argmax; the last CTA picks the token and advances tok/gen/step/pos.
//
// Rows of every matrix are split evenly over the CTAs; the o and down splits are the
// same (N = hidden), so the CTA that adds into h[row] is always the one that last
// wrote it. Data produced by other CTAs is read through L2 (ld.global.cg): L1 is not
// coherent across SMs.
#include <mutex>

#include <cuda_fp16.h>

#include "attn_decode.cuh"
#include "gemv_mma.cuh"
#include "hv_internal.h"

namespace hv {

constexpr int kStepThreads = 512;        // 16 warps, up to 128 registers each
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kStepU = 4;                 // GEMV load pipeline depth (iterations in flight)
constexpr int kCBufFloats = 12288;        // block terms of split GEMV phases (48 KB)
constexpr int kMaxHidden = 8192;          // pro_norm_quant holds 4 float4 per thread
constexpr unsigned long long kWaitNs = 2000000000ull;   // a barrier wait gives up after 2 s

// Reduction plans of the step, built on the host (hv_step_plans) and copied into shared
// memory at the start of every launch.
struct StepPlans {
  PwPlan pw_hid;                 // RMSNorm over the hidden vector
  GvPlan gv_hid, gv_o, gv_ffn;   // GEMV rows with K = hidden, n_head * 128, ffn
};

struct StepShared {
  StepPlans P;
  float leafval[kPwMaxLeaf];
  float red[4];
  float sv[32];
  int si[32];
  int flag;
  int ok;
};

HV_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

HV_DEV unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Grid-wide barrier over a self-resetting counter: CTA 0 adds 2^31 - (grid - 1), the
// others add 1, so the top bit flips exactly when all have arrived and the low bits
// return to zero. The wait is bounded: after kWaitNs (or once another CTA has reported
// a failure) it records HV_E_TIMEOUT in *status and returns false.
HV_DEV bool grid_sync(unsigned* bar, int* status, StepShared& S) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned add = (blockIdx.x == 0) ? (0x80000000u - (gridDim.x - 1)) : 1u;
    __threadfence();
    const unsigned old = atomicAdd(bar, add);
    const unsigned long long t0 = global_ns();
    int ok = 1;
    while (((ld_acquire(bar) ^ old) & 0x80000000u) == 0) {
      if (*(volatile int*)status != 0) { ok = 0; break; }
      if (global_ns() - t0 > kWaitNs) {
        atomicExch(status, HV_E_TIMEOUT);
        ok = 0;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    S.ok = ok;
  }
  __syncthreads();
  return S.ok != 0;
}

HV_DEV void trace_mark(const hv_step_desc& D, int idx) {
  if (D.trace != nullptr && threadIdx.x == 0)
    D.trace[(size_t)blockIdx.x * HV_STEP_TRACE_STRIDE(D.n_layer) + idx] = global_ns();
}

HV_DEV void row_range(int n, int* r0, int* r1) {
  *r0 = (int)(((long long)blockIdx.x * n) / gridDim.x);
  *r1 = (int)(((long long)(blockIdx.x + 1) * n) / gridDim.x);
}

// ---- prologues: build the quantised activation in shared memory ---------------------

// act <- quant(rmsnorm(src, w)) over n = hidden values (n % 32 == 0, n <= kMaxHidden);
// src from global (through L2) or, for layer 0, the f16 embedding row. Every load of
// the vector and of the gain is issued before any is used.
__device__ __noinline__ void pro_norm_quant(const float* src, const __half* emb_row,
                                            const float* __restrict__ w, int n, float eps,
                                            StepShared& S, float* x, float* sq, uint4* q_s,
                                            int2* sb_s) {
  constexpr int kV = kMaxHidden / 4 / kStepThreads;   // float4 per thread
  const int n4 = n / 4;
  const int t = threadIdx.x;
  float4 xv[kV], wv[kV];
#pragma unroll
  for (int k = 0; k < kV; ++k) {
    const int i4 = t + k * kStepThreads;
    if (i4 < n4) {
      if (src) {
        xv[k] = __ldcg(reinterpret_cast<const float4*>(src) + i4);
      } else {
        const __half2* e = reinterpret_cast<const __half2*>(emb_row) + 2 * i4;
        const float2 a = __half22float2(e[0]), b = __half22float2(e[1]);
        xv[k] = make_float4(a.x, a.y, b.x, b.y);
      }
      wv[k] = __ldg(reinterpret_cast<const float4*>(w) + i4);
    }
  }
#pragma unroll
  for (int k = 0; k < kV; ++k) {
    const int i4 = t + k * kStepThreads;
    if (i4 < n4)
      reinterpret_cast<float4*>(sq)[i4] =
          make_float4(__fmul_rn(xv[k].x, xv[k].x), __fmul_rn(xv[k].y, xv[k].y),
                      __fmul_rn(xv[k].z, xv[k].z), __fmul_rn(xv[k].w, xv[k].w));
  }
  __syncthreads();
  const float ss = block_pw_sum(sq, &S.P.pw_hid, S.leafval, S.red);
  const float d = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps));
#pragma unroll
  for (int k = 0; k < kV; ++k) {
    const int i4 = t + k * kStepThreads;
    if (i4 < n4)
      reinterpret_cast<float4*>(x)[i4] = make_float4(
          __fmul_rn(wv[k].x, __fdiv_rn(xv[k].x, d)), __fmul_rn(wv[k].y, __fdiv_rn(xv[k].y, d)),
          __fmul_rn(wv[k].z, __fdiv_rn(xv[k].z, d)), __fmul_rn(wv[k].w, __fdiv_rn(xv[k].w, d)));
  }
  __syncthreads();
  // quantise: 8 lanes per 32-block, 4 blocks per warp pass
  const int lane = t & 31, sub = lane & 7;
  unsigned* q32 = reinterpret_cast<unsigned*>(q_s);
  const int nb = n / kBlock;
  for (int b0 = (t >> 5) * 4; b0 < nb; b0 += kStepWarps * 4) {
    const int b = b0 + (lane >> 3);
    if (b < nb) {
      float s;
      int bs;
      const float4 v = reinterpret_cast<const float4*>(x)[b * 8 + sub];
      q32[b * 8 + sub] = quant_block_8lanes(v, &s, &bs);
      if (sub == 0) sb_s[b] = make_int2(__float_as_int(s), bs);
    }
  }
  __syncthreads();
}

// act <- quant(src) over n values produced by other CTAs (n % 32 == 0); 8 lanes per
// 32-block, the loads of up to 8 passes in flight together.
__device__ __noinline__ void pro_quant(const float* src, int n, uint4* q_s, int2* sb_s) {
  constexpr int kBatch = 8;
  const int lane = threadIdx.x & 31, sub = lane & 7;
  unsigned* q32 = reinterpret_cast<unsigned*>(q_s);
  const int nb = n / kBlock;
  const int step = kStepWarps * 4;
  for (int base = (threadIdx.x >> 5) * 4; base < nb; base += step * kBatch) {
    float4 v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int b = base + k * step + (lane >> 3);
      v[k] = (b < nb) ? __ldcg(reinterpret_cast<const float4*>(src) + b * 8 + sub)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int b = base + k * step + (lane >> 3);
      if (b < nb) {
        float s;
        int bs;
        q32[b * 8 + sub] = quant_block_8lanes(v[k], &s, &bs);
        if (sub == 0) sb_s[b] = make_int2(__float_as_int(s), bs);
      }
    }
  }
  __syncthreads();
}

// L2 prefetch (one thread) of tiles [t0, t1) of a prepacked matrix with K columns: the
// tiles' nibbles and scales are each one contiguous range.
HV_DEV void prefetch_tiles(const uint32_t* pb4, const float* psw, int k, int t0, int t1) {
  if (threadIdx.x != 0 || t1 <= t0) return;
  const size_t it = (size_t)pp_iters(k / kBlock);
  prefetch_l2(pb4 + (size_t)t0 * it * kPpNibWords, (size_t)(t1 - t0) * it * kPpNibWords * 4);
  prefetch_l2(psw + (size_t)t0 * it * kPpScales, (size_t)(t1 - t0) * it * kPpScales * 4);
}

// ---- GEMV phases -----------------------------------------------------------------------

enum { kStore = 0, kResidual = 1, kSiluPair = 2, kHead = 3 };

HV_DEV int pp_row_of(int tile, int g, int rows, int pair_ffn, bool* ok) {
  if (pair_ffn > 0) {
    const int p = tile * 4 + (g & 3);
    *ok = p < pair_ffn;
    return (g < 4) ? p : pair_ffn + p;
  }
  const int row = tile * 8 + g;
  *ok = row < rows;
  return row;
}

// GEMV over this CTA's tiles [t0, t1) of a matrix in the tile-interleaved layout.
// MODE kStore/kResidual/kHead: 8-row tiles of `rows` rows. kSiluPair: tiles of 4 gate
// rows (quads 0-3) and their 4 up rows (quads 4-7) of a [gate | up] matrix with pair_ffn
// rows per half; SiLU(gate) * up is formed in the lane that holds the gate row.
//
// With fewer tiles than warps, each tile's iterations are cut into chunks so every warp
// has work: (tile, chunk) items write their block terms to shared memory (cbuf), then
// one warp per tile walks numpy's chains over them in order. Otherwise a warp takes a
// whole tile and keeps the chains in registers. Both give the same bits.
template <int MODE>
HV_DEV void gemv_epilogue(float y, int row, bool ok, float* __restrict__ out, float* best_v,
                          int* best_i) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (MODE == kSiluPair) {
    const float up = __shfl_down_sync(0xFFFFFFFFu, y, 16);
    if (g < 4 && t == 0 && ok) out[row] = silu_mul1(y, up);
  } else if (t == 0 && ok) {
    if (MODE == kStore) {
      out[row] = y;
    } else if (MODE == kResidual) {
      out[row] = __fadd_rn(__ldcg(out + row), y);
    } else {
      out[row] = y;
      if (y > *best_v || (y == *best_v && row < *best_i)) { *best_v = y; *best_i = row; }
    }
  }
}

template <int MODE>
__device__ __noinline__ void gemv_split(const uint32_t* __restrict__ pb4,
                                        const float* __restrict__ psw, const GvPlan& P,
                                        const ActView act, int t0, int t1, int rows,
                                        int pair_ffn, int chunks, float* __restrict__ out,
                                        float* best_v, int* best_i, float* cbuf) {
  const int lane = threadIdx.x & 31, g = lane >> 2;
  const int warp = threadIdx.x >> 5;
  const int ntile = t1 - t0;
  const int niter = pp_iters(P.nb);
  const unsigned* act_w = reinterpret_cast<const unsigned*>(act.q);
  float2* cb = reinterpret_cast<float2*>(cbuf);
  for (int item = warp; item < ntile * chunks; item += kStepWarps) {
    const int lt = item / chunks, c = item % chunks;
    const int tile = t0 + lt;
    tile_terms_pp<kStepU>(pb4 + (size_t)tile * niter * kPpNibWords,
                          psw + (size_t)tile * niter * kPpScales, act_w, act.sb, P,
                          (c * niter) / chunks, ((c + 1) * niter) / chunks,
                          cb + (size_t)lt * niter * 32);
  }
  __syncthreads();
  for (int lt = warp; lt < ntile; lt += kStepWarps) {
    bool ok;
    const int row = pp_row_of(t0 + lt, g, rows, pair_ffn, &ok);
    const float y = chains_fold(P, cb + (size_t)lt * niter * 32);
    gemv_epilogue<MODE>(y, row, ok, out, best_v, best_i);
  }
  __syncthreads();
}

template <int MODE>
__device__ __noinline__ void gemv_direct(const uint32_t* __restrict__ pb4,
                                         const float* __restrict__ psw, const GvPlan& P,
                                         const ActView act, int t0, int t1, int rows,
                                         int pair_ffn, float* __restrict__ out, float* best_v,
                                         int* best_i) {
  const int lane = threadIdx.x & 31, g = lane >> 2;
  const int warp = threadIdx.x >> 5;
  const int niter = pp_iters(P.nb);
  const unsigned* act_w = reinterpret_cast<const unsigned*>(act.q);
  for (int tile = t0 + warp; tile < t1; tile += kStepWarps) {
    bool ok;
    const int row = pp_row_of(tile, g, rows, pair_ffn, &ok);
    float y;
    gemv_tile8<kStepU, true, true>(pb4 + (size_t)tile * niter * kPpNibWords,
                                   psw + (size_t)tile * niter * kPpScales, act_w, act.sb, P, 0,
                                   P.nleaf, &y, nullptr);
    gemv_epilogue<MODE>(y, row, ok, out, best_v, best_i);
  }
}

template <int MODE>
HV_DEV void gemv_phase(const uint32_t* __restrict__ pb4, const float* __restrict__ psw,
                       const GvPlan& P, const ActView act, int t0, int t1, int rows,
                       int pair_ffn, float* __restrict__ out, float* best_v, int* best_i,
                       float* cbuf) {
  const int ntile = t1 - t0;
  const int niter = pp_iters(P.nb);
  int chunks = 1;
  if (ntile > 0 && ntile < kStepWarps) {
    chunks = (kStepWarps + ntile - 1) / ntile;
    if (chunks > niter) chunks = niter;
    if ((size_t)ntile * niter * 64 > (size_t)kCBufFloats) chunks = 1;
  }
  if (chunks > 1)
    gemv_split<MODE>(pb4, psw, P, act, t0, t1, rows, pair_ffn, chunks, out, best_v, best_i, cbuf);
  else
    gemv_direct<MODE>(pb4, psw, P, act, t0, t1, rows, pair_ffn, out, best_v, best_i);
}

// ---- attention -------------------------------------------------------------------------

// One warp: rmsnorm(raw[0..128), gain) then rotate-half RoPE with this position's tables,
// bit-identical to k_rmsnorm (cols = 128) followed by k_rope.
HV_DEV void warp_norm_rope(const float* raw, const float* __restrict__ gain,
                           const float* __restrict__ cs, const float* __restrict__ sn,
                           float eps, float* tmp, float* dst) {
  const int lane = threadIdx.x & 31;
  const float4 x = __ldcg(reinterpret_cast<const float4*>(raw) + lane);
  tmp[4 * lane + 0] = __fmul_rn(x.x, x.x);
  tmp[4 * lane + 1] = __fmul_rn(x.y, x.y);
  tmp[4 * lane + 2] = __fmul_rn(x.z, x.z);
  tmp[4 * lane + 3] = __fmul_rn(x.w, x.w);
  __syncwarp();
  const float ss = __fadd_rn(0.0f, pw_leaf8(tmp, kHd, lane & 7));
  const float d = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)kHd), eps));
  __syncwarp();
  tmp[4 * lane + 0] = __fmul_rn(__ldg(gain + 4 * lane + 0), __fdiv_rn(x.x, d));
  tmp[4 * lane + 1] = __fmul_rn(__ldg(gain + 4 * lane + 1), __fdiv_rn(x.y, d));
  tmp[4 * lane + 2] = __fmul_rn(__ldg(gain + 4 * lane + 2), __fdiv_rn(x.z, d));
  tmp[4 * lane + 3] = __fmul_rn(__ldg(gain + 4 * lane + 3), __fdiv_rn(x.w, d));
  __syncwarp();
  for (int i = lane; i < kHd / 2; i += 32) {
    const float c = __ldg(cs + i), s = __ldg(sn + i);
    const float lo = tmp[i], hi = tmp[kHd / 2 + i];
    dst[i] = __fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s));
    dst[kHd / 2 + i] = __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s));
  }
  __syncwarp();
}

template <typename T>
HV_DEV T* ldg_ptr(T* const* p) {
  return reinterpret_cast<T*>(__ldg(reinterpret_cast<const unsigned long long*>(p)));
}

template <int GS>
__device__ __noinline__ void attn_phase(const hv_step_desc& D, const hv_layer_w* L, int pos, StepShared& S,
                       float* area) {
  const int nkv = D.n_kv, nch = D.attn_chunks, cap = D.cap, nq = D.n_head;
  const int chunk_max = (cap + nch - 1) / nch;
  const int lg_floats = (chunk_max * GS + 3) & ~3;   // keeps red_s 16-byte aligned
  float* q_s = area;
  float* kpos_s = q_s + GS * kHd;
  float* vpos_s = kpos_s + kHd;
  float* tmp_s = vpos_s + kHd;                       // (GS + 1) x 128
  float* stat_s = tmp_s + (GS + 1) * kHd;            // 2 GS (+pad)
  float* lg_s = stat_s + 4 * GS;
  float* red_s = lg_s + lg_floats;                  // accessed as float4
  const int warp = threadIdx.x >> 5;
  const float* cs = D.cos_t + (size_t)pos * (kHd / 2);
  const float* sn = D.sin_t + (size_t)pos * (kHd / 2);
  for (int wi = blockIdx.x; wi < nkv * nch; wi += gridDim.x) {
    const int g = wi / nch, c = wi % nch;
    // GS query heads, the kv head's k (normed + rotated) and its raw v, a warp each
    for (int h = warp; h < GS + 2; h += kStepWarps) {
      if (h < GS) {
        warp_norm_rope(D.qkv + (size_t)(g * GS + h) * kHd, ldg_ptr(&L->qn), cs, sn, D.eps,
                       tmp_s + h * kHd, q_s + h * kHd);
      } else if (h == GS) {
        warp_norm_rope(D.qkv + (size_t)(nq + g) * kHd, ldg_ptr(&L->kn), cs, sn, D.eps,
                       tmp_s + GS * kHd, kpos_s);
      } else {
        const int lane = threadIdx.x & 31;
        reinterpret_cast<float4*>(vpos_s)[lane] =
            __ldcg(reinterpret_cast<const float4*>(D.qkv + (size_t)(nq + nkv + g) * kHd) + lane);
      }
    }
    __syncthreads();
    float* kc = ldg_ptr(&L->kc) + (size_t)g * cap * kHd;
    float* vc = ldg_ptr(&L->vc) + (size_t)g * cap * kHd;
    if (c == nch - 1 && threadIdx.x < kHd) {         // the chunk holding pos appends
      kc[(size_t)pos * kHd + threadIdx.x] = kpos_s[threadIdx.x];
      vc[(size_t)pos * kHd + threadIdx.x] = vpos_s[threadIdx.x];
    }
    int t0, t1;
    chunk_bounds(pos + 1, nch, c, &t0, &t1);
    float* part = D.part + ((size_t)g * nch + c) * GS * kPartStride;
    attn_chunk<GS>(q_s, kc, vc, t0, t1, D.attn_scale, pos, kpos_s, vpos_s, lg_s, red_s,
                   stat_s, part);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) S.flag = (atomicAdd(D.ticket + g, 1) == nch - 1);
    __syncthreads();
    if (S.flag) {
      __threadfence();
      attn_merge<GS>(D.part + (size_t)g * nch * GS * kPartStride, nch,
                     D.ctx + (size_t)g * GS * kHd, red_s);
      if (threadIdx.x == 0) D.ticket[g] = 0;
    }
    __syncthreads();
  }
}

// L2 prefetch (one thread) of the K and V rows this CTA's attention work items read.
HV_DEV void prefetch_kv(const hv_step_desc& D, const hv_layer_w* L, int pos) {
  if (threadIdx.x != 0) return;
  const int nch = D.attn_chunks;
  const float* kc = ldg_ptr(&L->kc);
  const float* vc = ldg_ptr(&L->vc);
  for (int wi = blockIdx.x; wi < D.n_kv * nch; wi += gridDim.x) {
    const int g = wi / nch, c = wi % nch;
    int t0, t1;
    chunk_bounds(pos + 1, nch, c, &t0, &t1);
    if (t1 <= t0) continue;
    const size_t off = ((size_t)g * D.cap + t0) * kHd;
    prefetch_l2(kc + off, (size_t)(t1 - t0) * kHd * 4);
    prefetch_l2(vc + off, (size_t)(t1 - t0) * kHd * 4);
  }
}

// ---- the kernel ------------------------------------------------------------------------

template <int GS>
__global__ void __launch_bounds__(kStepThreads, 1) k_step(const hv_step_desc D, int flags) {
  extern __shared__ __align__(16) unsigned char smem[];
  StepShared& S = *reinterpret_cast<StepShared*>(smem);
  float* area = reinterpret_cast<float*>(smem + ((sizeof(StepShared) + 15) & ~size_t(15)));
  const int hid = D.hidden, ffn = D.ffn, qdim = D.n_head * kHd;
  const int kmax = max(max(hid, qdim), ffn);
  uint4* q_s = reinterpret_cast<uint4*>(area);
  int2* sb_s = reinterpret_cast<int2*>(reinterpret_cast<unsigned char*>(area) + kmax);
  // every region starts on a 16-byte boundary (float4 / int4 accesses)
  float* x_s = reinterpret_cast<float*>(
      reinterpret_cast<unsigned char*>(area) + (((size_t)kmax + (kmax / kBlock) * 8 + 15) & ~size_t(15)));
  float* sq_s = x_s + hid;
  float* leaf_s = sq_s + hid;             // block terms of split GEMV phases
  const ActView act{q_s, sb_s};

  trace_mark(D, 0);
  {
    const int* src = reinterpret_cast<const int*>(D.plans);
    int* dst = reinterpret_cast<int*>(&S.P);
    for (int i = threadIdx.x; i < (int)(sizeof(StepPlans) / 4); i += blockDim.x) dst[i] = __ldg(src + i);
  }
  const int pos = *D.pos;
  const int tok = *D.tok;
  __syncthreads();
  if (pos < 0 || pos >= D.cap || tok < 0 || tok >= D.vocab) {
    // every CTA reads the same values, so all leave here, before the first barrier
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(D.status, HV_E_INVALID);
    return;
  }

  // this CTA's tiles of every matrix; o and down share N = hidden, so the CTA that adds
  // into h[row] is always the one that last wrote it
  const int nqkv = (D.n_head + 2 * D.n_kv) * kHd;
  int qt0, qt1, ht0, ht1, gt0, gt1;
  row_range(pp_tiles(nqkv, 0), &qt0, &qt1);
  row_range(pp_tiles(hid, 0), &ht0, &ht1);
  row_range(pp_tiles(2 * ffn, ffn), &gt0, &gt1);
  const int hr0 = ht0 * 8, hr1 = min(ht1 * 8, hid);
  const __half* emb_row = reinterpret_cast<const __half*>(D.emb16) + (size_t)tok * hid;
  for (int i = hr0 + threadIdx.x; i < hr1; i += blockDim.x) D.h[i] = __half2float(emb_row[i]);

  prefetch_tiles(ldg_ptr(&D.layers[0].qkv_b4), ldg_ptr(&D.layers[0].qkv_sw), hid, qt0, qt1);
  trace_mark(D, 1);
  for (int l = 0; l < D.n_layer; ++l) {
    const hv_layer_w* L = D.layers + l;
    const int tb = 2 + 14 * l;
    // P1: qkv
    pro_norm_quant(l == 0 ? nullptr : D.h, emb_row, ldg_ptr(&L->an), hid, D.eps, S, x_s, sq_s,
                   q_s, sb_s);
    trace_mark(D, tb + 0);
    gemv_phase<kStore>(ldg_ptr(&L->qkv_b4), ldg_ptr(&L->qkv_sw), S.P.gv_hid, act, qt0, qt1, nqkv,
                       0, D.qkv, nullptr, nullptr, leaf_s);
    trace_mark(D, tb + 1);
    prefetch_kv(D, L, pos);
    if (!grid_sync(D.barrier, D.status, S)) return;
    trace_mark(D, tb + 2);
    // P2: attention
    attn_phase<GS>(D, L, pos, S, area);
    trace_mark(D, tb + 3);
    prefetch_tiles(ldg_ptr(&L->o_b4), ldg_ptr(&L->o_sw), qdim, ht0, ht1);
    if (!grid_sync(D.barrier, D.status, S)) return;
    trace_mark(D, tb + 4);
    // P3: o projection + residual
    pro_quant(D.ctx, qdim, q_s, sb_s);
    trace_mark(D, tb + 5);
    gemv_phase<kResidual>(ldg_ptr(&L->o_b4), ldg_ptr(&L->o_sw), S.P.gv_o, act, ht0, ht1, hid, 0,
                          D.h, nullptr, nullptr, leaf_s);
    trace_mark(D, tb + 6);
    prefetch_tiles(ldg_ptr(&L->gu_b4), ldg_ptr(&L->gu_sw), hid, gt0, gt1);
    if (!grid_sync(D.barrier, D.status, S)) return;
    trace_mark(D, tb + 7);
    // P4: gate/up + SiLU
    pro_norm_quant(D.h, nullptr, ldg_ptr(&L->fn), hid, D.eps, S, x_s, sq_s, q_s, sb_s);
    trace_mark(D, tb + 8);
    gemv_phase<kSiluPair>(ldg_ptr(&L->gu_b4), ldg_ptr(&L->gu_sw), S.P.gv_hid, act, gt0, gt1,
                          2 * ffn, ffn, D.act, nullptr, nullptr, leaf_s);
    trace_mark(D, tb + 9);
    prefetch_tiles(ldg_ptr(&L->dn_b4), ldg_ptr(&L->dn_sw), ffn, ht0, ht1);
    if (!grid_sync(D.barrier, D.status, S)) return;
    trace_mark(D, tb + 10);
    // P5: down + residual
    pro_quant(D.act, ffn, q_s, sb_s);
    trace_mark(D, tb + 11);
    gemv_phase<kResidual>(ldg_ptr(&L->dn_b4), ldg_ptr(&L->dn_sw), S.P.gv_ffn, act, ht0, ht1, hid,
                          0, D.h, nullptr, nullptr, leaf_s);
    trace_mark(D, tb + 12);
    if (l + 1 < D.n_layer) {
      prefetch_tiles(ldg_ptr(&D.layers[l + 1].qkv_b4), ldg_ptr(&D.layers[l + 1].qkv_sw), hid,
                     qt0, qt1);
    } else if (flags & HV_STEP_HEAD) {
      int a0, a1;
      row_range(pp_tiles(D.head_rows, 0), &a0, &a1);
      prefetch_tiles(D.head_b4, D.head_sw, hid, a0, min(a1, a0 + 8));
    }
    if (!grid_sync(D.barrier, D.status, S)) return;
    trace_mark(D, tb + 13);
  }

  if (!(flags & HV_STEP_HEAD)) return;
  const int th = 2 + 14 * D.n_layer;
  pro_norm_quant(D.h, nullptr, D.onorm, hid, D.eps, S, x_s, sq_s, q_s, sb_s);
  trace_mark(D, th + 0);
  int a0, a1;
  row_range(pp_tiles(D.head_rows, 0), &a0, &a1);
  float bv = -INFINITY;
  int bi = 0x7FFFFFFF;
  gemv_phase<kHead>(D.head_b4, D.head_sw, S.P.gv_hid, act, a0, a1, D.head_rows, 0, D.logits, &bv,
                    &bi, leaf_s);
  trace_mark(D, th + 1);
  if (!(flags & HV_STEP_ARGMAX)) return;

  // per-CTA argmax, then the last CTA to finish picks the token
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { S.sv[warp] = bv; S.si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kStepWarps; ++w)
        if (S.sv[w] > S.sv[0] || (S.sv[w] == S.sv[0] && S.si[w] < S.si[0])) {
          S.sv[0] = S.sv[w];
          S.si[0] = S.si[w];
        }
      D.amax_v[blockIdx.x] = S.sv[0];
      D.amax_i[blockIdx.x] = S.si[0];
      __threadfence();
      S.flag = (atomicAdd(D.ticket + D.n_kv, 1) == (int)gridDim.x - 1);
    }
    __syncthreads();
    if (S.flag && threadIdx.x == 0) {
      __threadfence();
      float v = -INFINITY;
      int idx = 0x7FFFFFFF;
      for (int c = 0; c < (int)gridDim.x; ++c) {
        const float cv = __ldcg(D.amax_v + c);
        const int ci = __ldcg(D.amax_i + c);
        if (cv > v || (cv == v && ci < idx)) { v = cv; idx = ci; }
      }
      *D.tok = idx;
      const int s = *D.step;
      if (s >= 0 && s <= D.cap) D.gen[s] = idx;      // gen holds cap + 1 entries
      *D.step = s + 1;
      *D.pos = pos + 1;
      D.ticket[D.n_kv] = 0;
    }
  }
  trace_mark(D, th + 2);
}

template <int GS>
static size_t step_smem(int hid, int qdim, int ffn, int cap, int nch) {
  const int kmax = std::max(std::max(hid, qdim), ffn);
  const size_t gemv = (((size_t)kmax + (size_t)(kmax / kBlock) * 8 + 15) & ~size_t(15)) +
                      2 * (size_t)hid * 4 + (size_t)kCBufFloats * 4;
  const int chunk_max = (cap + nch - 1) / nch;
  const size_t lg_floats = ((size_t)chunk_max * GS + 3) & ~size_t(3);
  const size_t attn = sizeof(float) * ((size_t)GS * kHd + 2 * kHd + (GS + 1) * kHd + 4 * GS +
                                       lg_floats + (size_t)kStepWarps * GS * kHd);
  return ((sizeof(StepShared) + 15) & ~size_t(15)) + std::max(gemv, attn);
}

static size_t step_smem_any(int gs, int hid, int qdim, int ffn, int cap, int nch) {
  switch (gs) {
    case 1: return step_smem<1>(hid, qdim, ffn, cap, nch);
    case 2: return step_smem<2>(hid, qdim, ffn, cap, nch);
    case 4: return step_smem<4>(hid, qdim, ffn, cap, nch);
    default: return step_smem<8>(hid, qdim, ffn, cap, nch);
  }
}

static void* step_fn(int gs) {
  switch (gs) {
    case 1: return (void*)k_step<1>;
    case 2: return (void*)k_step<2>;
    case 4: return (void*)k_step<4>;
    default: return (void*)k_step<8>;
  }
}

}  // namespace hv

using namespace hv;

extern "C" {

int hv_step_config(int n_kv, int group, int cap, int* grid, int* threads, size_t* smem,
                   int* chunks, size_t* part_floats) {
  HV_REQUIRE(n_kv > 0 && cap > 0 && grid && threads && chunks && part_floats, HV_E_INVALID,
             "hv_step_config: bad arguments");
  HV_REQUIRE(group == 1 || group == 2 || group == 4 || group == 8, HV_E_UNSUPPORTED,
             "hv_step_config: group size %d (1, 2, 4 or 8)", group);
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  *grid = sms;
  *threads = kStepThreads;
  int nch = sms / n_kv;
  if (nch < 1) nch = 1;
  const int need = (cap + 511) / 512;
  if (nch < need) nch = need;
  *chunks = nch;
  *part_floats = (size_t)n_kv * nch * group * kPartStride;
  if (smem) *smem = 0;
  return HV_OK;
}

int hv_step_plans(int hidden, int qdim, int ffn, void* host_buf, size_t len) {
  HV_REQUIRE(host_buf && len >= sizeof(StepPlans), HV_E_INVALID,
             "hv_step_plans: buffer of %zu bytes needed", sizeof(StepPlans));
  HV_REQUIRE(hidden > 0 && qdim > 0 && ffn > 0 && hidden % kBlock == 0 && qdim % kBlock == 0 &&
                 ffn % kBlock == 0, HV_E_INVALID, "hv_step_plans: bad geometry");
  StepPlans* P = static_cast<StepPlans*>(host_buf);
  memset(P, 0, sizeof(StepPlans));
  const bool ok = pw_make_plan(hidden, &P->pw_hid) && gv_make_plan(hidden / kBlock, &P->gv_hid) &&
                  gv_make_plan(qdim / kBlock, &P->gv_o) && gv_make_plan(ffn / kBlock, &P->gv_ffn);
  HV_REQUIRE(ok, HV_E_UNSUPPORTED, "hv_step_plans: reduction plan does not fit");
  return HV_OK;
}

int hv_step_plans_bytes(size_t* bytes) {
  HV_REQUIRE(bytes, HV_E_INVALID, "hv_step_plans_bytes: null pointer");
  *bytes = sizeof(StepPlans);
  return HV_OK;
}

int hv_step_launch(const hv_step_desc* desc, int flags, void* stream) {
  HV_REQUIRE(desc, HV_E_INVALID, "hv_step_launch: null descriptor");
  hv_step_desc h = *desc;
  HV_REQUIRE(h.head_dim == kHd, HV_E_UNSUPPORTED, "hv_step_launch: head_dim %d", h.head_dim);
  HV_REQUIRE(h.hidden % kBlock == 0 && h.ffn % kBlock == 0, HV_E_UNSUPPORTED,
             "hv_step_launch: hidden/ffn not multiples of 32");
  HV_REQUIRE(h.hidden <= kMaxHidden, HV_E_UNSUPPORTED, "hv_step_launch: hidden %d > %d",
             h.hidden, kMaxHidden);
  HV_REQUIRE(h.plans != nullptr, HV_E_INVALID, "hv_step_launch: plans not set (hv_step_plans)");
  const int gs = h.n_head / h.n_kv;
  HV_REQUIRE(gs == 1 || gs == 2 || gs == 4 || gs == 8, HV_E_UNSUPPORTED,
             "hv_step_launch: group size %d", gs);
  const size_t smem = step_smem_any(gs, h.hidden, h.n_head * kHd, h.ffn, h.cap, h.attn_chunks);
  HV_REQUIRE(smem <= 227 * 1024, HV_E_UNSUPPORTED, "hv_step_launch: needs %zu B of smem", smem);
  void* fn = step_fn(gs);
  {
    // set the function's shared-memory limit once per (group size, device, size)
    static std::mutex mu;
    static size_t done[4][64];
    int dev = 0;
    HV_CUDA(cudaGetDevice(&dev));
    const int gi = gs == 1 ? 0 : gs == 2 ? 1 : gs == 4 ? 2 : 3;
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 0 || dev >= 64 || done[gi][dev] < smem) {
      HV_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      if (dev >= 0 && dev < 64) done[gi][dev] = smem;
    }
  }
  int sms = 0;
  int rc = sm_count(&sms);
  if (rc) return rc;
  void* args[] = {(void*)&h, (void*)&flags};
  HV_CUDA(cudaLaunchCooperativeKernel(fn, dim3(sms), dim3(kStepThreads), args, smem,
                                      (cudaStream_t)stream));
  return HV_OK;
}

}  // extern "C"
