// Split-sequence (flash-decoding) causal attention for batch-1 decode, head_dim 128.
//
// The reference (fda_warp_pos, engine/limited.py:401-404; engine/reference.py:104-118)
// runs one warp per query head and so reads every KV row `group` times with only
// n_head warps in flight. Here one CTA serves one (kv head, chunk of positions) work
// item for the WHOLE query group: each K/V row is read from HBM once, and the
// positions of every kv head are split into enough chunks to fill the SMs. A chunk
// leaves its softmax state (running max m, sum l, unnormalised V-sum) in scratch; the
// last CTA to finish a kv head (atomic ticket) merges the chunks into ctx.
//
// Numerics: logits = (k . q) * scale, softmax by exp(x - max), weighted V sum -- the
// reference's math in another summation order (and CUDA's expf), so the result matches
// engine/reference.py to within float rounding, not bit for bit.
#pragma once

#include <cuda_fp16.h>

#include "hv_common.cuh"

namespace hv {

constexpr int kHd = 128;
constexpr int kAttnChunkMax = 1024;   // positions one work item may hold
constexpr int kPartStride = 132;      // per q head: m, l, 2 pad, acc[128]
constexpr int kAttnMaxChunks = 480;   // chunks per kv head: the merge scratch (2 nch GS + GS
                                      // floats) lies within the 8 x GS x 128 V-sum area
constexpr int kAttnBlock = 20;        // positions per block: block b of a chunk -> warp b % nw

HV_DEV void chunk_bounds(int npos, int nch, int c, int* t0, int* t1) {
  *t0 = (int)(((long long)c * npos) / nch);
  *t1 = (int)(((long long)(c + 1) * npos) / nch);
}

HV_DEV float4 ldg_f4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// The cache's element type: float, or __half for the compressed-KV lane.
template <class KT>
constexpr bool kKvHalf = false;
template <>
constexpr bool kKvHalf<__half> = true;

// A float as stored in the cache (binary16: nearest, ties to even; overflow to infinity).
template <class KT>
HV_DEV KT to_kv(float x);
template <>
HV_DEV float to_kv<float>(float x) { return x; }
template <>
HV_DEV __half to_kv<__half>(float x) { return __float2half_rn(x); }

// x rounded to binary16 and widened back: the value an f16 cache holds for x.
HV_DEV float4 round_half4(float4 v) {
  return make_float4(__half2float(__float2half_rn(v.x)), __half2float(__float2half_rn(v.y)),
                     __half2float(__float2half_rn(v.z)), __half2float(__float2half_rn(v.w)));
}

// Dims 4 lane .. 4 lane + 3 of cache row t, as floats. The cache holds f32, or IEEE
// binary16 (the compressed-KV lane); half -> float is exact, so everything after the load
// is the same arithmetic on the same values either way.
HV_DEV float4 kv_row4(const float* base, int t, int lane) {
  return ldg_f4(base + (size_t)t * kHd + lane * 4);
}
HV_DEV float4 kv_row4(const __half* base, int t, int lane) {
  const uint2 w = __ldg(reinterpret_cast<const uint2*>(base + (size_t)t * kHd + lane * 4));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Sum V values held in every lane across the 32 lanes by recursive halving: after it,
// lane l holds the total of value index `*idx`; lanes whose low (log2(32/V)) bits are
// zero are the representatives of their index.
template <int V>
HV_DEV float halving_reduce(float (&v)[V], int lane, int* idx) {
  int id = 0;
#pragma unroll
  for (int L = 0; L < 5; ++L) {
    const int o = 16 >> L;
    const int cur = (V >> L) > 0 ? (V >> L) : 1;
    if (cur >= 2) {
      const int half = cur / 2;
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int k = 0; k < half; ++k) {
        const float send = up ? v[k] : v[k + half];
        const float keep = up ? v[k + half] : v[k];
        v[k] = keep + __shfl_xor_sync(0xFFFFFFFFu, send, o);
      }
      if (up) id += half;
    } else {
      v[0] += __shfl_xor_sync(0xFFFFFFFFu, v[0], o);
    }
  }
  *idx = id;
  return v[0];
}

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

// Shared memory a work item needs (bytes), for `nwarps` warps.
template <int GS>
constexpr size_t attn_smem_bytes(int nwarps) {
  return sizeof(float) * ((size_t)GS * kHd                 // q
                          + (size_t)kAttnChunkMax * GS      // logits / probabilities
                          + (size_t)nwarps * GS * kHd       // cross-warp V sums
                          + 2 * GS + 2 * kHd);              // stats, k/v row at pos
}

// One work item: positions [t0, t1) of one kv head for its GS query heads.
//   q_s    smem [GS][128]  query heads, already normed and rotated
//   K, V   global [cap][128] rows of this kv head (float, or __half for the f16 cache)
//   pos, kpos_s/vpos_s: if kpos_s is set, row `pos` is taken from it instead of K/V
//   part   global [GS][kPartStride] partial state written by this item
// Block-cooperative; all threads call it.
template <int GS, class KT>
HV_DEV void attn_chunk(const float* q_s, const KT* __restrict__ K,
                       const KT* __restrict__ V, int t0, int t1, float scale, int pos,
                       const float* kpos_s, const float* vpos_s, float* lg_s, float* red_s,
                       float* stat_s, float* __restrict__ part) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int n = t1 - t0;

  // ---- scores: blocks of kAttnBlock positions, block b to warp b % nw, 4 positions at a
  // time; lane l owns dims 4l..4l+3
  float4 qv[GS];
#pragma unroll
  for (int i = 0; i < GS; ++i) qv[i] = reinterpret_cast<const float4*>(q_s + i * kHd)[lane];
  for (int b0 = t0 + warp * kAttnBlock; b0 < t1; b0 += nw * kAttnBlock) {
    const int b1 = min(b0 + kAttnBlock, t1);
    for (int tb = b0; tb < b1; tb += 4) {
      float4 kv[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int t = tb + p;
        if (t < t1) {
          kv[p] = (kpos_s && t == pos) ? reinterpret_cast<const float4*>(kpos_s)[lane]
                                       : kv_row4(K, t, lane);
        } else {
          kv[p] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float v[4 * GS];
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int i = 0; i < GS; ++i) {
          float sc = qv[i].x * kv[p].x;
          sc = fmaf(qv[i].y, kv[p].y, sc);
          sc = fmaf(qv[i].z, kv[p].z, sc);
          sc = fmaf(qv[i].w, kv[p].w, sc);
          v[p * GS + i] = sc;
        }
      int idx;
      const float tot = halving_reduce<4 * GS>(v, lane, &idx);
      constexpr int dup = 32 / (4 * GS);
      if ((lane & (dup - 1)) == 0) {
        const int p = idx / GS, i = idx % GS;
        const int t = tb + p;
        if (t < t1) lg_s[(t - t0) * GS + i] = tot * scale;
      }
    }
  }
  __syncthreads();

  // ---- per-head max and exp: warp i handles head i
  for (int i = warp; i < GS; i += nw) {
    float m = -INFINITY;
    for (int t = lane; t < n; t += 32) m = fmaxf(m, lg_s[t * GS + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    float l = 0.f;
    for (int t = lane; t < n; t += 32) {
      const float e = (n > 0) ? expf(lg_s[t * GS + i] - m) : 0.f;
      lg_s[t * GS + i] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xFFFFFFFFu, l, o);
    if (lane == 0) { stat_s[2 * i] = m; stat_s[2 * i + 1] = l; }
  }
  __syncthreads();

  // ---- probability-weighted V sum: the same blocks to the same warps, positions in
  // order within a block; lane owns 4 dims
  float4 acc[GS];
#pragma unroll
  for (int i = 0; i < GS; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int b0 = t0 + warp * kAttnBlock; b0 < t1; b0 += nw * kAttnBlock) {
    const int b1 = min(b0 + kAttnBlock, t1);
    for (int tb = b0; tb < b1; tb += 4) {
      float4 vv[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int t = tb + p;
        if (t < t1) {
          vv[p] = (vpos_s && t == pos) ? reinterpret_cast<const float4*>(vpos_s)[lane]
                                       : kv_row4(V, t, lane);
        } else {
          vv[p] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int t = tb + p;
        if (t < t1) {
#pragma unroll
          for (int i = 0; i < GS; ++i) {
            const float w = lg_s[(t - t0) * GS + i];
            acc[i].x = fmaf(w, vv[p].x, acc[i].x);
            acc[i].y = fmaf(w, vv[p].y, acc[i].y);
            acc[i].z = fmaf(w, vv[p].z, acc[i].z);
            acc[i].w = fmaf(w, vv[p].w, acc[i].w);
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < GS; ++i)
    reinterpret_cast<float4*>(red_s + ((size_t)warp * GS + i) * kHd)[lane] = acc[i];
  __syncthreads();
  for (int e = threadIdx.x; e < GS * kHd; e += blockDim.x) {
    float s = 0.f;
    for (int w = 0; w < nw; ++w) s += red_s[(size_t)w * GS * kHd + e];
    const int i = e / kHd, d = e % kHd;
    part[i * kPartStride + 4 + d] = s;
  }
  if (threadIdx.x < GS) {
    part[threadIdx.x * kPartStride + 0] = (n > 0) ? stat_s[2 * threadIdx.x] : -INFINITY;
    part[threadIdx.x * kPartStride + 1] = (n > 0) ? stat_s[2 * threadIdx.x + 1] : 0.f;
  }
}

// Merge the nch chunk states of one kv head into ctx rows [GS][128]. Reads the
// partials through L2 (they were written by other CTAs): first every chunk's (m, l) in
// parallel, then per head the global max and weights, then each output element sums
// its chunks with all loads of a batch in flight. `w_s` is shared scratch of
// 2 * nch * GS + GS floats. Cooperative over the threads of Sync. With kQuant the rows
// are not stored as floats but quantised per 32 values (quant_a8s, one warp per block):
// int8 into q_out[i * 128 + d], (scale bits, block sum) into sb_out[(i * 128 + d) / 32]
// (Sync's thread count must then be a multiple of 32).
template <int GS, class Sync = SyncBlock, bool kQuant = false>
HV_DEV void attn_merge(const float* part_head, int nch, float* __restrict__ ctx, float* w_s,
                       int8_t* __restrict__ q_out = nullptr, int2* __restrict__ sb_out = nullptr) {
  float* l_s = w_s + nch * GS;                    // l of (c, i)
  float* inv_s = l_s + nch * GS;                  // 1 / L per head
  const int nt = Sync::threads();
  for (int e = threadIdx.x; e < nch * GS; e += nt) {
    w_s[e] = __ldcg(part_head + (size_t)e * kPartStride);          // m of (c, i)
    l_s[e] = __ldcg(part_head + (size_t)e * kPartStride + 1);
  }
  Sync::sync();
  if (threadIdx.x < GS) {
    const int i = threadIdx.x;
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, w_s[c * GS + i]);
    float L = 0.f;
    for (int c = 0; c < nch; ++c) {
      const float w = expf(w_s[c * GS + i] - M);
      L = fmaf(w, l_s[c * GS + i], L);
      w_s[c * GS + i] = w;
    }
    inv_s[i] = 1.0f / L;
  }
  Sync::sync();
  for (int e = threadIdx.x; e < GS * kHd; e += nt) {
    const int i = e / kHd, d = e % kHd;
    float o = 0.f;
    for (int c0 = 0; c0 < nch; c0 += 8) {
      float a[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        a[k] = (c0 + k < nch)
                   ? __ldcg(part_head + ((size_t)(c0 + k) * GS + i) * kPartStride + 4 + d) : 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (c0 + k < nch) o = fmaf(w_s[(c0 + k) * GS + i], a[k], o);
    }
    const float val = o * inv_s[i];
    if constexpr (kQuant) {
      int8_t q8;
      float sc;
      int bs;
      quant_block_warp(val, threadIdx.x & 31, &q8, &sc, &bs);
      q_out[e] = q8;
      if ((threadIdx.x & 31) == 0) sb_out[e / 32] = make_int2(__float_as_int(sc), bs);
    } else {
      ctx[i * kHd + d] = val;
    }
  }
}

}  // namespace hv
