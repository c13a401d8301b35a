// Attention helpers shared by the eager kernels, the batched prefill and the fused step:
// the even split of positions into chunks, the cache's element type (float, or IEEE
// binary16 for the compressed-KV lane) and its rounding, and the per-head q/k RMSNorm +
// RoPE of one warp. The attention itself (scores, softmax and the weighted V sum in
// engine/reference.py:104-118's order) is in attn_exact.cuh.
#pragma once

#include <cuda_fp16.h>

#include "hv_common.cuh"

namespace hv {

constexpr int kHd = 128;
constexpr int kAttnChunkMax = 1024;   // positions one eager attention chunk may hold
constexpr int kAttnBlock = 20;        // KV rows per ring slot of the fused step's scores

// Positions [t0, t1) of chunk c when npos positions are split evenly into nch chunks.
HV_DEV void chunk_bounds(int npos, int nch, int c, int* t0, int* t1) {
  *t0 = (int)(((long long)c * npos) / nch);
  *t1 = (int)(((long long)(c + 1) * npos) / nch);
}

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

}  // namespace hv
