// Shared device helpers for the hive_b200 kernels (sm_100a).
//
// Numerics follow HIVE Limited's numpy reference (engine/reference.py) operation by
// operation. Every float operation on a bit-exact path is written with an explicit
// round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn) so that nvcc
// can never contract a multiply and an add into an FMA: numpy rounds each one.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define HV_DEV __device__ __forceinline__
#define HV_HD __host__ __device__ inline

namespace hv {

constexpr int kBlock = 32;      // weights / activations per scale
constexpr int kPwLeaf = 128;    // numpy's pairwise-summation leaf size
constexpr int kPwMaxLeaf = 512; // leaves a plan may hold (n <= 65536)

// ---------------------------------------------------------------------------
// numpy's float32 pairwise summation, restated.
//
// pairwise(x[0:n]): n <= 128 is one leaf; otherwise split at n2 = n/2 rounded down to
// a multiple of 8 and add pairwise(left) + pairwise(right). A leaf of n < 8 values is a
// sequential sum from +0. A leaf of n >= 8 keeps eight strided accumulators
// r[j] = x[j] + x[j+8] + x[j+16] + ... (in order), folds them as
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)), then adds the n % 8 tail in order. The reduction
// result is (+0) + pairwise(x). A plan lists the leaves left to right and, after each
// leaf, how many '+' of the recursion close there (postfix order).
// ---------------------------------------------------------------------------
struct PwPlan {
  int nleaf;
  int balanced;   // every split halves exactly and nleaf is a power of two <= 64
  int start[kPwMaxLeaf];
  short len[kPwMaxLeaf];
  unsigned char pops[kPwMaxLeaf];
};

// Builds the plan for n values. Returns false if it does not fit. Runs on the host so
// kernels receive a finished plan.
HV_HD bool pw_make_plan(int n, PwPlan* p) {
  // explicit DFS stack: kind 0 = node (s, m), kind 1 = '+'
  int sk[64], ss[64], sm[64];
  int sp = 0, nl = 0;
  sk[0] = 0; ss[0] = 0; sm[0] = n; sp = 1;
  while (sp > 0) {
    --sp;
    const int k = sk[sp], s = ss[sp], m = sm[sp];
    if (k == 1) {
      p->pops[nl - 1]++;
    } else if (m <= kPwLeaf) {
      if (nl >= kPwMaxLeaf) return false;
      p->start[nl] = s; p->len[nl] = (short)m; p->pops[nl] = 0; ++nl;
    } else {
      if (sp + 3 > 64) return false;
      int m2 = m / 2; m2 -= m2 % 8;
      sk[sp] = 1; ss[sp] = 0; sm[sp] = 0; ++sp;
      sk[sp] = 0; ss[sp] = s + m2; sm[sp] = m - m2; ++sp;
      sk[sp] = 0; ss[sp] = s; sm[sp] = m2; ++sp;
    }
  }
  p->nleaf = nl;
  // balanced: all leaves equal, a power-of-two count, each split exactly in half -- then
  // the recursion's '+' is the xor-butterfly over leaf indices
  bool bal = nl <= 64 && (nl & (nl - 1)) == 0;
  for (int i = 0; bal && i < nl; ++i) bal = p->len[i] == p->len[0] && p->start[i] == i * p->len[0];
  p->balanced = bal ? 1 : 0;
  return true;
}

// Folds leaf values with the plan's postfix '+' (one thread); returns (+0) + total.
HV_DEV float pw_fold(const PwPlan* p, const float* leafval) {
  float st[32];
  int sp = 0;
  for (int i = 0; i < p->nleaf; ++i) {
    st[sp++] = leafval[i];
    for (int k = 0; k < p->pops[i]; ++k) {
      const float b = st[--sp];
      const float a = st[--sp];
      st[sp++] = __fadd_rn(a, b);
    }
  }
  return __fadd_rn(0.0f, st[0]);
}

// Sum of one leaf of `len` values x[0..len) held in shared memory, computed by the 8
// lanes of an aligned lane group (sub = lane % 8). Every lane of the group returns it.
HV_DEV float pw_leaf8(const float* x, int len, int sub) {
  const unsigned gmask = 0xFFu << ((threadIdx.x & 31) & ~7);
  float r;
  int full = len - (len % 8);
  if (len >= 8) {
    r = x[sub];
    for (int i = 8 + sub; i < full; i += 8) r = __fadd_rn(r, x[i]);
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 1, 8));
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 2, 8));
    r = __fadd_rn(r, __shfl_xor_sync(gmask, r, 4, 8));
    for (int i = full; i < len; ++i) r = __fadd_rn(r, x[i]);
  } else {
    r = 0.0f;
    for (int i = 0; i < len; ++i) r = __fadd_rn(r, x[i]);
  }
  return r;
}

// The threads that run a block-cooperative routine and how they synchronise: the whole
// block (__syncthreads), or the first N threads on named barrier ID (warp-specialised
// kernels whose other warps never join).
struct SyncBlock {
  HV_DEV static void sync() { __syncthreads(); }
  HV_DEV static int threads() { return blockDim.x; }
};
template <int N, int ID>
struct SyncNamed {
  static_assert(N % 32 == 0 && ID > 0 && ID < 16, "named barrier of whole warps");
  HV_DEV static void sync() { asm volatile("bar.sync %0, %1;" :: "n"(ID), "n"(N) : "memory"); }
  HV_DEV static int threads() { return N; }
};

// Block-cooperative numpy sum of x[0..n) in shared memory. `plan` and `leafval`
// (kPwMaxLeaf floats) are shared scratch; the plan must already be built for n.
// All threads of Sync must call it; the result is returned to every thread.
template <class Sync = SyncBlock>
HV_DEV float block_pw_sum(const float* x, const PwPlan* plan, float* leafval,
                          float* result) {
  const int nthreads = Sync::threads();
  const int groups = nthreads / 8;
  const int g = threadIdx.x / 8, sub = threadIdx.x % 8;
  for (int leaf = g; leaf < ((plan->nleaf + groups - 1) / groups) * groups; leaf += groups) {
    // every lane of a full warp takes part in the shuffles, even past the last leaf
    const bool live = leaf < plan->nleaf;
    const int s = live ? plan->start[leaf] : 0;
    const int len = live ? plan->len[leaf] : 8;
    const float v = pw_leaf8(x + s, len, sub);
    if (live && sub == 0) leafval[leaf] = v;
  }
  Sync::sync();
  if (plan->balanced) {
    // one warp folds: leaf i -> lane i % 32 (two per lane when 64), then the butterfly
    if (threadIdx.x < 32) {
      const int n = plan->nleaf;
      const int lane = threadIdx.x;
      float v;
      if (n == 64) {
        v = __fadd_rn(leafval[2 * lane], leafval[2 * lane + 1]);
      } else {
        v = (lane < n) ? leafval[lane] : 0.0f;
      }
      const int m = n == 64 ? 32 : n;
      for (int o = 1; o < m; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
      if (lane == 0) *result = __fadd_rn(0.0f, v);
    }
  } else if (threadIdx.x == 0) {
    *result = pw_fold(plan, leafval);
  }
  Sync::sync();
  return *result;
}

// ---------------------------------------------------------------------------
// per-32 activation quantisation (engine/reference.py:44-59, quant_a8s)
//   s = f32(max|a| / 127), s == 0 -> 1
//   q = trunc(f32(f32(a / s) + (a < 0 ? -0.5 : 0.5))), clipped to +-127
//   bsum = sum of q (int32)
// One warp quantises one block: lane i holds a[32b + i].
// ---------------------------------------------------------------------------
HV_DEV void quant_block_warp(float a, int lane, int8_t* q_out, float* s_out, int* bsum_out) {
  float mx = fabsf(a);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  float s = __fdiv_rn(mx, 127.0f);
  if (s == 0.0f) s = 1.0f;
  const float half = (a < 0.0f) ? -0.5f : 0.5f;
  float t = truncf(__fadd_rn(__fdiv_rn(a, s), half));
  int q = (int)t;
  q = q > 127 ? 127 : (q < -127 ? -127 : q);
  int sum = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
  *q_out = (int8_t)q;
  if (lane == 0) { *s_out = s; *bsum_out = sum; }
}

// ---------------------------------------------------------------------------
// W4A8 block dot.
//
// Packed word t of a 32-weight block holds q[8t+b] in the low nibble of byte b and
// q[8t+4+b] in the high nibble. With u = (w & 0x0F0F0F0F) ^ 0x08080808 each byte is
// q + 8 in [0, 15], lined up with activation bytes a[8t..8t+3]; the high nibbles, masked
// in place, are 16 * (q + 8) lined up with a[8t+4..8t+7]. Unsigned x signed dp4a then
// gives sum((q+8)*a); subtracting 8 * sum(a) (the block sum quant_a8s stores) leaves the
// exact int32 dot.
// ---------------------------------------------------------------------------
HV_DEV int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

HV_DEV unsigned lop_lo(unsigned w) {   // (w & 0x0F0F0F0F) ^ 0x08080808
  unsigned d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(w), "r"(0x0F0F0F0Fu), "r"(0x08080808u));
  return d;
}
HV_DEV unsigned lop_hi(unsigned w) {   // (w & 0xF0F0F0F0) ^ 0x80808080
  unsigned d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(w), "r"(0xF0F0F0F0u), "r"(0x80808080u));
  return d;
}

// exact int32 dot of one 32-block: nib = 4 packed words, a0/a1 = the 32 int8
// activations as 8 words, bsum = their sum
HV_DEV int block_dot(uint4 nib, uint4 a0, uint4 a1, int bsum) {
  int lo = 0, hi = 0;
  lo = dp4a_us(lop_lo(nib.x), (int)a0.x, lo);
  hi = dp4a_us(lop_hi(nib.x), (int)a0.y, hi);
  lo = dp4a_us(lop_lo(nib.y), (int)a0.z, lo);
  hi = dp4a_us(lop_hi(nib.y), (int)a0.w, hi);
  lo = dp4a_us(lop_lo(nib.z), (int)a1.x, lo);
  hi = dp4a_us(lop_hi(nib.z), (int)a1.y, hi);
  lo = dp4a_us(lop_lo(nib.w), (int)a1.z, lo);
  hi = dp4a_us(lop_hi(nib.w), (int)a1.w, hi);
  return lo + (hi >> 4) - 8 * bsum;
}

// c = f32(f32(s_w * s_a) * f32(idot))  (engine/reference.py:71)
HV_DEV float block_term(float sw, float sa, int idot) {
  return __fmul_rn(__fmul_rn(sw, sa), __int2float_rn(idot));
}

// read-only 128-bit / 32-bit global loads that bypass L1 allocation
HV_DEV uint4 ldg_stream4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
HV_DEV float ldg_stream1(const float* p) {
  float v;
  asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// L2 prefetch of a contiguous byte range through the bulk-copy unit (no shared memory,
// no completion tracking). Address and size are rounded to 16 bytes inside the range's
// 256-byte-padded allocation.
HV_DEV void prefetch_l2(const void* p, size_t bytes) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  uintptr_t a0 = a & ~uintptr_t(15);
  size_t n = (bytes + (a - a0) + 15) & ~size_t(15);
  while (n > 0) {
    const unsigned chunk = n > (1u << 20) ? (1u << 20) : (unsigned)n;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(a0), "r"(chunk) : "memory");
    a0 += chunk;
    n -= chunk;
  }
}

// Per-32 quantisation with 8 lanes per block: lane (b = lane / 8, sub = lane % 8) holds
// v = values 4 sub .. 4 sub + 3 of block b. Same arithmetic as quant_block_warp (the
// max and the block sum are exact, so the grouping does not change any bit). Returns the
// four int8 values packed little-endian; lanes with sub == 0 receive the scale and sum.
HV_DEV unsigned quant_block_8lanes(float4 v, float* s_out, int* bsum_out) {
  const unsigned gmask = 0xFFu << ((threadIdx.x & 31) & ~7);
  float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  mx = fmaxf(mx, __shfl_xor_sync(gmask, mx, 1, 8));
  mx = fmaxf(mx, __shfl_xor_sync(gmask, mx, 2, 8));
  mx = fmaxf(mx, __shfl_xor_sync(gmask, mx, 4, 8));
  float s = __fdiv_rn(mx, 127.0f);
  if (s == 0.0f) s = 1.0f;
  const float a[4] = {v.x, v.y, v.z, v.w};
  unsigned packed = 0;
  int sum = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float half = (a[i] < 0.0f) ? -0.5f : 0.5f;
    int q = (int)truncf(__fadd_rn(__fdiv_rn(a[i], s), half));
    q = q > 127 ? 127 : (q < -127 ? -127 : q);
    sum += q;
    packed |= ((unsigned)q & 0xFFu) << (8 * i);
  }
  sum += __shfl_xor_sync(gmask, sum, 1, 8);
  sum += __shfl_xor_sync(gmask, sum, 2, 8);
  sum += __shfl_xor_sync(gmask, sum, 4, 8);
  *s_out = s;
  *bsum_out = sum;
  return packed;
}

// ---------------------------------------------------------------------------
// numpy's float32 exp (numpy/_core/src/umath/loops_exponent_log.dispatch.c.src,
// simd_exp_f32, the AVX512F / AVX2+FMA3 kernel numpy runs on x86-64 hosts that have
// them): n = rint(x log2 e) by the 1.5 * 2^23 add and subtract, a Cody-Waite reduction
// r = x - n ln2 in fused multiply-adds, exp(r) ~ P5(r) / Q2(r) (Horner, fused
// multiply-adds, one IEEE division), then the quotient times 2^n rounded once.
// x >= 88.72283935546875 gives +inf, x <= -103.97208404541015625 gives +0, NaN stays NaN.
// ---------------------------------------------------------------------------
HV_DEV float np_expf(float x) {
  if (x != x) return x;
  if (x >= 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x <= -103.97208404541015625f) return 0.0f;
  float n = __fmul_rn(x, 1.442695040888963407359924681001892137f);
  n = __fadd_rn(n, 0x1.8p23f);
  n = __fsub_rn(n, 0x1.8p23f);
  float r = __fmaf_rn(n, -6.93145752e-1f, x);
  r = __fmaf_rn(n, -1.42860677e-6f, r);
  r = __fmaf_rn(n, 0.0f, r);
  float p = __fmaf_rn(5.082762527590693718096e-04f, r, 6.757896990527504603057e-03f);
  p = __fmaf_rn(p, r, 5.114512081637298353406e-02f);
  p = __fmaf_rn(p, r, 2.473615434895520810817e-01f);
  p = __fmaf_rn(p, r, 7.257664613233124478488e-01f);
  p = __fmaf_rn(p, r, 9.999999999980870924916e-01f);
  float q = __fmaf_rn(2.159509375685829852307e-02f, r, -2.742335390411667452936e-01f);
  q = __fmaf_rn(q, r, 1.0f);
  const float quot = __fdiv_rn(p, q);
  // quot * 2^n: exact in double (n in [-150, 128]), then one rounding to float
  const double two_n = __longlong_as_double((long long)((int)n + 1023) << 52);
  return __double2float_rn(__dmul_rn((double)quot, two_n));
}

// ---------------------------------------------------------------------------
// SiLU * up (engine/reference.py:96-101): sigma by the sign-split exp form, exp being
// numpy's (np_expf), every operation rounded as numpy rounds it.
// ---------------------------------------------------------------------------
HV_DEV float silu_mul1(float g, float u) {
  const float sgn = (g < 0.0f) ? -1.0f : 1.0f;
  const float e = np_expf(-__fmul_rn(sgn, g));
  const float r = __fdiv_rn(__fsub_rn(1.0f, e), __fadd_rn(1.0f, e));
  const float sig = __fmul_rn(0.5f, __fadd_rn(1.0f, __fmul_rn(sgn, r)));
  return __fmul_rn(__fmul_rn(g, sig), u);
}

}  // namespace hv
