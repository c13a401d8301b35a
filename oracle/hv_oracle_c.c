/* ORACLE (test infrastructure only) -- a C restatement of the reference's W4A8 GEMV
 * (engine/reference.py:62-84) for the model sizes where numpy is too slow.
 *
 * y[n] = (+0) + pairwise_b( f32(f32(sw[n,b] * sa[b]) * f32(idot[n,b])) ), the block sum
 * in numpy's float32 pairwise order (leaves of <= 128 terms; a leaf of >= 8 terms keeps
 * eight strided accumulators folded as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) and then adds
 * its n % 8 tail; larger ranges split at n/2 rounded down to a multiple of 8).
 * Compiled with -ffp-contract=off so no multiply-add is fused. Checked bit for bit
 * against the numpy oracle and the reference's golden vectors (tests/test_oracle_c.py).
 *
 * Also restated here, because the reference's attention and SiLU call them
 * (engine/reference.py:99, 112-116) and their results depend on the library build:
 *  - numpy's float32 exp (hvo_np_expf), and
 *  - the order in which OpenBLAS's sgemv forms each row dot of `keys @ q`
 *    (hvo_blas_rowdots).
 * Both are pinned bit for bit against the numpy/OpenBLAS of the host that produced the
 * golden vectors (tests/test_oracle_c.py).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* numpy's float32 exp, restated from numpy's published SIMD algorithm (numpy 2.x,
 * numpy/_core/src/umath/loops_exponent_log.dispatch.c.src, simd_exp_f32: the AVX512F /
 * AVX2+FMA3 path numpy dispatches to on x86-64 hosts that have them):
 *   n = rint(x * log2(e)) by the 1.5 * 2^23 magic-number add and subtract;
 *   r = x + n * (-ln2_hi) + n * (-ln2_lo) (Cody-Waite, fused multiply-adds);
 *   exp(r) ~ P5(r) / Q2(r), Horner with fused multiply-adds, one IEEE division;
 *   result = that quotient * 2^n, rounded once.
 * x >= 88.72283935546875 gives +inf, x <= -103.97208404541015625 gives +0, NaN stays NaN.
 * Equal to np.exp on every float32 of [-104, 89] on an AVX-512 host (numpy 2.3.5). */
float hvo_np_expf(float x) {
  if (x != x) return x;
  if (x >= 88.72283935546875f) return INFINITY;
  if (x <= -103.97208404541015625f) return 0.0f;
  float n = x * 1.442695040888963407359924681001892137f;
  n = n + 0x1.8p23f;
  n = n - 0x1.8p23f;
  float r = fmaf(n, -6.93145752e-1f, x);
  r = fmaf(n, -1.42860677e-6f, r);
  r = fmaf(n, 0.0f, r);
  float p = fmaf(5.082762527590693718096e-04f, r, 6.757896990527504603057e-03f);
  p = fmaf(p, r, 5.114512081637298353406e-02f);
  p = fmaf(p, r, 2.473615434895520810817e-01f);
  p = fmaf(p, r, 7.257664613233124478488e-01f);
  p = fmaf(p, r, 9.999999999980870924916e-01f);
  float q = fmaf(2.159509375685829852307e-02f, r, -2.742335390411667452936e-01f);
  q = fmaf(q, r, 1.0f);
  return (float)ldexp((double)(p / q), (int)n);
}

void hvo_np_exp_arr(const float* x, float* y, long n) {
  for (long i = 0; i < n; ++i) y[i] = hvo_np_expf(x[i]);
}

/* The three row-dot kernels of OpenBLAS's single-precision gemv ("T" form: one output per
 * matrix row of m = 128 contiguous floats), as observed on the reference's host (OpenBLAS
 * 0.3.30 through numpy; identified by matching its outputs bit for bit):
 *   kind 0, rows in whole groups of 4: eight lanes, lane j accumulates elements j, j+8,
 *     ... with fused multiply-adds from +0; then s_k = a_k + a_{k+4} and
 *     (s_0 + s_1) + (s_2 + s_3);
 *   kind 1, the next two rows when a run has 2 or 3 left over: four lanes, lane j adds the
 *     rounded products of elements j, j+4, ... from +0; then (a_0 + a_1) + (a_2 + a_3);
 *   kind 2, the last row when a run has 1 or 3 left over: kind 0's lanes and fold, but
 *     each product rounded before the add. */
static float rowdot(const float* a, const float* x, int m, int kind) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (kind == 1) {
    for (int i = 0; i < m; ++i) acc[i & 3] = acc[i & 3] + a[i] * x[i];
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
  for (int i = 0; i < m; ++i)
    acc[i & 7] = kind == 0 ? fmaf(a[i], x[i], acc[i & 7]) : acc[i & 7] + a[i] * x[i];
  float s[4];
  for (int k = 0; k < 4; ++k) s[k] = acc[k] + acc[k + 4];
  return (s[0] + s[1]) + (s[2] + s[3]);
}

/* Kind of row t of a T-row gemv: OpenBLAS runs the rows as one run, or -- when
 * 128 * T >= 460800 -- as `threads` runs of ceil(rows left / runs left) rows (at least 4)
 * on the host's threads; inside a run, whole groups of 4 rows use kind 0 and the 1 to 3
 * rows left over use kinds 1, 1 and 2 as above. */
int hvo_blas_row_kind(int T, int t, int threads) {
  int nrun = (128L * T >= 460800L && threads > 1) ? threads : 1;
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

/* out[t] = row t of K (T x 128, row stride ldk floats) dotted with x, each row in the
 * order OpenBLAS uses for it. */
void hvo_blas_rowdots(const float* K, long ldk, const float* x, float* out, int T,
                      int threads) {
  for (int t = 0; t < T; ++t)
    out[t] = rowdot(K + (long)t * ldk, x, 128, hvo_blas_row_kind(T, t, threads));
}

static float leaf_sum(const float* x, long n) {
  if (n < 8) {
    float r = 0.0f;
    for (long i = 0; i < n; ++i) r = r + x[i];
    return r;
  }
  float r[8];
  for (int j = 0; j < 8; ++j) r[j] = x[j];
  long i = 8;
  for (; i < n - (n % 8); i += 8)
    for (int j = 0; j < 8; ++j) r[j] = r[j] + x[i + j];
  float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
  for (; i < n; ++i) res = res + x[i];
  return res;
}

static float pairwise(const float* x, long n) {
  if (n <= 128) return leaf_sum(x, n);
  long n2 = n / 2;
  n2 -= n2 % 8;
  return pairwise(x, n2) + pairwise(x + n2, n - n2);
}

float hvo_pairwise_sum(const float* x, long n) { return 0.0f + pairwise(x, n); }

/* idot may be NULL. */
void hvo_gemv(const int8_t* qa, const float* sa, const uint32_t* packed, const float* scale,
              long n, long k, float* y, int32_t* idot) {
  const long nb = k / 32;
#pragma omp parallel
  {
    float* c = (float*)malloc(sizeof(float) * (size_t)nb);
#pragma omp for schedule(static)
    for (long row = 0; row < n; ++row) {
      const uint32_t* w = packed + row * (k / 8);
      const float* s = scale + row * nb;
      for (long b = 0; b < nb; ++b) {
        int32_t acc = 0;
        for (int t = 0; t < 4; ++t) {
          const uint32_t word = w[b * 4 + t];
          const int8_t* a = qa + b * 32 + t * 8;
          for (int byte = 0; byte < 4; ++byte) {
            int lo = (int)((word >> (8 * byte)) & 15u);
            int hi = (int)((word >> (8 * byte + 4)) & 15u);
            lo = lo >= 8 ? lo - 16 : lo;
            hi = hi >= 8 ? hi - 16 : hi;
            acc += lo * a[byte] + hi * a[4 + byte];
          }
        }
        if (idot) idot[row * nb + b] = acc;
        const float sws = s[b] * sa[b];
        c[b] = sws * (float)acc;
      }
      y[row] = 0.0f + pairwise(c, nb);
    }
    free(c);
  }
}

/* engine/limited.py:40-58 restated: per-32 s = f32(max|w| / 7) (0 -> 1),
 * q = clip(rint(f32(w / s)), -7, 7) (round half to even), byte-sliced nibble packing. */
void hvo_quantize_w4(const float* w, long n, long k, uint32_t* packed, float* scale) {
  const long nb = k / 32;
#pragma omp parallel for schedule(static)
  for (long row = 0; row < n; ++row) {
    for (long b = 0; b < nb; ++b) {
      const float* x = w + row * k + b * 32;
      float mx = 0.0f;
      for (int i = 0; i < 32; ++i) {
        const float a = x[i] < 0 ? -x[i] : x[i];
        if (a > mx) mx = a;
      }
      float s = mx / 7.0f;
      if (s == 0.0f) s = 1.0f;
      uint32_t words[4] = {0, 0, 0, 0};
      for (int i = 0; i < 32; ++i) {
        float r = __builtin_rintf(x[i] / s);
        if (r > 7.0f) r = 7.0f;
        if (r < -7.0f) r = -7.0f;
        const uint32_t nib = (uint32_t)((int)r) & 15u;
        const int j = i % 8;
        const int shift = (j < 4) ? (8 * j) : (8 * (j - 4) + 4);
        words[i / 8] |= nib << shift;
      }
      for (int t = 0; t < 4; ++t) packed[row * (k / 8) + b * 4 + t] = words[t];
      scale[row * nb + b] = s;
    }
  }
}
