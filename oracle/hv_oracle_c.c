/* ORACLE (test infrastructure only) -- a C restatement of the reference's W4A8 GEMV
 * (engine/reference.py:62-84) for the model sizes where numpy is too slow.
 *
 * y[n] = (+0) + pairwise_b( f32(f32(sw[n,b] * sa[b]) * f32(idot[n,b])) ), the block sum
 * in numpy's float32 pairwise order (leaves of <= 128 terms; a leaf of >= 8 terms keeps
 * eight strided accumulators folded as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) and then adds
 * its n % 8 tail; larger ranges split at n/2 rounded down to a multiple of 8).
 * Compiled with -ffp-contract=off so no multiply-add is fused. Checked bit for bit
 * against the numpy oracle and the reference's golden vectors (tests/test_oracle_c.py).
 */
#include <stdint.h>
#include <stdlib.h>

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
