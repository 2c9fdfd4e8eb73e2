/* TEST INFRASTRUCTURE ONLY: plain-C restatement of two reference loops.
 *
 * oracle_topk_ref   -- csrc/kernels/topk_select.cu:17-95 of sparse-offload-infer,
 *                      serially: fp32 max (starting at 0), hi = max + 1e-3f,
 *                      24 bisection steps with a full count per step, then the
 *                      ascending scan writing the first k indices with v >= lo.
 * oracle_gemv_w4a16 -- csrc/kernels/gemv_w4a16_group.cu:77-127 on the CPU: per
 *                      row, per packed word, acc += s * sum(dq * x) in fp32;
 *                      rows split across OpenMP threads.  Used as the CPU
 *                      baseline of the GEMV (dequantisation included).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int e = -1;
      do { ++e; mant <<= 1; } while ((mant & 0x400u) == 0);
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

void oracle_topk_ref(const float* v, int n, int k, int* out_idx, int* out_count) {
  float m = 0.0f;
  for (int i = 0; i < n; ++i) m = fmaxf(m, v[i]);
  volatile float lo = 0.0f, hi = m + 1e-3f; /* volatile: keep every fp32 rounding */
  for (int it = 0; it < 24; ++it) {
    const float mid = 0.5f * (lo + hi);
    int cnt = 0;
    for (int i = 0; i < n; ++i) cnt += (v[i] >= mid);
    if (cnt >= k) lo = mid; else hi = mid;
  }
  const float tau = lo;
  int w = 0;
  for (int i = 0; i < n && w < k; ++i)
    if (v[i] >= tau) out_idx[w++] = i;
  for (int i = w; i < k; ++i) out_idx[i] = -1;
  *out_count = w;
}

static int int4_at(uint32_t word, int j) {
  static const int slot[8] = {0, 4, 1, 5, 2, 6, 3, 7}; /* logical j -> nibble slot (AWQ order) */
  const int n = (int)((word >> (4 * slot[j])) & 0xFu);
  return n >= 8 ? n - 16 : n;
}

void oracle_gemv_w4a16(const uint8_t* Wq, const float* scale, const uint16_t* x, float* y, int64_t N, int64_t K,
                       int64_t group_size, int nthreads) {
  const int64_t words = (K + 7) / 8;
  const int64_t groups = (K + group_size - 1) / group_size;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const uint8_t* row = Wq + n * words * 4;
    float acc = 0.0f;
    for (int64_t w = 0; w < words; ++w) {
      uint32_t word;
      memcpy(&word, row + 4 * w, 4);
      const int64_t k0 = 8 * w;
      const float s = scale[n * groups + k0 / group_size];
      float part = 0.0f;
      for (int j = 0; j < 8 && k0 + j < K; ++j) part += (float)int4_at(word, j) * half_to_float(x[k0 + j]);
      acc += s * part;
    }
    y[n] = acc;
  }
}
