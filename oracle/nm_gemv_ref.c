/*
 * ORACLE -- test infrastructure, not product code (see oracle/__init__.py).
 *
 * C restatement of the reference shared-mask N:M GEMV kernel
 * (triton_spmv.py:81-115): the wrapper's grid of programs
 * (row block x block of `gpp` groups, triton_spmv.py:298-302); inside a
 * program, groups in order and kept slots in order with an fp32 fused
 * multiply-add (the kernel's fma.rn.f32, triton_spmv.py:24-35); program
 * partials added to the fp32 output (the kernel's atomic_add, here in
 * program order, so the result is deterministic).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

/* out[h] (fp32) = sum over programs; vec [K], mat_data [w, h] (fp16 bits),
 * mat_index [w/n, n].  Rows [row_begin, row_end) only (for threading). */
void nm_gemv_ref_rows(const uint16_t* vec, const uint16_t* mat_data, const uint8_t* mat_index, float* out,
                      int64_t K, int64_t w, int64_t h, int32_t n, int32_t m, int32_t gpp, int64_t row_begin,
                      int64_t row_end) {
  const int64_t G = w / n;
  (void)K;
  for (int64_t r = row_begin; r < row_end; ++r) out[r] = 0.0f;
  for (int64_t g0 = 0; g0 < G; g0 += gpp) {
    const int64_t g1 = g0 + gpp < G ? g0 + gpp : G;
    for (int64_t r = row_begin; r < row_end; ++r) {
      float acc = 0.0f;
      for (int64_t g = g0; g < g1; ++g) {
        for (int32_t i = 0; i < n; ++i) {
          const float xi = f16_to_f32(vec[g * m + mat_index[g * n + i]]);
          const float wi = f16_to_f32(mat_data[(g * n + i) * h + r]);
          acc = fmaf(wi, xi, acc);
        }
      }
      out[r] += acc;
    }
  }
}

void nm_gemv_ref(const uint16_t* vec, const uint16_t* mat_data, const uint8_t* mat_index, float* out, int64_t K,
                 int64_t w, int64_t h, int32_t n, int32_t m, int32_t gpp) {
  nm_gemv_ref_rows(vec, mat_data, mat_index, out, K, w, h, n, m, gpp, 0, h);
}
