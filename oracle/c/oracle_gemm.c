/*
 * CPU restatement of the MLX-affine small-M GEMM (test and CPU-baseline infrastructure only;
 * the library never links it).
 *
 * Follows Worker/Sources/SmallMGEMM/SmallMGEMM.swift:662-755 (smallm_gemv_affine): per group
 * of 64 along K, acc += scale * sum(x * q) + bias * sum(x), fp32 accumulation; codes are
 * packed low bits first in uint32 words (:658-661).  Dense rows (bf16 bit patterns) follow
 * the dense GEMV (:585-656).  Parallel over output rows with OpenMP; x and the results are
 * fp32 (the caller rounds).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t v) {
  uint32_t u = (uint32_t)v << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* Rows of x are processed in blocks of this many, each block's accumulators in registers. */
#define ORACLE_MB 16

/* Summation order along K: 0 ascending, 1 descending (both are valid restatements; their
 * difference measures how much fp32 rounding order alone moves a result). */
static int g_reverse = 0;
void oracle_set_reverse(int r) { g_reverse = r ? 1 : 0; }

/* out[M, N] = x[M, K] . W^T, W MLX-affine (bits 4 | 8), scales/biases as bf16 bits.
 * Returns 0, or -1 when the group sums cannot be allocated. */
int oracle_qgemm_bf16(int M, int N, int K, int bits, const float* x, const uint32_t* w, const uint16_t* scales,
                      const uint16_t* biases, float* out) {
  const int G = K / 64, per = 32 / bits, wpr = K / per;
  const uint32_t mask = (1u << bits) - 1u;
  /* per-row group sums of x, shared by all output rows */
  float* xsum = (float*)malloc((size_t)(M > 0 ? M : 1) * (G > 0 ? G : 1) * sizeof(float));
  if (!xsum) return -1;
  for (int m = 0; m < M; ++m)
    for (int g = 0; g < G; ++g) {
      float s = 0.0f;
      for (int k = 0; k < 64; ++k) s += x[(size_t)m * K + g * 64 + k];
      xsum[(size_t)m * G + g] = s;
    }
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    const uint32_t* row = w + (size_t)n * wpr;
    for (int m0 = 0; m0 < M; m0 += ORACLE_MB) {
      const int mb = M - m0 < ORACLE_MB ? M - m0 : ORACLE_MB;
      float acc[ORACLE_MB];
      for (int m = 0; m < mb; ++m) acc[m] = 0.0f;
      for (int gi = 0; gi < G; ++gi) {
        const int g = g_reverse ? G - 1 - gi : gi;
        float q[64];
        for (int i = 0; i < 64 / per; ++i) {
          const uint32_t word = row[g * (64 / per) + i];
          for (int j = 0; j < per; ++j) q[i * per + j] = (float)((word >> (bits * j)) & mask);
        }
        const float s = bf16_to_f32(scales[(size_t)n * G + g]), b = bf16_to_f32(biases[(size_t)n * G + g]);
        for (int m = 0; m < mb; ++m) {
          const float* xr = x + (size_t)(m0 + m) * K + g * 64;
          float d = 0.0f;
          for (int ki = 0; ki < 64; ++ki) {
            const int k = g_reverse ? 63 - ki : ki;
            d += xr[k] * q[k];
          }
          acc[m] += s * d + b * xsum[(size_t)(m0 + m) * G + g];
        }
      }
      for (int m = 0; m < mb; ++m) out[(size_t)(m0 + m) * N + n] = acc[m];
    }
  }
  free(xsum);
  return 0;
}

/* fp32 -> bf16 -> fp32, round to nearest even (finite inputs). */
static inline float round_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* out[M, N] = x[M, K] . W'^T with W' = bf16(scale * q + bias) (computed in double, rounded to
 * float, then to bf16): the dequantize-then-multiply form of tile GEMMs. */
void oracle_qgemm_tile_bf16(int M, int N, int K, int bits, const float* x, const uint32_t* w, const uint16_t* scales,
                            const uint16_t* biases, float* out) {
  const int G = K / 64, per = 32 / bits, wpr = K / per;
  const uint32_t mask = (1u << bits) - 1u;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    const uint32_t* row = w + (size_t)n * wpr;
    for (int m0 = 0; m0 < M; m0 += ORACLE_MB) {
      const int mb = M - m0 < ORACLE_MB ? M - m0 : ORACLE_MB;
      float acc[ORACLE_MB];
      for (int m = 0; m < mb; ++m) acc[m] = 0.0f;
      for (int gi = 0; gi < G; ++gi) {
        const int g = g_reverse ? G - 1 - gi : gi;
        float dq[64];
        const double s = bf16_to_f32(scales[(size_t)n * G + g]), b = bf16_to_f32(biases[(size_t)n * G + g]);
        for (int i = 0; i < 64 / per; ++i) {
          const uint32_t word = row[g * (64 / per) + i];
          for (int j = 0; j < per; ++j)
            dq[i * per + j] = round_bf16((float)(s * (double)((word >> (bits * j)) & mask) + b));
        }
        for (int m = 0; m < mb; ++m) {
          const float* xr = x + (size_t)(m0 + m) * K + g * 64;
          float d = acc[m];
          for (int ki = 0; ki < 64; ++ki) {
            const int k = g_reverse ? 63 - ki : ki;
            d += xr[k] * dq[k];
          }
          acc[m] = d;
        }
      }
      for (int m = 0; m < mb; ++m) out[(size_t)(m0 + m) * N + n] = acc[m];
    }
  }
}

/* out[M, N] = x[M, K] . W^T, W dense bf16 bits [N, K]. */
void oracle_gemm_dense_bf16(int M, int N, int K, const float* x, const uint16_t* w, float* out) {
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; ++n) {
    const uint16_t* row = w + (size_t)n * K;
    for (int m = 0; m < M; ++m) {
      const float* xr = x + (size_t)m * K;
      float d = 0.0f;
      for (int ki = 0; ki < K; ++ki) {
        const int k = g_reverse ? K - 1 - ki : ki;
        d += xr[k] * bf16_to_f32(row[k]);
      }
      out[(size_t)m * N + n] = d;
    }
  }
}

int oracle_threads(void) {
#ifdef _OPENMP
  extern int omp_get_max_threads(void);
  return omp_get_max_threads();
#else
  return 1;
#endif
}
