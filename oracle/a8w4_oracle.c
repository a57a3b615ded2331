/*
 * a8w4_oracle.c — CPU restatement of the GEMM hot path. TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm
 * may load this library, and only as the checker or the timed CPU baseline; the
 * product path (arc-gemm_b200/) never calls it.
 *
 * What it restates:
 *   - int4 packing convention: byte j of a weight row holds code k=2j in bits 3:0 and
 *     k=2j+1 in bits 7:4 (reference packer arc/testing/quant.py:82-83; reference
 *     unpacker arc/math.py:144-146). Codes are two's-complement int4 in this recipe.
 *   - A8W4 group partials  P[m,n,g] = sum_{k in group g} A[m,k] * W[n,k]   (int32)
 *   - A8W4 output          out[m,n] = sa[m] * sum_g sb[n,g] * P[m,n,g]
 *     computed in double from the exact partials (the "fp32 reference" of the
 *     contract, made exact so a GPU result can be judged in bf16 ulps).
 *     The data flow follows the reference's A8W4 check, tests/a8w4.py:15-33 and :53.
 *   - bf16 GEMM reference  C = A . B^T in double from bf16 inputs (tests/matmul.py:21-23
 *     computes it as fp32 torch.mm of the upcast inputs).
 *   - float -> bf16 round-to-nearest-even, as torch's .to(torch.bfloat16).
 *
 * Loops are written for clarity; OpenMP splits the outer loop when available.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static inline int int4_code(const uint8_t *row, int k) {
  const uint8_t b = row[k >> 1];
  const int v = (k & 1) ? (b >> 4) : (b & 0x0F);
  return v >= 8 ? v - 16 : v;
}

static inline double bf16_to_double(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return (double)f;
}

/* Unpack [rows][K/2] packed bytes into [rows][K] int8 values in [-8, 7]. */
void oracle_unpack_int4(const uint8_t *packed, int rows, int K, int8_t *out) {
  for (long r = 0; r < rows; ++r) {
    const uint8_t *row = packed + r * (long)(K / 2);
    for (int k = 0; k < K; ++k) out[r * (long)K + k] = (int8_t)int4_code(row, k);
  }
}

/* P[m][n][g], int32. */
void oracle_a8w4_partials(const int8_t *A, const uint8_t *Wp, int M, int N, int K, int group,
                          int32_t *P) {
  const int G = K / group;
#pragma omp parallel for schedule(static)
  for (int m = 0; m < M; ++m) {
    const int8_t *a = A + (long)m * K;
    for (int n = 0; n < N; ++n) {
      const uint8_t *w = Wp + (long)n * (K / 2);
      for (int g = 0; g < G; ++g) {
        int32_t s = 0;
        for (int k = g * group; k < (g + 1) * group; ++k) s += (int32_t)a[k] * int4_code(w, k);
        P[((long)m * N + n) * G + g] = s;
      }
    }
  }
}

/* out[m][n] in double: sa[m] * sum_g sb[n][g] * P[m][n][g], groups in ascending order. */
void oracle_a8w4_out(const int8_t *A, const float *sa, const uint8_t *Wp, const uint16_t *sb,
                     int M, int N, int K, int group, double *out) {
  const int G = K / group;
#pragma omp parallel for schedule(static)
  for (int m = 0; m < M; ++m) {
    const int8_t *a = A + (long)m * K;
    for (int n = 0; n < N; ++n) {
      const uint8_t *w = Wp + (long)n * (K / 2);
      double acc = 0.0;
      for (int g = 0; g < G; ++g) {
        int32_t s = 0;
        for (int k = g * group; k < (g + 1) * group; ++k) s += (int32_t)a[k] * int4_code(w, k);
        acc += bf16_to_double(sb[(long)n * G + g]) * (double)s;
      }
      out[(long)m * N + n] = (double)sa[m] * acc;
    }
  }
}

/* C[m][n] in double = sum_k A[m][k] * B[n][k], A and B bf16 (row-major, K contiguous). */
void oracle_bf16_gemm(const uint16_t *A, const uint16_t *B, int M, int N, int K, double *C) {
#pragma omp parallel for schedule(static)
  for (int m = 0; m < M; ++m) {
    for (int n = 0; n < N; ++n) {
      double acc = 0.0;
      for (int k = 0; k < K; ++k) {
        acc += bf16_to_double(A[(long)m * K + k]) * bf16_to_double(B[(long)n * K + k]);
      }
      C[(long)m * N + n] = acc;
    }
  }
}

/* float -> bf16 bits, round to nearest even (NaN kept quiet). */
void oracle_f32_to_bf16(const float *x, long n, uint16_t *out) {
  for (long i = 0; i < n; ++i) {
    uint32_t u;
    memcpy(&u, &x[i], sizeof u);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) {
      out[i] = (uint16_t)((u >> 16) | 0x0040u);
      continue;
    }
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    out[i] = (uint16_t)(u >> 16);
  }
}
