/*
 * CPU oracle for the FP16 GEMM path. TEST INFRASTRUCTURE ONLY: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this code,
 * and only as the checker, never as the thing measured or shipped.
 *
 * Restates the reference's arithmetic contract for gemm_launcher:
 *   C[i,j] = half_rn(alpha * sum_k float(A[i,k]) * float(B[k,j]) + beta * float(C[i,j]))
 * with FP32 accumulation (reference src/lib/gemm_llm_kernels.cuh:130-194 and
 * :652-660: FP16 operands widened to FP32, products accumulated in FP32 with
 * fmaf, epilogue fmaf(alpha, acc, beta * previous) rounded to nearest; C not
 * read when beta == 0, src/lib/gemm_llm_kernels.cuh:215 and
 * src/lib/gemm_progressive_kernel.cuh:362). K <= 0 gives half_rn(beta * C)
 * (src/lib/gemm_cublas.cuh:27-33). M <= 0 or N <= 0 leaves C untouched
 * (src/gemm.cu:106-108).
 *
 * The binary16 conversions are written here from the IEEE 754 encoding
 * (round to nearest, ties to even), not taken from any CUDA header.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

float oracle_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1Fu;
  const uint32_t man = h & 0x3FFu;
  uint32_t bits;
  float out;
  if (exp == 0) {
    /* zero or subnormal: man * 2^-24 is exact in float */
    out = (float)man * 5.9604644775390625e-8f;
    memcpy(&bits, &out, 4);
    bits |= sign;
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  memcpy(&out, &bits, 4);
  return out;
}

uint16_t oracle_float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax > 0x7F800000u) return (uint16_t)(sign | 0x7E00u); /* NaN */
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 -> inf */
  if (ax <= 0x33000000u) return sign;                       /* <= 2^-25 -> 0 (tie to even) */
  const uint32_t exp = ax >> 23;
  const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
  if (exp < 113u) {
    /* subnormal result: value = q * 2^-24 */
    const uint32_t shift = 126u - exp; /* 14 .. 24 */
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1u);
    if (rem > halfway || (rem == halfway && (q & 1u))) ++q;
    return (uint16_t)(sign | q);
  }
  uint32_t h = ((exp - 112u) << 10) | ((ax >> 13) & 0x3FFu);
  const uint32_t rem = ax & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* carry may reach the exponent */
  return (uint16_t)(sign | h);
}

/* FP32-accumulate GEMM in k order. A[M,K], B[K,N], C[M,N] row-major with the
 * given row pitches (elements). */
void oracle_gemm_f32(const uint16_t* A, long lda, const uint16_t* B, long ldb, uint16_t* C, long ldc,
                     int M, int N, int K, float alpha, float beta) {
  if (M <= 0 || N <= 0) return;
  for (int i = 0; i < M; ++i) {
    for (int j = 0; j < N; ++j) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k)
        acc = fmaf(oracle_half_to_float(A[i * lda + k]), oracle_half_to_float(B[k * ldb + j]), acc);
      const float prev = beta != 0.0f ? oracle_half_to_float(C[i * ldc + j]) : 0.0f;
      C[i * ldc + j] = oracle_float_to_half(fmaf(alpha, acc, beta * prev));
    }
  }
}

/* Unrounded FP32 reference values alpha*acc + beta*C (what the reference's
 * tests compare against before rounding), written to out[M*N]. */
void oracle_gemm_f32_unrounded(const uint16_t* A, const uint16_t* B, const uint16_t* C, float* out,
                               int M, int N, int K, float alpha, float beta) {
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) {
      float acc = 0.0f;
      for (int k = 0; k < K; ++k)
        acc = fmaf(oracle_half_to_float(A[(long)i * K + k]),
                   oracle_half_to_float(B[(long)k * N + j]), acc);
      const float prev = beta != 0.0f ? oracle_half_to_float(C[(long)i * N + j]) : 0.0f;
      out[(long)i * N + j] = alpha * acc + beta * prev;
    }
}

/* FP64 audit of selected outputs (the reference's square benchmark audits 64
 * points with CPU FP64 dot products, benchmarks/square_benchmark.cu:73-95).
 * For each (rows[t], cols[t]) writes alpha * dot64 + beta * C0 to out[t]. */
void oracle_audit_f64(const uint16_t* A, const uint16_t* B, const uint16_t* C0, int M, int N, int K,
                      double alpha, double beta, const int* rows, const int* cols, int count,
                      double* out) {
  (void)M;
  for (int t = 0; t < count; ++t) {
    const long i = rows[t], j = cols[t];
    double acc = 0.0;
    for (int k = 0; k < K; ++k)
      acc += (double)oracle_half_to_float(A[i * K + k]) * (double)oracle_half_to_float(B[(long)k * N + j]);
    const double prev = beta != 0.0 ? (double)oracle_half_to_float(C0[i * N + j]) : 0.0;
    out[t] = alpha * acc + beta * prev;
  }
}

/* Bulk conversions used by the checker. */
void oracle_halves_to_floats(const uint16_t* in, float* out, long n) {
  for (long i = 0; i < n; ++i) out[i] = oracle_half_to_float(in[i]);
}

void oracle_floats_to_halves(const float* in, uint16_t* out, long n) {
  for (long i = 0; i < n; ++i) out[i] = oracle_float_to_half(in[i]);
}
