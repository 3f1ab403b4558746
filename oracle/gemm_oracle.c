/*
 * CPU oracle for the FP16 GEMM hot path.  TEST INFRASTRUCTURE ONLY: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it, as
 * the checker.  The product path never calls it.
 *
 * Restates the arithmetic of the reference kernels:
 *   C[i][j] = fp16_rn( sum_k fp32(A[i][k]) * fp32(B[k][j]) )
 * with fp16 inputs widened exactly to fp32, an fp32 accumulator running over
 * K in order, and one round-to-nearest-even conversion to fp16 at the end --
 * the reference epilogue `__float2half(alpha * acc)` with alpha = 1, beta = 0
 * (tensorcore_gemm/gemm.cu:1360-1361; reg_pingpong_256_mma.cu:152-156).  The
 * reference's fp32 accumulation order is per 16-deep MMA, sequential in K
 * (gemm.cu:1208-1290), so results agree with any fp32 summation order within
 * rounding, not bit for bit; parity is judged with the K-scaled RMS bound.
 *
 * The fp16 <-> fp32 conversions are written here from the IEEE 754 binary16
 * / binary32 formats (no compiler or library conversion is used), so the
 * oracle does not depend on the host compiler's _Float16 support.
 *
 * Layouts: A M x K row-major (lda), B K x N row-major (ldb) when
 * b_col_major == 0, else B stored N x K row-major (ldb), C M x N (ldc).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);           /* inf / nan */
  } else if (exp == 0) {
    if (man == 0) {
      bits = sign;                                       /* +-0 */
    } else {                                             /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; ++e; } while ((man & 0x400u) == 0);
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else {
    bits = sign | ((exp + (127 - 15)) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t oracle_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
  const int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);       /* overflow -> inf */
  if (e <= 0) {
    /* Result is subnormal or zero: shift the full significand. */
    if (exp == 0) return sign;                           /* fp32 subnormals are far below fp16 range */
    man |= 0x800000u;
    const int shift = 14 - e;                            /* >= 14 */
    if (shift > 31) return sign;
    uint32_t h = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* carry may reach inf: correct */
  return (uint16_t)(sign | h);
}

void oracle_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f16_to_f32(src[i]);
}

void oracle_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_f16(src[i]);
}

typedef struct {
  const float* a;   /* M x K, dense */
  const float* bt;  /* N x K, dense (B transposed) */
  float* acc;       /* optional M x N fp32 output (ldacc = N) */
  uint16_t* c;      /* optional fp16 output */
  int64_t m0, m1, n, k, ldc;
} Job;

static void* run_rows(void* p) {
  Job* j = (Job*)p;
  for (int64_t i = j->m0; i < j->m1; ++i) {
    const float* ar = j->a + i * j->k;
    for (int64_t c = 0; c < j->n; ++c) {
      const float* br = j->bt + c * j->k;
      float s = 0.0f;
      for (int64_t t = 0; t < j->k; ++t) s += ar[t] * br[t];
      if (j->acc) j->acc[i * j->n + c] = s;
      if (j->c) j->c[i * j->ldc + c] = oracle_f32_to_f16(s);
    }
  }
  return NULL;
}

/*
 * Oracle GEMM.  `c` (fp16, ldc) and/or `acc` (fp32, dense M x N) may be NULL.
 * `threads` <= 1 runs on the calling thread.  Returns 0, or -1 on bad
 * arguments / allocation failure.
 */
int oracle_gemm_f16(const uint16_t* A, const uint16_t* B, uint16_t* C, float* acc, int64_t M, int64_t N,
                    int64_t K, int64_t lda, int64_t ldb, int64_t ldc, int b_col_major, int threads) {
  if (M < 0 || N < 0 || K < 0) return -1;
  if (M == 0 || N == 0) return 0;
  float* a = (float*)malloc(sizeof(float) * (size_t)(M * (K ? K : 1)));
  float* bt = (float*)malloc(sizeof(float) * (size_t)(N * (K ? K : 1)));
  if (!a || !bt) { free(a); free(bt); return -1; }
  for (int64_t i = 0; i < M; ++i)
    for (int64_t t = 0; t < K; ++t) a[i * K + t] = oracle_f16_to_f32(A[i * lda + t]);
  for (int64_t c = 0; c < N; ++c)
    for (int64_t t = 0; t < K; ++t)
      bt[c * K + t] = oracle_f16_to_f32(b_col_major ? B[c * ldb + t] : B[t * ldb + c]);
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if ((int64_t)threads > M) threads = (int)M;
  Job jobs[256];
  pthread_t tids[256];
  int created[256];
  const int64_t per = (M + threads - 1) / threads;
  for (int t = 0; t < threads; ++t) {
    Job* j = &jobs[t];
    j->a = a; j->bt = bt; j->acc = acc; j->c = C; j->n = N; j->k = K; j->ldc = ldc;
    j->m0 = t * per < M ? t * per : M;
    j->m1 = (t + 1) * per < M ? (t + 1) * per : M;
    created[t] = 0;
    if (t > 0 && j->m0 < j->m1) created[t] = pthread_create(&tids[t], NULL, run_rows, j) == 0;
  }
  run_rows(&jobs[0]);
  for (int t = 1; t < threads; ++t) {
    if (created[t]) pthread_join(tids[t], NULL);
    else if (jobs[t].m0 < jobs[t].m1) run_rows(&jobs[t]);
  }
  free(a);
  free(bt);
  return 0;
}
