/*
 * qw_oracle.c -- CPU restatement of MLX's affine group quantization as
 * cr0sh/qw calls it.  TEST INFRASTRUCTURE ONLY; see qw_oracle.h for the
 * reference citations, the conventions and the parity status.
 *
 * Build: oracle/Makefile (-O3 -ffp-contract=off -fopenmp, x86-64-v3).
 * Contraction is disabled so that every `a*b + c` below is two IEEE fp32
 * operations, which is what makes the results reproducible bit for bit on
 * any x86-64 host.  The matmul's full 16-row blocks run in AVX2 intrinsics
 * with one row per lane, so each row's operations and their order are those
 * of the scalar loops that handle the last, partial block.
 */
#include "qw_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ fp16 */

uint16_t qwo_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, sizeof x);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) { /* inf / nan */
    if (ax > 0x7f800000u) return (uint16_t)(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    return (uint16_t)(sign | 0x7c00u);
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 -> inf */
  const uint32_t e = ax >> 23;
  if (e >= 113u) { /* normal binary16 */
    uint32_t h = ((e - 112u) << 10) | ((ax >> 13) & 0x3ffu);
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  if (e < 102u) return (uint16_t)sign; /* below 2^-25: rounds to zero */
  /* subnormal binary16: value = m * 2^(e-150), unit 2^-24 */
  const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
  const uint32_t shift = 126u - e; /* 14 .. 24 */
  uint32_t h = m >> shift;
  const uint32_t rem = m & ((1u << shift) - 1u);
  const uint32_t half = 1u << (shift - 1u);
  if (rem > half || (rem == half && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

uint16_t qwo_f64_to_f16(double d) {
  uint64_t x;
  memcpy(&x, &d, sizeof x);
  const uint32_t sign = (uint32_t)(x >> 48) & 0x8000u;
  const uint64_t ax = x & 0x7fffffffffffffffull;
  if (ax >= 0x7ff0000000000000ull) {
    if (ax > 0x7ff0000000000000ull) return (uint16_t)(sign | 0x7e00u | (uint32_t)((ax >> 42) & 0x3ffu));
    return (uint16_t)(sign | 0x7c00u);
  }
  if (fabs(d) >= 65520.0) return (uint16_t)(sign | 0x7c00u);
  const uint32_t e = (uint32_t)(ax >> 52);
  if (e >= 1009u) { /* normal binary16 */
    uint32_t h = ((e - 1008u) << 10) | (uint32_t)((ax >> 42) & 0x3ffu);
    const uint64_t rem = ax & ((1ull << 42) - 1ull);
    const uint64_t half = 1ull << 41;
    if (rem > half || (rem == half && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  if (e < 998u) return (uint16_t)sign;
  const uint64_t m = (ax & 0xfffffffffffffull) | (1ull << 52);
  const uint32_t shift = 1051u - e; /* 43 .. 53 */
  uint32_t h = (uint32_t)(m >> shift);
  const uint64_t rem = m & ((1ull << shift) - 1ull);
  const uint64_t half = 1ull << (shift - 1u);
  if (rem > half || (rem == half && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

float qwo_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  const uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
  uint32_t m = (uint32_t)h & 0x3ffu;
  uint32_t bits;
  if (e == 0x1fu) {
    bits = sign | 0x7f800000u | (m << 13);
  } else if (e != 0u) {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  } else if (m == 0u) {
    bits = sign;
  } else { /* subnormal: normalise */
    uint32_t ee = 113u;
    while ((m & 0x400u) == 0u) {
      m <<= 1;
      ee--;
    }
    bits = sign | (ee << 23) | ((m & 0x3ffu) << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

void qwo_f32_to_f16_array(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = qwo_f32_to_f16(src[i]);
}

void qwo_f16_to_f32_array(const uint16_t* src, float* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = qwo_f16_to_f32(src[i]);
}

int qwo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------ validation */

/* Mirrors the reference's load-time checks: bits must divide a 32-bit word
 * (the U32 packing of weights.rs:150-158), the group must tile K and the
 * packed width must satisfy packed_in*32 == bits*groups*group_size
 * (layers.rs:1568-1570). */
static int check_params(int64_t N, int64_t K, int group_size, int bits) {
  if (N < 0 || K <= 0) return QWO_EINVAL;
  if (bits != 2 && bits != 4 && bits != 8) return QWO_EUNSUPPORTED;
  if (group_size != 32 && group_size != 64 && group_size != 128) return QWO_EUNSUPPORTED;
  if (K % group_size != 0) return QWO_EINVAL;
  if ((K * bits) % 32 != 0) return QWO_EINVAL;
  return QWO_OK;
}

static inline uint32_t nibble_at(const uint32_t* row, int64_t k, int bits) {
  const int pf = 32 / bits;
  const uint32_t mask = (1u << bits) - 1u;
  return (row[k / pf] >> ((uint32_t)bits * (uint32_t)(k % pf))) & mask;
}

/* -------------------------------------------------------------- quantize */

int qwo_quantize(const uint16_t* w, int64_t N, int64_t K, int group_size, int bits,
                 uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  const int rc = check_params(N, K, group_size, bits);
  if (rc != QWO_OK) return rc;
  const int pf = 32 / bits;
  const int64_t kw = K / pf;
  const int64_t G = K / group_size;
  const float nbins = (float)((1 << bits) - 1);
  memset(wq, 0, (size_t)(N * kw) * sizeof(uint32_t));
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const uint16_t* wr = w + n * K;
    uint32_t* qr = wq + n * kw;
    for (int64_t g = 0; g < G; ++g) {
      float mn = INFINITY, mx = -INFINITY;
      for (int i = 0; i < group_size; ++i) {
        const float v = qwo_f16_to_f32(wr[g * group_size + i]);
        if (v < mn) mn = v;
        if (v > mx) mx = v;
      }
      float scale = (mx - mn) / nbins;
      if (!(scale >= 1e-7f)) scale = 1e-7f;
      const uint16_t sh = qwo_f32_to_f16(scale);
      const uint16_t bh = qwo_f32_to_f16(mn);
      const float sf = qwo_f16_to_f32(sh);
      const float bf = qwo_f16_to_f32(bh);
      scales[n * G + g] = sh;
      biases[n * G + g] = bh;
      for (int i = 0; i < group_size; ++i) {
        const int64_t k = g * group_size + i;
        const float v = qwo_f16_to_f32(wr[k]);
        float r = rintf((v - bf) / sf);
        r = fminf(fmaxf(r, 0.0f), nbins);
        const uint32_t q = (uint32_t)r;
        qr[k / pf] |= q << ((uint32_t)bits * (uint32_t)(k % pf));
      }
    }
  }
  return QWO_OK;
}

/* ------------------------------------------------------------ dequantize */

int qwo_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases,
                   int64_t N, int64_t K, int group_size, int bits, int rounding,
                   uint16_t* out) {
  const int rc = check_params(N, K, group_size, bits);
  if (rc != QWO_OK) return rc;
  if (rounding != QWO_ROUND_TWICE && rounding != QWO_ROUND_ONCE) return QWO_EINVAL;
  const int64_t kw = K * bits / 32;
  const int64_t G = K / group_size;
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const uint32_t* qr = wq + n * kw;
    for (int64_t k = 0; k < K; ++k) {
      const int64_t g = k / group_size;
      const uint16_t sh = scales[n * G + g];
      const uint16_t bh = biases[n * G + g];
      const uint32_t q = nibble_at(qr, k, bits);
      uint16_t r;
      if (rounding == QWO_ROUND_TWICE) {
        /* s*q is exact in fp32 (11-bit significand times an 8-bit integer),
         * so rounding it to fp16 is the correctly rounded fp16 product; the
         * fp32 sum of two fp16 values rounds to fp16 exactly as an fp16 add. */
        const uint16_t t = qwo_f32_to_f16(qwo_f16_to_f32(sh) * (float)q);
        r = qwo_f32_to_f16(qwo_f16_to_f32(t) + qwo_f16_to_f32(bh));
      } else {
        r = qwo_f64_to_f16((double)qwo_f16_to_f32(sh) * (double)q + (double)qwo_f16_to_f32(bh));
      }
      out[n * K + k] = r;
    }
  }
  return QWO_OK;
}

/* float32 scales and biases (MLX dequantize with f32 scales returns f32):
 * QWO_ROUND_TWICE: w = fp32(fp32(s*q) + b), the two ops of `scales * q +
 * biases` in float32; QWO_ROUND_ONCE: w = fmaf(s, q, b), rounded once.  The
 * reference's layout test (ffi_tests.rs:3792-3850) dequantizes such arrays. */
int qwo_dequantize_f32(const uint32_t* wq, const float* scales, const float* biases, int64_t N, int64_t K,
                       int group_size, int bits, int rounding, float* out) {
  const int rc = check_params(N, K, group_size, bits);
  if (rc != QWO_OK) return rc;
  if (rounding != QWO_ROUND_TWICE && rounding != QWO_ROUND_ONCE) return QWO_EINVAL;
  const int64_t kw = K * bits / 32;
  const int64_t G = K / group_size;
  for (int64_t n = 0; n < N; ++n) {
    const uint32_t* qr = wq + n * kw;
    for (int64_t k = 0; k < K; ++k) {
      const float s = scales[n * G + k / group_size];
      const float b = biases[n * G + k / group_size];
      const float q = (float)nibble_at(qr, k, bits);
      if (rounding == QWO_ROUND_TWICE) {
        const float t = s * q;
        out[n * K + k] = t + b;
      } else {
        out[n * K + k] = fmaf(s, q, b);
      }
    }
  }
  return QWO_OK;
}

/* -------------------------------------------------------- quantized_matmul */

/* binary16 -> binary32 lookup, filled once from qwo_f16_to_f32. */
static float f16_table[65536];
static pthread_once_t f16_table_once = PTHREAD_ONCE_INIT;
static void fill_f16_table(void) {
  for (uint32_t h = 0; h < 65536u; ++h) f16_table[h] = qwo_f16_to_f32((uint16_t)h);
}
static void init_f16_table(void) { pthread_once(&f16_table_once, fill_f16_table); }

#define QWO_RB 16 /* rows dequantized together; lanes of the inner vector loop */

/* Full blocks of QWO_RB rows in AVX2 (the build's x86-64-v3 baseline).  The
 * arithmetic is the scalar loops' exactly, only spread over lanes: lane j of
 * a vector is row nb + j, so every row still forms w = s*q, then + b, and
 * sums x*w in K order, each step one rounded fp32 operation.
 *
 * wblk[k][j] = dequantized weight of row nb + j at column k: the words of the
 * 16 rows at word index wi are gathered, then each code position p is
 * shifted out, converted and scaled for all rows at once. */
static void dequant_block_avx2(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases, int64_t nb,
                               int64_t kw, int64_t G, int group_size, int bits, float* wblk) {
  const int pf = 32 / bits;
  const __m256i mask = _mm256_set1_epi32((int)((1u << bits) - 1u));
  const __m256i rows = _mm256_setr_epi32(0, 1, 2, 3, 4, 5, 6, 7);
  const __m256i vidx = _mm256_mullo_epi32(rows, _mm256_set1_epi32((int)kw)); /* word offsets of rows 0..7 */
  const uint32_t* base = wq + nb * kw;
  const int64_t wpg = group_size / pf; /* words per group */
  for (int64_t g = 0; g < G; ++g) {
    float sv[QWO_RB], bv[QWO_RB];
    for (int j = 0; j < QWO_RB; ++j) {
      sv[j] = f16_table[scales[(nb + j) * G + g]];
      bv[j] = f16_table[biases[(nb + j) * G + g]];
    }
    const __m256 s0 = _mm256_loadu_ps(sv), s1 = _mm256_loadu_ps(sv + 8);
    const __m256 b0 = _mm256_loadu_ps(bv), b1 = _mm256_loadu_ps(bv + 8);
    for (int64_t wi = g * wpg; wi < (g + 1) * wpg; ++wi) {
      const __m256i w0 = _mm256_i32gather_epi32((const int*)(base + wi), vidx, 4);
      const __m256i w1 = _mm256_i32gather_epi32((const int*)(base + 8 * kw + wi), vidx, 4);
      float* dst = wblk + wi * pf * QWO_RB;
      for (int p = 0; p < pf; ++p, dst += QWO_RB) {
        const __m128i sh = _mm_cvtsi32_si128(bits * p);
        /* codes are at most 255: the signed conversion is exact */
        const __m256 q0 = _mm256_cvtepi32_ps(_mm256_and_si256(_mm256_srl_epi32(w0, sh), mask));
        const __m256 q1 = _mm256_cvtepi32_ps(_mm256_and_si256(_mm256_srl_epi32(w1, sh), mask));
        _mm256_storeu_ps(dst, _mm256_add_ps(_mm256_mul_ps(s0, q0), b0));
        _mm256_storeu_ps(dst + 8, _mm256_add_ps(_mm256_mul_ps(s1, q1), b1));
      }
    }
  }
}

/* Up to 4 rows of x: each weight is formed and used at once, with no
 * dequantized block in memory.  acc[i][j] = sum over k (ascending) of
 * x[m0 + i][k] * w(nb + j, k), the same steps as dequant_block_avx2 followed
 * by block_rows_avx2. */
static void fused_rows_avx2(const float* xf, int64_t K, const uint32_t* wq, const uint16_t* scales,
                            const uint16_t* biases, int64_t nb, int64_t kw, int64_t G, int group_size, int bits,
                            int64_t m0, int nm, float acc[4][QWO_RB]) {
  const int pf = 32 / bits;
  const __m256i mask = _mm256_set1_epi32((int)((1u << bits) - 1u));
  const __m256i vidx = _mm256_mullo_epi32(_mm256_setr_epi32(0, 1, 2, 3, 4, 5, 6, 7), _mm256_set1_epi32((int)kw));
  const uint32_t* base = wq + nb * kw;
  const int64_t wpg = group_size / pf;
  const float* xr[4];
  for (int i = 0; i < 4; ++i) xr[i] = xf + (m0 + (i < nm ? i : 0)) * K;
  __m256 a[4][2];
  for (int i = 0; i < 4; ++i) a[i][0] = a[i][1] = _mm256_setzero_ps();
  for (int64_t g = 0; g < G; ++g) {
    float sv[QWO_RB], bv[QWO_RB];
    for (int j = 0; j < QWO_RB; ++j) {
      sv[j] = f16_table[scales[(nb + j) * G + g]];
      bv[j] = f16_table[biases[(nb + j) * G + g]];
    }
    const __m256 s0 = _mm256_loadu_ps(sv), s1 = _mm256_loadu_ps(sv + 8);
    const __m256 b0 = _mm256_loadu_ps(bv), b1 = _mm256_loadu_ps(bv + 8);
    for (int64_t wi = g * wpg; wi < (g + 1) * wpg; ++wi) {
      const __m256i w0 = _mm256_i32gather_epi32((const int*)(base + wi), vidx, 4);
      const __m256i w1 = _mm256_i32gather_epi32((const int*)(base + 8 * kw + wi), vidx, 4);
      for (int p = 0; p < pf; ++p) {
        const int64_t k = wi * pf + p;
        const __m128i sh = _mm_cvtsi32_si128(bits * p);
        const __m256 q0 = _mm256_cvtepi32_ps(_mm256_and_si256(_mm256_srl_epi32(w0, sh), mask));
        const __m256 q1 = _mm256_cvtepi32_ps(_mm256_and_si256(_mm256_srl_epi32(w1, sh), mask));
        const __m256 d0 = _mm256_add_ps(_mm256_mul_ps(s0, q0), b0);
        const __m256 d1 = _mm256_add_ps(_mm256_mul_ps(s1, q1), b1);
        for (int i = 0; i < nm; ++i) {
          const __m256 xv = _mm256_broadcast_ss(xr[i] + k);
          a[i][0] = _mm256_add_ps(a[i][0], _mm256_mul_ps(xv, d0));
          a[i][1] = _mm256_add_ps(a[i][1], _mm256_mul_ps(xv, d1));
        }
      }
    }
  }
  for (int i = 0; i < nm; ++i) {
    _mm256_storeu_ps(acc[i], a[i][0]);
    _mm256_storeu_ps(acc[i] + 8, a[i][1]);
  }
}

/* acc[m][j] = sum over k (ascending) of x[m][k] * wblk[k][j] for m in
 * [m0, m0 + nm), nm <= 4: four rows of x share each load of wblk. */
static void block_rows_avx2(const float* xf, int64_t K, const float* wblk, int64_t m0, int nm,
                            float acc[4][QWO_RB]) {
  __m256 a[4][2];
  for (int i = 0; i < 4; ++i) a[i][0] = a[i][1] = _mm256_setzero_ps();
  const float* xr[4];
  for (int i = 0; i < 4; ++i) xr[i] = xf + (m0 + (i < nm ? i : 0)) * K;
  for (int64_t k = 0; k < K; ++k) {
    const __m256 w0 = _mm256_loadu_ps(wblk + k * QWO_RB), w1 = _mm256_loadu_ps(wblk + k * QWO_RB + 8);
    for (int i = 0; i < 4; ++i) {
      const __m256 xv = _mm256_broadcast_ss(xr[i] + k);
      a[i][0] = _mm256_add_ps(a[i][0], _mm256_mul_ps(xv, w0));
      a[i][1] = _mm256_add_ps(a[i][1], _mm256_mul_ps(xv, w1));
    }
  }
  for (int i = 0; i < nm; ++i) {
    _mm256_storeu_ps(acc[i], a[i][0]);
    _mm256_storeu_ps(acc[i] + 8, a[i][1]);
  }
}

int qwo_quantized_matmul(const uint16_t* x, const uint32_t* wq, const uint16_t* scales,
                         const uint16_t* biases, int64_t M, int64_t N, int64_t K,
                         int group_size, int bits, uint16_t* y, float* y32, int nthreads) {
  const int rc = check_params(N, K, group_size, bits);
  if (rc != QWO_OK) return rc;
  if (M < 0) return QWO_EINVAL;
  if (M == 0 || N == 0) return QWO_OK;
  const int64_t kw = K * bits / 32;
  const int64_t G = K / group_size;
  init_f16_table();
  float* xf = (float*)malloc((size_t)(M * K) * sizeof(float));
  if (!xf) return QWO_EINVAL;
  qwo_f16_to_f32_array(x, xf, M * K);
  int nt = nthreads > 0 ? nthreads : qwo_max_threads();
  (void)nt;
  int failed = 0;
#pragma omp parallel num_threads(nt)
  {
    /* wblk[k][j]: the fp32 dequantized weight of row nb+j at column k. */
    float* wblk = (float*)malloc((size_t)K * QWO_RB * sizeof(float));
    if (!wblk) {
#pragma omp atomic write
      failed = 1;
    }
#pragma omp for schedule(dynamic, 1)
    for (int64_t nb = 0; nb < N; nb += QWO_RB) {
      if (!wblk) continue;
      const int rb = (int)((N - nb) < QWO_RB ? (N - nb) : QWO_RB);
      if (rb == QWO_RB) {
        if (M > 4) dequant_block_avx2(wq, scales, biases, nb, kw, G, group_size, bits, wblk);
        for (int64_t m0 = 0; m0 < M; m0 += 4) {
          const int nm = (int)((M - m0) < 4 ? (M - m0) : 4);
          float acc[4][QWO_RB];
          if (M > 4) block_rows_avx2(xf, K, wblk, m0, nm, acc);
          else fused_rows_avx2(xf, K, wq, scales, biases, nb, kw, G, group_size, bits, m0, nm, acc);
          for (int i = 0; i < nm; ++i)
            for (int j = 0; j < QWO_RB; ++j) {
              y[(m0 + i) * N + nb + j] = qwo_f32_to_f16(acc[i][j]);
              if (y32) y32[(m0 + i) * N + nb + j] = acc[i][j];
            }
        }
        continue;
      }
      /* the last, partial block: scalar */
      for (int j = 0; j < QWO_RB; ++j) {
        if (j >= rb) {
          for (int64_t k = 0; k < K; ++k) wblk[k * QWO_RB + j] = 0.0f;
          continue;
        }
        const int64_t n = nb + j;
        const uint32_t* qr = wq + n * kw;
        const int pf = 32 / bits;
        const uint32_t mask = (1u << bits) - 1u;
        for (int64_t g = 0; g < G; ++g) {
          const float s = f16_table[scales[n * G + g]];
          const float b = f16_table[biases[n * G + g]];
          for (int64_t wi = g * group_size / pf; wi < (g + 1) * group_size / pf; ++wi) {
            uint32_t word = qr[wi];
            for (int p = 0; p < pf; ++p) {
              const float t = s * (float)(word & mask);
              wblk[(wi * pf + p) * QWO_RB + j] = t + b;
              word >>= bits;
            }
          }
        }
      }
      for (int64_t m = 0; m < M; ++m) {
        float acc[QWO_RB];
        for (int j = 0; j < QWO_RB; ++j) acc[j] = 0.0f;
        const float* xm = xf + m * K;
        for (int64_t k = 0; k < K; ++k) {
          const float xv = xm[k];
          const float* wk = wblk + k * QWO_RB;
          for (int j = 0; j < QWO_RB; ++j) {
            const float p = xv * wk[j];
            acc[j] = acc[j] + p;
          }
        }
        for (int j = 0; j < rb; ++j) {
          y[m * N + nb + j] = qwo_f32_to_f16(acc[j]);
          if (y32) y32[m * N + nb + j] = acc[j];
        }
      }
    }
    free(wblk);
  }
  free(xf);
  return failed ? QWO_EINVAL : QWO_OK;
}

/* y fp16 [M][N] = x fp16 [M][K] . w^T for fp16 weights w [N][K] (for example
 * qwo_dequantize's ROUND_TWICE output), each product and sum one fp32
 * operation, summed in ascending k: the matmul with the weights formed in
 * fp16 first instead of fp32. */
int qwo_matmul_f16w(const uint16_t* x, const uint16_t* w, int64_t M, int64_t N, int64_t K, uint16_t* y,
                    float* y32, int nthreads) {
  if (M < 0 || N < 0 || K <= 0) return QWO_EINVAL;
  if (M == 0 || N == 0) return QWO_OK;
  init_f16_table();
  float* xf = (float*)malloc((size_t)(M * K) * sizeof(float));
  if (!xf) return QWO_EINVAL;
  qwo_f16_to_f32_array(x, xf, M * K);
  int nt = nthreads > 0 ? nthreads : qwo_max_threads();
  (void)nt;
  int failed = 0;
#pragma omp parallel num_threads(nt)
  {
    float* wblk = (float*)malloc((size_t)K * QWO_RB * sizeof(float));
    if (!wblk) {
#pragma omp atomic write
      failed = 1;
    }
#pragma omp for schedule(dynamic, 1)
    for (int64_t nb = 0; nb < N; nb += QWO_RB) {
      if (!wblk) continue;
      const int rb = (int)((N - nb) < QWO_RB ? (N - nb) : QWO_RB);
      for (int j = 0; j < QWO_RB; ++j)
        for (int64_t k = 0; k < K; ++k) wblk[k * QWO_RB + j] = j < rb ? f16_table[w[(nb + j) * K + k]] : 0.0f;
      for (int64_t m0 = 0; m0 < M; m0 += 4) {
        const int nm = (int)((M - m0) < 4 ? (M - m0) : 4);
        float acc[4][QWO_RB];
        block_rows_avx2(xf, K, wblk, m0, nm, acc);
        for (int i = 0; i < nm; ++i)
          for (int j = 0; j < rb; ++j) {
            y[(m0 + i) * N + nb + j] = qwo_f32_to_f16(acc[i][j]);
            if (y32) y32[(m0 + i) * N + nb + j] = acc[i][j];
          }
      }
    }
    free(wblk);
  }
  free(xf);
  return failed ? QWO_EINVAL : QWO_OK;
}
