/*
 * oracle.c — CPU restatement of OnnxSharp's hot-path arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for libonnxsharp_cuda and the timed
 * CPU baseline in bench.py. Not linked into the product. See oracle.h for the
 * contract of each function and the reference file:line it follows.
 *
 * Build: make -C oracle  (gcc -O3 -ffp-contract=off -fopenmp -mavx2 -mfma).
 * -ffp-contract=off keeps every a*b+c that the reference writes unfused
 * unfused; fmaf() is used exactly where the reference calls Fma.MultiplyAdd.
 */
#include "oracle.h"

#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

static int nthreads(int threads) { return threads > 0 ? threads : omp_get_max_threads(); }

/* x86 MAXPS/MINPS semantics (Avx.Max/Avx.Min): (a > b) ? a : b, so a NaN in
 * the first operand yields the second. */
static inline float maxps(float a, float b) { return a > b ? a : b; }
static inline float minps(float a, float b) { return a < b ? a : b; }

/* VectorMath.Exp (Tensors/VectorMath.cs:21-43). */
float orc_exp(float x) {
  x = minps(maxps(x, -87.3f), 88.7f);
  const float n = nearbyintf(x * 1.4426950408889634f); /* Avx.RoundToNearestInteger: ties to even */
  float r = fmaf(n, -0.693145751953125f, x);
  r = fmaf(n, -1.4286067653e-6f, r);
  float p = 1.0f / 720.0f;
  p = fmaf(p, r, 1.0f / 120.0f);
  p = fmaf(p, r, 1.0f / 24.0f);
  p = fmaf(p, r, 1.0f / 6.0f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int32_t bits = ((int32_t)n + 127) << 23; /* Avx2.ShiftLeftLogical(n + 127, 23) */
  float s;
  memcpy(&s, &bits, sizeof(s));
  return p * s;
}

/* VectorMath.Sigmoid / Silu (VectorMath.cs:70-77). */
float orc_sigmoid(float x) { return 1.0f / (1.0f + orc_exp(x * -1.0f)); }
float orc_silu(float x) { return x * orc_sigmoid(x); }

static inline float act_apply(float v, int act) {
  switch (act) {
    case 1: return orc_silu(v);
    case 2: return v > 0.0f ? v : 0.0f;
    case 3: return orc_sigmoid(v);
    default: return v;
  }
}

void orc_unary(const float* x, float* y, long n, int act, int threads) {
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (long i = 0; i < n; ++i) y[i] = act_apply(x[i], act);
}

/* Rows of [0, m) that MultiplyPacked runs through the 12/6/4-row micro-kernels
 * (GemmKernel.cs:746-790); the remaining rows take MultiplyRow + ScaleColumns. */
static int grouped_rows(int m, int mr12) {
  int row = 0;
  if (mr12)
    while (row + 12 <= m) row += 12;
  while (row + 6 <= m) row += 6; /* UseMr6 default */
  while (row + 4 <= m) row += 4;
  return row;
}

/* Register-blocked accumulation: acc[r][0..15] (row pitch ldacc) for R <= 6
 * rows continues, for t = 0..K-1 in ascending order, the per-element chain
 * acc = fma(A[r][t], B[t][j], acc) (A row r at A + r*lda, B row t at B + t*ldb).
 * Each lane of _mm256_fmadd_ps is one fmaf, so every element's chain and
 * rounding are those of the scalar loop; only the loop nest is blocked, as the
 * reference's 12/6-row x 16-column micro-kernels block it
 * (GemmKernel.cs:1070-1304). */
static inline __attribute__((always_inline)) void mk_rows(int R, const float* A, long lda, const float* B, long ldb,
                                                         int K, float* acc, long ldacc) {
  __m256 c0[6], c1[6];
  for (int r = 0; r < 6; ++r) {
    if (r < R) {
      c0[r] = _mm256_loadu_ps(acc + r * ldacc);
      c1[r] = _mm256_loadu_ps(acc + r * ldacc + 8);
    }
  }
  for (int t = 0; t < K; ++t) {
    const __m256 b0 = _mm256_loadu_ps(B + (long)t * ldb);
    const __m256 b1 = _mm256_loadu_ps(B + (long)t * ldb + 8);
    for (int r = 0; r < 6; ++r) {
      if (r < R) {
        const __m256 av = _mm256_broadcast_ss(A + r * lda + t);
        c0[r] = _mm256_fmadd_ps(av, b0, c0[r]);
        c1[r] = _mm256_fmadd_ps(av, b1, c1[r]);
      }
    }
  }
  for (int r = 0; r < 6; ++r) {
    if (r < R) {
      _mm256_storeu_ps(acc + r * ldacc, c0[r]);
      _mm256_storeu_ps(acc + r * ldacc + 8, c1[r]);
    }
  }
}

static void mk_block(int R, const float* A, long lda, const float* B, long ldb, int K, float* acc, long ldacc) {
  switch (R) {
    case 6: mk_rows(6, A, lda, B, ldb, K, acc, ldacc); break;
    case 5: mk_rows(5, A, lda, B, ldb, K, acc, ldacc); break;
    case 4: mk_rows(4, A, lda, B, ldb, K, acc, ldacc); break;
    case 3: mk_rows(3, A, lda, B, ldb, K, acc, ldacc); break;
    case 2: mk_rows(2, A, lda, B, ldb, K, acc, ldacc); break;
    default: mk_rows(1, A, lda, B, ldb, K, acc, ldacc); break;
  }
}

/* The same chains for two 16-column panels at once (B0 / B1, row pitches
 * ldb0 / ldb1, accumulators acc0 / acc1) with 512-bit vectors: each lane of
 * _mm512_fmadd_ps is one fmaf, so the results equal mk_rows' bit for bit.
 * Used only when the CPU reports AVX-512F (checked at run time). */
static inline __attribute__((always_inline, target("avx512f"))) void mk_pair_rows(
    int R, const float* A, long lda, const float* B0, long ldb0, const float* B1, long ldb1, int K, float* acc0,
    float* acc1, long ldacc) {
  __m512 c0[6], c1[6];
  for (int r = 0; r < 6; ++r) {
    if (r < R) {
      c0[r] = _mm512_loadu_ps(acc0 + r * ldacc);
      c1[r] = _mm512_loadu_ps(acc1 + r * ldacc);
    }
  }
  for (int t = 0; t < K; ++t) {
    const __m512 b0 = _mm512_loadu_ps(B0 + (long)t * ldb0);
    const __m512 b1 = _mm512_loadu_ps(B1 + (long)t * ldb1);
    for (int r = 0; r < 6; ++r) {
      if (r < R) {
        const __m512 av = _mm512_set1_ps(A[r * lda + t]);
        c0[r] = _mm512_fmadd_ps(av, b0, c0[r]);
        c1[r] = _mm512_fmadd_ps(av, b1, c1[r]);
      }
    }
  }
  for (int r = 0; r < 6; ++r) {
    if (r < R) {
      _mm512_storeu_ps(acc0 + r * ldacc, c0[r]);
      _mm512_storeu_ps(acc1 + r * ldacc, c1[r]);
    }
  }
}

static __attribute__((target("avx512f"))) void mk_pair(int R, const float* A, long lda, const float* B0, long ldb0,
                                                        const float* B1, long ldb1, int K, float* acc0, float* acc1,
                                                        long ldacc) {
  switch (R) {
    case 6: mk_pair_rows(6, A, lda, B0, ldb0, B1, ldb1, K, acc0, acc1, ldacc); break;
    case 5: mk_pair_rows(5, A, lda, B0, ldb0, B1, ldb1, K, acc0, acc1, ldacc); break;
    case 4: mk_pair_rows(4, A, lda, B0, ldb0, B1, ldb1, K, acc0, acc1, ldacc); break;
    case 3: mk_pair_rows(3, A, lda, B0, ldb0, B1, ldb1, K, acc0, acc1, ldacc); break;
    case 2: mk_pair_rows(2, A, lda, B0, ldb0, B1, ldb1, K, acc0, acc1, ldacc); break;
    default: mk_pair_rows(1, A, lda, B0, ldb0, B1, ldb1, K, acc0, acc1, ldacc); break;
  }
}

static int have_avx512(void) {
  static int v = -1;
  if (v < 0) v = __builtin_cpu_supports("avx512f") ? 1 : 0;
  return v;
}

/* acc[r][j] for r < R, j < J (pitch ldacc): full 16-column panels through the
 * blocked kernel (two at a time with AVX-512), the remaining columns through
 * the scalar chain. */
static void accumulate(int R, int J, const float* A, long lda, const float* B, long ldb, int K, float* acc,
                       long ldacc) {
  const int J16 = J / 16 * 16;
  int j0 = 0;
  if (have_avx512())
    for (; j0 + 32 <= J16; j0 += 32) mk_pair(R, A, lda, B + j0, ldb, B + j0 + 16, ldb, K, acc + j0, acc + j0 + 16, ldacc);
  for (int j = j0; j < J16; j += 16) mk_block(R, A, lda, B + j, ldb, K, acc + j, ldacc);
  for (int r = 0; r < R; ++r)
    for (int j = J16; j < J; ++j) {
      float v = acc[r * ldacc + j];
      for (int t = 0; t < K; ++t) v = fmaf(A[r * lda + t], B[(long)t * ldb + j], v);
      acc[r * ldacc + j] = v;
    }
}

enum { kGemmCols = 128 };

void orc_gemm_f32(const float* a, int lda, const float* b, int ldb, int m, int k, int n, const float* row_bias,
                  const float* col_bias, const float* col_scale, int mr12, int act, float* c, int ldc, int threads) {
  const int fused_rows = col_scale ? grouped_rows(m, mr12) : m;
  const int full_cols = (n / 16) * 16;
  const long nrb = (m + 5) / 6, ncb = (n + kGemmCols - 1) / kGemmCols;
  /* B's full 16-column panels packed [n/16][k][16] (GemmKernel.Pack, :418-438), so a
   * panel's k rows are contiguous */
  float* bp = (float*)malloc(sizeof(float) * (size_t)(full_cols > 0 ? full_cols : 1) * (k > 0 ? k : 1));
#pragma omp parallel num_threads(nthreads(threads))
  {
    float acc[6 * kGemmCols];
#pragma omp for schedule(static)
    for (long pt = 0; pt < (long)(full_cols / 16) * k; ++pt) {
      const long p = pt / k, t = pt % k;
      memcpy(bp + (p * k + t) * 16, b + (size_t)t * ldb + p * 16, 16 * sizeof(float));
    }
    /* column block outer: a thread's consecutive row blocks reuse B's k x 128 block from cache */
#pragma omp for schedule(static)
    for (long task = 0; task < nrb * ncb; ++task) {
      const int i0 = (int)(task % nrb) * 6, j0 = (int)(task / nrb) * kGemmCols;
      const int R = m - i0 < 6 ? m - i0 : 6, J = n - j0 < kGemmCols ? n - j0 : kGemmCols;
      for (int r = 0; r < R; ++r)
        for (int jj = 0; jj < J; ++jj) {
          const int i = i0 + r, j = j0 + jj;
          acc[r * kGemmCols + jj] = col_scale ? 0.0f : (col_bias ? col_bias[j] : (row_bias ? row_bias[i] : 0.0f));
        }
      const int J16 = (j0 + J <= full_cols) ? J : full_cols - j0;
      int jj0 = 0;
      if (have_avx512())
        for (; jj0 + 32 <= J16; jj0 += 32)
          mk_pair(R, a + (size_t)i0 * lda, lda, bp + (size_t)(j0 + jj0) * k, 16, bp + (size_t)(j0 + jj0 + 16) * k, 16,
                  k, acc + jj0, acc + jj0 + 16, kGemmCols);
      for (int jj = jj0; jj < J16; jj += 16)
        mk_block(R, a + (size_t)i0 * lda, lda, bp + (size_t)(j0 + jj) * k, 16, k, acc + jj, kGemmCols);
      if (J16 < J)
        accumulate(R, J - J16, a + (size_t)i0 * lda, lda, b + j0 + J16, ldb, k, acc + J16, kGemmCols);
      for (int r = 0; r < R; ++r) {
        const int i = i0 + r;
        float* ci = c + (size_t)i * ldc;
        for (int jj = 0; jj < J; ++jj) {
          const int j = j0 + jj;
          const float s = acc[r * kGemmCols + jj];
          float v;
          if (!col_scale) {
            v = s;
          } else if (i < fused_rows && j < full_cols) {
            v = fmaf(s, col_scale[j], col_bias ? col_bias[j] : 0.0f); /* Multiply12Rows epilogue :1210-1241 */
          } else {
            v = s * col_scale[j]; /* ScaleColumns :1594-1608 */
            if (col_bias) v = v + col_bias[j];
          }
          ci[j] = act_apply(v, act);
        }
      }
    }
  }
  free(bp);
}

void orc_minmax(const float* x, long n, float* out_min, float* out_max) {
  float mn = 0.0f, mx = 0.0f;
  for (long i = 0; i < n; ++i) {
    const float v = x[i];
    if (v != v) continue;
    if (v < mn) mn = v;
    if (v > mx) mx = v;
  }
  *out_min = mn;
  *out_max = mx;
}

void orc_dql_params(float mn, float mx, float* scale, int* zero_point) {
  float s = (mx - mn) / 255.0f;
  if (!(s > 0.0f)) s = 1.0f;
  const float z = nearbyintf(-mn / s); /* MathF.Round(.., ToEven) */
  int zi = (z != z) ? 0 : (z > 2147483520.0f ? 2147483647 : (z < -2147483648.0f ? (int)0x80000000 : (int)z));
  if (zi < 0) zi = 0;
  if (zi > 255) zi = 255;
  *scale = s;
  *zero_point = zi;
}

static inline float quant_value(float x, float inverse, int zp) {
  float q = nearbyintf(x * inverse) + (float)zp;
  q = minps(255.0f, maxps(0.0f, q)); /* Avx.Min(vMax, Avx.Max(vMin, q)) */
  return q;
}

void orc_quantize_u8(const float* x, long n, float scale, int zero_point, uint8_t* q, int threads) {
  const float inverse = 1.0f / scale;
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (long i = 0; i < n; ++i) {
    const float v = quant_value(x[i], inverse, zero_point);
    q[i] = (v != v) ? 0 : (uint8_t)v;
  }
}

void orc_dqmm(const float* a, int m, int k, const void* w, int w_signed, const int32_t* w_zp, int n_zp,
              const float* w_scale, int n_scale, const float* bias, int n, int mr12, float* y, uint8_t* q_out,
              int32_t* acc_out, float* params_out, int threads) {
  float mn, mx, scale;
  int zp;
  orc_minmax(a, (long)m * k, &mn, &mx);
  orc_dql_params(mn, mx, &scale, &zp);
  if (params_out) {
    params_out[0] = scale;
    params_out[1] = (float)zp;
  }
  const float inverse = 1.0f / scale;
  float* act = (float*)malloc(sizeof(float) * (size_t)m * k);
  float* wid = (float*)malloc(sizeof(float) * (size_t)k * n);
  float* combined = (float*)malloc(sizeof(float) * (size_t)n);
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (long i = 0; i < (long)m * k; ++i) {
    const float q = quant_value(a[i], inverse, zp); /* QuantizeAndWiden :280-335 */
    act[i] = q - (float)zp;
    if (q_out) q_out[i] = (q != q) ? 0 : (uint8_t)q;
  }
  for (int t = 0; t < k; ++t)
    for (int j = 0; j < n; ++j) {
      const int wv = w_signed ? ((const int8_t*)w)[(size_t)t * n + j] : ((const uint8_t*)w)[(size_t)t * n + j];
      wid[(size_t)t * n + j] = (float)(wv - (n_zp > 1 ? w_zp[j] : (n_zp == 1 ? w_zp[0] : 0))); /* WidenWeights */
    }
  for (int j = 0; j < n; ++j) combined[j] = scale * w_scale[n_scale > 1 ? j : 0]; /* CombinedScale :203-221 */
  if (acc_out) {
    float* accf = (float*)malloc(sizeof(float) * (size_t)m * n);
    orc_gemm_f32(act, k, wid, n, m, k, n, NULL, NULL, NULL, mr12, 0, accf, n, threads);
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
    for (long i = 0; i < (long)m * n; ++i) acc_out[i] = (int32_t)accf[i];
    free(accf);
  }
  orc_gemm_f32(act, k, wid, n, m, k, n, NULL, bias, combined, mr12, 0, y, n, threads);
  free(act);
  free(wid);
  free(combined);
}

void orc_matmul_integer(const void* a, int a_signed, int m, int k, int a_zp, const void* w, int w_signed,
                        const int32_t* w_zp, int n_zp, int n, int32_t* acc, int threads) {
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (int i = 0; i < m; ++i)
    for (int j = 0; j < n; ++j) {
      int64_t s = 0;
      const int zpj = n_zp > 1 ? w_zp[j] : (n_zp == 1 ? w_zp[0] : 0);
      for (int t = 0; t < k; ++t) {
        const int wv = w_signed ? ((const int8_t*)w)[(size_t)t * n + j] : ((const uint8_t*)w)[(size_t)t * n + j];
        const int av = a_signed ? ((const int8_t*)a)[(size_t)i * k + t] : ((const uint8_t*)a)[(size_t)i * k + t];
        s += (int64_t)(av - a_zp) * (wv - zpj);
      }
      acc[(size_t)i * n + j] = (int32_t)s;
    }
}

void orc_conv2d(const float* x, int N, int C, int H, int W, const float* w, int M, int kh, int kw, int sh, int sw,
                int pt, int pl, int dh, int dw, int group, const float* bias, int act, float* y, int OH, int OW,
                int threads) {
  const int cpg = C / group, mpg = M / group;
  const int K = cpg * kh * kw; /* im2col row order (ic, ky, kx), ConvKernels.cs:262-462 */
  if (group == 1 && kh == 1 && kw == 1 && sh == 1 && sw == 1 && pt == 0 && pl == 0 && OH == H && OW == W) {
    /* 1x1, stride 1, unpadded: the image [C][H*W] already is the column
     * matrix, so W [M][C] times it through orc_gemm_f32 with the bias as the
     * row bias -- the same chains (acc = bias, then fma over c ascending). */
    const long HW = (long)H * W;
    for (int nb = 0; nb < N; ++nb)
      orc_gemm_f32(w, C, x + (size_t)nb * C * HW, (int)HW, M, C, (int)HW, bias, NULL, NULL, 0, act,
                   y + (size_t)nb * M * HW, (int)HW, threads);
    return;
  }
  if (group == 1 && (OW < 64 || OW % 16 != 0)) {
    /* Narrow images (an output row fills few or no 16-wide panels): the whole
     * image's columns [K][OH*OW] (FillColumns, zero outside the image), then
     * W [M][K] times them through orc_gemm_f32 with the bias as the row bias.
     * Every output's chain is the same as below -- acc = bias, then
     * fma(W[o][t], col[t][p], acc) for t ascending -- blocked over all of the
     * image's pixels instead of one output row at a time. */
    const long HW = (long)OH * OW;
    float* col = (float*)malloc(sizeof(float) * (size_t)K * (size_t)(HW > 0 ? HW : 1));
    for (int nb = 0; nb < N; ++nb) {
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
      for (long r = 0; r < (long)K * OH; ++r) {
        const int t = (int)(r / OH), oy = (int)(r % OH);
        const int ic = t / (kh * kw), ky = (t / kw) % kh, kx = t % kw;
        const float* xc = x + ((size_t)nb * C + ic) * H * W;
        const int iy = oy * sh - pt + ky * dh;
        float* cr = col + (size_t)t * HW + (size_t)oy * OW;
        for (int ox = 0; ox < OW; ++ox) {
          const int ix = ox * sw - pl + kx * dw;
          cr[ox] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? xc[(size_t)iy * W + ix] : 0.0f;
        }
      }
      orc_gemm_f32(w, K, col, (int)HW, M, K, (int)HW, bias, NULL, NULL, 0, act, y + (size_t)nb * M * HW, (int)HW,
                   threads);
    }
    free(col);
    return;
  }
  const long tasks = (long)N * group * OH;
#pragma omp parallel num_threads(nthreads(threads))
  {
    float* accb = (float*)malloc(sizeof(float) * (size_t)mpg * OW);
    float* col = (float*)malloc(sizeof(float) * (size_t)K * OW);
#pragma omp for schedule(static)
    for (long task = 0; task < tasks; ++task) {
      const int oy = (int)(task % OH);
      const int g = (int)((task / OH) % group);
      const int nb = (int)(task / ((long)OH * group));
      for (int ic = 0; ic < cpg; ++ic) { /* FillColumns (:525-654): zero outside the image */
        const float* xc = x + ((size_t)nb * C + (size_t)g * cpg + ic) * H * W;
        for (int ky = 0; ky < kh; ++ky) {
          const int iy = oy * sh - pt + ky * dh;
          for (int kx = 0; kx < kw; ++kx) {
            float* cr = col + (size_t)((ic * kh + ky) * kw + kx) * OW;
            for (int ox = 0; ox < OW; ++ox) {
              const int ix = ox * sw - pl + kx * dw;
              cr[ox] = (iy >= 0 && iy < H && ix >= 0 && ix < W) ? xc[(size_t)iy * W + ix] : 0.0f;
            }
          }
        }
      }
      for (int o = 0; o < mpg; ++o) {
        const float b0 = bias ? bias[g * mpg + o] : 0.0f;
        for (int ox = 0; ox < OW; ++ox) accb[(size_t)o * OW + ox] = b0;
      }
      /* acc[o][ox] from the row bias, then fma(W[o][t], col[t][ox], acc) for t ascending */
      const float* wg = w + (size_t)g * mpg * K;
      for (int o0 = 0; o0 < mpg; o0 += 6) {
        const int R = mpg - o0 < 6 ? mpg - o0 : 6;
        accumulate(R, OW, wg + (size_t)o0 * K, K, col, OW, K, accb + (size_t)o0 * OW, OW);
      }
      for (int o = 0; o < mpg; ++o) {
        float* yo = y + (((size_t)nb * M + (size_t)g * mpg + o) * OH + oy) * OW;
        const float* ao = accb + (size_t)o * OW;
        for (int ox = 0; ox < OW; ++ox) yo[ox] = act_apply(ao[ox], act);
      }
    }
    free(accb);
    free(col);
  }
}

/* VectorMath.MaxRow (VectorMath.cs:246-272). */
static float max_row(const float* s, int len) {
  float mx = -INFINITY;
  if (len >= 8) {
    float acc[8];
    for (int l = 0; l < 8; ++l) acc[l] = s[l];
    int i = 8;
    for (; i <= len - 8; i += 8)
      for (int l = 0; l < 8; ++l) acc[l] = maxps(acc[l], s[i + l]);
    float lo[4];
    for (int l = 0; l < 4; ++l) lo[l] = maxps(acc[l], acc[l + 4]);
    /* Vector128.Max(lo, Shuffle(lo, 2,3,0,1)) then MathF.Max(e0, e1) */
    const float m0 = fmaxf(lo[0], lo[2]), m1 = fmaxf(lo[1], lo[3]);
    mx = fmaxf(m0, m1);
    for (; i < len; ++i) mx = fmaxf(mx, s[i]);
  } else {
    for (int i = 0; i < len; ++i) mx = fmaxf(mx, s[i]);
  }
  return mx;
}

/* VectorMath.SumExp pointer form (VectorMath.cs:355-384): 8 lane partials,
 * lanes summed in order, scalar tail with MathF.Exp. */
static float sum_exp(const float* src, float* dst, int n, float bias) {
  int i = 0;
  float total = 0.0f;
  float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (; i <= n - 8; i += 8)
    for (int l = 0; l < 8; ++l) {
      const float e = orc_exp(src[i + l] - bias);
      dst[i + l] = e;
      lane[l] = lane[l] + e;
    }
  for (int l = 0; l < 8; ++l) total += lane[l];
  for (; i < n; ++i) {
    const float e = expf(src[i] - bias);
    dst[i] = e;
    total += e;
  }
  return total;
}

/* VectorMath.SoftmaxRow (VectorMath.cs:282): MaxRow, SumExp, Scale by 1/sum. */
void orc_softmax_rows(const float* x, float* y, long rows, int len, int threads) {
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (long r = 0; r < rows; ++r) {
    const float* s = x + (size_t)r * len;
    float* d = y + (size_t)r * len;
    const float mx = max_row(s, len);
    const float total = sum_exp(s, d, len, mx);
    const float inv = 1.0f / total;
    for (int j = 0; j < len; ++j) d[j] = d[j] * inv;
  }
}

/* AttentionOps.Dot (:692-711): 8-lane FMA partials, horizontal sum, unfused tail. */
static float dot8(const float* a, const float* b, int n) {
  int i = 0;
  float sum = 0.0f;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (; i + 8 <= n; i += 8)
    for (int l = 0; l < 8; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
  /* HorizontalSum (:716-722): lo = low+high; lo += shuffle(2,3,0,1); lo += shuffle(1,0,3,2) */
  float lo[4];
  for (int l = 0; l < 4; ++l) lo[l] = acc[l] + acc[l + 4];
  float s2[4] = {lo[0] + lo[2], lo[1] + lo[3], lo[2] + lo[0], lo[3] + lo[1]};
  sum = s2[0] + s2[1];
  for (; i < n; ++i) sum += a[i] * b[i];
  return sum;
}

void orc_attention(const float* q, const float* k, const float* v, const float* mask, int mask_rows, int B, int T,
                   int H, int D, float scale, int heads_form, int out_head_space, int block_min_seq, float* out,
                   int threads) {
  const int width = H * D;
  const int q_stride_t = heads_form ? width : D;
  const int v_stride_t = heads_form ? width : D;
  const int out_stride = out_head_space ? D : width;
  const int mask_batch = mask ? mask_rows * T : 0;
  const int mask_row = (mask && mask_rows != 1) ? T : 0;
  const int use_blocks = T > block_min_seq;
#pragma omp parallel num_threads(nthreads(threads))
  {
    float* qrow = (float*)malloc(sizeof(float) * (size_t)D);
    float* keys = (float*)malloc(sizeof(float) * (size_t)T * D);
    float* s = (float*)malloc(sizeof(float) * (size_t)T);
    float* o = (float*)malloc(sizeof(float) * (size_t)D);
#pragma omp for schedule(static)
    for (int bh = 0; bh < B * H; ++bh) {
      const int bi = bh / H, hi = bh % H;
      const int plane = heads_form ? bi * T * width + hi * D : bh * T * D;
      /* K relayout to [T][D] (:315-332). */
      for (int ti = 0; ti < T; ++ti)
        for (int di = 0; di < D; ++di)
          keys[(size_t)ti * D + di] = heads_form ? k[(size_t)plane + (size_t)ti * width + di]
                                                 : k[(size_t)bh * D * T + (size_t)di * T + ti];
      for (int r = 0; r < T; ++r) {
        const float* src = q + plane + (size_t)r * q_stride_t;
        for (int di = 0; di < D; ++di) qrow[di] = src[di] * scale;
        if (use_blocks) {
          /* ComputeBlocks: S = MultiplyPacked(q', K^T): FMA chain from 0 over d. */
          for (int j = 0; j < T; ++j) {
            float acc = 0.0f;
            for (int di = 0; di < D; ++di) acc = fmaf(qrow[di], keys[(size_t)j * D + di], acc);
            s[j] = acc;
          }
        } else {
          for (int j = 0; j < T; ++j) s[j] = dot8(qrow, keys + (size_t)j * D, D);
        }
        if (mask) {
          const float* mr = mask + (size_t)mask_batch * bi + (size_t)mask_row * r;
          for (int j = 0; j < T; ++j) s[j] += mr[j];
        }
        const float mx = max_row(s, T);
        const float total = sum_exp(s, s, T, mx);
        float* dst = out + (out_head_space ? (size_t)bh * T * D + (size_t)r * D : ((size_t)bi * T + r) * width + hi * D);
        if (use_blocks) {
          /* lazy softmax: O = e.V (FMA chain over t from 0), then O *= 1/sum (:590-643). */
          const float pinv = 1.0f / total;
          for (int di = 0; di < D; ++di) {
            float acc = 0.0f;
            for (int j = 0; j < T; ++j) acc = fmaf(s[j], v[plane + (size_t)j * v_stride_t + di], acc);
            dst[di] = acc * pinv;
          }
        } else {
          /* ComputeRows: SoftmaxRow then Axpy accumulation skipping zero weights (:402-421). */
          const float inv = 1.0f / total;
          for (int j = 0; j < T; ++j) s[j] = s[j] * inv;
          for (int di = 0; di < D; ++di) o[di] = 0.0f;
          const int dvec = D & ~7;
          for (int j = 0; j < T; ++j) {
            const float wgt = s[j];
            if (wgt == 0.0f) continue;
            const float* vr = v + plane + (size_t)j * v_stride_t;
            for (int di = 0; di < dvec; ++di) o[di] = fmaf(wgt, vr[di], o[di]);
            for (int di = dvec; di < D; ++di) o[di] += wgt * vr[di];
          }
          for (int di = 0; di < D; ++di) dst[di] = o[di];
        }
      }
    }
    free(qrow);
    free(keys);
    free(s);
    free(o);
  }
  (void)out_stride;
}

void orc_dfl(const float* x, int B, int sides, int bins, int pixels, float* out, int threads) {
  const int block = 64; /* DflLayer.BlockColumns */
  const int blocks_per_side = (pixels + block - 1) / block;
  const long tasks = (long)B * sides * blocks_per_side;
#pragma omp parallel num_threads(nthreads(threads))
  {
    float* ex = (float*)malloc(sizeof(float) * (size_t)bins * block);
#pragma omp for schedule(static)
    for (long task = 0; task < tasks; ++task) {
      const int bi = (int)(task % blocks_per_side);
      const long grp = task / blocks_per_side;
      const float* src = x + (size_t)grp * bins * pixels;
      float* dst = out + (size_t)grp * pixels;
      const int column = bi * block;
      const int width = (pixels - column) < block ? (pixels - column) : block;
      const int vend = width & ~7;
      for (int j = 0; j < width; ++j) {
        float mx = -INFINITY;
        for (int b = 0; b < bins; ++b) {
          const float xv = src[(size_t)b * pixels + column + j];
          mx = (j < vend) ? maxps(mx, xv) : fmaxf(mx, xv);
        }
        float total = 0.0f;
        for (int b = 0; b < bins; ++b) {
          const float sh = src[(size_t)b * pixels + column + j] - mx;
          /* VectorMath.Exp(float*, float*, n): vector lanes for i <= n-8, MathF.Exp tail */
          const float e = (j < vend) ? orc_exp(sh) : expf(sh);
          ex[(size_t)b * block + j] = e;
          total = total + e;
        }
        const float inv = 1.0f / total;
        float wsum = 0.0f;
        for (int b = 0; b < bins; ++b) {
          const float e = ex[(size_t)b * block + j];
          if (j < vend)
            wsum = fmaf(e * inv, (float)b, wsum);
          else
            wsum = wsum + (e * inv) * (float)b;
        }
        dst[column + j] = wsum;
      }
    }
    free(ex);
  }
}

void orc_layernorm(const float* x, int outer, int inner, const float* gamma, const float* beta, float eps, float* y,
                   int threads) {
#pragma omp parallel for num_threads(nthreads(threads)) schedule(static)
  for (int o = 0; o < outer; ++o) {
    const float* xr = x + (size_t)o * inner;
    float* yr = y + (size_t)o * inner;
    double sum = 0.0, sumsq = 0.0;
    int i = 0;
    if (inner >= 16) {
      float vs[16], vq[16];
      for (int l = 0; l < 16; ++l) vs[l] = vq[l] = 0.0f;
      for (; i <= inner - 16; i += 16)
        for (int l = 0; l < 16; ++l) {
          const float v = xr[i + l];
          vs[l] = vs[l] + v;
          vq[l] = vq[l] + v * v;
        }
      for (int l = 0; l < 16; ++l) {
        sum += vs[l];
        sumsq += vq[l];
      }
    }
    for (; i < inner; ++i) {
      const float v = xr[i];
      sum += v;
      sumsq += (double)v * v;
    }
    const double mean_d = sum / inner;
    double var_d = sumsq / inner - mean_d * mean_d;
    if (var_d < 0) var_d = 0;
    const float mean = (float)mean_d;
    const float inv_std = 1.0f / sqrtf((float)var_d + eps);
    for (int j = 0; j < inner; ++j) {
      float r = (xr[j] - mean) * inv_std;
      r = r * (gamma ? gamma[j] : 1.0f);
      if (beta) r = r + beta[j];
      yr[j] = r;
    }
  }
}

/* ImageGeometry.Contain + AxisMap.Bilinear + ImageTensor.ToChw (see oracle.h). */
void orc_letterbox(const uint8_t* pixels, int width, int height, int row_stride, int bytes_per_pixel, int bgr, int tw,
                   int th, float* dst, int* placement) {
  const float gx = (float)tw / (float)width, gy = (float)th / (float)height;
  const float gain = gx < gy ? gx : gy; /* MathF.Min */
  int rw = (int)nearbyintf((float)width * gain), rh = (int)nearbyintf((float)height * gain);
  rw = rw < 1 ? 1 : (rw > tw ? tw : rw);
  rh = rh < 1 ? 1 : (rh > th ? th : rh);
  const int ox = (tw - rw) / 2, oy = (th - rh) / 2;
  placement[0] = rw;
  placement[1] = rh;
  placement[2] = ox;
  placement[3] = oy;
  const float pad = 114.0f / 255.0f;
  const float g = 1.0f / (255.0f * 1.0f);
  const float bias = -0.0f / 1.0f;
  const long plane = (long)th * tw;
  for (long i = 0; i < 3 * plane; ++i) dst[i] = pad;
  for (int dy = 0; dy < rh; ++dy) {
    float sy = ((float)dy + 0.5f) * (float)height / (float)rh - 0.5f;
    sy = sy < 0.0f ? 0.0f : (sy > (float)(height - 1) ? (float)(height - 1) : sy);
    const int y0 = (int)sy, y1 = y0 + 1 < height - 1 ? y0 + 1 : height - 1;
    const float fy = sy - (float)y0, omfy = 1.0f - fy;
    for (int dx = 0; dx < rw; ++dx) {
      float sx = ((float)dx + 0.5f) * (float)width / (float)rw - 0.5f;
      sx = sx < 0.0f ? 0.0f : (sx > (float)(width - 1) ? (float)(width - 1) : sx);
      const int x0 = (int)sx, x1 = x0 + 1 < width - 1 ? x0 + 1 : width - 1;
      const float fx = sx - (float)x0, omfx = 1.0f - fx;
      for (int c = 0; c < 3; ++c) {
        const int co = bgr ? 2 - c : c;
        const uint8_t* t = pixels + (long)y0 * row_stride;
        const uint8_t* b = pixels + (long)y1 * row_stride;
        const float top = (float)t[x0 * bytes_per_pixel + co] * omfx + (float)t[x1 * bytes_per_pixel + co] * fx;
        const float bot = (float)b[x0 * bytes_per_pixel + co] * omfx + (float)b[x1 * bytes_per_pixel + co] * fx;
        dst[c * plane + (long)(oy + dy) * tw + ox + dx] = (top * omfy + bot * fy) * g + bias;
      }
    }
  }
}
