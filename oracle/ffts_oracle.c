/*
 * ffts_oracle.c -- CPU oracle for the FFTSparse block-mask selection path.
 *
 * TEST INFRASTRUCTURE.  This is the checker the parity tests compare the CUDA
 * kernels against; nothing on the product path links or calls it.
 *
 * It restates, in plain C, the mask path of `myattn_prefill`
 * (attn_src/fft_attn/my_attn_v7.py:454-641) with every floating-point
 * decision value defined by one fixed sequence of IEEE operations (the
 * "canonical" arithmetic), so that the GPU kernels and this file produce
 * bit-identical block masks:
 *
 *   pooling      fp32 sums in row order, / block_size, rounded to the
 *                input dtype                               (ref :105-114)
 *   lag corr.    zero-padded radix-2 DIT FFT in fp32 of z = q + i k per
 *                channel, cross spectrum summed over channels, one inverse
 *                FFT, then the reference's fp32 post-processing  (ref :117-157)
 *   scores       exact products, fp64 sums over d in order, / sqrt(D) in
 *                fp64, rounded once to fp32                (ref :234-249)
 *   statistics   fp64 reductions in a fixed 256-lane order (ref :301-383)
 *   top-k        ties broken by lowest block index (torch.topk leaves the
 *                order of ties unspecified)                (ref :54-72,
 *                :256-294, :390-447)
 *   quantile     torch.quantile's linear interpolation with its fp32 rank
 *                arithmetic and FMA lerp                   (ref :196-202)
 *
 * It is pinned against the reference itself: tests/golden/make_golden.py
 * runs the reference's my_attn_v7.py on the CPU and the unit tests compare
 * this file's masks with those fixtures.
 *
 * Build: cc -O2 -ffp-contract=off -fopenmp -shared -fPIC (see oracle/build.py).
 * -ffp-contract=off is required: contraction into FMA would change results.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../include/fftsparse_b200.h"

#if defined(__FP_FAST_FMA) && 0
#endif

/* ------------------------------------------------------------------ bits */

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float round_to_dtype(float f, int dtype) {
  return dtype == FFTS_DTYPE_BF16 ? bf16_to_f32(f32_to_bf16_rne(f)) : f;
}

/* Monotone key: larger float -> larger key; -0 is mapped to +0 first. */
static inline uint32_t f32_key(float f) {
  if (f == 0.0f) f = 0.0f;
  uint32_t u;
  memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* ---------------------------------------------------------------- pooling */

/* Canonical block mean: each channel's block_size values are summed in fp32 in
 * row order starting from +0 (rows past L contribute +0), the sum is divided
 * by block_size in fp32 and rounded to the dtype. */
int ffo_pool(const void *x, int dtype, int64_t B, int64_t H, int64_t L, int64_t D,
             int64_t sb, int64_t sh, int64_t sl, int bs, void *out) {
  const int64_t N = (L + bs - 1) / bs;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t bh = 0; bh < B * H; ++bh) {
    for (int64_t n = 0; n < N; ++n) {
      const int64_t b = bh / H, h = bh % H;
      for (int64_t d = 0; d < D; ++d) {
        float acc = 0.0f;
        for (int r = 0; r < bs; ++r) {
          const int64_t t = n * bs + r;
          float v = 0.0f;
          if (t < L) {
            const int64_t off = b * sb + h * sh + t * sl + d;
            v = dtype == FFTS_DTYPE_BF16 ? bf16_to_f32(((const uint16_t *)x)[off]) : ((const float *)x)[off];
          }
          acc = acc + v;
        }
        const float mean = acc / (float)bs;
        const int64_t o = ((b * H + h) * N + n) * D + d;
        if (dtype == FFTS_DTYPE_BF16)
          ((uint16_t *)out)[o] = f32_to_bf16_rne(mean);
        else
          ((float *)out)[o] = mean;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------- RoPE */

/* The rotary embedding the caller of myattn_prefill applies to q and k before
 * the call (eval/LongBench/pred.py:191-194, HF apply_rotary_pos_emb):
 * out = x * cos + rotate_half(x) * sin with rotate_half(x) = cat(-x[D/2:], x[:D/2]),
 * evaluated as torch evaluates that bf16 expression op by op: each product in
 * fp32 rounded to bf16, then the sum in fp32 rounded to bf16 (the negation is
 * exact).  x is token-major (head h of token t at x + t * ld + h * D), cos and
 * sin are bf16 [L, D] with row stride cs_ld, out is head-major [H, L, D]. */
int ffo_rope(const uint16_t *x, int64_t ld, int64_t L, int64_t H, int64_t D, const uint16_t *cos_t,
             const uint16_t *sin_t, int64_t cs_ld, uint16_t *out) {
  if (D % 2) return -1;
  const int64_t half = D / 2;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t h = 0; h < H; ++h) {
    for (int64_t t = 0; t < L; ++t) {
      const uint16_t *row = x + t * ld + h * D;
      for (int64_t d = 0; d < D; ++d) {
        const float xv = bf16_to_f32(row[d]);
        const float rv = d < half ? -bf16_to_f32(row[d + half]) : bf16_to_f32(row[d - half]);
        const float a = bf16_to_f32(f32_to_bf16_rne(xv * bf16_to_f32(cos_t[t * cs_ld + d])));
        const float b = bf16_to_f32(f32_to_bf16_rne(rv * bf16_to_f32(sin_t[t * cs_ld + d])));
        out[(h * L + t) * D + d] = f32_to_bf16_rne(a + b);
      }
    }
  }
  return 0;
}

/* -------------------------------------------------------------------- FFT */

static int ilog2(int64_t m) {
  int r = 0;
  while ((1LL << r) < m) ++r;
  return r;
}

static uint32_t bitrev(uint32_t x, int bits) {
  uint32_t r = 0;
  for (int i = 0; i < bits; ++i) r |= ((x >> i) & 1u) << (bits - 1 - i);
  return r;
}

/* Forward twiddles w_j = cos(2*pi*j/M) - i sin(2*pi*j/M), j < M/2, computed in
 * double and rounded to fp32. */
static void make_twiddles(int M, float *twr, float *twi) {
  for (int j = 0; j < M / 2; ++j) {
    const double a = (2.0 * M_PI * (double)j) / (double)M;
    twr[j] = (float)cos(a);
    twi[j] = (float)(-sin(a));
  }
}

/* In-place radix-2 DIT on input already in bit-reversed order.  Every
 * butterfly: t = w*b (two products, one sub / one add), a' = a + t,
 * b' = a - t, all in fp32.  `inverse` conjugates the twiddles. */
static void fft_dit(float *re, float *im, int M, const float *twr, const float *twi,
                    int inverse) {
  for (int h = 1; h < M; h <<= 1) {
    const int step = M / (2 * h);
    for (int g = 0; g < M; g += 2 * h) {
      for (int k = 0; k < h; ++k) {
        const float wr = twr[k * step];
        const float wi = inverse ? -twi[k * step] : twi[k * step];
        const int ia = g + k, ib = g + k + h;
        const float br = re[ib], bi = im[ib];
        const float p1 = wr * br, p2 = wi * bi, p3 = wr * bi, p4 = wi * br;
        const float tr = p1 - p2, ti = p3 + p4;
        const float ar = re[ia], ai = im[ia];
        re[ia] = ar + tr;
        im[ia] = ai + ti;
        re[ib] = ar - tr;
        im[ib] = ai - ti;
      }
    }
  }
}

#define FFO_DCHUNK 8

/* Canonical lag correlation for one (b, h): fills csum[0..N) and corr[0..N).
 * q, k: pooled fp32 rows [N][D]. */
static void lag_correlation(const float *q, const float *k, int N, int D,
                            const ffts_mask_params *p, float *csum, float *corr) {
  const int M = 1 << ilog2(2 * (int64_t)N);
  const int bits = ilog2(M);
  const int F = M / 2 + 1;
  float *twr = malloc(sizeof(float) * M / 2), *twi = malloc(sizeof(float) * M / 2);
  float *re = malloc(sizeof(float) * M), *im = malloc(sizeof(float) * M);
  float *accr = calloc(F, sizeof(float)), *acci = calloc(F, sizeof(float));
  float *pr = malloc(sizeof(float) * F), *pi = malloc(sizeof(float) * F);
  make_twiddles(M, twr, twi);
  const int nchunk = (D + FFO_DCHUNK - 1) / FFO_DCHUNK;
  for (int c = 0; c < nchunk; ++c) {
    for (int f = 0; f < F; ++f) pr[f] = pi[f] = 0.0f;
    for (int d = c * FFO_DCHUNK; d < D && d < (c + 1) * FFO_DCHUNK; ++d) {
      for (int t = 0; t < M; ++t) {
        const uint32_t r = bitrev((uint32_t)t, bits);
        re[r] = t < N ? q[(int64_t)t * D + d] : 0.0f;
        im[r] = t < N ? k[(int64_t)t * D + d] : 0.0f;
      }
      fft_dit(re, im, M, twr, twi, 0);
      for (int f = 0; f < F; ++f) {
        const int g = (M - f) & (M - 1);
        const float ar = re[f], ai = im[f], br = re[g], bi = im[g];
        const float qr = 0.5f * (ar + br), qi = 0.5f * (ai - bi);
        const float kr = 0.5f * (ai + bi), ki = 0.5f * (br - ar);
        const float cr = qr * kr + qi * ki;
        const float ci = qi * kr - qr * ki;
        pr[f] = pr[f] + cr;
        pi[f] = pi[f] + ci;
      }
    }
    for (int f = 0; f < F; ++f) {
      accr[f] = accr[f] + pr[f];
      acci[f] = acci[f] + pi[f];
    }
  }
  /* inverse: Hermitian extension, bit-reversed placement, conj twiddles */
  for (int f = 0; f < M; ++f) {
    const uint32_t r = bitrev((uint32_t)f, bits);
    if (f < F) {
      re[r] = accr[f];
      im[r] = acci[f];
    } else {
      re[r] = accr[M - f];
      im[r] = -acci[M - f];
    }
  }
  fft_dit(re, im, M, twr, twi, 1);
  const float invM = 1.0f / (float)M;
  for (int t = 0; t < N; ++t) csum[t] = re[t] * invM;

  /* post-processing, my_attn_v7.py:133-155 */
  for (int t = 0; t < N; ++t) corr[t] = csum[t] / (float)(N - t);
  const int ex = p->exclude_tau;
  const int sraw = p->sink_tau_raw;
  const int s0 = sraw >= 0 ? sraw : (N + sraw > 0 ? N + sraw : 0);
  for (int t = 0; t < ex && t < N; ++t) corr[t] = 0.0f;
  for (int t = s0; t < N; ++t) corr[t] = 0.0f;
  if (ex < sraw) {
    float mn = corr[ex];
    for (int t = ex + 1; t < sraw; ++t)
      if (corr[t] < mn) mn = corr[t];
    for (int t = ex; t < sraw; ++t) corr[t] = corr[t] - mn;
    const float lden0 = (float)log10((double)(N - ex));
    const float lden = lden0 > 1e-6f ? lden0 : 1e-6f;
    for (int t = ex; t < sraw; ++t) {
      const float w = (float)log10((double)(N - t)) / lden;
      corr[t] = corr[t] * w;
    }
  }
  free(twr); free(twi); free(re); free(im); free(accr); free(acci); free(pr); free(pi);
}

/* ------------------------------------------------------------- selection */

typedef struct { uint32_t key; int idx; } keyed;

static int cmp_desc(const void *a, const void *b) {
  const keyed *x = a, *y = b;
  if (x->key != y->key) return x->key > y->key ? -1 : 1;
  return x->idx < y->idx ? -1 : (x->idx > y->idx);
}

/* Select the k largest of vals[lo..hi) (ties: lowest index) into sel[]. */
static void topk_select(const float *vals, int lo, int hi, int k, uint8_t *sel) {
  const int n = hi - lo;
  if (n <= 0 || k <= 0) return;
  keyed *a = malloc(sizeof(keyed) * n);
  for (int i = 0; i < n; ++i) {
    a[i].key = f32_key(vals[lo + i]);
    a[i].idx = lo + i;
  }
  qsort(a, n, sizeof(keyed), cmp_desc);
  for (int i = 0; i < k && i < n; ++i) sel[a[i].idx] = 1;
  free(a);
}

static int cmp_f32_asc(const void *a, const void *b) {
  const float x = *(const float *)a, y = *(const float *)b;
  return x < y ? -1 : (x > y);
}

/* torch.quantile(v, q) with linear interpolation (fp32 ranks, FMA lerp). */
static float quantile_f32(const float *vals, int n, float q) {
  float *s = malloc(sizeof(float) * n);
  memcpy(s, vals, sizeof(float) * n);
  qsort(s, n, sizeof(float), cmp_f32_asc);
  const float ranks = q * (float)(n - 1);
  const int lo = (int)ranks;
  const int hi = (int)ceilf(ranks);
  const float w = ranks - (float)lo;
  const float a = s[lo], b = s[hi];
  float r;
  if (fabsf(w) < 0.5f)
    r = fmaf(w, b - a, a);
  else
    r = fmaf(-(b - a), 1.0f - w, b);
  free(s);
  return r;
}

/* Canonical fp64 dot of two pooled rows (exact products, sums in d order). */
static inline double dot64(const float *a, const float *b, int D) {
  double acc = 0.0;
  for (int d = 0; d < D; ++d) acc = fma((double)a[d], (double)b[d], acc);
  return acc;
}

static inline float block_score(const float *a, const float *b, int D, double sqrtD) {
  return (float)(dot64(a, b, D) / sqrtD);
}

/* Fixed 256-lane reduction: lane l sums x[l], x[l+256], ... from +0 in order;
 * lanes are then combined by part[l] += part[l+s], s = 128 .. 1. */
#define FFO_LANES 256
static double lane_reduce(const double *x, int n) {
  double part[FFO_LANES];
  for (int l = 0; l < FFO_LANES; ++l) {
    double acc = 0.0;
    for (int e = l; e < n; e += FFO_LANES) acc = acc + x[e];
    part[l] = acc;
  }
  for (int s = FFO_LANES / 2; s >= 1; s /= 2)
    for (int l = 0; l < s; ++l) part[l] = part[l] + part[l + s];
  return part[0];
}

/* Stripe statistic of one head, my_attn_v7.py:301-383. */
static float stripe_variance(const float *q, const float *k, int N, int D,
                             const ffts_mask_params *p) {
  if (p->stripe_all_diffuse) return INFINITY;
  const double sqrtD = sqrt((double)D);
  double total = 0.0;
  float *diag = malloc(sizeof(float) * (N + 1));
  double *tmp = malloc(sizeof(double) * (N + 1));
  for (int s = 0; s < p->n_diag_samples; ++s) {
    const int tau = p->diag_taus[s];
    const int m = N - tau - 1;       /* diagonal minus its last element */
    const int n = m - 1;             /* number of adjacent differences  */
    for (int t = 0; t < m; ++t)
      diag[t] = block_score(q + (int64_t)(t + tau) * D, k + (int64_t)t * D, D, sqrtD);
    double var;
    if (n >= 2) {
      for (int t = 0; t < n; ++t) tmp[t] = (double)(diag[t + 1] - diag[t]);
      const double mean = lane_reduce(tmp, n) / (double)n;
      for (int t = 0; t < n; ++t) {
        const double e = (double)(diag[t + 1] - diag[t]) - mean;
        tmp[t] = e * e;
      }
      var = lane_reduce(tmp, n) / (double)(n - 1);
    } else {
      var = NAN;
    }
    for (int t = 0; t < m; ++t) tmp[t] = fabs((double)diag[t]);
    double mabs = m > 0 ? lane_reduce(tmp, m) / (double)m : NAN;
    const double floor6 = (double)1e-6f;
    if (mabs < floor6) mabs = floor6;
    total = total + var / mabs;
  }
  free(diag);
  free(tmp);
  return (float)(total / (double)p->n_diag_samples);
}

/* Column scores, my_attn_v7.py:403-420: suffix sums of q over rows j..N-2
 * (fp64, accumulated from row N-2 downwards), dot with k[j] by fma in d
 * order, / sqrt(D), / max(1, N-j-1), rounded to fp32. */
static void column_scores(const float *q, const float *k, int N, int D, float *out) {
  double *P = calloc((size_t)D, sizeof(double));
  const double sqrtD = sqrt((double)D);
  for (int j = N - 1; j >= 0; --j) {
    if (j <= N - 2)
      for (int d = 0; d < D; ++d) P[d] = P[d] + (double)q[(int64_t)j * D + d];
    double acc = 0.0;
    for (int d = 0; d < D; ++d) acc = fma(P[d], (double)k[(int64_t)j * D + d], acc);
    const int cnt = N - j - 1 > 1 ? N - j - 1 : 1;
    out[j] = (float)((acc / sqrtD) / (double)cnt);
  }
  free(P);
}

/* ------------------------------------------------------------- top level */

int ffo_block_mask(const float *qb, const float *kb, int dtype, int64_t B, int64_t H,
                   int64_t Hkv, int64_t D, const ffts_mask_params *p, uint32_t *bits,
                   int32_t *row_count, float *corr_out, float *csum_out,
                   uint8_t *stripe_out, float *svar_out) {
  const int N = p->n_blocks;
  const int W = (N + 31) / 32;
  if (H % Hkv) return -1;
  const int64_t rep = H / Hkv;
  const double sqrtD = sqrt((double)D);
#pragma omp parallel for schedule(dynamic)
  for (int64_t bh = 0; bh < B * H; ++bh) {
    const int64_t b = bh / H, h = bh % H;
    const float *q = qb + bh * (int64_t)N * D;
    const float *k = kb + (b * Hkv + h / rep) * (int64_t)N * D;
    float *csum = malloc(sizeof(float) * N), *corr = malloc(sizeof(float) * N);
    uint8_t *tausel = calloc(N, 1), *colsel = calloc(N, 1), *lastsel = calloc(N, 1);
    uint8_t *rowsel = calloc(N, 1);
    float *tmp = malloc(sizeof(float) * N);
    int stripe = 0;
    float svar = INFINITY;

    if (p->corr_on) {
      lag_correlation(q, k, N, (int)D, p, csum, corr);
      const int rs = p->remote_start, nr = N - rs;
      if (nr > 0) {
        if (p->corr_mode == FFTS_SEL_TOPK) {
          const float thr = quantile_f32(corr + rs, nr, p->corr_quantile);
          for (int t = rs; t < N; ++t) tausel[t] = corr[t] >= thr;
        } else {
          float mx = corr[rs];
          for (int t = rs + 1; t < N; ++t)
            if (corr[t] > mx) mx = corr[t];
          if (mx < 1e-6f) mx = 1e-6f;
          for (int t = rs; t < N; ++t) tausel[t] = (corr[t] / mx) >= p->corr_threshold;
        }
      }
      svar = stripe_variance(q, k, N, (int)D, p);
      stripe = svar <= p->stripe_threshold;
    } else {
      for (int t = 0; t < N; ++t) csum[t] = corr[t] = 0.0f;
    }
    const int col_apply = p->col_on && (!p->corr_on || stripe);
    if (col_apply && p->col_end > p->col_start) {
      column_scores(q, k, N, (int)D, tmp);
      topk_select(tmp, p->col_start, p->col_end, p->col_topk, colsel);
    }
    if (p->last_on) {
      for (int j = 0; j < N; ++j) {
        const float s = (float)dot64(q + (int64_t)(N - 1) * D, k + (int64_t)j * D, (int)D);
        tmp[j] = round_to_dtype(s, dtype);
      }
      topk_select(tmp, 0, N, p->last_topk, lastsel);
    }

    for (int i = 0; i < N; ++i) {
      memset(rowsel, 0, N);
      if (p->corr_on && !stripe) {
        for (int j = 0; j <= i; ++j)
          tmp[j] = block_score(q + (int64_t)i * D, k + (int64_t)j * D, (int)D, sqrtD);
        const float kr = (float)(i + 1) * p->qk_topk_ratio;
        int ki = (int)kr;
        if (ki < 1) ki = 1;
        topk_select(tmp, 0, i + 1, ki, rowsel);
      }
      int cnt = 0;
      uint32_t *row = bits + (bh * N + i) * (int64_t)W;
      for (int w = 0; w < W; ++w) row[w] = 0;
      for (int j = 0; j <= i; ++j) {
        const int tau = i - j;
        int on = j < p->keep_sink || j >= N - p->keep_recent || tau <= p->local_window;
        if (p->corr_on) {
          if (stripe)
            on |= tau >= p->remote_start && tausel[tau] && j >= p->keep_sink;
          else
            on |= rowsel[j];
        }
        on |= col_apply && colsel[j];
        on |= p->last_on && i == N - 1 && lastsel[j];
        if (on) {
          row[j >> 5] |= 1u << (j & 31);
          ++cnt;
        }
      }
      if (row_count) row_count[bh * N + i] = cnt;
    }
    if (corr_out) memcpy(corr_out + bh * N, corr, sizeof(float) * N);
    if (csum_out) memcpy(csum_out + bh * N, csum, sizeof(float) * N);
    if (stripe_out) stripe_out[bh] = (uint8_t)stripe;
    if (svar_out) svar_out[bh] = svar;
    free(csum); free(corr); free(tausel); free(colsel); free(lastsel); free(rowsel); free(tmp);
  }
  return 0;
}
