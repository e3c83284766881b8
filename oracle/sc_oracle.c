/*
 * sc_oracle.c -- CPU restatement of the enable-signal stochastic-computing (SC)
 * matmul.  TEST INFRASTRUCTURE ONLY: this file is the checker for the CUDA
 * engine and the timed CPU baseline.  Nothing in the product path links it.
 *
 * Parity status: UNPINNED.  The reference's SC arithmetic lives in the
 * un-vendored `scmp_kernels` submodule (reference .gitmodules:4-7, directory
 * empty, commit unrecoverable), and the reference ships no golden vectors for
 * this path.  This file restates the semantics that the reference's call
 * sites, docstrings and README fix, and pins every free choice in writing:
 *
 *   quantisation  sc_integration/sc_linear.py:104-111 (bipolar per-row
 *                 symmetric, q_max = 2^(p-1)-1; unipolar asymmetric with a
 *                 zero point, q_max = 2^p-1), sc_linear.py:95-98 (1e-6 floor)
 *   granularity   sc_integration/sc_attention.py:39-81 (per_row / per_head /
 *                 per_tensor), group_a/group_b rows per scale group
 *   enable window README.md:522-528 ("|x_int| <= 2 (boundary <= 4) ... Sobol
 *                 prefix of length 0-4": window = 2|x_int| at L = 2^p)
 *   early stop    sc_integration/sc_precision_map.py:10-14 (L < 2^p uses the
 *                 2^p pool truncated to its first L entries)
 *   signs         cls/sc_attention_patch.py:301-302 ("unipolar + signs")
 *   count table   sc_integration/sc_linear.py:116-121 (cum_indicator is
 *                 O(D) and indexed by window x threshold)
 *
 * Spec (all arithmetic below is reproduced bit-for-bit by the CUDA engine):
 *   codes     bipolar:  c = 2|x_int|, sigma = sign(x_int)
 *             unipolar: c = x_int in [0, 2^p-1], sigma = +1
 *   window    k = (c_a * L) >> p                (enable-signal length, < L)
 *   stream    bit t of (n,d) = [R[d mod D_pool][t] < c_b],   t < L
 *   count     cnt(m,n,d) = #{ t < k : R[d'][t] < c_b }
 *   acc[m,n]  = sum_d sigma_a * sigma_b * cnt      (exact int32)
 *   rescale   F = 2^(2p) / (u*L), u = 4 bipolar, 1 unipolar
 *             bipolar  y = (float(acc) * s_a) * (s_b * F)
 *             unipolar t = float(acc)*F - float(z_a*rs_b + z_b*rs_a - K*z_a*z_b)
 *                      y = (t * s_a) * s_b
 *             y += bias[n]   (when given)
 *
 * Build: see oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).  Floating
 * point contraction must stay off so the float sequence matches the device.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define SCO_OK 0
#define SCO_EINVAL -1
#define SCO_ENOMEM -2

/* ------------------------------------------------------------------ pools */

/* Scrambled 1-D Sobol stream per dimension (Gray-code order).
 * m[d*p + (i-1)] is the odd direction-number seed m_i < 2^i of dimension d;
 * V_i = m_i << (p - i); x_t = XOR over set bits of gray(t) of V; then the
 * per-dimension digital shift is XORed in.  `antithetic` complements.
 * Follows the seed structure of cls/experiments/qwt_sc_overnight.py:193-200
 * (k_seed = [1, odd m_j < 2^(j+1)]) and the Python-`random` seeding noted at
 * det/sc_eval.py:222-225. */
int sco_pool_sobol(int D, int p, const uint32_t *m, const uint32_t *shift,
                   int antithetic, uint8_t *R) {
  if (D <= 0 || p < 1 || p > 8) return SCO_EINVAL;
  const int T = 1 << p;
  const uint32_t full = (uint32_t)T - 1u;
  for (int d = 0; d < D; ++d) {
    uint32_t V[8];
    for (int i = 1; i <= p; ++i) V[i - 1] = (m[(size_t)d * p + (i - 1)] << (p - i)) & full;
    for (int t = 0; t < T; ++t) {
      uint32_t g = (uint32_t)t ^ ((uint32_t)t >> 1);
      uint32_t x = 0;
      for (int i = 0; i < p; ++i)
        if (g & (1u << i)) x ^= V[i];
      x ^= shift[d] & full;
      if (antithetic) x ^= full;
      R[(size_t)d * T + t] = (uint8_t)x;
    }
  }
  return SCO_OK;
}

/* 16-bit Galois LFSR (x^16 + x^14 + x^13 + x^11 + 1, mask 0xB400) per
 * dimension; stream value t is the top p bits of the state after t+1 steps. */
int sco_pool_lfsr16(int D, int p, const uint16_t *state0, uint8_t *R) {
  if (D <= 0 || p < 1 || p > 8) return SCO_EINVAL;
  const int T = 1 << p;
  for (int d = 0; d < D; ++d) {
    uint32_t s = state0[d];
    if (s == 0) return SCO_EINVAL;
    for (int t = 0; t < T; ++t) {
      uint32_t lsb = s & 1u;
      s >>= 1;
      if (lsb) s ^= 0xB400u;
      R[(size_t)d * T + t] = (uint8_t)(s >> (16 - p));
    }
  }
  return SCO_OK;
}

/* ---------------------------------------------------------- quantisation */

/* Quantise rows [rows, K] whose scale group is row_group[r] (groups are
 * contiguous row ranges).  mode 0 = bipolar, 1 = unipolar.
 * Outputs per group: scale, zero (unipolar; 0 for bipolar).  Per element:
 * signed code sigma*c (int16).  Per row: rowsum = sum of magnitudes c. */
int sco_quantize(const float *x, int64_t rows, int64_t K, const int64_t *row_group,
                 int64_t ngroups, int mode, int p, float *gscale, int32_t *gzero,
                 int16_t *code, int64_t *rowsum) {
  if (rows < 0 || K <= 0 || p < 1 || p > 8 || ngroups <= 0) return SCO_EINVAL;
  if (mode == 0 && p < 2) return SCO_EINVAL;
  float *lo = (float *)malloc(sizeof(float) * (size_t)ngroups);
  float *hi = (float *)malloc(sizeof(float) * (size_t)ngroups);
  if (!lo || !hi) { free(lo); free(hi); return SCO_ENOMEM; }
  for (int64_t g = 0; g < ngroups; ++g) { lo[g] = INFINITY; hi[g] = -INFINITY; }
  for (int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * K;
    int64_t g = row_group[r];
    for (int64_t k = 0; k < K; ++k) {
      float v = xr[k];
      if (mode == 0) v = fabsf(v);
      if (v < lo[g]) lo[g] = v;
      if (v > hi[g]) hi[g] = v;
    }
  }
  const float qmax = (mode == 0) ? (float)((1 << (p - 1)) - 1) : (float)((1 << p) - 1);
  for (int64_t g = 0; g < ngroups; ++g) {
    if (mode == 0) {
      float amax = hi[g] > 1e-6f ? hi[g] : 1e-6f;
      gscale[g] = amax / qmax;
      gzero[g] = 0;
      lo[g] = qmax / amax; /* reuse lo[] as the quantisation multiplier */
    } else {
      float rng = hi[g] - lo[g];
      if (!(rng > 1e-6f)) rng = 1e-6f;
      float inv = qmax / rng;
      gscale[g] = rng / qmax;
      gzero[g] = (int32_t)rintf((-lo[g]) * inv);
      lo[g] = inv;
    }
  }
  const int32_t iq = (int32_t)qmax;
  for (int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * K;
    int64_t g = row_group[r];
    float inv = lo[g];
    int64_t rs = 0;
    for (int64_t k = 0; k < K; ++k) {
      int32_t q = (int32_t)rintf(xr[k] * inv);
      int16_t c;
      if (mode == 0) {
        if (q > iq) q = iq;
        if (q < -iq) q = -iq;
        c = (int16_t)(2 * q);
        rs += 2 * (q < 0 ? -q : q);
      } else {
        q += gzero[g];
        if (q > iq) q = iq;
        if (q < 0) q = 0;
        c = (int16_t)q;
        rs += q;
      }
      code[r * K + k] = c;
    }
    if (rowsum) rowsum[r] = rs;
  }
  free(lo);
  free(hi);
  return SCO_OK;
}

/* ---------------------------------------------------------------- counts */

/* acc[m,n] = sum_d sigma_a sigma_b #{t < k(m,d) : R[d'][t] < c_b(n,d)}.
 * ca [M,K], cb [N,K] signed codes; R [D_pool, 2^p]; d' = d mod D_pool.
 * L_row (nullable) gives a per-row stream length (rows with L <= 0 give 0);
 * otherwise every row uses L.  Bit-packed: per (n,d) the L-bit stream is
 * packed into 64-bit words with prefix popcounts, so each (m,n,d) costs one
 * masked popcount. */
int sco_sc_counts(const int16_t *ca, const int16_t *cb, int64_t M, int64_t N, int64_t K,
                  const uint8_t *R, int D_pool, int p, int L, const int32_t *L_row,
                  int32_t *acc, int nthreads) {
  if (M < 0 || N < 0 || K <= 0 || D_pool <= 0 || p < 1 || p > 8) return SCO_EINVAL;
  const int T = 1 << p;
  int Lmax = L;
  if (L_row) {
    Lmax = 0;
    for (int64_t m = 0; m < M; ++m) Lmax = L_row[m] > Lmax ? L_row[m] : Lmax;
  }
  if (Lmax > T) return SCO_EINVAL;
  if (M == 0 || N == 0) return SCO_OK;
  if (Lmax <= 0) { memset(acc, 0, sizeof(int32_t) * (size_t)(M * N)); return SCO_OK; }
  const int W = (Lmax + 63) / 64;
  /* streams [N, K, W] and prefix counts [N, K, W] */
  uint64_t *S = (uint64_t *)calloc((size_t)(N * K * W), sizeof(uint64_t));
  uint16_t *C = (uint16_t *)calloc((size_t)(N * K * W), sizeof(uint16_t));
  if (!S || !C) { free(S); free(C); return SCO_ENOMEM; }
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t d = 0; d < K; ++d) {
      int v = cb[n * K + d];
      if (v < 0) v = -v;
      const uint8_t *Rd = R + (size_t)(d % D_pool) * T;
      uint64_t *s = S + (n * K + d) * W;
      uint16_t *c = C + (n * K + d) * W;
      for (int t = 0; t < Lmax; ++t)
        if ((int)Rd[t] < v) s[t >> 6] |= 1ull << (t & 63);
      uint16_t run = 0;
      for (int w = 0; w < W; ++w) { c[w] = run; run = (uint16_t)(run + __builtin_popcountll(s[w])); }
    }
  }
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1)
#endif
  for (int64_t m = 0; m < M; ++m) {
    const int Lm = L_row ? L_row[m] : L;
    int32_t *out = acc + m * N;
    if (Lm <= 0) { memset(out, 0, sizeof(int32_t) * (size_t)N); continue; }
    /* windows for this row */
    int32_t *kk = (int32_t *)malloc(sizeof(int32_t) * (size_t)K);
    int8_t *sg = (int8_t *)malloc((size_t)K);
    for (int64_t d = 0; d < K; ++d) {
      int c = ca[m * K + d];
      sg[d] = (int8_t)(c < 0 ? -1 : 1);
      if (c < 0) c = -c;
      kk[d] = (c * Lm) >> p;
    }
    for (int64_t n = 0; n < N; ++n) {
      const uint64_t *s = S + n * K * W;
      const uint16_t *c = C + n * K * W;
      const int16_t *cbn = cb + n * K;
      int32_t a = 0;
      for (int64_t d = 0; d < K; ++d) {
        int k = kk[d];
        if (k == 0) continue;
        int w = k >> 6, r = k & 63;
        int cnt = c[d * W + w] + __builtin_popcountll(s[d * W + w] & ((1ull << r) - 1ull));
        a += (sg[d] * (cbn[d] < 0 ? -1 : 1)) * cnt;
      }
      out[n] = a;
    }
    free(kk);
    free(sg);
  }
  free(S);
  free(C);
  return SCO_OK;
}

/* --------------------------------------------------------------- rescale */

/* y[m,n] from acc.  sa/za are the group scale/zero of row m (already
 * expanded per row), sb/zb per column row n; rsa/rsb row sums of codes.
 * mode 0 bipolar, 1 unipolar; bias nullable.  L_row nullable (per-row L
 * and per-row p for the factor F; rows with L <= 0 give bias only). */
int sco_rescale(const int32_t *acc, int64_t M, int64_t N, int64_t K, int mode, int p, int L,
                const int32_t *L_row, const int32_t *p_row,
                const float *sa, const int32_t *za, const int64_t *rsa,
                const float *sb, const int32_t *zb, const int64_t *rsb,
                const float *bias, float *y) {
  for (int64_t m = 0; m < M; ++m) {
    int Lm = L_row ? L_row[m] : L;
    int pm = p_row ? p_row[m] : p;
    for (int64_t n = 0; n < N; ++n) {
      float v;
      if (Lm <= 0) {
        v = 0.0f;
      } else {
        float F = (float)(1u << (2 * pm)) / (float)((mode == 0 ? 4 : 1) * Lm);
        if (mode == 0) {
          float fb = sb[n] * F;
          v = ((float)acc[m * N + n] * sa[m]) * fb;
        } else {
          int64_t corr = (int64_t)za[m] * rsb[n] + (int64_t)zb[n] * rsa[m] -
                         K * (int64_t)za[m] * (int64_t)zb[n];
          float t = (float)acc[m * N + n] * F - (float)corr;
          v = (t * sa[m]) * sb[n];
        }
      }
      if (bias) v = v + bias[n];
      y[m * N + n] = v;
    }
  }
  return SCO_OK;
}

int sco_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
