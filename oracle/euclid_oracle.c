/*
 * CPU oracle for the euclid-cuda distance path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's arithmetic, used by tests/ (parity),
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg.  The product never links
 * or calls this file.  Every routine accumulates in the order the reference does
 * (sequential over the feature dimension, with the fused multiply-adds nvcc emits
 * for `acc += a * b`), so that the values it produces can be compared with the
 * reference's and the engine's bit for bit wherever the reference itself is
 * deterministic.
 *
 * Rounding helpers emulate IEEE round-to-nearest-even stores to fp16 / bf16 and the
 * round-to-nearest-away conversion to tf32, including subnormals and overflow to inf.
 *
 * Build: see oracle/Makefile (gcc -O2 -fopenmp -shared -fPIC, no -ffast-math).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* -------------------------------------------------------------- rounding */
/* x rounded to a binary format with p significand bits and exponent range
 * [emin, emax]; ties to even (away = 0) or away from zero (away = 1). */
static double round_fmt(double x, int p, int emin, int emax, int away) {
  if (x == 0.0 || !isfinite(x)) return x;
  int e;
  frexp(x, &e);
  int E = e - 1;
  if (E < emin) E = emin;
  const double q = ldexp(1.0, E - p + 1);
  const double t = x / q;
  const double r = (away ? round(t) : nearbyint(t)) * q;
  const double maxv = ldexp(2.0 - ldexp(1.0, -(p - 1)), emax);
  if (fabs(r) > maxv) return copysign(INFINITY, x);
  return r;
}
static inline double r_f16(double x) { return round_fmt(x, 11, -14, 15, 0); }
static inline double r_bf16(double x) { return round_fmt(x, 8, -126, 127, 0); }
static inline double r_tf32(double x) { return round_fmt(x, 11, -126, 127, 1); }

/* mode: 1 fp16 (RNE), 2 bf16 (RNE), 3 tf32 (RNA) */
void orc_round(const float* x, float* y, int64_t n, int mode) {
  for (int64_t i = 0; i < n; ++i) {
    const double v = x[i];
    y[i] = (float)(mode == 1 ? r_f16(v) : mode == 2 ? r_bf16(v) : r_tf32(v));
  }
}

/* ------------------------------------------------------------------ norms
 * mode 0: fmaf over fp16-rounded values, result stored fp16 (euclidean_kernels_mix.cu:106-119)
 * mode 1: same with bf16 (euclidean_kernels_mix.cu:122-135)
 * mode 2: fmaf over fp32 values (euclidean_kernels.cu:16-26)
 * mode 3: sum of fp32-rounded squares, sequential ((P*P).sum(1), euclidean_kernels_tiled.cu:338) */
void orc_norms_f32(const float* X, int64_t n, int64_t d, int mode, float* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const float* r = X + i * d;
    float s = 0.f;
    for (int64_t k = 0; k < d; ++k) {
      float v = r[k];
      if (mode == 0) v = (float)r_f16(v);
      if (mode == 1) v = (float)r_bf16(v);
      if (mode == 3)
        s = s + v * v;
      else
        s = fmaf(v, v, s);
    }
    if (mode == 0) s = (float)r_f16(s);
    if (mode == 1) s = (float)r_bf16(s);
    out[i] = s;
  }
}
/* fp64: s += v*v contracted to fma (euclidean_kernels.cu:28-38) */
void orc_norms_f64(const double* X, int64_t n, int64_t d, double* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    double s = 0.0;
    for (int64_t k = 0; k < d; ++k) s = fma(X[i * d + k], X[i * d + k], s);
    out[i] = s;
  }
}

/* ------------------------------------------------------------------- GEMMs
 * S[i, j] = sum_k A[i, k] * B[j, k], sequential fma in k.  Operands are passed
 * already rounded to the GEMM's input precision. */
void orc_gemm_f32(const float* A, const float* B, int64_t n, int64_t m, int64_t d, float* S) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i)
    for (int64_t j = 0; j < m; ++j) {
      float s = 0.f;
      for (int64_t k = 0; k < d; ++k) s = fmaf(A[i * d + k], B[j * d + k], s);
      S[i * m + j] = s;
    }
}
void orc_gemm_f64(const double* A, const double* B, int64_t n, int64_t m, int64_t d, double* S) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i)
    for (int64_t j = 0; j < m; ++j) {
      double s = 0.0;
      for (int64_t k = 0; k < d; ++k) s = fma(A[i * d + k], B[j * d + k], s);
      S[i * m + j] = s;
    }
}

/* ----------------------------------------------------------------- direct
 * in_type: 0 fp32, 1 fp16 bits, 2 bf16 bits, 3 fp64
 * rec:     1 fp64 fma   (direct_on_list_rowmajor, euclidean_kernels_mix.cu:156-177;
 *                        direct_on_list_fp16/_bf16/_fp64, euclidean_kernels_advanced.cu:148-220)
 *          2 fp32 fma   (direct_fp32_on_list, euclidean_kernels_mix.cu:481-504)
 *          3 fp16 arith, every operation rounded (direct_fp16_on_list, euclidean_kernels_mix.cu:412-439)
 *          4 bf16 arith, every operation rounded (direct_bf16_on_list, euclidean_kernels_mix.cu:442-469)
 *          5, 6: as 3, 4 with the square and the sum rounded once -- the sequence the
 *             reference's __hadd(acc, __hmul(diff, diff)) executes when built for sm_100 */
static inline double h2d(uint16_t h) {
  const int s = h >> 15, e = (h >> 10) & 31, f = h & 1023;
  double v;
  if (e == 0)
    v = ldexp((double)f, -24);
  else if (e == 31)
    v = f ? NAN : INFINITY;
  else
    v = ldexp((double)(f | 1024), e - 25);
  return s ? -v : v;
}
static inline double bf2d(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return (double)f;
}
static inline double in_val(int in_type, const void* X, int64_t idx) {
  switch (in_type) {
    case 0: return (double)((const float*)X)[idx];
    case 1: return h2d(((const uint16_t*)X)[idx]);
    case 2: return bf2d(((const uint16_t*)X)[idx]);
    default: return ((const double*)X)[idx];
  }
}
static double direct_one(int rec, int in_type, const void* P, const void* C, int64_t i, int64_t j, int64_t d) {
  if (rec == 1) {
    double acc = 0.0;
    for (int64_t k = 0; k < d; ++k) {
      const double diff = in_val(in_type, P, i * d + k) - in_val(in_type, C, j * d + k);
      acc = fma(diff, diff, acc);
    }
    return acc;
  }
  if (rec == 2) {
    float acc = 0.f;
    for (int64_t k = 0; k < d; ++k) {
      const float diff = (float)in_val(in_type, P, i * d + k) - (float)in_val(in_type, C, j * d + k);
      acc = fmaf(diff, diff, acc);
    }
    return acc;
  }
  /* half / bfloat arithmetic: each operation exact in double, then one rounding.
   * rec 3/4: diff, square and sum each rounded; rec 5/6: the square and the sum
   * fused into one rounding (what a contracted __hadd(acc, __hmul(d, d)) computes). */
  double (*rr)(double) = (rec == 3 || rec == 5) ? r_f16 : r_bf16;
  const int fused = (rec == 5 || rec == 6);
  double acc = 0.0;
  for (int64_t k = 0; k < d; ++k) {
    const double p = rr(in_val(in_type, P, i * d + k));
    const double c = rr(in_val(in_type, C, j * d + k));
    const double diff = rr(p - c);
    if (fused)
      acc = rr(fma(diff, diff, acc));
    else
      acc = rr(acc + rr(diff * diff));
  }
  return acc;
}
void orc_direct_pairs(int rec, int in_type, const void* P, const void* C, int64_t d, const int64_t* ii,
                      const int64_t* jj, int64_t cnt, double* out) {
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < cnt; ++t) out[t] = direct_one(rec, in_type, P, C, ii[t], jj[t], d);
}

/* Uniform direct operators (euclidean_kernels_uniform.cu:262-505): fp32 accumulate
 * for fp16/bf16/fp32 inputs (acc += diff*diff -> fmaf), fp64 for fp64. */
void orc_direct_all(int in_type, const void* P, const void* C, int64_t n, int64_t m, int64_t d, double* out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i)
    for (int64_t j = 0; j < m; ++j) {
      if (in_type == 3) {
        double acc = 0.0;
        for (int64_t k = 0; k < d; ++k) {
          const double diff = in_val(3, P, i * d + k) - in_val(3, C, j * d + k);
          acc = fma(diff, diff, acc);
        }
        out[i * m + j] = acc;
      } else {
        float acc = 0.f;
        for (int64_t k = 0; k < d; ++k) {
          const float diff = (float)in_val(in_type, P, i * d + k) - (float)in_val(in_type, C, j * d + k);
          acc = fmaf(diff, diff, acc);
        }
        out[i * m + j] = acc;
      }
    }
}

/* ---------------------------------------------------------------- centers
 * compute_centers_fp32_kernel / _fp64_kernel (center_kernels.cu:37-95): for every
 * (cluster, dim) a sequential sum over n = 0..N-1 of the rows with that label, in
 * the working precision, divided by the count; empty clusters stay 0. */
void orc_centers_f32(const float* X, const int64_t* labels, int64_t n, int64_t d, int64_t k, float* centers,
                     int64_t* counts) {
  memset(centers, 0, sizeof(float) * (size_t)(k * d));
  memset(counts, 0, sizeof(int64_t) * (size_t)k);
  for (int64_t i = 0; i < n; ++i)
    if (labels[i] >= 0 && labels[i] < k) counts[labels[i]]++;
  float* sums = (float*)calloc((size_t)(k * d), sizeof(float));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t c = labels[i];
    if (c < 0 || c >= k) continue;
    for (int64_t j = 0; j < d; ++j) sums[c * d + j] += X[i * d + j];
  }
  for (int64_t c = 0; c < k; ++c)
    if (counts[c] > 0)
      for (int64_t j = 0; j < d; ++j) centers[c * d + j] = sums[c * d + j] / (float)counts[c];
  free(sums);
}
void orc_centers_f64(const double* X, const int64_t* labels, int64_t n, int64_t d, int64_t k, double* centers,
                     int64_t* counts) {
  memset(centers, 0, sizeof(double) * (size_t)(k * d));
  memset(counts, 0, sizeof(int64_t) * (size_t)k);
  for (int64_t i = 0; i < n; ++i)
    if (labels[i] >= 0 && labels[i] < k) counts[labels[i]]++;
  double* sums = (double*)calloc((size_t)(k * d), sizeof(double));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t c = labels[i];
    if (c < 0 || c >= k) continue;
    for (int64_t j = 0; j < d; ++j) sums[c * d + j] += X[i * d + j];
  }
  for (int64_t c = 0; c < k; ++c)
    if (counts[c] > 0)
      for (int64_t j = 0; j < d; ++j) centers[c * d + j] = sums[c * d + j] / (double)counts[c];
  free(sums);
}
/* Exact-as-possible center sums: long double (80-bit) accumulation, for checking
 * the engine's fp64-accumulated statistics. */
void orc_center_stats(const void* X, int x_is_f64, const int64_t* labels, int64_t n, int64_t d, int64_t k,
                      double* stats) {
  long double* acc = (long double*)calloc((size_t)(k * (d + 1)), sizeof(long double));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t c = labels[i];
    if (c < 0 || c >= k) continue;
    for (int64_t j = 0; j < d; ++j)
      acc[c * (d + 1) + j] += x_is_f64 ? ((const double*)X)[i * d + j] : (double)((const float*)X)[i * d + j];
    acc[c * (d + 1) + d] += 1.0L;
  }
  for (int64_t t = 0; t < k * (d + 1); ++t) stats[t] = (double)acc[t];
  free(acc);
}

/* ----------------------------------------------------------- CPU baseline
 * The distance + argmin in fp64 on the host cores: norms, S = P.C^T (fp64 FMA),
 * d = |p|^2 - 2 s + |c|^2, first minimum per row.  C is transposed once so the
 * inner loop runs over centers with unit stride (vectorises without reassociating
 * any sum).  Returns the number of threads used. */
int orc_dist_argmin_f64(const double* P, const double* C, int64_t n, int64_t m, int64_t d, int64_t* labels,
                        double* mind, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
  double* Ct = (double*)malloc(sizeof(double) * (size_t)(m * d));
  double* cc = (double*)malloc(sizeof(double) * (size_t)m);
  for (int64_t j = 0; j < m; ++j) {
    double s = 0.0;
    for (int64_t k = 0; k < d; ++k) {
      Ct[k * m + j] = C[j * d + k];
      s = fma(C[j * d + k], C[j * d + k], s);
    }
    cc[j] = s;
  }
  int used = 1;
#pragma omp parallel
  {
#ifdef _OPENMP
#pragma omp single
    used = omp_get_num_threads();
#endif
    double* acc = (double*)malloc(sizeof(double) * (size_t)m);
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      const double* p = P + i * d;
      double pp = 0.0;
      for (int64_t j = 0; j < m; ++j) acc[j] = 0.0;
      for (int64_t k = 0; k < d; ++k) {
        const double pk = p[k];
        pp = fma(pk, pk, pp);
        const double* ct = Ct + k * m;
        for (int64_t j = 0; j < m; ++j) acc[j] = fma(pk, ct[j], acc[j]);
      }
      double best = INFINITY;
      int64_t bj = 0;
      for (int64_t j = 0; j < m; ++j) {
        double dd = pp - 2.0 * acc[j] + cc[j];
        if (dd < 0.0) dd = 0.0;
        if (dd < best) {
          best = dd;
          bj = j;
        }
      }
      labels[i] = bj;
      mind[i] = best;
    }
    free(acc);
  }
  free(Ct);
  free(cc);
  return used;
}

/* ----------------------------------------------------------- CPU baseline
 * One Lloyd iteration in fp64 on the host cores: the distance + argmin above for every
 * row, each thread adding its rows into a private k x (d+1) table (sums, count), then
 * the tables added in thread order and the means formed (an empty cluster gets 0, as
 * update_centers_* gives it, center_kernels.cu:52,116).  ms[0] receives the time of
 * the per-row part, ms[1] that of the reduction and means, whose cost does not grow
 * with n.  Returns the number of threads used. */
int orc_lloyd_step_f64(const double* X, const double* C, int64_t n, int64_t k, int64_t d, int64_t* labels,
                       double* newC, int threads, double* ms) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
  const int nt = omp_get_max_threads();
  const double t0 = omp_get_wtime();
#else
  const int nt = 1;
#endif
  const int64_t w = d + 1;
  double* part = (double*)calloc((size_t)nt * (size_t)(k * w), sizeof(double));
  double* mind = (double*)malloc(sizeof(double) * (size_t)(n > 0 ? n : 1));
  const int used = orc_dist_argmin_f64(X, C, n, k, d, labels, mind, nt);
#pragma omp parallel num_threads(nt)
  {
#ifdef _OPENMP
    double* t = part + (size_t)omp_get_thread_num() * (size_t)(k * w);
#else
    double* t = part;
#endif
#pragma omp for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
      double* row = t + labels[i] * w;
      for (int64_t j = 0; j < d; ++j) row[j] += X[i * d + j];
      row[d] += 1.0;
    }
  }
#ifdef _OPENMP
  const double t1 = omp_get_wtime();
#endif
  for (int64_t c = 0; c < k; ++c) {
    for (int64_t j = 0; j < w; ++j) {
      double s = 0.0;
      for (int q = 0; q < nt; ++q) s += part[(size_t)q * (size_t)(k * w) + c * w + j];
      part[c * w + j] = s;
    }
    const double cnt = part[c * w + d];
    for (int64_t j = 0; j < d; ++j) newC[c * d + j] = cnt > 0.0 ? part[c * w + j] / cnt : 0.0;
  }
#ifdef _OPENMP
  const double t2 = omp_get_wtime();
  ms[0] = (t1 - t0) * 1e3;
  ms[1] = (t2 - t1) * 1e3;
#else
  ms[0] = ms[1] = 0.0;
#endif
  free(part);
  free(mind);
  return used;
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
