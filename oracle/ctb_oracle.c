/*
 * ctb_oracle.c — CPU restatement of the cuTile kernels TileTriton runs
 * on its hot path. TEST INFRASTRUCTURE ONLY: the parity tests, the smoke
 * check and bench.py's CPU-baseline leg load it as the checker / the timed
 * CPU stand-in; the product library never calls it.
 *
 * Each function follows the reference's CPU expression for that kernel:
 *   vadd      c = a .+ b                       test/runtests.jl:46, bench/bench.jl:82
 *   rowsum    sum(a; dims=2)                   test/runtests.jl:66, bench/rocm_compare.jl:84
 *   softmax   eh = exp.(x .- maximum(x; dims=1)); eh ./ sum(eh; dims=1)
 *                                              test/runtests.jl:129-131, bench/bench.jl:188-189
 *   layernorm mean, biased var, rstd = 1/sqrt(var+eps), (x-mean)*rstd*w+b
 *             (cuTile example layernorm.jl:27 — not vendored: parity unpinned)
 *   layernorm backward: dx = (g - (xhat*mean(g*xhat) + mean(g)))*rstd with
 *             g = w*dy; dw = sum dy*xhat; db = sum dy (example layernorm.jl
 *             lines 118/186 — not vendored: parity unpinned)
 * GEMM and attention are restated with numpy float64 in oracle/oracle.py.
 *
 * Checker variants accumulate in double. The *_f32 variants accumulate in
 * float like Julia's Base reductions and are the timed CPU baseline.
 * Arrays follow the library's layout: vectors of `len` contiguous floats
 * spaced `ld` apart.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

int oracle_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ---- seeded inputs: the same counter-based SplitMix64 stream as the
 * library's ctb_fill_uniform / ctb_fill_normal ------------------------------ */
static inline uint64_t splitmix64_at(uint64_t seed, uint64_t ctr) {
  uint64_t z = seed + (ctr + 1) * 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline double u24(uint64_t z) { return (double)(z >> 40) * (1.0 / 16777216.0); }

/* Uniform as doubles; the caller rounds to the element type (round to nearest). */
void oracle_uniform_f64(double* out, int64_t n, uint64_t seed, uint64_t offset, double lo,
                        double hi) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = lo + (hi - lo) * u24(splitmix64_at(seed, offset + i));
}
void oracle_uniform_f32(float* out, int64_t n, uint64_t seed, uint64_t offset, double lo,
                        double hi) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i)
    out[i] = (float)(lo + (hi - lo) * u24(splitmix64_at(seed, offset + i)));
}
void oracle_normal_f32(float* out, int64_t n, uint64_t seed, uint64_t offset, double mean,
                       double sd) {
  const double pi = 3.14159265358979323846;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t c = 2 * (uint64_t)(offset + i);
    const double u1 = 1.0 - u24(splitmix64_at(seed, c));
    const double u2 = u24(splitmix64_at(seed, c + 1));
    out[i] = (float)(mean + sd * (sqrt(-2.0 * log(u1)) * cos(2.0 * pi * u2)));
  }
}

/* ---- vadd ---------------------------------------------------------------- */
void oracle_vadd_f32(const float* a, const float* b, float* c, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) c[i] = a[i] + b[i];
}
void oracle_vadd_f64(const double* a, const double* b, double* c, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) c[i] = a[i] + b[i];
}

/* ---- rowsum: out[i] = sum_j a[i*si + j*sj] --------------------------------- */
void oracle_rowsum(const float* a, float* out, int64_t m, int64_t n, int64_t si, int64_t sj) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    double s = 0.0;
    for (int64_t j = 0; j < n; ++j) s += a[i * si + j * sj];
    out[i] = (float)s;
  }
}
/* Float accumulation, cache-friendly order for column-major a (si == 1). */
void oracle_rowsum_f32(const float* a, float* out, int64_t m, int64_t n, int64_t si, int64_t sj) {
  if (si == 1) {
#pragma omp parallel
    {
#ifdef _OPENMP
      const int nt = omp_get_num_threads(), t = omp_get_thread_num();
#else
      const int nt = 1, t = 0;
#endif
      const int64_t lo = m * t / nt, hi = m * (t + 1) / nt;
      for (int64_t i = lo; i < hi; ++i) out[i] = 0.f;
      for (int64_t j = 0; j < n; ++j) {
        const float* col = a + j * sj;
        for (int64_t i = lo; i < hi; ++i) out[i] += col[i];
      }
    }
    return;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    float s = 0.f;
    for (int64_t j = 0; j < n; ++j) s += a[i * si + j * sj];
    out[i] = s;
  }
}

/* ---- softmax over contiguous vectors -------------------------------------------- */
void oracle_softmax(const float* x, float* y, int64_t len, int64_t count, int64_t ldx,
                    int64_t ldy) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < count; ++r) {
    const float* xr = x + r * ldx;
    float* yr = y + r * ldy;
    double m = -INFINITY;
    for (int64_t i = 0; i < len; ++i) m = xr[i] > m ? xr[i] : m;
    double s = 0.0;
    for (int64_t i = 0; i < len; ++i) s += exp((double)xr[i] - m);
    for (int64_t i = 0; i < len; ++i) yr[i] = (float)(exp((double)xr[i] - m) / s);
  }
}
void oracle_softmax_f32(const float* x, float* y, int64_t len, int64_t count, int64_t ldx,
                        int64_t ldy) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < count; ++r) {
    const float* xr = x + r * ldx;
    float* yr = y + r * ldy;
    float m = -INFINITY;
    for (int64_t i = 0; i < len; ++i) m = xr[i] > m ? xr[i] : m;
    float s = 0.f;
    for (int64_t i = 0; i < len; ++i) {
      const float e = expf(xr[i] - m);
      yr[i] = e;
      s += e;
    }
    for (int64_t i = 0; i < len; ++i) yr[i] /= s;
  }
}

/* ---- layernorm forward ---------------------------------------------------------- */
void oracle_layernorm_fwd(const float* x, const float* w, const float* b, float* y, float* mean,
                          float* rstd, int64_t n, int64_t rows, int64_t ldx, int64_t ldy,
                          double eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * ldx;
    float* yr = y + r * ldy;
    double s = 0.0;
    for (int64_t i = 0; i < n; ++i) s += xr[i];
    const double mu = s / (double)n;
    double q = 0.0;
    for (int64_t i = 0; i < n; ++i) q += ((double)xr[i] - mu) * ((double)xr[i] - mu);
    const double rs = 1.0 / sqrt(q / (double)n + eps);
    for (int64_t i = 0; i < n; ++i) yr[i] = (float)(((double)xr[i] - mu) * rs * w[i] + b[i]);
    mean[r] = (float)mu;
    rstd[r] = (float)rs;
  }
}
void oracle_layernorm_fwd_f32(const float* x, const float* w, const float* b, float* y,
                              float* mean, float* rstd, int64_t n, int64_t rows, int64_t ldx,
                              int64_t ldy, double eps) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * ldx;
    float* yr = y + r * ldy;
    float s = 0.f;
    for (int64_t i = 0; i < n; ++i) s += xr[i];
    const float mu = s / (float)n;
    float q = 0.f;
    for (int64_t i = 0; i < n; ++i) q += (xr[i] - mu) * (xr[i] - mu);
    const float rs = 1.0f / sqrtf(q / (float)n + (float)eps);
    for (int64_t i = 0; i < n; ++i) yr[i] = (xr[i] - mu) * rs * w[i] + b[i];
    mean[r] = mu;
    rstd[r] = rs;
  }
}

/* ---- layernorm backward ------------------------------------------------------- */
void oracle_layernorm_bwd(const float* x, const float* dy, const float* w, const float* mean,
                          const float* rstd, float* dx, double* dw, double* db, int64_t n,
                          int64_t rows) {
  for (int64_t i = 0; i < n; ++i) dw[i] = db[i] = 0.0;
#pragma omp parallel
  {
    double* ldw = (double*)calloc((size_t)n, sizeof(double));
    double* ldb = (double*)calloc((size_t)n, sizeof(double));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const float* xr = x + r * n;
      const float* gr = dy + r * n;
      const double mu = mean[r], rs = rstd[r];
      double s1 = 0.0, s2 = 0.0;
      for (int64_t i = 0; i < n; ++i) {
        const double xh = ((double)xr[i] - mu) * rs, g = (double)w[i] * gr[i];
        s1 += g * xh;
        s2 += g;
        ldw[i] += (double)gr[i] * xh;
        ldb[i] += gr[i];
      }
      const double c1 = s1 / (double)n, c2 = s2 / (double)n;
      for (int64_t i = 0; i < n; ++i) {
        const double xh = ((double)xr[i] - mu) * rs, g = (double)w[i] * gr[i];
        dx[r * n + i] = (float)((g - (xh * c1 + c2)) * rs);
      }
    }
#pragma omp critical
    for (int64_t i = 0; i < n; ++i) {
      dw[i] += ldw[i];
      db[i] += ldb[i];
    }
    free(ldw);
    free(ldb);
  }
}
