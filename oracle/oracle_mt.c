/*
 * oracle_mt.c — the strided-views workload (256x512x32768 float32 in the
 * full configuration) restated on the CPU, for the timed CPU baseline.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by bench.py's CPU-baseline leg and by the
 * tests, never by the product.
 *
 * The step is the R program
 *     y <- contiguous(permute_view(x, c(3,1,2)))
 *     z <- y*0.5 + exp(-y^2)
 *     s <- sum(z); v <- var(z)
 *     a <- argmax(z, axis = 1)
 * computed as base R would (double arithmetic, long double sums), with y and
 * z stored in the tensor dtype (float32).  `threads` > 1 splits every loop
 * statically over POSIX threads; partial sums are combined in thread order.
 */
#include <pthread.h>

#include "oracle.c"

typedef struct {
  const float *x;
  float *y, *z;
  int32_t *idx;
  int64_t n0, n1, n2, lo, hi; /* work range of this thread (phase-specific units) */
  long double s, t, q, m;
  int phase;
} job_t;

static void *run_job(void *p) {
  job_t *j = (job_t *)p;
  const int64_t n0 = j->n0, n1 = j->n1, n2 = j->n2;
  switch (j->phase) {
    case 0: /* permute: y[c + n2*(a + n0*b)] = x[a + n0*(b + n1*c)], units = (a,b) pairs */
      for (int64_t ab = j->lo; ab < j->hi; ++ab) {
        const int64_t a = ab % n0, b = ab / n0;
        float *yo = j->y + n2 * ab;
        const float *xi = j->x + a + n0 * b;
        for (int64_t c = 0; c < n2; ++c) yo[c] = xi[n0 * n1 * c];
      }
      break;
    case 1: /* elementwise chain + sum */
      for (int64_t i = j->lo; i < j->hi; ++i) {
        const float v = j->y[i];
        const float a = v * 0.5f;
        const float sq = v * v;
        const float e = (float)exp((double)-sq);
        const float r = a + e;
        j->z[i] = r;
        j->s += r;
      }
      break;
    case 2: /* correction term of R's mean */
      for (int64_t i = j->lo; i < j->hi; ++i) j->t += j->z[i] - j->m;
      break;
    case 3: /* sum of squared deviations */
      for (int64_t i = j->lo; i < j->hi; ++i) {
        const long double d = j->z[i] - j->m;
        j->q += d * d;
      }
      break;
    case 4: /* argmax along the first axis, units = fibers */
      for (int64_t f = j->lo; f < j->hi; ++f) {
        const float *zf = j->z + n2 * f;
        int64_t best = 0;
        float bv = zf[0];
        for (int64_t c = 1; c < n2; ++c)
          if (zf[c] > bv) {
            bv = zf[c];
            best = c;
          }
        j->idx[f] = (int32_t)(best + 1);
      }
      break;
  }
  return NULL;
}

static void run_phase(job_t *jobs, int threads, int phase, int64_t units, long double m) {
  pthread_t th[256];
  for (int k = 0; k < threads; ++k) {
    jobs[k].phase = phase;
    jobs[k].lo = units * k / threads;
    jobs[k].hi = units * (k + 1) / threads;
    jobs[k].m = m;
  }
  if (threads == 1) {
    run_job(&jobs[0]);
    return;
  }
  for (int k = 0; k < threads; ++k) pthread_create(&th[k], NULL, run_job, &jobs[k]);
  for (int k = 0; k < threads; ++k) pthread_join(th[k], NULL);
}

/* x: n0 x n1 x n2 column-major.  y, z: n2 x n0 x n1 column-major.
 * idx: n0 x n1, 1-based argmax of z along its first axis. */
void orc_pipeline_views(const float *x, int64_t n0, int64_t n1, int64_t n2, float *y, float *z, double *sum,
                        double *var, int32_t *idx, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  job_t jobs[256];
  memset(jobs, 0, sizeof(jobs));
  for (int k = 0; k < threads; ++k) {
    jobs[k].x = x;
    jobs[k].y = y;
    jobs[k].z = z;
    jobs[k].idx = idx;
    jobs[k].n0 = n0;
    jobs[k].n1 = n1;
    jobs[k].n2 = n2;
  }
  const int64_t n = n0 * n1 * n2;
  run_phase(jobs, threads, 0, n0 * n1, 0.0L);
  run_phase(jobs, threads, 1, n, 0.0L);
  long double s = 0.0L;
  for (int k = 0; k < threads; ++k) s += jobs[k].s;
  long double m = s / n;
  run_phase(jobs, threads, 2, n, m);
  long double t = 0.0L;
  for (int k = 0; k < threads; ++k) t += jobs[k].t;
  m += t / n;
  run_phase(jobs, threads, 3, n, m);
  long double q = 0.0L;
  for (int k = 0; k < threads; ++k) q += jobs[k].q;
  run_phase(jobs, threads, 4, n0 * n1, 0.0L);
  *sum = (double)s;
  *var = (double)(q / (n - 1));
}

/* ---- config-size checks: the oracle's per-output loops split over threads ----
 * Each output (or fiber) is computed by exactly the single-threaded code
 * above, so these return the same values as orc_reduce / orc_arg_reduce /
 * orc_scan / orc_softmax; only the outputs are divided among threads. */
typedef struct {
  int kind, op, dt, nd, axis, one_based;
  const void *in;
  const int64_t *shape, *st;
  uint32_t mask;
  void *out;
  int64_t lo, hi;
  int rc;
} range_job_t;

enum { J_REDUCE = 0, J_ARG = 1, J_SCAN = 2, J_SOFTMAX = 3 };

static void *run_range(void *p) {
  range_job_t *j = (range_job_t *)p;
  switch (j->kind) {
    case J_REDUCE:
      j->rc = orc_reduce_range(j->op, j->dt, j->in, j->nd, j->shape, j->st, j->mask, (double *)j->out, j->lo, j->hi);
      break;
    case J_ARG:
      j->rc = orc_arg_reduce_range(j->op, j->dt, j->in, j->nd, j->shape, j->st, j->axis, j->one_based,
                                   (int64_t *)j->out, j->lo, j->hi);
      break;
    case J_SCAN:
      j->rc = orc_scan_fibers(j->op, j->dt, j->in, j->nd, j->shape, j->st, j->axis, j->out, j->lo, j->hi);
      break;
    case J_SOFTMAX:
      j->rc = orc_softmax_fibers(j->dt, j->in, j->nd, j->shape, j->st, j->axis, j->out, j->lo, j->hi);
      break;
  }
  return NULL;
}

static int run_ranges(range_job_t proto, int64_t units, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (units < threads) threads = units > 0 ? (int)units : 1;
  range_job_t jobs[256];
  pthread_t th[256];
  for (int k = 0; k < threads; ++k) {
    jobs[k] = proto;
    jobs[k].lo = units * k / threads;
    jobs[k].hi = units * (k + 1) / threads;
    jobs[k].rc = 0;
  }
  for (int k = 1; k < threads; ++k) pthread_create(&th[k], NULL, run_range, &jobs[k]);
  run_range(&jobs[0]);
  int rc = jobs[0].rc;
  for (int k = 1; k < threads; ++k) {
    pthread_join(th[k], NULL);
    if (jobs[k].rc) rc = jobs[k].rc;
  }
  return rc;
}

static int64_t kept_outputs(int nd, const int64_t *shape, uint32_t mask) {
  int64_t o = 1;
  for (int d = 0; d < nd; ++d)
    if (!((mask >> d) & 1u)) o *= shape[d];
  return o;
}

int orc_reduce_mt(int op, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, uint32_t mask,
                  double *out, int threads) {
  range_job_t p = {J_REDUCE, op, dt, nd, 0, 0, in, shape, st, mask, out, 0, 0, 0};
  return run_ranges(p, kept_outputs(nd, shape, mask), threads);
}

int orc_arg_reduce_mt(int is_max, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis,
                      int one_based, int64_t *out, int threads) {
  const uint32_t mask = axis < 0 ? 0xFFu : (1u << axis);
  range_job_t p = {J_ARG, is_max, dt, nd, axis, one_based, in, shape, st, mask, out, 0, 0, 0};
  return run_ranges(p, kept_outputs(nd, shape, mask), threads);
}

/* axis >= 0 only (a flattened scan is one sequential fiber) */
int orc_scan_mt(int is_prod, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis,
                void *out, int threads) {
  if (axis < 0 || axis >= nd || shape[axis] == 0) return orc_scan(is_prod, dt, in, nd, shape, st, axis, out);
  range_job_t p = {J_SCAN, is_prod, dt, nd, axis, 0, in, shape, st, 0, out, 0, 0, 0};
  return run_ranges(p, numel(nd, shape) / shape[axis], threads);
}

int orc_softmax_mt(int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis, void *out,
                   int threads) {
  if (axis < 0 || axis >= nd || shape[axis] == 0) return orc_softmax(dt, in, nd, shape, st, axis, out);
  range_job_t p = {J_SOFTMAX, 0, dt, nd, axis, 0, in, shape, st, 0, out, 0, 0, 0};
  return run_ranges(p, numel(nd, shape) / shape[axis], threads);
}

/* ---- whole-tensor statistics of arrays too large for orc_reduce ----------
 * (orc_reduce gathers a fiber into long doubles first: 16 bytes per element).
 * The array may arrive in consecutive chunks; the accumulators carry over.
 *
 *   orc_moments_mt: acc[0] += sum(x - c), acc[1] += sum((x - c)^2), in long
 *     double, per-thread partials added in thread order.  With c = 0 the
 *     first is base R's long double sum (up to the order in which the
 *     per-thread partials meet); a second pass with c = sum/n gives R's mean
 *     correction t = sum(x - m) and the two-pass variance
 *     (sum((x - m)^2) - t^2/n) / (n - 1) around the corrected mean m + t/n.
 *   orc_extrema_mt: running max/min values and their first 0-based global
 *     index (base = index of in[0]); NaN never wins; idx = -1 until some
 *     element is not NaN. */
typedef struct {
  int dt;
  const void *in;
  int64_t lo, hi;
  long double c, s, q;
  double mx, mn;
  int64_t imx, imn;
} stat_job_t;

static void *run_moments(void *p) {
  stat_job_t *j = (stat_job_t *)p;
  long double s = 0.0L, q = 0.0L;
  for (int64_t i = j->lo; i < j->hi; ++i) {
    const long double d = ld_get(j->in, j->dt, i) - j->c;
    s += d;
    q += d * d;
  }
  j->s = s;
  j->q = q;
  return NULL;
}

static void *run_extrema(void *p) {
  stat_job_t *j = (stat_job_t *)p;
  j->imx = j->imn = -1;
  for (int64_t i = j->lo; i < j->hi; ++i) {
    const long double x = ld_get(j->in, j->dt, i);
    if (isnan(x)) continue;
    if (j->imx < 0 || x > j->mx) {
      j->mx = (double)x;
      j->imx = i;
    }
    if (j->imn < 0 || x < j->mn) {
      j->mn = (double)x;
      j->imn = i;
    }
  }
  return NULL;
}

static int split_stat(stat_job_t *jobs, pthread_t *th, int dt, const void *in, int64_t n, int threads,
                      void *(*fn)(void *), long double c) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (n < threads) threads = n > 0 ? (int)n : 1;
  for (int k = 0; k < threads; ++k) {
    memset(&jobs[k], 0, sizeof(jobs[k]));
    jobs[k].dt = dt;
    jobs[k].in = in;
    jobs[k].c = c;
    jobs[k].lo = n * k / threads;
    jobs[k].hi = n * (k + 1) / threads;
  }
  for (int k = 1; k < threads; ++k) pthread_create(&th[k], NULL, fn, &jobs[k]);
  fn(&jobs[0]);
  for (int k = 1; k < threads; ++k) pthread_join(th[k], NULL);
  return threads;
}

void orc_moments_mt(int dt, const void *in, int64_t n, const long double *center, long double *acc, int threads) {
  stat_job_t jobs[256];
  pthread_t th[256];
  const int t = split_stat(jobs, th, dt, in, n, threads, run_moments, *center);
  for (int k = 0; k < t; ++k) {
    acc[0] += jobs[k].s;
    acc[1] += jobs[k].q;
  }
}

void orc_extrema_mt(int dt, const void *in, int64_t n, int64_t base, double *val, int64_t *idx, int threads) {
  stat_job_t jobs[256];
  pthread_t th[256];
  const int t = split_stat(jobs, th, dt, in, n, threads, run_extrema, 0.0L);
  for (int k = 0; k < t; ++k) { /* thread order = index order: strict comparisons keep the first */
    if (jobs[k].imx >= 0 && (idx[0] < 0 || jobs[k].mx > val[0])) {
      val[0] = jobs[k].mx;
      idx[0] = base + jobs[k].imx;
    }
    if (jobs[k].imn >= 0 && (idx[1] < 0 || jobs[k].mn < val[1])) {
      val[1] = jobs[k].mn;
      idx[1] = base + jobs[k].imn;
    }
  }
}

/* x*p + exp(-(x^2)) of a contiguous array, split over threads */
typedef struct {
  int dt;
  const void *in;
  void *out;
  int64_t lo, hi;
  double p;
} chain_job_t;

static void *run_chain(void *p) {
  chain_job_t *j = (chain_job_t *)p;
  const int64_t w = j->dt == DT_F32 ? 4 : 8;
  orc_gauss_chain(j->dt, (const char *)j->in + w * j->lo, j->hi - j->lo, j->p, (char *)j->out + w * j->lo);
  return NULL;
}

void orc_gauss_chain_mt(int dt, const void *in, int64_t n, double p, void *out, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  chain_job_t jobs[256];
  pthread_t th[256];
  for (int k = 0; k < threads; ++k) {
    jobs[k].dt = dt;
    jobs[k].in = in;
    jobs[k].out = out;
    jobs[k].p = p;
    jobs[k].lo = n * k / threads;
    jobs[k].hi = n * (k + 1) / threads;
  }
  for (int k = 1; k < threads; ++k) pthread_create(&th[k], NULL, run_chain, &jobs[k]);
  run_chain(&jobs[0]);
  for (int k = 1; k < threads; ++k) pthread_join(th[k], NULL);
}
