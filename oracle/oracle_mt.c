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
