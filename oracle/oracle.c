/*
 * oracle.c — CPU restatement of the acediaR hot path in base-R semantics.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker of the CUDA path: only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 * Nothing in the product (acedia-r_b200/) calls it.
 *
 * What it follows:
 *   - elementwise formulas of the reference functors
 *     (src/kernels/tensor_kernels.cuh:10-192): sigmoid = 1/(1+exp(-x)),
 *     relu = fmax(x, 0), round = rint, max/min = fmax/fmin, comparisons 1/0;
 *     each R operator rounds once in the tensor dtype: + - * / and sqrt are
 *     the native IEEE float/double operations, transcendental functions are
 *     evaluated in long double and rounded once; sigmoid() of a float32
 *     tensor is evaluated as base R does (in double precision or better)
 *     and rounded once;
 *   - reductions as base R computes them: sum in a long double accumulator,
 *     mean as sum/n followed by R's correction pass mean += sum(x-mean)/n,
 *     var two-pass with divisor n-1 (the reference also divides by n-1,
 *     src/kernels/tensor_ops.cu:802), max/min NaN-ignoring like fmax;
 *   - which.max / argmax: first index of the maximum (strict comparison,
 *     src/kernels/tensor_kernels.cu:794; src/kernels/tensor_ops.cu:861-863);
 *   - cumsum/cumprod: long double running accumulator, one rounding per
 *     output (R/gpuTensor.R:2234-2277 runs base R's cumsum);
 *   - softmax: exp(x - max) / sum(exp(x - max)) (src/kernels/tensor_ops.cu:826-846
 *     for the whole tensor; per axis for the row softmax);
 *   - strided copy: dest[idx] = src[sum coord*stride] in column-major order
 *     (src/kernels/tensor_kernels.cu:272-295);
 *   - axis reductions: output in column-major order of the kept axes
 *     (src/kernels/tensor_kernels.cu:488-560, src/TensorRegistry.h:1153-1179).
 * Layout: column-major (src/gpuTensor.h:359-370).  Every function takes int64
 * shapes and element strides; outputs are contiguous column-major.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MAXD 8

/* DT_F16 is IEEE binary16 (_Float16: gcc converts to and from it with one
 * rounding to nearest); DT_I8 is int8_t (no NA; arithmetic wraps modulo 256) */
enum { DT_F32 = 0, DT_F64 = 1, DT_I32 = 2, DT_I64 = 3, DT_BOOL = 4, DT_F16 = 5, DT_I8 = 6 };
enum {
  U_EXP = 0, U_LOG, U_SQRT, U_ABS, U_FLOOR, U_CEIL, U_ROUND, U_ERF, U_TANH, U_SIGMOID, U_RELU, U_SIN, U_COS,
  U_NEG, U_SQUARE, U_COPY
};
enum {
  B_ADD = 0, B_SUB, B_MUL, B_DIV, B_MAX, B_MIN, B_POW, B_GT, B_LT, B_EQ, B_NE, B_GE, B_LE, B_RSUB, B_RDIV
};
enum { R_SUM = 0, R_MEAN, R_MAX, R_MIN, R_PROD, R_VAR, R_COUNT, R_ANY, R_ALL };

static long double ld_get(const void *p, int dt, int64_t i) {
  switch (dt) {
    case DT_F32: return ((const float *)p)[i];
    case DT_F64: return ((const double *)p)[i];
    case DT_I32: return ((const int32_t *)p)[i];
    case DT_I64: return (long double)((const int64_t *)p)[i];
    case DT_BOOL: return ((const uint8_t *)p)[i];
    case DT_F16: return ((const _Float16 *)p)[i];
    case DT_I8: return ((const int8_t *)p)[i];
  }
  return 0.0L;
}

/* round to the tensor dtype */
static long double rnd(long double v, int dt) {
  switch (dt) {
    case DT_F32: return (float)v;
    case DT_F64: return (double)v;
    case DT_F16: return (_Float16)v;
    default: return v;
  }
}

static void put(void *p, int dt, int64_t i, long double v) {
  switch (dt) {
    case DT_F32: ((float *)p)[i] = (float)v; break;
    case DT_F64: ((double *)p)[i] = (double)v; break;
    case DT_I32: ((int32_t *)p)[i] = (int32_t)v; break;
    case DT_I64: ((int64_t *)p)[i] = (int64_t)v; break;
    case DT_BOOL: ((uint8_t *)p)[i] = (uint8_t)(v != 0.0L); break;
    case DT_F16: ((_Float16 *)p)[i] = (_Float16)v; break;
    case DT_I8: ((int8_t *)p)[i] = (int8_t)(int64_t)v; break; /* wraps modulo 256 */
  }
}

static int64_t numel(int nd, const int64_t *shape) {
  int64_t n = 1;
  for (int d = 0; d < nd; ++d) n *= shape[d];
  return n;
}

/* offset of the column-major linear index `idx` under `st` */
static int64_t offset_of(int64_t idx, int nd, const int64_t *shape, const int64_t *st) {
  int64_t off = 0;
  for (int d = 0; d < nd; ++d) {
    off += (idx % shape[d]) * st[d];
    idx /= shape[d];
  }
  return off;
}

/* correctly rounded arithmetic in the tensor dtype: float and double use the
 * native IEEE operation (computing in long double and rounding afterwards
 * could round twice) */
static long double add_dt(long double a, long double b, int dt) {
  if (dt == DT_F16) return (_Float16)(a + b); /* exact (or 64-bit) in long double, one rounding */
  if (dt == DT_F32) return (float)a + (float)b;
  if (dt == DT_F64) return (double)a + (double)b;
  return a + b;
}
static long double sub_dt(long double a, long double b, int dt) {
  if (dt == DT_F16) return (_Float16)(a - b); /* exact (or 64-bit) in long double, one rounding */
  if (dt == DT_F32) return (float)a - (float)b;
  if (dt == DT_F64) return (double)a - (double)b;
  return a - b;
}
static long double mul_dt(long double a, long double b, int dt) {
  if (dt == DT_F16) return (_Float16)(a * b); /* exact (or 64-bit) in long double, one rounding */
  if (dt == DT_F32) return (float)a * (float)b;
  if (dt == DT_F64) return (double)a * (double)b;
  return a * b;
}
static long double div_dt(long double a, long double b, int dt) {
  if (dt == DT_F16) return (_Float16)(a / b); /* exact (or 64-bit) in long double, one rounding */
  if (dt == DT_F32) return (float)a / (float)b;
  if (dt == DT_F64) return (double)a / (double)b;
  return a / b;
}
static long double sqrt_dt(long double x, int dt) {
  if (dt == DT_F16) return (_Float16)sqrtl(x);
  if (dt == DT_F32) return sqrtf((float)x);
  if (dt == DT_F64) return sqrt((double)x);
  return sqrtl(x);
}

static long double unary(int op, long double x, int dt) {
  switch (op) {
    case U_EXP: return rnd(expl(x), dt);
    case U_LOG: return rnd(logl(x), dt);
    case U_SQRT: return sqrt_dt(x, dt);
    case U_ABS: return fabsl(x);
    case U_FLOOR: return floorl(x);
    case U_CEIL: return ceill(x);
    case U_ROUND: return rintl(x); /* half to even, as rint */
    case U_ERF: return rnd(erfl(x), dt);
    case U_TANH: return rnd(tanhl(x), dt);
    case U_SIGMOID:
      if (dt == DT_F64) {
        /* base R on doubles: 1/(1+exp(-x)), one rounding per operator */
        const long double e = rnd(expl(-x), dt);
        return div_dt(1.0L, add_dt(1.0L, e, dt), dt);
      }
      /* float32 tensor: base R evaluates in double; one rounding to float */
      return rnd(1.0L / (1.0L + expl(-x)), dt);
    case U_RELU: return isnan(x) ? 0.0L : (x > 0.0L ? x : 0.0L); /* fmax(x, 0) */
    case U_SIN: return rnd(sinl(x), dt);
    case U_COS: return rnd(cosl(x), dt);
    case U_NEG: return -x;
    case U_SQUARE: return mul_dt(x, x, dt);
    default: return x;
  }
}

static long double fmaxl_r(long double a, long double b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return a > b ? a : b;
}
static long double fminl_r(long double a, long double b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return a < b ? a : b;
}

static long double binary(int op, long double a, long double b, int dt) {
  switch (op) {
    case B_ADD: return add_dt(a, b, dt);
    case B_SUB: return sub_dt(a, b, dt);
    case B_MUL: return mul_dt(a, b, dt);
    case B_DIV: return div_dt(a, b, dt);
    case B_MAX: return fmaxl_r(a, b);
    case B_MIN: return fminl_r(a, b);
    case B_POW: return (b == 2.0L) ? mul_dt(a, a, dt) : rnd(powl(a, b), dt);
    case B_GT: return a > b;
    case B_LT: return a < b;
    case B_EQ: return a == b;
    case B_NE: return a != b;
    case B_GE: return a >= b;
    case B_LE: return a <= b;
    case B_RSUB: return sub_dt(b, a, dt);
    case B_RDIV: return div_dt(b, a, dt);
  }
  return 0.0L;
}

/* ---- elementwise ------------------------------------------------------- */
/* The *_range forms compute output elements lo..hi-1 only (the config-size
 * checks split the outputs over threads); the plain forms compute all. */
void orc_unary_range(int op, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, void *out,
                     int64_t lo, int64_t hi) {
  for (int64_t i = lo; i < hi; ++i) put(out, dt, i, unary(op, ld_get(in, dt, offset_of(i, nd, shape, st)), dt));
}

void orc_unary(int op, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, void *out) {
  orc_unary_range(op, dt, in, nd, shape, st, out, 0, numel(nd, shape));
}

/* a and b carry strides already expanded to `shape` (stride 0 on broadcast
 * dims); out_dt is the input dtype or bool for comparisons */
void orc_binary_range(int op, int dt, const void *a, const int64_t *sa, const void *b, const int64_t *sb, int nd,
                      const int64_t *shape, int out_dt, void *out, int64_t lo, int64_t hi) {
  for (int64_t i = lo; i < hi; ++i) {
    const long double x = ld_get(a, dt, offset_of(i, nd, shape, sa));
    const long double y = ld_get(b, dt, offset_of(i, nd, shape, sb));
    put(out, out_dt, i, binary(op, x, y, dt));
  }
}

void orc_binary(int op, int dt, const void *a, const int64_t *sa, const void *b, const int64_t *sb, int nd,
                const int64_t *shape, int out_dt, void *out) {
  orc_binary_range(op, dt, a, sa, b, sb, nd, shape, out_dt, out, 0, numel(nd, shape));
}

/* x op s, with s first cast to the tensor dtype */
void orc_scalar_range(int op, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, double s,
                      int out_dt, void *out, int64_t lo, int64_t hi) {
  const long double sv = rnd((long double)s, dt);
  for (int64_t i = lo; i < hi; ++i)
    put(out, out_dt, i, binary(op, ld_get(in, dt, offset_of(i, nd, shape, st)), sv, dt));
}

void orc_scalar(int op, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, double s,
                int out_dt, void *out) {
  orc_scalar_range(op, dt, in, nd, shape, st, s, out_dt, out, 0, numel(nd, shape));
}

/* x*p + exp(-(x^2)), five roundings */
void orc_gauss_chain(int dt, const void *in, int64_t n, double p, void *out) {
  const long double pv = rnd(p, dt);
  for (int64_t i = 0; i < n; ++i) {
    const long double x = ld_get(in, dt, i);
    const long double a = mul_dt(x, pv, dt);
    const long double sq = mul_dt(x, x, dt);
    const long double e = rnd(expl(-sq), dt);
    put(out, dt, i, add_dt(a, e, dt));
  }
}

void orc_copy(int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, void *out) {
  orc_unary(U_COPY, dt, in, nd, shape, st, out);
}

/* ---- dtype conversion: base R's as.* rules -------------------------------
 * (the reference converts with a static_cast per element,
 * src/kernels/tensor_kernels.cu:52-57 and src/kernels/kernel_utils.cuh:11;
 * R's as.integer truncates toward zero and gives NA for NaN and out-of-range
 * values; NA integers are INT32_MIN / INT64_MIN and convert to NaN). */
static int is_fp(int dt) { return dt == DT_F32 || dt == DT_F64 || dt == DT_F16; }

/* the source value as a long double (exact for every dtype), NA integers as NaN;
 * int8 has no NA */
static long double conv_src(int from, const void *in, int64_t off) {
  if (from == DT_I32) {
    const int32_t x = ((const int32_t *)in)[off];
    return x == INT32_MIN ? (long double)NAN : (long double)x;
  }
  if (from == DT_I64) {
    const int64_t x = ((const int64_t *)in)[off];
    return x == INT64_MIN ? (long double)NAN : (long double)x; /* exact in long double */
  }
  return ld_get(in, from, off);
}

static void convert_one(int from, int to, const void *in, int64_t off, void *out, int64_t i) {
  if (to == DT_F32 || to == DT_F64 || to == DT_F16) {
    const long double v = conv_src(from, in, off); /* one rounding below: v is the exact source value */
    if (to == DT_F32)
      ((float *)out)[i] = (float)v;
    else if (to == DT_F64)
      ((double *)out)[i] = (double)v;
    else
      ((_Float16 *)out)[i] = (_Float16)v;
  } else if (to == DT_I32) {
    int32_t r;
    if (is_fp(from)) {
      const long double x = ld_get(in, from, off);
      r = (x > -2147483648.0L && x < 2147483648.0L) ? (int32_t)truncl(x) : INT32_MIN;
    } else if (from == DT_I64) {
      const int64_t x = ((const int64_t *)in)[off];
      r = (x >= -2147483647LL && x <= 2147483647LL) ? (int32_t)x : INT32_MIN;
    } else if (from == DT_BOOL) {
      r = ((const uint8_t *)in)[off];
    } else if (from == DT_I8) {
      r = ((const int8_t *)in)[off];
    } else {
      r = ((const int32_t *)in)[off];
    }
    ((int32_t *)out)[i] = r;
  } else if (to == DT_I64) {
    int64_t r;
    if (is_fp(from)) {
      const long double x = ld_get(in, from, off);
      r = (x > -9223372036854775808.0L && x < 9223372036854775808.0L) ? (int64_t)truncl(x) : INT64_MIN;
    } else if (from == DT_I32) {
      const int32_t x = ((const int32_t *)in)[off];
      r = x == INT32_MIN ? INT64_MIN : (int64_t)x;
    } else if (from == DT_BOOL) {
      r = ((const uint8_t *)in)[off];
    } else if (from == DT_I8) {
      r = ((const int8_t *)in)[off];
    } else {
      r = ((const int64_t *)in)[off];
    }
    ((int64_t *)out)[i] = r;
  } else if (to == DT_I8) {
    /* no NA: from a floating value truncate toward zero and saturate to
     * [-128, 127], NaN -> 0 (the device's float-to-int8 cast); from a wider
     * integer keep the low 8 bits */
    int8_t r;
    if (is_fp(from)) {
      const long double x = ld_get(in, from, off);
      r = isnan(x) ? 0 : (x <= -128.0L ? -128 : (x >= 127.0L ? 127 : (int8_t)truncl(x)));
    } else if (from == DT_I32) {
      r = (int8_t)(uint8_t)(((const int32_t *)in)[off] & 0xFF);
    } else if (from == DT_I64) {
      r = (int8_t)(uint8_t)(((const int64_t *)in)[off] & 0xFF);
    } else if (from == DT_BOOL) {
      r = (int8_t)((const uint8_t *)in)[off];
    } else {
      r = ((const int8_t *)in)[off];
    }
    ((int8_t *)out)[i] = r;
  } else { /* bool: x != 0, so NaN and NA integers give 1 */
    int nz;
    switch (from) {
      case DT_F32: nz = ((const float *)in)[off] != 0.0f; break;
      case DT_F64: nz = ((const double *)in)[off] != 0.0; break;
      case DT_F16: nz = ((const _Float16 *)in)[off] != 0; break;
      case DT_I32: nz = ((const int32_t *)in)[off] != 0; break;
      case DT_I64: nz = ((const int64_t *)in)[off] != 0; break;
      case DT_I8: nz = ((const int8_t *)in)[off] != 0; break;
      default: nz = ((const uint8_t *)in)[off] != 0; break;
    }
    ((uint8_t *)out)[i] = (uint8_t)nz;
  }
}

void orc_convert(int from, int to, const void *in, int nd, const int64_t *shape, const int64_t *st, void *out) {
  const int64_t n = numel(nd, shape);
  for (int64_t i = 0; i < n; ++i) convert_one(from, to, in, offset_of(i, nd, shape, st), out, i);
}

/* ---- counter-based random tensors --------------------------------------
 * Philox4x32-10 (Salmon, Moraes, Dror and Shaw, SC 2011) keyed by the 64-bit
 * seed; element i takes counter position offset + i.  Restates the
 * generator of this library (the reference draws from cuRAND seeded with
 * time(NULL), src/TensorRandom.cpp:19-27, which no run can reproduce).
 * Uniforms use the same arithmetic as the device (one fused multiply-add in
 * the tensor dtype, C99 fma/fmaf being correctly rounded); normals are
 * evaluated in long double and rounded once (the device uses float32 or
 * float64 math, so the tests compare normals within a tolerance). */
static void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0, n1 = (uint32_t)p1;
    const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1, n3 = (uint32_t)p0;
    c[0] = n0;
    c[1] = n1;
    c[2] = n2;
    c[3] = n3;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

/* one raw Philox4x32-10 block, for the known-answer tests */
void orc_philox(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  for (int k = 0; k < 4; ++k) out[k] = ctr[k];
  philox4x32_10(out, key[0], key[1]);
}

void orc_rand(int dt, int dist, double a, double b, uint64_t seed, uint64_t offset, int64_t n, void *out) {
  const int pb = dt == DT_F32 ? 4 : 2;
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  const long double two_pi = 6.283185307179586476925286766559005768L;
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t pos = offset + (uint64_t)i, g = pos / (uint64_t)pb;
    const int j = (int)(pos % (uint64_t)pb);
    uint32_t w[4] = {(uint32_t)g, (uint32_t)(g >> 32), 0u, 0u};
    philox4x32_10(w, k0, k1);
    if (dt == DT_F32) {
      if (dist == 0) {
        const float u = (float)(w[j] >> 8) * 0x1p-24f;
        ((float *)out)[i] = fmaf((float)(b - a), u, (float)a);
      } else {
        const int p = j / 2;
        const long double u = (long double)((w[2 * p] >> 8) + 1u) * 0x1p-24L;
        const long double t = (long double)(w[2 * p + 1] >> 8) * 0x1p-24L;
        const long double r = sqrtl(-2.0L * logl(u));
        const long double z = (j % 2 == 0) ? r * cosl(two_pi * t) : r * sinl(two_pi * t);
        ((float *)out)[i] = fmaf((float)b, (float)z, (float)a);
      }
    } else {
      const uint64_t x0 = (((uint64_t)w[0] << 32) | w[1]) >> 11, x1 = (((uint64_t)w[2] << 32) | w[3]) >> 11;
      if (dist == 0) {
        ((double *)out)[i] = fma(b - a, (double)(j == 0 ? x0 : x1) * 0x1p-53, a);
      } else {
        const long double u = (long double)(x0 + 1) * 0x1p-53L, t = (long double)x1 * 0x1p-53L;
        const long double r = sqrtl(-2.0L * logl(u));
        const double z = (double)(j == 0 ? r * cosl(two_pi * t) : r * sinl(two_pi * t));
        ((double *)out)[i] = fma(b, z, a);
      }
    }
  }
}

/* ---- reductions over a set of reduced values ---------------------------- */
static long double r_mean(const long double *v, int64_t n) {
  long double s = 0.0L;
  for (int64_t i = 0; i < n; ++i) s += v[i];
  s /= n;
  if (isfinite(s)) {
    long double t = 0.0L;
    for (int64_t i = 0; i < n; ++i) t += v[i] - s;
    s += t / n;
  }
  return s;
}

static long double reduce_vals(int op, const long double *v, int64_t n) {
  switch (op) {
    case R_SUM: {
      long double s = 0.0L;
      for (int64_t i = 0; i < n; ++i) s += v[i];
      return s;
    }
    case R_MEAN: return r_mean(v, n);
    case R_MAX: {
      long double m = -INFINITY;
      for (int64_t i = 0; i < n; ++i) m = fmaxl_r(m, v[i]);
      return m;
    }
    case R_MIN: {
      long double m = INFINITY;
      for (int64_t i = 0; i < n; ++i) m = fminl_r(m, v[i]);
      return m;
    }
    case R_PROD: {
      long double p = 1.0L;
      for (int64_t i = 0; i < n; ++i) p *= v[i];
      return p;
    }
    case R_VAR: {
      if (n < 2) return NAN;
      const long double m = r_mean(v, n);
      long double s = 0.0L;
      for (int64_t i = 0; i < n; ++i) s += (v[i] - m) * (v[i] - m);
      return s / (n - 1);
    }
    case R_COUNT: {
      int64_t c = 0;
      for (int64_t i = 0; i < n; ++i) c += v[i] != 0.0L;
      return (long double)c;
    }
  }
  return 0.0L;
}

/* Splits dims into kept/reduced; output index runs column-major over kept dims. */
static void split(int nd, const int64_t *shape, const int64_t *st, uint32_t mask, int *nk, int64_t *ks, int64_t *kst,
                  int *nr, int64_t *rs, int64_t *rst) {
  *nk = *nr = 0;
  for (int d = 0; d < nd; ++d) {
    if ((mask >> d) & 1u) {
      rs[*nr] = shape[d];
      rst[*nr] = st[d];
      (*nr)++;
    } else {
      ks[*nk] = shape[d];
      kst[*nk] = st[d];
      (*nk)++;
    }
  }
}

/* out (double) holds one value per kept element; outputs o_lo..o_hi-1 are
 * computed (the multithreaded checks split the outputs over threads) */
int orc_reduce_range(int op, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st,
                     uint32_t mask, double *out, int64_t o_lo, int64_t o_hi) {
  int nk, nr;
  int64_t ks[MAXD], kst[MAXD], rs[MAXD], rst[MAXD];
  split(nd, shape, st, mask, &nk, ks, kst, &nr, rs, rst);
  const int64_t R = numel(nr, rs);
  long double *v = (long double *)malloc(sizeof(long double) * (R > 0 ? R : 1));
  if (!v) return -1;
  for (int64_t o = o_lo; o < o_hi; ++o) {
    const int64_t base = offset_of(o, nk, ks, kst);
    for (int64_t j = 0; j < R; ++j) v[j] = ld_get(in, dt, base + offset_of(j, nr, rs, rst));
    if (op == R_ANY || op == R_ALL) {
      /* R's any()/all() over as.logical(x): NaN and NA integers are NA; the
       * result is 1, 0 or NA (returned as NaN) */
      int64_t t = 0, na = 0;
      for (int64_t j = 0; j < R; ++j) {
        const int is_na = isnan(v[j]) || (dt == DT_I32 && v[j] == (long double)INT32_MIN) ||
                          (dt == DT_I64 && v[j] == (long double)INT64_MIN);
        na += is_na;
        t += !is_na && v[j] != 0.0L;
      }
      if (op == R_ANY)
        out[o] = t > 0 ? 1.0 : (na > 0 ? NAN : 0.0);
      else
        out[o] = (t + na < R) ? 0.0 : (na > 0 ? NAN : 1.0);
      continue;
    }
    out[o] = (double)reduce_vals(op, v, R);
  }
  free(v);
  return 0;
}

int orc_reduce(int op, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, uint32_t mask,
               double *out) {
  int nk, nr;
  int64_t ks[MAXD], kst[MAXD], rs[MAXD], rst[MAXD];
  split(nd, shape, st, mask, &nk, ks, kst, &nr, rs, rst);
  return orc_reduce_range(op, dt, in, nd, shape, st, mask, out, 0, numel(nk, ks));
}

/* first index of the max (min); NaN never wins; -1 when none.  Outputs
 * o_lo..o_hi-1 (o_hi < 0: all). */
int orc_arg_reduce_range(int is_max, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st,
                         int axis, int one_based, int64_t *out, int64_t o_lo, int64_t o_hi) {
  const uint32_t mask = axis < 0 ? 0xFFu : (1u << axis);
  int nk, nr;
  int64_t ks[MAXD], kst[MAXD], rs[MAXD], rst[MAXD];
  split(nd, shape, st, mask, &nk, ks, kst, &nr, rs, rst);
  const int64_t O = numel(nk, ks), R = numel(nr, rs);
  if (o_hi < 0 || o_hi > O) o_hi = O;
  for (int64_t o = o_lo; o < o_hi; ++o) {
    const int64_t base = offset_of(o, nk, ks, kst);
    int64_t best = -1;
    long double bv = 0.0L;
    for (int64_t j = 0; j < R; ++j) {
      const long double x = ld_get(in, dt, base + offset_of(j, nr, rs, rst));
      if (isnan(x)) continue;
      if (best < 0 || (is_max ? x > bv : x < bv)) {
        best = j;
        bv = x;
      }
    }
    out[o] = best < 0 ? -1 : best + (one_based ? 1 : 0);
  }
  return 0;
}

int orc_arg_reduce(int is_max, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis,
                   int one_based, int64_t *out) {
  return orc_arg_reduce_range(is_max, dt, in, nd, shape, st, axis, one_based, out, 0, -1);
}

int orc_scan_fibers(int is_prod, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis,
                    void *out, int64_t f_lo, int64_t f_hi);

/* cumsum/cumprod along `axis` (axis < 0: flattened column-major) */
int orc_scan(int is_prod, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis,
             void *out) {
  const int64_t n = numel(nd, shape);
  if (axis < 0) {
    long double acc = is_prod ? 1.0L : 0.0L;
    for (int64_t i = 0; i < n; ++i) {
      const long double x = ld_get(in, dt, offset_of(i, nd, shape, st));
      acc = is_prod ? acc * x : acc + x;
      put(out, dt, i, acc);
    }
    return 0;
  }
  return orc_scan_fibers(is_prod, dt, in, nd, shape, st, axis, out, 0, -1);
}

/* cumsum/cumprod along `axis` >= 0 of fibers f_lo..f_hi-1 (f_hi < 0: all);
 * fiber f starts at output index (f % ostride) + (f / ostride) * ostride * R */
int orc_scan_fibers(int is_prod, int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis,
                    void *out, int64_t f_lo, int64_t f_hi) {
  const int64_t n = numel(nd, shape);
  /* out is contiguous: stride of `axis` in out = prod(shape[<axis]) */
  int64_t ostride = 1;
  for (int d = 0; d < axis; ++d) ostride *= shape[d];
  const int64_t R = shape[axis];
  const int64_t F = R > 0 ? n / R : 0;
  if (f_hi < 0 || f_hi > F) f_hi = F;
  for (int64_t f = f_lo; f < f_hi; ++f) {
    const int64_t i = (f % ostride) + (f / ostride) * ostride * R;
    long double acc = is_prod ? 1.0L : 0.0L;
    for (int64_t k = 0; k < R; ++k) {
      const int64_t oi = i + k * ostride;
      const long double x = ld_get(in, dt, offset_of(oi, nd, shape, st));
      acc = is_prod ? acc * x : acc + x;
      put(out, dt, oi, acc);
    }
  }
  return 0;
}

/* softmax along `axis` (axis < 0: whole tensor); exp in long double of the
 * dtype-rounded difference, sum in long double */
int orc_softmax_fibers(int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis, void *out,
                       int64_t f_lo, int64_t f_hi) {
  const int64_t n = numel(nd, shape);
  if (n == 0) return 0;
  int64_t ostride = 1, R = n;
  if (axis >= 0) {
    for (int d = 0; d < axis; ++d) ostride *= shape[d];
    R = shape[axis];
  }
  if (R == 0) return 0;
  const int64_t F = n / R;
  if (f_hi < 0 || f_hi > F) f_hi = F;
  long double *e = (long double *)malloc(sizeof(long double) * R);
  if (!e) return -1;
  for (int64_t f = f_lo; f < f_hi; ++f) {
    /* fiber f starts at (f % ostride) + (f / ostride) * ostride * R */
    const int64_t i = (f % ostride) + (f / ostride) * ostride * R;
    const int64_t step = axis >= 0 ? ostride : 1;
    long double m = -INFINITY;
    for (int64_t k = 0; k < R; ++k) m = fmaxl_r(m, ld_get(in, dt, offset_of(i + k * step, nd, shape, st)));
    long double s = 0.0L;
    for (int64_t k = 0; k < R; ++k) {
      const long double d = rnd(ld_get(in, dt, offset_of(i + k * step, nd, shape, st)) - m, dt);
      e[k] = expl(d);
      s += e[k];
    }
    for (int64_t k = 0; k < R; ++k) put(out, dt, i + k * step, e[k] / s);
  }
  free(e);
  return 0;
}

int orc_softmax(int dt, const void *in, int nd, const int64_t *shape, const int64_t *st, int axis, void *out) {
  return orc_softmax_fibers(dt, in, nd, shape, st, axis, out, 0, -1);
}

/* Fused sum and var of a contiguous array (for large-size checks and the CPU
 * baseline): long double sum, two-pass variance. */
void orc_sum_var(int dt, const void *in, int64_t n, double *sum, double *var) {
  long double s = 0.0L;
  for (int64_t i = 0; i < n; ++i) s += ld_get(in, dt, i);
  long double m = s / n;
  long double t = 0.0L;
  for (int64_t i = 0; i < n; ++i) t += ld_get(in, dt, i) - m;
  m += t / n;
  long double q = 0.0L;
  for (int64_t i = 0; i < n; ++i) {
    const long double d = ld_get(in, dt, i) - m;
    q += d * d;
  }
  *sum = (double)s;
  *var = n > 1 ? (double)(q / (n - 1)) : NAN;
}
