// Reduction accumulators and result stores shared by the full, axis and
// scan kernels.
//
// Accuracy contract (base-R semantics, the reference's own kernels accumulate
// in the tensor dtype, src/kernels/tensor_kernels.cu:60-84):
//   float32 sums/means/variances accumulate in float64;
//   float64 sums accumulate in double-double (TwoSum), variances as
//   double-double sums of (x-K) and (x-K)^2 with an exact square (fma TwoProd);
//   K is the first element of each reduced fiber, so no pass over the mean is
//   needed and partials merge by addition.
//   max/min use fmax/fmin (NaN-ignoring, as MaxOp/MinOp in
//   src/kernels/tensor_kernels.cuh:32-51); arg-reductions keep the first index
//   among equal values (strict comparison, src/kernels/tensor_kernels.cu:794).
#pragma once

#include <cfloat>
#include <climits>
#include <type_traits>

#include "common.cuh"
#include "ops.cuh"

namespace acd {

// Where and how a reduced value is written.
struct OutSpec {
  void *out = nullptr;
  void *out2 = nullptr;  // arg value (ARG) or variance (sum_var)
  int32_t dt = ACD_FLOAT64;
  int32_t dt2 = ACD_FLOAT64;
  int32_t op = ACD_RED_SUM;
  int32_t mode = 0;  // 0 value, 1 index, 2 key, 3 stats, 4 sum+var
  int32_t one_based = 0;
  int32_t pad = 0;
  int64_t index_base = 0;
  int64_t n = 0;  // elements per reduced fiber
};

enum { kModeValue = 0, kModeIndex = 1, kModeKey = 2, kModeStats = 3, kModeSumVar = 4 };

__device__ __forceinline__ void store_f(void *p, int32_t dt, int64_t i, double v) {
  switch (dt) {
    case ACD_FLOAT32: static_cast<float *>(p)[i] = (float)v; break;
    case ACD_FLOAT64: static_cast<double *>(p)[i] = v; break;
    case ACD_INT32: static_cast<int32_t *>(p)[i] = (int32_t)v; break;
    case ACD_INT64: static_cast<int64_t *>(p)[i] = (int64_t)v; break;
    default: break;
  }
}

__device__ __forceinline__ void store_i(void *p, int32_t dt, int64_t i, long long v) {
  switch (dt) {
    case ACD_INT32:  // R's NA_integer_ on overflow
      static_cast<int32_t *>(p)[i] = (v > INT_MAX || v <= INT_MIN) ? INT_MIN : (int32_t)v;
      break;
    case ACD_INT64: static_cast<int64_t *>(p)[i] = v; break;
    case ACD_FLOAT32: static_cast<float *>(p)[i] = (float)v; break;
    case ACD_FLOAT64: static_cast<double *>(p)[i] = (double)v; break;
    default: break;
  }
}

template <typename T> __device__ __forceinline__ T lowest_of() {
  if constexpr (std::is_floating_point<T>::value) return -(T)INFINITY;
  else if constexpr (sizeof(T) == 8) return (T)LLONG_MIN;
  else return (T)INT_MIN;
}
template <typename T> __device__ __forceinline__ T highest_of() {
  if constexpr (std::is_floating_point<T>::value) return (T)INFINITY;
  else if constexpr (sizeof(T) == 8) return (T)LLONG_MAX;
  else return (T)INT_MAX;
}

// Promotes bool (uint8) to a 4-byte lane for shuffles.
template <typename T> using Lane = std::conditional_t<(sizeof(T) < 4), int32_t, T>;

// ---------------------------------------------------------------------------
template <typename T, typename Enable = void>
struct SumAcc;

template <>
struct SumAcc<float> {
  static constexpr bool kShift = false;
  double s;
  __device__ __forceinline__ void init() { s = 0.0; }
  __device__ __forceinline__ void set_shift(float) {}
  __device__ __forceinline__ void add(float x, int64_t) { s += (double)x; }
  __device__ __forceinline__ void merge(const SumAcc &o) { s += o.s; }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    store_f(os.out, os.dt, oi, os.op == ACD_RED_MEAN ? s / (double)os.n : s);
  }
};

template <>
struct SumAcc<double> {
  static constexpr bool kShift = false;
  DD s;
  __device__ __forceinline__ void init() { s.hi = 0.0; s.lo = 0.0; }
  __device__ __forceinline__ void set_shift(double) {}
  __device__ __forceinline__ void add(double x, int64_t) { dd_add(s, x); }
  __device__ __forceinline__ void merge(const SumAcc &o) { dd_merge(s, o.s); }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    const double v = s.hi + s.lo;
    if (os.op == ACD_RED_MEAN) {
      // (hi + lo) / n with one rounding of the quotient of the exact-ish sum
      const double q = s.hi / (double)os.n;
      const double r = fma(-q, (double)os.n, s.hi) + s.lo;
      store_f(os.out, os.dt, oi, q + r / (double)os.n);
    } else {
      store_f(os.out, os.dt, oi, v);
    }
  }
};

// float16: every half value is exact in float64, so the sum is a float64
// accumulation of the exact values (the reference's tensor_sum_float16 is a
// placeholder returning 0, src/kernels/tensor_ops.cu:701-705).
template <>
struct SumAcc<__half> {
  static constexpr bool kShift = false;
  double s;
  __device__ __forceinline__ void init() { s = 0.0; }
  __device__ __forceinline__ void set_shift(__half) {}
  __device__ __forceinline__ void add(__half x, int64_t) { s += (double)__half2float(x); }
  __device__ __forceinline__ void merge(const SumAcc &o) { s += o.s; }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    store_f(os.out, os.dt, oi, os.op == ACD_RED_MEAN ? s / (double)os.n : s);
  }
};

template <typename T>
struct SumAcc<T, std::enable_if_t<std::is_integral<T>::value>> {
  static constexpr bool kShift = false;
  long long s;
  __device__ __forceinline__ void init() { s = 0; }
  __device__ __forceinline__ void set_shift(T) {}
  __device__ __forceinline__ void add(T x, int64_t) { s += (long long)x; }
  __device__ __forceinline__ void merge(const SumAcc &o) { s += o.s; }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    if (os.op == ACD_RED_MEAN)
      store_f(os.out, os.dt, oi, (double)s / (double)os.n);
    else
      store_i(os.out, os.dt, oi, s);
  }
};

template <typename T>
struct CountAcc {
  static constexpr bool kShift = false;
  long long c;
  __device__ __forceinline__ void init() { c = 0; }
  __device__ __forceinline__ void set_shift(T) {}
  __device__ __forceinline__ void add(T x, int64_t) {
    if constexpr (std::is_same<T, __half>::value)
      c += (__half2float(x) != 0.0f) ? 1 : 0;
    else
      c += (x != T(0)) ? 1 : 0;
  }
  __device__ __forceinline__ void merge(const CountAcc &o) { c += o.c; }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const { store_i(os.out, os.dt, oi, c); }
};

// any / all: which truth values occur (bit 1 TRUE = non-zero, bit 2 FALSE,
// bit 4 NA = NaN or an NA integer); the result follows R's three-valued
// logic (an empty reduction: any FALSE, all TRUE).
template <typename T, bool ALL>
struct TruthAcc {
  static constexpr bool kShift = false;
  uint32_t f;
  __device__ __forceinline__ void init() { f = 0u; }
  __device__ __forceinline__ void set_shift(T) {}
  __device__ __forceinline__ void add(T x, int64_t) {
    bool is_na;
    if constexpr (std::is_floating_point<T>::value)
      is_na = x != x;
    else if constexpr (std::is_same<T, int32_t>::value)
      is_na = x == INT32_MIN;
    else if constexpr (std::is_same<T, int64_t>::value)
      is_na = x == INT64_MIN;
    else
      is_na = false;
    f |= is_na ? 4u : (x != T(0) ? 1u : 2u);
  }
  __device__ __forceinline__ void merge(const TruthAcc &o) { f |= o.f; }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    long long r;
    if (ALL)
      r = (f & 2u) ? 0 : ((f & 4u) ? (long long)INT32_MIN : 1);
    else
      r = (f & 1u) ? 1 : ((f & 4u) ? (long long)INT32_MIN : 0);
    store_i(os.out, os.dt, oi, r);
  }
};

// Nonzero bytes of a 32-bit word: each byte's bits are folded into its bit 0
// (the shifts stay inside the byte for bits 0..3, which are all that is
// kept), then the marks are counted.
__device__ __forceinline__ int nonzero_bytes(uint32_t w) {
  uint32_t t = w | (w >> 4);
  t |= t >> 2;
  t |= t >> 1;
  return __popc(t & 0x01010101u);
}

// Adds one vector of V elements to a single accumulator: a count over bytes
// (bool) takes 4 bytes per instruction, everything else element by element
// (`first` is the index of element 0, used by the argmin/argmax rules).
// Accumulators that define `static constexpr bool kVecAdd = true` and
// `add_vec(const Vec<T, V> &)` take a whole vector at once.
template <class A, class = void>
struct has_vec_add : std::false_type {};
template <class A>
struct has_vec_add<A, std::void_t<decltype(A::kVecAdd)>> : std::integral_constant<bool, A::kVecAdd> {};

template <class Acc, typename T, int V>
__device__ __forceinline__ void acc_add_vec(Acc &acc, const Vec<T, V> &x, int64_t first) {
  if constexpr (std::is_same<Acc, CountAcc<uint8_t>>::value && V == 16) {
    const uint4 w = *reinterpret_cast<const uint4 *>(&x);
    acc.c += nonzero_bytes(w.x) + nonzero_bytes(w.y) + nonzero_bytes(w.z) + nonzero_bytes(w.w);
  } else if constexpr (has_vec_add<Acc>::value) {
    acc.add_vec(x);
  } else {
#pragma unroll
    for (int k = 0; k < V; ++k) acc.add(x.v[k], first + k);
  }
}

template <typename T, bool MAX>
struct ExtAcc {
  static constexpr bool kShift = false;
  Lane<T> m;
  __device__ __forceinline__ void init() { m = MAX ? (Lane<T>)lowest_of<Lane<T>>() : (Lane<T>)highest_of<Lane<T>>(); }
  __device__ __forceinline__ void set_shift(T) {}
  __device__ __forceinline__ void add(T x, int64_t) {
    const Lane<T> v = (Lane<T>)x;
    if constexpr (std::is_floating_point<T>::value)
      m = MAX ? (Lane<T>)fmax(m, v) : (Lane<T>)fmin(m, v);
    else
      m = MAX ? (v > m ? v : m) : (v < m ? v : m);
  }
  // merged in the lane type: an empty partial holds the lane type's extreme,
  // which a narrow T (int8, bool) could not represent
  __device__ __forceinline__ void merge(const ExtAcc &o) {
    if constexpr (std::is_floating_point<T>::value)
      m = MAX ? (Lane<T>)fmax(m, o.m) : (Lane<T>)fmin(m, o.m);
    else
      m = MAX ? (o.m > m ? o.m : m) : (o.m < m ? o.m : m);
  }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    if constexpr (std::is_floating_point<T>::value)
      store_f(os.out, os.dt, oi, (double)m);
    else
      store_i(os.out, os.dt, oi, (long long)m);
  }
};

template <typename T>
struct ProdAcc {
  static constexpr bool kShift = false;
  double p;
  __device__ __forceinline__ void init() { p = 1.0; }
  __device__ __forceinline__ void set_shift(T) {}
  __device__ __forceinline__ void add(T x, int64_t) { p *= (double)x; }
  __device__ __forceinline__ void merge(const ProdAcc &o) { p *= o.p; }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const { store_f(os.out, os.dt, oi, p); }
};

// Shifted moments: s1 = sum(x-K), s2 = sum((x-K)^2).
template <typename T>
struct VarAcc;

template <>
struct VarAcc<float> {
  static constexpr bool kShift = true;
  double k, s1, s2;
  __device__ __forceinline__ void init() { k = 0.0; s1 = 0.0; s2 = 0.0; }
  __device__ __forceinline__ void set_shift(float x) { k = (double)x; }
  __device__ __forceinline__ void add(float x, int64_t) {
    const double d = (double)x - k;
    s1 += d;
    s2 += d * d;
  }
  __device__ __forceinline__ void merge(const VarAcc &o) { s1 += o.s1; s2 += o.s2; }
  __device__ __forceinline__ double sum1() const { return s1; }
  __device__ __forceinline__ double var(double n) const {
    if (n < 2.0) return (double)NAN;
    const double v = (s2 - s1 * (s1 / n)) / (n - 1.0);
    return v < 0.0 ? 0.0 : v;
  }
  __device__ __forceinline__ double total(double n) const { return fma(n, k, s1); }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    const double n = (double)os.n;
    if (os.mode == kModeStats) {
      double *p = static_cast<double *>(os.out);
      p[0] = n; p[1] = k; p[2] = s1; p[3] = s2; p[4] = 0.0; p[5] = 0.0;
    } else if (os.mode == kModeSumVar) {
      if (os.out) store_f(os.out, os.dt, oi, total(n));
      if (os.out2) store_f(os.out2, os.dt2, oi, var(n));
    } else if (os.op == ACD_RED_MEAN) {
      store_f(os.out, os.dt, oi, k + s1 / n);
    } else if (os.op == ACD_RED_SUM) {
      store_f(os.out, os.dt, oi, total(n));
    } else {
      store_f(os.out, os.dt, oi, var(n));
    }
  }
};

template <>
struct VarAcc<double> {
  static constexpr bool kShift = true;
  double k;
  double pad;
  DD s1, s2;
  __device__ __forceinline__ void init() { k = 0.0; pad = 0.0; s1.hi = s1.lo = s2.hi = s2.lo = 0.0; }
  __device__ __forceinline__ void set_shift(double x) { k = x; }
  __device__ __forceinline__ void add(double x, int64_t) {
    const double d = x - k;
    dd_add(s1, d);
    dd_add_square(s2, d);
  }
  __device__ __forceinline__ void merge(const VarAcc &o) { dd_merge(s1, o.s1); dd_merge(s2, o.s2); }
  __device__ __forceinline__ double var(double n) const {
    if (n < 2.0) return (double)NAN;
    const double t = s1.hi + s1.lo;
    const double q = t * (t / n);
    const double v = ((s2.hi - q) + s2.lo) / (n - 1.0);
    return v < 0.0 ? 0.0 : v;
  }
  __device__ __forceinline__ double total(double n) const {
    // n*k + s1 in double-double
    const double p = n * k;
    const double pe = fma(n, k, -p);
    double s, e;
    two_sum(p, s1.hi, s, e);
    return s + (e + pe + s1.lo);
  }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    const double n = (double)os.n;
    if (os.mode == kModeStats) {
      double *p = static_cast<double *>(os.out);
      p[0] = n; p[1] = k; p[2] = s1.hi; p[3] = s2.hi; p[4] = s1.lo; p[5] = s2.lo;
    } else if (os.mode == kModeSumVar) {
      if (os.out) store_f(os.out, os.dt, oi, total(n));
      if (os.out2) store_f(os.out2, os.dt2, oi, var(n));
    } else if (os.op == ACD_RED_MEAN) {
      store_f(os.out, os.dt, oi, total(n) / n);
    } else if (os.op == ACD_RED_SUM) {
      store_f(os.out, os.dt, oi, total(n));
    } else {
      store_f(os.out, os.dt, oi, var(n));
    }
  }
};

// Order-preserving 32-bit image of a float (larger float -> larger unsigned).
__device__ __forceinline__ uint32_t ordered_bits(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <typename T, bool MAX>
struct ArgAcc {
  static constexpr bool kShift = false;
  T v;
  int32_t pad;
  int64_t i;
  __device__ __forceinline__ void init() {
    v = MAX ? lowest_of<T>() : highest_of<T>();
    pad = 0;
    i = LLONG_MAX;
  }
  __device__ __forceinline__ void set_shift(T) {}
  __device__ __forceinline__ void add(T x, int64_t idx) {
    const bool better = MAX ? (x > v) : (x < v);
    if (better || (x == v && idx < i)) {
      v = x;
      i = idx;
    }
  }
  __device__ __forceinline__ void merge(const ArgAcc &o) { add(o.v, o.i); }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t oi) const {
    const bool none = (i == LLONG_MAX);
    if (os.mode == kModeKey) {
      long long key;
      if (none) {
        key = LLONG_MIN;
      } else {
        // -0 and +0 compare equal in the reduction; give them one key so the
        // index decides between them across shards too
        uint32_t ob;
        if constexpr (std::is_same<T, float>::value) ob = ordered_bits(v + 0.0f);
        else ob = ordered_bits((float)v + 0.0f);
        const uint64_t gi = (uint64_t)(i + os.index_base);
        const uint64_t u = ((uint64_t)ob << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)gi);
        key = (long long)(u ^ 0x8000000000000000ull);
      }
      static_cast<long long *>(os.out)[oi] = key;
      return;
    }
    store_i(os.out, os.dt, oi, none ? -1 : (long long)(i + os.one_based));
    if (os.out2) {
      if constexpr (std::is_floating_point<T>::value)
        store_f(os.out2, os.dt2, oi, (double)v);
      else
        store_i(os.out2, os.dt2, oi, (long long)v);
    }
  }
};

// Online softmax statistics: running maximum m and sum of exp(x - m).
template <typename T>
struct SoftStatAcc {
  static constexpr bool kShift = false;
  static constexpr bool kVecAdd = true;
  double m, s;
  __device__ __forceinline__ void init() { m = -INFINITY; s = 0.0; }
  __device__ __forceinline__ void set_shift(T) {}
  // A vector at once: one rescale for the vector's maximum, then one exp per
  // element (the per-element rule below rescales whenever the maximum grows).
  template <int V>
  __device__ __forceinline__ void add_vec(const Vec<T, V> &x) {
    T mb = x.v[0];
#pragma unroll
    for (int k = 1; k < V; ++k) mb = m_max(mb, x.v[k]);
    const double mbd = (double)mb;
    if (mbd > m) {
      s = (m == -INFINITY) ? 0.0 : s * exp(m - mbd);
      m = mbd;
    }
    if (m == -INFINITY) {  // only -inf (or NaN) so far: a NaN poisons the sum
#pragma unroll
      for (int k = 0; k < V; ++k)
        if (x.v[k] != x.v[k]) s = (double)NAN;
      return;
    }
    // m holds a value of T, so x - m rounded once in T equals the rounding of
    // the exact difference taken in double; the V exps are summed pairwise in
    // T (two roundings of a sum of at most V terms <= 1) before one float64 add
    const T mt = (T)m;
    T e[V];
#pragma unroll
    for (int k = 0; k < V; ++k) e[k] = m_exp(x.v[k] - mt);
#pragma unroll
    for (int w = 1; w < V; w <<= 1)
#pragma unroll
      for (int k = 0; k + w < V; k += 2 * w) e[k] += e[k + w];
    s += (double)e[0];
  }
  __device__ __forceinline__ void add(T x, int64_t) {
    const double xd = (double)x;
    if (xd == -INFINITY) return;
    if (xd > m) {
      s = s * exp(m - xd) + 1.0;
      m = xd;
    } else {
      s += (double)m_exp((T)(xd - m));
    }
  }
  __device__ __forceinline__ void merge(const SoftStatAcc &o) {
    if (o.m == -INFINITY) return;
    if (m == -INFINITY) {
      m = o.m;
      s = o.s;
      return;
    }
    if (o.m > m) {
      s = s * exp(m - o.m) + o.s;
      m = o.m;
    } else {
      s += o.s * exp(o.m - m);
    }
  }
  __device__ __forceinline__ void store(const OutSpec &os, int64_t) const {
    double *p = static_cast<double *>(os.out);
    p[0] = m;
    p[1] = s;
  }
};

}  // namespace acd
