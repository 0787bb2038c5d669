// Elementwise operator definitions (device).  One rounding per R operator in
// the tensor dtype: the library is compiled with --fmad=false so no multiply
// and add pair is contracted into an fma, and CUDA's own math functions are
// called for exp/log/tanh/erf/sin/cos (their documented ulp bounds apply).
//
// Formulas follow the reference functors (src/kernels/tensor_kernels.cuh:10-192):
// sigmoid = 1/(1+exp(-x)) (float32: evaluated in double, one rounding),
// relu = fmax(x, 0), round = rint (half to even),
// max/min = fmax/fmin (NaN-ignoring), comparisons write 1 or 0.  Two
// deliberate differences, both toward base R: x/s is a true division (the
// reference multiplies by 1/s, src/kernels/tensor_ops.cu:1901-1913), and x^2
// is x*x.
#pragma once

#include <climits>
#include <type_traits>

#include "common.cuh"

namespace acd {

__device__ __forceinline__ float m_exp(float x) { return expf(x); }
__device__ __forceinline__ double m_exp(double x) { return exp(x); }
__device__ __forceinline__ float m_log(float x) { return logf(x); }
__device__ __forceinline__ double m_log(double x) { return log(x); }
__device__ __forceinline__ float m_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double m_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float m_erf(float x) { return erff(x); }
__device__ __forceinline__ double m_erf(double x) { return erf(x); }
__device__ __forceinline__ float m_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double m_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float m_sin(float x) { return sinf(x); }
__device__ __forceinline__ double m_sin(double x) { return sin(x); }
__device__ __forceinline__ float m_cos(float x) { return cosf(x); }
__device__ __forceinline__ double m_cos(double x) { return cos(x); }
__device__ __forceinline__ float m_floor(float x) { return floorf(x); }
__device__ __forceinline__ double m_floor(double x) { return floor(x); }
__device__ __forceinline__ float m_ceil(float x) { return ceilf(x); }
__device__ __forceinline__ double m_ceil(double x) { return ceil(x); }
__device__ __forceinline__ float m_rint(float x) { return rintf(x); }
__device__ __forceinline__ double m_rint(double x) { return rint(x); }
__device__ __forceinline__ float m_abs(float x) { return fabsf(x); }
__device__ __forceinline__ double m_abs(double x) { return fabs(x); }
__device__ __forceinline__ int8_t m_abs(int8_t x) { return (int8_t)(x < 0 ? -x : x); }
__device__ __forceinline__ int32_t m_abs(int32_t x) { return x < 0 ? -x : x; }
__device__ __forceinline__ int64_t m_abs(int64_t x) { return x < 0 ? -x : x; }
__device__ __forceinline__ float m_max(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double m_max(double a, double b) { return fmax(a, b); }
__device__ __forceinline__ int8_t m_max(int8_t a, int8_t b) { return a > b ? a : b; }
__device__ __forceinline__ int32_t m_max(int32_t a, int32_t b) { return a > b ? a : b; }
__device__ __forceinline__ int64_t m_max(int64_t a, int64_t b) { return a > b ? a : b; }
__device__ __forceinline__ float m_min(float a, float b) { return fminf(a, b); }
__device__ __forceinline__ double m_min(double a, double b) { return fmin(a, b); }
__device__ __forceinline__ int8_t m_min(int8_t a, int8_t b) { return a < b ? a : b; }
__device__ __forceinline__ int32_t m_min(int32_t a, int32_t b) { return a < b ? a : b; }
__device__ __forceinline__ int64_t m_min(int64_t a, int64_t b) { return a < b ? a : b; }
// float pow is evaluated in double and rounded once (CUDA's double pow is
// within 2 ulp of double, so the float result is within 1 ulp).
__device__ __forceinline__ float m_pow(float a, float b) { return (float)pow((double)a, (double)b); }
__device__ __forceinline__ double m_pow(double a, double b) { return pow(a, b); }

// A comparison result (1 or 0) in the output dtype.
template <typename O>
__device__ __forceinline__ O flag_as(bool c) {
  if constexpr (std::is_same<O, __half>::value)
    return __float2half_rn(c ? 1.0f : 0.0f);
  else
    return O(c ? 1 : 0);
}

// IEEE binary16 (FLOAT16 tensors): each operation is evaluated in float32 on
// the exact half operands and rounded once to half.  For + - * / and the
// square this equals the correctly rounded binary16 result (float32 carries
// 24 bits >= 2*11 + 2, so the double rounding is innocuous), i.e. the
// reference's half operator arithmetic (src/kernels/tensor_kernels.cuh:10-25
// applied to half).
template <int OP>
__device__ __forceinline__ __half half_unary(__half x) {
  const float f = __half2float(x);
  if constexpr (OP == ACD_ABS) return __float2half_rn(fabsf(f));
  else if constexpr (OP == ACD_NEG) return __float2half_rn(-f);
  else if constexpr (OP == ACD_SQUARE) return __float2half_rn(f * f);
  else return x;  // ACD_COPY
}

template <int OP, typename O>
__device__ __forceinline__ O half_binary(__half a, __half b) {
  const float x = __half2float(a), y = __half2float(b);
  if constexpr (OP == ACD_GT) return flag_as<O>(x > y);
  else if constexpr (OP == ACD_LT) return flag_as<O>(x < y);
  else if constexpr (OP == ACD_EQ) return flag_as<O>(x == y);
  else if constexpr (OP == ACD_NE) return flag_as<O>(x != y);
  else if constexpr (OP == ACD_GE) return flag_as<O>(x >= y);
  else if constexpr (OP == ACD_LE) return flag_as<O>(x <= y);
  else if constexpr (OP == ACD_ADD) return __float2half_rn(x + y);
  else if constexpr (OP == ACD_SUB) return __float2half_rn(x - y);
  else if constexpr (OP == ACD_MUL) return __float2half_rn(x * y);
  else if constexpr (OP == ACD_DIV) return __float2half_rn(x / y);
  else if constexpr (OP == ACD_MAX) return __float2half_rn(fmaxf(x, y));
  else if constexpr (OP == ACD_MIN) return __float2half_rn(fminf(x, y));
  else if constexpr (OP == ACD_RSUB) return __float2half_rn(y - x);
  else return __float2half_rn(y / x);  // ACD_RDIV
}

template <int OP, typename T>
__device__ __forceinline__ T unary_apply(T x) {
  if constexpr (std::is_same<T, __half>::value) return half_unary<OP>(x);
  else if constexpr (OP == ACD_EXP) return m_exp(x);
  else if constexpr (OP == ACD_LOG) return m_log(x);
  else if constexpr (OP == ACD_SQRT) return m_sqrt(x);
  else if constexpr (OP == ACD_ABS) return m_abs(x);
  else if constexpr (OP == ACD_FLOOR) return m_floor(x);
  else if constexpr (OP == ACD_CEIL) return m_ceil(x);
  else if constexpr (OP == ACD_ROUND) return m_rint(x);
  else if constexpr (OP == ACD_ERF) return m_erf(x);
  else if constexpr (OP == ACD_TANH) return m_tanh(x);
  else if constexpr (OP == ACD_SIGMOID) {
    // sigmoid() is one R function: float32 is evaluated in double and rounded
    // once (as base R would); float64 keeps the reference formula's roundings
    if constexpr (std::is_same<T, float>::value)
      return (float)(1.0 / (1.0 + exp(-(double)x)));
    else
      return T(1) / (T(1) + m_exp(-x));
  }
  else if constexpr (OP == ACD_RELU) return m_max(x, T(0));
  else if constexpr (OP == ACD_SIN) return m_sin(x);
  else if constexpr (OP == ACD_COS) return m_cos(x);
  else if constexpr (OP == ACD_NEG) return T(-x);
  else if constexpr (OP == ACD_SQUARE) return T(x * x);
  else return x;  // ACD_COPY
}

template <int OP, typename T, typename O>
__device__ __forceinline__ O binary_apply(T a, T b) {
  if constexpr (std::is_same<T, __half>::value) return half_binary<OP, O>(a, b);
  else if constexpr (OP == ACD_ADD) return O(a + b);
  else if constexpr (OP == ACD_SUB) return O(a - b);
  else if constexpr (OP == ACD_MUL) return O(a * b);
  else if constexpr (OP == ACD_DIV) return O(a / b);
  else if constexpr (OP == ACD_MAX) return O(m_max(a, b));
  else if constexpr (OP == ACD_MIN) return O(m_min(a, b));
  else if constexpr (OP == ACD_POW) return O(m_pow(a, b));
  else if constexpr (OP == ACD_GT) return O(a > b ? 1 : 0);
  else if constexpr (OP == ACD_LT) return O(a < b ? 1 : 0);
  else if constexpr (OP == ACD_EQ) return O(a == b ? 1 : 0);
  else if constexpr (OP == ACD_NE) return O(a != b ? 1 : 0);
  else if constexpr (OP == ACD_GE) return O(a >= b ? 1 : 0);
  else if constexpr (OP == ACD_LE) return O(a <= b ? 1 : 0);
  else if constexpr (OP == ACD_RSUB) return O(b - a);
  else return O(b / a);  // ACD_RDIV
}

// ---- functor objects passed to the generic kernels ------------------------
template <int OP, typename T>
struct UnaryF {
  static constexpr int kIn = 1;
  using In = T;
  using Out = T;
  __device__ __forceinline__ T operator()(T x) const { return unary_apply<OP, T>(x); }
};

template <int OP, typename T, typename O>
struct BinaryF {
  static constexpr int kIn = 2;
  using In = T;
  using Out = O;
  __device__ __forceinline__ O operator()(T a, T b) const { return binary_apply<OP, T, O>(a, b); }
};

template <int OP, typename T, typename O>
struct ScalarF {
  static constexpr int kIn = 1;
  using In = T;
  using Out = O;
  T s;
  __device__ __forceinline__ O operator()(T a) const { return binary_apply<OP, T, O>(a, s); }
};

// x^2 with a scalar exponent of exactly 2 (R's `^` dispatches here).
template <typename T>
struct SquareScalarF {
  static constexpr int kIn = 1;
  using In = T;
  using Out = T;
  __device__ __forceinline__ T operator()(T a) const { return a * a; }
};

// ---- dtype conversion ------------------------------------------------------
// Base R's as.* rules on tensor storage: to an integer type a value is
// truncated toward zero, and NaN or a value outside the type's range becomes
// NA (INT32_MIN for int32, INT64_MIN for int64); an NA integer becomes NaN in
// a floating type; float <-> double and int64 -> float round to nearest;
// bool stores x != 0 (bool has no NA, so NaN and NA integers become 1).
// The two narrow types R lacks follow the reference's device casts:
// float16 is reached by one rounding to nearest from the exact source value
// (NA integers become NaN) and converts onward exactly through float32;
// int8 has no NA: from a floating value it truncates toward zero and
// saturates to [-128, 127] with NaN -> 0 (the device's float-to-int8 cast),
// from a wider integer it keeps the low 8 bits, and it widens exactly.
template <typename From, typename To>
__host__ __device__ __forceinline__ To convert_value(From x) {
  if constexpr (std::is_same<From, To>::value) {
    return x;
  } else if constexpr (std::is_same<From, __half>::value) {
    return convert_value<float, To>(__half2float(x));  // half -> float is exact
  } else if constexpr (std::is_same<To, __half>::value) {
    // double holds every float32, int32 and int8 value exactly (int64 beyond
    // 2^53 overflows half either way)
    return __double2half(convert_value<From, double>(x));
  } else if constexpr (std::is_same<To, int8_t>::value) {
    if constexpr (std::is_floating_point<From>::value) {
      if (x != x) return 0;
      if (x <= (From)-128) return -128;
      if (x >= (From)127) return 127;
      return (int8_t)x;
    } else {
      return (int8_t)x;
    }
  } else if constexpr (std::is_same<To, uint8_t>::value) {
    return (uint8_t)(x != From(0));
  } else if constexpr (std::is_floating_point<To>::value) {
    if constexpr (std::is_same<From, int32_t>::value)
      return x == INT32_MIN ? To(NAN) : (To)x;
    else if constexpr (std::is_same<From, int64_t>::value)
      return x == INT64_MIN ? To(NAN) : (To)x;
    else
      return (To)x;
  } else if constexpr (std::is_same<To, int32_t>::value) {
    if constexpr (std::is_floating_point<From>::value)
      return (x > (From)-2147483648.0 && x < (From)2147483648.0) ? (int32_t)x : INT32_MIN;
    else if constexpr (std::is_same<From, int64_t>::value)
      return (x >= -2147483647LL && x <= 2147483647LL) ? (int32_t)x : INT32_MIN;
    else
      return (int32_t)x;
  } else {
    if constexpr (std::is_floating_point<From>::value)
      return (x > (From)-9223372036854775808.0 && x < (From)9223372036854775808.0) ? (int64_t)x : INT64_MIN;
    else if constexpr (std::is_same<From, int32_t>::value)
      return x == INT32_MIN ? INT64_MIN : (int64_t)x;
    else
      return (int64_t)x;
  }
}

template <typename From, typename To>
struct ConvertF {
  static constexpr int kIn = 1;
  using In = From;
  using Out = To;
  __device__ __forceinline__ To operator()(From x) const { return convert_value<From, To>(x); }
};

// ---- fused chains ----------------------------------------------------------
// x*p + exp(-(x^2)): five R operators, five roundings.
template <typename T>
struct FusedScaleAddExpNegSquare {
  static constexpr int kIn = 1;
  using In = T;
  using Out = T;
  T p;
  __device__ __forceinline__ T operator()(T x) const {
    T a = x * p;
    T sq = x * x;
    T e = m_exp(-sq);
    return a + e;
  }
};

template <typename T>
struct FusedAddRelu {
  static constexpr int kIn = 2;
  using In = T;
  using Out = T;
  __device__ __forceinline__ T operator()(T a, T b) const { return m_max(a + b, T(0)); }
};

template <typename T>
struct FusedTanhScale {
  static constexpr int kIn = 1;
  using In = T;
  using Out = T;
  T p;
  __device__ __forceinline__ T operator()(T x) const { return m_tanh(x) * p; }
};

}  // namespace acd
