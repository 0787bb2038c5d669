// The acediaR launcher names (include/acediar_launchers.h) mapped onto the
// acd_* ABI.  Each entry point builds descriptors, runs on the legacy default
// stream of the current device through a per-device default context, and
// synchronises before returning, as the reference launchers do.
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/acediar_launchers.h"
#include "common.cuh"

namespace acd {

// The per-device context of the reference-named launchers (created on first
// use; also used by the contraction launchers in linalg.cu).
acd_ctx *shim_ctx() {
  static std::mutex mu;
  static acd_ctx *ctxs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) throw std::runtime_error("acediar: no CUDA device");
  std::lock_guard<std::mutex> lk(mu);
  if (!ctxs[dev]) {
    acd_ctx *c = nullptr;
    if (acd_ctx_create(dev, &c) != ACD_OK) throw std::runtime_error(std::string("acediar: ") + acd_last_error());
    ctxs[dev] = c;
  }
  return ctxs[dev];
}

static void shim_done(acd_status s, const char *fn) {
  if (s != ACD_OK) throw std::runtime_error(std::string(fn) + ": " + acd_last_error());
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) throw std::runtime_error(std::string(fn) + ": " + cudaGetErrorString(e));
}

static acd_desc flat(const void *p, int32_t dt, size_t n) {
  acd_desc d{};
  d.data = const_cast<void *>(p);
  d.ndim = 1;
  d.shape[0] = (int64_t)n;
  d.stride[0] = 1;
  d.dtype = dt;
  return d;
}

static acd_desc from_ref(const acd_ref_descriptor *r, int32_t dt) {
  if (!r) throw std::runtime_error("acediar: null descriptor");
  acd_desc d{};
  d.data = r->data;  // already the view's first element (see header)
  d.ndim = r->ndims;
  for (int k = 0; k < r->ndims && k < ACD_MAX_DIMS; ++k) {
    d.shape[k] = r->shape[k];
    d.stride[k] = r->strides[k];
  }
  d.dtype = dt;
  return d;
}

static acd_desc from_meta(const void *p, int32_t dt, const int *strides, const int *shape, int ndims) {
  acd_desc d{};
  d.data = const_cast<void *>(p);
  d.ndim = ndims;
  for (int k = 0; k < ndims && k < ACD_MAX_DIMS; ++k) {
    d.shape[k] = shape[k];
    d.stride[k] = strides[k];
  }
  d.dtype = dt;
  return d;
}

static acd_desc contiguous_of(const void *p, int32_t dt, const int *shape, int ndims) {
  acd_desc d{};
  d.data = const_cast<void *>(p);
  d.ndim = ndims;
  int64_t st = 1;
  for (int k = 0; k < ndims && k < ACD_MAX_DIMS; ++k) {
    d.shape[k] = shape[k];
    d.stride[k] = st;
    st *= shape[k];
  }
  d.dtype = dt;
  return d;
}

template <typename T> constexpr int32_t dt_of();
template <> constexpr int32_t dt_of<float>() { return ACD_FLOAT32; }
template <> constexpr int32_t dt_of<double>() { return ACD_FLOAT64; }
template <> constexpr int32_t dt_of<int32_t>() { return ACD_INT32; }
template <> constexpr int32_t dt_of<int64_t>() { return ACD_INT64; }
template <> constexpr int32_t dt_of<__half>() { return ACD_FLOAT16; }
template <> constexpr int32_t dt_of<int8_t>() { return ACD_INT8; }

static __half *hp(acd_half *p) { return reinterpret_cast<__half *>(p); }
static const __half *hp(const acd_half *p) { return reinterpret_cast<const __half *>(p); }

template <typename T>
static void bin(int op, T *r, const T *a, const T *b, size_t n, const char *fn) {
  if (n == 0) return;
  const acd_desc o = flat(r, dt_of<T>(), n), x = flat(a, dt_of<T>(), n), y = flat(b, dt_of<T>(), n);
  shim_done(acd_binary(shim_ctx(), op, &o, &x, &y, nullptr), fn);
}

template <typename T>
static void sca(int op, T *r, const T *a, double s, size_t n, const char *fn) {
  if (n == 0) return;
  const acd_desc o = flat(r, dt_of<T>(), n), x = flat(a, dt_of<T>(), n);
  shim_done(acd_scalar(shim_ctx(), op, &o, &x, s, nullptr), fn);
}

template <typename T>
static void una(int op, T *r, const T *a, size_t n, const char *fn) {
  if (n == 0) return;
  const acd_desc o = flat(r, dt_of<T>(), n), x = flat(a, dt_of<T>(), n);
  shim_done(acd_unary(shim_ctx(), op, &o, &x, nullptr), fn);
}

template <typename T>
static void bcast(int op, T *r, const T *a, const T *b, const int *as, const int *bs, const int *shape, int nd,
                  size_t total, const char *fn) {
  if (total == 0) return;
  const acd_desc o = contiguous_of(r, dt_of<T>(), shape, nd);
  const acd_desc x = from_meta(a, dt_of<T>(), as, shape, nd);
  const acd_desc y = from_meta(b, dt_of<T>(), bs, shape, nd);
  shim_done(acd_binary(shim_ctx(), op, &o, &x, &y, nullptr), fn);
}

template <typename T>
static T full_reduce(int op, const T *in, size_t n, const char *fn) {
  if (n == 0) return op == ACD_RED_PROD ? T(1) : T(0);
  acd_ctx *c = shim_ctx();
  double *d = &c->control->stats[4];  // one device double owned by the context
  const acd_desc x = flat(in, dt_of<T>(), n);
  acd_desc o = flat(d, ACD_FLOAT64, 1);
  acd_status s = acd_reduce(c, op, &o, &x, 1u, nullptr);
  double h = 0.0;
  cudaError_t e = cudaSuccess;
  if (s == ACD_OK) e = cudaMemcpy(&h, d, sizeof(double), cudaMemcpyDeviceToHost);
  if (s != ACD_OK) throw std::runtime_error(std::string(fn) + ": " + acd_last_error());
  if (e != cudaSuccess) throw std::runtime_error(std::string(fn) + ": " + cudaGetErrorString(e));
  return (T)h;
}

template <typename T>
static int64_t full_arg(int op, const T *in, size_t n, const char *fn) {
  if (!in || n == 0) throw std::runtime_error(std::string("Invalid input parameters for ") + fn);
  acd_ctx *c = shim_ctx();
  int64_t *d = reinterpret_cast<int64_t *>(&c->control->stats[5]);
  const acd_desc x = flat(in, dt_of<T>(), n);
  acd_desc o = flat(d, ACD_INT64, 1);
  acd_status s = acd_arg_reduce(c, op, &o, nullptr, &x, -1, 1, nullptr);
  int64_t h = 0;
  cudaError_t e = cudaSuccess;
  if (s == ACD_OK) e = cudaMemcpy(&h, d, sizeof(int64_t), cudaMemcpyDeviceToHost);
  if (s != ACD_OK) throw std::runtime_error(std::string(fn) + ": " + acd_last_error());
  if (e != cudaSuccess) throw std::runtime_error(std::string(fn) + ": " + cudaGetErrorString(e));
  return h;
}

// Axis launchers receive shape/strides/axes as device arrays.
static void fetch_meta(const int *d_strides, const int *d_shape, const int *d_axes, int n_axes, int ndims,
                       std::vector<int> &st, std::vector<int> &sh, std::vector<int> &ax, const char *fn) {
  if (ndims <= 0 || ndims > ACD_MAX_DIMS || n_axes <= 0 || n_axes > ndims || !d_strides || !d_shape || !d_axes)
    throw std::runtime_error(std::string("Null pointer or bad rank passed to ") + fn);
  st.resize(ndims);
  sh.resize(ndims);
  ax.resize(n_axes);
  if (cudaMemcpy(st.data(), d_strides, sizeof(int) * ndims, cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemcpy(sh.data(), d_shape, sizeof(int) * ndims, cudaMemcpyDeviceToHost) != cudaSuccess ||
      cudaMemcpy(ax.data(), d_axes, sizeof(int) * n_axes, cudaMemcpyDeviceToHost) != cudaSuccess)
    throw std::runtime_error(std::string(fn) + ": cannot read axis metadata");
}

template <typename T>
static void axis_reduce(int op, T *r, const T *in, const int *d_st, const int *d_sh, const int *d_ax, int n_axes,
                        int ndims, size_t out_size, const char *fn) {
  if (!r || !in) throw std::runtime_error(std::string("Null pointer passed to ") + fn);
  if (out_size == 0) throw std::runtime_error(std::string("Zero output size in ") + fn);
  std::vector<int> st, sh, ax;
  fetch_meta(d_st, d_sh, d_ax, n_axes, ndims, st, sh, ax, fn);
  uint32_t mask = 0;
  for (int a : ax) {
    if (a < 0 || a >= ndims) throw std::runtime_error(std::string(fn) + ": axis out of range");
    mask |= 1u << a;
  }
  const acd_desc x = from_meta(in, dt_of<T>(), st.data(), sh.data(), ndims);
  const acd_desc o = flat(r, dt_of<T>(), out_size);
  shim_done(acd_reduce(shim_ctx(), op, &o, &x, mask, nullptr), fn);
}

template <typename T>
static void axis_arg(int op, int64_t *idx, const T *in, const int *d_st, const int *d_sh, const int *d_ax,
                     int n_axes, int ndims, size_t out_elems, const char *fn) {
  if (!idx || !in) throw std::runtime_error(std::string("Null pointer passed to ") + fn);
  if (out_elems == 0) throw std::runtime_error(std::string("Zero output size in ") + fn);
  std::vector<int> st, sh, ax;
  fetch_meta(d_st, d_sh, d_ax, n_axes, ndims, st, sh, ax, fn);
  if (n_axes != 1) throw std::runtime_error(std::string(fn) + ": exactly one axis expected");
  const acd_desc x = from_meta(in, dt_of<T>(), st.data(), sh.data(), ndims);
  const acd_desc o = flat(idx, ACD_INT64, out_elems);
  shim_done(acd_arg_reduce(shim_ctx(), op, &o, nullptr, &x, ax[0], 0, nullptr), fn);
}

template <typename T>
static void strided_bin(int op, const acd_ref_descriptor *out, const acd_ref_descriptor *a,
                        const acd_ref_descriptor *b, const char *fn) {
  const acd_desc o = from_ref(out, dt_of<T>()), x = from_ref(a, dt_of<T>()), y = from_ref(b, dt_of<T>());
  shim_done(acd_binary(shim_ctx(), op, &o, &x, &y, nullptr), fn);
}

template <typename T>
static void strided_un(int op, const acd_ref_descriptor *out, const acd_ref_descriptor *in, const char *fn) {
  const acd_desc o = from_ref(out, dt_of<T>()), x = from_ref(in, dt_of<T>());
  shim_done(acd_unary(shim_ctx(), op, &o, &x, nullptr), fn);
}

template <typename T>
static void strided_sc(int op, const acd_ref_descriptor *out, const acd_ref_descriptor *in, double s,
                       const char *fn) {
  const acd_desc o = from_ref(out, dt_of<T>()), x = from_ref(in, dt_of<T>());
  shim_done(acd_scalar(shim_ctx(), op, &o, &x, s, nullptr), fn);
}

}  // namespace acd

using namespace acd;

extern "C" {

#define ACD_BIN(NAME, OP)                                                                       \
  void tensor_##NAME##_float32(float *r, const float *a, const float *b, size_t n) {            \
    bin<float>(OP, r, a, b, n, "tensor_" #NAME "_float32");                                     \
  }                                                                                             \
  void tensor_##NAME##_float64(double *r, const double *a, const double *b, size_t n) {         \
    bin<double>(OP, r, a, b, n, "tensor_" #NAME "_float64");                                    \
  }
ACD_BIN(add, ACD_ADD)
ACD_BIN(sub, ACD_SUB)
ACD_BIN(mul, ACD_MUL)
ACD_BIN(div, ACD_DIV)
ACD_BIN(gt, ACD_GT)
ACD_BIN(lt, ACD_LT)
ACD_BIN(eq, ACD_EQ)
ACD_BIN(max_elemwise, ACD_MAX)
ACD_BIN(min_elemwise, ACD_MIN)
ACD_BIN(pow_elemwise, ACD_POW)
#undef ACD_BIN

void tensor_add_int32(int32_t *r, const int32_t *a, const int32_t *b, size_t n) {
  bin<int32_t>(ACD_ADD, r, a, b, n, "tensor_add_int32");
}
void tensor_add_int64(int64_t *r, const int64_t *a, const int64_t *b, size_t n) {
  bin<int64_t>(ACD_ADD, r, a, b, n, "tensor_add_int64");
}

#define ACD_SCA(NAME, OP)                                                                      \
  void tensor_##NAME##_float32(float *r, const float *x, float s, size_t n) {                  \
    sca<float>(OP, r, x, (double)s, n, "tensor_" #NAME "_float32");                            \
  }                                                                                            \
  void tensor_##NAME##_float64(double *r, const double *x, double s, size_t n) {               \
    sca<double>(OP, r, x, s, n, "tensor_" #NAME "_float64");                                   \
  }
ACD_SCA(scalar_add, ACD_ADD)
ACD_SCA(scalar_mul, ACD_MUL)
ACD_SCA(scalar_sub, ACD_SUB)
ACD_SCA(scalar_div, ACD_DIV)
ACD_SCA(pow_scalar, ACD_POW)
#undef ACD_SCA

#define ACD_UN(NAME, OP)                                                                       \
  void tensor_##NAME##_float32(float *r, const float *x, size_t n) {                           \
    una<float>(OP, r, x, n, "tensor_" #NAME "_float32");                                       \
  }                                                                                            \
  void tensor_##NAME##_float64(double *r, const double *x, size_t n) {                         \
    una<double>(OP, r, x, n, "tensor_" #NAME "_float64");                                      \
  }
ACD_UN(exp, ACD_EXP)
ACD_UN(log, ACD_LOG)
ACD_UN(sqrt, ACD_SQRT)
ACD_UN(abs, ACD_ABS)
ACD_UN(tanh, ACD_TANH)
ACD_UN(sigmoid, ACD_SIGMOID)
ACD_UN(relu, ACD_RELU)
ACD_UN(sin, ACD_SIN)
ACD_UN(cos, ACD_COS)
ACD_UN(floor, ACD_FLOOR)
ACD_UN(ceil, ACD_CEIL)
ACD_UN(round, ACD_ROUND)
ACD_UN(erf, ACD_ERF)
#undef ACD_UN

#define ACD_BC(NAME, OP)                                                                                        \
  void tensor_##NAME##_broadcast_float32(float *r, const float *a, const float *b, const int *as, const int *bs, \
                                         const int *rs, const int *shape, int nd, size_t total) {               \
    (void)rs;                                                                                                   \
    bcast<float>(OP, r, a, b, as, bs, shape, nd, total, "tensor_" #NAME "_broadcast_float32");                 \
  }                                                                                                             \
  void tensor_##NAME##_broadcast_float64(double *r, const double *a, const double *b, const int *as,            \
                                         const int *bs, const int *rs, const int *shape, int nd, size_t total) { \
    (void)rs;                                                                                                   \
    bcast<double>(OP, r, a, b, as, bs, shape, nd, total, "tensor_" #NAME "_broadcast_float64");                \
  }
ACD_BC(add, ACD_ADD)
ACD_BC(sub, ACD_SUB)
ACD_BC(mul, ACD_MUL)
ACD_BC(div, ACD_DIV)
ACD_BC(max, ACD_MAX)
ACD_BC(min, ACD_MIN)
ACD_BC(pow, ACD_POW)
ACD_BC(gt, ACD_GT)
ACD_BC(lt, ACD_LT)
ACD_BC(eq, ACD_EQ)
#undef ACD_BC

#define ACD_SB(NAME, OP)                                                                                 \
  void tensor_##NAME##_strided_float32(const acd_ref_descriptor *o, const acd_ref_descriptor *a,        \
                                       const acd_ref_descriptor *b) {                                   \
    strided_bin<float>(OP, o, a, b, "tensor_" #NAME "_strided_float32");                                \
  }                                                                                                      \
  void tensor_##NAME##_strided_float64(const acd_ref_descriptor *o, const acd_ref_descriptor *a,        \
                                       const acd_ref_descriptor *b) {                                   \
    strided_bin<double>(OP, o, a, b, "tensor_" #NAME "_strided_float64");                               \
  }
ACD_SB(add, ACD_ADD)
ACD_SB(sub, ACD_SUB)
ACD_SB(mul, ACD_MUL)
ACD_SB(div, ACD_DIV)
ACD_SB(max_elemwise, ACD_MAX)
ACD_SB(min_elemwise, ACD_MIN)
ACD_SB(pow_elemwise, ACD_POW)
#undef ACD_SB

#define ACD_SU(NAME, OP)                                                                                 \
  void tensor_##NAME##_strided_float32(const acd_ref_descriptor *o, const acd_ref_descriptor *x) {      \
    strided_un<float>(OP, o, x, "tensor_" #NAME "_strided_float32");                                    \
  }                                                                                                      \
  void tensor_##NAME##_strided_float64(const acd_ref_descriptor *o, const acd_ref_descriptor *x) {      \
    strided_un<double>(OP, o, x, "tensor_" #NAME "_strided_float64");                                   \
  }
ACD_SU(exp, ACD_EXP)
ACD_SU(log, ACD_LOG)
ACD_SU(sqrt, ACD_SQRT)
ACD_SU(floor, ACD_FLOOR)
ACD_SU(ceil, ACD_CEIL)
ACD_SU(round, ACD_ROUND)
ACD_SU(erf, ACD_ERF)
#undef ACD_SU

#define ACD_SS(NAME, OP)                                                                                   \
  void tensor_##NAME##_strided_float32(const acd_ref_descriptor *o, const acd_ref_descriptor *x, float s) { \
    strided_sc<float>(OP, o, x, (double)s, "tensor_" #NAME "_strided_float32");                           \
  }                                                                                                        \
  void tensor_##NAME##_strided_float64(const acd_ref_descriptor *o, const acd_ref_descriptor *x,          \
                                       double s) {                                                        \
    strided_sc<double>(OP, o, x, s, "tensor_" #NAME "_strided_float64");                                  \
  }
ACD_SS(scalar_add, ACD_ADD)
ACD_SS(scalar_mul, ACD_MUL)
ACD_SS(scalar_sub, ACD_SUB)
ACD_SS(scalar_div, ACD_DIV)
ACD_SS(pow_scalar, ACD_POW)
#undef ACD_SS

void tensor_strided_copy_float32(float *dest, const float *src, const int *strides, const int *shape, int ndims,
                                 size_t total) {
  if (total == 0) return;
  const acd_desc o = contiguous_of(dest, ACD_FLOAT32, shape, ndims);
  const acd_desc x = from_meta(src, ACD_FLOAT32, strides, shape, ndims);
  shim_done(acd_copy(shim_ctx(), &o, &x, nullptr), "tensor_strided_copy_float32");
}
void tensor_strided_copy_float64(double *dest, const double *src, const int *strides, const int *shape, int ndims,
                                 size_t total) {
  if (total == 0) return;
  const acd_desc o = contiguous_of(dest, ACD_FLOAT64, shape, ndims);
  const acd_desc x = from_meta(src, ACD_FLOAT64, strides, shape, ndims);
  shim_done(acd_copy(shim_ctx(), &o, &x, nullptr), "tensor_strided_copy_float64");
}

// ---- float16 and int8: src/kernels/tensor_ops.cu:1053-1117, 1368-1392 ----
#define ACD_BIN16(NAME, OP)                                                                     \
  void tensor_##NAME##_float16(acd_half *r, const acd_half *a, const acd_half *b, size_t n) {   \
    bin<__half>(OP, hp(r), hp(a), hp(b), n, "tensor_" #NAME "_float16");                        \
  }                                                                                             \
  void tensor_##NAME##_strided_float16(const acd_ref_descriptor *o, const acd_ref_descriptor *a, \
                                       const acd_ref_descriptor *b) {                           \
    strided_bin<__half>(OP, o, a, b, "tensor_" #NAME "_strided_float16");                       \
  }
ACD_BIN16(add, ACD_ADD)
ACD_BIN16(sub, ACD_SUB)
ACD_BIN16(mul, ACD_MUL)
ACD_BIN16(div, ACD_DIV)
#undef ACD_BIN16

// the scalar arrives as float and rounds once to half, as the reference's
// convert_type<half>(float) does (src/kernels/tensor_kernels.cu:33-39)
void tensor_scalar_add_float16(acd_half *r, const acd_half *x, float s, size_t n) {
  sca<__half>(ACD_ADD, hp(r), hp(x), (double)s, n, "tensor_scalar_add_float16");
}
void tensor_scalar_mul_float16(acd_half *r, const acd_half *x, float s, size_t n) {
  sca<__half>(ACD_MUL, hp(r), hp(x), (double)s, n, "tensor_scalar_mul_float16");
}
void tensor_add_int8(int8_t *r, const int8_t *a, const int8_t *b, size_t n) {
  bin<int8_t>(ACD_ADD, r, a, b, n, "tensor_add_int8");
}
void tensor_add_strided_int8(const acd_ref_descriptor *o, const acd_ref_descriptor *a, const acd_ref_descriptor *b) {
  strided_bin<int8_t>(ACD_ADD, o, a, b, "tensor_add_strided_int8");
}

// The reference's float16 and int64 sums are placeholders that return 0
// (src/kernels/tensor_ops.cu:701-710); these compute the sums.
float tensor_sum_float16(const acd_half *in, size_t n) {
  if (n == 0) return 0.0f;
  acd_ctx *c = shim_ctx();
  double *d = &c->control->stats[4];
  const acd_desc x = flat(hp(in), ACD_FLOAT16, n);
  const acd_desc o = flat(d, ACD_FLOAT64, 1);
  acd_status st = acd_reduce(c, ACD_RED_SUM, &o, &x, 1u, nullptr);
  double h = 0.0;
  if (st != ACD_OK) throw std::runtime_error(std::string("tensor_sum_float16: ") + acd_last_error());
  const cudaError_t e = cudaMemcpy(&h, d, sizeof(double), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) throw std::runtime_error(std::string("tensor_sum_float16: ") + cudaGetErrorString(e));
  return (float)h;
}
int64_t tensor_sum_int64(const int64_t *in, size_t n) {
  if (n == 0) return 0;
  acd_ctx *c = shim_ctx();
  int64_t *d = reinterpret_cast<int64_t *>(&c->control->stats[5]);
  const acd_desc x = flat(in, ACD_INT64, n);
  const acd_desc o = flat(d, ACD_INT64, 1);
  acd_status st = acd_reduce(c, ACD_RED_SUM, &o, &x, 1u, nullptr);
  int64_t h = 0;
  if (st != ACD_OK) throw std::runtime_error(std::string("tensor_sum_int64: ") + acd_last_error());
  const cudaError_t e = cudaMemcpy(&h, d, sizeof(int64_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) throw std::runtime_error(std::string("tensor_sum_int64: ") + cudaGetErrorString(e));
  return h;  // exact modulo 2^64, as the int64 accumulator wraps
}

float tensor_sum_float32(const float *in, size_t n) { return full_reduce<float>(ACD_RED_SUM, in, n, "tensor_sum_float32"); }
double tensor_sum_float64(const double *in, size_t n) { return full_reduce<double>(ACD_RED_SUM, in, n, "tensor_sum_float64"); }
float tensor_max_float32(const float *in, size_t n) { return full_reduce<float>(ACD_RED_MAX, in, n, "tensor_max_float32"); }
double tensor_max_float64(const double *in, size_t n) { return full_reduce<double>(ACD_RED_MAX, in, n, "tensor_max_float64"); }
float tensor_min_float32(const float *in, size_t n) { return full_reduce<float>(ACD_RED_MIN, in, n, "tensor_min_float32"); }
double tensor_min_float64(const double *in, size_t n) { return full_reduce<double>(ACD_RED_MIN, in, n, "tensor_min_float64"); }
float tensor_prod_float32(const float *in, size_t n) { return full_reduce<float>(ACD_RED_PROD, in, n, "tensor_prod_float32"); }
double tensor_prod_float64(const double *in, size_t n) { return full_reduce<double>(ACD_RED_PROD, in, n, "tensor_prod_float64"); }
double tensor_var_float32(const float *in, size_t n) {
  if (n <= 1) return 0.0;  // the reference returns 0 for n <= 1 (src/kernels/tensor_ops.cu:786)
  return (double)full_reduce<float>(ACD_RED_VAR, in, n, "tensor_var_float32");
}
double tensor_var_float64(const double *in, size_t n) {
  if (n <= 1) return 0.0;
  return full_reduce<double>(ACD_RED_VAR, in, n, "tensor_var_float64");
}
int64_t tensor_argmax_float32(const float *in, size_t n) { return full_arg<float>(ACD_ARGMAX, in, n, "tensor_argmax_float32"); }
int64_t tensor_argmax_float64(const double *in, size_t n) { return full_arg<double>(ACD_ARGMAX, in, n, "tensor_argmax_float64"); }
int64_t tensor_argmin_float32(const float *in, size_t n) { return full_arg<float>(ACD_ARGMIN, in, n, "tensor_argmin_float32"); }
int64_t tensor_argmin_float64(const double *in, size_t n) { return full_arg<double>(ACD_ARGMIN, in, n, "tensor_argmin_float64"); }

#define ACD_AX(NAME, OP)                                                                                       \
  void tensor_axis_##NAME##_float32(float *r, const float *in, const int *st, const int *sh, const int *rs,    \
                                    const int *ax, int na, int nd, size_t os) {                               \
    (void)rs;                                                                                                 \
    axis_reduce<float>(OP, r, in, st, sh, ax, na, nd, os, "tensor_axis_" #NAME "_float32");                   \
  }                                                                                                           \
  void tensor_axis_##NAME##_float64(double *r, const double *in, const int *st, const int *sh, const int *rs, \
                                    const int *ax, int na, int nd, size_t os) {                               \
    (void)rs;                                                                                                 \
    axis_reduce<double>(OP, r, in, st, sh, ax, na, nd, os, "tensor_axis_" #NAME "_float64");                  \
  }
ACD_AX(sum, ACD_RED_SUM)
ACD_AX(mean, ACD_RED_MEAN)
ACD_AX(max, ACD_RED_MAX)
ACD_AX(min, ACD_RED_MIN)
ACD_AX(prod, ACD_RED_PROD)
ACD_AX(var, ACD_RED_VAR)
#undef ACD_AX

void tensor_axis_argmax_float32(int64_t *idx, const float *in, const int *st, const int *sh, const int *os,
                                const int *ax, int na, int nd, size_t oe) {
  (void)os;
  axis_arg<float>(ACD_ARGMAX, idx, in, st, sh, ax, na, nd, oe, "tensor_axis_argmax_float32");
}
void tensor_axis_argmax_float64(int64_t *idx, const double *in, const int *st, const int *sh, const int *os,
                                const int *ax, int na, int nd, size_t oe) {
  (void)os;
  axis_arg<double>(ACD_ARGMAX, idx, in, st, sh, ax, na, nd, oe, "tensor_axis_argmax_float64");
}
void tensor_axis_argmin_float32(int64_t *idx, const float *in, const int *st, const int *sh, const int *os,
                                const int *ax, int na, int nd, size_t oe) {
  (void)os;
  axis_arg<float>(ACD_ARGMIN, idx, in, st, sh, ax, na, nd, oe, "tensor_axis_argmin_float32");
}
void tensor_axis_argmin_float64(int64_t *idx, const double *in, const int *st, const int *sh, const int *os,
                                const int *ax, int na, int nd, size_t oe) {
  (void)os;
  axis_arg<double>(ACD_ARGMIN, idx, in, st, sh, ax, na, nd, oe, "tensor_axis_argmin_float64");
}

// ---- slice and mask assignment, concat / stack / repeat / pad ----------------
#define ACD_SLICE_SCALAR(NAME, T, DT, BODY)                                                                  \
  void NAME(T *data, double scalar, const int *start, const int *slice_shape, const int *strides, int ndims,  \
            size_t total) {                                                                                   \
    if (total == 0) return;                                                                                   \
    acd_desc v = from_meta(data, DT, strides, slice_shape, ndims);                                            \
    for (int k = 0; k < ndims; ++k) v.offset += (int64_t)start[k] * strides[k];                                \
    BODY;                                                                                                     \
  }
ACD_SLICE_SCALAR(tensor_slice_set_scalar_float32, float, ACD_FLOAT32,
                 shim_done(acd_fill(shim_ctx(), &v, scalar, nullptr), "tensor_slice_set_scalar_float32"))
ACD_SLICE_SCALAR(tensor_slice_set_scalar_float64, double, ACD_FLOAT64,
                 shim_done(acd_fill(shim_ctx(), &v, scalar, nullptr), "tensor_slice_set_scalar_float64"))
ACD_SLICE_SCALAR(tensor_slice_add_scalar_float32, float, ACD_FLOAT32,
                 shim_done(acd_scalar(shim_ctx(), ACD_ADD, &v, &v, scalar, nullptr),
                           "tensor_slice_add_scalar_float32"))
ACD_SLICE_SCALAR(tensor_slice_add_scalar_float64, double, ACD_FLOAT64,
                 shim_done(acd_scalar(shim_ctx(), ACD_ADD, &v, &v, scalar, nullptr),
                           "tensor_slice_add_scalar_float64"))
#undef ACD_SLICE_SCALAR

#define ACD_SLICE_TENSOR(NAME, T, DT)                                                                          \
  void NAME(T *dest, const T *src, const int *start, const int *slice_shape, const int *dest_strides,          \
            const int *src_strides, int ndims, size_t total) {                                                 \
    if (total == 0) return;                                                                                     \
    acd_desc o = from_meta(dest, DT, dest_strides, slice_shape, ndims);                                         \
    for (int k = 0; k < ndims; ++k) o.offset += (int64_t)start[k] * dest_strides[k];                             \
    const acd_desc x = from_meta(src, DT, src_strides, slice_shape, ndims);                                     \
    shim_done(acd_copy(shim_ctx(), &o, &x, nullptr), #NAME);                                                    \
  }
ACD_SLICE_TENSOR(tensor_slice_set_tensor_float32, float, ACD_FLOAT32)
ACD_SLICE_TENSOR(tensor_slice_set_tensor_float64, double, ACD_FLOAT64)
#undef ACD_SLICE_TENSOR

void tensor_mask_set_scalar_float32(float *data, const unsigned char *mask, float value, size_t n) {
  if (n == 0) return;
  const acd_desc x = flat(data, ACD_FLOAT32, n), m = flat(mask, ACD_BOOL, n);
  shim_done(acd_mask_fill(shim_ctx(), &x, &m, value, nullptr), "tensor_mask_set_scalar_float32");
}
void tensor_mask_set_scalar_float64(double *data, const unsigned char *mask, double value, size_t n) {
  if (n == 0) return;
  const acd_desc x = flat(data, ACD_FLOAT64, n), m = flat(mask, ACD_BOOL, n);
  shim_done(acd_mask_fill(shim_ctx(), &x, &m, value, nullptr), "tensor_mask_set_scalar_float64");
}

#define ACD_CONCAT(NAME, T, DT)                                                                                \
  void NAME(T *result, const T **inputs, const int *input_sizes, int num, const int *result_strides,            \
            const int *input_strides_list, const int *shape, int ndims, int axis, size_t total) {               \
    if (total == 0) return;                                                                                     \
    const acd_desc o = from_meta(result, DT, result_strides, shape, ndims);                                     \
    std::vector<acd_desc> in(num);                                                                              \
    std::vector<const acd_desc *> ptr(num);                                                                     \
    for (int t = 0; t < num; ++t) {                                                                             \
      std::vector<int> sh(shape, shape + ndims);                                                                \
      sh[axis] = input_sizes[t];                                                                                \
      in[t] = from_meta(inputs[t], DT, input_strides_list + (size_t)t * ndims, sh.data(), ndims);               \
      ptr[t] = &in[t];                                                                                          \
    }                                                                                                           \
    shim_done(acd_concat(shim_ctx(), &o, ptr.data(), num, axis, nullptr), #NAME);                               \
  }
ACD_CONCAT(launch_concat_float32, float, ACD_FLOAT32)
ACD_CONCAT(launch_concat_float64, double, ACD_FLOAT64)
#undef ACD_CONCAT

#define ACD_STACK(NAME, T, DT)                                                                                 \
  void NAME(T *result, const T **inputs, int num, const int *input_strides, const int *result_shape, int ndims,  \
            int axis, size_t total) {                                                                           \
    if (total == 0) return;                                                                                     \
    const acd_desc o = contiguous_of(result, DT, result_shape, ndims);                                          \
    std::vector<int> sh;                                                                                        \
    for (int d = 0; d < ndims; ++d)                                                                             \
      if (d != axis) sh.push_back(result_shape[d]);                                                             \
    std::vector<acd_desc> in(num);                                                                              \
    std::vector<const acd_desc *> ptr(num);                                                                     \
    for (int t = 0; t < num; ++t) {                                                                             \
      in[t] = from_meta(inputs[t], DT, input_strides, sh.data(), ndims - 1);                                    \
      ptr[t] = &in[t];                                                                                          \
    }                                                                                                           \
    shim_done(acd_stack(shim_ctx(), &o, ptr.data(), num, axis, nullptr), #NAME);                                \
  }
ACD_STACK(launch_stack_float32, float, ACD_FLOAT32)
ACD_STACK(launch_stack_float64, double, ACD_FLOAT64)
#undef ACD_STACK

#define ACD_REPEAT(NAME, T, DT)                                                                                \
  void NAME(T *result, const T *input, const int *input_strides, const int *reps, const int *input_shape,       \
            const int *result_shape, int ndims, size_t total) {                                                 \
    if (total == 0) return;                                                                                     \
    const acd_desc o = contiguous_of(result, DT, result_shape, ndims);                                          \
    const acd_desc x = from_meta(input, DT, input_strides, input_shape, ndims);                                 \
    int64_t r[ACD_MAX_DIMS];                                                                                    \
    for (int d = 0; d < ndims && d < ACD_MAX_DIMS; ++d) r[d] = reps[d];                                         \
    shim_done(acd_repeat(shim_ctx(), &o, &x, r, nullptr), #NAME);                                               \
  }
ACD_REPEAT(launch_repeat_float32, float, ACD_FLOAT32)
ACD_REPEAT(launch_repeat_float64, double, ACD_FLOAT64)
#undef ACD_REPEAT

#define ACD_PAD(NAME, T, DT)                                                                                   \
  void NAME(T *result, const T *input, const int *input_strides, const int *input_shape, const int *pad_before,  \
            const int *pad_after, const int *result_shape, int ndims, T pad_value, int pad_mode, size_t total) {   \
    (void)pad_after;                                                                                            \
    if (total == 0) return;                                                                                     \
    const acd_desc o = contiguous_of(result, DT, result_shape, ndims);                                          \
    const acd_desc x = from_meta(input, DT, input_strides, input_shape, ndims);                                 \
    int64_t b[ACD_MAX_DIMS];                                                                                    \
    for (int d = 0; d < ndims && d < ACD_MAX_DIMS; ++d) b[d] = pad_before[d];                                   \
    shim_done(acd_pad(shim_ctx(), &o, &x, b, pad_mode, (double)pad_value, nullptr), #NAME);                     \
  }
ACD_PAD(launch_pad_float32, float, ACD_FLOAT32)
ACD_PAD(launch_pad_float64, double, ACD_FLOAT64)
#undef ACD_PAD

void tensor_softmax_float32(float *out, const float *in, size_t n) {
  if (n == 0) return;
  const acd_desc o = flat(out, ACD_FLOAT32, n), x = flat(in, ACD_FLOAT32, n);
  shim_done(acd_softmax(shim_ctx(), &o, &x, -1, nullptr), "tensor_softmax_float32");
}
void tensor_softmax_float64(double *out, const double *in, size_t n) {
  if (n == 0) return;
  const acd_desc o = flat(out, ACD_FLOAT64, n), x = flat(in, ACD_FLOAT64, n);
  shim_done(acd_softmax(shim_ctx(), &o, &x, -1, nullptr), "tensor_softmax_float64");
}

}  // extern "C"
