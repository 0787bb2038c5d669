// TensorAcd.cpp — acediaR's Rcpp entry points over the B200 library's C ABI
// (include/acd.h) for the operations the reference lacks, computes on the
// host, or leaves as stubs.  It is added to acediaR's src/ next to the
// reference's own Tensor*.cpp modules and builds against the reference's
// gpuTensor.h / TensorRegistry.h (tensor objects, dtype dispatch) and this
// repository's include/acd.h; rglue/Makevars links libacediar_b200.so.
//
// Entry points (R name -> C ABI call):
//   tensor_softmax_axis_unified(x, axis)        acd_softmax along a 0-based axis
//   tensor_cumsum_axis_unified(x, axis)         acd_scan ACD_CUMSUM (axis < 0: flattened)
//   tensor_cumprod_axis_unified(x, axis)        acd_scan ACD_CUMPROD
//   tensor_argmax_axis(x, axis, keep_dims)      acd_arg_reduce, 0-based int64 indices
//   tensor_argmin_axis(x, axis, keep_dims)        (replace the stubs at
//                                                 src/TensorReduction.cpp:390-398)
//   tensor_var_axis(x, axis, keep_dims)         acd_reduce ACD_RED_VAR (replaces
//                                                 src/TensorReduction.cpp's version,
//                                                 whose kernel writes zeros)
//   tensor_compare_bool_unified(a, b, op)       acd_binary GT..LE with a bool output
//   tensor_to_dtype_unified(x, dtype)           acd_convert (replaces
//                                                 src/TensorDataAccess.cpp:152-190)
//   rand_tensor / rnorm_tensor                  acd_rand (replace src/TensorRandom.cpp:42-224)
//   set_random_seed(seed)                       the (seed, position) of acd_rand's stream
//
// Errors become R errors through stop() with the reference's message
// prefixes ("Error in unified tensor <op>: ...").  Every call runs on the
// legacy default stream of the current device and synchronises before
// returning, as the reference's entry points do.
//
// Verification: R and Rcpp are absent from the build image, so this file has
// not been compiled; the C ABI calls it makes are the ones the repository's
// ctypes mirror (acedia-r_b200/acediar/tensor.py) makes and tests.
#include <Rcpp.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "TensorRegistry.h"
#include "gpuTensor.h"
#include "acd.h"

using namespace Rcpp;

namespace {

acd_ctx *acd_default_ctx() {
  static acd_ctx *ctxs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) stop("acediaR: no CUDA device");
  if (!ctxs[dev] && acd_ctx_create(dev, &ctxs[dev]) != ACD_OK) stop(std::string("acediaR: ") + acd_last_error());
  return ctxs[dev];
}

template <typename T> int32_t acd_dtype_of();
template <> int32_t acd_dtype_of<float>() { return ACD_FLOAT32; }
template <> int32_t acd_dtype_of<double>() { return ACD_FLOAT64; }
template <> int32_t acd_dtype_of<int>() { return ACD_INT32; }
template <> int32_t acd_dtype_of<int64_t>() { return ACD_INT64; }
template <> int32_t acd_dtype_of<bool>() { return ACD_BOOL; }
template <> int32_t acd_dtype_of<half>() { return ACD_FLOAT16; }
template <> int32_t acd_dtype_of<int8_t>() { return ACD_INT8; }

// gpuTensor::data() already points at the view's first element (the offset
// is applied), so the descriptor's offset is 0.
template <typename T>
acd_desc to_acd(const gpuTensor<T> &t) {
  acd_desc d{};
  d.data = const_cast<T *>(t.data());
  d.offset = 0;
  d.ndim = (int32_t)t.ndims();
  d.dtype = acd_dtype_of<T>();
  for (int k = 0; k < d.ndim; ++k) {
    d.shape[k] = (int64_t)t.shape()[k];
    d.stride[k] = (int64_t)t.strides()[k];
  }
  return d;
}

void acd_done(acd_status st, const std::string &what) {
  if (st != ACD_OK) stop("Error in unified tensor " + what + ": " + acd_last_error());
  const cudaError_t e = cudaStreamSynchronize(nullptr);
  if (e != cudaSuccess) stop("Error in unified tensor " + what + ": " + cudaGetErrorString(e));
}

SEXP wrap_tensor(std::unique_ptr<TensorBase> t) {
  const DType dt = t->dtype();
  XPtr<TensorBase> ptr(t.release(), true);
  ptr.attr("class") = "gpuTensor";
  ptr.attr("dtype") = dtype_to_string(dt);
  return ptr;
}

template <typename T>
const gpuTensor<T> &tensor_of(const XPtr<TensorBase> &x) {
  auto tw = dynamic_cast<const TensorWrapper<T> *>(x.get());
  if (!tw) stop("Invalid tensor wrapper");
  return tw->tensor();
}

// Calls f.template run<T>() for the tensor's element type.
template <class F>
SEXP dispatch_real(const XPtr<TensorBase> &x, F &&f, const char *what) {
  switch (x->dtype()) {
    case DType::FLOAT32: return f.template run<float>(tensor_of<float>(x));
    case DType::FLOAT64: return f.template run<double>(tensor_of<double>(x));
    default: stop(std::string(what) + " currently supports float/double tensors only");
  }
  return R_NilValue;
}

template <class F>
SEXP dispatch_any(const XPtr<TensorBase> &x, F &&f, const char *what) {
  switch (x->dtype()) {
    case DType::FLOAT32: return f.template run<float>(tensor_of<float>(x));
    case DType::FLOAT64: return f.template run<double>(tensor_of<double>(x));
    case DType::INT32: return f.template run<int>(tensor_of<int>(x));
    case DType::INT64: return f.template run<int64_t>(tensor_of<int64_t>(x));
    case DType::FLOAT16: return f.template run<half>(tensor_of<half>(x));
    case DType::INT8: return f.template run<int8_t>(tensor_of<int8_t>(x));
    case DType::BOOL: return f.template run<bool>(tensor_of<bool>(x));
    default: stop(std::string(what) + ": unsupported dtype " + dtype_to_string(x->dtype()));
  }
  return R_NilValue;
}

Shape kept_shape(const Shape &in, const std::vector<int> &axes0, bool keep_dims) {
  std::vector<size_t> dims;
  for (size_t d = 0; d < in.ndims(); ++d) {
    bool reduced = false;
    for (int a : axes0) reduced = reduced || (a == (int)d);
    if (!reduced)
      dims.push_back(in[d]);
    else if (keep_dims)
      dims.push_back(1);
  }
  if (dims.empty()) dims.push_back(1);  // all axes reduced: shape [1] (src/TensorRegistry.h:1153-1179)
  return Shape(dims);
}

}  // namespace

// ---- row softmax (P7: softmax(x, axis = k)) --------------------------------
// [[Rcpp::export]]
// (the per-dtype bodies are structs at namespace scope: a local class cannot
// have member templates)
namespace {
struct SoftmaxAxis {
  int axis;
  template <typename T>
  SEXP run(const gpuTensor<T> &t) {
    if (axis < 0 || axis >= (int)t.ndims()) stop("axis must be a single positive integer within tensor dimensions");
    auto out = std::make_shared<gpuTensor<T>>(t.shape());
    const acd_desc o = to_acd(*out), i = to_acd(t);
    acd_done(acd_softmax(acd_default_ctx(), &o, &i, axis, nullptr), "softmax");
    return wrap_tensor(std::make_unique<TensorWrapper<T>>(out));
  }
};
}  // namespace

SEXP tensor_softmax_axis_unified(SEXP tensor_ptr, int axis) {
  XPtr<TensorBase> x(tensor_ptr);
  if (!x) stop("Invalid tensor pointer");
  return dispatch_real(x, SoftmaxAxis{axis}, "Softmax");
}

// ---- cumsum / cumprod along an axis (P8; axis < 0: flattened) ---------------
namespace {
struct ScanAxis {
  int axis;
  int32_t op;
  const char *what;
  template <typename T>
  SEXP run(const gpuTensor<T> &t) {
    if (axis >= (int)t.ndims()) stop("axis must be a single positive integer within tensor dimensions");
    auto out = std::make_shared<gpuTensor<T>>(t.shape());
    const acd_desc o = to_acd(*out), i = to_acd(t);
    acd_done(acd_scan(acd_default_ctx(), op, &o, &i, axis, nullptr), what);
    return wrap_tensor(std::make_unique<TensorWrapper<T>>(out));
  }
};

SEXP scan_axis(SEXP tensor_ptr, int axis, int32_t op, const char *what) {
  XPtr<TensorBase> x(tensor_ptr);
  if (!x) stop("Invalid tensor pointer");
  return dispatch_real(x, ScanAxis{axis, op, what}, what);
}
}  // namespace

// [[Rcpp::export]]
SEXP tensor_cumsum_axis_unified(SEXP tensor_ptr, int axis) { return scan_axis(tensor_ptr, axis, ACD_CUMSUM, "cumsum"); }

// [[Rcpp::export]]
SEXP tensor_cumprod_axis_unified(SEXP tensor_ptr, int axis) {
  return scan_axis(tensor_ptr, axis, ACD_CUMPROD, "cumprod");
}

// ---- argmax / argmin along an axis (the stubs of src/TensorReduction.cpp) ---
// Indices are 0-based int64, as TensorWrapper::argmax(axis) defines them
// (src/TensorRegistry.h:737-815); the R wrapper adds 1.
namespace {
struct ArgAxis {
  int axis;
  bool keep_dims;
  int32_t op;
  const char *what;
  template <typename T>
  SEXP run(const gpuTensor<T> &t) {
    if (axis < 0 || axis >= (int)t.ndims()) stop("axis must be within dimensions of tensor");
    auto out = std::make_shared<gpuTensor<int64_t>>(kept_shape(t.shape(), {axis}, keep_dims));
    const acd_desc o = to_acd(*out), i = to_acd(t);
    acd_done(acd_arg_reduce(acd_default_ctx(), op, &o, nullptr, &i, axis, 0, nullptr), what);
    return wrap_tensor(std::make_unique<TensorWrapper<int64_t>>(out));
  }
};

SEXP arg_axis(SEXP tensor_ptr, int axis, bool keep_dims, int32_t op, const char *what) {
  XPtr<TensorBase> x(tensor_ptr);
  if (!x) stop("Invalid tensor pointer");
  return dispatch_any(x, ArgAxis{axis, keep_dims, op, what}, what);
}
}  // namespace

// [[Rcpp::export]]
SEXP tensor_argmax_axis(SEXP tensor_ptr, int axis, bool keep_dims = false) {
  return arg_axis(tensor_ptr, axis, keep_dims, ACD_ARGMAX, "argmax");
}

// [[Rcpp::export]]
SEXP tensor_argmin_axis(SEXP tensor_ptr, int axis, bool keep_dims = false) {
  return arg_axis(tensor_ptr, axis, keep_dims, ACD_ARGMIN, "argmin");
}

// ---- variance along axes (the reference's axis_variance_kernel writes 0) ----
namespace {
struct VarAxes {
  std::vector<int> axes0;
  bool keep_dims;
  template <typename T>
  SEXP run(const gpuTensor<T> &t) {
    uint32_t mask = 0;
    for (int a : axes0) mask |= 1u << a;
    // float results in the tensor dtype (accumulated in float64 inside)
    auto out = std::make_shared<gpuTensor<T>>(kept_shape(t.shape(), axes0, keep_dims));
    const acd_desc o = to_acd(*out), i = to_acd(t);
    acd_done(acd_reduce(acd_default_ctx(), ACD_RED_VAR, &o, &i, mask, nullptr), "var");
    return wrap_tensor(std::make_unique<TensorWrapper<T>>(out));
  }
};
}  // namespace

// [[Rcpp::export]]
SEXP tensor_var_axis(SEXP tensor_ptr, Nullable<IntegerVector> axis = R_NilValue, bool keep_dims = false) {
  XPtr<TensorBase> x(tensor_ptr);
  if (!x) stop("Invalid tensor pointer");
  std::vector<int> axes0;
  if (axis.isNotNull()) {
    IntegerVector av(axis.get());
    for (int a : av) {
      if (a < 1 || a > (int)x->ndims()) stop("axis must be a vector of positive integers");
      axes0.push_back(a - 1);  // the R API is 1-based
    }
  } else {
    for (int d = 0; d < (int)x->ndims(); ++d) axes0.push_back(d);
  }
  return dispatch_real(x, VarAxes{axes0, keep_dims}, "var");
}

// ---- comparisons with a bool result (P6) -----------------------------------
namespace {
struct CompareBool {
  XPtr<TensorBase> b;
  int32_t code;
  template <typename T>
  SEXP run(const gpuTensor<T> &ta) {
    const gpuTensor<T> &tb = tensor_of<T>(b);
    int32_t nd = 0;
    int64_t shp[ACD_MAX_DIMS];
    const acd_desc da = to_acd(ta), db = to_acd(tb);
    if (acd_broadcast_shape(da.ndim, da.shape, db.ndim, db.shape, &nd, shp) != ACD_OK)
      stop("Tensor shapes are not broadcastable");
    std::vector<size_t> dims(shp, shp + nd);
    auto out = std::make_shared<gpuTensor<bool>>(Shape(dims));
    const acd_desc o = to_acd(*out);
    acd_done(acd_binary(acd_default_ctx(), code, &o, &da, &db, nullptr), "comparison");
    return wrap_tensor(std::make_unique<TensorWrapper<bool>>(out));
  }
};
}  // namespace

// op: "gt", "lt", "eq", "ne", "ge", "le".  The reference's tensor_gt_unified
// returns 0/1 in the input dtype; these store bool (1 byte), values 0/1.
// [[Rcpp::export]]
SEXP tensor_compare_bool_unified(SEXP a_ptr, SEXP b_ptr, std::string op) {
  XPtr<TensorBase> a(a_ptr), b(b_ptr);
  if (!a || !b) stop("Invalid tensor pointer");
  if (a->dtype() != b->dtype()) stop("Cannot compare tensors with different dtypes");
  int32_t code;
  if (op == "gt") code = ACD_GT;
  else if (op == "lt") code = ACD_LT;
  else if (op == "eq") code = ACD_EQ;
  else if (op == "ne") code = ACD_NE;
  else if (op == "ge") code = ACD_GE;
  else if (op == "le") code = ACD_LE;
  else stop("Unknown comparison: " + op);
  return dispatch_any(a, CompareBool{b, code}, "comparison");
}

// ---- dtype conversion with base R's as.* rules -------------------------------
namespace {
struct ToDtype {
  std::string dtype;
  template <typename To, typename From>
  SEXP to(const gpuTensor<From> &t) {
    auto out = std::make_shared<gpuTensor<To>>(t.shape());
    const acd_desc o = to_acd(*out), i = to_acd(t);
    acd_done(acd_convert(acd_default_ctx(), &o, &i, nullptr), "to_dtype");
    return wrap_tensor(std::make_unique<TensorWrapper<To>>(out));
  }
  template <typename T>
  SEXP run(const gpuTensor<T> &t) {
    if (dtype == "float" || dtype == "float32") return to<float>(t);
    if (dtype == "double" || dtype == "float64") return to<double>(t);
    if (dtype == "int32" || dtype == "int") return to<int>(t);
    if (dtype == "int64" || dtype == "long") return to<int64_t>(t);
    if (dtype == "bool" || dtype == "logical") return to<bool>(t);
    if (dtype == "float16" || dtype == "half") return to<half>(t);
    if (dtype == "int8") return to<int8_t>(t);
    stop("Error converting tensor dtype: Unsupported target dtype: " + dtype);
    return R_NilValue;
  }
};
}  // namespace

// [[Rcpp::export]]
SEXP tensor_to_dtype_unified(SEXP tensor_ptr, std::string dtype) {
  XPtr<TensorBase> x(tensor_ptr);
  if (!x) stop("Invalid tensor pointer");
  return dispatch_any(x, ToDtype{dtype}, "to_dtype");
}

// ---- counter-based random tensors --------------------------------------------
// One (seed, position) stream per process: each call takes the next n
// positions (rounded up to a multiple of 4), so set_random_seed(s) makes runs
// repeatable, and a tensor sharded over ranks equals the unsharded one when
// each shard passes its first global index as the offset.
namespace {
uint64_t g_seed = 0x9E3779B97F4A7C15ull;
uint64_t g_pos = 0;

template <typename T>
SEXP rand_into(const Shape &shape, int32_t dist, double a, double b) {
  auto out = std::make_shared<gpuTensor<T>>(shape);
  const acd_desc o = to_acd(*out);
  const uint64_t pos = g_pos;
  g_pos += ((uint64_t)shape.size() + 3) / 4 * 4;
  acd_done(acd_rand(acd_default_ctx(), &o, dist, a, b, g_seed, pos, nullptr), dist ? "rnorm" : "rand");
  return wrap_tensor(std::make_unique<TensorWrapper<T>>(out));
}

Shape shape_of(IntegerVector shape) {
  std::vector<size_t> dims;
  for (int s : shape) {
    if (s <= 0) stop("All shape dimensions must be positive");
    dims.push_back((size_t)s);
  }
  return Shape(dims);
}
}  // namespace

// [[Rcpp::export]]
SEXP rand_tensor(IntegerVector shape, std::string dtype = "float") {
  if (dtype == "float" || dtype == "float32") return rand_into<float>(shape_of(shape), 0, 0.0, 1.0);
  if (dtype == "double" || dtype == "float64") return rand_into<double>(shape_of(shape), 0, 0.0, 1.0);
  stop("Unsupported dtype for random tensor. Use 'float' or 'double'");
  return R_NilValue;
}

// [[Rcpp::export]]
SEXP rnorm_tensor(IntegerVector shape, double mean = 0.0, double sd = 1.0, std::string dtype = "float") {
  if (dtype == "float" || dtype == "float32") return rand_into<float>(shape_of(shape), 1, mean, sd);
  if (dtype == "double" || dtype == "float64") return rand_into<double>(shape_of(shape), 1, mean, sd);
  stop("Unsupported dtype for random tensor. Use 'float' or 'double'");
  return R_NilValue;
}

// [[Rcpp::export]]
void set_random_seed(int seed) {
  g_seed = (uint64_t)(int64_t)seed;
  g_pos = 0;
}
