// The reference's contraction launchers: matmul, outer product, matrix-vector
// and vector-matrix products (declared at src/TensorLinearAlgebra.cpp:15-34,
// defined at src/kernels/tensor_ops.cu:1180-1326).
//
// Contractions are not part of this library's memory-bound hot path; they are
// exported so that the reference's Rcpp modules link against this library
// alone.  GEMM and GEMV are plain cuBLAS calls, as in the reference.  cuBLAS
// is opened with dlopen on the first contraction, so the rest of the library
// carries no cuBLAS dependency.  The outer product, result[i + M*j] =
// a[i] * b[j] in column-major order, is this library's broadcast multiply of
// an M x 1 view by a 1 x N view.
//
// Like the other reference-named launchers they run on the legacy default
// stream of the current device and synchronise before returning; a failure
// throws std::runtime_error.
#include <cublas_v2.h>
#include <dlfcn.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "../../include/acediar_launchers.h"
#include "common.cuh"

namespace acd {
acd_ctx *shim_ctx();  // csrc/shim.cu

namespace {

struct Cublas {
  decltype(&cublasCreate_v2) create = nullptr;
  decltype(&cublasSetStream_v2) set_stream = nullptr;
  decltype(&cublasSgemm_v2) sgemm = nullptr;
  decltype(&cublasDgemm_v2) dgemm = nullptr;
  // the C entry point (C++ adds an overload taking cudaDataType as the compute type)
  cublasStatus_t (*gemm_ex)(cublasHandle_t, cublasOperation_t, cublasOperation_t, int, int, int, const void *,
                            const void *, cudaDataType, int, const void *, cudaDataType, int, const void *, void *,
                            cudaDataType, int, cublasComputeType_t, cublasGemmAlgo_t) = nullptr;
  decltype(&cublasSgemv_v2) sgemv = nullptr;
  decltype(&cublasDgemv_v2) dgemv = nullptr;
  cublasHandle_t handles[64] = {nullptr};
};

template <typename F>
void bind(void *lib, F &f, const char *name) {
  f = reinterpret_cast<F>(dlsym(lib, name));
  if (!f) throw std::runtime_error(std::string("acediar: cuBLAS entry point missing: ") + name);
}

// The cuBLAS handle of the current device (created on first use).
std::pair<Cublas *, cublasHandle_t> cublas_for_device() {
  static std::mutex mu;
  static Cublas api;
  static bool loaded = false;
  std::lock_guard<std::mutex> lk(mu);
  if (!loaded) {
    void *lib = dlopen("libcublas.so.12", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) throw std::runtime_error(std::string("acediar: cannot load libcublas.so.12: ") + dlerror());
    bind(lib, api.create, "cublasCreate_v2");
    bind(lib, api.set_stream, "cublasSetStream_v2");
    bind(lib, api.sgemm, "cublasSgemm_v2");
    bind(lib, api.dgemm, "cublasDgemm_v2");
    bind(lib, api.gemm_ex, "cublasGemmEx");
    bind(lib, api.sgemv, "cublasSgemv_v2");
    bind(lib, api.dgemv, "cublasDgemv_v2");
    loaded = true;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) throw std::runtime_error("acediar: no CUDA device");
  if (!api.handles[dev]) {
    cublasHandle_t h = nullptr;
    if (api.create(&h) != CUBLAS_STATUS_SUCCESS) throw std::runtime_error("acediar: cublasCreate failed");
    api.set_stream(h, nullptr);
    api.handles[dev] = h;
  }
  return {&api, api.handles[dev]};
}

void done(cublasStatus_t st, const char *fn) {
  if (st != CUBLAS_STATUS_SUCCESS)
    throw std::runtime_error(std::string(fn) + ": cuBLAS status " + std::to_string((int)st));
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) throw std::runtime_error(std::string(fn) + ": " + cudaGetErrorString(e));
}

int dim(size_t v, const char *fn) {
  if (v > (size_t)INT32_MAX) throw std::runtime_error(std::string(fn) + ": extent exceeds the int range of cuBLAS");
  return (int)v;
}

// C (M x N) = A (M x K) B (K x N), all column-major with leading dimensions
// M, K and M; float16 operands accumulate in float32.
template <typename T>
void gemm(T *C, const T *A, const T *B, size_t M, size_t N, size_t K, cublasOperation_t ta, int lda, int ldb,
          int ldc, const char *fn) {
  if (M == 0 || N == 0) return;
  auto [api, h] = cublas_for_device();
  const int m = dim(M, fn), n = dim(N, fn), k = dim(K, fn);
  cublasStatus_t st;
  if constexpr (std::is_same<T, float>::value) {
    const float one = 1.0f, zero = 0.0f;
    st = api->sgemm(h, ta, CUBLAS_OP_N, m, n, k, &one, A, lda, B, ldb, &zero, C, ldc);
  } else if constexpr (std::is_same<T, double>::value) {
    const double one = 1.0, zero = 0.0;
    st = api->dgemm(h, ta, CUBLAS_OP_N, m, n, k, &one, A, lda, B, ldb, &zero, C, ldc);
  } else {
    const float one = 1.0f, zero = 0.0f;
    st = api->gemm_ex(h, ta, CUBLAS_OP_N, m, n, k, &one, A, CUDA_R_16F, lda, B, CUDA_R_16F, ldb, &zero, C,
                      CUDA_R_16F, ldc, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  }
  done(st, fn);
}

// y = op(A) x with A M x N column-major.
template <typename T>
void gemv(T *y, const T *A, const T *x, size_t M, size_t N, cublasOperation_t ta, const char *fn) {
  if (M == 0 || N == 0) return;
  auto [api, h] = cublas_for_device();
  const int m = dim(M, fn), n = dim(N, fn);
  cublasStatus_t st;
  if constexpr (std::is_same<T, float>::value) {
    const float one = 1.0f, zero = 0.0f;
    st = api->sgemv(h, ta, m, n, &one, A, m, x, 1, &zero, y, 1);
  } else {
    const double one = 1.0, zero = 0.0;
    st = api->dgemv(h, ta, m, n, &one, A, m, x, 1, &zero, y, 1);
  }
  done(st, fn);
}

template <typename T>
void outer(T *r, const T *a, const T *b, size_t M, size_t N, int32_t dt, const char *fn) {
  if (M == 0 || N == 0) return;
  acd_ctx *ctx = shim_ctx();
  acd_desc o{}, x{}, y{};
  o.data = r;
  x.data = const_cast<T *>(a);
  y.data = const_cast<T *>(b);
  o.ndim = x.ndim = y.ndim = 2;
  o.dtype = x.dtype = y.dtype = dt;
  o.shape[0] = (int64_t)M;
  o.shape[1] = (int64_t)N;
  o.stride[0] = 1;
  o.stride[1] = (int64_t)M;
  x.shape[0] = (int64_t)M;  // a as M x 1
  x.shape[1] = 1;
  x.stride[0] = 1;
  x.stride[1] = (int64_t)M;
  y.shape[0] = 1;  // b as 1 x N
  y.shape[1] = (int64_t)N;
  y.stride[0] = 1;
  y.stride[1] = 1;
  if (acd_binary(ctx, ACD_MUL, &o, &x, &y, nullptr) != ACD_OK)
    throw std::runtime_error(std::string(fn) + ": " + acd_last_error());
  const cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) throw std::runtime_error(std::string(fn) + ": " + cudaGetErrorString(e));
}

__half *hp(acd_half *p) { return reinterpret_cast<__half *>(p); }
const __half *hp(const acd_half *p) { return reinterpret_cast<const __half *>(p); }

}  // namespace
}  // namespace acd

using namespace acd;

extern "C" {

void tensor_matmul_float16(acd_half *C, const acd_half *A, const acd_half *B, size_t M, size_t N, size_t K) {
  gemm<__half>(hp(C), hp(A), hp(B), M, N, K, CUBLAS_OP_N, (int)M, (int)K, (int)M, "tensor_matmul_float16");
}
void tensor_matmul_float32(float *C, const float *A, const float *B, size_t M, size_t N, size_t K) {
  gemm<float>(C, A, B, M, N, K, CUBLAS_OP_N, (int)M, (int)K, (int)M, "tensor_matmul_float32");
}
void tensor_matmul_float64(double *C, const double *A, const double *B, size_t M, size_t N, size_t K) {
  gemm<double>(C, A, B, M, N, K, CUBLAS_OP_N, (int)M, (int)K, (int)M, "tensor_matmul_float64");
}

void tensor_outer_product_float16(acd_half *r, const acd_half *a, const acd_half *b, size_t M, size_t N) {
  outer<__half>(hp(r), hp(a), hp(b), M, N, ACD_FLOAT16, "tensor_outer_product_float16");
}
void tensor_outer_product_float32(float *r, const float *a, const float *b, size_t M, size_t N) {
  outer<float>(r, a, b, M, N, ACD_FLOAT32, "tensor_outer_product_float32");
}
void tensor_outer_product_float64(double *r, const double *a, const double *b, size_t M, size_t N) {
  outer<double>(r, a, b, M, N, ACD_FLOAT64, "tensor_outer_product_float64");
}

// result (M) = A (M x N) v (N)
void tensor_matvec_float32(float *r, const float *A, const float *v, size_t M, size_t N) {
  gemv<float>(r, A, v, M, N, CUBLAS_OP_N, "tensor_matvec_float32");
}
void tensor_matvec_float64(double *r, const double *A, const double *v, size_t M, size_t N) {
  gemv<double>(r, A, v, M, N, CUBLAS_OP_N, "tensor_matvec_float64");
}
// result (N) = v (M) A (M x N), i.e. A^T v
void tensor_vecmat_float32(float *r, const float *v, const float *A, size_t M, size_t N) {
  gemv<float>(r, A, v, M, N, CUBLAS_OP_T, "tensor_vecmat_float32");
}
void tensor_vecmat_float64(double *r, const double *v, const double *A, size_t M, size_t N) {
  gemv<double>(r, A, v, M, N, CUBLAS_OP_T, "tensor_vecmat_float64");
}
// The float16 forms are declared by the reference (src/TensorLinearAlgebra.cpp:27,
// 32) but never defined there; here they are a GEMM with one column,
// accumulated in float32.
void tensor_matvec_float16(acd_half *r, const acd_half *A, const acd_half *v, size_t M, size_t N) {
  gemm<__half>(hp(r), hp(A), hp(v), M, 1, N, CUBLAS_OP_N, (int)M, (int)N, (int)M, "tensor_matvec_float16");
}
void tensor_vecmat_float16(acd_half *r, const acd_half *v, const acd_half *A, size_t M, size_t N) {
  gemm<__half>(hp(r), hp(A), hp(v), N, 1, M, CUBLAS_OP_T, (int)M, (int)M, (int)N, "tensor_vecmat_float16");
}

}  // extern "C"
