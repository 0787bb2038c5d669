/*
 * acediar_launchers.h — the acediaR launcher ABI, re-exported by
 * libacediar_b200.so so that the reference's Rcpp op modules
 * (src/Tensor*.cpp, src/TensorRegistry.h, src/gpuTensor.h) link against the
 * B200 kernels unchanged.
 *
 * Every name and signature below is the one the reference declares and
 * defines; the file:line of the reference definition is given per group.
 * Semantics follow the reference launchers (synchronous: each call returns
 * after the device has finished, like the reference's cudaDeviceSynchronize),
 * with these documented differences:
 *   - reductions cover every element (the reference's launch_reduction stops
 *     after 65535*256 elements, src/kernels/tensor_ops.cu:65-69);
 *   - float32 sums/variances accumulate in float64, float64 sums in
 *     double-double;
 *   - tensor_scalar_div_* divides (the reference multiplies by 1/s,
 *     src/kernels/tensor_ops.cu:1901-1913);
 *   - tensor_argmin_* scans the whole tensor (the reference launches one block,
 *     src/kernels/tensor_kernels.cu:1237);
 *   - tensor_axis_var_* computes the sample variance (the reference's
 *     axis_variance_kernel writes 0, src/kernels/tensor_kernels.cu:810-834);
 *   - in the *_strided_* entry points `data` is taken as the view's first
 *     element and the descriptor's `offset` is not added again (the reference
 *     adds it a second time, src/gpuTensor.h:597-599 with src/cuda_utils.h:140-146).
 * Failures throw std::runtime_error, as the reference's axis launchers do
 * (src/kernels/tensor_kernels.cu:947-988); the Rcpp glue turns them into R errors.
 */
#ifndef ACEDIAR_LAUNCHERS_H
#define ACEDIAR_LAUNCHERS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Binary-compatible with cuda_utils::TensorDescriptor (src/cuda_utils.h:111-118).
 * The reference passes it by C++ reference, i.e. as a pointer. */
typedef struct acd_ref_descriptor {
  void *data;
  int ndims;
  int shape[8];
  int strides[8];
  size_t offset;
  size_t total_size;
} acd_ref_descriptor;

/* IEEE binary16 storage: CUDA's `half` (__half), two bytes.  The reference
 * declares these launchers with `half *`; a pointer to this struct has the
 * same representation, and extern "C" names carry no parameter types. */
typedef struct acd_half {
  uint16_t bits;
} acd_half;

/* ---- float16 and int8 (declared at src/TensorArithmetic.cpp:13-31, 64-67,
 * 84-114; defined at src/kernels/tensor_ops.cu:1053-1117, 1368-1392).
 * float16: one rounding per operation (correctly rounded binary16); the
 * scalar is rounded to half first.  int8: wraps modulo 256. ---- */
void tensor_add_float16(acd_half *r, const acd_half *a, const acd_half *b, size_t n);
void tensor_sub_float16(acd_half *r, const acd_half *a, const acd_half *b, size_t n);
void tensor_mul_float16(acd_half *r, const acd_half *a, const acd_half *b, size_t n);
void tensor_div_float16(acd_half *r, const acd_half *a, const acd_half *b, size_t n);
void tensor_scalar_add_float16(acd_half *r, const acd_half *x, float s, size_t n);
void tensor_scalar_mul_float16(acd_half *r, const acd_half *x, float s, size_t n);
void tensor_add_int8(int8_t *r, const int8_t *a, const int8_t *b, size_t n);
void tensor_add_strided_float16(const acd_ref_descriptor *out, const acd_ref_descriptor *a,
                                const acd_ref_descriptor *b);
void tensor_sub_strided_float16(const acd_ref_descriptor *out, const acd_ref_descriptor *a,
                                const acd_ref_descriptor *b);
void tensor_mul_strided_float16(const acd_ref_descriptor *out, const acd_ref_descriptor *a,
                                const acd_ref_descriptor *b);
void tensor_div_strided_float16(const acd_ref_descriptor *out, const acd_ref_descriptor *a,
                                const acd_ref_descriptor *b);
void tensor_add_strided_int8(const acd_ref_descriptor *out, const acd_ref_descriptor *a,
                             const acd_ref_descriptor *b);
/* sums (declared at src/TensorReduction.cpp:12-15; the reference's own
 * definitions, src/kernels/tensor_ops.cu:701-710, are placeholders returning
 * 0): float16 accumulated in float64 and returned as float; int64 exact
 * (modulo 2^64) */
float tensor_sum_float16(const acd_half *in, size_t n);
int64_t tensor_sum_int64(const int64_t *in, size_t n);

/* ---- contractions (declared at src/TensorLinearAlgebra.cpp:15-34, defined
 * at src/kernels/tensor_ops.cu:1180-1326): outside the hot path, exported so
 * the Rcpp modules link against this library alone.  matmul / matvec /
 * vecmat call cuBLAS (loaded on first use); the outer product
 * result[i + M*j] = a[i] * b[j] is a broadcast multiply.  Column-major:
 * C (M x N) = A (M x K) B (K x N); matvec r = A (M x N) v; vecmat
 * r = v A (M x N).  float16 accumulates in float32.  The float16 matvec and
 * vecmat are declared but not defined by the reference. ---- */
void tensor_matmul_float16(acd_half *C, const acd_half *A, const acd_half *B, size_t M, size_t N, size_t K);
void tensor_matmul_float32(float *C, const float *A, const float *B, size_t M, size_t N, size_t K);
void tensor_matmul_float64(double *C, const double *A, const double *B, size_t M, size_t N, size_t K);
void tensor_outer_product_float16(acd_half *r, const acd_half *a, const acd_half *b, size_t M, size_t N);
void tensor_outer_product_float32(float *r, const float *a, const float *b, size_t M, size_t N);
void tensor_outer_product_float64(double *r, const double *a, const double *b, size_t M, size_t N);
void tensor_matvec_float16(acd_half *r, const acd_half *A, const acd_half *v, size_t M, size_t N);
void tensor_matvec_float32(float *r, const float *A, const float *v, size_t M, size_t N);
void tensor_matvec_float64(double *r, const double *A, const double *v, size_t M, size_t N);
void tensor_vecmat_float16(acd_half *r, const acd_half *v, const acd_half *A, size_t M, size_t N);
void tensor_vecmat_float32(float *r, const float *v, const float *A, size_t M, size_t N);
void tensor_vecmat_float64(double *r, const double *v, const double *A, size_t M, size_t N);

/* ---- contiguous elementwise: src/kernels/tensor_ops.cu:1001-1117 ---- */
void tensor_add_float32(float *r, const float *a, const float *b, size_t n);
void tensor_add_float64(double *r, const double *a, const double *b, size_t n);
void tensor_add_int32(int32_t *r, const int32_t *a, const int32_t *b, size_t n);
void tensor_add_int64(int64_t *r, const int64_t *a, const int64_t *b, size_t n);
void tensor_sub_float32(float *r, const float *a, const float *b, size_t n);
void tensor_sub_float64(double *r, const double *a, const double *b, size_t n);
void tensor_mul_float32(float *r, const float *a, const float *b, size_t n);
void tensor_mul_float64(double *r, const double *a, const double *b, size_t n);
void tensor_div_float32(float *r, const float *a, const float *b, size_t n);
void tensor_div_float64(double *r, const double *a, const double *b, size_t n);
/* comparisons write 1/0 in the input dtype: src/kernels/tensor_ops.cu:757-791 */
void tensor_gt_float32(float *r, const float *a, const float *b, size_t n);
void tensor_gt_float64(double *r, const double *a, const double *b, size_t n);
void tensor_lt_float32(float *r, const float *a, const float *b, size_t n);
void tensor_lt_float64(double *r, const double *a, const double *b, size_t n);
void tensor_eq_float32(float *r, const float *a, const float *b, size_t n);
void tensor_eq_float64(double *r, const double *a, const double *b, size_t n);
/* pmax/pmin/pow: src/kernels/tensor_ops.cu:1761-1803 */
void tensor_max_elemwise_float32(float *r, const float *a, const float *b, size_t n);
void tensor_max_elemwise_float64(double *r, const double *a, const double *b, size_t n);
void tensor_min_elemwise_float32(float *r, const float *a, const float *b, size_t n);
void tensor_min_elemwise_float64(double *r, const double *a, const double *b, size_t n);
void tensor_pow_elemwise_float32(float *r, const float *a, const float *b, size_t n);
void tensor_pow_elemwise_float64(double *r, const double *a, const double *b, size_t n);

/* ---- scalar ops: src/kernels/tensor_ops.cu:1032-1074, 1887-1913 ---- */
void tensor_scalar_add_float32(float *r, const float *x, float s, size_t n);
void tensor_scalar_add_float64(double *r, const double *x, double s, size_t n);
void tensor_scalar_mul_float32(float *r, const float *x, float s, size_t n);
void tensor_scalar_mul_float64(double *r, const double *x, double s, size_t n);
void tensor_scalar_sub_float32(float *r, const float *x, float s, size_t n);
void tensor_scalar_sub_float64(double *r, const double *x, double s, size_t n);
void tensor_scalar_div_float32(float *r, const float *x, float s, size_t n);
void tensor_scalar_div_float64(double *r, const double *x, double s, size_t n);
void tensor_pow_scalar_float32(float *r, const float *x, float e, size_t n);
void tensor_pow_scalar_float64(double *r, const double *x, double e, size_t n);

/* ---- unary math and activations: src/kernels/tensor_ops.cu:488-683 ---- */
#define ACEDIAR_UNARY_DECL(NAME)                                          \
  void tensor_##NAME##_float32(float *r, const float *x, size_t n);       \
  void tensor_##NAME##_float64(double *r, const double *x, size_t n);
ACEDIAR_UNARY_DECL(exp)
ACEDIAR_UNARY_DECL(log)
ACEDIAR_UNARY_DECL(sqrt)
ACEDIAR_UNARY_DECL(abs)
ACEDIAR_UNARY_DECL(tanh)
ACEDIAR_UNARY_DECL(sigmoid)
ACEDIAR_UNARY_DECL(relu)
ACEDIAR_UNARY_DECL(sin)
ACEDIAR_UNARY_DECL(cos)
ACEDIAR_UNARY_DECL(floor)
ACEDIAR_UNARY_DECL(ceil)
ACEDIAR_UNARY_DECL(round)
ACEDIAR_UNARY_DECL(erf)
#undef ACEDIAR_UNARY_DECL

/* ---- broadcast binary, host metadata: src/kernels/tensor_ops.cu:1120-1179, 1973-2035 ---- */
#define ACEDIAR_BCAST_DECL(NAME)                                                                         \
  void tensor_##NAME##_broadcast_float32(float *r, const float *a, const float *b, const int *a_strides,  \
                                         const int *b_strides, const int *r_strides, const int *shape,   \
                                         int ndims, size_t total);                                        \
  void tensor_##NAME##_broadcast_float64(double *r, const double *a, const double *b,                    \
                                         const int *a_strides, const int *b_strides,                     \
                                         const int *r_strides, const int *shape, int ndims, size_t total);
ACEDIAR_BCAST_DECL(add)
ACEDIAR_BCAST_DECL(sub)
ACEDIAR_BCAST_DECL(mul)
ACEDIAR_BCAST_DECL(div)
ACEDIAR_BCAST_DECL(max)
ACEDIAR_BCAST_DECL(min)
ACEDIAR_BCAST_DECL(pow)
ACEDIAR_BCAST_DECL(gt)
ACEDIAR_BCAST_DECL(lt)
ACEDIAR_BCAST_DECL(eq)
#undef ACEDIAR_BCAST_DECL

/* ---- strided (view) ops: src/kernels/tensor_ops.cu:1342-1966 ---- */
#define ACEDIAR_STRIDED_BIN_DECL(NAME)                                                               \
  void tensor_##NAME##_strided_float32(const acd_ref_descriptor *out, const acd_ref_descriptor *a,  \
                                       const acd_ref_descriptor *b);                                \
  void tensor_##NAME##_strided_float64(const acd_ref_descriptor *out, const acd_ref_descriptor *a,  \
                                       const acd_ref_descriptor *b);
ACEDIAR_STRIDED_BIN_DECL(add)
ACEDIAR_STRIDED_BIN_DECL(sub)
ACEDIAR_STRIDED_BIN_DECL(mul)
ACEDIAR_STRIDED_BIN_DECL(div)
ACEDIAR_STRIDED_BIN_DECL(max_elemwise)
ACEDIAR_STRIDED_BIN_DECL(min_elemwise)
ACEDIAR_STRIDED_BIN_DECL(pow_elemwise)
#undef ACEDIAR_STRIDED_BIN_DECL
#define ACEDIAR_STRIDED_UN_DECL(NAME)                                                                \
  void tensor_##NAME##_strided_float32(const acd_ref_descriptor *out, const acd_ref_descriptor *in); \
  void tensor_##NAME##_strided_float64(const acd_ref_descriptor *out, const acd_ref_descriptor *in);
ACEDIAR_STRIDED_UN_DECL(exp)
ACEDIAR_STRIDED_UN_DECL(log)
ACEDIAR_STRIDED_UN_DECL(sqrt)
ACEDIAR_STRIDED_UN_DECL(floor)
ACEDIAR_STRIDED_UN_DECL(ceil)
ACEDIAR_STRIDED_UN_DECL(round)
ACEDIAR_STRIDED_UN_DECL(erf)
#undef ACEDIAR_STRIDED_UN_DECL
#define ACEDIAR_STRIDED_SC_DECL(NAME)                                                                \
  void tensor_##NAME##_strided_float32(const acd_ref_descriptor *out, const acd_ref_descriptor *in,  \
                                       float s);                                                     \
  void tensor_##NAME##_strided_float64(const acd_ref_descriptor *out, const acd_ref_descriptor *in,  \
                                       double s);
ACEDIAR_STRIDED_SC_DECL(scalar_add)
ACEDIAR_STRIDED_SC_DECL(scalar_mul)
ACEDIAR_STRIDED_SC_DECL(scalar_sub)
ACEDIAR_STRIDED_SC_DECL(scalar_div)
ACEDIAR_STRIDED_SC_DECL(pow_scalar)
#undef ACEDIAR_STRIDED_SC_DECL

/* ---- strided copy (contiguous()): src/gpuTensor.h:33-36, src/kernels/tensor_ops.cu:1329-1339 ---- */
void tensor_strided_copy_float32(float *dest, const float *src, const int *strides, const int *shape, int ndims,
                                 size_t total);
void tensor_strided_copy_float64(double *dest, const double *src, const int *strides, const int *shape, int ndims,
                                 size_t total);

/* ---- global reductions (host scalar results): src/TensorRegistry.h:15-39 ---- */
float tensor_sum_float32(const float *in, size_t n);
double tensor_sum_float64(const double *in, size_t n);
float tensor_max_float32(const float *in, size_t n);
double tensor_max_float64(const double *in, size_t n);
float tensor_min_float32(const float *in, size_t n);
double tensor_min_float64(const double *in, size_t n);
float tensor_prod_float32(const float *in, size_t n);
double tensor_prod_float64(const double *in, size_t n);
double tensor_var_float32(const float *in, size_t n);
double tensor_var_float64(const double *in, size_t n);
/* 1-based index of the first maximum/minimum (src/kernels/tensor_ops.cu:850-880) */
int64_t tensor_argmax_float32(const float *in, size_t n);
int64_t tensor_argmax_float64(const double *in, size_t n);
int64_t tensor_argmin_float32(const float *in, size_t n);
int64_t tensor_argmin_float64(const double *in, size_t n);

/* ---- axis reductions, DEVICE metadata arrays: src/TensorRegistry.h:41-114 ---- */
#define ACEDIAR_AXIS_DECL(NAME)                                                                            \
  void tensor_axis_##NAME##_float32(float *r, const float *in, const int *in_strides, const int *in_shape,  \
                                    const int *r_strides, const int *axes, int n_axes, int ndims,           \
                                    size_t out_size);                                                       \
  void tensor_axis_##NAME##_float64(double *r, const double *in, const int *in_strides,                     \
                                    const int *in_shape, const int *r_strides, const int *axes, int n_axes, \
                                    int ndims, size_t out_size);
ACEDIAR_AXIS_DECL(sum)
ACEDIAR_AXIS_DECL(mean)
ACEDIAR_AXIS_DECL(max)
ACEDIAR_AXIS_DECL(min)
ACEDIAR_AXIS_DECL(prod)
ACEDIAR_AXIS_DECL(var)
#undef ACEDIAR_AXIS_DECL
/* 0-based index within the reduced fiber (src/kernels/tensor_kernels.cu:1316-1480) */
void tensor_axis_argmax_float32(int64_t *idx, const float *in, const int *in_strides, const int *in_shape,
                                const int *out_strides, const int *axes, int n_axes, int ndims, size_t out_elems);
void tensor_axis_argmax_float64(int64_t *idx, const double *in, const int *in_strides, const int *in_shape,
                                const int *out_strides, const int *axes, int n_axes, int ndims, size_t out_elems);
void tensor_axis_argmin_float32(int64_t *idx, const float *in, const int *in_strides, const int *in_shape,
                                const int *out_strides, const int *axes, int n_axes, int ndims, size_t out_elems);
void tensor_axis_argmin_float64(int64_t *idx, const double *in, const int *in_strides, const int *in_shape,
                                const int *out_strides, const int *axes, int n_axes, int ndims, size_t out_elems);

/* ---- slice and mask assignment (host metadata): src/kernels/tensor_slice_update.cu,
 * called by src/TensorMutation.cpp:49-86 ---- */
void tensor_slice_add_scalar_float32(float *data, double scalar, const int *start, const int *slice_shape,
                                     const int *strides, int ndims, size_t total_elements);
void tensor_slice_add_scalar_float64(double *data, double scalar, const int *start, const int *slice_shape,
                                     const int *strides, int ndims, size_t total_elements);
void tensor_slice_set_scalar_float32(float *data, double scalar, const int *start, const int *slice_shape,
                                     const int *strides, int ndims, size_t total_elements);
void tensor_slice_set_scalar_float64(double *data, double scalar, const int *start, const int *slice_shape,
                                     const int *strides, int ndims, size_t total_elements);
void tensor_slice_set_tensor_float32(float *dest_data, const float *src_data, const int *start,
                                     const int *slice_shape, const int *dest_strides, const int *src_strides,
                                     int ndims, size_t total_elements);
void tensor_slice_set_tensor_float64(double *dest_data, const double *src_data, const int *start,
                                     const int *slice_shape, const int *dest_strides, const int *src_strides,
                                     int ndims, size_t total_elements);
/* mask: one byte per element, nonzero = TRUE (C++ bool storage) */
void tensor_mask_set_scalar_float32(float *data, const unsigned char *mask, float value, size_t total_elements);
void tensor_mask_set_scalar_float64(double *data, const unsigned char *mask, double value, size_t total_elements);

/* ---- concat / stack / repeat / pad (host metadata): src/TensorMutation.cpp:10-47 ---- */
void launch_concat_float32(float *result, const float **inputs, const int *input_sizes, int num_tensors,
                           const int *result_strides, const int *input_strides_list, const int *shape, int ndims,
                           int concat_axis, size_t total_elements);
void launch_concat_float64(double *result, const double **inputs, const int *input_sizes, int num_tensors,
                           const int *result_strides, const int *input_strides_list, const int *shape, int ndims,
                           int concat_axis, size_t total_elements);
void launch_stack_float32(float *result, const float **inputs, int num_tensors, const int *input_strides,
                          const int *result_shape, int ndims, int stack_axis, size_t total_elements);
void launch_stack_float64(double *result, const double **inputs, int num_tensors, const int *input_strides,
                          const int *result_shape, int ndims, int stack_axis, size_t total_elements);
void launch_repeat_float32(float *result, const float *input, const int *input_strides, const int *repeat_counts,
                           const int *input_shape, const int *result_shape, int ndims, size_t total_elements);
void launch_repeat_float64(double *result, const double *input, const int *input_strides, const int *repeat_counts,
                           const int *input_shape, const int *result_shape, int ndims, size_t total_elements);
void launch_pad_float32(float *result, const float *input, const int *input_strides, const int *input_shape,
                        const int *pad_before, const int *pad_after, const int *result_shape, int ndims,
                        float pad_value, int pad_mode, size_t total_elements);
void launch_pad_float64(double *result, const double *input, const int *input_strides, const int *input_shape,
                        const int *pad_before, const int *pad_after, const int *result_shape, int ndims,
                        double pad_value, int pad_mode, size_t total_elements);

/* ---- softmax over the whole tensor: src/kernels/tensor_ops.cu:826-846 ---- */
void tensor_softmax_float32(float *out, const float *in, size_t n);
void tensor_softmax_float64(double *out, const double *in, size_t n);

#ifdef __cplusplus
}
#endif

#endif /* ACEDIAR_LAUNCHERS_H */
