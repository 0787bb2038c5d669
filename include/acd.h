/*
 * acd.h — C ABI of the B200 tensor hot path (elementwise, broadcast, strided
 * copy, full/axis reductions, arg-reductions, scans, softmax).
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, is
 * stream-ordered (asynchronous with respect to the host unless stated) and
 * returns an acd_status.  No exception crosses this boundary.  The message of
 * the last failure on the calling thread is available from acd_last_error().
 *
 * Layout convention: acediaR tensors are column-major (src/gpuTensor.h:51-55,
 * compute_strides at src/gpuTensor.h:359-370): axis 0 is the fastest-varying,
 * stride[0] == 1 for a contiguous tensor.  A descriptor may describe any
 * strided view: permuted, transposed, broadcast (stride 0) or offset.  The
 * offset is applied exactly once (the reference applies it twice, src/gpuTensor.h:597-599
 * with src/cuda_utils.h:140-146).
 *
 * Replaces, in the reference:
 *   - cuda_utils::TensorDescriptor (src/cuda_utils.h:111-156): int32 shape and
 *     strides, row-major linear_to_coords        -> acd_desc (int64, column-major)
 *   - the TensorRegistry dtype dispatch (src/TensorRegistry.h:214-1386)
 *                                                 -> dtype field + internal dispatch
 *   - the extern "C" launchers (src/kernels/tensor_ops.cu:484-2037,
 *     src/kernels/tensor_kernels.cu:934-1482)     -> the acd_* functions below.
 * The reference's own launcher names are also exported by the same library;
 * see acediar_launchers.h.
 */
#ifndef ACD_H
#define ACD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ACD_MAX_DIMS 8

/* Element types.  Names follow dtype_to_string (src/gpuTensor.h:183-200).
 * FLOAT16 and INT8 are the reference's two narrow storage types
 * (DType::FLOAT16 / DType::INT8, src/gpuTensor.h:61-75).  They take the
 * element-wise arithmetic, scalar ops, comparisons, copies, conversions,
 * fills and the sum / mean / count reductions (INT8 also max / min);
 * the transcendental functions, variance, products and arg-reductions
 * return ACD_ERR_UNSUPPORTED for them.  FLOAT16 arithmetic is IEEE
 * binary16 with one rounding per operation (the operation is evaluated in
 * float32 and rounded once, which equals the correctly rounded half result
 * for + - * /); INT8 arithmetic wraps modulo 256 as the reference's int8_t
 * arithmetic does. */
typedef enum {
  ACD_FLOAT32 = 0, /* "float"  */
  ACD_FLOAT64 = 1, /* "double" */
  ACD_INT32 = 2,   /* "int32"  */
  ACD_INT64 = 3,   /* "int64"  */
  ACD_BOOL = 4,    /* "bool", one byte holding 0 or 1 */
  ACD_FLOAT16 = 5, /* "float16", IEEE binary16 */
  ACD_INT8 = 6     /* "int8"   */
} acd_dtype;

typedef enum {
  ACD_OK = 0,
  ACD_ERR_INVALID = 1,     /* null pointer, bad ndim, negative extent, bad op code */
  ACD_ERR_SHAPE = 2,       /* shapes not broadcastable, or output shape mismatch */
  ACD_ERR_DTYPE = 3,       /* dtype combination not supported by the op */
  ACD_ERR_AXIS = 4,        /* axis out of range */
  ACD_ERR_ALLOC = 5,       /* workspace allocation failed */
  ACD_ERR_CUDA = 6,        /* CUDA runtime error (message has the CUDA error string) */
  ACD_ERR_DEVICE = 7,      /* a kernel raised its device status word (bounded wait expired) */
  ACD_ERR_UNSUPPORTED = 8  /* valid request outside what this build implements */
} acd_status;

/* Strided view descriptor.  Element (c0..c_{n-1}) lives at
 * data + (offset + sum_k c_k * stride[k]) * sizeof(dtype).  ndim == 0 is a
 * one-element scalar.  Strides are in elements and may be 0 (broadcast). */
typedef struct acd_desc {
  void *data;
  int64_t offset;
  int64_t shape[ACD_MAX_DIMS];
  int64_t stride[ACD_MAX_DIMS];
  int32_t ndim;
  int32_t dtype;
} acd_desc;

/* Opaque per-device context: owns the reduction/scan workspace and the
 * device status word.  Calls that share one context must be ordered on one
 * stream (the workspace is reused without locking). */
typedef struct acd_ctx acd_ctx;

/* cudaStream_t, passed as an opaque pointer so this header needs no CUDA headers. */
typedef void *acd_stream;

/* Optional allocator used for the workspace (e.g. a caller's caching pool).
 * alloc returns NULL on failure. */
typedef void *(*acd_alloc_fn)(size_t bytes, void *user);
typedef void (*acd_free_fn)(void *ptr, void *user);

/* ---- elementwise op codes ---------------------------------------------- */
typedef enum {
  ACD_EXP = 0, ACD_LOG = 1, ACD_SQRT = 2, ACD_ABS = 3, ACD_FLOOR = 4,
  ACD_CEIL = 5, ACD_ROUND = 6, ACD_ERF = 7, ACD_TANH = 8, ACD_SIGMOID = 9,
  ACD_RELU = 10, ACD_SIN = 11, ACD_COS = 12, ACD_NEG = 13, ACD_SQUARE = 14,
  ACD_COPY = 15
} acd_unary_op;

typedef enum {
  ACD_ADD = 0, ACD_SUB = 1, ACD_MUL = 2, ACD_DIV = 3,
  ACD_MAX = 4, ACD_MIN = 5, ACD_POW = 6,
  ACD_GT = 7, ACD_LT = 8, ACD_EQ = 9, ACD_NE = 10, ACD_GE = 11, ACD_LE = 12,
  ACD_RSUB = 13, ACD_RDIV = 14 /* scalar-only: s - x, s / x */
} acd_binary_op;

/* Fused elementwise chains.  Each evaluates the listed R expression with one
 * rounding per R operator, in the tensor dtype, so the result is bit-identical
 * to issuing the operators one by one. */
typedef enum {
  ACD_FUSED_SCALE_ADD_EXP_NEG_SQUARE = 0, /* x*p0 + exp(-(x^2))          (one input)  */
  ACD_FUSED_ADD_RELU = 1,                 /* relu(a + b)                 (two inputs) */
  ACD_FUSED_TANH_SCALE = 2                /* tanh(x) * p0                (one input)  */
} acd_fused_op;

/* ---- reduction op codes ------------------------------------------------ */
typedef enum {
  ACD_RED_SUM = 0, ACD_RED_MEAN = 1, ACD_RED_MAX = 2, ACD_RED_MIN = 3,
  ACD_RED_PROD = 4, ACD_RED_VAR = 5, /* sample variance, divisor n-1 */
  ACD_RED_COUNT = 6,                 /* number of non-zero elements */
  /* any / all with R's logical rules: an element is TRUE when non-zero,
   * NA when NaN (or an NA integer, INT_MIN); any = TRUE if some element is
   * TRUE, else NA if some is NA, else FALSE; all = FALSE if some element is
   * FALSE, else NA if some is NA, else TRUE.  Written as 1 / 0 / NA
   * (INT32_MIN, R's NA_LOGICAL) to an int32 output.  The reference converts
   * the tensor on the host (any.gpuTensor / all.gpuTensor,
   * R/gpuTensor.R:2178-2206). */
  ACD_RED_ANY = 7, ACD_RED_ALL = 8
} acd_reduce_op;

typedef enum { ACD_ARGMAX = 0, ACD_ARGMIN = 1 } acd_arg_op;
typedef enum { ACD_CUMSUM = 0, ACD_CUMPROD = 1 } acd_scan_op;

/* ---- context ----------------------------------------------------------- */
const char *acd_version(void);
const char *acd_last_error(void);
const char *acd_status_string(acd_status s);

/* Device queries, replacing gpu_available / gpu_info / gpu_memory_available
 * (src/RcppInterface.cpp:7-20 over src/cuda_utils.h:17-103).  They need no
 * context and do not fail: without a driver or a device they report 0 or a
 * message.
 *   acd_gpu_available          1 if device 0 answers a properties query
 *   acd_gpu_info               "Found N CUDA device(s):\n" then one line
 *                              "  Device i: <name> (Compute M.m) - <MiB> MB\n"
 *                              per device; writes at most len-1 bytes plus a
 *                              NUL into buf and returns the full length
 *   acd_gpu_memory_available   free bytes on the current device */
int32_t acd_gpu_available(void);
int64_t acd_gpu_info(char *buf, int64_t len);
double acd_gpu_memory_available(void);

/* Creates a context on `device` (the current device is left unchanged). */
acd_status acd_ctx_create(int device, acd_ctx **out);
acd_status acd_ctx_destroy(acd_ctx *ctx);
/* Replaces the workspace allocator (NULL, NULL restores cudaMalloc/cudaFree).
 * Frees the current workspace; safe only when no call on `ctx` is in flight. */
acd_status acd_ctx_set_allocator(acd_ctx *ctx, acd_alloc_fn alloc, acd_free_fn free_fn, void *user);
/* Reads and clears the device status word (synchronises `stream`).
 * Returns ACD_ERR_DEVICE and fills *code when a kernel reported an error:
 * 1 = the scan's look-back wait expired, 2 = a wait of the TMA transpose
 * pipeline expired, 3 = the TMA load wait of the cluster softmax expired,
 * 4 = the row softmax's wait for a lane group's statistics expired. */
acd_status acd_ctx_check(acd_ctx *ctx, acd_stream stream, int32_t *code);
/* Test hook for the bounded look-back wait of the scan: when `tile` >= 0,
 * the scan kernel's tile with that index never publishes its prefix, so the
 * tile after it gives up after `timeout_ns` and raises the status word.
 * tile < 0 disables the hook.  timeout_ns <= 0 restores the default (1 s). */
acd_status acd_ctx_set_scan_fault(acd_ctx *ctx, int64_t tile, int64_t timeout_ns);

/* ---- shape helpers (host only, no CUDA) -------------------------------- */
/* acediaR broadcast rule (src/gpuTensor.h:248-340): dims are aligned from the
 * leading side; the shorter shape is tried at every offset, first fit wins. */
acd_status acd_broadcast_shape(int32_t a_ndim, const int64_t *a_shape, int32_t b_ndim,
                               const int64_t *b_shape, int32_t *out_ndim, int64_t *out_shape);
/* Strides of `in` expanded to `out_ndim`/`out_shape` under the same rule
 * (stride 0 on broadcast dims), cf. compute_broadcast_strides
 * (src/TensorArithmetic.cpp:240-292). */
acd_status acd_broadcast_strides(int32_t in_ndim, const int64_t *in_shape, const int64_t *in_stride,
                                 int32_t out_ndim, const int64_t *out_shape, int64_t *out_stride);

/* ---- elementwise ------------------------------------------------------- */
/* out = op(in).  out and in have the same shape; in may be any strided view. */
acd_status acd_unary(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in, acd_stream stream);
/* out = a op b with acediaR broadcasting.  Comparisons (GT..LE) write 0/1 as
 * bool or in the input dtype, whichever `out` declares. */
acd_status acd_binary(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *a,
                      const acd_desc *b, acd_stream stream);
/* out = in op s (s cast to the tensor dtype first, as elementwise_scalar_kernel
 * does, src/kernels/tensor_kernels.cu:33-39).  ACD_POW with s == 2 is x*x. */
acd_status acd_scalar(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in, double s,
                      acd_stream stream);
/* Fused chains (acd_fused_op).  `b` is NULL for one-input chains. */
acd_status acd_fused(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *a,
                     const acd_desc *b, double p0, acd_stream stream);
/* ---- assembly and mutation (views of acd_desc) ------------------------- */
/* Host only: the view of `in` restricted to start[d] .. start[d]+count[d]-1
 * (0-based) on every axis, same rank.  `[.gpuTensor` (R/gpuTensor.R:719-811)
 * extracts such ranges by a host round trip; here the view is zero-copy and
 * acd_copy materialises it. */
acd_status acd_slice_desc(const acd_desc *in, const int64_t *start, const int64_t *count, acd_desc *out);
/* out = value on every element of a view (value converted as by acd_convert).
 * With acd_slice_desc this is tensor_slice_set_scalar_unified
 * (src/TensorMutation.cpp:439-492, src/kernels/tensor_slice_update.cu). */
acd_status acd_fill(acd_ctx *ctx, const acd_desc *out, double value, acd_stream stream);
/* x[mask] <- value in place; mask is a bool view of x's shape.
 * Replaces tensor_mask_set_scalar_unified (src/TensorMutation.cpp:577-623). */
acd_status acd_mask_fill(acd_ctx *ctx, const acd_desc *x, const acd_desc *mask, double value,
                         acd_stream stream);
/* out = concatenation of ins[0..n-1] along `axis` (0-based); every other
 * extent equal.  Replaces tensor_concat_unified (src/TensorMutation.cpp:167-273,
 * concat_kernel src/kernels/tensor_kernels.cu:298-341). */
acd_status acd_concat(acd_ctx *ctx, const acd_desc *out, const acd_desc *const *ins, int32_t n, int32_t axis,
                      acd_stream stream);
/* out = the n equal-shaped inputs stacked along a new axis `axis` (0-based,
 * 0..rank).  Replaces tensor_stack_unified (src/TensorMutation.cpp:275-331). */
acd_status acd_stack(acd_ctx *ctx, const acd_desc *out, const acd_desc *const *ins, int32_t n, int32_t axis,
                     acd_stream stream);
/* out(c) = in(c / reps) per axis: every element repeated reps[d] times along
 * axis d.  Replaces tensor_repeat_unified (src/TensorMutation.cpp:333-385,
 * repeat_kernel src/kernels/tensor_kernels.cu:381-413). */
acd_status acd_repeat(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, const int64_t *reps,
                      acd_stream stream);
/* out = in padded by before[d] elements in front and
 * out.shape[d] - in.shape[d] - before[d] behind on each axis.  mode 0:
 * `value`; 1: reflect with the edge included (the reference's rule, padding
 * at most the axis length); 2: replicate the edge.  Replaces
 * tensor_pad_unified (src/TensorMutation.cpp:387-437, pad_kernel
 * src/kernels/tensor_kernels.cu:415-466). */
acd_status acd_pad(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, const int64_t *before, int32_t mode,
                   double value, acd_stream stream);

/* ---- random tensors --------------------------------------------------- */
/* Fills a contiguous float32/float64 view: dist 0 = uniform on [a, b),
 * dist 1 = normal with mean a and sd b.  Element i takes counter position
 * offset + i of Philox4x32-10 keyed by `seed`, so a shard generated with
 * offset = its first global index holds exactly the values of the whole
 * tensor.  Replaces rand_tensor / rnorm_tensor (src/TensorRandom.cpp:42-224),
 * which draw from cuRAND seeded with time(NULL). */
acd_status acd_rand(acd_ctx *ctx, const acd_desc *out, int32_t dist, double a, double b, uint64_t seed,
                    uint64_t offset, acd_stream stream);

/* dtype conversion, out = as.<dtype>(in) over any two views of one shape.
 * Replaces tensor_to_dtype_unified (src/TensorDataAccess.cpp:152-190), whose
 * kernel is type_conversion_kernel (src/kernels/tensor_kernels.cu:52-57,
 * a static_cast per element, src/kernels/kernel_utils.cuh:11).  Base R's
 * as.* rules: to int32/int64 values truncate toward zero and NaN or values
 * out of range become NA (INT32_MIN / INT64_MIN); NA integers become NaN in
 * float32/float64; bool stores x != 0.  Equal dtypes copy. */
acd_status acd_convert(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, acd_stream stream);

/* out = in, any strides on both sides (contiguous(), strided copy). */
acd_status acd_copy(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, acd_stream stream);
/* nbytes of src copied to dst0 and, when dst1 is not NULL, to dst1 too;
 * 16-byte aligned buffers, nbytes a multiple of 16.  Plain streaming: the
 * benchmark times it as the ceiling of a kernel that reads once and writes
 * once or twice (the strided-views step writes y and z for each x). */
acd_status acd_copy_fanout(acd_ctx *ctx, void *dst0, void *dst1, const void *src, int64_t nbytes,
                           acd_stream stream);

/* ---- reductions -------------------------------------------------------- */
/* Reduces the axes whose bit is set in axes_mask (bit k = axis k, 0-based).
 * out holds prod(shape[k] for unreduced k) elements, in column-major order of
 * the unreduced axes (keep.dims only changes the shape the caller reports).
 * Output dtype: the input dtype, or FLOAT64 for FLOAT32/FLOAT64 input
 * (wider result); COUNT writes INT32 or INT64; SUM of INT32 writes INT32
 * (NA = INT32_MIN on overflow, as R) or INT64. */
acd_status acd_reduce(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in,
                      uint32_t axes_mask, acd_stream stream);
/* Fused single pass over all elements: out_sum and out_var are one-element
 * descriptors (either may be NULL).  Sum and sample variance as acd_reduce. */
acd_status acd_sum_var(acd_ctx *ctx, const acd_desc *out_sum, const acd_desc *out_var,
                       const acd_desc *in, acd_stream stream);
/* Index of the first maximum (minimum) along `axis`, or over all elements in
 * column-major order when axis < 0.  out dtype INT32 or INT64.  Indices are
 * 1-based when one_based != 0 (which.max), else 0-based (the reference's
 * axis kernel, src/kernels/tensor_kernels.cu:720-807).  NaN never wins. */
acd_status acd_arg_reduce(acd_ctx *ctx, int32_t op, const acd_desc *out_index,
                          const acd_desc *out_value, const acd_desc *in, int32_t axis,
                          int32_t one_based, acd_stream stream);

/* ---- scans and softmax ------------------------------------------------- */
/* Cumulative sum/product along `axis`, or over the column-major flattened
 * tensor when axis < 0 (cumsum.gpuTensor, R/gpuTensor.R:2234-2277).
 * Accumulates in float64 and rounds each output once to the tensor dtype. */
acd_status acd_scan(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in, int32_t axis,
                    acd_stream stream);
/* exp(x - max) / sum(exp(x - max)) along `axis`; axis < 0 normalises the
 * whole tensor (tensor_softmax_*, src/kernels/tensor_ops.cu:826-846). */
acd_status acd_softmax(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, int32_t axis,
                       acd_stream stream);

/* Cumulative sum/product with acd_scan's semantics, for callers that cannot
 * allocate device memory (no context, no workspace): the scratch is a static
 * 8 MiB device array held by every GPU that loads this library.  With
 * interleaved lanes the additions run in another order than acd_scan's, so
 * the two agree within rounding (tested to 1e-5 / 1e-12 relative).  Problems
 * whose scratch would not fit return ACD_ERR_UNSUPPORTED: about 1.7e9
 * elements along a contiguous axis; with interleaved lanes 516 (float32) or
 * 260 (float64) bytes per tile of 32 x 256 or 16 x 512 lane-steps, however
 * many of its lanes are real (1.3e8 float32 elements when the lane count is a
 * multiple of 32, 8e6 with 2 lanes).  Runs on the current device; the first
 * call on a device looks up the array's device address and keeps it for the
 * process, so make that call before any stream capture and do not use the
 * entry point after a cudaDeviceReset.  Calls that overlap on the GPU race on
 * the shared array.  This entry point has no counterpart in the reference. */
acd_status acd_scan_noalloc(int32_t op, const acd_desc *out, const acd_desc *in, int32_t axis, acd_stream stream);

/* The elementwise chain + reduction configuration in one pass.  For float64
 * contiguous a and b of n elements, writes outs[0..4] = a + b, a * b,
 * exp(a), sigmoid(b), sqrt(a) (each bit-identical to acd_binary / acd_unary
 * of that operator) and, from the same registers, stats[3k], stats[3k+1],
 * stats[3k+2] = sum, mean, sample variance of outs[k] (device float64[15])
 * and which_max[0] = which.max(outs[0]) (1-based, first index; device
 * int64[1]).  Replaces five elementwise calls and sixteen reductions
 * (R's `+`, `*`, exp, sigmoid, sqrt, then sum/mean/var and which.max,
 * R/gpuTensor.R; src/kernels/tensor_ops.cu:785-880); a and b are read once. */
acd_status acd_chain5_stats(acd_ctx *ctx, const acd_desc *a, const acd_desc *b, const acd_desc *const *outs,
                            double *stats, int64_t *which_max, acd_stream stream);

/* ---- sharded partials (multi-GPU global sum/var and argmax) ------------- */
/* Writes this shard's partial statistics of all elements of `in` to the
 * device array `stats` (float64[4]: n, shift, sum(x-shift), sum((x-shift)^2)),
 * with shift = first element of the shard. */
acd_status acd_stats_partial(acd_ctx *ctx, double *stats, const acd_desc *in, acd_stream stream);
/* Argmax along `axis` written as order-preserving 64-bit keys (int64 array
 * with one key per output): key = (ordered value bits << 32) | (0xFFFFFFFF - idx),
 * sign bit flipped, so a signed MAX all-reduce selects the largest value and,
 * among equal values, the smallest global index.  idx = local index +
 * index_base.  FLOAT32 input only. */
acd_status acd_argmax_keys(acd_ctx *ctx, int64_t *keys, const acd_desc *in, int32_t axis,
                           int64_t index_base, acd_stream stream);
/* The elementwise chain out = in*p0 + exp(-(in^2)) (bit-identical to
 * acd_fused with ACD_FUSED_SCALE_ADD_EXP_NEG_SQUARE) together with, from the
 * same pass over out, the statistics row of acd_stats_partial(out) and the
 * keys of acd_argmax_keys(out, axis 0, index_base).  It replaces those three
 * calls on the strided-views step (R/gpuTensor.R:2032-2042 for x^2 and the
 * Ops group; src/kernels/tensor_ops.cu:785-880 for the statistics and the
 * argmax): out is still written, but not read again.  FLOAT32.  Contiguous,
 * 16-byte aligned data with shape[0] a multiple of 4 take one kernel; other
 * views run the three calls. */
acd_status acd_fused_stats_keys(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, double p0, double *stats,
                                int64_t *keys, int64_t index_base, acd_stream stream);
/* y = contiguous(in) for the view `in`, then z, the statistics row and the
 * argmax keys of acd_fused_stats_keys(z, y, ...): the strided-views step's
 * permute -> contiguous (R/gpuTensor.R:1544-1556, src/gpuTensor.h:723-769),
 * elementwise chain, statistics and argmax keys as one call.  y and z are
 * contiguous FLOAT32 of in's shape.  When `in` is a transpose of y (y
 * contiguous along axis 0, `in` contiguous along another axis after
 * collapsing, 16-byte aligned data and strides, both transposed extents at
 * least 64) it is one kernel that reads `in` once and writes y and z once;
 * otherwise the copy and then acd_fused_stats_keys.  Results are identical
 * either way (y, z and keys bit for bit; the moments to summation order). */
acd_status acd_permute_fused_stats_keys(acd_ctx *ctx, const acd_desc *y, const acd_desc *z, const acd_desc *in,
                                        double p0, double *stats, int64_t *keys, int64_t index_base,
                                        acd_stream stream);
/* One exchange for the sharded step.  buf is an int64 array of nkeys + 6 *
 * world entries: the argmax keys, then one statistics row per rank (the
 * float64 row of acd_stats_partial stored as bit patterns).  Each rank
 * passes keys = buf and stats = (double *)(buf + nkeys + 6 * rank) to
 * acd_fused_stats_keys; the other ranks' rows hold INT64_MIN (the bit
 * pattern of -0.0, the smallest int64), so a single int64 MAX all-reduce
 * over the whole buffer selects every key's winner and copies every rank's
 * row to all ranks.  acd_shard_exchange_init sets all rows to INT64_MIN
 * once; acd_shard_finish then decodes the keys into out_index (as
 * acd_argmax_keys_decode), merges the rows in rank order into
 * sum_var[0] = sum and sum_var[1] = sample variance (device float64[2]),
 * and sets the rows back to INT64_MIN for the next exchange.  The
 * reference computes the global sum, var and argmax of one device's tensor
 * (src/kernels/tensor_ops.cu:785-880); the exchange has no counterpart. */
acd_status acd_shard_exchange_init(acd_ctx *ctx, int64_t *buf, int64_t nkeys, int32_t world, acd_stream stream);
acd_status acd_shard_finish(acd_ctx *ctx, int64_t *buf, int64_t nkeys, int32_t world, const acd_desc *out_index,
                            double *sum_var, int32_t one_based, acd_stream stream);
/* Decodes keys back to indices (INT32/INT64 out, 1-based when one_based). */
acd_status acd_argmax_keys_decode(acd_ctx *ctx, const acd_desc *out_index, const int64_t *keys,
                                  int32_t one_based, acd_stream stream);

#ifdef __cplusplus
}
#endif

#endif /* ACD_H */
