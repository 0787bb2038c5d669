// Tensor assembly and mutation on column-major views: slices, concat, stack,
// repeat and pad.
//
// Reference: src/TensorMutation.cpp (tensor_concat_unified 167-273,
// tensor_stack_unified 275-331, tensor_repeat_unified 333-385,
// tensor_pad_unified 387-437, slice and mask assignment 439-623) with the
// kernels concat_kernel / stack_kernel / repeat_kernel / pad_kernel
// (src/kernels/tensor_kernels.cu:298-467) and src/kernels/tensor_slice_update.cu.
// The reference gathers every output element through int32 coordinates and
// cudaMallocs its metadata per call.  Here a slice is a view (offset, extents,
// strides), so concat and stack are one strided copy per input into a view of
// the output, slice assignment is a copy or fill into a view of the
// destination, and repeat is one copy from a broadcast view (stride 0 on a
// split axis) into a split view of the output.  Only pad needs its own
// gather kernel (reflect and replicate map each coordinate separately).
#include "common.cuh"
#include "ops.cuh"

namespace acd {

namespace {

constexpr int kPadThreads = 256;

struct PadArgs {
  int32_t ndim;
  int32_t mode;  // 0 constant, 1 reflect (edge included), 2 replicate
  int64_t oshape[ACD_MAX_DIMS];
  int64_t ost[ACD_MAX_DIMS];
  int64_t ishape[ACD_MAX_DIMS];
  int64_t ist[ACD_MAX_DIMS];
  int64_t before[ACD_MAX_DIMS];
};

// out(c) = in(c - before) inside, the pad rule outside.  Output-driven, runs
// of 4 consecutive elements along axis 0 per thread, int64 coordinates.
template <typename T>
__global__ void __launch_bounds__(kPadThreads) k_pad(T *__restrict__ out, const T *__restrict__ in, PadArgs a,
                                                     int64_t n, T value) {
  constexpr int RUN = 4;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = tid * RUN; base < n; base += nth * RUN) {
    int64_t c[ACD_MAX_DIMS];
    int64_t rem = base;
    for (int d = 0; d < a.ndim; ++d) {
      c[d] = rem % a.oshape[d];
      rem /= a.oshape[d];
    }
    for (int r = 0; r < RUN && base + r < n; ++r) {
      int64_t oo = 0, io = 0;
      bool pad = false;
      for (int d = 0; d < a.ndim; ++d) {
        oo += c[d] * a.ost[d];
        int64_t k = c[d] - a.before[d];
        const int64_t m = a.ishape[d];
        if (k < 0 || k >= m) {
          pad = true;
          if (a.mode == 1)
            k = k < 0 ? -k - 1 : 2 * m - k - 1;
          else
            k = k < 0 ? 0 : m - 1;
        }
        io += k * a.ist[d];
      }
      out[oo] = (pad && a.mode == 0) ? value : in[io];
      for (int d = 0; d < a.ndim; ++d) {  // next element in column-major order
        if (++c[d] < a.oshape[d]) break;
        c[d] = 0;
      }
    }
  }
}

template <typename T>
acd_status launch_pad(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, const PadArgs &a, double value,
                      cudaStream_t s) {
  const int64_t n = desc_numel(out);
  const int64_t work = ((n + 3) / 4 + kPadThreads - 1) / kPadThreads;
  const int grid = persistent_grid(ctx, k_pad<T>, kPadThreads, 0, work);
  k_pad<T><<<grid, kPadThreads, 0, s>>>(reinterpret_cast<T *>(desc_ptr(out)),
                                        reinterpret_cast<const T *>(desc_ptr(in)), a, n,
                                        convert_value<double, T>(value));
  return ACD_OK;
}

acd_status check_same_kind(const acd_desc *a, const acd_desc *b, const char *what) {
  if (a->dtype != b->dtype) return fail(ACD_ERR_DTYPE, "%s: all tensors must have the same dtype", what);
  return ACD_OK;
}

}  // namespace

}  // namespace acd

using namespace acd;

extern "C" {

acd_status acd_slice_desc(const acd_desc *in, const int64_t *start, const int64_t *count, acd_desc *out) {
  ACD_TRY(check_desc(in, "in"));
  if (!start || !count || !out) return fail(ACD_ERR_INVALID, "acd_slice_desc: null argument");
  acd_desc v = *in;
  for (int d = 0; d < in->ndim; ++d) {
    if (start[d] < 0 || count[d] < 0 || start[d] + count[d] > in->shape[d])
      return fail(ACD_ERR_SHAPE, "Index out of bounds for dimension %d with size %lld", d + 1,
                  (long long)in->shape[d]);
    v.offset += start[d] * in->stride[d];
    v.shape[d] = count[d];
  }
  *out = v;
  return ACD_OK;
}

acd_status acd_concat(acd_ctx *ctx, const acd_desc *out, const acd_desc *const *ins, int32_t n, int32_t axis,
                      acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_concat: null context");
  ACD_TRY(check_desc(out, "out"));
  if (!ins || n < 2) return fail(ACD_ERR_INVALID, "Need at least two tensors to concatenate");
  if (axis < 0 || axis >= out->ndim) return fail(ACD_ERR_AXIS, "axis out of range");
  int64_t total = 0;
  for (int t = 0; t < n; ++t) {
    ACD_TRY(check_desc(ins[t], "input"));
    ACD_TRY(check_same_kind(out, ins[t], "acd_concat"));
    if (ins[t]->ndim != out->ndim) return fail(ACD_ERR_SHAPE, "All tensors must have same number of dims");
    for (int d = 0; d < out->ndim; ++d)
      if (d != axis && ins[t]->shape[d] != out->shape[d]) return fail(ACD_ERR_SHAPE, "Non-concat dimensions must match");
    total += ins[t]->shape[axis];
  }
  if (total != out->shape[axis]) return fail(ACD_ERR_SHAPE, "acd_concat: output extent along the axis differs");
  int64_t start[ACD_MAX_DIMS] = {0}, count[ACD_MAX_DIMS];
  for (int d = 0; d < out->ndim; ++d) count[d] = out->shape[d];
  for (int t = 0; t < n; ++t) {
    count[axis] = ins[t]->shape[axis];
    if (count[axis] > 0) {
      acd_desc v;
      ACD_TRY(acd_slice_desc(out, start, count, &v));
      ACD_TRY(acd_copy(ctx, &v, ins[t], stream));
    }
    start[axis] += count[axis];
  }
  return ACD_OK;
}

acd_status acd_stack(acd_ctx *ctx, const acd_desc *out, const acd_desc *const *ins, int32_t n, int32_t axis,
                     acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_stack: null context");
  ACD_TRY(check_desc(out, "out"));
  if (!ins || n < 2) return fail(ACD_ERR_INVALID, "Need at least two tensors to stack");
  const int nd = ins[0]->ndim;
  if (nd + 1 != out->ndim) return fail(ACD_ERR_SHAPE, "acd_stack: output rank must be the input rank + 1");
  if (axis < 0 || axis > nd) return fail(ACD_ERR_AXIS, "axis out of range");
  if (out->shape[axis] != n) return fail(ACD_ERR_SHAPE, "acd_stack: output extent along the new axis differs");
  for (int t = 0; t < n; ++t) {
    ACD_TRY(check_desc(ins[t], "input"));
    ACD_TRY(check_same_kind(out, ins[t], "acd_stack"));
    if (ins[t]->ndim != nd) return fail(ACD_ERR_SHAPE, "All tensors must have identical shape for stack");
    for (int d = 0; d < nd; ++d)
      if (ins[t]->shape[d] != ins[0]->shape[d] || out->shape[d < axis ? d : d + 1] != ins[t]->shape[d])
        return fail(ACD_ERR_SHAPE, "All tensors must have identical shape for stack");
  }
  for (int t = 0; t < n; ++t) {
    // the output view with index t on the new axis, that axis dropped
    acd_desc v = *out;
    v.offset = out->offset + t * out->stride[axis];
    v.ndim = nd;
    for (int d = 0; d < nd; ++d) {
      const int od = d < axis ? d : d + 1;
      v.shape[d] = out->shape[od];
      v.stride[d] = out->stride[od];
    }
    ACD_TRY(acd_copy(ctx, &v, ins[t], stream));
  }
  return ACD_OK;
}

acd_status acd_repeat(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, const int64_t *reps,
                      acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_repeat: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  ACD_TRY(check_same_kind(out, in, "acd_repeat"));
  if (!reps) return fail(ACD_ERR_INVALID, "acd_repeat: null repeats");
  if (out->ndim != in->ndim) return fail(ACD_ERR_SHAPE, "repeats length must match tensor dims");
  // out axis d of extent r*m is split into (r: stride s_d, m: stride r*s_d);
  // the input is broadcast (stride 0) along the r part
  acd_desc vo = *out, vi = *in;
  int k = 0;
  for (int d = 0; d < in->ndim; ++d) {
    if (reps[d] <= 0) return fail(ACD_ERR_INVALID, "repeat counts must be positive");
    if (out->shape[d] != in->shape[d] * reps[d]) return fail(ACD_ERR_SHAPE, "acd_repeat: output extent differs on axis %d", d);
    if (reps[d] > 1) {
      if (k + 2 > ACD_MAX_DIMS) return fail(ACD_ERR_UNSUPPORTED, "acd_repeat: more than %d axes after splitting", ACD_MAX_DIMS);
      vo.shape[k] = reps[d];
      vo.stride[k] = out->stride[d];
      vi.shape[k] = reps[d];
      vi.stride[k] = 0;
      ++k;
      vo.shape[k] = in->shape[d];
      vo.stride[k] = reps[d] * out->stride[d];
      vi.shape[k] = in->shape[d];
      vi.stride[k] = in->stride[d];
      ++k;
    } else {
      if (k + 1 > ACD_MAX_DIMS) return fail(ACD_ERR_UNSUPPORTED, "acd_repeat: more than %d axes after splitting", ACD_MAX_DIMS);
      vo.shape[k] = out->shape[d];
      vo.stride[k] = out->stride[d];
      vi.shape[k] = in->shape[d];
      vi.stride[k] = in->stride[d];
      ++k;
    }
  }
  vo.ndim = vi.ndim = k;
  if (desc_numel(out) == 0) return ACD_OK;
  return acd_copy(ctx, &vo, &vi, stream);
}

acd_status acd_pad(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, const int64_t *before, int32_t mode,
                   double value, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_pad: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  ACD_TRY(check_same_kind(out, in, "acd_pad"));
  if (mode < 0 || mode > 2) return fail(ACD_ERR_INVALID, "Unsupported pad mode");
  if (!before) return fail(ACD_ERR_INVALID, "acd_pad: null padding");
  if (out->ndim != in->ndim) return fail(ACD_ERR_SHAPE, "pad_width must be matrix of ndims x 2");
  PadArgs a{};
  a.ndim = in->ndim;
  a.mode = mode;
  for (int d = 0; d < in->ndim; ++d) {
    const int64_t after = out->shape[d] - in->shape[d] - before[d];
    if (before[d] < 0 || after < 0) return fail(ACD_ERR_INVALID, "padding must be non-negative");
    if (mode != 0 && in->shape[d] == 0 && out->shape[d] > 0)
      return fail(ACD_ERR_SHAPE, "acd_pad: cannot reflect or replicate an empty axis");
    if (mode == 1 && (before[d] > in->shape[d] || after > in->shape[d]))
      return fail(ACD_ERR_SHAPE, "acd_pad: reflect padding larger than the axis (%lld) on axis %d",
                  (long long)in->shape[d], d + 1);
    a.oshape[d] = out->shape[d];
    a.ost[d] = out->stride[d];
    a.ishape[d] = in->shape[d];
    a.ist[d] = in->stride[d];
    a.before[d] = before[d];
  }
  if (desc_numel(out) == 0) return ACD_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (dtype_size(in->dtype)) {
    case 1: st = launch_pad<uint8_t>(ctx, out, in, a, value, s); break;
    case 4:
      st = in->dtype == ACD_FLOAT32 ? launch_pad<float>(ctx, out, in, a, value, s)
                                    : launch_pad<int32_t>(ctx, out, in, a, value, s);
      break;
    case 8:
      st = in->dtype == ACD_FLOAT64 ? launch_pad<double>(ctx, out, in, a, value, s)
                                    : launch_pad<int64_t>(ctx, out, in, a, value, s);
      break;
    default: return fail(ACD_ERR_DTYPE, "acd_pad: bad dtype");
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

}  // extern "C"
