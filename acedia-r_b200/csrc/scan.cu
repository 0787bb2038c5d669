// Cumulative sum / product along an axis, or over the column-major flattened
// tensor.
//
// Reference: cumsum.gpuTensor / cumprod.gpuTensor (R/gpuTensor.R:2234-2277)
// copy the whole tensor to the host and run base R's cumsum over the
// flattened vector.  Here a single-pass chained scan (decoupled look-back,
// Merrill & Garland 2016) runs on the device:
//   * the problem is (L lanes, R steps, O outer): element (l, r, o) at
//     l*sl + r*sr + o*so; each (lane block, o) pair is one chain of tiles
//     along r;
//   * CTAs take tiles from an atomic ticket, so every tile a CTA waits for
//     was started earlier (no deadlock whatever the residency);
//   * a tile publishes its aggregate, looks back over its predecessors'
//     aggregates until it finds an inclusive prefix, then publishes its own
//     inclusive prefix; flags carry the launch epoch so stale flags from
//     earlier launches never match and the state needs no clearing;
//   * every wait is bounded (globaltimer): on expiry the tile raises the
//     context status word, marks the launch aborted (later waiters give up
//     at once) and publishes anyway, so the kernel always terminates.
// Accumulation is float64 (a float64 sum per lane; R accumulates in long
// double and rounds each output once).
#include "scan_kernel.cuh"

namespace acd {

template <typename T, bool PROD>
static acd_status launch_scan(acd_ctx *ctx, ScanArgs a, cudaStream_t s) {
  constexpr int LTW = 128 / sizeof(T);  // lanes per tile when L > 1: 128-byte rows
  const int LT = a.L == 1 ? 1 : LTW;
  constexpr int SEG1 = 16, SEGW = 32;
  const int RT = LT == 1 ? 256 * SEG1 : (256 / LTW) * SEGW;
  a.lblocks = (a.L + LT - 1) / LT;
  a.rtiles = (a.R + RT - 1) / RT;
  a.ntiles = a.lblocks * a.O * a.rtiles;
  if (a.ntiles > 0x7fffffffLL) return fail(ACD_ERR_UNSUPPORTED, "scan: too many tiles");
  const size_t dbytes = (size_t)a.ntiles * LT * sizeof(double);
  const size_t ioff = (dbytes + 255) / 256 * 256;
  ACD_TRY(get_flags(ctx, (size_t)a.ntiles, s, &a.flags));
  void *scratch;
  ACD_TRY(get_scratch(ctx, ioff + dbytes, s, &scratch));
  char *base = static_cast<char *>(scratch);
  a.agg = reinterpret_cast<double *>(base);
  a.incl = reinterpret_cast<double *>(base + ioff);
  a.control = ctx->control;
  ctx->epoch = (ctx->epoch + 1) & 0x3fffffffu;
  if (ctx->epoch == 0) ctx->epoch = 1;
  a.epoch = ctx->epoch;
  a.fault_tile = ctx->scan_fault_tile;
  a.timeout_ns = ctx->scan_timeout_ns;
  if (LT == 1)
    k_scan<T, PROD, 1, SEG1><<<(int)a.ntiles, 256, 0, s>>>(a);
  else
    k_scan<T, PROD, LTW, SEGW><<<(int)a.ntiles, 256, 0, s>>>(a);
  return ACD_OK;
}

}  // namespace acd

using namespace acd;

extern "C" {

acd_status acd_scan(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in, int32_t axis,
                    acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_scan: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  if (op != ACD_CUMSUM && op != ACD_CUMPROD) return fail(ACD_ERR_INVALID, "acd_scan: bad op %d", op);
  if (!is_float(in->dtype) || out->dtype != in->dtype)
    return fail(ACD_ERR_DTYPE, "acd_scan: float32/float64 input and output of one dtype required");
  if (out->ndim != in->ndim) return fail(ACD_ERR_SHAPE, "acd_scan: output rank differs");
  for (int d = 0; d < in->ndim; ++d)
    if (out->shape[d] != in->shape[d]) return fail(ACD_ERR_SHAPE, "acd_scan: output extent differs on axis %d", d);
  if (axis >= in->ndim && in->ndim > 0) return fail(ACD_ERR_AXIS, "acd_scan: axis %d out of range", axis);
  const int64_t n = desc_numel(in);
  if (n == 0) return ACD_OK;
  ScanArgs a{};
  a.in = desc_ptr(in);
  a.out = desc_ptr(out);
  int64_t si[3] = {0, 0, 0}, so[3] = {0, 0, 0};
  if (axis < 0 || in->ndim == 0) {
    // flattened column-major order: both views must be contiguous
    if (!desc_is_contiguous(in) || !desc_is_contiguous(out))
      return fail(ACD_ERR_UNSUPPORTED, "acd_scan: flattened scan needs contiguous input and output");
    a.L = 1;
    a.R = n;
    a.O = 1;
    si[1] = so[1] = 1;
  } else {
    if (!split_axis(in, out, axis, a.L, a.R, a.O, si, so))
      return fail(ACD_ERR_UNSUPPORTED, "acd_scan: view not collapsible around the axis; make it contiguous first");
  }
  a.sl = si[0];
  a.sr = si[1];
  a.so = si[2];
  a.ol = so[0];
  a.orr = so[1];
  a.oo = so[2];
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  const bool prod = op == ACD_CUMPROD;
  if (in->dtype == ACD_FLOAT32)
    st = prod ? launch_scan<float, true>(ctx, a, s) : launch_scan<float, false>(ctx, a, s);
  else
    st = prod ? launch_scan<double, true>(ctx, a, s) : launch_scan<double, false>(ctx, a, s);
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

}  // extern "C"
