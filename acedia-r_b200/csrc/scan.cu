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
//
// Interleaved lanes (L > 1: the scanned axis is not the innermost one, so
// neighbouring lanes sit next to each other in memory) take a three-kernel
// reduce-then-scan instead, which has no waits between CTAs:
//   1. k_lane_reduce: one warp per (lane block, step segment) task reads its
//      segment row by row, last row first (LT lanes x G step phases per warp,
//      so a warp load covers G rows of LT lanes) and writes one total per
//      lane;
//   2. k_lane_seg_scan: one CTA per (chain, lane) turns the segment totals
//      into exclusive prefixes in place;
//   3. k_lane_apply: the same warps re-read their segments and write
//      prefix + running sum.
// The traffic is 3 tensor passes (read, read, write) against 2 for the
// chained scan, but the chained scan's look-back frontier advances only one
// 32-tile window per round trip, which caps it far below HBM speed when a
// tile carries LT lane totals.
#include "scan_kernel.cuh"

namespace acd {

struct LaneArgs {
  const void *in;
  void *out;
  int64_t L, R, O;
  int64_t sl, sr, so;  // input strides
  int64_t ol, orr, oo; // output strides
  int64_t lblocks;     // lane blocks of LT lanes
  int64_t nchains;     // lblocks * O
  int64_t SB;          // row blocks (G steps each) per segment
  int64_t nseg;        // segments per chain
  double *seg;         // [nchains][LT][nseg] totals, then exclusive prefixes
};

constexpr int kLaneU = 16;  // row blocks loaded per batch

// Task t (segment-major, so consecutive warps read neighbouring lane blocks
// of the same rows) -> chain, segment and this thread's lane.
template <int LT>
struct LaneTask {
  int64_t s, chain, o, l, rs, re;
  __device__ __forceinline__ LaneTask(const LaneArgs &a, int64_t t, int li) {
    constexpr int G = 32 / LT;
    s = t / a.nchains;
    chain = t - s * a.nchains;
    o = chain / a.lblocks;
    l = (chain - o * a.lblocks) * LT + li;
    rs = s * a.SB * G;
    re = min(a.R, rs + a.SB * G);
  }
};

template <typename T, bool PROD, int LT>
__global__ void __launch_bounds__(256) k_lane_reduce(LaneArgs a) {
  constexpr int G = 32 / LT, U = kLaneU;
  const double ident = PROD ? 1.0 : 0.0;
  const int wl = threadIdx.x & 31, li = wl % LT, g = wl / LT;
  const int64_t ntask = a.nchains * a.nseg;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t step = (int64_t)G * a.sr;
  for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < ntask; t += nw) {
    const LaneTask<LT> k(a, t, li);
    double acc = ident;
    if (k.l < a.L && k.rs + g < k.re) {
      // the segment is read from its last row back to its first, so the rows
      // this pass leaves in L2 are the segments' first rows, the ones
      // k_lane_apply reads first
      int64_t n = (k.re - k.rs - g + G - 1) / G;
      const int64_t last = (k.rs + g + (n - 1) * G) * a.sr;
      const T *p = static_cast<const T *>(a.in) + k.o * a.so + k.l * a.sl + last;
      for (; n >= U; n -= U) {
        T v[U];
#pragma unroll
        for (int j = 0; j < U; ++j) v[j] = p[-j * step];
#pragma unroll
        for (int j = 0; j < U; ++j) acc = combine<PROD>(acc, (double)v[j]);
        if (n > U) p -= U * step;
      }
      for (; n > 0; --n) {
        acc = combine<PROD>(acc, (double)*p);
        if (n > 1) p -= step;
      }
    }
#pragma unroll
    for (int d = LT; d < 32; d <<= 1) acc = combine<PROD>(acc, __shfl_xor_sync(0xffffffffu, acc, d));
    if (g == 0) a.seg[(k.chain * LT + li) * a.nseg + k.s] = acc;
  }
}

// Exclusive scan, in place, of each of `nrows` rows of `nseg` (<= 4096)
// segment totals: 1024 threads x 4 consecutive items (few rows, so the
// parallelism has to come from within a row).
template <bool PROD>
__global__ void __launch_bounds__(1024) k_lane_seg_scan(double *seg, int64_t nrows, int nseg) {
  constexpr int IPT = 4, NW = 32;
  __shared__ double s_warp[NW];
  const double ident = PROD ? 1.0 : 0.0;
  const int wl = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int i0 = threadIdx.x * IPT;
  for (int64_t row = blockIdx.x; row < nrows; row += gridDim.x) {
    double *p = seg + row * nseg;
    double v[IPT];
    double tot = ident;
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      v[j] = (i0 + j < nseg) ? p[i0 + j] : ident;
      tot = combine<PROD>(tot, v[j]);
    }
    double x = tot;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, x, d);
      if (wl >= d) x = combine<PROD>(y, x);
    }
    if (wl == 31) s_warp[w] = x;
    __syncthreads();
    if (w == 0) {  // exclusive scan of the 32 warp totals
      const double t = s_warp[wl];
      double u = t;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, u, d);
        if (wl >= d) u = combine<PROD>(y, u);
      }
      double e = __shfl_up_sync(0xffffffffu, u, 1);
      s_warp[wl] = wl == 0 ? ident : e;
    }
    __syncthreads();
    double run = s_warp[w];
    double prev = __shfl_up_sync(0xffffffffu, x, 1);
    if (wl > 0) run = combine<PROD>(run, prev);
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      if (i0 + j < nseg) p[i0 + j] = run;
      run = combine<PROD>(run, v[j]);
    }
    __syncthreads();
  }
}

template <typename T, bool PROD, int LT>
__global__ void __launch_bounds__(256) k_lane_apply(LaneArgs a) {
  constexpr int G = 32 / LT, U = kLaneU;
  const double ident = PROD ? 1.0 : 0.0;
  const int wl = threadIdx.x & 31, li = wl % LT, g = wl / LT;
  const int64_t ntask = a.nchains * a.nseg;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t step = (int64_t)G * a.sr, ostep = (int64_t)G * a.orr;
  for (int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < ntask; t += nw) {
    const LaneTask<LT> k(a, t, li);
    const bool lok = k.l < a.L;
    const int64_t lc = lok ? k.l : 0;  // lanes past L read lane 0 and discard it
    double carry = a.nseg > 1 ? a.seg[(k.chain * LT + li) * a.nseg + k.s] : ident;
    const T *p = static_cast<const T *>(a.in) + k.o * a.so + lc * a.sl + (k.rs + g) * a.sr;
    T *q = static_cast<T *>(a.out) + k.o * a.oo + lc * a.ol + (k.rs + g) * a.orr;
    const int64_t nfull = (k.re - k.rs) / G;          // row blocks with all G steps present
    const int64_t nb = (k.re - k.rs + G - 1) / G;     // all row blocks
    int64_t b = 0;
    for (; b + U <= nfull; b += U, p += U * step, q += U * ostep) {
      T v[U];
#pragma unroll
      for (int j = 0; j < U; ++j) v[j] = p[j * step];
#pragma unroll
      for (int j = 0; j < U; ++j) {
        double x = lok ? (double)v[j] : ident;
#pragma unroll
        for (int d = 1; d < G; d <<= 1) {
          const double y = __shfl_up_sync(0xffffffffu, x, d * LT);
          if (g >= d) x = combine<PROD>(y, x);
        }
        if (lok) q[j * ostep] = (T)combine<PROD>(carry, x);
        if constexpr (G == 1)
          carry = combine<PROD>(carry, x);
        else
          carry = combine<PROD>(carry, __shfl_sync(0xffffffffu, x, (G - 1) * LT + li));
      }
    }
    for (; b < nb; ++b, p += step, q += ostep) {
      const bool ok = lok && k.rs + b * G + g < k.re;
      double x = ok ? (double)*p : ident;
#pragma unroll
      for (int d = 1; d < G; d <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, x, d * LT);
        if (g >= d) x = combine<PROD>(y, x);
      }
      if (ok) *q = (T)combine<PROD>(carry, x);
      carry = combine<PROD>(carry, __shfl_sync(0xffffffffu, x, (G - 1) * LT + li));
    }
  }
}

template <typename T, bool PROD, int LT>
static acd_status launch_lane_scan_lt(acd_ctx *ctx, LaneArgs a, cudaStream_t s) {
  constexpr int G = 32 / LT, U = kLaneU;
  a.lblocks = (a.L + LT - 1) / LT;
  a.nchains = a.lblocks * a.O;
  const int64_t RB = (a.R + G - 1) / G;
  // about one task per resident warp, at most 4096 segments per chain and
  // at least U row blocks per segment
  const int64_t target = (int64_t)ctx->sm_count * 64;
  int64_t nseg = (target + a.nchains - 1) / a.nchains;
  if (nseg > 4096) nseg = 4096;
  if (nseg < 1) nseg = 1;
  int64_t SB = (RB + nseg - 1) / nseg;
  if (SB < U) SB = U;
  SB = (SB + U - 1) / U * U;
  a.SB = SB;
  a.nseg = (RB + SB - 1) / SB;
  const int64_t ntask = a.nchains * a.nseg;
  if (a.nseg > 1) {
    void *scratch;
    ACD_TRY(get_scratch(ctx, (size_t)(a.nchains * LT * a.nseg) * sizeof(double), s, &scratch));
    a.seg = static_cast<double *>(scratch);
    k_lane_reduce<T, PROD, LT>
        <<<persistent_grid(ctx, k_lane_reduce<T, PROD, LT>, 256, 0, (ntask + 7) / 8), 256, 0, s>>>(a);
    const int64_t nrows = a.nchains * LT;
    const int sg = (int)(nrows < (int64_t)ctx->sm_count * 8 ? nrows : (int64_t)ctx->sm_count * 8);
    k_lane_seg_scan<PROD><<<sg, 1024, 0, s>>>(a.seg, nrows, (int)a.nseg);
  }
  k_lane_apply<T, PROD, LT><<<persistent_grid(ctx, k_lane_apply<T, PROD, LT>, 256, 0, (ntask + 7) / 8), 256, 0, s>>>(a);
  return ACD_OK;
}

template <typename T, bool PROD>
static acd_status launch_lane_scan(acd_ctx *ctx, const ScanArgs &sa, cudaStream_t s) {
  LaneArgs a{};
  a.in = sa.in;
  a.out = sa.out;
  a.L = sa.L;
  a.R = sa.R;
  a.O = sa.O;
  a.sl = sa.sl;
  a.sr = sa.sr;
  a.so = sa.so;
  a.ol = sa.ol;
  a.orr = sa.orr;
  a.oo = sa.oo;
  if (a.L > 16) return launch_lane_scan_lt<T, PROD, 32>(ctx, a, s);
  if (a.L > 8) return launch_lane_scan_lt<T, PROD, 16>(ctx, a, s);
  if (a.L > 4) return launch_lane_scan_lt<T, PROD, 8>(ctx, a, s);
  if (a.L > 2) return launch_lane_scan_lt<T, PROD, 4>(ctx, a, s);
  return launch_lane_scan_lt<T, PROD, 2>(ctx, a, s);
}

template <typename T, bool PROD>
static acd_status launch_scan(acd_ctx *ctx, ScanArgs a, cudaStream_t s) {
  if (a.L > 1) return launch_lane_scan<T, PROD>(ctx, a, s);
  constexpr int LT = 1, SEG1 = 16;
  const int RT = 256 * SEG1;
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
  k_scan<T, PROD, 1, SEG1><<<(int)a.ntiles, 256, 0, s>>>(a);
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
