// acd_scan_noalloc: cumsum/cumprod for callers that cannot allocate device
// memory.
//
// Who needs it: callers that cannot call cudaMalloc.  An application whose
// own allocator has reserved (nearly) all device memory — a framework's
// caching pool, an R session sharing the GPU with such a framework — gets
// failures or fragmentation from a second allocator; latency-critical paths
// cannot take cudaMalloc's unbounded latency or cudaFree's device-wide
// synchronisation; and a stateless plugin interface has nowhere to keep the
// context object that owns acd_scan's workspace.  acd_scan needs such a
// context (acd_ctx_create allocates its control block, and the first scan
// grows its workspace); this entry point needs neither.
//
// Its scratch is one file-scope __device__ array of kNoAllocScratchBytes
// (8 MiB), which every GPU that loads the library holds until the process
// exits.  It has room for the tile flags, the per-tile aggregates and
// inclusive prefixes, and the ticket counters of the chained-scan kernel.
// Along a contiguous axis a tile is 4096 steps and costs 20 bytes: about 1.7
// billion elements.  With interleaved lanes a tile is 32 float32 lanes x 256
// steps (516 bytes) or 16 float64 lanes x 512 steps (260 bytes), whatever
// number of its lanes is real: about 130 million elements when the lane count
// is a multiple of the tile width, proportionally fewer for narrow lane counts
// (about 8 million float32 elements with 2 lanes).  A cumsum along the last
// axis of a 64 x 1048576 float32 matrix needs 4.2 MB.  Larger problems are
// rejected with ACD_ERR_UNSUPPORTED before anything is launched.
//
// Behaviour to know:
//   * the array's host-side name is not a device address: on the first call on
//     each device (with that device current) the entry point looks up the
//     address with cudaGetSymbolAddress and caches it for the life of the
//     process; make that first call before any stream capture, and do not
//     use the entry point after a cudaDeviceReset of that device (the cached
//     address would be stale);
//   * results have acd_scan's semantics; with interleaved lanes acd_scan runs
//     its reduce-then-scan kernels while this entry point runs the chained
//     scan, so the additions happen in another order and the results agree
//     within rounding, not bit for bit;
//   * every call shares the array and it keeps the last call's contents: each
//     call clears the counters and flags it relies on (cudaMemsetAsync on the
//     caller's stream) before launching;
//   * calls that overlap on the GPU race on the array — order them on one
//     stream or otherwise serialise them;
//   * a look-back wait that expires (it cannot in normal operation) leaves
//     the output undefined and is not reported by this entry point.
#include <mutex>

#include "scan_kernel.cuh"

namespace acd {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void *g_noalloc_addr[kNoAllocMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once).
static acd_status noalloc_base(void **out) {
  int dev = -1;
  ACD_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(ACD_ERR_UNSUPPORTED, "acd_scan_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return ACD_OK;
}

static size_t up256(size_t x) { return (x + 255) / 256 * 256; }

template <typename T, bool PROD>
static acd_status noalloc_launch(ScanArgs a, cudaStream_t s) {
  constexpr int LTW = 128 / sizeof(T);
  constexpr int SEG1 = 16, SEGW = 32;  // the tile shapes acd_scan uses
  const int LT = a.L == 1 ? 1 : LTW;
  const int RT = LT == 1 ? 256 * SEG1 : (256 / LTW) * SEGW;
  a.lblocks = (a.L + LT - 1) / LT;
  a.rtiles = (a.R + RT - 1) / RT;
  a.ntiles = a.lblocks * a.O * a.rtiles;
  const size_t ctl = up256(sizeof(Control));
  const size_t fl = up256((size_t)a.ntiles * sizeof(uint32_t));
  const size_t dd = up256((size_t)a.ntiles * LT * sizeof(double));
  const size_t need = ctl + fl + 2 * dd;
  if (a.ntiles > 0x7fffffffLL || need > kNoAllocScratchBytes)
    return fail(ACD_ERR_UNSUPPORTED,
                "acd_scan_noalloc: this scan needs %zu bytes of device scratch; the static maximum is %zu bytes "
                "(about 1.7 billion elements along a contiguous axis) - use acd_scan",
                need, kNoAllocScratchBytes);
  void *base;
  ACD_TRY(noalloc_base(&base));
  char *b = static_cast<char *>(base);
  a.control = reinterpret_cast<Control *>(b);
  a.flags = reinterpret_cast<uint32_t *>(b + ctl);
  a.agg = reinterpret_cast<double *>(b + ctl + fl);
  a.incl = reinterpret_cast<double *>(b + ctl + fl + dd);
  // counters, status and flags must start at zero; the flags then only need
  // one epoch value
  ACD_CUDA(cudaMemsetAsync(b, 0, ctl + fl, s));
  a.epoch = 1;
  a.fault_tile = -1;
  a.timeout_ns = 1000000000LL;
  if (LT == 1)
    k_scan<T, PROD, 1, SEG1><<<(int)a.ntiles, 256, 0, s>>>(a);
  else
    k_scan<T, PROD, LTW, SEGW><<<(int)a.ntiles, 256, 0, s>>>(a);
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

}  // namespace acd

using namespace acd;

extern "C" {

acd_status acd_scan_noalloc(int32_t op, const acd_desc *out, const acd_desc *in, int32_t axis, acd_stream stream) {
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  if (op != ACD_CUMSUM && op != ACD_CUMPROD) return fail(ACD_ERR_INVALID, "acd_scan_noalloc: bad op %d", op);
  if (!is_float(in->dtype) || out->dtype != in->dtype)
    return fail(ACD_ERR_DTYPE, "acd_scan_noalloc: float32/float64 input and output of one dtype required");
  if (out->ndim != in->ndim) return fail(ACD_ERR_SHAPE, "acd_scan_noalloc: output rank differs");
  for (int d = 0; d < in->ndim; ++d)
    if (out->shape[d] != in->shape[d])
      return fail(ACD_ERR_SHAPE, "acd_scan_noalloc: output extent differs on axis %d", d);
  if (axis >= in->ndim && in->ndim > 0) return fail(ACD_ERR_AXIS, "acd_scan_noalloc: axis %d out of range", axis);
  const int64_t n = desc_numel(in);
  if (n == 0) return ACD_OK;
  ScanArgs a{};
  a.in = desc_ptr(in);
  a.out = desc_ptr(out);
  int64_t si[3] = {0, 0, 0}, so[3] = {0, 0, 0};
  if (axis < 0 || in->ndim == 0) {
    if (!desc_is_contiguous(in) || !desc_is_contiguous(out))
      return fail(ACD_ERR_UNSUPPORTED, "acd_scan_noalloc: flattened scan needs contiguous input and output");
    a.L = 1;
    a.R = n;
    a.O = 1;
    si[1] = so[1] = 1;
  } else if (!split_axis(in, out, axis, a.L, a.R, a.O, si, so)) {
    return fail(ACD_ERR_UNSUPPORTED, "acd_scan_noalloc: view not collapsible around the axis");
  }
  a.sl = si[0];
  a.sr = si[1];
  a.so = si[2];
  a.ol = so[0];
  a.orr = so[1];
  a.oo = so[2];
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool prod = op == ACD_CUMPROD;
  if (in->dtype == ACD_FLOAT32) return prod ? noalloc_launch<float, true>(a, s) : noalloc_launch<float, false>(a, s);
  return prod ? noalloc_launch<double, true>(a, s) : noalloc_launch<double, false>(a, s);
}

}  // extern "C"
