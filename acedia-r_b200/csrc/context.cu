// Context, workspace, error reporting and host-side descriptor analysis.
//
// The reference has no context: every launcher allocates its own temporaries
// with cudaMalloc and frees them after a cudaDeviceSynchronize
// (src/kernels/tensor_ops.cu:50-126, 168-197; src/TensorRegistry.h:950-1150).
// Here one context per device owns a workspace that grows on demand and a
// control block of self-resetting counters, so no call allocates in steady state.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace acd {

static thread_local char g_err[1024] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

acd_status fail(acd_status s, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return s;
}

acd_status cuda_fail(cudaError_t e, const char *where) {
  snprintf(g_err, sizeof(g_err), "CUDA error in %s: %s", where, cudaGetErrorString(e));
  return ACD_ERR_CUDA;
}

static void *dev_alloc(acd_ctx *ctx, size_t bytes) {
  if (ctx->alloc) return ctx->alloc(bytes, ctx->alloc_user);
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

static void dev_free(acd_ctx *ctx, void *p) {
  if (!p) return;
  if (ctx->free_fn)
    ctx->free_fn(p, ctx->alloc_user);
  else
    cudaFree(p);
}

acd_status get_scratch(acd_ctx *ctx, size_t bytes, cudaStream_t stream, void **out) {
  if (bytes == 0) bytes = 256;
  if (ctx->scratch && ctx->scratch_bytes >= bytes) {
    *out = ctx->scratch;
    return ACD_OK;
  }
  size_t want = bytes;
  if (want < 2 * ctx->scratch_bytes) want = 2 * ctx->scratch_bytes;
  want = (want + 4095) & ~(size_t)4095;
  if (ctx->scratch) {
    ACD_CUDA(cudaStreamSynchronize(stream));
    dev_free(ctx, ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  void *p = dev_alloc(ctx, want);
  if (!p) return fail(ACD_ERR_ALLOC, "workspace allocation of %zu bytes failed", want);
  ctx->scratch = p;
  ctx->scratch_bytes = want;
  *out = p;
  return ACD_OK;
}

template <typename W>
static acd_status get_zeroed(acd_ctx *ctx, W **region, size_t *have, size_t n, cudaStream_t stream,
                             const char *what) {
  if (n == 0) n = 1;
  if (*region && *have >= n) return ACD_OK;
  size_t want = n < 2 * *have ? 2 * *have : n;
  want = (want + 1023) & ~(size_t)1023;
  if (*region) {
    ACD_CUDA(cudaStreamSynchronize(stream));
    dev_free(ctx, *region);
    *region = nullptr;
    *have = 0;
  }
  void *p = dev_alloc(ctx, want * sizeof(W));
  if (!p) return fail(ACD_ERR_ALLOC, "%s allocation of %zu bytes failed", what, want * sizeof(W));
  ACD_CUDA(cudaMemsetAsync(p, 0, want * sizeof(W), stream));
  *region = static_cast<W *>(p);
  *have = want;
  return ACD_OK;
}

int resident_blocks(const void *kernel, int threads, size_t smem) {
  struct Key {
    const void *k;
    int t;
    size_t s;
  };
  static std::mutex mu;
  static Key keys[256];
  static int vals[256];
  static int used = 0;
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < used; ++i)
    if (keys[i].k == kernel && keys[i].t == threads && keys[i].s == smem) return vals[i];
  int nb = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kernel, threads, smem) != cudaSuccess || nb < 1) {
    cudaGetLastError();
    nb = 1;
  }
  if (used < 256) {
    keys[used] = Key{kernel, threads, smem};
    vals[used] = nb;
    ++used;
  }
  return nb;
}

acd_status get_counters(acd_ctx *ctx, size_t n, cudaStream_t stream, unsigned int **out) {
  ACD_TRY(get_zeroed(ctx, &ctx->counters, &ctx->counters_n, n, stream, "counter"));
  *out = ctx->counters;
  return ACD_OK;
}

acd_status get_flags(acd_ctx *ctx, size_t n, cudaStream_t stream, uint32_t **out) {
  ACD_TRY(get_zeroed(ctx, &ctx->flags, &ctx->flags_n, n, stream, "flag"));
  *out = ctx->flags;
  return ACD_OK;
}

// ---------------------------------------------------------------------------
// descriptor analysis
// ---------------------------------------------------------------------------
acd_status check_desc(const acd_desc *d, const char *name) {
  if (!d) return fail(ACD_ERR_INVALID, "%s: null descriptor", name);
  if (d->ndim < 0 || d->ndim > ACD_MAX_DIMS)
    return fail(ACD_ERR_INVALID, "%s: ndim %d outside [0, %d]", name, d->ndim, ACD_MAX_DIMS);
  if (dtype_size(d->dtype) == 0) return fail(ACD_ERR_DTYPE, "%s: unknown dtype %d", name, d->dtype);
  int64_t n = 1;
  for (int k = 0; k < d->ndim; ++k) {
    if (d->shape[k] < 0) return fail(ACD_ERR_INVALID, "%s: negative extent on axis %d", name, k);
    n *= d->shape[k];
  }
  if (n > 0 && !d->data) return fail(ACD_ERR_INVALID, "%s: null data pointer", name);
  if (d->offset < 0) return fail(ACD_ERR_INVALID, "%s: negative offset", name);
  return ACD_OK;
}

int64_t desc_numel(const acd_desc *d) {
  int64_t n = 1;
  for (int k = 0; k < d->ndim; ++k) n *= d->shape[k];
  return n;
}

bool desc_is_contiguous(const acd_desc *d) {
  int64_t expect = 1;
  for (int k = 0; k < d->ndim; ++k) {
    if (d->shape[k] != 1 && d->stride[k] != expect) return false;
    expect *= d->shape[k];
  }
  return true;
}

void collapse(IterSpace &it) {
  // drop size-1 dims
  int nd = 0;
  for (int d = 0; d < it.ndim; ++d) {
    if (it.shape[d] == 1) continue;
    it.shape[nd] = it.shape[d];
    for (int o = 0; o < it.nops; ++o) it.stride[o][nd] = it.stride[o][d];
    ++nd;
  }
  if (nd == 0) {
    it.ndim = 1;
    it.shape[0] = 1;
    for (int o = 0; o < it.nops; ++o) it.stride[o][0] = 0;
    return;
  }
  // merge neighbours
  int w = 0;
  for (int d = 1; d < nd; ++d) {
    bool ok = true;
    for (int o = 0; o < it.nops; ++o)
      if (it.stride[o][d] != it.stride[o][w] * it.shape[w]) { ok = false; break; }
    if (ok) {
      it.shape[w] *= it.shape[d];
    } else {
      ++w;
      it.shape[w] = it.shape[d];
      for (int o = 0; o < it.nops; ++o) it.stride[o][w] = it.stride[o][d];
    }
  }
  it.ndim = w + 1;
}

bool is_dense_permutation(int ndim, const int64_t *shape, const int64_t *stride) {
  // Order dims by stride; each stride must equal the product of the extents
  // of the dims ordered before it.
  int idx[ACD_MAX_DIMS];
  int m = 0;
  for (int d = 0; d < ndim; ++d)
    if (shape[d] != 1) idx[m++] = d;
  for (int a = 1; a < m; ++a)
    for (int b = a; b > 0 && stride[idx[b]] < stride[idx[b - 1]]; --b) {
      int t = idx[b];
      idx[b] = idx[b - 1];
      idx[b - 1] = t;
    }
  int64_t expect = 1;
  for (int a = 0; a < m; ++a) {
    if (stride[idx[a]] != expect) return false;
    expect *= shape[idx[a]];
  }
  return true;
}

}  // namespace acd

using namespace acd;

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

const char *acd_version(void) { return "acediar-b200 0.1 (sm_100a)"; }

int32_t acd_gpu_available(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return 0;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, 0) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return 1;
}

int64_t acd_gpu_info(char *buf, int64_t len) {
  std::string info;
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    info = std::string("CUDA Error: ") + cudaGetErrorString(e);
  } else if (n == 0) {
    info = "No CUDA-capable devices found";
  } else {
    info = "Found " + std::to_string(n) + " CUDA device(s):\n";
    for (int i = 0; i < n; ++i) {
      cudaDeviceProp prop;
      if (cudaGetDeviceProperties(&prop, i) != cudaSuccess) {
        cudaGetLastError();
        continue;
      }
      info += "  Device " + std::to_string(i) + ": " + prop.name + " (Compute " + std::to_string(prop.major) + "." +
              std::to_string(prop.minor) + ") - " + std::to_string(prop.totalGlobalMem / (1024 * 1024)) + " MB\n";
    }
  }
  if (buf && len > 0) {
    const size_t k = std::min((size_t)(len - 1), info.size());
    memcpy(buf, info.data(), k);
    buf[k] = 0;
  }
  return (int64_t)info.size();
}

double acd_gpu_memory_available(void) {
  if (!acd_gpu_available()) return 0.0;
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) {
    cudaGetLastError();
    return 0.0;
  }
  return (double)free_b;
}

const char *acd_last_error(void) { return g_err; }

const char *acd_status_string(acd_status s) {
  switch (s) {
    case ACD_OK: return "ok";
    case ACD_ERR_INVALID: return "invalid argument";
    case ACD_ERR_SHAPE: return "shape mismatch";
    case ACD_ERR_DTYPE: return "unsupported dtype";
    case ACD_ERR_AXIS: return "axis out of range";
    case ACD_ERR_ALLOC: return "allocation failed";
    case ACD_ERR_CUDA: return "CUDA error";
    case ACD_ERR_DEVICE: return "device error";
    case ACD_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

acd_status acd_ctx_create(int device, acd_ctx **out) {
  if (!out) return fail(ACD_ERR_INVALID, "acd_ctx_create: null output pointer");
  *out = nullptr;
  int ndev = 0;
  ACD_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev)
    return fail(ACD_ERR_INVALID, "acd_ctx_create: device %d outside [0, %d)", device, ndev);
  DeviceGuard g(device);
  if (!g.ok) return fail(ACD_ERR_CUDA, "acd_ctx_create: cannot select device %d", device);
  acd_ctx *ctx = new acd_ctx();
  ctx->device = device;
  cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&ctx->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  cudaError_t e = cudaMalloc(&ctx->control, sizeof(Control));
  if (e != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "cudaMalloc(control)");
  }
  e = cudaMemset(ctx->control, 0, sizeof(Control));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(ctx->control);
    delete ctx;
    return cuda_fail(e, "cudaMemset(control)");
  }
  *out = ctx;
  return ACD_OK;
}

acd_status acd_ctx_destroy(acd_ctx *ctx) {
  if (!ctx) return ACD_OK;
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  dev_free(ctx, ctx->scratch);
  dev_free(ctx, ctx->counters);
  dev_free(ctx, ctx->flags);
  cudaFree(ctx->control);
  delete ctx;
  return ACD_OK;
}

acd_status acd_ctx_set_allocator(acd_ctx *ctx, acd_alloc_fn alloc, acd_free_fn free_fn, void *user) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_ctx_set_allocator: null context");
  if ((alloc == nullptr) != (free_fn == nullptr))
    return fail(ACD_ERR_INVALID, "acd_ctx_set_allocator: alloc and free must both be set or both be NULL");
  DeviceGuard g(ctx->device);
  ACD_CUDA(cudaDeviceSynchronize());
  dev_free(ctx, ctx->scratch);
  dev_free(ctx, ctx->counters);
  dev_free(ctx, ctx->flags);
  ctx->scratch = nullptr;
  ctx->scratch_bytes = 0;
  ctx->counters = nullptr;
  ctx->counters_n = 0;
  ctx->flags = nullptr;
  ctx->flags_n = 0;
  ctx->alloc = alloc;
  ctx->free_fn = free_fn;
  ctx->alloc_user = user;
  return ACD_OK;
}

acd_status acd_ctx_check(acd_ctx *ctx, acd_stream stream, int32_t *code) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_ctx_check: null context");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ACD_CUDA(cudaStreamSynchronize(s));
  int32_t host[2] = {0, 0};
  ACD_CUDA(cudaMemcpy(host, ctx->control, sizeof(host), cudaMemcpyDeviceToHost));
  if (code) *code = host[0];
  if (host[0] != 0) {
    int32_t zero[2] = {0, 0};
    ACD_CUDA(cudaMemcpy(ctx->control, zero, sizeof(zero), cudaMemcpyHostToDevice));
    return fail(ACD_ERR_DEVICE, "device status %d (detail %d): a bounded wait expired", host[0], host[1]);
  }
  return ACD_OK;
}

acd_status acd_ctx_set_scan_fault(acd_ctx *ctx, int64_t tile, int64_t timeout_ns) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_ctx_set_scan_fault: null context");
  ctx->scan_fault_tile = tile < 0 ? -1 : tile;
  ctx->scan_timeout_ns = timeout_ns > 0 ? timeout_ns : 1000000000LL;
  return ACD_OK;
}

acd_status acd_broadcast_shape(int32_t a_ndim, const int64_t *a_shape, int32_t b_ndim, const int64_t *b_shape,
                               int32_t *out_ndim, int64_t *out_shape) {
  if (a_ndim < 0 || b_ndim < 0 || a_ndim > ACD_MAX_DIMS || b_ndim > ACD_MAX_DIMS || !out_ndim || !out_shape ||
      (a_ndim && !a_shape) || (b_ndim && !b_shape))
    return fail(ACD_ERR_INVALID, "acd_broadcast_shape: bad arguments");
  const bool a_short = a_ndim < b_ndim;
  const int32_t ns = a_short ? a_ndim : b_ndim, nl = a_short ? b_ndim : a_ndim;
  const int64_t *ss = a_short ? a_shape : b_shape, *sl = a_short ? b_shape : a_shape;
  for (int32_t off = 0; off + ns <= nl; ++off) {
    bool ok = true;
    for (int32_t i = 0; i < nl && ok; ++i) {
      int64_t ds = (i >= off && i < off + ns) ? ss[i - off] : 1;
      int64_t dl = sl[i];
      if (ds != dl && ds != 1 && dl != 1) ok = false;
    }
    if (ok) {
      for (int32_t i = 0; i < nl; ++i) {
        int64_t ds = (i >= off && i < off + ns) ? ss[i - off] : 1;
        out_shape[i] = ds > sl[i] ? ds : sl[i];
      }
      *out_ndim = nl;
      return ACD_OK;
    }
    if (ns == nl) break;  // equal ranks: only offset 0
  }
  return fail(ACD_ERR_SHAPE, "Tensor shapes are not broadcastable");
}

acd_status acd_broadcast_strides(int32_t in_ndim, const int64_t *in_shape, const int64_t *in_stride, int32_t out_ndim,
                                 const int64_t *out_shape, int64_t *out_stride) {
  if (in_ndim < 0 || out_ndim < in_ndim || out_ndim > ACD_MAX_DIMS || !out_stride || (in_ndim && (!in_shape || !in_stride)) ||
      (out_ndim && !out_shape))
    return fail(ACD_ERR_INVALID, "acd_broadcast_strides: bad arguments");
  for (int32_t off = 0; off + in_ndim <= out_ndim; ++off) {
    bool ok = true;
    for (int32_t i = 0; i < in_ndim && ok; ++i) {
      int64_t s = in_shape[i], d = out_shape[i + off];
      if (s != d && s != 1 && d != 1) ok = false;
      if (s != 1 && s != d) ok = false;  // the input must expand into the output
    }
    if (ok) {
      for (int32_t i = 0; i < out_ndim; ++i) {
        if (i < off || i >= off + in_ndim)
          out_stride[i] = 0;
        else
          out_stride[i] = in_shape[i - off] == 1 ? 0 : in_stride[i - off];
      }
      return ACD_OK;
    }
  }
  return fail(ACD_ERR_SHAPE, "Shape mismatch in broadcast stride calculation");
}

// Host-only self test of the fast divider, exported for the CPU test suite.
int32_t acd_selftest_fastdiv(uint32_t d, uint32_t n, uint32_t *q) {
  if (d == 0 || !q) return -1;
  FastDiv f(d);
  *q = f.div(n);
  return 0;
}

// Host-only: collapsed iteration space of (out, in) for tests of the dim
// merging rule.  Returns ndim; writes shapes and both operands' strides.
int32_t acd_selftest_collapse(const acd_desc *out, const acd_desc *in, int64_t *shape, int64_t *s_out, int64_t *s_in) {
  if (!out || !in || out->ndim != in->ndim) return -1;
  IterSpace it;
  it.ndim = out->ndim;
  it.nops = 2;
  for (int d = 0; d < it.ndim; ++d) {
    it.shape[d] = out->shape[d];
    it.stride[0][d] = out->stride[d];
    it.stride[1][d] = in->stride[d];
  }
  collapse(it);
  for (int d = 0; d < it.ndim; ++d) {
    shape[d] = it.shape[d];
    s_out[d] = it.stride[0][d];
    s_in[d] = it.stride[1][d];
  }
  return it.ndim;
}

}  // extern "C"
