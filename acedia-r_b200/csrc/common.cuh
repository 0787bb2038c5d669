// Shared host/device helpers of the acd library: dtype traits, descriptor
// analysis (dimension collapsing), fast division, vector memory types, error
// reporting and the context layout.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cmath>
#include <cstring>
#include <string>
#include <type_traits>

#include "../../include/acd.h"

namespace acd {

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
void set_error(const char *fmt, ...);
acd_status fail(acd_status s, const char *fmt, ...);
acd_status cuda_fail(cudaError_t e, const char *where);

#define ACD_CUDA(call)                                               \
  do {                                                               \
    cudaError_t _e = (call);                                         \
    if (_e != cudaSuccess) return ::acd::cuda_fail(_e, #call);       \
  } while (0)

#define ACD_TRY(expr)                                                \
  do {                                                               \
    acd_status _s = (expr);                                          \
    if (_s != ACD_OK) return _s;                                     \
  } while (0)

// ---------------------------------------------------------------------------
// dtypes
// ---------------------------------------------------------------------------
inline size_t dtype_size(int32_t dt) {
  switch (dt) {
    case ACD_FLOAT32: return 4;
    case ACD_FLOAT64: return 8;
    case ACD_INT32: return 4;
    case ACD_INT64: return 8;
    case ACD_BOOL: return 1;
    case ACD_FLOAT16: return 2;
    case ACD_INT8: return 1;
    default: return 0;
  }
}
inline bool is_float(int32_t dt) { return dt == ACD_FLOAT32 || dt == ACD_FLOAT64; }

// Real (non-integer) element types: float, double and IEEE binary16.
template <typename T>
struct is_real : std::integral_constant<bool, std::is_floating_point<T>::value || std::is_same<T, __half>::value> {};

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
// Control block at the start of the workspace: a status word and counters
// that every kernel leaves at zero when it finishes.
struct Control {
  int32_t status;        // first device error code raised (0 = none)
  int32_t status_info;   // detail (e.g. tile index of a timed-out wait)
  uint32_t scan_abort;   // epoch of a scan launch that gave up waiting
  uint32_t pad0;
  unsigned int counters[60];
  double stats[8];  // small device results (softmax statistics)
};

}  // namespace acd

struct acd_ctx {
  int device = 0;
  int sm_count = 148;
  int max_smem_optin = 0;
  acd::Control *control = nullptr;  // device, persistent, zeroed at creation
  void *scratch = nullptr;          // device, grows on demand: partial results (no state at rest)
  size_t scratch_bytes = 0;
  unsigned int *counters = nullptr; // device, grows on demand, zero at rest (kernels reset them)
  size_t counters_n = 0;
  uint32_t *flags = nullptr;        // device, grows on demand, epoch-tagged scan tile flags
  size_t flags_n = 0;
  uint32_t epoch = 0;               // incremented per scan launch (tags tile flags)
  acd_alloc_fn alloc = nullptr;
  acd_free_fn free_fn = nullptr;
  void *alloc_user = nullptr;
  int64_t scan_fault_tile = -1;
  int64_t scan_timeout_ns = 1000000000LL;
};

namespace acd {

// Scratch for partial results: at least `bytes`, contents undefined.
// Growing synchronises `stream` first (the old region may be in use).
acd_status get_scratch(acd_ctx *ctx, size_t bytes, cudaStream_t stream, void **out);
// `n` tile counters, zero at rest: every kernel that increments one resets it.
// Nothing else ever writes this region.
acd_status get_counters(acd_ctx *ctx, size_t n, cudaStream_t stream, unsigned int **out);
// `n` scan tile flags tagged with the launch epoch (stale tags never match).
acd_status get_flags(acd_ctx *ctx, size_t n, cudaStream_t stream, uint32_t **out);
// Device guard: makes ctx->device current for the scope.
struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = (cudaSetDevice(dev) == cudaSuccess);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// ---------------------------------------------------------------------------
// descriptor analysis
// ---------------------------------------------------------------------------
constexpr int kMaxOps = 3;  // output + up to two inputs

// A set of operands iterated over one common shape (the output's).  All
// strides are in elements of the operand's own dtype.
struct IterSpace {
  int ndim = 0;
  int nops = 0;
  int64_t shape[ACD_MAX_DIMS];
  int64_t stride[kMaxOps][ACD_MAX_DIMS];
  int64_t numel() const {
    int64_t n = 1;
    for (int d = 0; d < ndim; ++d) n *= shape[d];
    return n;
  }
};

acd_status check_desc(const acd_desc *d, const char *name);
int64_t desc_numel(const acd_desc *d);
bool desc_is_contiguous(const acd_desc *d);  // column-major dense, any offset
// Pointer to the view's first element.
inline char *desc_ptr(const acd_desc *d) {
  return static_cast<char *>(d->data) + d->offset * (int64_t)dtype_size(d->dtype);
}
// Drops size-1 dims and merges neighbours that are jointly contiguous for all
// operands.  Leaves ndim >= 1.
void collapse(IterSpace &it);
// Sorts nothing; reports whether the operand's strides describe a dense
// permutation of a column-major block (each element visited exactly once).
bool is_dense_permutation(int ndim, const int64_t *shape, const int64_t *stride);

// ---------------------------------------------------------------------------
// 32-bit fast division (round-up magic number, Granlund & Montgomery 1994)
// ---------------------------------------------------------------------------
struct FastDiv {
  uint32_t d = 1, m = 1, s = 0;
  FastDiv() = default;
  explicit FastDiv(uint32_t divisor) {
    d = divisor;
    s = 0;
    while ((1ull << s) < d) ++s;
    m = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
  }
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
#ifdef __CUDA_ARCH__
    uint32_t hi = __umulhi(n, m);
#else
    uint32_t hi = (uint32_t)(((uint64_t)n * m) >> 32);
#endif
    return (uint32_t)(((uint64_t)hi + n) >> s);
  }
};

// ---------------------------------------------------------------------------
// vector memory helpers
// ---------------------------------------------------------------------------
template <typename T, int V>
struct alignas(sizeof(T) * V) Vec {
  T v[V];
};

template <typename T>
__host__ __device__ __forceinline__ bool aligned_to(const void *p, int bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

// ---------------------------------------------------------------------------
// double-double helpers (Knuth TwoSum, fma-based TwoProd)
// ---------------------------------------------------------------------------
struct DD {
  double hi, lo;
};
__host__ __device__ __forceinline__ void two_sum(double a, double b, double &s, double &e) {
  s = a + b;
  double bb = s - a;
  e = (a - (s - bb)) + (b - bb);
}
__host__ __device__ __forceinline__ void dd_add(DD &acc, double x) {
  double s, e;
  two_sum(acc.hi, x, s, e);
  acc.hi = s;
  acc.lo += e;
}
__host__ __device__ __forceinline__ void dd_merge(DD &a, const DD &b) {
  double s, e;
  two_sum(a.hi, b.hi, s, e);
  e += a.lo + b.lo;
  double hi = s + e;
  a.lo = e - (hi - s);
  a.hi = hi;
}
__device__ __forceinline__ void dd_add_square(DD &acc, double d) {
  double p = d * d;
  double pe = fma(d, d, -p);
  double s, e;
  two_sum(acc.hi, p, s, e);
  acc.hi = s;
  acc.lo += e + pe;
}

// ---------------------------------------------------------------------------
// warp / block helpers
// ---------------------------------------------------------------------------
template <class A>
__device__ __forceinline__ A shfl_xor_any(const A &a, int mask) {
  static_assert(sizeof(A) % 4 == 0, "shuffle payload must be 4-byte words");
  A r;
  const int *src = reinterpret_cast<const int *>(&a);
  int *dst = reinterpret_cast<int *>(&r);
#pragma unroll
  for (int k = 0; k < (int)(sizeof(A) / 4); ++k) dst[k] = __shfl_xor_sync(0xffffffffu, src[k], mask);
  return r;
}

template <class A>
__device__ __forceinline__ void warp_reduce(A &a) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) {
    A o = shfl_xor_any(a, m);
    a.merge(o);
  }
}

// Block-wide reduction; the result is valid in thread 0.  `smem` must hold
// blockDim.x/32 accumulators.
template <class A>
__device__ __forceinline__ void block_reduce(A &a, A *smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  warp_reduce(a);
  __syncthreads();  // smem may still be read by a previous round
  if (lane == 0) smem[warp] = a;
  __syncthreads();
  if (warp == 0) {
    A b;
    if (lane < nwarps) {
      b = smem[lane];
    } else {
      b.init();
    }
    warp_reduce(b);
    a = b;
  }
}

// Device status word: records the first error code.
__device__ __forceinline__ void raise_status(Control *c, int32_t code, int32_t info) {
  if (atomicCAS(&c->status, 0, code) == 0) c->status_info = info;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Blocks of `kernel` resident per SM at `threads` threads and `smem` dynamic
// shared memory (occupancy API, cached per kernel and launch shape).
int resident_blocks(const void *kernel, int threads, size_t smem);

// Persistent grid: as many blocks as are resident at once (a multiple of the
// SM count), or fewer when there is less work.  A larger grid would run as a
// second, partly filled wave.
template <typename K>
inline int persistent_grid(const acd_ctx *ctx, K kernel, int threads, size_t smem, int64_t work_blocks) {
  const int nb = resident_blocks(reinterpret_cast<const void *>(kernel), threads, smem);
  int64_t cap = (int64_t)ctx->sm_count * nb;
  if (work_blocks < cap) cap = work_blocks;
  return cap < 1 ? 1 : (int)cap;
}

// Grid sizing: a multiple of the SM count.
inline int grid_for(const acd_ctx *ctx, int64_t work_items, int per_block, int blocks_per_sm) {
  int64_t want = (work_items + per_block - 1) / per_block;
  int64_t cap = (int64_t)ctx->sm_count * blocks_per_sm;
  if (want > cap) want = cap;
  if (want < 1) want = 1;
  return (int)want;
}

}  // namespace acd
