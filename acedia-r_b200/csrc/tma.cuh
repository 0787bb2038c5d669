// Tensor Memory Accelerator (TMA) and mbarrier helpers for sm_100a, as
// inline PTX, plus the host-side tensor-map encoder.
//
// Only plain tiled loads and stores of this GPU's own memory are used: every
// load names this CTA's own shared memory and an mbarrier in it, and no load
// is broadcast to other CTAs.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace acd {

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (TMA).
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// One plain arrival.
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One arrival that also expects `bytes` of TMA transactions in this phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Deadline of a bounded wait.  The clock is %globaltimer; a reading below
// the start (the timer was set back) restarts the count, and the limit is
// only declared after at least 4096 polls, so a timer that jumps forward
// cannot end a short wait.
struct WaitClock {
  uint64_t t0 = 0;
  uint32_t polls = 0;
  __device__ __forceinline__ bool expired(uint64_t timeout_ns) {
    const uint64_t now = global_timer_ns();
    if (polls++ == 0 || now < t0) {
      t0 = now;
      return false;
    }
    return polls > 4096u && now - t0 > timeout_ns;
  }
};

// Waits for the phase with `parity` to complete, at most `timeout_ns`.
// Returns false when the limit expired.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  WaitClock clk;
  while (!mbar_try_wait(bar, parity))
    if (clk.expired(timeout_ns)) return false;
  return true;
}

// Bounded wait of one thread for the phase with `parity`.  Gives up when
// *abort is set (another role of the CTA gave up) or when the limit expires;
// then it sets *abort, raises `code` in the context status word and returns
// false.
__device__ __forceinline__ bool mbar_wait_thread(uint64_t *bar, uint32_t parity, int *abort, Control *control,
                                                 int32_t code, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  WaitClock clk;
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<volatile int *>(abort)) return false;
    if (clk.expired(timeout_ns)) {
      *reinterpret_cast<volatile int *>(abort) = 1;
      raise_status(control, code, (int32_t)blockIdx.x);
      return false;
    }
  }
  return true;
}

// The same for a whole warp, with one answer for all its lanes: every lane
// polls the barrier (each observes the phase, which orders the TMA-written
// data before its reads), lane 0 alone keeps the clock and reads *abort, and
// the warp leaves together, so code after the wait never runs with part of
// the warp.  All 32 lanes must call it.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, int *abort, Control *control,
                                               int32_t code, uint64_t timeout_ns) {
  WaitClock clk;
  const bool lead = (threadIdx.x & 31) == 0;
  while (true) {
    const bool ok = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, ok)) return true;
    int stop = 0;
    if (lead) {
      if (*reinterpret_cast<volatile int *>(abort)) {
        stop = 1;
      } else if (clk.expired(timeout_ns)) {
        *reinterpret_cast<volatile int *>(abort) = 1;
        raise_status(control, code, (int32_t)blockIdx.x);
        stop = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, stop, 0)) return false;
  }
}

// 3-D tiled load of one box into shared memory; completion is counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// 3-D tiled store of one box from shared memory (bulk-group completion).
// Parts of the box outside the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(map),
               "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(src))
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N committed store groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Host: encodes a 3-D tiled tensor map over 4- or 8-byte elements, with a
// 128-byte swizzle (box inner extent = 128 bytes) or none.  dims[0] is the
// contiguous axis; strides_elems[0..1] are the element strides of dims 1 and
// 2.  `promote256` lets L2 fetch 256-byte granules (worth it when the
// neighbouring 128 bytes are read at about the same time).  Returns false
// when the driver rejects the map (alignment, extents).
bool encode_tensor_map_3d(CUtensorMap *map, const void *base, int elem_bytes, const int64_t dims[3],
                          const int64_t strides_elems[2], const uint32_t box[3], bool swizzle128 = true,
                          bool promote256 = true);

// Host: TMA-staged transpose of 4-byte elements, out(i,j,k) = in(i,j,k) with
// out contiguous along i (extent n0, j stride os1, k stride os2) and in
// contiguous along j (extent n1, i stride is0, k stride is2).  Returns false,
// having launched nothing, when the views do not meet TMA's alignment rules
// or are too small to gain from it.
bool launch_transpose_tma4(acd_ctx *ctx, void *out, const void *in, int64_t n0, int64_t n1, int64_t n2,
                           int64_t os1, int64_t os2, int64_t is0, int64_t is2, cudaStream_t stream);

// Host: the strided-views step in one kernel (permute_chain.cu).  y and z
// take the geometry of launch_transpose_tma4's `out` (both contiguous, the
// fibers of the argmax along i, n0 elements each), x that of its `in`.
// Writes y, z = y*p + exp(-(y^2)), the statistics row of z (as
// acd_stats_partial, n_total elements) and the argmax keys of z along i (as
// acd_argmax_keys with index_base).  Sets *launched = false, having launched
// nothing, when the views do not meet TMA's rules; errors only from scratch
// allocation or the launch.
acd_status launch_permute_chain(acd_ctx *ctx, float *y, float *z, const float *x, int64_t n0, int64_t n1,
                                int64_t n2, int64_t os1, int64_t os2, int64_t is0, int64_t is2, float p,
                                double *stats, int64_t n_total, long long *keys, int64_t index_base,
                                cudaStream_t stream, bool *launched);

}  // namespace acd
