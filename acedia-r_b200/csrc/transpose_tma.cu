// TMA-staged transpose of 4-byte elements (the permute -> contiguous copy of
// a float32 / int32 view whose innermost axes swap).
//
// out(i, j, k) = in(i, j, k) with out contiguous along i and in contiguous
// along j.  The work is split into 64 x 64 tiles, batched over k.  One
// persistent CTA per SM runs a warp-specialised pipeline with no block-wide
// barrier inside the loop:
//   * warp 8 (one thread) loads tiles with TMA into NS stage buffers: two
//     boxes of 32 j x 64 i, 128-byte swizzled;
//   * warps 0..7 transpose each tile in registers.  Every thread owns one
//     4 x 4 block: it reads 4 input rows of 16 bytes and writes 4 output rows
//     of 16 bytes.  The blocks a quarter-warp touches are chosen so that its 8
//     16-byte accesses land in 8 distinct bank groups under the swizzle, for
//     reads and writes alike.  The results go to NOB output buffers in the
//     output box layout (32 i x 64 j, 128-byte swizzled);
//   * warp 9 (one thread) stores each output buffer with TMA.  Stores clip at
//     the tensor edge, so ragged tiles need no masking.
// Stage and buffer ownership passes through mbarriers (full / empty per
// stage, full / free per output buffer).  Every wait is bounded; when a wait
// expires the CTA raises the context status word (code 2), the other roles
// leave their loops, and the loading thread waits (bounded) for the loads it
// issued before the CTA exits.
//
// Tiles are visited in diagonal order: tile t of a batch has i-tile
// t % tiles0 and j-tile (t / tiles0 + t % tiles0) % tiles1.  The tiles in
// flight at one time then spread over both tensors' address ranges instead
// of sharing low address bits, which would load a few memory channels.
#include <atomic>
#include <mutex>

#include "ops.cuh"
#include "reduce_acc.cuh"
#include "tma.cuh"

namespace acd {

namespace {

constexpr int kTT = 64;                // tile edge (elements)
constexpr int kTileBytes = kTT * kTT * 4;
constexpr int kBoxBytes = kTileBytes / 2;
constexpr int kNS = 4;                 // input stages
constexpr int kNOB = 4;                // output buffers
constexpr int kThreads = 320;          // 8 transpose warps, a load warp, a store warp
constexpr uint64_t kWaitNs = 1000000000ull;

struct TtShared {
  uint64_t full[kNS], empty[kNS], ofull[kNOB], ofree[kNOB];
  int abort;
};
constexpr size_t kSmemBytes = (size_t)(kNS + kNOB) * kTileBytes + sizeof(TtShared) + 1024;

struct TtArgs {
  int64_t tiles0, tiles1, nb;
  int n0, n1;
  Control *control;
};

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait that also gives up once another role of the CTA has aborted.
template <class SH>
__device__ __forceinline__ bool tt_wait(uint64_t *bar, uint32_t parity, SH *sh, const TtArgs &a) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*reinterpret_cast<volatile int *>(&sh->abort)) return false;
    if (global_timer_ns() - t0 > kWaitNs) {
      *reinterpret_cast<volatile int *>(&sh->abort) = 1;
      raise_status(a.control, 2, (int32_t)blockIdx.x);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tt_coords(const TtArgs &a, int64_t k, int &i0, int &j0, int &b) {
  const int64_t nt01 = a.tiles0 * a.tiles1;
  const int64_t t = (int64_t)blockIdx.x + k * gridDim.x;
  const int64_t bb = t / nt01, t01 = t - bb * nt01;
  const int64_t ti = t01 % a.tiles0;
  const int64_t tj = (t01 / a.tiles0 + ti) % a.tiles1;
  i0 = (int)(ti * kTT);
  j0 = (int)(tj * kTT);
  b = (int)bb;
}

__global__ void __launch_bounds__(kThreads, 1)
    k_transpose_tma4(const __grid_constant__ CUtensorMap map_in, const __grid_constant__ CUtensorMap map_out,
                     TtArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // 128-byte swizzled boxes need 1024-byte aligned buffers
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  unsigned char *sin = smem;
  unsigned char *sout = smem + kNS * kTileBytes;
  TtShared *sh = reinterpret_cast<TtShared *>(sout + kNOB * kTileBytes);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t ntiles = a.tiles0 * a.tiles1 * a.nb;
  if ((int64_t)blockIdx.x >= ntiles) return;
  const int64_t my_n = (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 8);
    }
    for (int b = 0; b < kNOB; ++b) {
      mbar_init(&sh->ofull[b], 8);
      mbar_init(&sh->ofree[b], 1);
    }
    sh->abort = 0;
    mbar_init_fence();
  }
  __syncthreads();

  if (warp == 8) {  // loader
    if (lane == 0) {
      int64_t k = 0;
      for (; k < my_n; ++k) {
        const int s = (int)(k % kNS);
        if (!tt_wait(&sh->empty[s], (uint32_t)(((k / kNS) & 1) ^ 1), sh, a)) break;
        int i0, j0, b;
        tt_coords(a, k, i0, j0, b);
        const bool two = j0 + 32 < a.n1;  // a box wholly past the last column is not loaded
        mbar_arrive_expect_tx(&sh->full[s], two ? kTileBytes : kBoxBytes);
        tma_load_3d(sin + s * kTileBytes, &map_in, &sh->full[s], j0, i0, b);
        if (two) tma_load_3d(sin + s * kTileBytes + kBoxBytes, &map_in, &sh->full[s], j0 + 32, i0, b);
      }
      if (*reinterpret_cast<volatile int *>(&sh->abort)) {
        // the loads issued last may still be landing in this CTA's shared memory
        for (int64_t q = (k > kNS ? k - kNS : 0); q < k; ++q) {
          const uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(&sh->full[q % kNS], (uint32_t)((q / kNS) & 1)) &&
                 global_timer_ns() - t0 < kWaitNs) {
          }
        }
      }
    }
    return;
  }
  if (warp == 9) {  // storer
    if (lane == 0) {
      for (int64_t k = 0; k < my_n; ++k) {
        const int b = (int)(k % kNOB);
        if (!tt_wait(&sh->ofull[b], (uint32_t)((k / kNOB) & 1), sh, a)) break;
        int i0, j0, bb;
        tt_coords(a, k, i0, j0, bb);
        tma_store_3d(&map_out, sout + b * kTileBytes, i0, j0, bb);
        if (i0 + 32 < a.n0) tma_store_3d(&map_out, sout + b * kTileBytes + kBoxBytes, i0 + 32, j0, bb);
        bulk_commit();
        if (k >= 1) {
          bulk_wait_read<1>();  // the previous tile's store has read its buffer
          mbar_arrive(&sh->ofree[(k - 1) % kNOB]);
        }
      }
      bulk_wait_all();
    }
    return;
  }

  // transpose warps: thread -> 4x4 block (ib, jb) of the tile, ib, jb in 0..15
  const int k8 = lane & 7;
  const int shift = (lane >> 3) | ((warp & 1) << 2);
  const int ih = (warp >> 1) & 1, jh = warp >> 2;
  const int ib = 8 * ih + k8, jb = 8 * jh + ((k8 + shift) & 7);
  const int cj = jb & 7, ci = ib & 7;  // 16-byte chunk within a 128-byte row
  for (int64_t k = 0; k < my_n; ++k) {
    const int s = (int)(k % kNS);
    if (!tt_wait(&sh->full[s], (uint32_t)((k / kNS) & 1), sh, a)) break;
    const unsigned char *tin = sin + s * kTileBytes + jh * kBoxBytes;
    uint4 r[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int i = 4 * ci + m + 32 * ih;  // input box row
      r[m] = *reinterpret_cast<const uint4 *>(tin + i * 128 + ((cj ^ (i & 7)) << 4));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[s]);
    const int b = (int)(k % kNOB);
    if (!tt_wait(&sh->ofree[b], (uint32_t)(((k / kNOB) & 1) ^ 1), sh, a)) break;
    unsigned char *tout = sout + b * kTileBytes + ih * kBoxBytes;
    const uint4 w0 = make_uint4(r[0].x, r[1].x, r[2].x, r[3].x);
    const uint4 w1 = make_uint4(r[0].y, r[1].y, r[2].y, r[3].y);
    const uint4 w2 = make_uint4(r[0].z, r[1].z, r[2].z, r[3].z);
    const uint4 w3 = make_uint4(r[0].w, r[1].w, r[2].w, r[3].w);
    const int j = 4 * cj + 32 * jh;  // output box row of w0
    *reinterpret_cast<uint4 *>(tout + (j + 0) * 128 + ((ci ^ ((j + 0) & 7)) << 4)) = w0;
    *reinterpret_cast<uint4 *>(tout + (j + 1) * 128 + ((ci ^ ((j + 1) & 7)) << 4)) = w1;
    *reinterpret_cast<uint4 *>(tout + (j + 2) * 128 + ((ci ^ ((j + 2) & 7)) << 4)) = w2;
    *reinterpret_cast<uint4 *>(tout + (j + 3) * 128 + ((ci ^ ((j + 3) & 7)) << 4)) = w3;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->ofull[b]);
  }
}

// ---- the transpose with the elementwise chain, statistics and argmax keys --
// y = the transposed copy and z = y*p + exp(-(y^2)) (the chain's rounding),
// both written from the same tile, so the step reads its input once.  The
// same warp roles as k_transpose_tma4, with an output buffer pair (y, z) per
// slot.  From the transposed registers each thread also keeps the shifted
// moments of z (shift K = z(0, 0, 0), as acd_stats_partial) and, per tile,
// one key per output row j for the argmax along i (the key of acd_argmax_keys
// with index_base): the 16 partial keys of a row go through a double-buffered
// shared array and one 64-bit atomic max per row reaches `keys`, which the
// host fills with LLONG_MIN first.  The moments meet in the last CTA.
// Every transpose warp takes each named barrier exactly once per tile, also
// after an aborted wait (it then skips the tile's work), so no barrier can
// wait for a warp that left.
constexpr int kNOBz = 4;  // (y, z) output buffer pairs
constexpr int kNTW = 8;   // transpose warps

struct TcShared {
  uint64_t full[kNS], empty[kNS], ofull[kNOBz], ofree[kNOBz];
  int abort;
  int am_last;
  long long tkeys[2][kTT][16];
  VarAcc<float> wst[kNTW];
};
constexpr size_t kTcSmemBytes = (size_t)(kNS + 2 * kNOBz) * kTileBytes + sizeof(TcShared) + 1024;

struct TcArgs {
  const float *in0;  // the input's first element (y(0,0,0))
  float p;
  long long *keys;
  int64_t index_base;
  VarAcc<float> *partials;  // one per CTA
  unsigned int *counter;    // zero at rest; the last CTA resets it
  OutSpec os;               // statistics row
};

__device__ __forceinline__ void tc_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ long long tc_key(float v, int64_t gi) {
  const uint32_t ob = ordered_bits(v + 0.0f);
  const uint64_t u = ((uint64_t)ob << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)gi);
  return (long long)(u ^ 0x8000000000000000ull);
}

__global__ void __launch_bounds__(kThreads, 1)
    k_transpose_chain_tma4(const __grid_constant__ CUtensorMap map_in, const __grid_constant__ CUtensorMap map_y,
                           const __grid_constant__ CUtensorMap map_z, TtArgs a, TcArgs c) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  unsigned char *sin = smem;
  unsigned char *sy = smem + kNS * kTileBytes;
  unsigned char *sz = sy + kNOBz * kTileBytes;
  TcShared *sh = reinterpret_cast<TcShared *>(sz + kNOBz * kTileBytes);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t ntiles = a.tiles0 * a.tiles1 * a.nb;
  if ((int64_t)blockIdx.x >= ntiles) return;  // the host launches at most ntiles CTAs
  const int64_t my_n = (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x;
  if (tid == 0) {
    for (int s = 0; s < kNS; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], kNTW);
    }
    for (int b = 0; b < kNOBz; ++b) {
      mbar_init(&sh->ofull[b], kNTW);
      mbar_init(&sh->ofree[b], 1);
    }
    sh->abort = 0;
    mbar_init_fence();
  }
  __syncthreads();

  if (warp == 8) {  // loader, as in k_transpose_tma4
    if (lane == 0) {
      int64_t k = 0;
      for (; k < my_n; ++k) {
        const int s = (int)(k % kNS);
        if (!tt_wait(&sh->empty[s], (uint32_t)(((k / kNS) & 1) ^ 1), sh, a)) break;
        int i0, j0, b;
        tt_coords(a, k, i0, j0, b);
        const bool two = j0 + 32 < a.n1;
        mbar_arrive_expect_tx(&sh->full[s], two ? kTileBytes : kBoxBytes);
        tma_load_3d(sin + s * kTileBytes, &map_in, &sh->full[s], j0, i0, b);
        if (two) tma_load_3d(sin + s * kTileBytes + kBoxBytes, &map_in, &sh->full[s], j0 + 32, i0, b);
      }
      if (*reinterpret_cast<volatile int *>(&sh->abort)) {
        for (int64_t q = (k > kNS ? k - kNS : 0); q < k; ++q) {
          const uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(&sh->full[q % kNS], (uint32_t)((q / kNS) & 1)) &&
                 global_timer_ns() - t0 < kWaitNs) {
          }
        }
      }
    }
    return;
  }
  if (warp == 9) {  // storer: the y and z tiles of a slot
    if (lane == 0) {
      for (int64_t k = 0; k < my_n; ++k) {
        const int b = (int)(k % kNOBz);
        if (!tt_wait(&sh->ofull[b], (uint32_t)((k / kNOBz) & 1), sh, a)) break;
        int i0, j0, bb;
        tt_coords(a, k, i0, j0, bb);
        tma_store_3d(&map_y, sy + b * kTileBytes, i0, j0, bb);
        tma_store_3d(&map_z, sz + b * kTileBytes, i0, j0, bb);
        if (i0 + 32 < a.n0) {
          tma_store_3d(&map_y, sy + b * kTileBytes + kBoxBytes, i0 + 32, j0, bb);
          tma_store_3d(&map_z, sz + b * kTileBytes + kBoxBytes, i0 + 32, j0, bb);
        }
        bulk_commit();
        if (k >= 1) {
          bulk_wait_read<1>();
          mbar_arrive(&sh->ofree[(k - 1) % kNOBz]);
        }
      }
      bulk_wait_all();
    }
    return;
  }

  // transpose warps (0..7): the 4 x 4 block mapping of k_transpose_tma4
  const int k8 = lane & 7;
  const int shift = (lane >> 3) | ((warp & 1) << 2);
  const int ih = (warp >> 1) & 1, jh = warp >> 2;
  const int ib = 8 * ih + k8, jb = 8 * jh + ((k8 + shift) & 7);
  const int cj = jb & 7, ci = ib & 7;
  const FusedScaleAddExpNegSquare<float> f{c.p};
  const float K = f(*c.in0);
  VarAcc<float> st;
  st.init();
  st.set_shift(K);
  bool alive = true;
  for (int64_t k = 0; k < my_n; ++k) {
    const int s = (int)(k % kNS), b = (int)(k % kNOBz), kb = (int)(k & 1);
    int i0, j0, bb;
    tt_coords(a, k, i0, j0, bb);
    long long kq[4] = {LLONG_MIN, LLONG_MIN, LLONG_MIN, LLONG_MIN};
    uint4 r[4];
    if (alive) alive = __all_sync(0xffffffffu, tt_wait(&sh->full[s], (uint32_t)((k / kNS) & 1), sh, a));
    if (alive) {
      const unsigned char *tin = sin + s * kTileBytes + jh * kBoxBytes;
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i = 4 * ci + m + 32 * ih;
        r[m] = *reinterpret_cast<const uint4 *>(tin + i * 128 + ((cj ^ (i & 7)) << 4));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[s]);
      alive = __all_sync(0xffffffffu, tt_wait(&sh->ofree[b], (uint32_t)(((k / kNOBz) & 1) ^ 1), sh, a));
    }
    if (alive) {
      unsigned char *ty = sy + b * kTileBytes + ih * kBoxBytes;
      unsigned char *tz = sz + b * kTileBytes + ih * kBoxBytes;
      const int irow = i0 + 4 * ci + 32 * ih;  // global i of component 0
      uint4 w[4];
      w[0] = make_uint4(r[0].x, r[1].x, r[2].x, r[3].x);
      w[1] = make_uint4(r[0].y, r[1].y, r[2].y, r[3].y);
      w[2] = make_uint4(r[0].z, r[1].z, r[2].z, r[3].z);
      w[3] = make_uint4(r[0].w, r[1].w, r[2].w, r[3].w);
      const int j = 4 * cj + 32 * jh;  // output box row of w[0]
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int off = (j + q) * 128 + ((ci ^ ((j + q) & 7)) << 4);
        *reinterpret_cast<uint4 *>(ty + off) = w[q];
        const float yv[4] = {__uint_as_float(w[q].x), __uint_as_float(w[q].y), __uint_as_float(w[q].z),
                             __uint_as_float(w[q].w)};
        float zv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) zv[e] = f(yv[e]);
        *reinterpret_cast<uint4 *>(tz + off) =
            make_uint4(__float_as_uint(zv[0]), __float_as_uint(zv[1]), __float_as_uint(zv[2]), __float_as_uint(zv[3]));
        if (j0 + j + q < a.n1) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (irow + e < a.n0) {
              st.add(zv[e], 0);
              if (zv[e] == zv[e]) {  // NaN never wins, as in the argmax reduction
                const long long key = tc_key(zv[e], (int64_t)(irow + e) + c.index_base);
                kq[q] = key > kq[q] ? key : kq[q];
              }
            }
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->ofull[b]);
    }
    // this tile's per-row argmax: 16 partial keys per output row j
#pragma unroll
    for (int q = 0; q < 4; ++q) sh->tkeys[kb][4 * cj + 32 * jh + q][ib] = kq[q];
    tc_bar();
    if (tid < kTT) {
      long long m = sh->tkeys[kb][tid][0];
#pragma unroll
      for (int t = 1; t < 16; ++t) m = sh->tkeys[kb][tid][t] > m ? sh->tkeys[kb][tid][t] : m;
      if (m != LLONG_MIN && j0 + tid < a.n1) atomicMax(&c.keys[(int64_t)bb * a.n1 + j0 + tid], m);
    }
  }
  // the moments: warps, then the CTA, then the last CTA merges all in order
  warp_reduce(st);
  if (lane == 0) sh->wst[warp] = st;
  tc_bar();
  if (tid == 0) {
    VarAcc<float> v = sh->wst[0];
    for (int w = 1; w < kNTW; ++w) v.merge(sh->wst[w]);
    c.partials[blockIdx.x] = v;
    __threadfence();
    const unsigned int nparts = gridDim.x;
    const unsigned int t = atomicAdd(c.counter, 1u);
    if (t == nparts - 1) {
      __threadfence();
      VarAcc<float> g;
      g.init();
      g.set_shift(K);
      for (unsigned int q = 0; q < nparts; ++q) {
        VarAcc<float> pq;
        pq.k = __ldcg(&c.partials[q].k);
        pq.s1 = __ldcg(&c.partials[q].s1);
        pq.s2 = __ldcg(&c.partials[q].s2);
        g.merge(pq);
      }
      g.store(c.os, 0);
      *c.counter = 0u;
    }
  }
}

__global__ void k_fill_keys(long long *keys, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    keys[i] = LLONG_MIN;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

}  // namespace

bool encode_tensor_map_3d(CUtensorMap *map, const void *base, int elem_bytes, const int64_t dims[3],
                          const int64_t strides_elems[2], const uint32_t box[3], bool swizzle128,
                          bool promote256) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t gd[3], gs[2];
  for (int d = 0; d < 3; ++d) gd[d] = (cuuint64_t)dims[d];
  for (int d = 0; d < 2; ++d) gs[d] = (cuuint64_t)(strides_elems[d] * elem_bytes);
  cuuint32_t bx[3] = {box[0], box[1], box[2]};
  cuuint32_t es[3] = {1, 1, 1};
  const CUtensorMapDataType dt = elem_bytes == 8 ? CU_TENSOR_MAP_DATA_TYPE_UINT64 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
  return enc(map, dt, 3, const_cast<void *>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
             promote256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_NONE,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool launch_transpose_tma4(acd_ctx *ctx, void *out, const void *in, int64_t n0, int64_t n1, int64_t n2,
                           int64_t os1, int64_t os2, int64_t is0, int64_t is2, cudaStream_t stream) {
  // TMA needs 16-byte aligned bases and strides; coordinates are 32-bit
  if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) return false;
  if (is0 % 4 || os1 % 4 || (n2 > 1 && (is2 % 4 || os2 % 4))) return false;
  if (n0 < kTT || n1 < kTT || n0 >= (1ll << 31) || n1 >= (1ll << 31) || n2 >= (1ll << 31)) return false;
  if (n2 == 1) {
    is2 = is0 * n0;
    os2 = os1 * n1;
  }
  const int64_t lim = 1ll << 38;  // element strides below 2^40 bytes
  if (is0 >= lim || os1 >= lim || is2 >= lim || os2 >= lim) return false;
  CUtensorMap mi, mo;
  const int64_t din[3] = {n1, n0, n2}, sin_[2] = {is0, is2};
  const int64_t dout[3] = {n0, n1, n2}, sout_[2] = {os1, os2};
  const uint32_t box[3] = {32, kTT, 1};
  if (!encode_tensor_map_3d(&mi, in, 4, din, sin_, box)) return false;
  if (!encode_tensor_map_3d(&mo, out, 4, dout, sout_, box)) return false;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device
  const uint64_t bit = 1ull << (ctx->device & 63);
  if (!(attr_set.load() & bit)) {
    if (cudaFuncSetAttribute(k_transpose_tma4, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
        cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    attr_set.fetch_or(bit);
  }
  TtArgs a;
  a.tiles0 = (n0 + kTT - 1) / kTT;
  a.tiles1 = (n1 + kTT - 1) / kTT;
  a.nb = n2;
  a.n0 = (int)n0;
  a.n1 = (int)n1;
  a.control = ctx->control;
  const int grid = persistent_grid(ctx, k_transpose_tma4, kThreads, kSmemBytes, a.tiles0 * a.tiles1 * a.nb);
  k_transpose_tma4<<<grid, kThreads, kSmemBytes, stream>>>(mi, mo, a);
  return cudaGetLastError() == cudaSuccess;
}


bool launch_transpose_chain_tma4(acd_ctx *ctx, float *y, float *z, const float *in, int64_t n0, int64_t n1,
                                 int64_t is0, float p, double *stats, int64_t *keys, int64_t index_base,
                                 cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(z)) & 15)
    return false;
  if (is0 % 4 || n0 % 4) return false;
  if (n0 < kTT || n1 < kTT || n0 >= (1ll << 31) || n1 >= (1ll << 31)) return false;
  const int64_t lim = 1ll << 38;  // element strides below 2^40 bytes
  if (is0 >= lim || n0 * n1 >= lim || is0 * n0 >= lim) return false;
  CUtensorMap mi, my, mz;
  const int64_t din[3] = {n1, n0, 1}, sin_[2] = {is0, is0 * n0};
  const int64_t dout[3] = {n0, n1, 1}, sout_[2] = {n0, n0 * n1};
  const uint32_t box[3] = {32, kTT, 1};
  if (!encode_tensor_map_3d(&mi, in, 4, din, sin_, box)) return false;
  if (!encode_tensor_map_3d(&my, y, 4, dout, sout_, box)) return false;
  if (!encode_tensor_map_3d(&mz, z, 4, dout, sout_, box)) return false;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device
  const uint64_t bit = 1ull << (ctx->device & 63);
  if (!(attr_set.load() & bit)) {
    if (cudaFuncSetAttribute(k_transpose_chain_tma4, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kTcSmemBytes) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    attr_set.fetch_or(bit);
  }
  TtArgs a;
  a.tiles0 = (n0 + kTT - 1) / kTT;
  a.tiles1 = (n1 + kTT - 1) / kTT;
  a.nb = 1;
  a.n0 = (int)n0;
  a.n1 = (int)n1;
  a.control = ctx->control;
  const int grid = persistent_grid(ctx, k_transpose_chain_tma4, kThreads, kTcSmemBytes, a.tiles0 * a.tiles1);
  void *scratch;
  if (get_scratch(ctx, sizeof(VarAcc<float>) * (size_t)grid, stream, &scratch) != ACD_OK) return false;
  TcArgs c;
  c.in0 = in;
  c.p = p;
  c.keys = reinterpret_cast<long long *>(keys);
  c.index_base = index_base;
  c.partials = static_cast<VarAcc<float> *>(scratch);
  c.counter = &ctx->control->counters[0];
  c.os.mode = kModeStats;
  c.os.out = stats;
  c.os.op = ACD_RED_VAR;
  c.os.n = n0 * n1;
  k_fill_keys<<<grid_for(ctx, n1, 256, 4), 256, 0, stream>>>(c.keys, n1);
  k_transpose_chain_tma4<<<grid, kThreads, kTcSmemBytes, stream>>>(mi, my, mz, a, c);
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace acd
