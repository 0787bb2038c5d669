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

// Bounded waits that also give up once another role of the CTA has aborted:
// one thread (the loading and storing roles), or a whole transpose warp with
// one answer for all its lanes.
__device__ __forceinline__ bool tt_wait(uint64_t *bar, uint32_t parity, TtShared *sh, const TtArgs &a) {
  return mbar_wait_thread(bar, parity, &sh->abort, a.control, 2, kWaitNs);
}
__device__ __forceinline__ bool tt_wait_warp(uint64_t *bar, uint32_t parity, TtShared *sh, const TtArgs &a) {
  return mbar_wait_warp(bar, parity, &sh->abort, a.control, 2, kWaitNs);
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
          WaitClock clk;
          while (!mbar_try_wait(&sh->full[q % kNS], (uint32_t)((q / kNS) & 1)) && !clk.expired(kWaitNs)) {
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
    if (!tt_wait_warp(&sh->full[s], (uint32_t)((k / kNS) & 1), sh, a)) break;
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
    if (!tt_wait_warp(&sh->ofree[b], (uint32_t)(((k / kNOB) & 1) ^ 1), sh, a)) break;
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

}  // namespace acd
