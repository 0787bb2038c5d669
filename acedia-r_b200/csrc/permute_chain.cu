// The strided-views step in one pass over its input: y = contiguous(permuted
// view of x), z = y*p + exp(-(y^2)), the shifted moments of z and the argmax
// keys of z along y's axis 0, with x read once and y and z written once
// (12 bytes per element; the copy followed by the one-pass chain kernel
// moves 16).
//
// y(i, j, b) = x(i, j, b) with y contiguous along i (the argmax axis, extent
// n0 = F) and x contiguous along j.  The work is cut into 64 x 64 tiles as in
// the TMA transpose, and the tiles into sequences: sequence (j-tile, b) is
// the column of tiles that covers 64 whole fibers, and one CTA runs all of
// it, so each fiber's argmax is finished inside one CTA and stored with a
// plain write (no global atomics).  Sequences go to the persistent CTAs in
// turn; sequence s starts at i-tile s mod tiles0 and wraps, so the tiles in
// flight at one time sit at different offsets of their rows.
//
// Warp roles, with no block-wide barrier in the tile loop:
//   * one loading thread: TMA loads of x tiles into NS stages (two boxes of
//     32 j x 64 i, 128-byte swizzled);
//   * G groups of 8 compute warps: group g takes the CTA's tiles k with
//     k % G == g.  A thread owns one 4 x 4 block of the tile (the
//     bank-conflict-free mapping of the transpose), evaluates the chain on
//     its 16 values, writes the transposed block of y and of z into an
//     output buffer, adds the 16 values of z to its shifted moments and
//     keeps a running argmax for each of its 4 fibers;
//   * one storing thread: TMA stores of the y and z tiles (clipped at the
//     tensor edge).
// At the end of a sequence every compute thread folds its 4 running maxima
// into 64 shared 64-bit keys (atomicMax on the order-preserving key of
// acd_argmax_keys), the compute warps meet at a named barrier, and 64 threads
// store the keys.  At the end of the kernel the moments are reduced over the
// CTA and over the grid (the last CTA to finish merges the per-CTA partials
// and stores the statistics row).  Every mbarrier wait is bounded; when one
// expires the CTA raises status 2, the roles leave their loops (the compute
// warps still pass every named barrier, so none waits for a thread that
// left), and the loading thread waits, bounded, for its loads in flight.
#include <atomic>
#include <climits>

#include "ops.cuh"
#include "reduce_acc.cuh"
#include "tma.cuh"

namespace acd {

namespace {

constexpr int kPT = 64;                   // tile edge (elements)
constexpr int kPTile = kPT * kPT * 4;     // one 4-byte tile
constexpr int kPBox = kPTile / 2;         // one box (half a tile)
constexpr int kPNS = 4;                   // input stages
constexpr int kPNOB = 4;                  // output buffers (a y tile and a z tile each)
constexpr int kPG = 2;                    // compute groups of 8 warps
constexpr int kPCompute = 256 * kPG;      // compute threads
constexpr int kPThreads = kPCompute + 64; // plus a load warp and a store warp
constexpr uint64_t kPWaitNs = 1000000000ull;
// Group g takes the tiles k with k % G == g, so with NS and NOB multiples of
// G every stage and output buffer belongs to one group, whose warps take its
// tiles in order.  The parity waits rely on that: a waiter is never two
// phases ahead of its barrier.  (With a stage shared by two groups, a group
// whose earlier tile landed first could wait on a stage whose previous load
// is still in flight, and the parity of the phase two back would let it
// through.)
static_assert(kPNS % kPG == 0 && kPNOB % kPG == 0, "stages and output buffers must divide among the groups");

struct PcShared {
  uint64_t full[kPNS], empty[kPNS], ofull[kPNOB], ofree[kPNOB];
  unsigned long long key[2][kPT];  // per sequence parity: the 64 fibers' keys
  VarAcc<float> st[kPCompute / 32];
  int abort;
};
constexpr size_t kPSmem = (size_t)kPNS * kPTile + (size_t)kPNOB * 2 * kPTile + sizeof(PcShared) + 1024;

struct PcArgs {
  int64_t tiles0, tiles1, nseq;  // i-tiles per sequence, j-tiles, sequences (j-tiles x batches)
  int n0, n1;
  float p;
  int32_t pad;
  int64_t ks1, ks2;       // key index = j * ks1 + b * ks2
  int64_t index_base;     // added to the position along axis 0 in the keys
  long long *keys;
  const float *x0;        // x's first element: z's shift for the moments
  VarAcc<float> *partials;
  unsigned int *counter;
  OutSpec os;             // the statistics row
  Control *control;
};

// Bounded waits: one thread (the loading and storing roles) or a whole
// compute warp with one answer for all its lanes.
__device__ __forceinline__ bool pc_wait(uint64_t *bar, uint32_t parity, PcShared *sh, Control *c) {
  return mbar_wait_thread(bar, parity, &sh->abort, c, 2, kPWaitNs);
}
__device__ __forceinline__ bool pc_wait_warp(uint64_t *bar, uint32_t parity, PcShared *sh, Control *c) {
  return mbar_wait_warp(bar, parity, &sh->abort, c, 2, kPWaitNs);
}

// Barrier 1 of the compute warps.  The non-aligned form: each thread
// arrives on its own, so a warp that has not reconverged after the
// data-dependent branches before it still counts correctly; the __syncwarp
// reconverges it first all the same.
__device__ __forceinline__ void compute_sync() {
  __syncwarp();
  asm volatile("barrier.sync 1, %0;" ::"n"(kPCompute) : "memory");
}

// Sequence r of this CTA: its global number s, first column j0 and batch b.
__device__ __forceinline__ int64_t pc_seq(const PcArgs &a, int64_t r, int &j0, int &b) {
  const int64_t s = (int64_t)blockIdx.x + r * gridDim.x;
  const int64_t bb = s / a.tiles1;
  j0 = (int)((s - bb * a.tiles1) * kPT);
  b = (int)bb;
  return s;
}

// The i-tile of tile t of sequence s: (t + s) mod tiles0.  Each role takes
// it once per sequence and then steps it, wrapping, without a division.
__device__ __forceinline__ int pc_ti(const PcArgs &a, int64_t s, int64_t t) { return (int)((t + s) % a.tiles0); }

__device__ __forceinline__ uint32_t comp(const uint4 &v, int q) {
  return q == 0 ? v.x : (q == 1 ? v.y : (q == 2 ? v.z : v.w));
}

__global__ void __launch_bounds__(kPThreads, 1)
    k_permute_chain(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_y,
                    const __grid_constant__ CUtensorMap map_z, PcArgs a) {
  extern __shared__ unsigned char smem_raw[];
  // 128-byte swizzled boxes need 1024-byte aligned buffers
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                          ~static_cast<uintptr_t>(1023));
  unsigned char *sin = smem;
  unsigned char *sout = smem + kPNS * kPTile;  // buffer q: the y tile, then the z tile
  PcShared *sh = reinterpret_cast<PcShared *>(sout + kPNOB * 2 * kPTile);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // the grid is at most nseq, so every CTA has a sequence
  const int64_t my_nseq = (a.nseq - blockIdx.x + gridDim.x - 1) / gridDim.x;
  const int64_t T = a.tiles0;
  const int64_t my_n = my_nseq * T;
  if (tid == 0) {
    for (int s = 0; s < kPNS; ++s) {
      mbar_init(&sh->full[s], 1);
      mbar_init(&sh->empty[s], 8);
    }
    for (int q = 0; q < kPNOB; ++q) {
      mbar_init(&sh->ofull[q], 8);
      mbar_init(&sh->ofree[q], 1);
    }
    sh->abort = 0;
    mbar_init_fence();
  }
  for (int q = tid; q < 2 * kPT; q += blockDim.x) (&sh->key[0][0])[q] = 0ull;
  __syncthreads();

  if (warp == kPCompute / 32) {  // loader
    if (lane == 0) {
      int64_t k = 0;
      bool go = true;
      for (int64_t r = 0; go && r < my_nseq; ++r) {
        int j0, b;
        const int64_t sq = pc_seq(a, r, j0, b);
        const bool two = j0 + 32 < a.n1;  // a box wholly past the last column is not loaded
        int ti = pc_ti(a, sq, 0);
        for (int64_t t = 0; t < T; ++t, ++k) {
          const int s = (int)(k % kPNS);
          if (!pc_wait(&sh->empty[s], (uint32_t)(((k / kPNS) & 1) ^ 1), sh, a.control)) {
            go = false;
            break;
          }
          mbar_arrive_expect_tx(&sh->full[s], two ? kPTile : kPBox);
          tma_load_3d(sin + s * kPTile, &map_x, &sh->full[s], j0, ti * kPT, b);
          if (two) tma_load_3d(sin + s * kPTile + kPBox, &map_x, &sh->full[s], j0 + 32, ti * kPT, b);
          if (++ti == (int)T) ti = 0;
        }
      }
      if (*reinterpret_cast<volatile int *>(&sh->abort)) {
        // the loads issued last may still be landing in this CTA's shared memory
        for (int64_t q = (k > kPNS ? k - kPNS : 0); q < k; ++q) {
          WaitClock clk;
          while (!mbar_try_wait(&sh->full[q % kPNS], (uint32_t)((q / kPNS) & 1)) && !clk.expired(kPWaitNs)) {
          }
        }
      }
    }
    return;
  }
  if (warp == kPCompute / 32 + 1) {  // storer
    if (lane == 0) {
      int64_t k = 0;
      bool go = true;
      for (int64_t r = 0; go && r < my_nseq; ++r) {
        int j0, b;
        const int64_t sq = pc_seq(a, r, j0, b);
        int ti = pc_ti(a, sq, 0);
        for (int64_t t = 0; t < T; ++t, ++k) {
          const int ob = (int)(k % kPNOB);
          if (!pc_wait(&sh->ofull[ob], (uint32_t)((k / kPNOB) & 1), sh, a.control)) {
            go = false;
            break;
          }
          const int i0 = ti * kPT;
          const unsigned char *ty = sout + ob * 2 * kPTile;
          tma_store_3d(&map_y, ty, i0, j0, b);
          tma_store_3d(&map_z, ty + kPTile, i0, j0, b);
          if (i0 + 32 < a.n0) {
            tma_store_3d(&map_y, ty + kPBox, i0 + 32, j0, b);
            tma_store_3d(&map_z, ty + kPTile + kPBox, i0 + 32, j0, b);
          }
          bulk_commit();
          if (k >= 1) {
            bulk_wait_read<1>();  // the previous tile's stores have read its buffer
            mbar_arrive(&sh->ofree[(k - 1) % kPNOB]);
          }
          if (++ti == (int)T) ti = 0;
        }
      }
      bulk_wait_all();
    }
    return;
  }

  // compute warps: thread -> 4 x 4 block (ib, jb) of the tile, ib, jb in 0..15
  const int g = warp >> 3, wq = warp & 7;
  const int k8 = lane & 7;
  const int shift = (lane >> 3) | ((wq & 1) << 2);
  const int ih = (wq >> 1) & 1, jh = wq >> 2;
  const int ib = 8 * ih + k8, jb = 8 * jh + ((k8 + shift) & 7);
  const int cj = jb & 7, ci = k8;  // 16-byte chunk within a 128-byte row
  const FusedScaleAddExpNegSquare<float> f{a.p};
  const float K = f(__ldg(a.x0));
  VarAcc<float> st;
  st.init();
  st.set_shift(K);
  float av[4];
  int ai[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    av[q] = -INFINITY;
    ai[q] = INT_MAX;
  }
  bool live = true;
  for (int64_t r = 0; r < my_nseq; ++r) {
    int j0, b;
    const int64_t sq = pc_seq(a, r, j0, b);
    const bool jfull = j0 + kPT <= a.n1;
    // this group's tiles of the sequence: k = r*T + t with k % G == g
    const int64_t k0 = r * T;
    int64_t t = (int64_t)((g - (int)(k0 % kPG) + kPG) % kPG);
    int ti = pc_ti(a, sq, t);
    for (; live && t < T; t += kPG) {
      const int64_t k = k0 + t;
      const int i0 = ti * kPT;
      ti += kPG;
      while (ti >= (int)T) ti -= (int)T;
      const int s = (int)(k % kPNS);
      if (!pc_wait_warp(&sh->full[s], (uint32_t)((k / kPNS) & 1), sh, a.control)) {
        live = false;
        break;
      }
      const unsigned char *tin = sin + s * kPTile + jh * kPBox;
      uint4 rv[4];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i = 4 * ci + m + 32 * ih;  // input box row
        rv[m] = *reinterpret_cast<const uint4 *>(tin + i * 128 + ((cj ^ (i & 7)) << 4));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[s]);
      float zf[4][4];  // [position along i][fiber]
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int q = 0; q < 4; ++q) zf[m][q] = f(__uint_as_float(comp(rv[m], q)));
      const int ob = (int)(k % kPNOB);
      if (!pc_wait_warp(&sh->ofree[ob], (uint32_t)(((k / kPNOB) & 1) ^ 1), sh, a.control)) {
        live = false;
        break;
      }
      unsigned char *ty = sout + ob * 2 * kPTile + ih * kPBox;
      unsigned char *tz = ty + kPTile;
      const int jr = 4 * cj + 32 * jh;  // output box row of fiber 0
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = jr + q;
        const int off = j * 128 + ((ci ^ (j & 7)) << 4);
        *reinterpret_cast<uint4 *>(ty + off) = make_uint4(comp(rv[0], q), comp(rv[1], q), comp(rv[2], q), comp(rv[3], q));
        *reinterpret_cast<float4 *>(tz + off) = make_float4(zf[0][q], zf[1][q], zf[2][q], zf[3][q]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->ofull[ob]);
      // moments and running maxima (a larger value wins; among equal values
      // the smaller index, since the tiles of a sequence do not come in index
      // order; NaN never wins; an all -inf fiber keeps its first element)
      const int ibase = i0 + 4 * ib;
      if (jfull && i0 + kPT <= a.n0) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
#pragma unroll
          for (int m = 0; m < 4; ++m) st.add(zf[m][q], 0);
          // the block's maximum (fmaxf passes NaN over; four NaN give NaN,
          // which takes no part), then, only when it reaches the running
          // one, its first position
          const float tm = fmaxf(fmaxf(zf[0][q], zf[1][q]), fmaxf(zf[2][q], zf[3][q]));
          if (tm >= av[q]) {
            const int idx = ibase + (zf[0][q] == tm ? 0 : zf[1][q] == tm ? 1 : zf[2][q] == tm ? 2 : 3);
            if (tm > av[q] || idx < ai[q]) {
              av[q] = tm;
              ai[q] = idx;
            }
          }
        }
      } else {  // a ragged tile: elements past either edge take no part
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (j0 + 4 * jb + q >= a.n1) continue;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            if (ibase + m >= a.n0) continue;
            const float v = zf[m][q];
            st.add(v, 0);
            const bool better = v > av[q] || (v == av[q] && ibase + m < ai[q]);
            av[q] = better ? v : av[q];
            ai[q] = better ? ibase + m : ai[q];
          }
        }
      }
    }
    // the sequence's 64 keys: every compute thread folds in its 4 maxima
    // (key layout of ArgAcc<float>::store in kModeKey, before the sign flip)
    const int kb = (int)(r & 1);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (ai[q] != INT_MAX) {
        const uint32_t obits = ordered_bits(av[q] + 0.0f);
        const uint32_t gi = (uint32_t)((int64_t)ai[q] + a.index_base);
        const unsigned long long u = ((unsigned long long)obits << 32) | (unsigned long long)(0xFFFFFFFFu - gi);
        atomicMax(&sh->key[kb][4 * jb + q], u);
      }
      av[q] = -INFINITY;
      ai[q] = INT_MAX;
    }
    compute_sync();
    if (tid < kPT) {
      // key[kb] is next written two sequences on, after the barrier of the
      // sequence in between, so this reset cannot race with those atomics
      const unsigned long long u = sh->key[kb][tid];
      sh->key[kb][tid] = 0ull;
      if (j0 + tid < a.n1)
        a.keys[(int64_t)(j0 + tid) * a.ks1 + (int64_t)b * a.ks2] = (long long)(u ^ 0x8000000000000000ull);
    }
  }

  // moments: warps, then the CTA, then the grid (the last CTA merges)
  warp_reduce(st);
  if (lane == 0) sh->st[warp] = st;
  compute_sync();
  if (warp == 0) {
    VarAcc<float> c;
    if (lane < kPCompute / 32) {
      c = sh->st[lane];
    } else {
      c.init();
      c.set_shift(K);
    }
    warp_reduce(c);
    int last = 0;
    if (lane == 0) {
      a.partials[blockIdx.x] = c;
      __threadfence();
      last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence();
      VarAcc<float> tot;
      tot.init();
      tot.set_shift(K);
      for (int q = lane; q < (int)gridDim.x; q += 32) {
        VarAcc<float> o;
        o.k = K;
        o.s1 = __ldcg(&a.partials[q].s1);
        o.s2 = __ldcg(&a.partials[q].s2);
        tot.merge(o);
      }
      warp_reduce(tot);
      if (lane == 0) {
        tot.store(a.os, 0);
        *a.counter = 0u;
      }
    }
  }
}

}  // namespace

acd_status launch_permute_chain(acd_ctx *ctx, float *y, float *z, const float *x, int64_t n0, int64_t n1,
                                int64_t n2, int64_t os1, int64_t os2, int64_t is0, int64_t is2, float p,
                                double *stats, int64_t n_total, long long *keys, int64_t index_base,
                                cudaStream_t stream, bool *launched) {
  *launched = false;
  // TMA needs 16-byte aligned bases and strides; coordinates are 32-bit
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(z)) & 15)
    return ACD_OK;
  if (is0 % 4 || os1 % 4 || (n2 > 1 && (is2 % 4 || os2 % 4))) return ACD_OK;
  if (n0 < kPT || n1 < kPT || n0 >= (1ll << 31) || n1 >= (1ll << 31) || n2 >= (1ll << 31)) return ACD_OK;
  if (n2 == 1) {
    is2 = is0 * n0;
    os2 = os1 * n1;
  }
  // y is contiguous with fibers of n0 elements: the key of fiber (j, b) goes
  // to (j * os1 + b * os2) / n0
  if (os1 % n0 || os2 % n0) return ACD_OK;
  const int64_t lim = 1ll << 38;  // element strides below 2^40 bytes
  if (is0 >= lim || os1 >= lim || is2 >= lim || os2 >= lim) return ACD_OK;
  CUtensorMap mx, my, mz;
  const int64_t din[3] = {n1, n0, n2}, sin_[2] = {is0, is2};
  const int64_t dout[3] = {n0, n1, n2}, sout_[2] = {os1, os2};
  const uint32_t box[3] = {32, kPT, 1};
  if (!encode_tensor_map_3d(&mx, x, 4, din, sin_, box)) return ACD_OK;
  if (!encode_tensor_map_3d(&my, y, 4, dout, sout_, box)) return ACD_OK;
  if (!encode_tensor_map_3d(&mz, z, 4, dout, sout_, box)) return ACD_OK;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device
  const uint64_t bit = 1ull << (ctx->device & 63);
  if (!(attr_set.load() & bit)) {
    if (cudaFuncSetAttribute(k_permute_chain, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem) !=
        cudaSuccess) {
      cudaGetLastError();
      return ACD_OK;
    }
    attr_set.fetch_or(bit);
  }
  PcArgs a;
  a.tiles0 = (n0 + kPT - 1) / kPT;
  a.tiles1 = (n1 + kPT - 1) / kPT;
  a.nseq = a.tiles1 * n2;
  a.n0 = (int)n0;
  a.n1 = (int)n1;
  a.p = p;
  a.pad = 0;
  a.ks1 = os1 / n0;
  a.ks2 = os2 / n0;
  a.index_base = index_base;
  a.keys = keys;
  a.x0 = x;
  a.control = ctx->control;
  a.counter = &ctx->control->counters[0];
  a.os.mode = kModeStats;
  a.os.out = stats;
  a.os.op = ACD_RED_VAR;
  a.os.n = n_total;
  const int grid = persistent_grid(ctx, k_permute_chain, kPThreads, kPSmem, a.nseq);
  void *scratch;
  ACD_TRY(get_scratch(ctx, (sizeof(VarAcc<float>) * grid + 255) / 256 * 256, stream, &scratch));
  a.partials = static_cast<VarAcc<float> *>(scratch);
  k_permute_chain<<<grid, kPThreads, kPSmem, stream>>>(mx, my, mz, a);
  ACD_CUDA(cudaGetLastError());
  *launched = true;
  return ACD_OK;
}

}  // namespace acd
