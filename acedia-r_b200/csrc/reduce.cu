// Full and per-axis reductions, arg-reductions, the fused sum+variance pass
// and the per-shard partials used by the multi-GPU path.
//
// Reference counterparts and what changes:
//   reduction_kernel + launch_reduction (src/kernels/tensor_kernels.cu:60-84,
//   src/kernels/tensor_ops.cu:50-126): one element per thread, grid capped at
//   65535 blocks with no grid-stride loop (only the first 16,776,960 elements
//   are reduced), partials finished on the host.  Here: one launch over a
//   persistent grid with 16-byte loads; the last CTA to finish merges the
//   per-CTA partials in a fixed order, so results are deterministic and never
//   leave the device.
//   axis_reduction_kernel (src/kernels/tensor_kernels.cu:488-698): one block
//   per output element, uncoalesced reads for outer axes, per-call cudaMalloc
//   of metadata.  Here the reduced axes are collapsed to (I, R, O) and one of
//   two layouts is used: inner (R contiguous: a warp or a CTA per output,
//   vector loads) or outer (R strided: threads own adjacent outputs so loads
//   along I coalesce; R is split across CTAs when I*O is small and the splits
//   are merged in order by the last CTA of each tile).
//   axis_variance_kernel (src/kernels/tensor_kernels.cu:810-834) writes zeros;
//   here variance is computed for real.
//   argmax/argmin: global argmax copies the tensor to the host
//   (src/kernels/tensor_ops.cu:850-880), global argmin scans 256 elements
//   (src/kernels/tensor_kernels.cu:1224-1309); both become device reductions.
#include "common.cuh"
#include "ops.cuh"
#include "reduce_acc.cuh"
#include "tma.cuh"

namespace acd {

template <class A>
__device__ __forceinline__ A load_cg(const A *p) {
  A r;
  const int *s = reinterpret_cast<const int *>(p);
  int *d = reinterpret_cast<int *>(&r);
#pragma unroll
  for (int k = 0; k < (int)(sizeof(A) / 4); ++k) d[k] = __ldcg(s + k);
  return r;
}

constexpr int kRedThreads = 512;

// Block partial -> partials[blockIdx.x]; the last CTA merges all partials in
// index order and stores the result.  `K` re-seeds the shift of the final
// accumulator.
template <class Acc, typename T>
__device__ __forceinline__ void finish_grid(Acc &acc, Acc *smem, Acc *__restrict__ partials, unsigned int *counter,
                                            const OutSpec &os, int64_t oi, T K) {
  __shared__ int am_last;
  block_reduce(acc, smem);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = acc;
    __threadfence();
    const unsigned int t = atomicAdd(counter, 1u);
    am_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (am_last) {
    __threadfence();
    Acc f;
    f.init();
    if constexpr (Acc::kShift) f.set_shift(K);
    for (int b = threadIdx.x; b < (int)gridDim.x; b += blockDim.x) f.merge(load_cg(partials + b));
    block_reduce(f, smem);
    if (threadIdx.x == 0) {
      f.store(os, oi);
      *counter = 0u;
    }
  }
}

// ---- full reduction over a dense range ------------------------------------
template <class Acc, typename T, int V, int U>
__global__ void __launch_bounds__(kRedThreads) k_red_flat(const T *__restrict__ in, int64_t n, int64_t head,
                                                          Acc *__restrict__ partials, unsigned int *counter,
                                                          OutSpec os) {
  __shared__ Acc smem[kRedThreads / 32];
  Acc acc;
  acc.init();
  T K = T(0);
  if constexpr (Acc::kShift) {
    K = in[0];
    acc.set_shift(K);
  }
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t nvec = (n - head) / V;
  const int64_t tail = head + nvec * V;
  const int64_t nscalar = head + (n - tail);
  for (int64_t i = tid; i < nscalar; i += nth) {
    const int64_t e = i < head ? i : tail + (i - head);
    acc.add(in[e], e);
  }
  const Vec<T, V> *pv = reinterpret_cast<const Vec<T, V> *>(in + head);
  // one accumulator per vector in flight: no dependency chain links the U
  // loads of an iteration, so they stay in flight together
  Acc part[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    part[u].init();
    if constexpr (Acc::kShift) part[u].set_shift(K);
  }
  // main loop: U full vectors per thread, no guards, so all U loads are
  // issued before any is consumed
  int64_t v0 = tid;
  for (; v0 + (int64_t)(U - 1) * nth < nvec; v0 += nth * U) {
    Vec<T, V> x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) x[u] = pv[v0 + (int64_t)u * nth];
#pragma unroll
    for (int u = 0; u < U; ++u) acc_add_vec(part[u], x[u], head + (v0 + (int64_t)u * nth) * V);
  }
  // remainder: fewer than U vectors left for this thread
  for (int u = 0; v0 + (int64_t)u * nth < nvec; ++u) {
    const int64_t v = v0 + (int64_t)u * nth;
    acc_add_vec(part[0], pv[v], head + v * V);
  }
#pragma unroll
  for (int u = 0; u < U; ++u) acc.merge(part[u]);
  finish_grid(acc, smem, partials, counter, os, 0, K);
}

struct Space1 {
  int32_t ndim;
  int64_t shape[ACD_MAX_DIMS];
  int64_t st[ACD_MAX_DIMS];
};

// ---- full reduction over any strided view (logical column-major order) ----
template <class Acc, typename T>
__global__ void __launch_bounds__(kRedThreads) k_red_strided(const T *__restrict__ in, Space1 g, int64_t n,
                                                             Acc *__restrict__ partials, unsigned int *counter,
                                                             OutSpec os) {
  __shared__ Acc smem[kRedThreads / 32];
  constexpr int RUN = 4;
  Acc acc;
  acc.init();
  T K = T(0);
  if constexpr (Acc::kShift) {
    K = in[0];
    acc.set_shift(K);
  }
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = tid * RUN; base < n; base += nth * RUN) {
    int64_t c[ACD_MAX_DIMS];
    int64_t off = 0, rem = base;
    for (int d = 0; d < g.ndim; ++d) {
      c[d] = rem % g.shape[d];
      rem /= g.shape[d];
      off += c[d] * g.st[d];
    }
    for (int r = 0; r < RUN && base + r < n; ++r) {
      acc.add(in[off], base + r);
      off += g.st[0];
      if (++c[0] == g.shape[0]) {
        c[0] = 0;
        off -= g.shape[0] * g.st[0];
        for (int d = 1; d < g.ndim; ++d) {
          off += g.st[d];
          if (++c[d] < g.shape[d]) break;
          c[d] = 0;
          off -= g.shape[d] * g.st[d];
        }
      }
    }
  }
  finish_grid(acc, smem, partials, counter, os, 0, K);
}

// ---- inner axis: out[o] = reduce_r in[o*so + r*sr], a warp per output -----
template <class Acc, typename T, int V, bool VEC>
__global__ void __launch_bounds__(256) k_red_inner_warp(const T *__restrict__ in, int64_t R, int64_t sr, int64_t so,
                                                        int64_t O, OutSpec os) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t o = warp; o < O; o += nwarps) {
    const T *p = in + o * so;
    Acc acc;
    acc.init();
    if constexpr (Acc::kShift) acc.set_shift(p[0]);
    if constexpr (VEC) {
      // vectors in flight per lane: 16 for bytes (bool counts: a whole 8 KB
      // column of a warp in one batch, 17.7 -> 15.7 us for count(M) of
      // 8192x8192 bool), 8 otherwise (colSums of 8192x8192 float32
      // 0.049 -> 0.042 ms)
      constexpr int U = sizeof(T) == 1 ? 16 : 8;
      const int64_t nv = R / V;
      const Vec<T, V> *pv = reinterpret_cast<const Vec<T, V> *>(p);
      int64_t v0 = lane;
      for (; v0 + 32 * (U - 1) < nv; v0 += 32 * U) {  // U full vectors: unguarded loads
        Vec<T, V> x[U];
#pragma unroll
        for (int u = 0; u < U; ++u) x[u] = pv[v0 + 32 * u];
#pragma unroll
        for (int u = 0; u < U; ++u) acc_add_vec(acc, x[u], (v0 + 32 * u) * V);
      }
      for (; v0 < nv; v0 += 32) acc_add_vec(acc, pv[v0], v0 * V);
      for (int64_t r = nv * V + lane; r < R; r += 32) acc.add(p[r], r);
    } else {
      for (int64_t r = lane; r < R; r += 32) acc.add(p[r * sr], r);
    }
    warp_reduce(acc);
    if (lane == 0) acc.store(os, o);
  }
}

// ---- inner axis, few long fibers: CTAs split each fiber ---------------------
template <class Acc, typename T, int V, bool VEC>
__global__ void __launch_bounds__(kRedThreads) k_red_inner_cta(const T *__restrict__ in, int64_t R, int64_t sr,
                                                               int64_t so, int64_t S, int64_t chunk,
                                                               Acc *__restrict__ partials, unsigned int *counters,
                                                               OutSpec os) {
  __shared__ Acc smem[kRedThreads / 32];
  __shared__ int am_last;
  const int64_t o = blockIdx.x / S, s = blockIdx.x % S;
  const T *p = in + o * so;
  const int64_t r0 = s * chunk;
  const int64_t r1 = (r0 + chunk < R) ? r0 + chunk : R;
  Acc acc;
  acc.init();
  T K = T(0);
  if constexpr (Acc::kShift) {
    K = p[0];
    acc.set_shift(K);
  }
  if constexpr (VEC) {  // chunk is a multiple of V, p is V-aligned
    const int64_t v_beg = r0 / V, v_end = r1 / V;
    const Vec<T, V> *pv = reinterpret_cast<const Vec<T, V> *>(p);
    constexpr int U = 4;
    int64_t v0 = v_beg + threadIdx.x;
    for (; v0 + (int64_t)blockDim.x * (U - 1) < v_end; v0 += (int64_t)blockDim.x * U) {  // unguarded
      Vec<T, V> x[U];
#pragma unroll
      for (int u = 0; u < U; ++u) x[u] = pv[v0 + (int64_t)blockDim.x * u];
#pragma unroll
      for (int u = 0; u < U; ++u) acc_add_vec(acc, x[u], (v0 + (int64_t)blockDim.x * u) * V);
    }
    for (; v0 < v_end; v0 += blockDim.x) acc_add_vec(acc, pv[v0], v0 * V);
    for (int64_t r = v_end * V + threadIdx.x; r < r1; r += blockDim.x) acc.add(p[r], r);
  } else {
    for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) acc.add(p[r * sr], r);
  }
  block_reduce(acc, smem);
  if (S == 1) {
    if (threadIdx.x == 0) acc.store(os, o);
    return;
  }
  if (threadIdx.x == 0) {
    partials[o * S + s] = acc;
    __threadfence();
    const unsigned int t = atomicAdd(&counters[o], 1u);
    am_last = (t == (unsigned int)(S - 1));
  }
  __syncthreads();
  if (am_last && threadIdx.x == 0) {
    __threadfence();
    Acc f = load_cg(partials + o * S);
    for (int64_t q = 1; q < S; ++q) f.merge(load_cg(partials + o * S + q));
    if constexpr (Acc::kShift) f.set_shift(K);
    f.store(os, o);
    counters[o] = 0u;
  }
}

// ---- outer axis: out[i + I*o] = reduce_r in[i*si + r*sr + o*so] -----------
// A CTA covers TI = 32*V*WI consecutive i; WR warps split the r range.
// Registers bound the loads in flight per SM.  Left free, the compiler gave
// even a one-double accumulator ~155 registers (1 CTA per SM, 8 warps, 0.26 ms
// for a float32 sum along axis 2 of 4096x4096x16).  Accumulators of up to 16
// bytes are held to 4 CTAs per SM (64 registers), larger ones (variance:
// shift and two float64 sums) to 3; eight rows are in flight per thread
// unless the V accumulators take more than 96 bytes (then four).  Measured
// against 2 and 1 CTAs per SM and four rows: this is the fastest or within 2%
// for sum, mean, var, max and argmax along axes 2 and 3 (0.157-0.21 ms).
template <class Acc>
__host__ __device__ constexpr int outer_min_blocks() { return sizeof(Acc) > 16 ? 3 : 4; }
template <class Acc, int V>
__host__ __device__ constexpr int outer_rows_in_flight() { return sizeof(Acc) * V > 96 ? 4 : 8; }

template <class Acc, typename T, int V, int WR, bool VEC>
__global__ void __launch_bounds__(256, outer_min_blocks<Acc>()) k_red_outer(const T *__restrict__ in, int64_t I, int64_t R, int64_t si,
                                                   int64_t sr, int64_t so, int64_t O, int64_t S, int64_t chunk,
                                                   int64_t itiles, Acc *__restrict__ partials,
                                                   unsigned int *counters, OutSpec os) {
  constexpr int WI = 8 / WR;
  constexpr int TI = 32 * V * WI;
  __shared__ Acc smem[WR > 1 ? WR : 1][WR > 1 ? 32 * V : 1];
  __shared__ int am_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wi = warp % WI, wr = warp / WI;
  const int64_t s = blockIdx.x % S;
  const int64_t rest = blockIdx.x / S;
  const int64_t it = rest % itiles, o = rest / itiles;
  const int64_t i0 = it * TI + (int64_t)(wi * 32 + lane) * V;
  const int64_t r0 = s * chunk;
  const int64_t r1 = (r0 + chunk < R) ? r0 + chunk : R;
  const T *base = in + o * so;

  Acc acc[V];
  const bool full = VEC && (i0 + V <= I);
  int64_t r = r0 + wr;
  // the shift is row 0 of each output: a thread whose first row is row 0
  // takes it from that row's load, others load it as one vector
  bool need_shift = false;
#pragma unroll
  for (int k = 0; k < V; ++k) acc[k].init();
  if constexpr (Acc::kShift) {
    if (full && r == 0 && r < r1) {
      need_shift = true;
    } else if (full) {
      const Vec<T, V> k0 = *reinterpret_cast<const Vec<T, V> *>(base + i0);
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k].set_shift(k0.v[k]);
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k)
        if (i0 + k < I) acc[k].set_shift(base[(i0 + k) * si]);
    }
  }
  if (full) {
    // RU rows in flight per thread; accumulation stays in row order.  The
    // loop is not unrolled further, so the register bound, not unrolling,
    // sets the loads in flight per SM.
    constexpr int RU = outer_rows_in_flight<Acc, V>();
#pragma unroll 1
    for (; r + (RU - 1) * WR < r1; r += RU * WR) {
      Vec<T, V> x[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) x[u] = *reinterpret_cast<const Vec<T, V> *>(base + (r + u * WR) * sr + i0);
      if constexpr (Acc::kShift) {
        if (need_shift) {  // x[0] is row 0
#pragma unroll
          for (int k = 0; k < V; ++k) acc[k].set_shift(x[0].v[k]);
          need_shift = false;
        }
      }
#pragma unroll
      for (int u = 0; u < RU; ++u) {
#pragma unroll
        for (int k = 0; k < V; ++k) acc[k].add(x[u].v[k], r + u * WR);
      }
    }
  }
#pragma unroll 1
  for (; r < r1; r += WR) {
    const T *row = base + r * sr;
    if (full) {
      const Vec<T, V> x = *reinterpret_cast<const Vec<T, V> *>(row + i0);
      if constexpr (Acc::kShift) {
        if (need_shift) {  // this row is row 0
#pragma unroll
          for (int k = 0; k < V; ++k) acc[k].set_shift(x.v[k]);
          need_shift = false;
        }
      }
#pragma unroll
      for (int k = 0; k < V; ++k) acc[k].add(x.v[k], r);
    } else {
#pragma unroll
      for (int k = 0; k < V; ++k)
        if (i0 + k < I) acc[k].add(row[(i0 + k) * si], r);
    }
  }
  if constexpr (WR > 1) {
    // merge the WR partial accumulators of each output in r order
    if (wr > 0) {
#pragma unroll
      for (int k = 0; k < V; ++k) smem[wr][lane * V + k] = acc[k];
    }
    __syncthreads();
    if (wr == 0) {
#pragma unroll
      for (int k = 0; k < V; ++k)
        for (int q = 1; q < WR; ++q) acc[k].merge(smem[q][lane * V + k]);
    }
  }
  if (S == 1) {
    if (wr == 0) {
#pragma unroll
      for (int k = 0; k < V; ++k)
        if (i0 + k < I) acc[k].store(os, (i0 + k) + I * o);
    }
    return;
  }
  // split over r: write partials, the last CTA of this (tile, o) merges them
  const int64_t nout = I * O;
  if (wr == 0) {
#pragma unroll
    for (int k = 0; k < V; ++k)
      if (i0 + k < I) partials[s * nout + (i0 + k) + I * o] = acc[k];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int t = atomicAdd(&counters[it + itiles * o], 1u);
    am_last = (t == (unsigned int)(S - 1));
  }
  __syncthreads();
  if (am_last) {
    // every thread merges whole outputs of the tile, adjacent threads adjacent
    // outputs (coalesced partial reads), four partials in flight, in q order
    __threadfence();
    for (int j = threadIdx.x; j < TI; j += blockDim.x) {
      const int64_t i = it * TI + j;
      if (i >= I) break;
      const int64_t oi = i + I * o;
      const Acc *pp = partials + oi;
      Acc f = load_cg(pp);
      int64_t q = 1;
#pragma unroll 1
      for (; q + 3 < S; q += 4) {
        const Acc a0 = load_cg(pp + q * nout), a1 = load_cg(pp + (q + 1) * nout);
        const Acc a2 = load_cg(pp + (q + 2) * nout), a3 = load_cg(pp + (q + 3) * nout);
        f.merge(a0);
        f.merge(a1);
        f.merge(a2);
        f.merge(a3);
      }
#pragma unroll 1
      for (; q < S; ++q) f.merge(load_cg(pp + q * nout));
      if constexpr (Acc::kShift) f.set_shift(base[i * si]);
      f.store(os, oi);
    }
    if (threadIdx.x == 0) counters[it + itiles * o] = 0u;
  }
}

// ---- the elementwise chain with its statistics and argmax keys, one pass ----
// z = x*p + exp(-(x^2)) over a contiguous float32 tensor whose axis 0 (the
// argmax axis) has F elements, F a multiple of 4.  Each warp takes whole
// fibers (F consecutive elements) in turn: it writes z with 16-byte stores,
// keeps each thread's running argmax of the fiber (its indices only grow, so
// a strict > keeps the first of equal values; an all -inf fiber takes its
// first element, as the argmax reduction does; NaN never wins) and reduces it to one key per
// fiber (as acd_argmax_keys) with shuffles only.  The threads' shifted moments
// of z (shift K = z[0], as acd_stats_partial) run across all their fibers and
// meet in finish_grid.  No block-wide barrier until the end, so the loads of
// one fiber follow the previous one's without a drain; z is read by nothing
// else, so the step moves 8 bytes per element instead of 16.
constexpr int kChainThreads = 256;

template <int U>
__global__ void __launch_bounds__(kChainThreads) k_chain_stats_keys(const float *__restrict__ x, float *__restrict__ z,
                                                                    int64_t F, int64_t nfib, float p,
                                                                    VarAcc<float> *__restrict__ partials,
                                                                    unsigned int *counter, OutSpec os_stats,
                                                                    long long *__restrict__ keys, int64_t index_base) {
  __shared__ VarAcc<float> smem_st[kChainThreads / 32];
  const FusedScaleAddExpNegSquare<float> f{p};
  const float K = f(x[0]);
  VarAcc<float> st;
  st.init();
  st.set_shift(K);
  OutSpec os_key;
  os_key.mode = kModeKey;
  os_key.out = keys;
  os_key.index_base = index_base;
  const int lane = threadIdx.x & 31;
  const int64_t nv = F / 4;
  const int64_t gw = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t fb = gw; fb < nfib; fb += nw) {
    const Vec<float, 4> *xi = reinterpret_cast<const Vec<float, 4> *>(x + fb * F);
    Vec<float, 4> *zo = reinterpret_cast<Vec<float, 4> *>(z + fb * F);
    ArgAcc<float, true> am;
    am.init();
    int64_t v = lane;
    for (; v + 32 * (U - 1) < nv; v += 32 * U) {  // U vectors in flight, unguarded
      Vec<float, 4> a[U];
#pragma unroll
      for (int u = 0; u < U; ++u) a[u] = xi[v + 32 * u];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        Vec<float, 4> r;
#pragma unroll
        for (int k = 0; k < 4; ++k) r.v[k] = f(a[u].v[k]);
        zo[v + 32 * u] = r;
        const int64_t i0 = (v + 32 * u) * 4;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          st.add(r.v[k], 0);
          if (r.v[k] > am.v || (r.v[k] == am.v && am.i == LLONG_MAX)) {  // first -inf too
            am.v = r.v[k];
            am.i = i0 + k;
          }
        }
      }
    }
    for (; v < nv; v += 32) {
      const Vec<float, 4> a = xi[v];
      Vec<float, 4> r;
#pragma unroll
      for (int k = 0; k < 4; ++k) r.v[k] = f(a.v[k]);
      zo[v] = r;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        st.add(r.v[k], 0);
        if (r.v[k] > am.v || (r.v[k] == am.v && am.i == LLONG_MAX)) {
          am.v = r.v[k];
          am.i = v * 4 + k;
        }
      }
    }
    warp_reduce(am);
    if (lane == 0) am.store(os_key, fb);
  }
  finish_grid(st, smem_st, partials, counter, os_stats, 0, K);
}

// ---- generic: any set of reduced axes, a warp per output --------------------
struct AxisSpace {
  int32_t nk, nr;
  int64_t kshape[ACD_MAX_DIMS], kst[ACD_MAX_DIMS];
  int64_t rshape[ACD_MAX_DIMS], rst[ACD_MAX_DIMS];
};

template <class Acc, typename T>
__global__ void __launch_bounds__(256) k_red_generic(const T *__restrict__ in, AxisSpace a, int64_t O, int64_t R,
                                                     OutSpec os) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t o = warp; o < O; o += nwarps) {
    int64_t rem = o, base = 0;
    for (int d = 0; d < a.nk; ++d) {
      base += (rem % a.kshape[d]) * a.kst[d];
      rem /= a.kshape[d];
    }
    Acc acc;
    acc.init();
    if constexpr (Acc::kShift) acc.set_shift(in[base]);
    for (int64_t j = lane; j < R; j += 32) {
      int64_t r = j, off = base;
      for (int d = 0; d < a.nr; ++d) {
        off += (r % a.rshape[d]) * a.rst[d];
        r /= a.rshape[d];
      }
      acc.add(in[off], j);
    }
    warp_reduce(acc);
    if (lane == 0) acc.store(os, o);
  }
}

// ---------------------------------------------------------------------------
// host planning
// ---------------------------------------------------------------------------
struct Plan {
  enum Kind { kFullFlat, kFullStrided, kInner, kOuter, kGeneric } kind;
  int64_t n = 0;             // full: elements
  const void *flat_base = nullptr;
  Space1 sp{};
  int64_t I = 1, R = 1, O = 1, si = 0, sr = 0, so = 0;
  AxisSpace ax{};
};

// Builds the reduction plan for `in` with reduced-axis mask `mask`.
static acd_status plan_reduce(const acd_desc *in, uint32_t mask, bool order_matters, Plan &p) {
  const size_t es = dtype_size(in->dtype);
  const char *base = desc_ptr(in);
  int nd = 0;
  int64_t shp[ACD_MAX_DIMS], st[ACD_MAX_DIMS];
  bool red[ACD_MAX_DIMS];
  for (int d = 0; d < in->ndim; ++d) {
    if (in->shape[d] == 1) continue;
    shp[nd] = in->shape[d];
    st[nd] = in->stride[d];
    red[nd] = (mask >> d) & 1u;
    ++nd;
  }
  bool all = true;
  for (int d = 0; d < nd; ++d) all = all && red[d];
  if (all) {
    p.n = 1;
    for (int d = 0; d < nd; ++d) p.n *= shp[d];
    // dense (contiguous, or a permutation of a dense block when the order of
    // visiting does not matter): one flat range
    bool contiguous = true;
    int64_t expect = 1;
    for (int d = 0; d < nd; ++d) {
      if (st[d] != expect) contiguous = false;
      expect *= shp[d];
    }
    if (contiguous || (!order_matters && is_dense_permutation(nd, shp, st))) {
      p.kind = Plan::kFullFlat;
      p.flat_base = base;
      return ACD_OK;
    }
    p.kind = Plan::kFullStrided;
    // collapse for the strided walk
    IterSpace it;
    it.ndim = nd;
    it.nops = 1;
    for (int d = 0; d < nd; ++d) {
      it.shape[d] = shp[d];
      it.stride[0][d] = st[d];
    }
    collapse(it);
    p.sp.ndim = it.ndim;
    for (int d = 0; d < ACD_MAX_DIMS; ++d) {
      p.sp.shape[d] = d < it.ndim ? it.shape[d] : 1;
      p.sp.st[d] = d < it.ndim ? it.stride[0][d] : 0;
    }
    p.flat_base = base;
    return ACD_OK;
  }
  (void)es;
  // merge neighbours with the same flag that are jointly contiguous
  int m = 0;
  for (int d = 0; d < nd; ++d) {
    if (m > 0 && red[m - 1] == red[d] && st[d] == st[m - 1] * shp[m - 1]) {
      shp[m - 1] *= shp[d];
    } else {
      shp[m] = shp[d];
      st[m] = st[d];
      red[m] = red[d];
      ++m;
    }
  }
  nd = m;
  // (kept)? (reduced) (kept)?
  int nruns = 0;
  for (int d = 0; d < nd; ++d)
    if (red[d] && (d == 0 || !red[d - 1])) ++nruns;
  int nkept = 0;
  for (int d = 0; d < nd; ++d) nkept += !red[d];
  if (nruns == 1 && nd <= 3 && nkept <= 2) {
    int r = 0;
    while (!red[r]) ++r;
    const bool kb = r > 0, ka = r + 1 < nd;
    if (nd == 1 + (int)kb + (int)ka) {
      p.I = kb ? shp[0] : 1;
      p.si = kb ? st[0] : 0;
      p.R = shp[r];
      p.sr = st[r];
      p.O = ka ? shp[r + 1] : 1;
      p.so = ka ? st[r + 1] : 0;
      p.flat_base = base;
      p.kind = (p.I == 1) ? Plan::kInner : Plan::kOuter;
      return ACD_OK;
    }
  }
  p.kind = Plan::kGeneric;
  p.ax.nk = p.ax.nr = 0;
  p.O = p.R = 1;
  for (int d = 0; d < nd; ++d) {
    if (red[d]) {
      p.ax.rshape[p.ax.nr] = shp[d];
      p.ax.rst[p.ax.nr] = st[d];
      p.ax.nr++;
      p.R *= shp[d];
    } else {
      p.ax.kshape[p.ax.nk] = shp[d];
      p.ax.kst[p.ax.nk] = st[d];
      p.ax.nk++;
      p.O *= shp[d];
    }
  }
  p.flat_base = base;
  return ACD_OK;
}

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

template <class Acc, typename T>
static acd_status run_plan(acd_ctx *ctx, const Plan &p, OutSpec os, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  const T *in = static_cast<const T *>(p.flat_base);
  switch (p.kind) {
    case Plan::kFullFlat:
    case Plan::kFullStrided: {
      os.n = p.n;
      if (p.n == 0) return fail(ACD_ERR_UNSUPPORTED, "reduction of an empty tensor");
      int grid;
      if (p.kind == Plan::kFullFlat)
        grid = persistent_grid(ctx, k_red_flat<Acc, T, V, 4>, kRedThreads, 0,
                               ((p.n + V - 1) / V + kRedThreads * 4 - 1) / (kRedThreads * 4));
      else
        grid = persistent_grid(ctx, k_red_strided<Acc, T>, kRedThreads, 0,
                               ((p.n + 3) / 4 + kRedThreads - 1) / kRedThreads);
      void *scratch;
      ACD_TRY(get_scratch(ctx, align_up(sizeof(Acc) * grid, 256), stream, &scratch));
      Acc *partials = static_cast<Acc *>(scratch);
      unsigned int *counter = &ctx->control->counters[0];
      if (p.kind == Plan::kFullFlat) {
        const int64_t c = (reinterpret_cast<uintptr_t>(in) / sizeof(T)) % V;
        const bool al = aligned_to<T>(in, sizeof(T));
        int64_t head = al ? (V - c) % V : p.n;
        if (head > p.n) head = p.n;
        k_red_flat<Acc, T, V, 4><<<grid, kRedThreads, 0, stream>>>(in, p.n, head, partials, counter, os);
      } else {
        k_red_strided<Acc, T><<<grid, kRedThreads, 0, stream>>>(in, p.sp, p.n, partials, counter, os);
      }
      return ACD_OK;
    }
    case Plan::kInner: {
      os.n = p.R;
      const bool vec = p.sr == 1 && (p.so % V == 0) && aligned_to<T>(in, sizeof(T) * V);
      const int64_t warps_wanted = p.O;
      const int64_t target_threads = (int64_t)ctx->sm_count * 2048;
      if (p.O * 32 >= target_threads / 2 || p.R <= 4096) {
        const int64_t work = (warps_wanted * 32 + 255) / 256;
        if (vec) {
          const int grid = persistent_grid(ctx, k_red_inner_warp<Acc, T, V, true>, 256, 0, work);
          k_red_inner_warp<Acc, T, V, true><<<grid, 256, 0, stream>>>(in, p.R, p.sr, p.so, p.O, os);
        } else {
          const int grid = persistent_grid(ctx, k_red_inner_warp<Acc, T, V, false>, 256, 0, work);
          k_red_inner_warp<Acc, T, V, false><<<grid, 256, 0, stream>>>(in, p.R, p.sr, p.so, p.O, os);
        }
        return ACD_OK;
      }
      // few long fibers: split each over S CTAs
      int64_t S = (target_threads / kRedThreads + p.O - 1) / p.O;
      int64_t chunk = (p.R + S - 1) / S;
      chunk = (chunk + 4 * V - 1) / (4 * V) * (4 * V);
      S = (p.R + chunk - 1) / chunk;
      void *scratch;
      unsigned int *counters;
      ACD_TRY(get_counters(ctx, (size_t)p.O, stream, &counters));
      ACD_TRY(get_scratch(ctx, sizeof(Acc) * p.O * S, stream, &scratch));
      Acc *partials = static_cast<Acc *>(scratch);
      const int64_t grid = p.O * S;
      if (grid > INT32_MAX) return fail(ACD_ERR_UNSUPPORTED, "reduction grid too large");
      if (vec)
        k_red_inner_cta<Acc, T, V, true><<<(int)grid, kRedThreads, 0, stream>>>(in, p.R, p.sr, p.so, S, chunk,
                                                                               partials, counters, os);
      else
        k_red_inner_cta<Acc, T, V, false><<<(int)grid, kRedThreads, 0, stream>>>(in, p.R, p.sr, p.so, S, chunk,
                                                                                partials, counters, os);
      return ACD_OK;
    }
    case Plan::kOuter: {
      os.n = p.R;
      const bool vec = p.si == 1 && (p.sr % V == 0) && (p.so % V == 0) && aligned_to<T>(in, sizeof(T) * V);
      const bool tall = p.R >= 64;
      const int WI = tall ? 1 : 8;
      const int64_t TI = (int64_t)32 * V * WI;
      const int64_t itiles = (p.I + TI - 1) / TI;
      const int64_t ctas = itiles * p.O;
      const int64_t target_ctas = (int64_t)ctx->sm_count * 8;
      int64_t S = 1;
      if (tall && ctas < target_ctas) S = (target_ctas + ctas - 1) / ctas;
      const int WR = tall ? 8 : 1;
      int64_t chunk = (p.R + S - 1) / S;
      chunk = (chunk + WR - 1) / WR * WR;
      if (chunk < 8 * WR) chunk = 8 * WR;
      S = (p.R + chunk - 1) / chunk;
      const int64_t grid = ctas * S;
      if (grid > INT32_MAX) return fail(ACD_ERR_UNSUPPORTED, "reduction grid too large");
      Acc *partials = nullptr;
      unsigned int *counters = nullptr;
      if (S > 1) {
        void *scratch;
        ACD_TRY(get_counters(ctx, (size_t)ctas, stream, &counters));
        ACD_TRY(get_scratch(ctx, sizeof(Acc) * p.I * p.O * S, stream, &scratch));
        partials = static_cast<Acc *>(scratch);
      }
#define ACD_OUTER(WRV, VECV)                                                                            \
  k_red_outer<Acc, T, V, WRV, VECV><<<(int)grid, 256, 0, stream>>>(in, p.I, p.R, p.si, p.sr, p.so, p.O, S, \
                                                                   chunk, itiles, partials, counters, os)
      if (tall) {
        if (vec) ACD_OUTER(8, true); else ACD_OUTER(8, false);
      } else {
        if (vec) ACD_OUTER(1, true); else ACD_OUTER(1, false);
      }
#undef ACD_OUTER
      return ACD_OK;
    }
    case Plan::kGeneric: {
      os.n = p.R;
      const int grid = persistent_grid(ctx, k_red_generic<Acc, T>, 256, 0, (p.O * 32 + 255) / 256);
      k_red_generic<Acc, T><<<grid, 256, 0, stream>>>(in, p.ax, p.O, p.R, os);
      return ACD_OK;
    }
  }
  return fail(ACD_ERR_INVALID, "bad reduction plan");
}

template <typename T>
static acd_status reduce_t(acd_ctx *ctx, int op, const Plan &p, const OutSpec &os, cudaStream_t s) {
  constexpr bool fl = std::is_floating_point<T>::value;
  switch (op) {
    case ACD_RED_SUM:
    case ACD_RED_MEAN: return run_plan<SumAcc<T>, T>(ctx, p, os, s);
    case ACD_RED_MAX: return run_plan<ExtAcc<T, true>, T>(ctx, p, os, s);
    case ACD_RED_MIN: return run_plan<ExtAcc<T, false>, T>(ctx, p, os, s);
    case ACD_RED_COUNT: return run_plan<CountAcc<T>, T>(ctx, p, os, s);
    case ACD_RED_ANY: return run_plan<TruthAcc<T, false>, T>(ctx, p, os, s);
    case ACD_RED_ALL: return run_plan<TruthAcc<T, true>, T>(ctx, p, os, s);
    case ACD_RED_PROD:
      if constexpr (fl) return run_plan<ProdAcc<T>, T>(ctx, p, os, s);
      break;
    case ACD_RED_VAR:
      if constexpr (fl) return run_plan<VarAcc<T>, T>(ctx, p, os, s);
      break;
    default: break;
  }
  return fail(ACD_ERR_UNSUPPORTED, "reduction op %d not supported for this dtype", op);
}

// float16 tensors: sum, mean and count (accumulated in float64 / int64)
static acd_status reduce_half(acd_ctx *ctx, int op, const Plan &p, const OutSpec &os, cudaStream_t s) {
  switch (op) {
    case ACD_RED_SUM:
    case ACD_RED_MEAN: return run_plan<SumAcc<__half>, __half>(ctx, p, os, s);
    case ACD_RED_COUNT: return run_plan<CountAcc<__half>, __half>(ctx, p, os, s);
    default: break;
  }
  return fail(ACD_ERR_UNSUPPORTED, "reduction op %d not supported for float16 (sum, mean and count are)", op);
}

template <typename T>
static acd_status arg_t(acd_ctx *ctx, int op, const Plan &p, const OutSpec &os, cudaStream_t s) {
  if (op == ACD_ARGMAX) return run_plan<ArgAcc<T, true>, T>(ctx, p, os, s);
  return run_plan<ArgAcc<T, false>, T>(ctx, p, os, s);
}

static acd_status check_out_count(const acd_desc *out, int64_t want, const char *what) {
  if (desc_numel(out) != want)
    return fail(ACD_ERR_SHAPE, "%s: output has %lld elements, expected %lld", what, (long long)desc_numel(out),
                (long long)want);
  if (!desc_is_contiguous(out)) return fail(ACD_ERR_UNSUPPORTED, "%s: output must be contiguous", what);
  if (out->dtype != ACD_FLOAT32 && out->dtype != ACD_FLOAT64 && out->dtype != ACD_INT32 && out->dtype != ACD_INT64)
    return fail(ACD_ERR_DTYPE, "%s: output dtype must be float, double, int32 or int64", what);
  return ACD_OK;
}

static int64_t kept_count(const acd_desc *in, uint32_t mask) {
  int64_t n = 1;
  for (int d = 0; d < in->ndim; ++d)
    if (!((mask >> d) & 1u)) n *= in->shape[d];
  return n;
}

__global__ void __launch_bounds__(256) k_keys_decode(void *out, int32_t dt, const long long *__restrict__ keys,
                                                     int64_t n, int32_t one_based) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const long long k = keys[i];
    long long idx = -1;
    if (k != LLONG_MIN) {
      const uint64_t u = (uint64_t)k ^ 0x8000000000000000ull;
      idx = (long long)(0xFFFFFFFFull - (u & 0xFFFFFFFFull)) + one_based;
    }
    store_i(out, dt, i, idx);
  }
}

// The exchange buffer of the sharded strided-views step: int64
// buf[nkeys + 6 * world], the argmax keys followed by one statistics row
// (n, K, s1_hi, s2_hi, s1_lo, s2_lo as float64 bit patterns) per rank.  Each
// rank writes its keys and its own row and leaves the other ranks' rows at
// INT64_MIN, the bit pattern of -0.0 and the smallest int64, so one int64 MAX
// all-reduce both picks every key's winner and hands each rank's row to all
// ranks unchanged.  k_shard_finish then decodes the keys, merges the rows in
// rank order (Chan's shifted-moment merge, the same float64 arithmetic as
// the host merge in acediar/sharded.py) and puts INT64_MIN back into every
// row for the next exchange.
__global__ void __launch_bounds__(256) k_shard_finish(void *out, int32_t dt, long long *__restrict__ buf, int64_t nkeys,
                                                      int32_t world, double *__restrict__ sum_var, int32_t one_based) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nkeys; i += (int64_t)gridDim.x * blockDim.x) {
    const long long k = buf[i];
    long long idx = -1;
    if (k != LLONG_MIN) {
      const uint64_t u = (uint64_t)k ^ 0x8000000000000000ull;
      idx = (long long)(0xFFFFFFFFull - (u & 0xFFFFFFFFull)) + one_based;
    }
    store_i(out, dt, i, idx);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    long long *rows = buf + nkeys;
    const double k0 = __longlong_as_double(rows[1]);
    double s1 = 0.0, s2 = 0.0, nt = 0.0;
    for (int r = 0; r < world; ++r) {
      const long long *row = rows + 6 * r;
      const double n = __longlong_as_double(row[0]), k = __longlong_as_double(row[1]);
      const double a = __longlong_as_double(row[2]) + __longlong_as_double(row[4]);
      const double b = __longlong_as_double(row[3]) + __longlong_as_double(row[5]);
      const double d = k - k0;
      s1 += a + n * d;
      s2 += b + 2.0 * d * a + n * d * d;
      nt += n;
    }
    sum_var[0] = nt * k0 + s1;
    sum_var[1] = nt > 1.0 ? (s2 - s1 * (s1 / nt)) / (nt - 1.0) : (double)NAN;
    for (int64_t j = 0; j < 6 * (int64_t)world; ++j) rows[j] = LLONG_MIN;
  }
}

// ---- the elementwise chain + reduction configuration in one pass -----------
// For float64 a, b: c = a + b, d = a * b, e = exp(a), f = sigmoid(b),
// g = sqrt(a), each rounded as its own operator (bit-identical to the
// separate launches), and from the same registers the shifted moments of
// each output (shift = its first element) and the first maximum of c.  One
// launch replaces five elementwise kernels and sixteen reductions that would
// re-read their inputs.  A thread adds only about n / (grid * 256) elements
// (14 at n = 2^20) before the pairwise block and grid merges, so float64
// moments keep the error near log2(n) ulp; double-double (VarAcc<double>)
// would double the FP64 instructions of a kernel that is bound by them.
struct Moments {
  double k, s1, s2;
  __device__ __forceinline__ void init() { k = 0.0; s1 = 0.0; s2 = 0.0; }
  __device__ __forceinline__ void set_shift(double x) { k = x; }
  __device__ __forceinline__ void add(double x, int64_t) {
    const double d = x - k;
    s1 += d;
    s2 += d * d;
  }
  __device__ __forceinline__ void merge(const Moments &o) {
    s1 += o.s1;
    s2 += o.s2;
  }
  __device__ __forceinline__ double total(double n) const { return n * k + s1; }
  __device__ __forceinline__ double var(double n) const {
    if (n < 2.0) return (double)NAN;
    const double v = (s2 - s1 * (s1 / n)) / (n - 1.0);
    return v < 0.0 ? 0.0 : v;
  }
};

struct Chain5Acc {
  Moments v[5];
  ArgAcc<double, true> am;
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int k = 0; k < 5; ++k) v[k].init();
    am.init();
  }
  __device__ __forceinline__ void merge(const Chain5Acc &o) {
#pragma unroll
    for (int k = 0; k < 5; ++k) v[k].merge(o.v[k]);
    am.merge(o.am);
  }
};

constexpr int kChain5Threads = 256;

__device__ __forceinline__ void chain5_shifts(const double *a, const double *b, double K[5]) {
  const double a0 = a[0], b0 = b[0];
  K[0] = binary_apply<ACD_ADD, double, double>(a0, b0);
  K[1] = binary_apply<ACD_MUL, double, double>(a0, b0);
  K[2] = unary_apply<ACD_EXP, double>(a0);
  K[3] = unary_apply<ACD_SIGMOID, double>(b0);
  K[4] = unary_apply<ACD_SQRT, double>(a0);
}

__global__ void __launch_bounds__(kChain5Threads) k_chain5(const double *__restrict__ a, const double *__restrict__ b,
                                                           double *__restrict__ c, double *__restrict__ d,
                                                           double *__restrict__ e, double *__restrict__ f,
                                                           double *__restrict__ g, int64_t n,
                                                           Chain5Acc *__restrict__ partials, unsigned int *counter,
                                                           double *__restrict__ stats, int64_t *__restrict__ which) {
  __shared__ Chain5Acc smem[kChain5Threads / 32];
  __shared__ int am_last;
  double K[5];
  chain5_shifts(a, b, K);
  Chain5Acc acc;
  acc.init();
#pragma unroll
  for (int k = 0; k < 5; ++k) acc.v[k].set_shift(K[k]);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  constexpr int U = 4;  // elements in flight per thread
  int64_t i = tid;
  for (; i + (U - 1) * nth < n; i += U * nth) {
    double xa[U], xb[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      xa[u] = a[i + u * nth];
      xb[u] = b[i + u * nth];
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = i + u * nth;
      const double vc = binary_apply<ACD_ADD, double, double>(xa[u], xb[u]);
      const double vd = binary_apply<ACD_MUL, double, double>(xa[u], xb[u]);
      const double ve = unary_apply<ACD_EXP, double>(xa[u]);
      const double vf = unary_apply<ACD_SIGMOID, double>(xb[u]);
      const double vg = unary_apply<ACD_SQRT, double>(xa[u]);
      c[j] = vc;
      d[j] = vd;
      e[j] = ve;
      f[j] = vf;
      g[j] = vg;
      acc.v[0].add(vc, j);
      acc.v[1].add(vd, j);
      acc.v[2].add(ve, j);
      acc.v[3].add(vf, j);
      acc.v[4].add(vg, j);
      acc.am.add(vc, j);
    }
  }
  for (; i < n; i += nth) {
    const double va = a[i], vb = b[i];
    const double vc = binary_apply<ACD_ADD, double, double>(va, vb);
    const double vd = binary_apply<ACD_MUL, double, double>(va, vb);
    const double ve = unary_apply<ACD_EXP, double>(va);
    const double vf = unary_apply<ACD_SIGMOID, double>(vb);
    const double vg = unary_apply<ACD_SQRT, double>(va);
    c[i] = vc;
    d[i] = vd;
    e[i] = ve;
    f[i] = vf;
    g[i] = vg;
    acc.v[0].add(vc, i);
    acc.v[1].add(vd, i);
    acc.v[2].add(ve, i);
    acc.v[3].add(vf, i);
    acc.v[4].add(vg, i);
    acc.am.add(vc, i);
  }
  // grid merge: per-CTA partials, the last CTA merges them in index order
  block_reduce(acc, smem);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = acc;
    __threadfence();
    am_last = (atomicAdd(counter, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!am_last) return;
  __threadfence();
  Chain5Acc fin;
  fin.init();
#pragma unroll
  for (int k = 0; k < 5; ++k) fin.v[k].set_shift(K[k]);
  for (int q = threadIdx.x; q < (int)gridDim.x; q += blockDim.x) fin.merge(load_cg(partials + q));
  block_reduce(fin, smem);
  if (threadIdx.x == 0) {
    const double nn = (double)n;
#pragma unroll
    for (int k = 0; k < 5; ++k) {
      const double tot = fin.v[k].total(nn);
      stats[3 * k] = tot;
      stats[3 * k + 1] = tot / nn;
      stats[3 * k + 2] = fin.v[k].var(nn);
    }
    which[0] = fin.am.i == LLONG_MAX ? -1 : fin.am.i + 1;
    *counter = 0u;
  }
}

__global__ void k_shard_rows_init(long long *rows, int64_t n) {
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x)
    rows[j] = LLONG_MIN;
}

template <typename T>
acd_status softmax_stats(acd_ctx *ctx, const acd_desc *in, cudaStream_t s) {
  Plan p;
  ACD_TRY(plan_reduce(in, 0xFFu, false, p));
  OutSpec os;
  os.out = ctx->control->stats;
  os.mode = kModeValue;
  return run_plan<SoftStatAcc<T>, T>(ctx, p, os, s);
}
template acd_status softmax_stats<float>(acd_ctx *, const acd_desc *, cudaStream_t);
template acd_status softmax_stats<double>(acd_ctx *, const acd_desc *, cudaStream_t);

}  // namespace acd

using namespace acd;

extern "C" {

acd_status acd_reduce(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in, uint32_t axes_mask,
                      acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_reduce: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  if (op < ACD_RED_SUM || op > ACD_RED_ALL) return fail(ACD_ERR_INVALID, "acd_reduce: bad op %d", op);
  if (in->ndim < 32 && (axes_mask >> in->ndim) != 0u) return fail(ACD_ERR_AXIS, "acd_reduce: axis outside the tensor");
  if (in->ndim == 0) axes_mask = 0;
  ACD_TRY(check_out_count(out, kept_count(in, axes_mask), "acd_reduce"));
  if (desc_numel(in) == 0) return fail(ACD_ERR_UNSUPPORTED, "acd_reduce: empty input");
  Plan p;
  ACD_TRY(plan_reduce(in, axes_mask, false, p));
  OutSpec os;
  os.out = desc_ptr(out);
  os.dt = out->dtype;
  os.op = op;
  os.mode = kModeValue;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (in->dtype) {
    case ACD_FLOAT32: st = reduce_t<float>(ctx, op, p, os, s); break;
    case ACD_FLOAT64: st = reduce_t<double>(ctx, op, p, os, s); break;
    case ACD_INT32: st = reduce_t<int32_t>(ctx, op, p, os, s); break;
    case ACD_INT64: st = reduce_t<int64_t>(ctx, op, p, os, s); break;
    case ACD_BOOL: st = reduce_t<uint8_t>(ctx, op, p, os, s); break;
    case ACD_INT8: st = reduce_t<int8_t>(ctx, op, p, os, s); break;
    case ACD_FLOAT16: st = reduce_half(ctx, op, p, os, s); break;
    default: return fail(ACD_ERR_DTYPE, "acd_reduce: bad dtype");
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_sum_var(acd_ctx *ctx, const acd_desc *out_sum, const acd_desc *out_var, const acd_desc *in,
                       acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_sum_var: null context");
  ACD_TRY(check_desc(in, "in"));
  if (!out_sum && !out_var) return fail(ACD_ERR_INVALID, "acd_sum_var: no output");
  if (out_sum) {
    ACD_TRY(check_desc(out_sum, "out_sum"));
    ACD_TRY(check_out_count(out_sum, 1, "acd_sum_var"));
  }
  if (out_var) {
    ACD_TRY(check_desc(out_var, "out_var"));
    ACD_TRY(check_out_count(out_var, 1, "acd_sum_var"));
  }
  if (!is_float(in->dtype)) return fail(ACD_ERR_DTYPE, "acd_sum_var: float32/float64 input required");
  if (desc_numel(in) == 0) return fail(ACD_ERR_UNSUPPORTED, "acd_sum_var: empty input");
  Plan p;
  ACD_TRY(plan_reduce(in, 0xFFu, false, p));
  OutSpec os;
  os.mode = kModeSumVar;
  os.out = out_sum ? desc_ptr(out_sum) : nullptr;
  os.dt = out_sum ? out_sum->dtype : ACD_FLOAT64;
  os.out2 = out_var ? desc_ptr(out_var) : nullptr;
  os.dt2 = out_var ? out_var->dtype : ACD_FLOAT64;
  os.op = ACD_RED_VAR;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st = in->dtype == ACD_FLOAT32 ? run_plan<VarAcc<float>, float>(ctx, p, os, s)
                                           : run_plan<VarAcc<double>, double>(ctx, p, os, s);
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_stats_partial(acd_ctx *ctx, double *stats, const acd_desc *in, acd_stream stream) {
  if (!ctx || !stats) return fail(ACD_ERR_INVALID, "acd_stats_partial: null argument");
  ACD_TRY(check_desc(in, "in"));
  if (!is_float(in->dtype)) return fail(ACD_ERR_DTYPE, "acd_stats_partial: float32/float64 input required");
  if (desc_numel(in) == 0) return fail(ACD_ERR_UNSUPPORTED, "acd_stats_partial: empty input");
  Plan p;
  ACD_TRY(plan_reduce(in, 0xFFu, false, p));
  OutSpec os;
  os.mode = kModeStats;
  os.out = stats;
  os.op = ACD_RED_VAR;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st = in->dtype == ACD_FLOAT32 ? run_plan<VarAcc<float>, float>(ctx, p, os, s)
                                           : run_plan<VarAcc<double>, double>(ctx, p, os, s);
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_arg_reduce(acd_ctx *ctx, int32_t op, const acd_desc *out_index, const acd_desc *out_value,
                          const acd_desc *in, int32_t axis, int32_t one_based, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_arg_reduce: null context");
  ACD_TRY(check_desc(out_index, "out_index"));
  ACD_TRY(check_desc(in, "in"));
  if (op != ACD_ARGMAX && op != ACD_ARGMIN) return fail(ACD_ERR_INVALID, "acd_arg_reduce: bad op %d", op);
  if (out_index->dtype != ACD_INT32 && out_index->dtype != ACD_INT64 && out_index->dtype != ACD_FLOAT64)
    return fail(ACD_ERR_DTYPE, "acd_arg_reduce: index output must be int32, int64 or float64");
  if (axis >= in->ndim && !(axis == 0 && in->ndim == 0)) return fail(ACD_ERR_AXIS, "acd_arg_reduce: axis %d out of range", axis);
  const uint32_t mask = axis < 0 ? 0xFFu : (1u << axis);
  const int64_t kept = axis < 0 ? 1 : kept_count(in, mask);
  ACD_TRY(check_out_count(out_index, kept, "acd_arg_reduce"));
  if (out_value) {
    ACD_TRY(check_desc(out_value, "out_value"));
    ACD_TRY(check_out_count(out_value, kept, "acd_arg_reduce"));
  }
  if (desc_numel(in) == 0) return fail(ACD_ERR_UNSUPPORTED, "acd_arg_reduce: empty input");
  Plan p;
  ACD_TRY(plan_reduce(in, mask, true, p));
  OutSpec os;
  os.mode = kModeIndex;
  os.out = desc_ptr(out_index);
  os.dt = out_index->dtype;
  os.out2 = out_value ? desc_ptr(out_value) : nullptr;
  os.dt2 = out_value ? out_value->dtype : ACD_FLOAT64;
  os.one_based = one_based ? 1 : 0;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (in->dtype) {
    case ACD_FLOAT32: st = arg_t<float>(ctx, op, p, os, s); break;
    case ACD_FLOAT64: st = arg_t<double>(ctx, op, p, os, s); break;
    case ACD_INT32: st = arg_t<int32_t>(ctx, op, p, os, s); break;
    case ACD_INT64: st = arg_t<int64_t>(ctx, op, p, os, s); break;
    default: return fail(ACD_ERR_DTYPE, "acd_arg_reduce: dtype not supported");
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_argmax_keys(acd_ctx *ctx, int64_t *keys, const acd_desc *in, int32_t axis, int64_t index_base,
                           acd_stream stream) {
  if (!ctx || !keys) return fail(ACD_ERR_INVALID, "acd_argmax_keys: null argument");
  ACD_TRY(check_desc(in, "in"));
  if (in->dtype != ACD_FLOAT32) return fail(ACD_ERR_DTYPE, "acd_argmax_keys: float32 input required");
  if (axis < 0 || axis >= in->ndim) return fail(ACD_ERR_AXIS, "acd_argmax_keys: axis %d out of range", axis);
  if (desc_numel(in) == 0) return fail(ACD_ERR_UNSUPPORTED, "acd_argmax_keys: empty input");
  if (index_base < 0 || index_base + in->shape[axis] > 0xFFFFFFFFLL)
    return fail(ACD_ERR_INVALID, "acd_argmax_keys: global index must fit in 32 bits");
  Plan p;
  ACD_TRY(plan_reduce(in, 1u << axis, true, p));
  OutSpec os;
  os.mode = kModeKey;
  os.out = keys;
  os.index_base = index_base;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st = run_plan<ArgAcc<float, true>, float>(ctx, p, os, s);
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_argmax_keys_decode(acd_ctx *ctx, const acd_desc *out_index, const int64_t *keys, int32_t one_based,
                                  acd_stream stream) {
  if (!ctx || !keys) return fail(ACD_ERR_INVALID, "acd_argmax_keys_decode: null argument");
  ACD_TRY(check_desc(out_index, "out_index"));
  if (!desc_is_contiguous(out_index)) return fail(ACD_ERR_UNSUPPORTED, "acd_argmax_keys_decode: contiguous output required");
  if (out_index->dtype != ACD_INT32 && out_index->dtype != ACD_INT64)
    return fail(ACD_ERR_DTYPE, "acd_argmax_keys_decode: int32 or int64 output required");
  const int64_t n = desc_numel(out_index);
  if (n == 0) return ACD_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(ctx, n, 256, 4);
  k_keys_decode<<<grid, 256, 0, s>>>(desc_ptr(out_index), out_index->dtype, reinterpret_cast<const long long *>(keys),
                                     n, one_based ? 1 : 0);
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_chain5_stats(acd_ctx *ctx, const acd_desc *a, const acd_desc *b, const acd_desc *const *outs,
                            double *stats, int64_t *which_max, acd_stream stream) {
  if (!ctx || !a || !b || !outs || !stats || !which_max) return fail(ACD_ERR_INVALID, "acd_chain5_stats: null argument");
  ACD_TRY(check_desc(a, "a"));
  ACD_TRY(check_desc(b, "b"));
  const int64_t n = desc_numel(a);
  if (a->dtype != ACD_FLOAT64 || b->dtype != ACD_FLOAT64)
    return fail(ACD_ERR_DTYPE, "acd_chain5_stats: float64 inputs required");
  if (desc_numel(b) != n || !desc_is_contiguous(a) || !desc_is_contiguous(b))
    return fail(ACD_ERR_SHAPE, "acd_chain5_stats: a and b must be contiguous with one element count");
  if (n < 1) return fail(ACD_ERR_UNSUPPORTED, "acd_chain5_stats: empty input");
  double *o[5];
  for (int k = 0; k < 5; ++k) {
    if (!outs[k]) return fail(ACD_ERR_INVALID, "acd_chain5_stats: null output %d", k);
    ACD_TRY(check_desc(outs[k], "out"));
    if (outs[k]->dtype != ACD_FLOAT64 || desc_numel(outs[k]) != n || !desc_is_contiguous(outs[k]))
      return fail(ACD_ERR_SHAPE, "acd_chain5_stats: output %d must be contiguous float64 of the input size", k);
    o[k] = reinterpret_cast<double *>(desc_ptr(outs[k]));
  }
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = persistent_grid(ctx, k_chain5, kChain5Threads, 0, (n + 4 * kChain5Threads - 1) / (4 * kChain5Threads));
  void *scratch;
  ACD_TRY(get_scratch(ctx, align_up(sizeof(Chain5Acc) * grid, 256), s, &scratch));
  k_chain5<<<grid, kChain5Threads, 0, s>>>(reinterpret_cast<const double *>(desc_ptr(a)),
                                           reinterpret_cast<const double *>(desc_ptr(b)), o[0], o[1], o[2], o[3], o[4], n,
                                           static_cast<Chain5Acc *>(scratch), &ctx->control->counters[1], stats,
                                           which_max);
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_shard_exchange_init(acd_ctx *ctx, int64_t *buf, int64_t nkeys, int32_t world, acd_stream stream) {
  if (!ctx || !buf || nkeys < 0 || world < 1) return fail(ACD_ERR_INVALID, "acd_shard_exchange_init: bad argument");
  DeviceGuard g(ctx->device);
  k_shard_rows_init<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<long long *>(buf + nkeys),
                                                                    6 * (int64_t)world);
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_shard_finish(acd_ctx *ctx, int64_t *buf, int64_t nkeys, int32_t world, const acd_desc *out_index,
                            double *sum_var, int32_t one_based, acd_stream stream) {
  if (!ctx || !buf || !sum_var || nkeys < 0 || world < 1) return fail(ACD_ERR_INVALID, "acd_shard_finish: bad argument");
  ACD_TRY(check_desc(out_index, "out_index"));
  if (!desc_is_contiguous(out_index) || desc_numel(out_index) != nkeys)
    return fail(ACD_ERR_SHAPE, "acd_shard_finish: out_index must be contiguous with nkeys elements");
  if (out_index->dtype != ACD_INT32 && out_index->dtype != ACD_INT64)
    return fail(ACD_ERR_DTYPE, "acd_shard_finish: int32 or int64 output required");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(ctx, nkeys > 0 ? nkeys : 1, 256, 4);
  k_shard_finish<<<grid, 256, 0, s>>>(desc_ptr(out_index), out_index->dtype, reinterpret_cast<long long *>(buf), nkeys,
                                      world, sum_var, one_based ? 1 : 0);
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_fused_stats_keys(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, double p0, double *stats,
                                int64_t *keys, int64_t index_base, acd_stream stream) {
  if (!ctx || !stats || !keys) return fail(ACD_ERR_INVALID, "acd_fused_stats_keys: null argument");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  if (in->dtype != ACD_FLOAT32 || out->dtype != ACD_FLOAT32)
    return fail(ACD_ERR_DTYPE, "acd_fused_stats_keys: float32 input and output required");
  if (in->ndim < 1) return fail(ACD_ERR_SHAPE, "acd_fused_stats_keys: at least one axis required");
  if (out->ndim != in->ndim) return fail(ACD_ERR_SHAPE, "acd_fused_stats_keys: output shape differs");
  for (int d = 0; d < in->ndim; ++d)
    if (out->shape[d] != in->shape[d]) return fail(ACD_ERR_SHAPE, "acd_fused_stats_keys: output shape differs");
  const int64_t n = desc_numel(in);
  if (n == 0) return fail(ACD_ERR_UNSUPPORTED, "acd_fused_stats_keys: empty input");
  const int64_t F = in->shape[0];
  if (index_base < 0 || index_base + F > 0xFFFFFFFFLL)
    return fail(ACD_ERR_INVALID, "acd_fused_stats_keys: global index must fit in 32 bits");
  const bool fast = desc_is_contiguous(in) && desc_is_contiguous(out) && F % 4 == 0 &&
                    aligned_to<float>(desc_ptr(in), 16) && aligned_to<float>(desc_ptr(out), 16);
  if (!fast) {  // the three separate passes
    ACD_TRY(acd_fused(ctx, ACD_FUSED_SCALE_ADD_EXP_NEG_SQUARE, out, in, nullptr, p0, stream));
    ACD_TRY(acd_stats_partial(ctx, stats, out, stream));
    return acd_argmax_keys(ctx, keys, out, 0, index_base, stream);
  }
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nfib = n / F;
  const int grid = persistent_grid(ctx, k_chain_stats_keys<8>, kChainThreads, 0, (nfib + 7) / 8);
  void *scratch;
  ACD_TRY(get_scratch(ctx, align_up(sizeof(VarAcc<float>) * grid, 256), s, &scratch));
  OutSpec os;
  os.mode = kModeStats;
  os.out = stats;
  os.op = ACD_RED_VAR;
  os.n = n;
  k_chain_stats_keys<8><<<grid, kChainThreads, 0, s>>>(
      reinterpret_cast<const float *>(desc_ptr(in)), reinterpret_cast<float *>(desc_ptr(out)), F, nfib, (float)p0,
      static_cast<VarAcc<float> *>(scratch), &ctx->control->counters[0], os, reinterpret_cast<long long *>(keys),
      index_base);
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_permute_fused_stats_keys(acd_ctx *ctx, const acd_desc *y, const acd_desc *z, const acd_desc *in,
                                        double p0, double *stats, int64_t *keys, int64_t index_base,
                                        acd_stream stream) {
  if (!ctx || !stats || !keys) return fail(ACD_ERR_INVALID, "acd_permute_fused_stats_keys: null argument");
  ACD_TRY(check_desc(y, "y"));
  ACD_TRY(check_desc(z, "z"));
  ACD_TRY(check_desc(in, "in"));
  if (in->dtype != ACD_FLOAT32 || y->dtype != ACD_FLOAT32 || z->dtype != ACD_FLOAT32)
    return fail(ACD_ERR_DTYPE, "acd_permute_fused_stats_keys: float32 views required");
  if (!desc_is_contiguous(y) || !desc_is_contiguous(z))
    return fail(ACD_ERR_UNSUPPORTED, "acd_permute_fused_stats_keys: y and z must be contiguous");
  if (y->ndim != in->ndim || z->ndim != in->ndim)
    return fail(ACD_ERR_SHAPE, "acd_permute_fused_stats_keys: y, z and in must have one shape");
  for (int d = 0; d < in->ndim; ++d)
    if (y->shape[d] != in->shape[d] || z->shape[d] != in->shape[d])
      return fail(ACD_ERR_SHAPE, "acd_permute_fused_stats_keys: y, z and in must have one shape");
  const int64_t n = desc_numel(in);
  if (n == 0) return fail(ACD_ERR_UNSUPPORTED, "acd_permute_fused_stats_keys: empty input");
  if (index_base < 0 || index_base + in->shape[0] > 0xFFFFFFFFLL)
    return fail(ACD_ERR_INVALID, "acd_permute_fused_stats_keys: global index must fit in 32 bits");
  // a transpose (y contiguous along axis 0, in contiguous along another
  // axis of the collapsed space) runs as one kernel that reads `in` once
  IterSpace it;
  it.ndim = y->ndim;
  it.nops = 2;
  for (int d = 0; d < y->ndim; ++d) {
    it.shape[d] = y->shape[d];
    it.stride[0][d] = y->stride[d];
    it.stride[1][d] = in->stride[d];
  }
  collapse(it);
  if ((it.ndim == 2 || it.ndim == 3) && it.stride[0][0] == 1 && it.shape[0] == y->shape[0]) {
    int ai = -1;
    for (int d = 1; d < it.ndim; ++d)
      if (it.stride[1][d] == 1) ai = d;
    if (ai > 0) {
      int64_t n2 = 1, os2 = 0, is2 = 0;
      if (it.ndim == 3) {
        const int bd = 3 - ai;
        n2 = it.shape[bd];
        os2 = it.stride[0][bd];
        is2 = it.stride[1][bd];
      }
      DeviceGuard g(ctx->device);
      bool launched = false;
      ACD_TRY(launch_permute_chain(ctx, reinterpret_cast<float *>(desc_ptr(y)), reinterpret_cast<float *>(desc_ptr(z)),
                                   reinterpret_cast<const float *>(desc_ptr(in)), it.shape[0], it.shape[ai], n2,
                                   it.stride[0][ai], os2, it.stride[1][0], is2, (float)p0, stats, n,
                                   reinterpret_cast<long long *>(keys), index_base,
                                   static_cast<cudaStream_t>(stream), &launched));
      if (launched) return ACD_OK;
    }
  }
  // otherwise the copy (TMA transpose for a permuted matrix), then the chain
  // with its statistics and keys in one pass over the copy
  ACD_TRY(acd_copy(ctx, y, in, stream));
  return acd_fused_stats_keys(ctx, z, y, p0, stats, keys, index_base, stream);
}

}  // extern "C"
