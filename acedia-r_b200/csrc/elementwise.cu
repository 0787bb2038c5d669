// Elementwise, broadcast and strided-copy kernels.
//
// Reference counterparts: elementwise_{binary,scalar,unary}_kernel
// (src/kernels/tensor_kernels.cu:25-48, one element per thread, scalar loads),
// broadcast_binary_kernel (src/kernels/tensor_kernels.cu:243-269, int32
// coordinates), strided_{unary,binary,scalar}_kernel
// (src/kernels/tensor_ops.cu:406-481) and strided_copy_kernel
// (src/kernels/tensor_kernels.cu:272-295, gathered reads, int32 index).
//
// Here every launch first collapses the operands' dimensions jointly and then
// picks one of four kernels:
//   k_flat      all operands dense in one order: 16-byte vector loads/stores,
//               grid-stride over a persistent grid (multiple of the SM count);
//   k_rows      2-D with every input dense or broadcast along axis 0 (the
//               acediaR row-bias X[i,j] + r[1,j] case): vector loads along
//               axis 0, the broadcast value loaded once per vector;
//   k_transpose out and in contiguous along different axes (permute →
//               contiguous): 64x64 shared-memory tiles, coalesced on both sides;
//   k_general   anything else: int64 coordinates, incremented along a run.
#include "common.cuh"
#include "ops.cuh"
#include "tma.cuh"

namespace acd {

template <class F>
__device__ __forceinline__ typename F::Out apply(const F &f, typename F::In a, typename F::In b) {
  if constexpr (F::kIn == 1)
    return f(a);
  else
    return f(a, b);
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
constexpr int kEwThreads = 256;
constexpr int kFlatU = 4;  // 16-byte vectors in flight per thread and operand

template <class F, int V, int U>
__global__ void __launch_bounds__(kEwThreads) k_flat(typename F::Out *__restrict__ out,
                                                     const typename F::In *__restrict__ a,
                                                     const typename F::In *__restrict__ b, int64_t n,
                                                     int64_t head, F f) {
  using T = typename F::In;
  using O = typename F::Out;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t nvec = (n - head) / V;
  const int64_t tail = head + nvec * V;
  const int64_t nscalar = head + (n - tail);
  for (int64_t i = tid; i < nscalar; i += nth) {
    const int64_t e = i < head ? i : tail + (i - head);
    out[e] = apply(f, a[e], F::kIn == 2 ? b[e] : T(0));
  }
  const Vec<T, V> *av = reinterpret_cast<const Vec<T, V> *>(a + head);
  const Vec<T, V> *bv = reinterpret_cast<const Vec<T, V> *>(F::kIn == 2 ? b + head : a + head);
  Vec<O, V> *ov = reinterpret_cast<Vec<O, V> *>(out + head);
  // full groups of U vectors: every load is in range, so none is guarded and
  // all U are in flight before the first use
  int64_t v0 = tid;
  for (; v0 + (int64_t)(U - 1) * nth < nvec; v0 += nth * U) {
    Vec<T, V> xa[U], xb[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      xa[u] = av[v0 + (int64_t)u * nth];
      if constexpr (F::kIn == 2) xb[u] = bv[v0 + (int64_t)u * nth];
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      Vec<O, V> r;
#pragma unroll
      for (int k = 0; k < V; ++k) r.v[k] = apply(f, xa[u].v[k], F::kIn == 2 ? xb[u].v[k] : T(0));
      ov[v0 + (int64_t)u * nth] = r;
    }
  }
  for (; v0 < nvec; v0 += nth) {
    const Vec<T, V> xa = av[v0];
    Vec<T, V> xb;
    if constexpr (F::kIn == 2) xb = bv[v0];
    Vec<O, V> r;
#pragma unroll
    for (int k = 0; k < V; ++k) r.v[k] = apply(f, xa.v[k], F::kIn == 2 ? xb.v[k] : T(0));
    ov[v0] = r;
  }
}

struct RowOperand {
  const void *p;
  int64_t s1;  // stride along axis 1
  int32_t s0;  // stride along axis 0: 0 (broadcast) or 1 (dense)
};

// Row-broadcast kernel: vector index w -> (column j, row block i); broadcast
// operands are loaded once per vector.
template <class F, int V, bool FAST>
__global__ void __launch_bounds__(kEwThreads) k_rows(typename F::Out *__restrict__ out, int64_t os1, RowOperand A,
                                                       RowOperand B, int64_t nv0, int64_t n1, FastDiv fd, F f) {
  using T = typename F::In;
  using O = typename F::Out;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t total = nv0 * n1;
  for (int64_t w = tid; w < total; w += nth) {
    int64_t j;
    if constexpr (FAST)
      j = fd.div((uint32_t)w);
    else
      j = w / nv0;
    const int64_t i = (w - j * nv0) * V;
    Vec<T, V> xa, xb;
    const T *pa = static_cast<const T *>(A.p) + j * A.s1;
    if (A.s0) {
      xa = *reinterpret_cast<const Vec<T, V> *>(pa + i);
    } else {
      const T s = *pa;
#pragma unroll
      for (int k = 0; k < V; ++k) xa.v[k] = s;
    }
    if constexpr (F::kIn == 2) {
      const T *pb = static_cast<const T *>(B.p) + j * B.s1;
      if (B.s0) {
        xb = *reinterpret_cast<const Vec<T, V> *>(pb + i);
      } else {
        const T s = *pb;
#pragma unroll
        for (int k = 0; k < V; ++k) xb.v[k] = s;
      }
    }
    Vec<O, V> r;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      if constexpr (F::kIn == 2)
        r.v[k] = f(xa.v[k], xb.v[k]);
      else
        r.v[k] = f(xa.v[k]);
    }
    *reinterpret_cast<Vec<O, V> *>(out + j * os1 + i) = r;
  }
}

struct GenSpace {
  int32_t ndim;
  int64_t shape[ACD_MAX_DIMS];
  int64_t st[kMaxOps][ACD_MAX_DIMS];
};

template <class F, int RUN>
__global__ void __launch_bounds__(kEwThreads) k_general(typename F::Out *__restrict__ out,
                                                        const typename F::In *__restrict__ a,
                                                        const typename F::In *__restrict__ b, GenSpace g,
                                                        int64_t n, F f) {
  using T = typename F::In;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = tid * RUN; base < n; base += nth * RUN) {
    int64_t c[ACD_MAX_DIMS];
    int64_t o0 = 0, o1 = 0, o2 = 0;
    int64_t rem = base;
#pragma unroll
    for (int d = 0; d < ACD_MAX_DIMS; ++d) {
      if (d < g.ndim) {
        c[d] = rem % g.shape[d];
        rem /= g.shape[d];
        o0 += c[d] * g.st[0][d];
        o1 += c[d] * g.st[1][d];
        o2 += c[d] * g.st[2][d];
      }
    }
#pragma unroll
    for (int r = 0; r < RUN; ++r) {
      if (base + r >= n) break;
      out[o0] = apply(f, a[o1], F::kIn == 2 ? b[o2] : T(0));
      // advance the coordinate by one along the column-major order
      o0 += g.st[0][0];
      o1 += g.st[1][0];
      o2 += g.st[2][0];
      if (++c[0] == g.shape[0]) {
        c[0] = 0;
        o0 -= g.shape[0] * g.st[0][0];
        o1 -= g.shape[0] * g.st[1][0];
        o2 -= g.shape[0] * g.st[2][0];
        for (int d = 1; d < g.ndim; ++d) {
          o0 += g.st[0][d];
          o1 += g.st[1][d];
          o2 += g.st[2][d];
          if (++c[d] < g.shape[d]) break;
          c[d] = 0;
          o0 -= g.shape[d] * g.st[0][d];
          o1 -= g.shape[d] * g.st[1][d];
          o2 -= g.shape[d] * g.st[2][d];
        }
      }
    }
  }
}

// out(i,j,k) = in(i,j,k) where out is contiguous along i and in along j.
// Persistent over TILE x TILE tiles (batched over k).  Tiles are visited in
// diagonal order: tile t of a batch has i-tile t % tiles0 and j-tile
// (t / tiles0 + t % tiles0) % tiles1, a bijection under which the tiles that
// run at the same time spread over both the input's and the output's
// contiguous address ranges (a plain row order puts every concurrent tile at
// the same low address bits when the other side's stride is a power of two,
// which concentrates the traffic on a few memory channels).  Full tiles with
// aligned rows use 16-byte loads and stores.
template <typename T, int TILE>
__global__ void __launch_bounds__(256, 8) k_transpose(T *__restrict__ out, const T *__restrict__ in, int64_t n0,
                                                   int64_t n1, int64_t n2, int64_t os1, int64_t os2, int64_t is0,
                                                   int64_t is2, int64_t tiles0, int64_t tiles1, int vec_ok) {
  constexpr int V = (sizeof(T) >= 4) ? 16 / (int)sizeof(T) : 1;
  __shared__ T tile[TILE][TILE + 1];
  const int64_t nt01 = tiles0 * tiles1;
  const int64_t ntiles = nt01 * n2;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t k = t / nt01;
    const int64_t t01 = t - k * nt01;
    const int64_t ti = t01 % tiles0;
    const int64_t tj = (t01 / tiles0 + ti) % tiles1;
    const int64_t i0 = ti * TILE, j0 = tj * TILE;
    const T *src = in + k * is2;
    T *dst = out + k * os2;
    const bool full = (i0 + TILE <= n0) && (j0 + TILE <= n1);
    if (V > 1 && full && vec_ok) {
      // rows i, contiguous along j: TILE/V vectors per row
      for (int e = threadIdx.x; e < TILE * (TILE / V); e += blockDim.x) {
        const int r = e / (TILE / V), cv = e % (TILE / V);
        const Vec<T, V> x = *reinterpret_cast<const Vec<T, V> *>(src + (i0 + r) * is0 + j0 + cv * V);
#pragma unroll
        for (int q = 0; q < V; ++q) tile[r][cv * V + q] = x.v[q];
      }
      __syncthreads();
      // columns j, contiguous along i
      for (int e = threadIdx.x; e < TILE * (TILE / V); e += blockDim.x) {
        const int r = e / (TILE / V), cv = e % (TILE / V);
        Vec<T, V> y;
#pragma unroll
        for (int q = 0; q < V; ++q) y.v[q] = tile[cv * V + q][r];
        *reinterpret_cast<Vec<T, V> *>(dst + (i0 + cv * V) + (j0 + r) * os1) = y;
      }
    } else {
      for (int e = threadIdx.x; e < TILE * TILE; e += blockDim.x) {
        const int r = e / TILE, c = e % TILE;
        if (full || (i0 + r < n0 && j0 + c < n1)) tile[r][c] = src[(i0 + r) * is0 + j0 + c];
      }
      __syncthreads();
      for (int e = threadIdx.x; e < TILE * TILE; e += blockDim.x) {
        const int r = e / TILE, c = e % TILE;
        if (full || (i0 + c < n0 && j0 + r < n1)) dst[(i0 + c) + (j0 + r) * os1] = tile[c][r];
      }
    }
    __syncthreads();
  }
}

// The same transpose when every tile is full, rows are 16-byte aligned and
// there is no batch axis (the permute -> contiguous of a dense 3-D tensor
// collapses to this): no bounds checks, no scalar path, 16-byte accesses only.
template <typename T, int TILE>
__global__ void __launch_bounds__(256) k_transpose_full(T *__restrict__ out, const T *__restrict__ in, int64_t n0,
                                                        int64_t n1, int64_t os1, int64_t is0, int64_t tiles0,
                                                        int64_t tiles1) {
  constexpr int V = 16 / (int)sizeof(T);
  __shared__ T tile[TILE][TILE + 1];
  const int64_t nt = tiles0 * tiles1;
  for (int64_t t = blockIdx.x; t < nt; t += gridDim.x) {
    const int64_t ti = t % tiles0;
    const int64_t tj = (t / tiles0 + ti) % tiles1;
    const int64_t i0 = ti * TILE, j0 = tj * TILE;
    for (int e = threadIdx.x; e < TILE * (TILE / V); e += blockDim.x) {
      const int r = e / (TILE / V), cv = e % (TILE / V);
      const Vec<T, V> x = *reinterpret_cast<const Vec<T, V> *>(in + (i0 + r) * is0 + j0 + cv * V);
#pragma unroll
      for (int q = 0; q < V; ++q) tile[r][cv * V + q] = x.v[q];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < TILE * (TILE / V); e += blockDim.x) {
      const int r = e / (TILE / V), cv = e % (TILE / V);
      Vec<T, V> y;
#pragma unroll
      for (int q = 0; q < V; ++q) y.v[q] = tile[cv * V + q][r];
      *reinterpret_cast<Vec<T, V> *>(out + (i0 + cv * V) + (j0 + r) * os1) = y;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// launch selection
// ---------------------------------------------------------------------------
template <class F>
static acd_status launch_map(acd_ctx *ctx, const F &f, const acd_desc *out, const acd_desc *a, const int64_t *a_st,
                             const acd_desc *b, const int64_t *b_st, cudaStream_t stream) {
  using T = typename F::In;
  using O = typename F::Out;
  constexpr int V = 16 / sizeof(T);
  IterSpace it;
  it.ndim = out->ndim;
  it.nops = 1 + F::kIn;
  for (int d = 0; d < out->ndim; ++d) {
    it.shape[d] = out->shape[d];
    it.stride[0][d] = out->stride[d];
    it.stride[1][d] = a_st[d];
    if (F::kIn == 2) it.stride[2][d] = b_st[d];
  }
  const int64_t n = it.numel();
  if (n == 0) return ACD_OK;
  collapse(it);
  O *po = reinterpret_cast<O *>(desc_ptr(out));
  const T *pa = reinterpret_cast<const T *>(desc_ptr(a));
  const T *pb = F::kIn == 2 ? reinterpret_cast<const T *>(desc_ptr(b)) : pa;

  // ---- flat
  bool flat = it.ndim == 1;
  for (int o = 0; o < it.nops && flat; ++o) flat = it.stride[o][0] == 1;
  if (flat) {
    const int64_t ca = (reinterpret_cast<uintptr_t>(pa) / sizeof(T)) % V;
    const int64_t co = (reinterpret_cast<uintptr_t>(po) / sizeof(O)) % V;
    const int64_t cb = (reinterpret_cast<uintptr_t>(pb) / sizeof(T)) % V;
    const bool ok = aligned_to<T>(pa, sizeof(T)) && aligned_to<O>(po, sizeof(O)) && ca == co && cb == ca;
    const int64_t head = ok ? (V - ca) % V : n;
    const int64_t head_c = head > n ? n : head;
    const int64_t work = ((ok ? (n - head_c) / V + 1 : n) + kEwThreads * kFlatU - 1) / (kEwThreads * kFlatU);
    const int grid = persistent_grid(ctx, k_flat<F, V, kFlatU>, kEwThreads, 0, work);
    k_flat<F, V, kFlatU><<<grid, kEwThreads, 0, stream>>>(po, pa, pb, n, head_c, f);
    return ACD_OK;
  }

  // ---- rows (2-D, inputs dense or broadcast along axis 0); a 1-D problem
  // with a broadcast input is the 2-D case with one column.
  int64_t n0 = it.shape[0], n1 = it.ndim >= 2 ? it.shape[1] : 1;
  int64_t os0 = it.stride[0][0], os1 = it.ndim >= 2 ? it.stride[0][1] : n0;
  if (it.ndim <= 2 && os0 == 1 && n0 % V == 0 && (os1 % V == 0) && aligned_to<O>(po, sizeof(O) * V)) {
    RowOperand A{pa, it.ndim >= 2 ? it.stride[1][1] : 0, (int32_t)it.stride[1][0]};
    RowOperand B{pb, (F::kIn == 2 && it.ndim >= 2) ? it.stride[2][1] : 0,
                 F::kIn == 2 ? (int32_t)it.stride[2][0] : 0};
    bool ok = (it.stride[1][0] == 0 || it.stride[1][0] == 1);
    if (F::kIn == 2) ok = ok && (it.stride[2][0] == 0 || it.stride[2][0] == 1);
    if (ok && A.s0) ok = (A.s1 % V == 0) && aligned_to<T>(pa, sizeof(T) * V);
    if (ok && F::kIn == 2 && B.s0) ok = (B.s1 % V == 0) && aligned_to<T>(pb, sizeof(T) * V);
    if (ok) {
      const int64_t nv0 = n0 / V;
      const int64_t total = nv0 * n1;
      const int64_t work = (total + kEwThreads - 1) / kEwThreads;
      if (total < (1ll << 32) && nv0 < (1ll << 31)) {
        const int grid = persistent_grid(ctx, k_rows<F, V, true>, kEwThreads, 0, work);
        k_rows<F, V, true><<<grid, kEwThreads, 0, stream>>>(po, os1, A, B, nv0, n1, FastDiv((uint32_t)nv0), f);
      } else {
        const int grid = persistent_grid(ctx, k_rows<F, V, false>, kEwThreads, 0, work);
        k_rows<F, V, false><<<grid, kEwThreads, 0, stream>>>(po, os1, A, B, nv0, n1, FastDiv(1), f);
      }
      return ACD_OK;
    }
  }

  // ---- general
  GenSpace g;
  g.ndim = it.ndim;
  for (int d = 0; d < ACD_MAX_DIMS; ++d) {
    g.shape[d] = d < it.ndim ? it.shape[d] : 1;
    for (int o = 0; o < kMaxOps; ++o) g.st[o][d] = (d < it.ndim && o < it.nops) ? it.stride[o][d] : 0;
  }
  const int grid = persistent_grid(ctx, k_general<F, 4>, kEwThreads, 0, ((n + 3) / 4 + kEwThreads - 1) / kEwThreads);
  k_general<F, 4><<<grid, kEwThreads, 0, stream>>>(po, pa, pb, g, n, f);
  return ACD_OK;
}

template <typename T, int TILE>
static void launch_transpose(acd_ctx *ctx, T *out, const T *in, int64_t n0, int64_t n1, int64_t n2, int64_t os1,
                             int64_t os2, int64_t is0, int64_t is2, cudaStream_t stream) {
  constexpr int V = (sizeof(T) >= 4) ? 16 / (int)sizeof(T) : 1;
  if constexpr (sizeof(T) == 4) {
    if (launch_transpose_tma4(ctx, out, in, n0, n1, n2, os1, os2, is0, is2, stream)) return;
  }
  const int64_t tiles0 = (n0 + TILE - 1) / TILE, tiles1 = (n1 + TILE - 1) / TILE;
  const int64_t ntiles = tiles0 * tiles1 * n2;
  static bool carveout_set = false;  // one shared-memory carveout request per instantiation
  if (!carveout_set) {
    cudaFuncSetAttribute(k_transpose<T, TILE>, cudaFuncAttributePreferredSharedMemoryCarveout,
                         cudaSharedmemCarveoutMaxShared);
    cudaGetLastError();
    carveout_set = true;
  }
  const int grid = persistent_grid(ctx, k_transpose<T, TILE>, 256, 0, ntiles);
  const int vec_ok = V > 1 && is0 % V == 0 && os1 % V == 0 && is2 % V == 0 && os2 % V == 0 &&
                     aligned_to<T>(in, 16) && aligned_to<T>(out, 16);
  if constexpr (V > 1) {
    if (vec_ok && n2 == 1 && n0 % TILE == 0 && n1 % TILE == 0) {
      static bool full_carveout_set = false;
      if (!full_carveout_set) {
        cudaFuncSetAttribute(k_transpose_full<T, TILE>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
        cudaGetLastError();
        full_carveout_set = true;
      }
      const int g2 = persistent_grid(ctx, k_transpose_full<T, TILE>, 256, 0, ntiles);
      k_transpose_full<T, TILE><<<g2, 256, 0, stream>>>(out, in, n0, n1, os1, is0, tiles0, tiles1);
      return;
    }
  }
  k_transpose<T, TILE><<<grid, 256, 0, stream>>>(out, in, n0, n1, n2, os1, os2, is0, is2, tiles0, tiles1, vec_ok);
}

// Bitwise copy between two views of one element size.
template <typename W, int TILE>
static acd_status copy_sized(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, cudaStream_t stream) {
  IterSpace it;
  it.ndim = out->ndim;
  it.nops = 2;
  for (int d = 0; d < out->ndim; ++d) {
    it.shape[d] = out->shape[d];
    it.stride[0][d] = out->stride[d];
    it.stride[1][d] = in->stride[d];
  }
  if (it.numel() == 0) return ACD_OK;
  collapse(it);
  W *po = reinterpret_cast<W *>(desc_ptr(out));
  const W *pi = reinterpret_cast<const W *>(desc_ptr(in));
  // transpose: out contiguous along one axis, in contiguous along another
  if (it.ndim == 2 || it.ndim == 3) {
    int ao = -1, ai = -1;
    for (int d = 0; d < it.ndim; ++d) {
      if (it.stride[0][d] == 1) ao = d;
      if (it.stride[1][d] == 1) ai = d;
    }
    if (ao >= 0 && ai >= 0 && ao != ai) {
      int bd = 3 - ao - ai;  // batch axis (3-D only)
      int64_t n2 = 1, os2 = 0, is2 = 0;
      if (it.ndim == 3) {
        n2 = it.shape[bd];
        os2 = it.stride[0][bd];
        is2 = it.stride[1][bd];
      }
      launch_transpose<W, TILE>(ctx, po, pi, it.shape[ao], it.shape[ai], n2, it.stride[0][ai], os2,
                                it.stride[1][ao], is2, stream);
      return ACD_OK;
    }
  }
  int64_t st_a[ACD_MAX_DIMS], st_o[ACD_MAX_DIMS];
  acd_desc o2 = *out, i2 = *in;
  o2.ndim = i2.ndim = it.ndim;
  for (int d = 0; d < it.ndim; ++d) {
    o2.shape[d] = i2.shape[d] = it.shape[d];
    st_o[d] = o2.stride[d] = it.stride[0][d];
    st_a[d] = i2.stride[d] = it.stride[1][d];
  }
  (void)st_o;
  return launch_map(ctx, UnaryF<ACD_COPY, W>{}, &o2, &i2, st_a, nullptr, nullptr, stream);
}

// ---------------------------------------------------------------------------
// dispatch helpers
// ---------------------------------------------------------------------------
static acd_status same_shape(const acd_desc *a, const acd_desc *b, const char *what) {
  if (desc_numel(a) != desc_numel(b)) return fail(ACD_ERR_SHAPE, "%s: element counts differ", what);
  if (a->ndim != b->ndim) return fail(ACD_ERR_SHAPE, "%s: ranks differ (%d vs %d)", what, a->ndim, b->ndim);
  for (int d = 0; d < a->ndim; ++d)
    if (a->shape[d] != b->shape[d]) return fail(ACD_ERR_SHAPE, "%s: extents differ on axis %d", what, d);
  return ACD_OK;
}

template <typename T>
static acd_status unary_t(acd_ctx *ctx, int op, const acd_desc *out, const acd_desc *in, cudaStream_t s) {
  const int64_t *st = in->stride;
#define ACD_U(OPC)                                                                  \
  case OPC:                                                                         \
    return launch_map(ctx, UnaryF<OPC, T>{}, out, in, st, nullptr, nullptr, s);
  if constexpr (std::is_floating_point<T>::value) {
    switch (op) {
      ACD_U(ACD_EXP) ACD_U(ACD_LOG) ACD_U(ACD_SQRT) ACD_U(ACD_ABS) ACD_U(ACD_FLOOR) ACD_U(ACD_CEIL)
      ACD_U(ACD_ROUND) ACD_U(ACD_ERF) ACD_U(ACD_TANH) ACD_U(ACD_SIGMOID) ACD_U(ACD_RELU) ACD_U(ACD_SIN)
      ACD_U(ACD_COS) ACD_U(ACD_NEG) ACD_U(ACD_SQUARE) ACD_U(ACD_COPY)
      default: break;
    }
  } else {
    switch (op) {
      ACD_U(ACD_ABS) ACD_U(ACD_NEG) ACD_U(ACD_SQUARE) ACD_U(ACD_COPY)
      default: break;
    }
  }
#undef ACD_U
  return fail(ACD_ERR_UNSUPPORTED, "unary op %d not supported for this dtype", op);
}

template <typename T, typename O>
static acd_status binary_to(acd_ctx *ctx, int op, const acd_desc *out, const acd_desc *a, const int64_t *sa,
                            const acd_desc *b, const int64_t *sb, cudaStream_t s) {
#define ACD_B(OPC)                                                                \
  case OPC:                                                                       \
    return launch_map(ctx, BinaryF<OPC, T, O>{}, out, a, sa, b, sb, s);
  constexpr bool cmp_only = !std::is_same<T, O>::value;
  if constexpr (cmp_only) {
    switch (op) {
      ACD_B(ACD_GT) ACD_B(ACD_LT) ACD_B(ACD_EQ) ACD_B(ACD_NE) ACD_B(ACD_GE) ACD_B(ACD_LE)
      default: break;
    }
  } else if constexpr (std::is_floating_point<T>::value) {
    switch (op) {
      ACD_B(ACD_ADD) ACD_B(ACD_SUB) ACD_B(ACD_MUL) ACD_B(ACD_DIV) ACD_B(ACD_MAX) ACD_B(ACD_MIN) ACD_B(ACD_POW)
      ACD_B(ACD_GT) ACD_B(ACD_LT) ACD_B(ACD_EQ) ACD_B(ACD_NE) ACD_B(ACD_GE) ACD_B(ACD_LE)
      default: break;
    }
  } else if constexpr (std::is_same<T, __half>::value) {
    switch (op) {
      ACD_B(ACD_ADD) ACD_B(ACD_SUB) ACD_B(ACD_MUL) ACD_B(ACD_DIV) ACD_B(ACD_MAX) ACD_B(ACD_MIN)
      ACD_B(ACD_GT) ACD_B(ACD_LT) ACD_B(ACD_EQ) ACD_B(ACD_NE) ACD_B(ACD_GE) ACD_B(ACD_LE)
      default: break;
    }
  } else {
    switch (op) {
      ACD_B(ACD_ADD) ACD_B(ACD_SUB) ACD_B(ACD_MUL) ACD_B(ACD_MAX) ACD_B(ACD_MIN)
      ACD_B(ACD_GT) ACD_B(ACD_LT) ACD_B(ACD_EQ) ACD_B(ACD_NE) ACD_B(ACD_GE) ACD_B(ACD_LE)
      default: break;
    }
  }
#undef ACD_B
  return fail(ACD_ERR_UNSUPPORTED, "binary op %d not supported for this dtype pair", op);
}

template <typename T, typename O>
static acd_status scalar_to(acd_ctx *ctx, int op, const acd_desc *out, const acd_desc *in, double sv,
                            cudaStream_t s) {
  T ts;
  if constexpr (std::is_same<T, __half>::value)
    ts = __double2half(sv);  // the scalar rounds once to the tensor dtype
  else
    ts = (T)sv;
  const int64_t *st = in->stride;
#define ACD_S(OPC)                                                                            \
  case OPC:                                                                                   \
    return launch_map(ctx, ScalarF<OPC, T, O>{ts}, out, in, st, nullptr, nullptr, s);
  constexpr bool cmp_only = !std::is_same<T, O>::value;
  if constexpr (cmp_only) {
    switch (op) {
      ACD_S(ACD_GT) ACD_S(ACD_LT) ACD_S(ACD_EQ) ACD_S(ACD_NE) ACD_S(ACD_GE) ACD_S(ACD_LE)
      default: break;
    }
  } else if constexpr (std::is_floating_point<T>::value) {
    if (op == ACD_POW && sv == 2.0) return launch_map(ctx, SquareScalarF<T>{}, out, in, st, nullptr, nullptr, s);
    switch (op) {
      ACD_S(ACD_ADD) ACD_S(ACD_SUB) ACD_S(ACD_MUL) ACD_S(ACD_DIV) ACD_S(ACD_MAX) ACD_S(ACD_MIN) ACD_S(ACD_POW)
      ACD_S(ACD_GT) ACD_S(ACD_LT) ACD_S(ACD_EQ) ACD_S(ACD_NE) ACD_S(ACD_GE) ACD_S(ACD_LE)
      ACD_S(ACD_RSUB) ACD_S(ACD_RDIV)
      default: break;
    }
  } else if constexpr (std::is_same<T, __half>::value) {
    switch (op) {
      ACD_S(ACD_ADD) ACD_S(ACD_SUB) ACD_S(ACD_MUL) ACD_S(ACD_DIV) ACD_S(ACD_MAX) ACD_S(ACD_MIN)
      ACD_S(ACD_GT) ACD_S(ACD_LT) ACD_S(ACD_EQ) ACD_S(ACD_NE) ACD_S(ACD_GE) ACD_S(ACD_LE)
      ACD_S(ACD_RSUB) ACD_S(ACD_RDIV)
      default: break;
    }
  } else {
    switch (op) {
      ACD_S(ACD_ADD) ACD_S(ACD_SUB) ACD_S(ACD_MUL) ACD_S(ACD_MAX) ACD_S(ACD_MIN) ACD_S(ACD_RSUB)
      ACD_S(ACD_GT) ACD_S(ACD_LT) ACD_S(ACD_EQ) ACD_S(ACD_NE) ACD_S(ACD_GE) ACD_S(ACD_LE)
      default: break;
    }
  }
#undef ACD_S
  return fail(ACD_ERR_UNSUPPORTED, "scalar op %d not supported for this dtype pair", op);
}

static bool is_compare(int op) { return op >= ACD_GT && op <= ACD_LE; }

// out = v for every element of a view.  The launcher wants one input operand:
// it is the output's first element at stride 0 on every axis, never read.
template <typename T>
struct FillF {
  static constexpr int kIn = 1;
  using In = T;
  using Out = T;
  T v;
  __device__ __forceinline__ T operator()(T) const { return v; }
};

template <typename T>
static acd_status fill_t(acd_ctx *ctx, const acd_desc *out, double value, cudaStream_t s) {
  int64_t zero[ACD_MAX_DIMS] = {0, 0, 0, 0, 0, 0, 0, 0};
  return launch_map(ctx, FillF<T>{convert_value<double, T>(value)}, out, out, zero, nullptr, nullptr, s);
}

// x[i] = v where mask[i] != 0, in place.  Dense operands take 16 mask bytes
// per load; other views walk int64 coordinates in runs of 4.
template <typename T>
__global__ void __launch_bounds__(kEwThreads) k_mask_fill_flat(T *__restrict__ x, const uint8_t *__restrict__ m,
                                                               int64_t n, T v) {
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const int64_t nv = (reinterpret_cast<uintptr_t>(m) & 15) == 0 ? n / 16 : 0;
  for (int64_t i = tid; i < nv; i += nth) {
    const uint4 w = reinterpret_cast<const uint4 *>(m)[i];
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (ws[q])
#pragma unroll
        for (int b = 0; b < 4; ++b)
          if ((ws[q] >> (8 * b)) & 0xffu) x[i * 16 + q * 4 + b] = v;
  }
  for (int64_t i = nv * 16 + tid; i < n; i += nth)
    if (m[i]) x[i] = v;
}

template <typename T>
__global__ void __launch_bounds__(kEwThreads) k_mask_fill_general(T *__restrict__ x, const uint8_t *__restrict__ m,
                                                                  GenSpace g, int64_t n, T v) {
  constexpr int RUN = 4;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = tid * RUN; base < n; base += nth * RUN) {
    int64_t c[ACD_MAX_DIMS];
    int64_t ox = 0, om = 0, rem = base;
#pragma unroll
    for (int d = 0; d < ACD_MAX_DIMS; ++d) {
      if (d < g.ndim) {
        c[d] = rem % g.shape[d];
        rem /= g.shape[d];
        ox += c[d] * g.st[0][d];
        om += c[d] * g.st[1][d];
      }
    }
    for (int r = 0; r < RUN && base + r < n; ++r) {
      if (m[om]) x[ox] = v;
      ox += g.st[0][0];
      om += g.st[1][0];
      if (++c[0] == g.shape[0]) {
        c[0] = 0;
        ox -= g.shape[0] * g.st[0][0];
        om -= g.shape[0] * g.st[1][0];
        for (int d = 1; d < g.ndim; ++d) {
          ox += g.st[0][d];
          om += g.st[1][d];
          if (++c[d] < g.shape[d]) break;
          c[d] = 0;
          ox -= g.shape[d] * g.st[0][d];
          om -= g.shape[d] * g.st[1][d];
        }
      }
    }
  }
}

template <typename T>
static acd_status mask_fill_t(acd_ctx *ctx, const acd_desc *x, const acd_desc *mask, double value,
                              cudaStream_t s) {
  IterSpace it;
  it.ndim = x->ndim;
  it.nops = 2;
  for (int d = 0; d < x->ndim; ++d) {
    it.shape[d] = x->shape[d];
    it.stride[0][d] = x->stride[d];
    it.stride[1][d] = mask->stride[d];
  }
  const int64_t n = it.numel();
  if (n == 0) return ACD_OK;
  collapse(it);
  T *px = reinterpret_cast<T *>(desc_ptr(x));
  const uint8_t *pm = reinterpret_cast<const uint8_t *>(desc_ptr(mask));
  const T v = convert_value<double, T>(value);
  if (it.ndim == 1 && it.stride[0][0] == 1 && it.stride[1][0] == 1) {
    const int grid = persistent_grid(ctx, k_mask_fill_flat<T>, kEwThreads, 0, (n / 16 + kEwThreads) / kEwThreads);
    k_mask_fill_flat<T><<<grid, kEwThreads, 0, s>>>(px, pm, n, v);
    return ACD_OK;
  }
  GenSpace g;
  g.ndim = it.ndim;
  for (int d = 0; d < ACD_MAX_DIMS; ++d) {
    g.shape[d] = d < it.ndim ? it.shape[d] : 1;
    for (int o = 0; o < kMaxOps; ++o) g.st[o][d] = (d < it.ndim && o < 2) ? it.stride[o][d] : 0;
  }
  const int grid = persistent_grid(ctx, k_mask_fill_general<T>, kEwThreads, 0, ((n + 3) / 4 + kEwThreads - 1) / kEwThreads);
  k_mask_fill_general<T><<<grid, kEwThreads, 0, s>>>(px, pm, g, n, v);
  return ACD_OK;
}

template <typename From>
static acd_status convert_from(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, cudaStream_t s) {
  const int64_t *st = in->stride;
  switch (out->dtype) {
    case ACD_FLOAT32: return launch_map(ctx, ConvertF<From, float>{}, out, in, st, nullptr, nullptr, s);
    case ACD_FLOAT64: return launch_map(ctx, ConvertF<From, double>{}, out, in, st, nullptr, nullptr, s);
    case ACD_INT32: return launch_map(ctx, ConvertF<From, int32_t>{}, out, in, st, nullptr, nullptr, s);
    case ACD_INT64: return launch_map(ctx, ConvertF<From, int64_t>{}, out, in, st, nullptr, nullptr, s);
    case ACD_BOOL: return launch_map(ctx, ConvertF<From, uint8_t>{}, out, in, st, nullptr, nullptr, s);
    case ACD_FLOAT16: return launch_map(ctx, ConvertF<From, __half>{}, out, in, st, nullptr, nullptr, s);
    case ACD_INT8: return launch_map(ctx, ConvertF<From, int8_t>{}, out, in, st, nullptr, nullptr, s);
    default: return fail(ACD_ERR_DTYPE, "acd_convert: target dtype %d not supported", out->dtype);
  }
}

}  // namespace acd

using namespace acd;

// Contiguous copy into one or two destinations (16-byte vectors, four in
// flight per thread): the streaming rate of one read against one or two
// writes, the ceiling of a kernel with that traffic mix.
template <bool TWO>
__global__ void __launch_bounds__(256) k_fanout(const uint4 *__restrict__ src, uint4 *__restrict__ d0,
                                               uint4 *__restrict__ d1, int64_t n) {
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * nth < n; i += 4 * nth) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = src[i + u * nth];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      d0[i + u * nth] = v[u];
      if (TWO) d1[i + u * nth] = v[u];
    }
  }
  for (; i < n; i += nth) {
    const uint4 v = src[i];
    d0[i] = v;
    if (TWO) d1[i] = v;
  }
}

extern "C" {

acd_status acd_convert(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_convert: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  ACD_TRY(same_shape(out, in, "acd_convert"));
  if (out->dtype == in->dtype) return acd_copy(ctx, out, in, stream);
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (in->dtype) {
    case ACD_FLOAT32: st = convert_from<float>(ctx, out, in, s); break;
    case ACD_FLOAT64: st = convert_from<double>(ctx, out, in, s); break;
    case ACD_INT32: st = convert_from<int32_t>(ctx, out, in, s); break;
    case ACD_INT64: st = convert_from<int64_t>(ctx, out, in, s); break;
    case ACD_BOOL: st = convert_from<uint8_t>(ctx, out, in, s); break;
    case ACD_FLOAT16: st = convert_from<__half>(ctx, out, in, s); break;
    case ACD_INT8: st = convert_from<int8_t>(ctx, out, in, s); break;
    default: return fail(ACD_ERR_DTYPE, "acd_convert: source dtype %d not supported", in->dtype);
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_fill(acd_ctx *ctx, const acd_desc *out, double value, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_fill: null context");
  ACD_TRY(check_desc(out, "out"));
  if (desc_numel(out) == 0) return ACD_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (out->dtype) {
    case ACD_FLOAT32: st = fill_t<float>(ctx, out, value, s); break;
    case ACD_FLOAT64: st = fill_t<double>(ctx, out, value, s); break;
    case ACD_INT32: st = fill_t<int32_t>(ctx, out, value, s); break;
    case ACD_INT64: st = fill_t<int64_t>(ctx, out, value, s); break;
    case ACD_BOOL: st = fill_t<uint8_t>(ctx, out, value, s); break;
    case ACD_FLOAT16: st = fill_t<__half>(ctx, out, value, s); break;
    case ACD_INT8: st = fill_t<int8_t>(ctx, out, value, s); break;
    default: return fail(ACD_ERR_DTYPE, "acd_fill: dtype %d not supported", out->dtype);
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_mask_fill(acd_ctx *ctx, const acd_desc *x, const acd_desc *mask, double value, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_mask_fill: null context");
  ACD_TRY(check_desc(x, "x"));
  ACD_TRY(check_desc(mask, "mask"));
  if (mask->dtype != ACD_BOOL) return fail(ACD_ERR_DTYPE, "Mask tensor must be boolean type");
  if (same_shape(x, mask, "acd_mask_fill") != ACD_OK) return fail(ACD_ERR_SHAPE, "Tensor and mask must have the same shape");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (x->dtype) {
    case ACD_FLOAT32: st = mask_fill_t<float>(ctx, x, mask, value, s); break;
    case ACD_FLOAT64: st = mask_fill_t<double>(ctx, x, mask, value, s); break;
    case ACD_INT32: st = mask_fill_t<int32_t>(ctx, x, mask, value, s); break;
    case ACD_INT64: st = mask_fill_t<int64_t>(ctx, x, mask, value, s); break;
    case ACD_BOOL: st = mask_fill_t<uint8_t>(ctx, x, mask, value, s); break;
    case ACD_FLOAT16: st = mask_fill_t<__half>(ctx, x, mask, value, s); break;
    case ACD_INT8: st = mask_fill_t<int8_t>(ctx, x, mask, value, s); break;
    default: return fail(ACD_ERR_DTYPE, "acd_mask_fill: dtype %d not supported", x->dtype);
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_unary(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_unary: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  ACD_TRY(same_shape(out, in, "acd_unary"));
  if (out->dtype != in->dtype) return fail(ACD_ERR_DTYPE, "acd_unary: out dtype must equal in dtype");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (in->dtype) {
    case ACD_FLOAT32: st = unary_t<float>(ctx, op, out, in, s); break;
    case ACD_FLOAT64: st = unary_t<double>(ctx, op, out, in, s); break;
    case ACD_INT32: st = unary_t<int32_t>(ctx, op, out, in, s); break;
    case ACD_INT64: st = unary_t<int64_t>(ctx, op, out, in, s); break;
    case ACD_FLOAT16: st = unary_t<__half>(ctx, op, out, in, s); break;
    case ACD_INT8: st = unary_t<int8_t>(ctx, op, out, in, s); break;
    default: return fail(ACD_ERR_DTYPE, "acd_unary: dtype %d not supported", in->dtype);
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_binary(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *a, const acd_desc *b,
                      acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_binary: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(a, "a"));
  ACD_TRY(check_desc(b, "b"));
  if (op < ACD_ADD || op > ACD_LE) return fail(ACD_ERR_INVALID, "acd_binary: bad op %d", op);
  if (a->dtype != b->dtype) return fail(ACD_ERR_DTYPE, "acd_binary: operands must share one dtype");
  int32_t bnd = 0;
  int64_t bshape[ACD_MAX_DIMS];
  ACD_TRY(acd_broadcast_shape(a->ndim, a->shape, b->ndim, b->shape, &bnd, bshape));
  // the output must have the broadcast shape (as many elements, same extents)
  if (out->ndim != bnd) return fail(ACD_ERR_SHAPE, "acd_binary: output rank %d, broadcast rank %d", out->ndim, bnd);
  for (int d = 0; d < bnd; ++d)
    if (out->shape[d] != bshape[d]) return fail(ACD_ERR_SHAPE, "acd_binary: output extent mismatch on axis %d", d);
  int64_t sa[ACD_MAX_DIMS], sb[ACD_MAX_DIMS];
  ACD_TRY(acd_broadcast_strides(a->ndim, a->shape, a->stride, bnd, bshape, sa));
  ACD_TRY(acd_broadcast_strides(b->ndim, b->shape, b->stride, bnd, bshape, sb));
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool cmp = is_compare(op);
  const bool to_bool = out->dtype == ACD_BOOL;
  if (to_bool && !cmp) return fail(ACD_ERR_DTYPE, "acd_binary: bool output only for comparisons");
  if (!to_bool && out->dtype != a->dtype) return fail(ACD_ERR_DTYPE, "acd_binary: out dtype must be the input dtype or bool");
  acd_status st;
  switch (a->dtype) {
    case ACD_FLOAT32:
      st = to_bool ? binary_to<float, uint8_t>(ctx, op, out, a, sa, b, sb, s)
                   : binary_to<float, float>(ctx, op, out, a, sa, b, sb, s);
      break;
    case ACD_FLOAT64:
      st = to_bool ? binary_to<double, uint8_t>(ctx, op, out, a, sa, b, sb, s)
                   : binary_to<double, double>(ctx, op, out, a, sa, b, sb, s);
      break;
    case ACD_INT32:
      st = to_bool ? binary_to<int32_t, uint8_t>(ctx, op, out, a, sa, b, sb, s)
                   : binary_to<int32_t, int32_t>(ctx, op, out, a, sa, b, sb, s);
      break;
    case ACD_INT64:
      st = to_bool ? binary_to<int64_t, uint8_t>(ctx, op, out, a, sa, b, sb, s)
                   : binary_to<int64_t, int64_t>(ctx, op, out, a, sa, b, sb, s);
      break;
    case ACD_FLOAT16:
      st = to_bool ? binary_to<__half, uint8_t>(ctx, op, out, a, sa, b, sb, s)
                   : binary_to<__half, __half>(ctx, op, out, a, sa, b, sb, s);
      break;
    case ACD_INT8:
      st = to_bool ? binary_to<int8_t, uint8_t>(ctx, op, out, a, sa, b, sb, s)
                   : binary_to<int8_t, int8_t>(ctx, op, out, a, sa, b, sb, s);
      break;
    default: return fail(ACD_ERR_DTYPE, "acd_binary: dtype %d not supported", a->dtype);
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_scalar(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *in, double sv,
                      acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_scalar: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  ACD_TRY(same_shape(out, in, "acd_scalar"));
  if (op < ACD_ADD || op > ACD_RDIV) return fail(ACD_ERR_INVALID, "acd_scalar: bad op %d", op);
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool to_bool = out->dtype == ACD_BOOL;
  if (to_bool && !is_compare(op)) return fail(ACD_ERR_DTYPE, "acd_scalar: bool output only for comparisons");
  if (!to_bool && out->dtype != in->dtype) return fail(ACD_ERR_DTYPE, "acd_scalar: out dtype must be the input dtype or bool");
  acd_status st;
  switch (in->dtype) {
    case ACD_FLOAT32:
      st = to_bool ? scalar_to<float, uint8_t>(ctx, op, out, in, sv, s) : scalar_to<float, float>(ctx, op, out, in, sv, s);
      break;
    case ACD_FLOAT64:
      st = to_bool ? scalar_to<double, uint8_t>(ctx, op, out, in, sv, s)
                   : scalar_to<double, double>(ctx, op, out, in, sv, s);
      break;
    case ACD_INT32:
      st = to_bool ? scalar_to<int32_t, uint8_t>(ctx, op, out, in, sv, s)
                   : scalar_to<int32_t, int32_t>(ctx, op, out, in, sv, s);
      break;
    case ACD_INT64:
      st = to_bool ? scalar_to<int64_t, uint8_t>(ctx, op, out, in, sv, s)
                   : scalar_to<int64_t, int64_t>(ctx, op, out, in, sv, s);
      break;
    case ACD_FLOAT16:
      st = to_bool ? scalar_to<__half, uint8_t>(ctx, op, out, in, sv, s)
                   : scalar_to<__half, __half>(ctx, op, out, in, sv, s);
      break;
    case ACD_INT8:
      st = to_bool ? scalar_to<int8_t, uint8_t>(ctx, op, out, in, sv, s)
                   : scalar_to<int8_t, int8_t>(ctx, op, out, in, sv, s);
      break;
    default: return fail(ACD_ERR_DTYPE, "acd_scalar: dtype %d not supported", in->dtype);
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_fused(acd_ctx *ctx, int32_t op, const acd_desc *out, const acd_desc *a, const acd_desc *b, double p0,
                     acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_fused: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(a, "a"));
  if (out->dtype != a->dtype || !is_float(a->dtype))
    return fail(ACD_ERR_DTYPE, "acd_fused: float32/float64 input and output of one dtype required");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f32 = a->dtype == ACD_FLOAT32;
  acd_status st = ACD_OK;
  if (op == ACD_FUSED_SCALE_ADD_EXP_NEG_SQUARE || op == ACD_FUSED_TANH_SCALE) {
    ACD_TRY(same_shape(out, a, "acd_fused"));
    if (op == ACD_FUSED_SCALE_ADD_EXP_NEG_SQUARE)
      st = f32 ? launch_map(ctx, FusedScaleAddExpNegSquare<float>{(float)p0}, out, a, a->stride, nullptr, nullptr, s)
               : launch_map(ctx, FusedScaleAddExpNegSquare<double>{p0}, out, a, a->stride, nullptr, nullptr, s);
    else
      st = f32 ? launch_map(ctx, FusedTanhScale<float>{(float)p0}, out, a, a->stride, nullptr, nullptr, s)
               : launch_map(ctx, FusedTanhScale<double>{p0}, out, a, a->stride, nullptr, nullptr, s);
  } else if (op == ACD_FUSED_ADD_RELU) {
    ACD_TRY(check_desc(b, "b"));
    if (b->dtype != a->dtype) return fail(ACD_ERR_DTYPE, "acd_fused: operands must share one dtype");
    int32_t bnd = 0;
    int64_t bshape[ACD_MAX_DIMS];
    ACD_TRY(acd_broadcast_shape(a->ndim, a->shape, b->ndim, b->shape, &bnd, bshape));
    if (out->ndim != bnd) return fail(ACD_ERR_SHAPE, "acd_fused: output rank mismatch");
    for (int d = 0; d < bnd; ++d)
      if (out->shape[d] != bshape[d]) return fail(ACD_ERR_SHAPE, "acd_fused: output extent mismatch on axis %d", d);
    int64_t sa[ACD_MAX_DIMS], sb[ACD_MAX_DIMS];
    ACD_TRY(acd_broadcast_strides(a->ndim, a->shape, a->stride, bnd, bshape, sa));
    ACD_TRY(acd_broadcast_strides(b->ndim, b->shape, b->stride, bnd, bshape, sb));
    st = f32 ? launch_map(ctx, FusedAddRelu<float>{}, out, a, sa, b, sb, s)
             : launch_map(ctx, FusedAddRelu<double>{}, out, a, sa, b, sb, s);
  } else {
    return fail(ACD_ERR_INVALID, "acd_fused: bad op %d", op);
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_copy_fanout(acd_ctx *ctx, void *dst0, void *dst1, const void *src, int64_t nbytes,
                           acd_stream stream) {
  if (!ctx || !dst0 || !src) return fail(ACD_ERR_INVALID, "acd_copy_fanout: null argument");
  if (nbytes < 0 || nbytes % 16 ||
      ((reinterpret_cast<uintptr_t>(dst0) | reinterpret_cast<uintptr_t>(dst1) | reinterpret_cast<uintptr_t>(src)) & 15))
    return fail(ACD_ERR_INVALID, "acd_copy_fanout: 16-byte aligned buffers and a multiple of 16 bytes required");
  if (nbytes == 0) return ACD_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = nbytes / 16;
  const uint4 *ps = static_cast<const uint4 *>(src);
  if (dst1) {
    const int grid = persistent_grid(ctx, k_fanout<true>, 256, 0, (n + 1023) / 1024);
    k_fanout<true><<<grid, 256, 0, s>>>(ps, static_cast<uint4 *>(dst0), static_cast<uint4 *>(dst1), n);
  } else {
    const int grid = persistent_grid(ctx, k_fanout<false>, 256, 0, (n + 1023) / 1024);
    k_fanout<false><<<grid, 256, 0, s>>>(ps, static_cast<uint4 *>(dst0), nullptr, n);
  }
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

acd_status acd_copy(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_copy: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  ACD_TRY(same_shape(out, in, "acd_copy"));
  if (out->dtype != in->dtype) return fail(ACD_ERR_DTYPE, "acd_copy: dtypes differ");
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  switch (dtype_size(in->dtype)) {
    case 1: st = copy_sized<uint8_t, 64>(ctx, out, in, s); break;
    case 2: st = copy_sized<uint16_t, 64>(ctx, out, in, s); break;
    case 4: st = copy_sized<uint32_t, 64>(ctx, out, in, s); break;
    case 8: st = copy_sized<uint64_t, 32>(ctx, out, in, s); break;
    default: return fail(ACD_ERR_DTYPE, "acd_copy: bad dtype");
  }
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

}  // extern "C"
