// Softmax along an axis (row softmax) and over the whole tensor.
//
// Reference: tensor_softmax_{float32,float64} (src/kernels/tensor_ops.cu:826-846)
// normalise the whole tensor with two host round-trips (global max, then
// global sum of shift_exp_kernel's output) and are subject to the 65535-block
// truncation of launch_reduction.  The row softmax the workload needs is
// exp(v - max(v)) / sum(exp(v - max(v))) along one axis.
//
// Axis softmax: the view is collapsed to (L lanes, R steps, O outer) around
// the axis.  A thread-block cluster of C CTAs owns LT adjacent lanes (a
// 128-byte row of memory per step when lanes are contiguous, so every load is
// coalesced even though, column-major, a row's steps are nrow elements apart)
// and splits the R steps into C chunks.  Each CTA keeps its chunk in shared
// memory (re-reading from L2 what does not fit), and the per-lane maxima and
// sums are exchanged through distributed shared memory: HBM sees one read and
// one write per element.  exp() is evaluated once per element; the quotient
// is a multiply by the reciprocal of the sum (within one ulp of the division).
//
// Whole-tensor softmax: one streaming pass computes the online (max, sum)
// pair, a second pass writes exp(x - max) / sum.
#include <cooperative_groups.h>

#include <algorithm>
#include <numeric>

#include "common.cuh"
#include "ops.cuh"
#include "reduce_acc.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace acd {

struct SoftArgs {
  const void *in;
  void *out;
  int64_t L, R, O;
  int64_t sl, sr, so;
  int64_t ol, orr, oo;
  int64_t lblocks;
  int64_t chunk;  // steps per CTA
  int64_t cap;    // steps of the chunk held in shared memory
};

template <typename T, int LT>
__global__ void __launch_bounds__(256) k_softmax_axis(SoftArgs a) {
  constexpr int G = 256 / LT;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T *tile = reinterpret_cast<T *>(smem_raw);  // [cap][LT]
  __shared__ double cmax[LT];
  __shared__ double psum[LT];
  __shared__ double red[G][LT];

  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int64_t group_id = blockIdx.x / C;  // (lane block, o)
  const int64_t o = group_id / a.lblocks, lb = group_id % a.lblocks;
  const int lane = (LT == 1) ? 0 : (int)(threadIdx.x % LT);
  const int grp = (LT == 1) ? (int)threadIdx.x : (int)(threadIdx.x / LT);
  const int64_t l = lb * LT + lane;
  const bool lane_ok = l < a.L;
  const int64_t r0 = (int64_t)rank * a.chunk;
  int64_t r1 = r0 + a.chunk;
  if (r1 > a.R) r1 = a.R;
  const T *in = static_cast<const T *>(a.in) + o * a.so + (lane_ok ? l : 0) * a.sl;
  T *out = static_cast<T *>(a.out) + o * a.oo + (lane_ok ? l : 0) * a.ol;

  // pass 1: load (into shared memory where it fits) and take the lane maximum
  T m = lowest_of<T>();
#pragma unroll 8
  for (int64_t r = r0 + grp; r < r1; r += G) {
    T x = lowest_of<T>();
    if (lane_ok) x = in[r * a.sr];
    const int64_t k = r - r0;
    if (k < a.cap) tile[k * LT + lane] = x;
    m = m_max(m, x);
  }
  red[grp][lane] = (double)m;
  __syncthreads();
  if (grp == 0) {
    T mm = lowest_of<T>();
    for (int g = 0; g < G; ++g) mm = m_max(mm, (T)red[g][lane]);
    cmax[lane] = (double)mm;
  }
  // exchange maxima across the cluster
  cluster.sync();
  double M = -INFINITY;
  for (int q = 0; q < C; ++q) {
    const double *rm = cluster.map_shared_rank(cmax, q);
    M = fmax(M, rm[lane]);
  }
  const T Mt = (T)M;

  // pass 2: e = exp(x - M), kept in shared memory; lane sums in float64
  double s = 0.0;
#pragma unroll 8
  for (int64_t r = r0 + grp; r < r1; r += G) {
    const int64_t k = r - r0;
    T x;
    if (k < a.cap)
      x = tile[k * LT + lane];
    else
      x = lane_ok ? in[r * a.sr] : lowest_of<T>();
    const T e = lane_ok ? m_exp(x - Mt) : T(0);
    if (k < a.cap) tile[k * LT + lane] = e;
    s += (double)e;
  }
  __syncthreads();  // red[] reuse
  red[grp][lane] = s;
  __syncthreads();
  if (grp == 0) {
    double ss = 0.0;
    for (int g = 0; g < G; ++g) ss += red[g][lane];
    psum[lane] = ss;
  }
  cluster.sync();
  double S = 0.0;
  for (int q = 0; q < C; ++q) {
    const double *rs = cluster.map_shared_rank(psum, q);
    S += rs[lane];
  }
  cluster.sync();  // no CTA leaves while another still reads its psum/cmax
  const T inv = (T)(1.0 / S);

  // pass 3: write
  if (lane_ok) {
#pragma unroll 8
    for (int64_t r = r0 + grp; r < r1; r += G) {
      const int64_t k = r - r0;
      T e;
      if (k < a.cap)
        e = tile[k * LT + lane];
      else
        e = m_exp(in[r * a.sr] - Mt);
      out[r * a.orr] = e * inv;
    }
  }
}

// ---- two passes, for rows whose chunk does not fit shared memory -----------
// Pass 1: each CTA reduces LT lanes x `chunk` steps to per-lane online
// (max, sum of exp(x - max)) partials.  Pass 2: each CTA merges the partials
// of its lanes over all chunks, then re-reads its chunk and writes the
// normalised values.  Reads each element twice, writes it once; every CTA is
// independent, so occupancy is not limited by a cluster or by shared memory.
template <typename T, int LT>
__global__ void __launch_bounds__(256) k_softmax_partials(SoftArgs a, int64_t nchunks, double2 *__restrict__ part) {
  constexpr int G = 256 / LT;
  __shared__ double2 red[G][LT];
  const int64_t c = blockIdx.x % nchunks, gid = blockIdx.x / nchunks;
  const int64_t o = gid / a.lblocks, lb = gid % a.lblocks;
  const int lane = (LT == 1) ? 0 : (int)(threadIdx.x % LT);
  const int grp = (LT == 1) ? (int)threadIdx.x : (int)(threadIdx.x / LT);
  const int64_t l = lb * LT + lane;
  const bool lane_ok = l < a.L;
  const int64_t r0 = c * a.chunk;
  int64_t r1 = r0 + a.chunk;
  if (r1 > a.R) r1 = a.R;
  const T *in = static_cast<const T *>(a.in) + o * a.so + (lane_ok ? l : 0) * a.sl;
  double m = -INFINITY, sum = 0.0;
  if (lane_ok) {
#pragma unroll 8
    for (int64_t r = r0 + grp; r < r1; r += G) {
      const double x = (double)in[r * a.sr];
      if (x > m) {
        sum = sum * exp(m - x) + 1.0;
        m = x;
      } else if (x != -INFINITY) {
        sum += (double)m_exp((T)(x - m));
      }
    }
  }
  red[grp][lane] = make_double2(m, sum);
  __syncthreads();
  if (grp == 0) {
    double M = -INFINITY, S = 0.0;
    for (int g = 0; g < G; ++g) {
      const double2 v = red[g][lane];
      if (v.x == -INFINITY) continue;
      if (v.x > M) {
        S = S * exp(M - v.x) + v.y;
        M = v.x;
      } else {
        S += v.y * exp(v.x - M);
      }
    }
    part[(gid * nchunks + c) * LT + lane] = make_double2(M, S);
  }
}

template <typename T, int LT>
__global__ void __launch_bounds__(256) k_softmax_finish(SoftArgs a, int64_t nchunks,
                                                        const double2 *__restrict__ part) {
  constexpr int G = 256 / LT;
  __shared__ double sM[LT], sInv[LT];
  const int64_t c = blockIdx.x % nchunks, gid = blockIdx.x / nchunks;
  const int64_t o = gid / a.lblocks, lb = gid % a.lblocks;
  const int lane = (LT == 1) ? 0 : (int)(threadIdx.x % LT);
  const int grp = (LT == 1) ? (int)threadIdx.x : (int)(threadIdx.x / LT);
  const int64_t l = lb * LT + lane;
  const bool lane_ok = l < a.L;
  if (grp == 0) {
    double M = -INFINITY, S = 0.0;
    for (int64_t q = 0; q < nchunks; ++q) {
      const double2 v = part[(gid * nchunks + q) * LT + lane];
      if (v.x == -INFINITY) continue;
      if (v.x > M) {
        S = S * exp(M - v.x) + v.y;
        M = v.x;
      } else {
        S += v.y * exp(v.x - M);
      }
    }
    sM[lane] = M;
    sInv[lane] = 1.0 / S;
  }
  __syncthreads();
  if (!lane_ok) return;
  const T Mt = (T)sM[lane];
  const T inv = (T)sInv[lane];
  const int64_t r0 = c * a.chunk;
  int64_t r1 = r0 + a.chunk;
  if (r1 > a.R) r1 = a.R;
  const T *in = static_cast<const T *>(a.in) + o * a.so + l * a.sl;
  T *out = static_cast<T *>(a.out) + o * a.oo + l * a.ol;
#pragma unroll 8
  for (int64_t r = r0 + grp; r < r1; r += G) out[r * a.orr] = m_exp(in[r * a.sr] - Mt) * inv;
}

// ---- two passes over wide, contiguous lane blocks ---------------------------
// For a softmax along a strided axis whose lanes are contiguous (the row
// softmax of a column-major matrix): each thread owns VL adjacent lanes read
// with one 16-byte load per step, a CTA owns 256*VL lanes, so every step of
// the chunk is a 4 KB contiguous read.  Pass 1 writes per-lane online (max,
// sum) partials per chunk, a small kernel merges each lane's partials, and
// pass 2 writes exp(x - max) / sum.  Chunks are sized to give every SM about
// eight CTAs even when there are few lane blocks.
template <typename T>
__device__ __forceinline__ void online_add(double &m, double &s, T x) {
  const double xd = (double)x;
  if (xd > m) {
    s = s * exp(m - xd) + 1.0;
    m = xd;
  } else if (xd != -INFINITY) {
    s += (double)m_exp((T)(xd - m));
  }
}

template <typename T, int VL>
__global__ void __launch_bounds__(256) k_softmax_wide_partials(SoftArgs a, int64_t nchunks, int64_t lblocks,
                                                               double2 *__restrict__ part) {
  const int64_t c = blockIdx.x % nchunks, gid = blockIdx.x / nchunks;
  const int64_t o = gid / lblocks, lb = gid % lblocks;
  const int64_t l0 = (lb * 256 + threadIdx.x) * VL;
  if (l0 >= a.L) return;
  const int64_t r0 = c * a.chunk;
  int64_t r1 = r0 + a.chunk;
  if (r1 > a.R) r1 = a.R;
  const T *in = static_cast<const T *>(a.in) + o * a.so + l0;
  // online (max, sum) in the tensor dtype, four steps at a time: one rescale
  // exp per batch and one exp per element, no divergent branches
  T m[VL], s[VL];
#pragma unroll
  for (int k = 0; k < VL; ++k) {
    m[k] = lowest_of<T>();
    s[k] = T(0);
  }
  int64_t r = r0;
  for (; r + 3 < r1; r += 4) {
    Vec<T, VL> x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = *reinterpret_cast<const Vec<T, VL> *>(in + (r + u) * a.sr);
#pragma unroll
    for (int k = 0; k < VL; ++k) {
      const T mb = m_max(m_max(x[0].v[k], x[1].v[k]), m_max(x[2].v[k], x[3].v[k]));
      const T mn = m_max(m[k], mb);
      if (mn == lowest_of<T>()) continue;  // all -inf so far
      T acc = (m[k] == lowest_of<T>()) ? T(0) : s[k] * m_exp(m[k] - mn);
#pragma unroll
      for (int u = 0; u < 4; ++u) acc += m_exp(x[u].v[k] - mn);
      s[k] = acc;
      m[k] = mn;
    }
  }
  for (; r < r1; ++r) {
    const Vec<T, VL> x = *reinterpret_cast<const Vec<T, VL> *>(in + r * a.sr);
#pragma unroll
    for (int k = 0; k < VL; ++k) {
      const T mn = m_max(m[k], x.v[k]);
      if (mn == lowest_of<T>()) continue;
      const T acc = (m[k] == lowest_of<T>()) ? T(0) : s[k] * m_exp(m[k] - mn);
      s[k] = acc + m_exp(x.v[k] - mn);
      m[k] = mn;
    }
  }
  double2 *dst = part + (gid * nchunks + c) * (int64_t)(256 * VL) + threadIdx.x * VL;
#pragma unroll
  for (int k = 0; k < VL; ++k)
    dst[k] = make_double2(m[k] == lowest_of<T>() ? -INFINITY : (double)m[k], (double)s[k]);
}

// Merges each lane's per-chunk (max, sum) partials into one pair.  A CTA
// takes 8 consecutive lane slots (a warp reads four 128-byte runs of
// partials) and splits the chunks over 32 thread groups; the group results
// are then combined in group order.  The chain of dependent exp() calls per
// thread is nchunks / 32 long.
__device__ __forceinline__ void merge_pair(double &mm, double &ss, double2 v) {
  if (v.x == -INFINITY) return;
  if (v.x > mm) {
    ss = ss * exp(mm - v.x) + v.y;
    mm = v.x;
  } else {
    ss += v.y * exp(v.x - mm);
  }
}

__global__ void __launch_bounds__(256) k_softmax_wide_merge(int64_t nchunks, int64_t nslots, int64_t slots_per_group,
                                                            const double2 *__restrict__ part,
                                                            double2 *__restrict__ stat) {
  constexpr int NSL = 8, NCG = 32;
  __shared__ double2 red[NCG][NSL];
  const int sl = threadIdx.x % NSL, cg = threadIdx.x / NSL;
  const int64_t i = (int64_t)blockIdx.x * NSL + sl;
  double mm = -INFINITY, ss = 0.0;
  if (i < nslots) {
    const int64_t gid = i / slots_per_group, w = i - gid * slots_per_group;
    const double2 *p = part + gid * nchunks * slots_per_group + w;
    int64_t q = cg;
    for (; q + 3 * NCG < nchunks; q += 4 * NCG) {  // four independent loads per round
      const double2 v0 = p[q * slots_per_group], v1 = p[(q + NCG) * slots_per_group];
      const double2 v2 = p[(q + 2 * NCG) * slots_per_group], v3 = p[(q + 3 * NCG) * slots_per_group];
      merge_pair(mm, ss, v0);
      merge_pair(mm, ss, v1);
      merge_pair(mm, ss, v2);
      merge_pair(mm, ss, v3);
    }
    for (; q < nchunks; q += NCG) merge_pair(mm, ss, p[q * slots_per_group]);
  }
  red[cg][sl] = make_double2(mm, ss);
  __syncthreads();
  if (cg == 0 && i < nslots) {
    double M = -INFINITY, S = 0.0;
    for (int g = 0; g < NCG; ++g) merge_pair(M, S, red[g][sl]);
    stat[i] = make_double2(M, S);
  }
}

template <typename T, int VL>
__global__ void __launch_bounds__(256) k_softmax_wide_finish(SoftArgs a, int64_t nchunks, int64_t lblocks,
                                                             const double2 *__restrict__ stat) {
  const int64_t c = blockIdx.x % nchunks, gid = blockIdx.x / nchunks;
  const int64_t o = gid / lblocks, lb = gid % lblocks;
  const int64_t l0 = (lb * 256 + threadIdx.x) * VL;
  if (l0 >= a.L) return;
  T M[VL], inv[VL];
#pragma unroll
  for (int k = 0; k < VL; ++k) {
    const double2 v = stat[gid * (int64_t)(256 * VL) + threadIdx.x * VL + k];
    M[k] = (T)v.x;
    inv[k] = (T)(1.0 / v.y);
  }
  const int64_t r0 = c * a.chunk;
  int64_t r1 = r0 + a.chunk;
  if (r1 > a.R) r1 = a.R;
  const T *in = static_cast<const T *>(a.in) + o * a.so + l0;
  T *out = static_cast<T *>(a.out) + o * a.oo + l0;
  int64_t r = r0;
  for (; r + 3 < r1; r += 4) {
    Vec<T, VL> x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = *reinterpret_cast<const Vec<T, VL> *>(in + (r + u) * a.sr);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      Vec<T, VL> y;
#pragma unroll
      for (int k = 0; k < VL; ++k) y.v[k] = m_exp(x[u].v[k] - M[k]) * inv[k];
      *reinterpret_cast<Vec<T, VL> *>(out + (r + u) * a.orr) = y;
    }
  }
  for (; r < r1; ++r) {
    const Vec<T, VL> x = *reinterpret_cast<const Vec<T, VL> *>(in + r * a.sr);
    Vec<T, VL> y;
#pragma unroll
    for (int k = 0; k < VL; ++k) y.v[k] = m_exp(x.v[k] - M[k]) * inv[k];
    *reinterpret_cast<Vec<T, VL> *>(out + r * a.orr) = y;
  }
}

template <typename T>
static acd_status launch_softmax_wide(acd_ctx *ctx, SoftArgs a, cudaStream_t s) {
  constexpr int VL = 16 / sizeof(T);
  const int64_t lblocks = (a.L + 256 * VL - 1) / (256 * VL);
  const int64_t groups = lblocks * a.O;
  // chunks: about 8 CTAs per SM, at least 64 steps each
  int64_t nchunks = ((int64_t)ctx->sm_count * 8 + groups - 1) / groups;
  const int64_t max_chunks = (a.R + 63) / 64;
  if (nchunks > max_chunks) nchunks = max_chunks;
  if (nchunks < 1) nchunks = 1;
  a.chunk = (a.R + nchunks - 1) / nchunks;
  nchunks = (a.R + a.chunk - 1) / a.chunk;
  const int64_t grid = groups * nchunks;
  if (grid > INT32_MAX) return fail(ACD_ERR_UNSUPPORTED, "softmax: grid too large");
  const int64_t slots = 256 * VL, nslots = groups * slots;
  const size_t pbytes = sizeof(double2) * (size_t)grid * slots;
  const size_t sbytes = sizeof(double2) * (size_t)nslots;
  void *scratch;
  ACD_TRY(get_scratch(ctx, pbytes + sbytes, s, &scratch));
  double2 *part = static_cast<double2 *>(scratch);
  double2 *stat = reinterpret_cast<double2 *>(static_cast<char *>(scratch) + pbytes);
  k_softmax_wide_partials<T, VL><<<(int)grid, 256, 0, s>>>(a, nchunks, lblocks, part);
  k_softmax_wide_merge<<<(int)((nslots + 7) / 8), 256, 0, s>>>(nchunks, nslots, slots, part, stat);
  k_softmax_wide_finish<T, VL><<<(int)grid, 256, 0, s>>>(a, nchunks, lblocks, stat);
  return ACD_OK;
}

// ---- one HBM read through L2: statistics and apply as ordered tickets --------
// For the same views as the wide kernels (contiguous lanes, 16-byte aligned).
// The lanes are cut into groups of one warp width (GW = 32 * VL lanes, a
// 512-byte row per step) and the steps into chunks.  Work items are:
//   A(g, c): the online (max, sum) of group g over chunk c, written as a
//            per-lane partial; the CTA that completes group g's last chunk
//            merges the partials into (M, 1/S) per lane and flags the group;
//   B(g, c): exp(x - M) * (1/S) over chunk c of group g.
// One persistent launch takes items by a global ticket counter in the order
//   A(0,*) ; A(1,*) ; ... A(lag,*) B(0,*) ; A(lag+1,*) B(1,*) ; ...
// so the A items of a group run `lag` groups before its B items, and the
// input those B items re-read was read by the A items a moment earlier: it
// is still in L2 (A reads mark it evict_last, B reads and the output stores
// evict_first), so HBM sees the input once and the output once.  lag is
// chosen so that the groups between an A and its B, plus the items in
// flight, stay well inside L2.  A B item waits (bounded, 1 s by
// %globaltimer, status code 4 when it expires) until its group is flagged;
// every A item it waits for was taken earlier by a running CTA and never
// waits itself, so the wait always ends.  Counters are zero at rest: the last
// B item of a group clears the group's counters and the last CTA to leave
// clears the ticket counter.
struct SoftL2Args {
  const void *in;
  void *out;
  int64_t L, R, O;
  int64_t sr, so, orr, oo;  // lanes are contiguous (stride 1) on both sides
  int64_t lgroups;          // lane groups per outer index
  int64_t ng;               // lgroups * O
  int64_t nchunks, chunk;   // chunks per group, steps per chunk (a multiple of 8)
  int64_t lag;              // groups between A(g) and B(g)
  int64_t total;            // tickets: (ng + lag) * 2 * nchunks
  unsigned int *cnt;        // [3 * ng + 2]: A done, ready, B done per group; ticket; CTAs done
  void *part;               // [ng][nchunks][GW] (m, s) pairs in T
  void *stat;               // [ng][GW] (M, 1/S) pairs in T
  Control *control;
};

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

template <typename T>
__device__ __forceinline__ Vec<T, 16 / sizeof(T)> ld_hint(const T *p, uint64_t pol) {
  Vec<T, 16 / sizeof(T)> v;
  if constexpr (sizeof(T) == 4)
    asm volatile("ld.global.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.v[0]), "=f"(v.v[1]), "=f"(v.v[2]), "=f"(v.v[3])
                 : "l"(p), "l"(pol));
  else
    asm volatile("ld.global.L2::cache_hint.v2.f64 {%0, %1}, [%2], %3;"
                 : "=d"(v.v[0]), "=d"(v.v[1])
                 : "l"(p), "l"(pol));
  return v;
}

template <typename T>
__device__ __forceinline__ void st_hint(T *p, const Vec<T, 16 / sizeof(T)> &v, uint64_t pol) {
  if constexpr (sizeof(T) == 4)
    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "f"(v.v[0]), "f"(v.v[1]),
                 "f"(v.v[2]), "f"(v.v[3]), "l"(pol)
                 : "memory");
  else
    asm volatile("st.global.L2::cache_hint.v2.f64 [%0], {%1, %2}, %3;" ::"l"(p), "d"(v.v[0]), "d"(v.v[1]), "l"(pol)
                 : "memory");
}

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int *p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned int *p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// A pair of T read at L2 (never a stale L1 line: the pairs are written by
// other CTAs of the same launch).
template <typename T>
__device__ __forceinline__ Vec<T, 2> ld_pair_cg(const Vec<T, 2> *p) {
  Vec<T, 2> r;
  if constexpr (sizeof(T) == 4) {
    const float2 v = __ldcg(reinterpret_cast<const float2 *>(p));
    r.v[0] = v.x;
    r.v[1] = v.y;
  } else {
    const double2 v = __ldcg(reinterpret_cast<const double2 *>(p));
    r.v[0] = v.x;
    r.v[1] = v.y;
  }
  return r;
}

// (m, s) of one lane: m the maximum, s = sum exp(x - m); merged in double.
__device__ __forceinline__ void merge_ms(double &M, double &S, double m, double s) {
  if (m == -INFINITY) return;
  if (m > M) {
    S = S * exp(M - m) + s;
    M = m;
  } else {
    S += s * exp(m - M);
  }
}

template <typename T, int U>
__global__ void __launch_bounds__(256, sizeof(T) == 4 ? 3 : 2) k_softmax_l2(SoftL2Args a) {
  constexpr int VL = 16 / sizeof(T);
  constexpr int GW = 32 * VL;
  using P = Vec<T, 2>;  // (m, s) or (M, 1/S)
  __shared__ double red_m[8][GW], red_s[8][GW];
  __shared__ int64_t s_ticket;
  __shared__ int s_last;
  const int warp = threadIdx.x / 32, lane32 = threadIdx.x % 32;
  const int64_t per_block = 2 * a.nchunks;
  const int64_t wsteps = a.chunk / 8;  // steps per warp in an item
  const uint64_t keep = policy_evict_last(), drop = policy_evict_first();
  P *part = static_cast<P *>(a.part);
  P *stat = static_cast<P *>(a.stat);
  unsigned int *cntA = a.cnt, *ready = a.cnt + a.ng, *cntB = a.cnt + 2 * a.ng;
  unsigned int *ticket = a.cnt + 3 * a.ng, *done = ticket + 1;

  if (threadIdx.x == 0) s_ticket = (int64_t)atomicAdd(ticket, 1u);
  __syncthreads();
  int64_t t = s_ticket;
  while (t < a.total) {
    const int64_t blk = t / per_block, slot = t % per_block;
    const bool is_a = slot < a.nchunks;
    const int64_t g = is_a ? blk : blk - a.lag;
    const int64_t c = is_a ? slot : slot - a.nchunks;
    __syncthreads();  // s_ticket, s_last and red_* reuse
    // the next ticket is taken now, so its round trip overlaps this item (a
    // CTA holds at most one ticket it has not started; the smallest
    // unfinished ticket is always some CTA's current item, so work proceeds)
    unsigned int next = 0u;
    if (threadIdx.x == 0) next = atomicAdd(ticket, 1u);
    if (g >= 0 && g < a.ng) {
      const int64_t o = g / a.lgroups, lg = g % a.lgroups;
      const int64_t l0 = lg * GW + (int64_t)lane32 * VL;  // first lane of this thread
      const bool lane_ok = l0 < a.L;                     // L is a multiple of VL
      int64_t r0 = c * a.chunk + (int64_t)warp * wsteps;
      int64_t r1 = r0 + wsteps;
      if (r1 > a.R) r1 = a.R;
      const T *in = static_cast<const T *>(a.in) + o * a.so + l0;
      if (is_a) {
        // ---- A: online (max, sum) in the tensor dtype, U steps per batch
        T m[VL], sm[VL];
#pragma unroll
        for (int k = 0; k < VL; ++k) {
          m[k] = lowest_of<T>();
          sm[k] = T(0);
        }
        if (lane_ok) {
          int64_t r = r0;
          for (; r + U - 1 < r1; r += U) {
            Vec<T, VL> x[U];
#pragma unroll
            for (int u = 0; u < U; ++u) x[u] = ld_hint(in + (r + u) * a.sr, keep);
#pragma unroll
            for (int k = 0; k < VL; ++k) {
              T mb = x[0].v[k];
#pragma unroll
              for (int u = 1; u < U; ++u) mb = m_max(mb, x[u].v[k]);
              const T mn = m_max(m[k], mb);
              if (mn == lowest_of<T>()) continue;  // all -inf so far
              T acc = (m[k] == lowest_of<T>()) ? T(0) : sm[k] * m_exp(m[k] - mn);
#pragma unroll
              for (int u = 0; u < U; ++u) acc += m_exp(x[u].v[k] - mn);
              sm[k] = acc;
              m[k] = mn;
            }
          }
          for (; r < r1; ++r) {
            const Vec<T, VL> x = ld_hint(in + r * a.sr, keep);
#pragma unroll
            for (int k = 0; k < VL; ++k) {
              const T mn = m_max(m[k], x.v[k]);
              if (mn == lowest_of<T>()) continue;
              const T acc = (m[k] == lowest_of<T>()) ? T(0) : sm[k] * m_exp(m[k] - mn);
              sm[k] = acc + m_exp(x.v[k] - mn);
              m[k] = mn;
            }
          }
        }
#pragma unroll
        for (int k = 0; k < VL; ++k) {
          red_m[warp][lane32 * VL + k] = m[k] == lowest_of<T>() ? -INFINITY : (double)m[k];
          red_s[warp][lane32 * VL + k] = (double)sm[k];
        }
        __syncthreads();
        // the eight warps' pairs of a lane -> the item's partial (in T)
        P *dst = part + (g * a.nchunks + c) * GW;
        for (int i = threadIdx.x; i < GW; i += blockDim.x) {
          double M = -INFINITY, S = 0.0;
          for (int w = 0; w < 8; ++w) merge_ms(M, S, red_m[w][i], red_s[w][i]);
          P pr;
          pr.v[0] = M == -INFINITY ? lowest_of<T>() : (T)M;
          pr.v[1] = (T)S;
          dst[i] = pr;
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = (atomicAdd(&cntA[g], 1u) == (unsigned int)(a.nchunks - 1));
        __syncthreads();
        if (s_last) {
          // ---- the group's last A item: merge all chunk partials per lane
          __threadfence();
          for (int i = threadIdx.x; i < GW; i += blockDim.x) {
            const P *src = part + g * a.nchunks * GW + i;
            double M = -INFINITY;
            for (int64_t q = 0; q < a.nchunks; ++q) {
              const P v = ld_pair_cg(src + q * GW);
              if (v.v[0] != lowest_of<T>()) M = fmax(M, (double)v.v[0]);
            }
            double S = 0.0;
            if (M != -INFINITY)
              for (int64_t q = 0; q < a.nchunks; ++q) {
                const P v = ld_pair_cg(src + q * GW);
                if (v.v[0] != lowest_of<T>()) S += (double)v.v[1] * exp((double)v.v[0] - M);
              }
            P st;
            st.v[0] = M == -INFINITY ? lowest_of<T>() : (T)M;
            st.v[1] = (T)(1.0 / S);
            stat[g * GW + i] = st;
          }
          __threadfence();
          __syncthreads();
          if (threadIdx.x == 0) st_release_u32(&ready[g], 1u);
        }
      } else {
        // ---- B: the first loads go out before the wait for the group's
        // statistics (they do not depend on them), then write
        Vec<T, VL> x[U];
        const bool first = lane_ok && r0 + U - 1 < r1;
        if (first) {
#pragma unroll
          for (int u = 0; u < U; ++u) x[u] = ld_hint(in + (r0 + u) * a.sr, drop);
        }
        if (threadIdx.x == 0) {
          if (ld_acquire_u32(&ready[g]) == 0u) {
            const uint64_t t0 = global_timer_ns();
            while (ld_acquire_u32(&ready[g]) == 0u) {
              if (global_timer_ns() - t0 > 1000000000ull) {
                raise_status(a.control, 4, (int32_t)(g & 0x7fffffff));
                break;
              }
              __nanosleep(200);
            }
          }
        }
        __syncthreads();
        T M[VL], inv[VL];
#pragma unroll
        for (int k = 0; k < VL; ++k) {
          const P st = lane_ok ? ld_pair_cg(stat + g * GW + lane32 * VL + k) : P{};
          M[k] = st.v[0];
          inv[k] = st.v[1];
        }
        T *out = static_cast<T *>(a.out) + o * a.oo + l0;
        if (lane_ok) {
          int64_t r = r0;
          if (first) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
              Vec<T, VL> y;
#pragma unroll
              for (int k = 0; k < VL; ++k) y.v[k] = m_exp(x[u].v[k] - M[k]) * inv[k];
              st_hint(out + (r0 + u) * a.orr, y, drop);
            }
            r += U;
          }
          for (; r + U - 1 < r1; r += U) {
#pragma unroll
            for (int u = 0; u < U; ++u) x[u] = ld_hint(in + (r + u) * a.sr, drop);
#pragma unroll
            for (int u = 0; u < U; ++u) {
              Vec<T, VL> y;
#pragma unroll
              for (int k = 0; k < VL; ++k) y.v[k] = m_exp(x[u].v[k] - M[k]) * inv[k];
              st_hint(out + (r + u) * a.orr, y, drop);
            }
          }
          for (; r < r1; ++r) {
            const Vec<T, VL> x = ld_hint(in + r * a.sr, drop);
            Vec<T, VL> y;
#pragma unroll
            for (int k = 0; k < VL; ++k) y.v[k] = m_exp(x.v[k] - M[k]) * inv[k];
            st_hint(out + r * a.orr, y, drop);
          }
        }
        __syncthreads();
        if (threadIdx.x == 0 && atomicAdd(&cntB[g], 1u) == (unsigned int)(a.nchunks - 1)) {
          // every B item of the group has read its statistics: clear the counters
          cntA[g] = 0u;
          ready[g] = 0u;
          cntB[g] = 0u;
        }
      }
    }
    if (threadIdx.x == 0) s_ticket = (int64_t)next;
    __syncthreads();
    t = s_ticket;
  }
  if (threadIdx.x == 0 && atomicAdd(done, 1u) == gridDim.x - 1) {
    *ticket = 0u;  // every CTA has taken its last ticket
    *done = 0u;
  }
}

// Tuning of k_softmax_l2: items of 128 KB and a lag of about 96 MB of input
// between a group's A and B items.  Sweeps over 32-512 KB items and 8-96 MB
// lags on 65536x4096 float32: 32 KB / 8 MB took 1.9 ms (per-item latency:
// ticket, flag and statistics round trips), 128 KB / 96 MB 0.56 ms.  A
// shorter lag keeps more of the re-read in L2 but leaves B items waiting on
// groups whose A items are still in flight (444 CTAs x 128 KB = 57 MB are
// in flight at once); at 48 MB ncu counted 1.79 GB of DRAM reads for the
// 1.07 GB input, i.e. a third of the re-read hit L2.
template <typename T>
static acd_status launch_softmax_l2(acd_ctx *ctx, SoftArgs sa, cudaStream_t s) {
  constexpr int VL = 16 / sizeof(T);
  constexpr int64_t GW = 32 * VL;
  constexpr int64_t row_bytes = GW * sizeof(T);  // 512
  SoftL2Args a{};
  a.in = sa.in;
  a.out = sa.out;
  a.L = sa.L;
  a.R = sa.R;
  a.O = sa.O;
  a.sr = sa.sr;
  a.so = sa.so;
  a.orr = sa.orr;
  a.oo = sa.oo;
  a.lgroups = (sa.L + GW - 1) / GW;
  a.ng = a.lgroups * sa.O;
  int64_t chunk = (128 * 1024) / row_bytes;  // 256 steps
  if (chunk > sa.R) chunk = (sa.R + 7) / 8 * 8;
  a.chunk = chunk;
  a.nchunks = (sa.R + chunk - 1) / chunk;
  const int64_t group_bytes = a.nchunks * chunk * row_bytes;
  a.lag = (96ll << 20) / group_bytes;
  if (a.lag < 1) a.lag = 1;
  if (a.lag > a.ng) a.lag = a.ng;
  a.total = (a.ng + a.lag) * 2 * a.nchunks;
  if (a.total >= (1ll << 31) || a.ng >= (1ll << 29)) return fail(ACD_ERR_UNSUPPORTED, "softmax: too many items");
  ACD_TRY(get_counters(ctx, (size_t)(3 * a.ng + 2), s, &a.cnt));
  const size_t pbytes = sizeof(T) * 2 * (size_t)(a.ng * a.nchunks * GW);
  const size_t sbytes = sizeof(T) * 2 * (size_t)(a.ng * GW);
  void *scratch;
  ACD_TRY(get_scratch(ctx, pbytes + sbytes, s, &scratch));
  a.part = scratch;
  a.stat = static_cast<char *>(scratch) + pbytes;
  a.control = ctx->control;
  constexpr int U = 8;
  const int grid = persistent_grid(ctx, k_softmax_l2<T, U>, 256, 0, a.total);
  k_softmax_l2<T, U><<<grid, 256, 0, s>>>(a);
  return ACD_OK;
}

// ---- one read through TMA: a cluster holds a lane block's whole row ---------
// For lanes contiguous in memory (the row softmax of a column-major matrix)
// whose R steps x 128 bytes fit the shared memory of a cluster of up to 16
// CTAs.  Each CTA loads its chunk of steps (a 128-byte lane block per step)
// with bulk tensor loads; every byte of the chunk is in flight at once.  Two
// passes over shared memory give each lane's local maximum m_q and local sum
// s_q = sum exp(x - m_q) (float64); the (m_q, s_q) pairs are exchanged once
// over distributed shared memory and combined in rank order,
// M = max m_q, S = sum s_q * exp(m_q - M).  A third pass writes
// exp(x - M) * (1/S) in place and bulk tensor stores write the chunk back.
// HBM sees one read and one write per element.  Shared-memory passes use
// 16-byte vectors: thread t covers vector slot t % 8 of each 128-byte row and
// steps t / 8, t / 8 + 32, ...  Lanes past L and steps past R are zero-filled
// by the loads and clipped by the stores.  The load wait is bounded (status
// code 3 when it expires).
struct SoftTmaArgs {
  int64_t lblocks;
  int64_t groups;  // lblocks * O
  int64_t gstep;   // coprime with groups: cluster c takes group (c * gstep) % groups
  int64_t R;
  int ch;  // steps per CTA, a multiple of bs
  int bs;  // steps per TMA box
  Control *control;
};

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

template <typename T>
__global__ void __launch_bounds__(256) k_softmax_tma(const __grid_constant__ CUtensorMap map_in,
                                                     const __grid_constant__ CUtensorMap map_out, SoftTmaArgs a) {
  constexpr int LT = 128 / (int)sizeof(T);  // lanes per 128-byte row
  constexpr int V = 16 / (int)sizeof(T);    // lanes per 16-byte vector
  constexpr int SG = 32;                    // step groups (256 threads / 8 vector slots)
  extern __shared__ unsigned char smem_raw[];
  T *tile = reinterpret_cast<T *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t bar;
  __shared__ double wred[8][LT];      // per-warp lane partials
  __shared__ double2 stat[LT];        // this CTA's (m_q, s_q), read by the cluster
  __shared__ double2 xch[16][LT];     // every rank's (m_q, s_q)
  __shared__ T lane_m[LT], lane_inv[LT];

  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  // (lane block, o) of this cluster: clusters that run at the same time take
  // lane blocks gstep apart, spreading their reads over each row
  const int64_t gid = (int64_t)(((uint64_t)(blockIdx.x / C) * (uint64_t)a.gstep) % (uint64_t)a.groups);  // < 2^62
  const int64_t o = gid / a.lblocks, lb = gid % a.lblocks;
  const int tid = threadIdx.x, wl = tid & 31, w = tid >> 5;
  const int slot = tid & 7, sg = tid >> 3;
  const int64_t r0 = (int64_t)rank * a.ch;
  const int64_t left = a.R - r0;
  const int nv = left <= 0 ? 0 : (left < a.ch ? (int)left : a.ch);  // steps of this CTA
  const int nbox = (nv + a.bs - 1) / a.bs;
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (tid == 0 && nbox > 0) {
    mbar_arrive_expect_tx(&bar, (uint32_t)nbox * (uint32_t)a.bs * 128u);
    for (int b = 0; b < nbox; ++b)
      tma_load_3d(tile + (size_t)b * a.bs * LT, &map_in, &bar, (int)(lb * LT), (int)(r0 + (int64_t)b * a.bs), (int)o);
  }
  bool landed = true;
  if (nbox > 0) landed = mbar_wait_bounded(&bar, 0, 1000000000ull);
  if (!landed) raise_status(a.control, 3, (int32_t)blockIdx.x);
  const Vec<T, V> *tv = reinterpret_cast<const Vec<T, V> *>(tile) + slot;  // row k at tv[k * 8]

  // pass A: lane maxima
  T m[V];
#pragma unroll
  for (int v = 0; v < V; ++v) m[v] = lowest_of<T>();
#pragma unroll 4
  for (int k = sg; k < nv; k += SG) {
    const Vec<T, V> x = tv[k * 8];
#pragma unroll
    for (int v = 0; v < V; ++v) m[v] = m_max(m[v], x.v[v]);
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    m[v] = m_max(m[v], __shfl_xor_sync(0xffffffffu, m[v], 8));
    m[v] = m_max(m[v], __shfl_xor_sync(0xffffffffu, m[v], 16));
    if (wl < 8) wred[w][slot * V + v] = (double)m[v];
  }
  __syncthreads();
  if (tid < LT) {
    T mm = lowest_of<T>();
    for (int q = 0; q < 8; ++q) mm = m_max(mm, (T)wred[q][tid]);
    lane_m[tid] = mm;
  }
  __syncthreads();
#pragma unroll
  for (int v = 0; v < V; ++v) m[v] = lane_m[slot * V + v];

  // pass B: local sums of exp(x - m_q), float64
  double s[V];
#pragma unroll
  for (int v = 0; v < V; ++v) s[v] = 0.0;
#pragma unroll 4
  for (int k = sg; k < nv; k += SG) {
    const Vec<T, V> x = tv[k * 8];
#pragma unroll
    for (int v = 0; v < V; ++v) s[v] += (double)m_exp(x.v[v] - m[v]);
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    s[v] += __shfl_xor_sync(0xffffffffu, s[v], 8);
    s[v] += __shfl_xor_sync(0xffffffffu, s[v], 16);
    if (wl < 8) wred[w][slot * V + v] = s[v];
  }
  __syncthreads();
  if (tid < LT) {
    double ss = 0.0;
    for (int q = 0; q < 8; ++q) ss += wred[q][tid];
    const T mq = lane_m[tid];
    stat[tid] = mq == lowest_of<T>() ? make_double2(-INFINITY, 0.0) : make_double2((double)mq, ss);
  }
  cluster.sync();
  // remote reads spread over the threads: entry i is rank i / LT, lane i % LT
  for (int i = tid; i < C * LT; i += 256) xch[i / LT][i % LT] = cluster.map_shared_rank(stat, i / LT)[i % LT];
  __syncthreads();
  cluster_arrive_relaxed();  // this CTA is done reading its peers
  if (tid < LT) {
    double M = -INFINITY;
    for (int q = 0; q < C; ++q) M = fmax(M, xch[q][tid].x);
    double S = 0.0;
    for (int q = 0; q < C; ++q) {
      const double2 v = xch[q][tid];
      if (v.x != -INFINITY) S += v.y * exp(v.x - M);
    }
    lane_m[tid] = (T)M;
    lane_inv[tid] = (T)(1.0 / S);
  }
  __syncthreads();
  T inv[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    m[v] = lane_m[slot * V + v];
    inv[v] = lane_inv[slot * V + v];
  }

  // pass C: exp(x - M) / S in place, then store
  Vec<T, V> *tw = reinterpret_cast<Vec<T, V> *>(tile) + slot;
#pragma unroll 4
  for (int k = sg; k < nv; k += SG) {
    Vec<T, V> x = tw[k * 8];
#pragma unroll
    for (int v = 0; v < V; ++v) x.v[v] = m_exp(x.v[v] - m[v]) * inv[v];
    tw[k * 8] = x;
  }
  fence_proxy_async_smem();
  __syncthreads();
  if (tid == 0) {
    if (nbox > 0) {
      for (int b = 0; b < nbox; ++b)
        tma_store_3d(&map_out, tile + (size_t)b * a.bs * LT, (int)(lb * LT), (int)(r0 + (int64_t)b * a.bs), (int)o);
      bulk_commit();
      bulk_wait_read<0>();  // the stores have read the tile before the CTA's shared memory is released
    }
    if (!landed) mbar_wait_bounded(&bar, 0, 1000000000ull);
  }
  cluster_wait();  // no CTA leaves while a peer may still read its stat
}

// Launches k_softmax_tma when the view suits it; false (nothing launched)
// otherwise.
template <typename T>
static bool launch_softmax_tma(acd_ctx *ctx, const SoftArgs &sa, cudaStream_t s) {
  constexpr int LT = 128 / (int)sizeof(T);
  constexpr int64_t eb = sizeof(T);
  if (sa.sl != 1 || sa.ol != 1 || sa.L < LT) return false;
  if ((sa.sr * eb) % 16 || (sa.orr * eb) % 16) return false;
  if (sa.O > 1 && ((sa.so * eb) % 16 || (sa.oo * eb) % 16)) return false;
  if ((reinterpret_cast<uintptr_t>(sa.in) | reinterpret_cast<uintptr_t>(sa.out)) & 15) return false;
  if (sa.L >= (1ll << 31) || sa.R >= (1ll << 31) || sa.O >= (1ll << 31)) return false;
  // cluster size: the smallest that brings a CTA's chunk under 72 KB (three
  // CTAs per SM), at most 8.  16-CTA clusters with 32 KB chunks measured
  // slower on 65536x4096 float32 (0.71 vs 0.60 ms): their barrier waits grow
  // faster than the extra residency helps.
  int C = 1;
  while (C < 8 && ((sa.R + C - 1) / C) * 128 > 72 * 1024) C *= 2;
  int64_t ch = (sa.R + C - 1) / C;
  if (ch > 256) ch = (ch + 31) / 32 * 32;
  if (ch * 128 > 200 * 1024) return false;
  const int bs = ch <= 256 ? (int)ch : ch % 256 == 0 ? 256 : ch % 128 == 0 ? 128 : ch % 64 == 0 ? 64 : 32;
  SoftTmaArgs a;
  a.lblocks = (sa.L + LT - 1) / LT;
  a.groups = a.lblocks * sa.O;
  a.R = sa.R;
  a.ch = (int)ch;
  a.bs = bs;
  a.control = ctx->control;
  const int64_t groups = a.groups;
  // about as many clusters run at once as the shared memory of the SMs holds;
  // stepping by groups / that count puts them evenly across the lane blocks
  const int64_t per_sm = std::max<int64_t>(1, (200 * 1024) / (ch * 128 + 12 * 1024));
  int64_t step = groups / (((int64_t)ctx->sm_count * per_sm + C - 1) / C);
  if (step < 1) step = 1;
  while (std::gcd(step, groups) != 1) ++step;
  a.gstep = step;
  if (groups * C < ctx->sm_count || groups * C > INT32_MAX) return false;  // too few CTAs to fill the GPU
  CUtensorMap mi, mo;
  const int64_t d[3] = {sa.L, sa.R, sa.O};
  const int64_t si[2] = {sa.sr, sa.O > 1 ? sa.so : sa.sr * sa.R};
  const int64_t so[2] = {sa.orr, sa.O > 1 ? sa.oo : sa.orr * sa.R};
  const uint32_t box[3] = {(uint32_t)LT, (uint32_t)bs, 1};
  if (!encode_tensor_map_3d(&mi, sa.in, (int)eb, d, si, box, false, false)) return false;
  if (!encode_tensor_map_3d(&mo, sa.out, (int)eb, d, so, box, false, false)) return false;
  const size_t dyn = (size_t)ch * 128 + 1024;
  auto kern = k_softmax_tma<T>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess ||
      (C > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)) {
    cudaGetLastError();
    return false;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(groups * C), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, mi, mo, a) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

// ---- whole tensor ----------------------------------------------------------
template <typename T, int V, int U>
__global__ void __launch_bounds__(256) k_softmax_apply(T *__restrict__ out, const T *__restrict__ in, int64_t n,
                                                       const double *__restrict__ stats) {
  const T M = (T)stats[0];
  const T inv = (T)(1.0 / stats[1]);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  const int64_t nv = vec ? n / V : 0;
  const Vec<T, V> *iv = reinterpret_cast<const Vec<T, V> *>(in);
  Vec<T, V> *ov = reinterpret_cast<Vec<T, V> *>(out);
  int64_t v0 = tid;
  for (; v0 + (int64_t)(U - 1) * nth < nv; v0 += nth * U) {  // U full vectors: unguarded loads
    Vec<T, V> x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) x[u] = iv[v0 + (int64_t)u * nth];
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int k = 0; k < V; ++k) x[u].v[k] = m_exp(x[u].v[k] - M) * inv;
      ov[v0 + (int64_t)u * nth] = x[u];
    }
  }
  for (; v0 < nv; v0 += nth) {
    Vec<T, V> x = iv[v0];
#pragma unroll
    for (int k = 0; k < V; ++k) x.v[k] = m_exp(x.v[k] - M) * inv;
    ov[v0] = x;
  }
  for (int64_t i = nv * V + tid; i < n; i += nth) out[i] = m_exp(in[i] - M) * inv;
}

static bool split_axis_sm(const acd_desc *in, const acd_desc *out, int axis, int64_t &L, int64_t &R, int64_t &O,
                          int64_t *s_in, int64_t *s_out) {
  auto merge = [&](int d0, int d1, int64_t &n, int64_t &si, int64_t &so) -> bool {
    n = 1;
    si = 0;
    so = 0;
    bool first = true;
    int64_t ei = 0, eo = 0;
    for (int d = d0; d < d1; ++d) {
      if (in->shape[d] == 1) continue;
      if (first) {
        si = in->stride[d];
        so = out->stride[d];
        ei = si * in->shape[d];
        eo = so * in->shape[d];
        n = in->shape[d];
        first = false;
      } else {
        if (in->stride[d] != ei || out->stride[d] != eo) return false;
        n *= in->shape[d];
        ei = in->stride[d] * in->shape[d];
        eo = out->stride[d] * in->shape[d];
      }
    }
    return true;
  };
  if (!merge(0, axis, L, s_in[0], s_out[0])) return false;
  if (!merge(axis + 1, in->ndim, O, s_in[2], s_out[2])) return false;
  R = in->shape[axis];
  s_in[1] = in->stride[axis];
  s_out[1] = out->stride[axis];
  return true;
}

template <typename T, int LT>
static acd_status launch_softmax_two_pass(acd_ctx *ctx, SoftArgs a, cudaStream_t s) {
  a.lblocks = (a.L + LT - 1) / LT;
  const int64_t groups = a.lblocks * a.O;
  // chunks: enough CTAs to fill the GPU a few times, at least 256 steps each
  int64_t nchunks = ((int64_t)ctx->sm_count * 8 + groups - 1) / groups;
  const int64_t max_chunks = (a.R + 255) / 256;
  if (nchunks > max_chunks) nchunks = max_chunks;
  if (nchunks < 1) nchunks = 1;
  a.chunk = (a.R + nchunks - 1) / nchunks;
  nchunks = (a.R + a.chunk - 1) / a.chunk;
  const int64_t grid = groups * nchunks;
  if (grid > INT32_MAX) return fail(ACD_ERR_UNSUPPORTED, "softmax: grid too large");
  void *scratch;
  ACD_TRY(get_scratch(ctx, sizeof(double2) * (size_t)grid * LT, s, &scratch));
  double2 *part = static_cast<double2 *>(scratch);
  k_softmax_partials<T, LT><<<(int)grid, 256, 0, s>>>(a, nchunks, part);
  k_softmax_finish<T, LT><<<(int)grid, 256, 0, s>>>(a, nchunks, part);
  return ACD_OK;
}

template <typename T, int LT>
static acd_status launch_softmax_axis(acd_ctx *ctx, SoftArgs a, cudaStream_t s) {
  a.lblocks = (a.L + LT - 1) / LT;
  const int64_t groups = a.lblocks * a.O;
  // chunks that would not fit shared memory even split over 8 CTAs: two passes
  if (((a.R + 7) / 8) * (int64_t)LT * (int64_t)sizeof(T) > 160 * 1024) return launch_softmax_two_pass<T, LT>(ctx, a, s);
  // cluster size: enough CTAs to fill the GPU, chunks that fit shared memory
  const int64_t smem_target = 64 * 1024;
  const int64_t row_bytes = (int64_t)LT * sizeof(T);
  int C = 1;
  while (C < 8 && ((a.R + C - 1) / C) * row_bytes > smem_target) C *= 2;
  while (C < 8 && groups * C < (int64_t)ctx->sm_count * 4 && (a.R + 2 * C - 1) / (2 * C) >= 256 / LT) C *= 2;
  a.chunk = (a.R + C - 1) / C;
  int64_t cap = a.chunk;
  const int64_t smem_max = 160 * 1024;
  if (cap * row_bytes > smem_max) cap = smem_max / row_bytes;
  a.cap = cap;
  const size_t dyn = (size_t)cap * row_bytes;
  const int64_t grid = groups * C;
  if (grid > INT32_MAX) return fail(ACD_ERR_UNSUPPORTED, "softmax: grid too large");
  auto kern = k_softmax_axis<T, LT>;
  if (dyn > 48 * 1024) ACD_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = dyn;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ACD_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
  return ACD_OK;
}

}  // namespace acd

using namespace acd;

// Defined in reduce.cu: the online (max, sum) statistics of the whole tensor,
// written to ctx->control->stats[0..1].
namespace acd {
template <typename T>
acd_status softmax_stats(acd_ctx *ctx, const acd_desc *in, cudaStream_t s);
}

extern "C" {

acd_status acd_softmax(acd_ctx *ctx, const acd_desc *out, const acd_desc *in, int32_t axis, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_softmax: null context");
  ACD_TRY(check_desc(out, "out"));
  ACD_TRY(check_desc(in, "in"));
  if (!is_float(in->dtype) || out->dtype != in->dtype)
    return fail(ACD_ERR_DTYPE, "acd_softmax: float32/float64 input and output of one dtype required");
  if (out->ndim != in->ndim) return fail(ACD_ERR_SHAPE, "acd_softmax: output rank differs");
  for (int d = 0; d < in->ndim; ++d)
    if (out->shape[d] != in->shape[d]) return fail(ACD_ERR_SHAPE, "acd_softmax: output extent differs on axis %d", d);
  if (axis >= in->ndim && in->ndim > 0) return fail(ACD_ERR_AXIS, "acd_softmax: axis %d out of range", axis);
  const int64_t n = desc_numel(in);
  if (n == 0) return ACD_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f32 = in->dtype == ACD_FLOAT32;
  if (axis < 0 || in->ndim == 0) {
    if (!desc_is_contiguous(in) || !desc_is_contiguous(out))
      return fail(ACD_ERR_UNSUPPORTED, "acd_softmax: whole-tensor softmax needs contiguous input and output");
    acd_status st = f32 ? softmax_stats<float>(ctx, in, s) : softmax_stats<double>(ctx, in, s);
    const double *stats = ctx->control->stats;
    if (st != ACD_OK) return st;
    if (f32) {
      const int grid = persistent_grid(ctx, k_softmax_apply<float, 4, 4>, 256, 0, (n / 4 + 1023) / 1024 + 1);
      k_softmax_apply<float, 4, 4><<<grid, 256, 0, s>>>(reinterpret_cast<float *>(desc_ptr(out)),
                                                        reinterpret_cast<const float *>(desc_ptr(in)), n, stats);
    } else {
      const int grid = persistent_grid(ctx, k_softmax_apply<double, 2, 4>, 256, 0, (n / 2 + 1023) / 1024 + 1);
      k_softmax_apply<double, 2, 4><<<grid, 256, 0, s>>>(reinterpret_cast<double *>(desc_ptr(out)),
                                                         reinterpret_cast<const double *>(desc_ptr(in)), n, stats);
    }
    ACD_CUDA(cudaGetLastError());
    return ACD_OK;
  }
  SoftArgs a{};
  a.in = desc_ptr(in);
  a.out = desc_ptr(out);
  int64_t si[3] = {0, 0, 0}, so[3] = {0, 0, 0};
  if (!split_axis_sm(in, out, axis, a.L, a.R, a.O, si, so))
    return fail(ACD_ERR_UNSUPPORTED, "acd_softmax: view not collapsible around the axis; make it contiguous first");
  a.sl = si[0];
  a.sr = si[1];
  a.so = si[2];
  a.ol = so[0];
  a.orr = so[1];
  a.oo = so[2];
  acd_status st;
  const int VL = f32 ? 4 : 2;
  const bool wide = a.L >= 256 * VL && a.sl == 1 && a.ol == 1 && a.L % VL == 0 && a.sr % VL == 0 &&
                    a.orr % VL == 0 && a.so % VL == 0 && a.oo % VL == 0 && aligned_to<char>(a.in, 16) &&
                    aligned_to<char>(a.out, 16);
  // contiguous lanes: the wide two-pass kernels when there are at least 256
  // vectors of lanes (measured faster than the cluster kernel on
  // 65536x4096 float32: 0.60 vs 0.77 ms), else the single-read cluster kernel
  // the single-launch kernel needs enough lane groups (512-byte columns of
  // lanes) to keep the pipeline of statistics and apply items full: with 16
  // groups (1024x32768 float64) the two-pass kernels win, 0.18 vs 0.30 ms
  const int64_t lane_groups = (a.L + 32 * VL - 1) / (32 * VL) * a.O;
  if (wide && lane_groups >= 64)
    st = f32 ? launch_softmax_l2<float>(ctx, a, s) : launch_softmax_l2<double>(ctx, a, s);
  else if (wide)
    st = f32 ? launch_softmax_wide<float>(ctx, a, s) : launch_softmax_wide<double>(ctx, a, s);
  else if (f32 ? launch_softmax_tma<float>(ctx, a, s) : launch_softmax_tma<double>(ctx, a, s))
    st = ACD_OK;
  else if (a.L == 1)
    st = f32 ? launch_softmax_axis<float, 1>(ctx, a, s) : launch_softmax_axis<double, 1>(ctx, a, s);
  else
    st = f32 ? launch_softmax_axis<float, 32>(ctx, a, s) : launch_softmax_axis<double, 16>(ctx, a, s);
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

}  // extern "C"
