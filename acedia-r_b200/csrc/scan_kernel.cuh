// Chained-scan kernel shared by acd_scan (scan.cu) and the entry point
// without allocation (scan_noalloc.cu).  See scan.cu for the algorithm.
#pragma once

#include "common.cuh"

namespace acd {

constexpr uint32_t kFlagAgg = 1u, kFlagIncl = 2u;

struct ScanArgs {
  const void *in;
  void *out;
  int64_t L, R, O;
  int64_t sl, sr, so;  // input strides
  int64_t ol, orr, oo; // output strides
  int64_t lblocks;     // lane blocks per o
  int64_t rtiles;      // step tiles per chain
  int64_t ntiles;
  uint32_t *flags;     // [ntiles]
  double *agg;         // [ntiles][LT]
  double *incl;        // [ntiles][LT]
  Control *control;
  uint32_t epoch;
  int64_t fault_tile;
  int64_t timeout_ns;
};

template <bool PROD>
__device__ __forceinline__ double combine(double a, double b) {
  return PROD ? a * b : a + b;
}

__device__ __forceinline__ uint32_t load_flag(const uint32_t *p) {
  return *reinterpret_cast<const volatile uint32_t *>(p);
}

// Thread layout: LT lanes x G step groups (LT * G == 256).  Each thread scans
// SEG consecutive steps of one lane in registers.
template <typename T, bool PROD, int LT, int SEG>
__global__ void __launch_bounds__(256, 3) k_scan(ScanArgs a) {
  constexpr int G = 256 / LT;
  constexpr int RT = G * SEG;  // steps per tile
  __shared__ int64_t s_tile;
  __shared__ double s_tot[G][LT];
  __shared__ double s_prefix[LT];
  __shared__ double s_win[LT > 1 ? 32 : 1][LT];
  const double ident = PROD ? 1.0 : 0.0;

  if (threadIdx.x == 0) s_tile = (int64_t)atomicAdd(&a.control->counters[1], 1u);
  __syncthreads();
  const int64_t tile = s_tile;
  const int64_t chain = tile / a.rtiles, q = tile % a.rtiles;
  const int64_t o = chain / a.lblocks, lb = chain % a.lblocks;
  const int lane = (LT == 1) ? 0 : (int)(threadIdx.x % LT);
  const int grp = (LT == 1) ? (int)threadIdx.x : (int)(threadIdx.x / LT);
  const int64_t l = lb * LT + lane;
  const bool lane_ok = l < a.L;
  const int64_t r0 = q * RT + (int64_t)grp * SEG;

  const T *in = static_cast<const T *>(a.in) + o * a.so + (lane_ok ? l : 0) * a.sl;
  T *out = static_cast<T *>(a.out) + o * a.oo + (lane_ok ? l : 0) * a.ol;

  // 1. load this thread's segment (kept in the tensor dtype, so a thread
  // holds SEG values of T rather than SEG doubles) and reduce it in double
  T xs[SEG];
#pragma unroll
  for (int k = 0; k < SEG; ++k) {
    const int64_t r = r0 + k;
    xs[k] = (lane_ok && r < a.R) ? in[r * a.sr] : T(PROD ? 1 : 0);
  }
  double run = ident;
#pragma unroll
  for (int k = 0; k < SEG; ++k) run = combine<PROD>(run, (double)xs[k]);

  // 2. exclusive prefix of the segment totals within the tile, per lane
  double excl = ident;
  double tile_total = ident;
  if constexpr (LT == 1) {
    // block scan over 256 segment totals: warp shuffles, then warp totals
    const int wl = threadIdx.x & 31, w = threadIdx.x >> 5;
    double x = run;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, x, d);
      if (wl >= d) x = combine<PROD>(y, x);
    }
    if (wl == 31) s_tot[w][0] = x;  // G == 256 rows; rows 0..7 reused for warp totals
    __syncthreads();
    double wexcl = ident, all = ident;
    for (int k = 0; k < 8; ++k) {
      const double t = s_tot[k][0];
      if (k < w) wexcl = combine<PROD>(wexcl, t);
      all = combine<PROD>(all, t);
    }
    const double incl_in_warp = x;
    double prev = __shfl_up_sync(0xffffffffu, incl_in_warp, 1);
    if (wl == 0) prev = ident;
    excl = combine<PROD>(wexcl, prev);
    tile_total = all;
  } else {
    s_tot[grp][lane] = run;
    __syncthreads();
    double all = ident;
    for (int g = 0; g < G; ++g) {
      const double t = s_tot[g][lane];
      if (g < grp) excl = combine<PROD>(excl, t);
      all = combine<PROD>(all, t);
    }
    tile_total = all;
  }

  // 3. publish and look back (warp 0).  Data lane dl < LT is carried by
  // thread dl (threads 0..LT-1 form step group 0); for LT == 1 the tile total
  // is uniform across threads.  The look-back inspects a window of 32
  // predecessors at once: lane l waits (bounded) for predecessor base - l to
  // publish, a ballot finds the nearest inclusive prefix, and the window's
  // aggregates are added in tile order.
  if (threadIdx.x < 32) {
    const int dl = threadIdx.x;
    const uint32_t ep = a.epoch << 2;
    const double my_total = tile_total;
    const bool publish = (tile != a.fault_tile);
    double prefix = ident;
    if (q == 0) {
      if (publish) {
        if (dl < LT) a.incl[tile * LT + dl] = my_total;
        __threadfence();
        __syncwarp();
        if (dl == 0) atomicExch(&a.flags[tile], ep | kFlagIncl);
      }
    } else {
      if (publish) {
        if (dl < LT) a.agg[tile * LT + dl] = my_total;
        __threadfence();
        __syncwarp();
        if (dl == 0) atomicExch(&a.flags[tile], ep | kFlagAgg);
      }
      const int64_t chain_start = tile - q;
      int64_t base = tile - 1;
      while (true) {
        const int64_t p = base - dl;
        const bool valid = p >= chain_start;
        uint32_t f = 0u;
        int gave_up = 0;
        if (valid) {
          f = load_flag(&a.flags[p]);
          if ((f & ~3u) != ep || (f & 3u) == 0u) {
            const uint64_t t0 = global_timer_ns();
            uint32_t spins = 0;
            while (true) {
              f = load_flag(&a.flags[p]);
              if ((f & ~3u) == ep && (f & 3u) != 0u) break;
              if (load_flag(&a.control->scan_abort) == a.epoch) { gave_up = 1; break; }
              if ((int64_t)(global_timer_ns() - t0) > a.timeout_ns || ++spins > (1u << 26)) {
                gave_up = 1;
                raise_status(a.control, 1, (int32_t)(tile & 0x7fffffff));
                atomicExch(&a.control->scan_abort, a.epoch);
                break;
              }
              __nanosleep(32);
            }
          }
        }
        if (__any_sync(0xffffffffu, gave_up)) break;
        __threadfence();
        const unsigned incl = __ballot_sync(0xffffffffu, valid && (f & 3u) == kFlagIncl);
        // lanes 0..stop contribute: aggregates before the nearest inclusive
        // prefix, then the inclusive prefix itself (the chain's first tile
        // always publishes one, so a window that reaches it stops there)
        const int stop = incl ? __ffs(incl) - 1 : 31;
        if constexpr (LT == 1) {
          double v = ident;
          if (dl <= stop && valid) v = __ldcg(((f & 3u) == kFlagIncl) ? &a.incl[p] : &a.agg[p]);
          // combine in tile order: lane stop is the oldest
#pragma unroll
          for (int d = 16; d > 0; d >>= 1) {
            const double o = __shfl_down_sync(0xffffffffu, v, d);
            if (dl + d < 32) v = combine<PROD>(v, o);
          }
          v = __shfl_sync(0xffffffffu, v, 0);
          prefix = combine<PROD>(v, prefix);
        } else {
          // stage the window's values with independent loads, then combine
          // them in tile order (oldest first)
#pragma unroll 8
          for (int l = 0; l < 32; ++l) {
            if (l <= stop && dl < LT) {
              const int64_t pl = base - l;
              s_win[l][dl] = __ldcg(((incl >> l) & 1u) ? &a.incl[pl * LT + dl] : &a.agg[pl * LT + dl]);
            }
          }
          __syncwarp();
          double w = ident;
          for (int l = stop; l >= 0; --l)
            if (dl < LT) w = combine<PROD>(w, s_win[l][dl]);
          __syncwarp();
          prefix = combine<PROD>(w, prefix);
        }
        if (incl) break;
        base -= 32;
      }
      // publish the inclusive prefix (also after giving up, so that later
      // tiles never wait on this one)
      if (publish) {
        if (dl < LT) a.incl[tile * LT + dl] = combine<PROD>(prefix, my_total);
        __threadfence();
        __syncwarp();
        if (dl == 0) atomicExch(&a.flags[tile], ep | kFlagIncl);
      }
    }
    if (dl < LT) s_prefix[dl] = prefix;
  }
  __syncthreads();

  // 4. write outputs: the running value restarts from the tile prefix and
  // this segment's exclusive prefix
  double acc = combine<PROD>(s_prefix[lane], excl);
#pragma unroll
  for (int k = 0; k < SEG; ++k) {
    const int64_t r = r0 + k;
    acc = combine<PROD>(acc, (double)xs[k]);
    if (lane_ok && r < a.R) out[r * a.orr] = (T)acc;
  }

  // 5. the last CTA to finish resets the ticket counters
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int d = atomicAdd(&a.control->counters[2], 1u);
    if (d == (unsigned int)(a.ntiles - 1)) {
      atomicExch(&a.control->counters[1], 0u);
      atomicExch(&a.control->counters[2], 0u);
    }
  }
}

// Collapses the view around `axis` into (L, R, O); returns false when the
// dims before or after the axis cannot be merged for both in and out.
inline bool split_axis(const acd_desc *in, const acd_desc *out, int axis, int64_t &L, int64_t &R, int64_t &O,
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

}  // namespace acd
