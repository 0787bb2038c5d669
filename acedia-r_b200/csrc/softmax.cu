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

#include "common.cuh"
#include "ops.cuh"
#include "reduce_acc.cuh"

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

// ---- whole tensor ----------------------------------------------------------
template <typename T, int V>
__global__ void __launch_bounds__(256) k_softmax_apply(T *__restrict__ out, const T *__restrict__ in, int64_t n,
                                                       const double *__restrict__ stats) {
  const T M = (T)stats[0];
  const T inv = (T)(1.0 / stats[1]);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n; i += nth) out[i] = m_exp(in[i] - M) * inv;
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
static acd_status launch_softmax_axis(acd_ctx *ctx, SoftArgs a, cudaStream_t s) {
  a.lblocks = (a.L + LT - 1) / LT;
  const int64_t groups = a.lblocks * a.O;
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
    const int grid = grid_for(ctx, n, 256, 8);
    if (f32)
      k_softmax_apply<float, 4><<<grid, 256, 0, s>>>(reinterpret_cast<float *>(desc_ptr(out)),
                                                     reinterpret_cast<const float *>(desc_ptr(in)), n, stats);
    else
      k_softmax_apply<double, 2><<<grid, 256, 0, s>>>(reinterpret_cast<double *>(desc_ptr(out)),
                                                      reinterpret_cast<const double *>(desc_ptr(in)), n, stats);
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
  if (a.L == 1)
    st = f32 ? launch_softmax_axis<float, 1>(ctx, a, s) : launch_softmax_axis<double, 1>(ctx, a, s);
  else
    st = f32 ? launch_softmax_axis<float, 32>(ctx, a, s) : launch_softmax_axis<double, 16>(ctx, a, s);
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

}  // extern "C"
