// Counter-based random tensors.
//
// Reference: rand_tensor / rnorm_tensor (src/TensorRandom.cpp:42-224) fill a
// new tensor from a process-wide cuRAND generator seeded with time(NULL), so
// their streams are neither reproducible nor independent of how a tensor is
// split.  Here element i of a call takes its value from counter (offset + i)
// of Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers:
// as easy as 1, 2, 3", SC 2011) under a 64-bit key (the seed): any shard of a
// tensor, on any number of GPUs, generates exactly the values of the whole
// tensor at its global indices.
//
// One Philox block (a 128-bit counter) yields four 32-bit words, used as
//   float32 uniform  4 values: (w >> 8) * 2^-24                      in [0, 1)
//   float64 uniform  2 values: ((w0 << 32 | w1) >> 11) * 2^-53        in [0, 1)
//   float32 normal   4 values: Box-Muller on (w0, w1) and (w2, w3)
//   float64 normal   2 values: Box-Muller on 53-bit uniforms from (w0, w1), (w2, w3)
// Box-Muller: r = sqrt(-2 log u), (z0, z1) = r (cos 2 pi v, sin 2 pi v) with u
// in (0, 1] (a uniform shifted by one step) and v in [0, 1).  Uniforms are
// scaled as min + (max - min) u and normals as mean + sd z: one fused
// multiply-add in the tensor dtype (float32: with min, max - min, mean and sd
// rounded to float32 first).
#include "common.cuh"

namespace acd {

namespace {

constexpr uint32_t kPhiloxM0 = 0xD2511F53u, kPhiloxM1 = 0xCD9E8D57u;
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u, kPhiloxW1 = 0xBB67AE85u;
constexpr int kRandThreads = 256;

__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = kPhiloxM0 * c[0], hi0 = __umulhi(kPhiloxM0, c[0]);
    const uint32_t lo1 = kPhiloxM1 * c[2], hi1 = __umulhi(kPhiloxM1, c[2]);
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
    k0 += kPhiloxW0;
    k1 += kPhiloxW1;
  }
}

// The values of counter block g: 4 (float32) or 2 (float64).
template <typename T, int DIST>
__device__ __forceinline__ void block_values(uint64_t g, uint32_t k0, uint32_t k1, double a, double b, T v[4]) {
  uint32_t w[4] = {(uint32_t)g, (uint32_t)(g >> 32), 0u, 0u};
  philox4x32_10(w, k0, k1);
  if constexpr (std::is_same<T, float>::value) {
    if constexpr (DIST == 0) {
      const float span = (float)(b - a), lo = (float)a;
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = fmaf(span, (float)(w[j] >> 8) * 0x1p-24f, lo);
    } else {
      const float sd = (float)b, mu = (float)a;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const float u = (float)((w[2 * p] >> 8) + 1u) * 0x1p-24f;  // (0, 1]
        const float t = (float)(w[2 * p + 1] >> 8) * 0x1p-24f;      // [0, 1)
        const float r = sqrtf(-2.0f * logf(u));
        float sn, cs;
        sincospif(2.0f * t, &sn, &cs);
        v[2 * p] = fmaf(sd, r * cs, mu);
        v[2 * p + 1] = fmaf(sd, r * sn, mu);
      }
    }
  } else {
    const uint64_t x0 = (((uint64_t)w[0] << 32) | w[1]) >> 11;
    const uint64_t x1 = (((uint64_t)w[2] << 32) | w[3]) >> 11;
    if constexpr (DIST == 0) {
      v[0] = fma(b - a, (double)x0 * 0x1p-53, a);
      v[1] = fma(b - a, (double)x1 * 0x1p-53, a);
    } else {
      const double u = (double)(x0 + 1) * 0x1p-53;  // (0, 1]
      const double t = (double)x1 * 0x1p-53;        // [0, 1)
      const double r = sqrt(-2.0 * log(u));
      double sn, cs;
      sincospi(2.0 * t, &sn, &cs);
      v[0] = fma(b, r * cs, a);
      v[1] = fma(b, r * sn, a);
    }
  }
}

// out[i] for i in [0, n) takes the value of counter position offset + i.
template <typename T, int DIST>
__global__ void __launch_bounds__(kRandThreads) k_rand(T *__restrict__ out, int64_t n, uint64_t offset, uint32_t k0,
                                                       uint32_t k1, double a, double b) {
  constexpr int PB = std::is_same<T, float>::value ? 4 : 2;  // values per counter block
  const uint64_t g0 = offset / PB;
  const uint64_t g1 = (offset + (uint64_t)n + PB - 1) / PB;
  const int64_t nb = (int64_t)(g1 - g0);
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  const bool aligned = offset % PB == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  for (int64_t bi = tid; bi < nb; bi += nth) {
    const uint64_t g = g0 + (uint64_t)bi;
    T v[4];
    block_values<T, DIST>(g, k0, k1, a, b, v);
    const int64_t first = (int64_t)(g * PB - offset);  // output index of v[0] (may be < 0 in the first block)
    if (aligned && first + PB <= n) {
      Vec<T, PB> vv;
#pragma unroll
      for (int j = 0; j < PB; ++j) vv.v[j] = v[j];
      *reinterpret_cast<Vec<T, PB> *>(out + first) = vv;
    } else {
#pragma unroll
      for (int j = 0; j < PB; ++j)
        if (first + j >= 0 && first + j < n) out[first + j] = v[j];
    }
  }
}

template <typename T>
acd_status launch_rand(acd_ctx *ctx, T *out, int64_t n, int dist, double a, double b, uint64_t seed,
                       uint64_t offset, cudaStream_t s) {
  constexpr int PB = std::is_same<T, float>::value ? 4 : 2;
  const int64_t nb = (int64_t)((offset + (uint64_t)n + PB - 1) / PB - offset / PB);
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  const int64_t work = (nb + kRandThreads - 1) / kRandThreads;
  if (dist == 0) {
    const int grid = persistent_grid(ctx, k_rand<T, 0>, kRandThreads, 0, work);
    k_rand<T, 0><<<grid, kRandThreads, 0, s>>>(out, n, offset, k0, k1, a, b);
  } else {
    const int grid = persistent_grid(ctx, k_rand<T, 1>, kRandThreads, 0, work);
    k_rand<T, 1><<<grid, kRandThreads, 0, s>>>(out, n, offset, k0, k1, a, b);
  }
  return ACD_OK;
}

}  // namespace

}  // namespace acd

using namespace acd;

extern "C" {

acd_status acd_rand(acd_ctx *ctx, const acd_desc *out, int32_t dist, double a, double b, uint64_t seed,
                    uint64_t offset, acd_stream stream) {
  if (!ctx) return fail(ACD_ERR_INVALID, "acd_rand: null context");
  ACD_TRY(check_desc(out, "out"));
  if (out->dtype != ACD_FLOAT32 && out->dtype != ACD_FLOAT64)
    return fail(ACD_ERR_DTYPE, "Unsupported dtype for random tensor. Use 'float' or 'double'");
  if (!desc_is_contiguous(out)) return fail(ACD_ERR_UNSUPPORTED, "acd_rand: the output must be contiguous");
  if (dist == 0) {
    if (!(a < b)) return fail(ACD_ERR_INVALID, "min must be less than max");
  } else if (dist == 1) {
    if (!(b > 0.0)) return fail(ACD_ERR_INVALID, "sd must be positive");
  } else {
    return fail(ACD_ERR_INVALID, "acd_rand: bad distribution %d", dist);
  }
  const int64_t n = desc_numel(out);
  if (n == 0) return ACD_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  acd_status st;
  if (out->dtype == ACD_FLOAT32)
    st = launch_rand<float>(ctx, reinterpret_cast<float *>(desc_ptr(out)), n, dist, a, b, seed, offset, s);
  else
    st = launch_rand<double>(ctx, reinterpret_cast<double *>(desc_ptr(out)), n, dist, a, b, seed, offset, s);
  if (st != ACD_OK) return st;
  ACD_CUDA(cudaGetLastError());
  return ACD_OK;
}

}  // extern "C"
