// RMSNorm producer of h, fused at both ends of the readout.
//
// Forward: h = x * rstd * weight with rstd = 1 / sqrt(mean_k x^2 + eps), computed in fp32
// (fp64 when x or h is fp64) and rounded once into the readout's compute dtype, so the
// readout's TMA loads read h as the norm wrote it (no separate cast, no [N, K] fp32 copy).
// Backward: takes the readout's un-cast dh accumulator (fp32, or fp64) directly, instead of
// dh rounded to h's dtype, and returns
//   dx = rstd * (a - xh * mean_k(a * xh)),  a = dh * weight,  xh = x * rstd
//   dweight = sum_n dh * xh                 (fixed-order reduction, no atomics)
// One warp per row in both kernels.  The weight gradient is summed per warp in shared
// memory (each lane owns its columns), then per block in warp order into a partial row,
// then over the blocks in block order: the result does not depend on scheduling.
#include <cmath>

#include "common.cuh"
#include "ptx.cuh"

namespace swvr {
namespace norm {

template <typename A>
__device__ __forceinline__ A load_a(const void* p, int dt, int64_t i) {
  if constexpr (sizeof(A) == 8) return load_d(p, dt, i);
  else return load_f(p, dt, i);
}

template <typename A>
__device__ __forceinline__ void store_a(void* p, int dt, int64_t i, A v) {
  if constexpr (sizeof(A) == 8) store_d(p, dt, i, v);
  else store_f(p, dt, i, v);
}

template <typename A>
__device__ __forceinline__ A warp_sum(A v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float inv_sqrt(float v) { return rsqrtf(v); }
__device__ __forceinline__ double inv_sqrt(double v) { return 1.0 / sqrt(v); }

template <typename A>
__global__ void rmsnorm_fwd_kernel(int64_t N, int64_t K, const void* __restrict__ x, int x_dt, int64_t ld_x,
                                   const void* __restrict__ w, int w_dt, A eps, void* h, int h_dt, int64_t ld_h,
                                   A* rstd) {
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (n >= N) return;
  const int64_t xr = n * ld_x, hr = n * ld_h;
  A ss = 0;
  for (int64_t k = lane; k < K; k += 32) {
    const A v = load_a<A>(x, x_dt, xr + k);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const A r = inv_sqrt(ss / static_cast<A>(K) + eps);
  for (int64_t k = lane; k < K; k += 32) {
    const A g = w ? load_a<A>(w, w_dt, k) : A(1);
    store_a<A>(h, h_dt, hr + k, load_a<A>(x, x_dt, xr + k) * r * g);
  }
  if (lane == 0) rstd[n] = r;
}

// Block b owns rows [b * rows_per_block, ...); warp w of the block takes every nwarps-th of
// them.  Shared memory: nwarps x K weight-gradient sums (when dw_part is not null).
template <typename A>
__global__ void rmsnorm_bwd_kernel(int64_t N, int64_t K, int64_t rows_per_block, const A* __restrict__ dh,
                                   const void* __restrict__ x, int x_dt, int64_t ld_x, const void* __restrict__ w,
                                   int w_dt, const A* __restrict__ rstd, void* dx, int dx_dt, A* dw_part) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  A* dws = reinterpret_cast<A*>(smem_raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  A* mine = dws + static_cast<int64_t>(warp) * K;
  if (dw_part)
    for (int64_t k = lane; k < K; k += 32) mine[k] = A(0);
  const int64_t r0 = blockIdx.x * rows_per_block, r1 = min(N, r0 + rows_per_block);
  for (int64_t n = r0 + warp; n < r1; n += nwarps) {
    const A r = rstd[n];
    const A* dr = dh + n * K;
    const int64_t xr = n * ld_x;
    A s = 0;
    for (int64_t k = lane; k < K; k += 32) {
      const A d = dr[k];
      const A xh = load_a<A>(x, x_dt, xr + k) * r;
      const A g = w ? load_a<A>(w, w_dt, k) : A(1);
      s += d * g * xh;
      if (dw_part) mine[k] += d * xh;
    }
    const A c = warp_sum(s) / static_cast<A>(K);
    if (dx) {
      for (int64_t k = lane; k < K; k += 32) {
        const A xh = load_a<A>(x, x_dt, xr + k) * r;
        const A g = w ? load_a<A>(w, w_dt, k) : A(1);
        store_a<A>(dx, dx_dt, n * K + k, r * (dr[k] * g - xh * c));
      }
    }
  }
  if (dw_part) {
    __syncthreads();
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      A t = 0;
      for (int i = 0; i < nwarps; ++i) t += dws[static_cast<int64_t>(i) * K + k];
      dw_part[blockIdx.x * K + k] = t;
    }
  }
}

template <typename A>
__global__ void rmsnorm_dw_reduce_kernel(int64_t K, int blocks, const A* __restrict__ dw_part, void* dw, int dw_dt) {
  const int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (k >= K) return;
  A t = 0;
  for (int b = 0; b < blocks; ++b) t += dw_part[static_cast<int64_t>(b) * K + k];
  store_a<A>(dw, dw_dt, k, t);
}

// Launch shape of the backward: warps per block (bounded by the shared-memory weight sums) and
// the number of blocks (each writes one partial row).
struct BwdShape {
  int nwarps, blocks;
  int64_t rows_per_block;
  size_t smem;
};

constexpr size_t kNormSmemMax = 200 * 1024;

inline BwdShape bwd_shape(int64_t N, int64_t K, size_t asz, bool need_w) {
  BwdShape s{};
  const size_t per_warp = need_w ? static_cast<size_t>(K) * asz : 0;
  s.nwarps = per_warp ? static_cast<int>(std::min<size_t>(8, kNormSmemMax / per_warp)) : 8;
  if (s.nwarps < 1) s.nwarps = 0;  // K too wide for the shared-memory sums
  const int64_t want = std::max<int64_t>(1, std::min<int64_t>(ceil_div(N, std::max(s.nwarps, 1)), 2 * kNumSMsB200));
  s.rows_per_block = ceil_div(std::max<int64_t>(N, 1), want);
  s.blocks = static_cast<int>(ceil_div(std::max<int64_t>(N, 1), s.rows_per_block));
  s.smem = static_cast<size_t>(s.nwarps) * per_warp;
  return s;
}

inline size_t bwd_workspace(int64_t N, int64_t K, size_t asz, bool need_w) {
  if (!need_w) return 0;
  const BwdShape s = bwd_shape(N, K, asz, need_w);
  return static_cast<size_t>(s.blocks) * K * asz;
}

template <typename A>
cudaError_t fwd(int64_t N, int64_t K, const void* x, int x_dt, int64_t ld_x, const void* w, int w_dt, double eps,
                void* h, int h_dt, int64_t ld_h, void* rstd, cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>(ceil_div(N, 8));
  rmsnorm_fwd_kernel<A><<<blocks, 256, 0, st>>>(N, K, x, x_dt, ld_x, w, w_dt, static_cast<A>(eps), h, h_dt, ld_h,
                                                static_cast<A*>(rstd));
  return cudaGetLastError();
}

template <typename A>
cudaError_t bwd(int64_t N, int64_t K, const void* dh, const void* x, int x_dt, int64_t ld_x, const void* w, int w_dt,
                const void* rstd, void* dx, int dx_dt, void* dw, int dw_dt, void* ws, cudaStream_t st) {
  const bool need_w = dw != nullptr;
  if (N == 0) {
    if (need_w) {
      rmsnorm_dw_reduce_kernel<A><<<static_cast<unsigned>(ceil_div(std::max<int64_t>(K, 1), 256)), 256, 0, st>>>(
          K, 0, static_cast<const A*>(ws), dw, dw_dt);
      return cudaGetLastError();
    }
    return cudaSuccess;
  }
  const BwdShape s = bwd_shape(N, K, sizeof(A), need_w);
  auto kern = rmsnorm_bwd_kernel<A>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(s.smem));
  if (e != cudaSuccess) return e;
  kern<<<s.blocks, 32 * s.nwarps, s.smem, st>>>(N, K, s.rows_per_block, static_cast<const A*>(dh), x, x_dt, ld_x, w,
                                               w_dt, static_cast<const A*>(rstd), dx, dx_dt,
                                               need_w ? static_cast<A*>(ws) : nullptr);
  e = cudaGetLastError();
  if (e != cudaSuccess || !need_w) return e;
  rmsnorm_dw_reduce_kernel<A><<<static_cast<unsigned>(ceil_div(K, 256)), 256, 0, st>>>(
      K, s.blocks, static_cast<const A*>(ws), dw, dw_dt);
  return cudaGetLastError();
}

}  // namespace norm
}  // namespace swvr
