// Small memory-bound kernels around the tensor-core kernels: the online-softmax combine,
// the deterministic dE / db reduction, the backward prologue, the MSE / z-loss epilogue
// and dtype casts.
#include <cmath>
#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"
#include "small.cuh"

namespace swvr {
namespace small {

// Launch a grid of plain blocks, optionally with programmatic stream serialization.
template <typename... KArgs, typename... Args>
static cudaError_t launch_small(void (*kern)(KArgs...), unsigned blocks, unsigned threads, bool pdl, cudaStream_t st,
                                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.stream = st;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------------ combine
// Source s of row n lives at idx(s, n): split slots of the tensor-core forward (mode 0,
// T = tile_rows: ((n/T)*splits + s)*T + n%T) or shard-major arrays (mode 1: s*N + n).
// One warp per row: the lanes split the sources for the max and the weights
// w_s = 2^(m2_s - max) (exp2f for fp32 state), then split the D columns; the column sums
// run in the state's precision as fused multiply-adds in source order, and l in double
// through a fixed shuffle tree, so the result is deterministic and identical on every device
// that merges the same states.
__device__ __forceinline__ float exp2_t(float x) { return exp2f(x); }
__device__ __forceinline__ double exp2_t(double x) { return exp2(x); }

template <typename T>
__global__ void combine_kernel(int S, int64_t N, int64_t D, const T* __restrict__ m2, const T* __restrict__ l,
                               const T* __restrict__ acc, int mode, int splits, int tile_rows, T* O, T* lse, T* m2o,
                               T* lo, T* acco) {
  pdl_wait();
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (n >= N) return;
  // idx(s) = base + s * stride (integer divisions once per row, not per access)
  const int64_t base = mode == 0 ? (n / tile_rows) * splits * tile_rows + n % tile_rows : n;
  const int64_t stride = mode == 0 ? tile_rows : N;
  auto idx = [&](int s) -> int64_t { return base + static_cast<int64_t>(s) * stride; };
  T M = -INFINITY;
  for (int s = lane; s < S; s += 32) M = fmax(M, m2[idx(s)]);
  for (int o = 16; o > 0; o >>= 1) M = fmax(M, __shfl_xor_sync(0xffffffffu, M, o));
  const T ref = isinf(M) ? T(0) : M;
  // weights of the first 64 sources stay in two registers per lane; more are recomputed
  T w0 = 0, w1 = 0;
  double Lp = 0.0;
  for (int s = lane; s < S; s += 32) {
    const T w = exp2_t(m2[idx(s)] - ref);
    Lp += w == T(0) ? 0.0 : static_cast<double>(l[idx(s)]) * static_cast<double>(w);
    if (s < 32) w0 = w;
    else if (s < 64) w1 = w;
  }
  for (int o = 16; o > 0; o >>= 1) Lp += __shfl_xor_sync(0xffffffffu, Lp, o);
  const double L = Lp;
  for (int64_t d0 = 0; d0 < D; d0 += 32) {  // uniform trip count: the shuffles below need every lane
    const int64_t d = d0 + lane;
    T A = 0;
    // sources 8 at a time: their loads are all in flight before the first add; the adds stay
    // in source order
    for (int s0 = 0; s0 < S; s0 += 8) {
      T wv[8], v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int s = s0 + k;
        const T ws = __shfl_sync(0xffffffffu, s < 32 ? w0 : w1, s & 31);
        wv[k] = s < S ? (s < 64 ? ws : exp2_t(m2[idx(s)] - ref)) : T(0);
        v[k] = (d < D && wv[k] != T(0)) ? acc[idx(s) * D + d] : T(0);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (d < D && wv[k] != T(0)) A = fma(v[k], wv[k], A);
    }
    if (d < D) {
      if (O) O[n * D + d] = A / static_cast<T>(L);
      if (acco) acco[n * D + d] = A;
    }
  }
  if (lane == 0) {
    if (lse) lse[n] = static_cast<T>((static_cast<double>(ref) + log2(L)) * 0.6931471805599453);
    if (m2o) m2o[n] = M;
    if (lo) lo[n] = static_cast<T>(L);
  }
}

cudaError_t combine(int acc_dt, int S, int64_t N, int64_t D, const void* m2, const void* l, const void* acc, int mode,
                    int splits, int tile_rows, void* O, void* lse, void* m2o, void* lo, void* acco, bool pdl,
                    cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>(ceil_div(N, 8));  // 8 rows (warps) per block
  if (acc_dt == SWVR_F64)
    return launch_small(combine_kernel<double>, blocks, 256, pdl, st, S, N, D, static_cast<const double*>(m2),
                        static_cast<const double*>(l), static_cast<const double*>(acc), mode, splits, tile_rows,
                        static_cast<double*>(O), static_cast<double*>(lse), static_cast<double*>(m2o),
                        static_cast<double*>(lo), static_cast<double*>(acco));
  return launch_small(combine_kernel<float>, blocks, 256, pdl, st, S, N, D, static_cast<const float*>(m2),
                      static_cast<const float*>(l), static_cast<const float*>(acc), mode, splits, tile_rows,
                      static_cast<float*>(O), static_cast<float*>(lse), static_cast<float*>(m2o),
                      static_cast<float*>(lo), static_cast<float*>(acco));
}

// ------------------------------------------------------------------ dE / db reduction
// Row v of the chunk: sum its token-split partial slots in split order.  Slots are grouped
// per vocabulary tile of `tile_rows` rows: slot((vt*TS + ts)*tile_rows + r), so for one
// split the tile's rows x D floats are contiguous.  One thread per (row, 4 columns) when D is
// a multiple of 4 (else per (row, column)); each thread loads the splits 8 at a time, so
// eight independent 16-byte loads are in flight before the first add, and the adds stay in
// split order (the result does not depend on the batching).
template <int VEC>
__global__ void reduce_de_db_kernel(const float* __restrict__ part_de, const float* __restrict__ part_db, int TS,
                                    int n_ts, int v_begin, int rows, int tile_rows, int64_t D, void* gE, int gE_dt,
                                    int64_t ld_gE, void* gb, int gb_dt) {
  using V = typename std::conditional<VEC == 4, float4, float>::type;
  pdl_wait();
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t DV = D / VEC;  // vectors per row
  if (part_de && i < static_cast<int64_t>(rows) * DV) {
    const int64_t total = static_cast<int64_t>(rows) * DV;
    const int rr = total < (int64_t(1) << 32) ? static_cast<int>(static_cast<uint32_t>(i) / static_cast<uint32_t>(DV))
                                              : static_cast<int>(i / DV);
    const int64_t d = (i - static_cast<int64_t>(rr) * DV) * VEC;
    const int vt = rr / tile_rows, r = rr % tile_rows;
    const V* src = reinterpret_cast<const V*>(part_de + (static_cast<int64_t>(vt) * TS * tile_rows + r) * D + d);
    const int64_t step = static_cast<int64_t>(tile_rows) * DV;  // one split, in vectors
    float acc[VEC];
#pragma unroll
    for (int c = 0; c < VEC; ++c) acc[c] = 0.f;
    for (int ts0 = 0; ts0 < n_ts; ts0 += 8) {
      V buf[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (ts0 + k < n_ts) buf[k] = src[(ts0 + k) * step];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (ts0 + k < n_ts) {
          const float* f = reinterpret_cast<const float*>(&buf[k]);
#pragma unroll
          for (int c = 0; c < VEC; ++c) acc[c] += f[c];
        }
      }
    }
#pragma unroll
    for (int c = 0; c < VEC; ++c) store_f(gE, gE_dt, (v_begin + rr) * ld_gE + d + c, acc[c]);
  }
  if (part_db && i < rows) {
    const int rr = static_cast<int>(i);
    const int vt = rr / tile_rows, r = rr % tile_rows;
    const float* src = part_db + static_cast<int64_t>(vt) * TS * tile_rows + r;
    float s = 0.f;
#pragma unroll 4
    for (int ts = 0; ts < n_ts; ++ts) s += src[static_cast<int64_t>(ts) * tile_rows];
    store_f(gb, gb_dt, v_begin + rr, s);
  }
}

cudaError_t reduce_de_db(const float* part_de, const float* part_db, int TS, int per_t, int NT, int v_begin, int rows,
                         int tile_rows, int64_t D, void* gE, int gE_dt, int64_t ld_gE, void* gb, int gb_dt, bool pdl,
                         cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int n_ts = std::min(TS, static_cast<int>(ceil_div(NT, std::max(per_t, 1))));  // splits with tokens
  // 16-byte loads: D a multiple of 4 keeps every row (and the 256-byte aligned base) 16-byte aligned
  const bool vec = D % 4 == 0 && (reinterpret_cast<uintptr_t>(part_de) & 15u) == 0;
  const int64_t work = std::max<int64_t>(part_de ? static_cast<int64_t>(rows) * (vec ? D / 4 : D) : 0, rows);
  const unsigned blocks = static_cast<unsigned>(ceil_div(work, 256));
  if (vec)
    return launch_small(reduce_de_db_kernel<4>, blocks, 256, pdl, st, part_de, part_db, TS, n_ts, v_begin, rows,
                        tile_rows, D, gE, gE_dt, ld_gE, gb, gb_dt);
  return launch_small(reduce_de_db_kernel<1>, blocks, 256, pdl, st, part_de, part_db, TS, n_ts, v_begin, rows,
                      tile_rows, D, gE, gE_dt, ld_gE, gb, gb_dt);
}

// ------------------------------------------------------------------ bounded-wait self test
// One thread waits on an mbarrier that nothing arrives on, through the same bounded wait the
// tensor-core pipelines use, so the error path (error word recorded, kernel returns, context
// usable) can be exercised without a fault or a hang.
__global__ void wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, kErrSelftest | 1, limit_ns);
}

cudaError_t wait_selftest(uint64_t limit_ns, cudaStream_t st) {
  wait_selftest_kernel<<<1, 32, 0, st>>>(limit_ns);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ backward prologue
// delta = rowsum(O * gO) - glse (swvr/chunked.py:112-113) and gO rounded to the compute
// dtype, zero-padded to DP columns (chunked.py:114).  One warp per row.
template <bool kBF16>
__global__ void prologue_kernel(const float* __restrict__ O, const float* __restrict__ gO,
                                const float* __restrict__ glse, int64_t N, int D, int DP, float* delta, void* gOc) {
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (n >= N) return;
  float s = 0.f;
  for (int d = lane; d < DP; d += 32) {
    const float go = d < D ? gO[n * D + d] : 0.f;
    if (d < D) s += O[n * D + d] * go;
    if constexpr (kBF16)
      static_cast<__nv_bfloat16*>(gOc)[n * DP + d] = __float2bfloat16_rn(go);
    else
      static_cast<__half*>(gOc)[n * DP + d] = __float2half_rn(go);
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) delta[n] = s - glse[n];
}

cudaError_t prologue(bool bf16, const float* O, const float* gO, const float* glse, int64_t N, int D, int DP,
                     float* delta, void* gOc, cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>(ceil_div(N, 8));
  if (bf16)
    prologue_kernel<true><<<blocks, 256, 0, st>>>(O, gO, glse, N, D, DP, delta, gOc);
  else
    prologue_kernel<false><<<blocks, 256, 0, st>>>(O, gO, glse, N, D, DP, delta, gOc);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ casts
__global__ void cast_f32_kernel(const float* __restrict__ src, void* dst, int dt, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_f(dst, dt, i, src[i]);
}

cudaError_t cast_f32(const float* src, void* dst, int dt, int64_t n, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  int64_t blocks = ceil_div(n, 256);
  if (blocks > 8192) blocks = 8192;
  cast_f32_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(src, dst, dt, n);
  return cudaGetLastError();
}

__global__ void zero_kernel(void* dst, int dt, int64_t rows, int64_t cols, int64_t ld) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows * cols;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_d(dst, dt, (i / cols) * ld + i % cols, 0.0);
}

cudaError_t zero_rows(void* dst, int dt, int64_t rows, int64_t cols, int64_t ld, cudaStream_t st) {
  if (rows * cols == 0) return cudaSuccess;
  int64_t blocks = ceil_div(rows * cols, 256);
  if (blocks > 8192) blocks = 8192;
  zero_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(dst, dt, rows, cols, ld);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ MSE epilogue
// raw_n = mean_d (O - t)^2 + z * lse^2  (swvr/api.py:54-56); one warp per row.
template <typename T>
__device__ __forceinline__ T row_raw(const T* O, const T* t, const T* lse, int64_t n, int64_t D, T z, int lane) {
  T s = 0;
  for (int64_t d = lane; d < D; d += 32) {
    const T e = O[n * D + d] - t[n * D + d];
    s += e * e;
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  T raw = s / static_cast<T>(D);
  if (z != T(0)) raw += z * lse[n] * lse[n];
  return raw;
}

template <typename T>
__global__ void mse_none_kernel(int64_t N, int64_t D, const T* O, const T* lse, const T* t, const T* w, T z, T* out) {
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
  if (n >= N) return;
  const T raw = row_raw<T>(O, t, lse, n, D, z, threadIdx.x % 32);
  if (threadIdx.x % 32 == 0) out[n] = w ? raw * w[n] : raw;
}

// Deterministic two-stage reduction over a fixed grid of kMseBlocks blocks (one warp per
// row, rows assigned round-robin in a fixed pattern): stage 1 writes each block's
// (sum w*raw, sum w) to stats[2 + 2b]; stage 2 (one block) adds them in block order and
// writes out[0] = loss, stats[0] = sum(w * raw), stats[1] = denominator.
constexpr int kMseBlocks = 256;

template <typename T>
__global__ void __launch_bounds__(256) mse_partial_kernel(int64_t N, int64_t D, const T* O, const T* lse, const T* t,
                                                          const T* w, T z, T* stats) {
  __shared__ T sh_s[8], sh_w[8];
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  T s = 0, ws = 0;
  for (int64_t n = static_cast<int64_t>(blockIdx.x) * 8 + warp; n < N; n += static_cast<int64_t>(kMseBlocks) * 8) {
    const T raw = row_raw<T>(O, t, lse, n, D, z, lane);
    const T wn = w ? w[n] : T(1);
    s += raw * wn;
    ws += wn;
  }
  if (lane == 0) {
    sh_s[warp] = s;
    sh_w[warp] = ws;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    T S = 0, Wt = 0;
    for (int i = 0; i < 8; ++i) {
      S += sh_s[i];
      Wt += sh_w[i];
    }
    stats[2 + 2 * blockIdx.x] = S;
    stats[3 + 2 * blockIdx.x] = Wt;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) mse_final_kernel(int64_t N, int reduction, bool weighted, T* out, T* stats) {
  __shared__ T sh_s[kMseBlocks], sh_w[kMseBlocks];
  sh_s[threadIdx.x] = stats[2 + 2 * threadIdx.x];
  sh_w[threadIdx.x] = stats[3 + 2 * threadIdx.x];
  __syncthreads();
  for (int stride = kMseBlocks / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) {
      sh_s[threadIdx.x] += sh_s[threadIdx.x + stride];
      sh_w[threadIdx.x] += sh_w[threadIdx.x + stride];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    T denom = T(1);
    if (reduction == SWVR_REDUCE_MEAN) denom = weighted ? sh_w[0] : static_cast<T>(N);
    out[0] = sh_s[0] / denom;
    stats[0] = sh_s[0];
    stats[1] = denom;
  }
}

template <typename T>
__global__ void mse_bwd_kernel(int64_t N, int64_t D, const T* O, const T* lse, const T* t, const T* w, T z,
                               int reduction, const T* gout, const T* stats, T* gO, T* glse, T* gt, T* gw) {
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (n >= N) return;
  const T g = reduction == SWVR_REDUCE_NONE ? gout[n] : gout[0];
  const T wn = w ? w[n] : T(1);
  T denom = T(1);
  if (reduction == SWVR_REDUCE_MEAN) denom = stats[1];
  const T c = g * wn / denom;
  const T k = c * static_cast<T>(2) / static_cast<T>(D);
  for (int64_t d = lane; d < D; d += 32) {
    const T v = k * (O[n * D + d] - t[n * D + d]);
    gO[n * D + d] = v;
    if (gt) gt[n * D + d] = -v;
  }
  if (lane == 0) glse[n] = c * static_cast<T>(2) * z * lse[n];
  if (gw) {
    const T raw = row_raw<T>(O, t, lse, n, D, z, lane);
    if (lane == 0) {
      T v = g * raw;
      if (reduction == SWVR_REDUCE_MEAN) v = g * (raw - stats[0] / denom) / denom;
      gw[n] = v;
    }
  }
}

template <typename T>
static cudaError_t mse_fwd_t(int64_t N, int64_t D, const void* O, const void* lse, const void* t, const void* w,
                             double z, int red, void* out, void* stats, cudaStream_t st) {
  if (red == SWVR_REDUCE_NONE) {
    if (N == 0) return cudaSuccess;
    mse_none_kernel<T><<<static_cast<unsigned>(ceil_div(N, 8)), 256, 0, st>>>(
        N, D, static_cast<const T*>(O), static_cast<const T*>(lse), static_cast<const T*>(t),
        static_cast<const T*>(w), static_cast<T>(z), static_cast<T*>(out));
  } else {
    mse_partial_kernel<T><<<kMseBlocks, 256, 0, st>>>(N, D, static_cast<const T*>(O), static_cast<const T*>(lse),
                                                      static_cast<const T*>(t), static_cast<const T*>(w),
                                                      static_cast<T>(z), static_cast<T*>(stats));
    mse_final_kernel<T><<<1, kMseBlocks, 0, st>>>(N, red, w != nullptr, static_cast<T*>(out), static_cast<T*>(stats));
  }
  return cudaGetLastError();
}

cudaError_t mse_fwd(int dt, int64_t N, int64_t D, const void* O, const void* lse, const void* t, const void* w,
                    double z, int red, void* out, void* stats, cudaStream_t st) {
  return dt == SWVR_F64 ? mse_fwd_t<double>(N, D, O, lse, t, w, z, red, out, stats, st)
                        : mse_fwd_t<float>(N, D, O, lse, t, w, z, red, out, stats, st);
}

template <typename T>
static cudaError_t mse_bwd_t(int64_t N, int64_t D, const void* O, const void* lse, const void* t, const void* w,
                             double z, int red, const void* gout, const void* stats, void* gO, void* glse, void* gt,
                             void* gw, cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  mse_bwd_kernel<T><<<static_cast<unsigned>(ceil_div(N, 8)), 256, 0, st>>>(
      N, D, static_cast<const T*>(O), static_cast<const T*>(lse), static_cast<const T*>(t), static_cast<const T*>(w),
      static_cast<T>(z), red, static_cast<const T*>(gout), static_cast<const T*>(stats), static_cast<T*>(gO),
      static_cast<T*>(glse), static_cast<T*>(gt), static_cast<T*>(gw));
  return cudaGetLastError();
}

cudaError_t mse_bwd(int dt, int64_t N, int64_t D, const void* O, const void* lse, const void* t, const void* w,
                    double z, int red, const void* gout, const void* stats, void* gO, void* glse, void* gt, void* gw,
                    cudaStream_t st) {
  return dt == SWVR_F64 ? mse_bwd_t<double>(N, D, O, lse, t, w, z, red, gout, stats, gO, glse, gt, gw, st)
                        : mse_bwd_t<float>(N, D, O, lse, t, w, z, red, gout, stats, gO, glse, gt, gw, st);
}

}  // namespace small
}  // namespace swvr
