// Exact SIMT CUDA path for fp32 / fp64 compute: the chunked algorithm of the reference
// (swvr/chunked.py:82-151, torch branch) with every GEMM and element-wise step as a CUDA
// kernel.  Used for SWVR_F32 / SWVR_F64 compute dtypes (gradcheck, fp32 parity), where the
// tensor cores' bf16/fp16 operands would not meet the fp32 1e-5 / fp64 tolerances.
#include <cmath>

#include "common.cuh"
#include "simt.cuh"

namespace swvr {
namespace simt {

// C[m, n] = alpha * sum_k A[m, k] B[k, n] + beta * C[m, n] with arbitrary strides (the callers
// pass transposes as strides) and C of any dtype.  128 x 128 block tiles, 8-deep K steps,
// 8 x 8 outputs per thread.  The block tiles are double-buffered in shared memory (one barrier
// per K step) and the next K step's tiles are fetched into registers while the current one is
// multiplied.  Global loads run along whichever dimension of A / B has unit stride, so they
// coalesce for row- and column-major operands alike, 16 bytes at a time where the layout allows
// it; the fp32 kernel reads its fragments from shared memory 16 bytes at a time.
constexpr int BM = 128, BN = 128, BK = 8, PAD = 4;

template <typename T>
struct GemmTileLoader {
  // one thread's 4 elements of the BM x BK tile of A and of the BK x BN tile of B
  T a[4], b[4];
  // vec_a / vec_b: the 4 elements are contiguous, 16-byte aligned and all in or all out of range
  __device__ __forceinline__ void load(const T* __restrict__ A, int64_t sam, int64_t sak, const T* __restrict__ B,
                                       int64_t sbk, int64_t sbn, int64_t M, int64_t N, int64_t K, int64_t m0,
                                       int64_t n0, int64_t k0, int t, bool vec_a, bool vec_b) {
    if (vec_a) {
      const int64_t m = sak == 1 ? m0 + t / 2 : m0 + (t % 32) * 4;
      const int64_t k = sak == 1 ? k0 + (t % 2) * 4 : k0 + t / 32;
      const bool in = sak == 1 ? (m < M && k < K) : (m < M && k < K);
      const float4 v = in ? *reinterpret_cast<const float4*>(A + m * sam + k * sak) : make_float4(0.f, 0.f, 0.f, 0.f);
      a[0] = v.x, a[1] = v.y, a[2] = v.z, a[3] = v.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int64_t m, k;
        if (sak == 1) { m = m0 + t / 2; k = k0 + (t % 2) * 4 + e; }   // K contiguous in A
        else          { m = m0 + (t % 32) * 4 + e; k = k0 + t / 32; }  // M contiguous (or general)
        a[e] = (m < M && k < K) ? A[m * sam + k * sak] : T(0);
      }
    }
    if (vec_b) {
      const int64_t n = sbn == 1 ? n0 + (t % 32) * 4 : n0 + t / 2;
      const int64_t k = sbn == 1 ? k0 + t / 32 : k0 + (t % 2) * 4;
      const bool in = n < N && k < K;
      const float4 v = in ? *reinterpret_cast<const float4*>(B + k * sbk + n * sbn) : make_float4(0.f, 0.f, 0.f, 0.f);
      b[0] = v.x, b[1] = v.y, b[2] = v.z, b[3] = v.w;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int64_t n, k;
        if (sbn == 1) { n = n0 + (t % 32) * 4 + e; k = k0 + t / 32; }  // N contiguous in B
        else          { n = n0 + t / 2; k = k0 + (t % 2) * 4 + e; }   // K contiguous (or general)
        b[e] = (n < N && k < K) ? B[k * sbk + n * sbn] : T(0);
      }
    }
  }
  __device__ __forceinline__ void store(T (*As)[BM + PAD], T (*Bs)[BN + PAD], bool a_kcontig, bool b_ncontig,
                                        int t) const {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (a_kcontig) As[(t % 2) * 4 + e][t / 2] = a[e];
      else As[t / 32][(t % 32) * 4 + e] = a[e];
      if (b_ncontig) Bs[t / 32][(t % 32) * 4 + e] = b[e];
      else Bs[(t % 2) * 4 + e][t / 2] = b[e];
    }
  }
};

// Four consecutive elements of a shared-memory row (16-byte aligned for fp32).
template <typename T>
__device__ __forceinline__ void frag4(const T* p, T* out) {
  if constexpr (sizeof(T) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    out[0] = v.x, out[1] = v.y, out[2] = v.z, out[3] = v.w;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = p[i];
  }
}

// True when the loader's 4 elements along the unit-stride dimension form an aligned float4
// that is either wholly inside or wholly outside the extent: fp32, 16-byte aligned base,
// the other stride and the unit-stride extent multiples of 4.
template <typename T>
static bool vec4_ok(const T* p, int64_t s_other, int64_t s_unit, int64_t unit_extent) {
  return sizeof(T) == 4 && s_unit == 1 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && s_other % 4 == 0 &&
         unit_extent % 4 == 0;
}

template <typename T>
__global__ void __launch_bounds__(256) gemm_kernel(int64_t M, int64_t N, int64_t K, T alpha, const T* __restrict__ A,
                                                   int64_t sam, int64_t sak, const T* __restrict__ B, int64_t sbk,
                                                   int64_t sbn, T beta, void* C, int cdt, int64_t scm, int64_t scn,
                                                   bool vec_a, bool vec_b) {
  __shared__ __align__(16) T As[2][BK][BM + PAD];
  __shared__ __align__(16) T Bs[2][BK][BN + PAD];
  const int t = threadIdx.x, tx = t % 16, ty = t / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM, n0 = static_cast<int64_t>(blockIdx.x) * BN;
  const bool a_kcontig = sak == 1, b_ncontig = sbn == 1;
  T acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = T(0);
  GemmTileLoader<T> ld;
  ld.load(A, sam, sak, B, sbk, sbn, M, N, K, m0, n0, 0, t, vec_a, vec_b);
  ld.store(As[0], Bs[0], a_kcontig, b_ncontig, t);
  __syncthreads();
  int cur = 0;
  for (int64_t k0 = 0; k0 < K; k0 += BK) {
    const bool more = k0 + BK < K;
    if (more) ld.load(A, sam, sak, B, sbk, sbn, M, N, K, m0, n0, k0 + BK, t, vec_a, vec_b);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      // rows ty*4 + {0..3} and 64 + ty*4 + {0..3}; columns tx*4 + {0..3} and 64 + tx*4 + {0..3}
      T a[8], b[8];
      frag4(&As[cur][kk][ty * 4], a);
      frag4(&As[cur][kk][64 + ty * 4], a + 4);
      frag4(&Bs[cur][kk][tx * 4], b);
      frag4(&Bs[cur][kk][64 + tx * 4], b + 4);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
    if (more) ld.store(As[cur ^ 1], Bs[cur ^ 1], a_kcontig, b_ncontig, t);  // the other buffer: read a step ago
    __syncthreads();
    cur ^= 1;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= N) continue;
      const int64_t off = gm * scm + gn * scn;
      T v = alpha * acc[i][j];
      if (beta != T(0)) v += beta * static_cast<T>(load_d(C, cdt, off));
      store_d(C, cdt, off, static_cast<double>(v));
    }
  }
}

template <typename T>
cudaError_t gemm(cudaStream_t st, int64_t M, int64_t N, int64_t K, T alpha, const T* A, int64_t sam, int64_t sak,
                 const T* B, int64_t sbk, int64_t sbn, T beta, void* C, int cdt, int64_t scm, int64_t scn) {
  if (M == 0 || N == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>(ceil_div(N, BN)), static_cast<unsigned>(ceil_div(M, BM)));
  // A: unit stride along K (sak == 1) or along M (sam == 1); B: along N (sbn == 1) or along K
  const bool vec_a = sak == 1 ? vec4_ok(A, sam, sak, K) : vec4_ok(A, sak, sam, M);
  const bool vec_b = sbn == 1 ? vec4_ok(B, sbk, sbn, N) : vec4_ok(B, sbn, sbk, K);
  gemm_kernel<T><<<grid, 256, 0, st>>>(M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt, scm, scn, vec_a,
                                       vec_b);
  return cudaGetLastError();
}

template <typename T>
__device__ __forceinline__ T block_reduce(T v, bool is_max, T* sh) {
  for (int o = 16; o > 0; o >>= 1) {
    T w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? (w > v ? w : v) : v + w;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  const int nw = blockDim.x / 32;
  T r = sh[0];
  for (int i = 1; i < nw; ++i) r = is_max ? (sh[i] > r ? sh[i] : r) : r + sh[i];
  return r;
}

template <typename T>
__device__ __forceinline__ T exp_t(T x);
template <>
__device__ __forceinline__ float exp_t<float>(float x) { return expf(x); }
template <>
__device__ __forceinline__ double exp_t<double>(double x) { return exp(x); }

template <typename T>
__device__ __forceinline__ T log_t(T x);
template <>
__device__ __forceinline__ float log_t<float>(float x) { return logf(x); }
template <>
__device__ __forceinline__ double log_t<double>(double x) { return log(x); }

// S[n, :] += bias[v0:v0+C] (chunked.py:77-78)
template <typename T>
__global__ void add_bias_kernel(T* S, int64_t N, int64_t C, const void* bias, int bdt, int64_t v0) {
  const int64_t total = N * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    S[i] += static_cast<T>(load_d(bias, bdt, v0 + i % C));
}

// One block per row: the online-softmax update of chunked.py:96-104 (P written over S).
template <typename T>
__global__ void fwd_update_kernel(T* S, int64_t C, T* m, T* l, T* acc, int64_t D) {
  __shared__ T sh[32];
  const int64_t n = blockIdx.x;
  T* row = S + n * C;
  T mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) mx = row[c] > mx ? row[c] : mx;
  mx = block_reduce<T>(mx, true, sh);
  const T m_old = m[n];
  const T m_new = m_old > mx ? m_old : mx;
  const T shift = isinf(m_new) ? T(0) : m_new;  // chunked.py:97-98
  const T alpha = exp_t<T>(m_old - shift);
  T sum = 0;
  for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
    const T p = exp_t<T>(row[c] - shift);
    row[c] = p;
    sum += p;
  }
  sum = block_reduce<T>(sum, false, sh);
  for (int64_t d = threadIdx.x; d < D; d += blockDim.x) acc[n * D + d] *= alpha;
  if (threadIdx.x == 0) {
    l[n] = l[n] * alpha + sum;
    m[n] = m_new;
  }
}

template <typename T>
__global__ void fwd_init_kernel(T* m, T* l, T* acc, int64_t N, int64_t D) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < N * D;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    acc[i] = T(0);
    if (i < N) {
      m[i] = -INFINITY;
      l[i] = T(0);
    }
  }
}

// O = acc / l, LSE = m + log(l)  (chunked.py:105)
template <typename T>
__global__ void fwd_finish_kernel(const T* m, const T* l, const T* acc, T* O, T* lse, int64_t N, int64_t D) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < N * D;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / D;
    O[i] = acc[i] / l[n];
    if (i % D == 0) lse[n] = m[n] + log_t<T>(l[n]);
  }
}

// delta = rowsum(O * gO) - glse  (chunked.py:112-113)
template <typename T>
__global__ void delta_kernel(const T* O, const T* gO, const T* glse, T* delta, int64_t N, int64_t D) {
  for (int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; n < N;
       n += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    T s = 0;
    for (int64_t d = 0; d < D; ++d) s += O[n * D + d] * gO[n * D + d];
    delta[n] = s - glse[n];
  }
}

// P = exp(S - lse)  (chunked.py:132)
template <typename T>
__global__ void bwd_p_kernel(T* S, const T* lse, int64_t N, int64_t C) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < N * C;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    S[i] = exp_t<T>(S[i] - lse[i / C]);
}

// G = (dP - delta) * P  (chunked.py:134), in place in dP
template <typename T>
__global__ void bwd_gs_kernel(const T* P, T* G, const T* delta, int64_t N, int64_t C) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < N * C;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    G[i] = (G[i] - delta[i / C]) * P[i];
}

// gb[v0 + c] = sum_n G[n, c]  (chunked.py:135-136), fixed order per column.
template <typename T>
__global__ void colsum_kernel(const T* G, int64_t N, int64_t C, void* gb, int gdt, int64_t v0) {
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < C;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    T s = 0;
    for (int64_t n = 0; n < N; ++n) s += G[n * C + c];
    store_d(gb, gdt, v0 + c, static_cast<double>(s));
  }
}

template <typename T>
__global__ void cast_kernel(const T* src, void* dst, int dt, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_d(dst, dt, i, static_cast<double>(src[i]));
}

template <typename T>
__global__ void zero_rows_kernel(void* dst, int dt, int64_t rows, int64_t cols, int64_t ld) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows * cols;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_d(dst, dt, (i / cols) * ld + i % cols, 0.0);
}

inline unsigned grid_for(int64_t n, int threads = 256) {
  int64_t g = ceil_div(n, threads);
  if (g < 1) g = 1;
  if (g > 4096) g = 4096;
  return static_cast<unsigned>(g);
}

// ---------------------------------------------------------------------------------------- host
size_t fwd_workspace(const swvr_problem& p) {
  const size_t es = p.compute_dtype == SWVR_F64 ? 8 : 4;
  const int64_t C = p.chunk < p.vocab ? p.chunk : (p.vocab > 0 ? p.vocab : 1);
  return align_up(es * p.n_tokens * C, 256) + 2 * align_up(es * p.n_tokens, 256) +
         align_up(es * p.n_tokens * p.embed_dim, 256) + 256;
}

template <typename T>
static int fwd_impl(const swvr_problem& p, void* m_out, void* l_out, void* acc_out, T* O, T* lse, void* ws,
                    cudaStream_t st) {
  const int64_t N = p.n_tokens, K = p.hidden, V = p.vocab, D = p.embed_dim;
  const int64_t C = p.chunk < V ? p.chunk : (V > 0 ? V : 1);
  char* w = static_cast<char*>(ws);
  T* S = reinterpret_cast<T*>(w);
  w += align_up(sizeof(T) * N * C, 256);
  T* m = m_out ? static_cast<T*>(m_out) : reinterpret_cast<T*>(w);
  w += align_up(sizeof(T) * N, 256);
  T* l = l_out ? static_cast<T*>(l_out) : reinterpret_cast<T*>(w);
  w += align_up(sizeof(T) * N, 256);
  T* acc = acc_out ? static_cast<T*>(acc_out) : reinterpret_cast<T*>(w);
  const T* h = static_cast<const T*>(p.h);
  const T* W = static_cast<const T*>(p.W);
  const T* E = static_cast<const T*>(p.E);
  const int adt = sizeof(T) == 8 ? SWVR_F64 : SWVR_F32;
  fwd_init_kernel<T><<<grid_for(N * D > N ? N * D : N), 256, 0, st>>>(m, l, acc, N, D);
  for (int64_t v0 = 0; v0 < V; v0 += C) {
    const int64_t c = (V - v0) < C ? (V - v0) : C;
    cudaError_t e = gemm<T>(st, N, c, K, static_cast<T>(p.logit_scale), h, p.ldh, 1, W + v0 * p.ldw, 1, p.ldw, T(0),
                            S, adt, c, 1);
    if (e != cudaSuccess) return SWVR_ERR_CUDA;
    if (p.bias) add_bias_kernel<T><<<grid_for(N * c), 256, 0, st>>>(S, N, c, p.bias, p.bias_dtype, v0);
    if (N > 0) fwd_update_kernel<T><<<static_cast<unsigned>(N), 256, 0, st>>>(S, c, m, l, acc, D);
    e = gemm<T>(st, N, D, c, T(1), S, c, 1, E + v0 * p.lde, p.lde, 1, T(1), acc, adt, D, 1);
    if (e != cudaSuccess) return SWVR_ERR_CUDA;
  }
  if (O) fwd_finish_kernel<T><<<grid_for(N * D > N ? N * D : N), 256, 0, st>>>(m, l, acc, O, lse, N, D);
  return cudaGetLastError() == cudaSuccess ? SWVR_OK : SWVR_ERR_CUDA;
}

// The SIMT path keeps the natural-log running max; the partial-state ABI is in log2 units.
template <typename T>
__global__ void to_log2_kernel(T* m, int64_t N) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < N;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    m[i] = m[i] * static_cast<T>(1.4426950408889634);
}

int fwd(const swvr_problem& p, void* O, void* lse, void* m2, void* l, void* acc, void* ws, cudaStream_t st) {
  int rc;
  if (p.compute_dtype == SWVR_F64)
    rc = fwd_impl<double>(p, m2, l, acc, static_cast<double*>(O), static_cast<double*>(lse), ws, st);
  else
    rc = fwd_impl<float>(p, m2, l, acc, static_cast<float*>(O), static_cast<float*>(lse), ws, st);
  if (rc == SWVR_OK && m2 && p.n_tokens > 0) {
    if (p.compute_dtype == SWVR_F64)
      to_log2_kernel<double><<<grid_for(p.n_tokens), 256, 0, st>>>(static_cast<double*>(m2), p.n_tokens);
    else
      to_log2_kernel<float><<<grid_for(p.n_tokens), 256, 0, st>>>(static_cast<float*>(m2), p.n_tokens);
  }
  return rc;
}

size_t bwd_workspace(const swvr_problem& p, const swvr_grads& g) {
  const size_t es = p.compute_dtype == SWVR_F64 ? 8 : 4;
  const int64_t C = p.chunk < p.vocab ? p.chunk : (p.vocab > 0 ? p.vocab : 1);
  size_t b = 2 * align_up(es * p.n_tokens * C, 256) + align_up(es * p.n_tokens, 256);
  if (g.grad_h && !g.grad_h_acc) b += align_up(es * p.n_tokens * p.hidden, 256);
  return b + 256;
}

template <typename T>
static int bwd_impl(const swvr_problem& p, const swvr_grads& g, void* ws, cudaStream_t st) {
  const int64_t N = p.n_tokens, K = p.hidden, V = p.vocab, D = p.embed_dim;
  const int64_t C = p.chunk < V ? p.chunk : (V > 0 ? V : 1);
  const T s = static_cast<T>(p.logit_scale);
  const bool need_h = g.grad_h || g.grad_h_acc, need_W = g.grad_W, need_E = g.grad_E;
  const bool need_b = g.grad_bias && p.bias;
  const int adt = sizeof(T) == 8 ? SWVR_F64 : SWVR_F32;
  char* w = static_cast<char*>(ws);
  T* S = reinterpret_cast<T*>(w);
  w += align_up(sizeof(T) * N * C, 256);
  T* G = reinterpret_cast<T*>(w);
  w += align_up(sizeof(T) * N * C, 256);
  T* delta = reinterpret_cast<T*>(w);
  w += align_up(sizeof(T) * N, 256);
  T* dh = g.grad_h_acc ? static_cast<T*>(g.grad_h_acc) : reinterpret_cast<T*>(w);
  const T* h = static_cast<const T*>(p.h);
  const T* W = static_cast<const T*>(p.W);
  const T* E = static_cast<const T*>(p.E);
  const T* gO = static_cast<const T*>(g.grad_O);
  const T* lse = static_cast<const T*>(g.lse);
  if (N == 0) {
    if (need_W) zero_rows_kernel<T><<<grid_for(V * K), 256, 0, st>>>(g.grad_W, g.grad_W_dtype, V, K, g.ld_grad_W);
    if (need_E) zero_rows_kernel<T><<<grid_for(V * D), 256, 0, st>>>(g.grad_E, g.grad_E_dtype, V, D, g.ld_grad_E);
    if (need_b) zero_rows_kernel<T><<<grid_for(V), 256, 0, st>>>(g.grad_bias, g.grad_bias_dtype, 1, V, V);
    return cudaGetLastError() == cudaSuccess ? SWVR_OK : SWVR_ERR_CUDA;
  }
  delta_kernel<T><<<grid_for(N), 256, 0, st>>>(static_cast<const T*>(g.O), gO, static_cast<const T*>(g.grad_lse), delta,
                                               N, D);
  if (need_h && !(g.grad_h_acc && g.accumulate_grad_h)) cudaMemsetAsync(dh, 0, sizeof(T) * N * K, st);
  for (int64_t v0 = 0; v0 < V; v0 += C) {
    const int64_t c = (V - v0) < C ? (V - v0) : C;
    // P = exp(s h W_c^T + b_c - lse)  (chunked.py:132)
    if (gemm<T>(st, N, c, K, s, h, p.ldh, 1, W + v0 * p.ldw, 1, p.ldw, T(0), S, adt, c, 1) != cudaSuccess)
      return SWVR_ERR_CUDA;
    if (p.bias) add_bias_kernel<T><<<grid_for(N * c), 256, 0, st>>>(S, N, c, p.bias, p.bias_dtype, v0);
    bwd_p_kernel<T><<<grid_for(N * c), 256, 0, st>>>(S, lse, N, c);
    // G = (gO E_c^T - delta) * P  (chunked.py:134)
    if (gemm<T>(st, N, c, D, T(1), gO, D, 1, E + v0 * p.lde, 1, p.lde, T(0), G, adt, c, 1) != cudaSuccess)
      return SWVR_ERR_CUDA;
    bwd_gs_kernel<T><<<grid_for(N * c), 256, 0, st>>>(S, G, delta, N, c);
    if (need_b) colsum_kernel<T><<<grid_for(c), 256, 0, st>>>(G, N, c, g.grad_bias, g.grad_bias_dtype, v0);
    // gE_c = P^T gO  (chunked.py:137-138)
    if (need_E &&
        gemm<T>(st, c, D, N, T(1), S, 1, c, gO, D, 1, T(0), static_cast<char*>(g.grad_E) +
                    static_cast<size_t>(v0 * g.ld_grad_E) * dtype_size(g.grad_E_dtype),
                g.grad_E_dtype, g.ld_grad_E, 1) != cudaSuccess)
      return SWVR_ERR_CUDA;
    // gH += s G W_c ; gW_c = s G^T h  (chunked.py:142-150)
    if (need_h && gemm<T>(st, N, K, c, s, G, c, 1, W + v0 * p.ldw, p.ldw, 1, T(1), dh, adt, K, 1) != cudaSuccess)
      return SWVR_ERR_CUDA;
    if (need_W &&
        gemm<T>(st, c, K, N, s, G, 1, c, h, p.ldh, 1, T(0), static_cast<char*>(g.grad_W) +
                    static_cast<size_t>(v0 * g.ld_grad_W) * dtype_size(g.grad_W_dtype),
                g.grad_W_dtype, g.ld_grad_W, 1) != cudaSuccess)
      return SWVR_ERR_CUDA;
  }
  if (g.grad_h) cast_kernel<T><<<grid_for(N * K), 256, 0, st>>>(dh, g.grad_h, g.grad_h_dtype, N * K);
  return cudaGetLastError() == cudaSuccess ? SWVR_OK : SWVR_ERR_CUDA;
}

int bwd(const swvr_problem& p, const swvr_grads& g, void* ws, cudaStream_t st) {
  if (p.compute_dtype == SWVR_F64) return bwd_impl<double>(p, g, ws, st);
  return bwd_impl<float>(p, g, ws, st);
}

}  // namespace simt
}  // namespace swvr
