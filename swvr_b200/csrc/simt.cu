// Exact path for fp32 / fp64 compute: the chunked algorithm of the reference
// (swvr/chunked.py:82-151, torch branch) with every GEMM and element-wise step as a CUDA
// kernel.  Used for SWVR_F32 / SWVR_F64 compute dtypes (gradcheck, fp32 parity), where the
// bf16/fp16 tensor-core kernels would not meet the fp32 1e-5 / fp64 tolerances.  fp64 GEMMs
// run on the CUDA cores; fp32 GEMMs run as three-term split TF32 products on the tensor
// cores (gemm_tf32x3_kernel, fp32-level error) wherever their operands can be staged 16
// bytes at a time, and on the CUDA cores otherwise.
#include <algorithm>
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

// fp32 GEMM on the tensor cores at fp32 accuracy: each operand is split into a TF32 head and
// the TF32 rounding of its remainder, x = hi(x) + lo(x), and the product takes the three
// terms lo·hi + hi·lo + hi·hi (the lo·lo term, ~2^-22 relative, is dropped): about 2^-21
// relative error per product, against 2^-24 for an fp32 FMA and 2^-11 for plain TF32.  Each
// 8-deep K step's terms are summed from zero and added to the running sum in fp32
// round-to-nearest, so the MMA's own rounding toward zero does not accumulate over K.  128 x 128 block tiles, 32-deep K tiles in a 3-stage cp.async ring (the
// CUDA-core kernel above, one 8-deep step ahead, waits on its global loads), eight warps of
// 64 x 32 as 4 x 4 warp-level m16n8k8 TF32 MMAs; the operands are split as the fragments
// are read.  Each operand is staged in its own global layout: a K-contiguous tile as rows of
// 32 + 4 floats, an M- (or N-) contiguous one as rows of 128 + 8; in both a fragment load of
// lane (g = lane / 4, q = lane % 4) touches 32 distinct banks.
namespace tf32x3 {
constexpr int TM = 128, TN = 128, TK = 32, STAGES = 3, KP = TK + 4, MP = 128 + 8;
constexpr int A_WORDS = TM * KP > TK * MP ? TM * KP : TK * MP;  // either layout of one stage
constexpr int B_WORDS = TN * KP > TK * MP ? TN * KP : TK * MP;
constexpr int SMEM = STAGES * (A_WORDS + B_WORDS) * 4;
}  // namespace tf32x3

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void split_tf32(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_rna(x);
  lo = tf32_rna(x - __uint_as_float(hi));
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// 16 bytes global -> shared, zero-filled when !in (no bytes are read then).
__device__ __forceinline__ void cp16(float* dst, const float* src, bool in) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(in ? 16 : 0));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// AK: A is K-contiguous (sak == 1) else M-contiguous (sam == 1); BNC: B is N-contiguous
// (sbn == 1) else K-contiguous (sbk == 1).  The host checks the 16-byte alignment of every
// staged chunk (see gemm below).
template <bool AK, bool BNC>
__global__ void __launch_bounds__(256, 2) gemm_tf32x3_kernel(int64_t M, int64_t N, int64_t K, float alpha,
                                                          const float* __restrict__ A, int64_t sam, int64_t sak,
                                                          const float* __restrict__ B, int64_t sbk, int64_t sbn,
                                                          float beta, void* C, int cdt, int64_t scm, int64_t scn,
                                                          int64_t kper, int64_t zstride, const void* cbias,
                                                          int cbias_dt) {
  using namespace tf32x3;
  // split K: block z takes K rows [z * kper, z * kper + kper) and writes its own fp32 slice of C
  {
    const int64_t kb = static_cast<int64_t>(blockIdx.z) * kper;
    A += kb * sak;
    B += kb * sbk;
    K = K - kb < kper ? K - kb : kper;
    if (gridDim.z > 1) C = static_cast<float*>(C) + blockIdx.z * zstride;
  }
  extern __shared__ __align__(16) float smem_f[];
  float* As = smem_f;                       // [STAGES][A_WORDS]
  float* Bs = smem_f + STAGES * A_WORDS;    // [STAGES][B_WORDS]
  const int t = threadIdx.x, lane = t % 32, warp = t / 32;
  const int g = lane / 4, q = lane % 4;
  const int wm = (warp % 2) * 64, wn = (warp / 2) * 32;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * TM, n0 = static_cast<int64_t>(blockIdx.x) * TN;
  const int ktiles = static_cast<int>((K + TK - 1) / TK);

  // stage s <- K tile kt: 1024 16-byte chunks of A and of B, 4 + 4 per thread
  auto load = [&](int s, int kt) {
    const int64_t k0 = static_cast<int64_t>(kt) * TK;
    float* as = As + s * A_WORDS;
    float* bs = Bs + s * B_WORDS;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = t + i * 256;
      if (AK) {  // 128 rows of m x 8 chunks of k
        const int r = c / 8, c4 = (c % 8) * 4;
        const int64_t m = m0 + r, k = k0 + c4;
        const bool in = m < M && k < K;
        cp16(as + r * KP + c4, in ? A + m * sam + k : A, in);
      } else {   // 32 rows of k x 32 chunks of m
        const int r = c / 32, c4 = (c % 32) * 4;
        const int64_t k = k0 + r, m = m0 + c4;
        const bool in = m < M && k < K;
        cp16(as + r * MP + c4, in ? A + k * sak + m : A, in);
      }
      if (BNC) { // 32 rows of k x 32 chunks of n
        const int r = c / 32, c4 = (c % 32) * 4;
        const int64_t k = k0 + r, n = n0 + c4;
        const bool in = n < N && k < K;
        cp16(bs + r * MP + c4, in ? B + k * sbk + n : B, in);
      } else {   // 128 rows of n x 8 chunks of k
        const int r = c / 8, c4 = (c % 8) * 4;
        const int64_t n = n0 + r, k = k0 + c4;
        const bool in = n < N && k < K;
        cp16(bs + r * KP + c4, in ? B + n * sbn + k : B, in);
      }
    }
  };
  auto a_at = [&](const float* as, int r, int k) -> float { return AK ? as[r * KP + k] : as[k * MP + r]; };
  auto b_at = [&](const float* bs, int k, int n) -> float { return BNC ? bs[k * MP + n] : bs[n * KP + k]; };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < ktiles) load(s, s);
    cp_commit();
  }
  for (int kt = 0; kt < ktiles; ++kt) {
    cp_wait<STAGES - 2>();  // K tile kt has landed (this thread's copies) ...
    __syncthreads();        // ... and every thread's; the stage read in kt - 1 is free again
    if (kt + STAGES - 1 < ktiles) load((kt + STAGES - 1) % STAGES, kt + STAGES - 1);
    cp_commit();
    const float* as = As + (kt % STAGES) * A_WORDS;
    const float* bs = Bs + (kt % STAGES) * B_WORDS;
#pragma unroll
    for (int kk = 0; kk < TK; kk += 8) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t bh[4][2], bl[4][2];  // re-split per m tile: 16 fewer live registers
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          split_tf32(b_at(bs, kk + q, wn + j * 8 + g), bh[j][0], bl[j][0]);
          split_tf32(b_at(bs, kk + q + 4, wn + j * 8 + g), bh[j][1], bl[j][1]);
        }
        const int r = wm + i * 16 + g;
        uint32_t ah[4], al[4];
        split_tf32(a_at(as, r, kk + q), ah[0], al[0]);
        split_tf32(a_at(as, r + 8, kk + q), ah[1], al[1]);
        split_tf32(a_at(as, r, kk + q + 4), ah[2], al[2]);
        split_tf32(a_at(as, r + 8, kk + q + 4), ah[3], al[3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // the three terms of this 8-deep K step start from zero and are added to the running
          // sum in fp32 round-to-nearest: the MMA's own accumulation rounds toward zero, which
          // over a long K (thousands of steps) would bias the sum by ~1e-5 relative
          float d[4] = {0.f, 0.f, 0.f, 0.f};
          mma_tf32(d, al, bh[j]);  // small terms first
          mma_tf32(d, ah, bl[j]);
          mma_tf32(d, ah, bh[j]);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[i][j][e] += d[e];
        }
      }
    }
  }
  cp_wait<0>();
  // accumulator fragment e of tile (i, j): row g (+8 for e >= 2), column 2q (+1 for odd e)
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int e2 = 0; e2 < 2; ++e2) {
      const int64_t gm = m0 + wm + i * 16 + g + e2 * 8;
      if (gm >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t gn0 = n0 + wn + j * 8 + 2 * q;
        float v[2];
#pragma unroll
        for (int e1 = 0; e1 < 2; ++e1) {
          const int64_t gn = gn0 + e1;
          v[e1] = alpha * acc[i][j][e2 * 2 + e1];
          if (gn < N) {
            if (beta != 0.f) v[e1] += beta * load_f(C, cdt, gm * scm + gn * scn);
            if (cbias) v[e1] += load_f(cbias, cbias_dt, gn);  // the score bias of column gn (the S GEMM)
          }
        }
        const int64_t off = gm * scm + gn0 * scn;
        float* dst = static_cast<float*>(C) + off;
        if (cdt == SWVR_F32 && scn == 1 && gn0 + 1 < N && (reinterpret_cast<uintptr_t>(dst) & 7u) == 0) {
          *reinterpret_cast<float2*>(dst) = make_float2(v[0], v[1]);
        } else {
#pragma unroll
          for (int e1 = 0; e1 < 2; ++e1)
            if (gn0 + e1 < N) store_f(C, cdt, off + e1 * scn, v[e1]);
        }
      }
    }
  }
}

// 16-byte staging needs: unit stride along the staged rows, a 16-byte aligned base, a row
// pitch that is a multiple of 4 floats and an extent along the rows that is a multiple of 4
// (a chunk is wholly inside or outside).
static bool tf32x3_ok(const float* A, int64_t sam, int64_t sak, int64_t M, const float* B, int64_t sbk, int64_t sbn,
                      int64_t N, int64_t K) {
  const bool a_ok = sak == 1 ? vec4_ok(A, sam, sak, K) : (sam == 1 && vec4_ok(A, sak, sam, M));
  const bool b_ok = sbn == 1 ? vec4_ok(B, sbk, sbn, N) : (sbk == 1 && vec4_ok(B, sbn, sbk, K));
  return a_ok && b_ok;
}

template <bool AK, bool BNC>
static cudaError_t launch_tf32x3(cudaStream_t st, dim3 grid, int64_t M, int64_t N, int64_t K, float alpha,
                                 const float* A, int64_t sam, int64_t sak, const float* B, int64_t sbk, int64_t sbn,
                                 float beta, void* C, int cdt, int64_t scm, int64_t scn, int64_t kper,
                                 int64_t zstride, const void* cbias, int cbias_dt) {
  auto kern = gemm_tf32x3_kernel<AK, BNC>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, tf32x3::SMEM);
  if (e != cudaSuccess) return e;
  kern<<<grid, 256, tf32x3::SMEM, st>>>(M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt, scm, scn, kper,
                                        zstride, cbias, cbias_dt);
  return cudaGetLastError();
}

static cudaError_t launch_tf32x3_any(cudaStream_t st, dim3 grid, int64_t M, int64_t N, int64_t K, float alpha,
                                     const float* A, int64_t sam, int64_t sak, const float* B, int64_t sbk,
                                     int64_t sbn, float beta, void* C, int cdt, int64_t scm, int64_t scn,
                                     int64_t kper, int64_t zstride, const void* cbias = nullptr,
                                     int cbias_dt = SWVR_F32) {
  if (sak == 1)
    return sbn == 1 ? launch_tf32x3<true, true>(st, grid, M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt, scm,
                                                 scn, kper, zstride, cbias, cbias_dt)
                    : launch_tf32x3<true, false>(st, grid, M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt,
                                                  scm, scn, kper, zstride, cbias, cbias_dt);
  return sbn == 1 ? launch_tf32x3<false, true>(st, grid, M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt, scm,
                                                scn, kper, zstride, cbias, cbias_dt)
                  : launch_tf32x3<false, false>(st, grid, M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt,
                                                 scm, scn, kper, zstride, cbias, cbias_dt);
}

// C = alpha * sum_z part[z] + beta * C, the K splits summed in z order.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int splits, int64_t M, int64_t N, float alpha,
                                     float beta, void* C, int cdt, int64_t scm, int64_t scn) {
  const int64_t MN = M * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < MN;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float t = 0.f;
    for (int z = 0; z < splits; ++z) t += part[z * MN + i];
    const int64_t off = (i / N) * scm + (i % N) * scn;
    float v = alpha * t;
    if (beta != 0.f) v += beta * load_f(C, cdt, off);
    store_f(C, cdt, off, v);
  }
}

// Floats of split-K partials the fp32 kernels may use for a GEMM whose output is M x N.
constexpr int64_t kSplitKMaxFloats = int64_t(16) << 20;  // 64 MB
inline int64_t splitk_floats(int64_t M, int64_t N) {
  const int64_t want = 16 * M * N;
  return want < kSplitKMaxFloats ? want : kSplitKMaxFloats;
}

template <typename T>
cudaError_t gemm(cudaStream_t st, int64_t M, int64_t N, int64_t K, T alpha, const T* A, int64_t sam, int64_t sak,
                 const T* B, int64_t sbk, int64_t sbn, T beta, void* C, int cdt, int64_t scm, int64_t scn) {
  if (M == 0 || N == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>(ceil_div(N, BN)), static_cast<unsigned>(ceil_div(M, BM)));
  // A: unit stride along K (sak == 1) or along M (sam == 1); B: along N (sbn == 1) or along K
  const bool vec_a = sak == 1 ? vec4_ok(A, sam, sak, K) : vec4_ok(A, sak, sam, M);
  const bool vec_b = sbn == 1 ? vec4_ok(B, sbk, sbn, N) : vec4_ok(B, sbn, sbk, K);
  if constexpr (sizeof(T) == 4) {
    // the tensor-core kernel where its 16-byte staging applies, else the CUDA-core one
    if (tf32x3_ok(A, sam, sak, M, B, sbk, sbn, N, K))
      return launch_tf32x3_any(st, grid, M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt, scm, scn, K, 0);
  }
  gemm_kernel<T><<<grid, 256, 0, st>>>(M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt, scm, scn, vec_a, vec_b);
  return cudaGetLastError();
}

// A GEMM whose output is narrow (the P.E and dE products, D columns) and whose K is long: its
// 128 x 128 tiles would leave most SMs idle, so the fp32 kernel splits K into up to 16
// ranges, about four 128 x 128 tiles per SM in all, each range writing an fp32 slice of
// `part` (splitk_floats(M, N) floats), summed in order by splitk_reduce_kernel.  (Splitting
// the dh and dW GEMMs as well, whose tiles already fill 86 % of two block slots per SM, made
// the fp32 step 1.5 ms slower.)  fp64, or a layout the tensor-core kernel does not stage,
// takes gemm().
template <typename T>
cudaError_t gemm_split(cudaStream_t st, int64_t M, int64_t N, int64_t K, T alpha, const T* A, int64_t sam,
                        int64_t sak, const T* B, int64_t sbk, int64_t sbn, T beta, void* C, int cdt, int64_t scm,
                        int64_t scn, float* part) {
  if constexpr (sizeof(T) == 4) {
    if (M > 0 && N > 0 && part && tf32x3_ok(A, sam, sak, M, B, sbk, sbn, N, K)) {
      const int64_t tiles = ceil_div(M, tf32x3::TM) * ceil_div(N, tf32x3::TN);
      int64_t splits = std::min<int64_t>({int64_t(16), ceil_div(4 * kNumSMsB200, tiles), K / 256,
                                          splitk_floats(M, N) / (M * N)});
      if (splits >= 2) {
        const int64_t kper = round_up(ceil_div(K, splits), tf32x3::TK);
        splits = ceil_div(K, kper);
        dim3 grid(static_cast<unsigned>(ceil_div(N, tf32x3::TN)), static_cast<unsigned>(ceil_div(M, tf32x3::TM)),
                  static_cast<unsigned>(splits));
        cudaError_t e = launch_tf32x3_any(st, grid, M, N, K, 1.f, A, sam, sak, B, sbk, sbn, 0.f, part, SWVR_F32, N, 1,
                                          kper, M * N);
        if (e != cudaSuccess) return e;
        splitk_reduce_kernel<<<static_cast<unsigned>(std::min<int64_t>(ceil_div(M * N, 256), 8 * kNumSMsB200)), 256, 0,
                               st>>>(part, static_cast<int>(splits), M, N, alpha, beta, C, cdt, scm, scn);
        return cudaGetLastError();
      }
    }
  }
  return gemm<T>(st, M, N, K, alpha, A, sam, sak, B, sbk, sbn, beta, C, cdt, scm, scn);
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

inline unsigned grid_for(int64_t n, int threads = 256) {
  int64_t g = ceil_div(n, threads);
  if (g < 1) g = 1;
  if (g > 4096) g = 4096;
  return static_cast<unsigned>(g);
}

// S[N, C] = alpha * A B + bias[v0 : v0 + C] (the bias of the chunk's scores, chunked.py:77-78):
// added in the fp32 tensor-core GEMM's epilogue where that kernel runs, else by add_bias_kernel.
template <typename T>
static cudaError_t gemm_bias(cudaStream_t st, int64_t M, int64_t N, int64_t K, T alpha, const T* A, int64_t sam,
                             int64_t sak, const T* B, int64_t sbk, int64_t sbn, T* S, int adt, const void* bias,
                             int bdt, int64_t v0) {
  if constexpr (sizeof(T) == 4) {
    if (bias && M > 0 && N > 0 && tf32x3_ok(A, sam, sak, M, B, sbk, sbn, N, K)) {
      dim3 grid(static_cast<unsigned>(ceil_div(N, BN)), static_cast<unsigned>(ceil_div(M, BM)));
      return launch_tf32x3_any(st, grid, M, N, K, alpha, A, sam, sak, B, sbk, sbn, 0.f, S, adt, N, 1, K, 0,
                               static_cast<const char*>(bias) + v0 * static_cast<int64_t>(dtype_size(bdt)), bdt);
    }
  }
  cudaError_t e = gemm<T>(st, M, N, K, alpha, A, sam, sak, B, sbk, sbn, T(0), S, adt, N, 1);
  if (e != cudaSuccess || !bias) return e;
  add_bias_kernel<T><<<grid_for(M * N), 256, 0, st>>>(S, M, N, bias, bdt, v0);
  return cudaGetLastError();
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

// gb[v0 + c] = sum_n G[n, c]  (chunked.py:135-136), in a fixed order per column: a block of
// 256 threads takes 32 columns; thread (r, c) of the 8 x 32 sums rows r, r + 8, r + 16, ...
// (a warp reads 32 consecutive columns of one row), and the 8 row sums of a column are
// added in r order.
template <typename T>
__global__ void colsum_kernel(const T* G, int64_t N, int64_t C, void* gb, int gdt, int64_t v0) {
  __shared__ T part[8][33];
  const int cl = threadIdx.x % 32, r = threadIdx.x / 32;
  const int64_t c = blockIdx.x * 32LL + cl;
  T s = 0;
  if (c < C) {
#pragma unroll 8
    for (int64_t n = r; n < N; n += 8) s += G[n * C + c];
  }
  part[r][cl] = s;
  __syncthreads();
  if (r == 0 && c < C) {
    T t = part[0][cl];
#pragma unroll
    for (int i = 1; i < 8; ++i) t += part[i][cl];
    store_d(gb, gdt, v0 + c, static_cast<double>(t));
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


// ---------------------------------------------------------------------------------------- host
size_t fwd_workspace(const swvr_problem& p) {
  const size_t es = p.compute_dtype == SWVR_F64 ? 8 : 4;
  const int64_t C = p.chunk < p.vocab ? p.chunk : (p.vocab > 0 ? p.vocab : 1);
  const size_t part = es == 4 ? align_up(4 * splitk_floats(p.n_tokens, p.embed_dim), 256) : 0;  // P.E split K
  return align_up(es * p.n_tokens * C, 256) + 2 * align_up(es * p.n_tokens, 256) +
         align_up(es * p.n_tokens * p.embed_dim, 256) + part + 256;
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
  w += align_up(sizeof(T) * N * D, 256);
  float* part = sizeof(T) == 4 ? reinterpret_cast<float*>(w) : nullptr;  // split-K partials of P.E
  const T* h = static_cast<const T*>(p.h);
  const T* W = static_cast<const T*>(p.W);
  const T* E = static_cast<const T*>(p.E);
  const int adt = sizeof(T) == 8 ? SWVR_F64 : SWVR_F32;
  fwd_init_kernel<T><<<grid_for(N * D > N ? N * D : N), 256, 0, st>>>(m, l, acc, N, D);
  for (int64_t v0 = 0; v0 < V; v0 += C) {
    const int64_t c = (V - v0) < C ? (V - v0) : C;
    cudaError_t e = gemm_bias<T>(st, N, c, K, static_cast<T>(p.logit_scale), h, p.ldh, 1, W + v0 * p.ldw, 1, p.ldw,
                                 S, adt, p.bias, p.bias_dtype, v0);
    if (e != cudaSuccess) return SWVR_ERR_CUDA;
    if (N > 0) fwd_update_kernel<T><<<static_cast<unsigned>(N), 256, 0, st>>>(S, c, m, l, acc, D);
    e = gemm_split<T>(st, N, D, c, T(1), S, c, 1, E + v0 * p.lde, p.lde, 1, T(1), acc, adt, D, 1, part);
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
  if (es == 4 && g.grad_E) b += align_up(4 * splitk_floats(C, p.embed_dim), 256);  // dE split K
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
  if (g.grad_h && !g.grad_h_acc) w += align_up(sizeof(T) * N * K, 256);
  float* part = sizeof(T) == 4 ? reinterpret_cast<float*>(w) : nullptr;  // split-K partials (bwd_workspace)
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
    if (gemm_bias<T>(st, N, c, K, s, h, p.ldh, 1, W + v0 * p.ldw, 1, p.ldw, S, adt, p.bias, p.bias_dtype, v0) !=
        cudaSuccess)
      return SWVR_ERR_CUDA;
    bwd_p_kernel<T><<<grid_for(N * c), 256, 0, st>>>(S, lse, N, c);
    // G = (gO E_c^T - delta) * P  (chunked.py:134)
    if (gemm<T>(st, N, c, D, T(1), gO, D, 1, E + v0 * p.lde, 1, p.lde, T(0), G, adt, c, 1) != cudaSuccess)
      return SWVR_ERR_CUDA;
    bwd_gs_kernel<T><<<grid_for(N * c), 256, 0, st>>>(S, G, delta, N, c);
    if (need_b)
      colsum_kernel<T><<<static_cast<unsigned>(ceil_div(c, 32)), 256, 0, st>>>(G, N, c, g.grad_bias, g.grad_bias_dtype,
                                                                              v0);
    // gE_c = P^T gO  (chunked.py:137-138)
    if (need_E &&
        gemm_split<T>(st, c, D, N, T(1), S, 1, c, gO, D, 1, T(0), static_cast<char*>(g.grad_E) +
                           static_cast<size_t>(v0 * g.ld_grad_E) * dtype_size(g.grad_E_dtype),
                       g.grad_E_dtype, g.ld_grad_E, 1, part) != cudaSuccess)
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
