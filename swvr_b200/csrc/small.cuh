// Small memory-bound kernels (combine, reductions, prologue, loss epilogue, casts).
#pragma once
#include "common.cuh"

namespace swvr {
namespace small {
// pdl: launch with programmatic stream serialization (the previous kernel in the stream is
// the one producing this kernel's input; the kernel waits for it before reading).
cudaError_t combine(int acc_dt, int S, int64_t N, int64_t D, const void* m2, const void* l, const void* acc, int mode,
                    int splits, int tile_rows, void* O, void* lse, void* m2o, void* lo, void* acco, bool pdl,
                    cudaStream_t st);
cudaError_t reduce_de_db(const float* part_de, const float* part_db, int TS, int per_t, int NT, int v_begin, int rows,
                         int tile_rows, int64_t D, void* gE, int gE_dt, int64_t ld_gE, void* gb, int gb_dt, bool pdl,
                         cudaStream_t st);
// Launch a kernel whose bounded wait expires after limit_ns (records kErrSelftest | 1).
cudaError_t wait_selftest(uint64_t limit_ns, cudaStream_t st);
cudaError_t prologue(bool bf16, const float* O, const float* gO, const float* glse, int64_t N, int D, int DP,
                     float* delta, void* gOc, cudaStream_t st);
cudaError_t cast_f32(const float* src, void* dst, int dt, int64_t n, cudaStream_t st);
cudaError_t zero_rows(void* dst, int dt, int64_t rows, int64_t cols, int64_t ld, cudaStream_t st);
cudaError_t mse_fwd(int dt, int64_t N, int64_t D, const void* O, const void* lse, const void* t, const void* w,
                    double z, int red, void* out, void* stats, cudaStream_t st);
cudaError_t mse_bwd(int dt, int64_t N, int64_t D, const void* O, const void* lse, const void* t, const void* w,
                    double z, int red, const void* gout, const void* stats, void* gO, void* glse, void* gt, void* gw,
                    cudaStream_t st);
}  // namespace small
}  // namespace swvr
