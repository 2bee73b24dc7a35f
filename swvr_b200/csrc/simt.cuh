// Exact SIMT CUDA path (fp32 / fp64 compute).
#pragma once
#include "common.cuh"

namespace swvr {
namespace simt {
size_t fwd_workspace(const swvr_problem& p);
// Writes O/lse when not null, and the log2-unit partial state (m2, l, acc) when not null.
int fwd(const swvr_problem& p, void* O, void* lse, void* m2, void* l, void* acc, void* ws, cudaStream_t st);
size_t bwd_workspace(const swvr_problem& p, const swvr_grads& g);
int bwd(const swvr_problem& p, const swvr_grads& g, void* ws, cudaStream_t st);
}  // namespace simt
}  // namespace swvr
