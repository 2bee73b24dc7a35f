// Single translation unit of libswvr_b200.so (built by swvr_b200/build.py).
#include "simt.cu"
#include "small.cu"
#include "norm.cu"
#include "tc_fwd.cu"
#include "tc_bwd.cu"
#include "tc_gemm.cu"
#include "abi.cu"
#include "noalloc.cu"
