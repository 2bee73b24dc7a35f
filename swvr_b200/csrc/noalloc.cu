// swvr_fwd_noalloc: the tensor-core forward with its scratch memory in a file-scope device
// array instead of a caller-provided workspace.
//
// Some callers cannot allocate device memory when they call the readout: an inference
// server or a host engine that plans every byte of device memory up front and hands
// plugins no allocator, or an FFI host (cgo, JNI, N-API) whose runtime owns the CUDA
// context and forbids its plugins from calling cudaMalloc, which can synchronise the
// device and fragments a pool the host manages.  For them this entry point takes only
// the problem, the outputs and a stream.
//
// The scratch (the per-split online-softmax state the forward kernel writes before the
// combine kernel merges it) lives in g_fwd_scratch below: kFwdScratchBytes (16 MiB) per
// GPU, held by every GPU that loads the library until the process exits.  Problems whose
// state does not fit are rejected with SWVR_ERR_UNSUPPORTED and a message; the planner
// first lowers the number of vocabulary splits (down to one) to make it fit.
//
// Host code never dereferences g_fwd_scratch: in host code its name is only a stand-in.
// The first call on each device, with that device current, looks up the array's device
// address with cudaGetSymbolAddress and caches it with the current context (a new context on
// that device, e.g. after cudaDeviceReset, is looked up again); make that first call before
// any stream capture.  Every call on a device shares the one array and leaves its last contents
// there; each call writes every slot it later reads, so nothing needs clearing.  Calls
// whose work overlaps on the GPU (different streams, or different host threads without
// ordering) race on the array and must be serialised by the caller.
#include <mutex>

#include "common.cuh"
#include "small.cuh"
#include "tc.cuh"

namespace swvr {

constexpr size_t kFwdScratchBytes = size_t(16) << 20;

static __device__ __align__(256) unsigned char g_fwd_scratch[kFwdScratchBytes];

constexpr int kMaxDevices = 64;
static std::mutex g_scratch_mu;
// Per device ordinal: the context the address was looked up in, and the address.  A new
// context on the same ordinal (after cudaDeviceReset, or a host that destroys and recreates
// its primary context) gets a fresh lookup instead of a stale address.
static CUcontext g_scratch_ctx[kMaxDevices] = {};
static void* g_scratch_ptr[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

static CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &ptr, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

// Device address of g_fwd_scratch on the current device, looked up once per device and
// context (cudaGetSymbolAddress also makes the device's primary context current if no
// context is).
static int fwd_scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SWVR_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(SWVR_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  CtxGetCurrentFn get_ctx = ctx_get_current();
  if (!get_ctx) return fail(SWVR_ERR_CUDA, "cuCtxGetCurrent is not available from the driver");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return fail(SWVR_ERR_CUDA, "cuCtxGetCurrent failed");
  if (!g_scratch_ptr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_fwd_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(SWVR_ERR_CUDA, "cudaGetSymbolAddress(g_fwd_scratch) failed: %s", cudaGetErrorString(e));
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return fail(SWVR_ERR_CUDA, "no current CUDA context");
    g_scratch_ctx[dev] = ctx;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return SWVR_OK;
}

// The forward plan restricted to the static scratch: as many vocabulary splits as fit.
static int plan_fwd_static(const swvr_problem& p, FwdPlan* out) {
  const size_t per_unit = align_up(tc::kFwdTokenTile * 4, 256) * 2 + align_up(size_t(tc::kFwdTokenTile) * p.embed_dim * 4, 256);
  const size_t max_units = (kFwdScratchBytes - 3 * 256) / per_unit;
  const int64_t MT = ceil_div(p.n_tokens, tc::kFwdTokenTile);
  if (static_cast<size_t>(MT) > max_units)
    return fail(SWVR_ERR_UNSUPPORTED,
                "swvr_fwd_noalloc: N=%lld, D=%lld needs %zu bytes of scratch even unsplit; the static scratch holds "
                "%zu bytes (at most %zu %d-token tiles of this D)",
                (long long)p.n_tokens, (long long)p.embed_dim, static_cast<size_t>(MT) * per_unit, kFwdScratchBytes,
                max_units, tc::kFwdTokenTile);
  const FwdPlan f = plan_fwd_units(p, static_cast<int>(max_units / static_cast<size_t>(MT)));
  if (f.bytes > kFwdScratchBytes)
    return fail(SWVR_ERR_UNSUPPORTED, "swvr_fwd_noalloc: plan needs %zu bytes of scratch, the static scratch holds %zu",
                f.bytes, kFwdScratchBytes);
  *out = f;
  return SWVR_OK;
}

}  // namespace swvr

extern "C" int swvr_fwd_noalloc(const swvr_problem* p, void* O, void* lse, void* stream) {
  using namespace swvr;
  SWVR_TRY(validate(p));
  if (!is_tc(p->compute_dtype))
    return fail(SWVR_ERR_UNSUPPORTED, "swvr_fwd_noalloc runs the bf16 / fp16 tensor-core forward only");
  if (p->n_tokens > 0 && (!O || !lse)) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL output");
  if (p->n_tokens == 0) return SWVR_OK;
  if (p->vocab == 0) return fail(SWVR_ERR_UNSUPPORTED, "empty vocabulary (callers handle V == 0)");
  FwdPlan f;
  SWVR_TRY(plan_fwd_static(*p, &f));
  void* scratch = nullptr;
  SWVR_TRY(fwd_scratch_address(&scratch));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  tc::FwdParams prm;
  SWVR_TRY(tc_fwd_launch(*p, f, static_cast<char*>(scratch), st, &prm));
  ProfScope ps_c(kProfCombine, st);
  SWVR_CUDA(small::combine(SWVR_F32, f.splits, p->n_tokens, p->embed_dim, prm.part_m2, prm.part_l, prm.part_acc, 0,
                           f.splits, tc::kFwdTokenTile, O, lse, nullptr, nullptr, nullptr, /*pdl=*/true, st));
  return SWVR_OK;
}
