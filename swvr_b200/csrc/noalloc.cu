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
// address with cudaGetSymbolAddress and caches it; make that first call before any stream
// capture.  Every call on a device shares the one array and leaves its last contents
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
static void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_fwd_scratch on the current device (looked up once per device).
static int fwd_scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SWVR_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(SWVR_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_fwd_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(SWVR_ERR_CUDA, "cudaGetSymbolAddress(g_fwd_scratch) failed: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return SWVR_OK;
}

// The forward plan restricted to the static scratch: as many vocabulary splits as fit.
static int plan_fwd_static(const swvr_problem& p, FwdPlan* out) {
  FwdPlan f{};
  const int sms = num_sms();
  f.DP = p.embed_dim <= 64 ? 64 : 128;
  f.BV = tc::fwd_vocab_tile(f.DP);
  f.MT = static_cast<int>(ceil_div(p.n_tokens, 128));
  f.VT = static_cast<int>(ceil_div(p.vocab, f.BV));
  const size_t per_unit = align_up(128 * 4, 256) * 2 + align_up(size_t(128) * p.embed_dim * 4, 256);
  const size_t max_units = (kFwdScratchBytes - 3 * 256) / per_unit;
  if (static_cast<size_t>(f.MT) > max_units)
    return fail(SWVR_ERR_UNSUPPORTED,
                "swvr_fwd_noalloc: N=%lld, D=%lld needs %zu bytes of scratch even unsplit; the static scratch holds "
                "%zu bytes (at most %zu 128-token tiles of this D)",
                (long long)p.n_tokens, (long long)p.embed_dim, static_cast<size_t>(f.MT) * per_unit, kFwdScratchBytes,
                max_units);
  const int smax = std::max(1, std::min<int>(std::min(f.VT, 64), static_cast<int>(max_units / f.MT)));
  int best_s = 1;
  int64_t best_cost = -1;
  for (int s = 1; s <= smax; ++s) {
    const int64_t cost = ceil_div(static_cast<int64_t>(f.MT) * s, sms) * ceil_div(f.VT, s);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_s = s;
    }
  }
  f.per = static_cast<int>(ceil_div(std::max(f.VT, 1), best_s));
  f.splits = static_cast<int>(ceil_div(std::max(f.VT, 1), f.per));
  f.units = f.MT * f.splits;
  f.grid = std::max(1, std::min(f.units, sms));
  const size_t rows = static_cast<size_t>(f.units) * 128;
  f.off_m2 = 0;
  f.off_l = align_up(rows * 4, 256);
  f.off_acc = f.off_l + align_up(rows * 4, 256);
  f.bytes = f.off_acc + align_up(rows * p.embed_dim * 4, 256);
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
  const bool bf16 = p->compute_dtype == SWVR_BF16;
  tc::FwdMaps maps;
  SWVR_TRY(make_map(&maps.h, p->h, p->compute_dtype, p->hidden, p->n_tokens, p->ldh * 2, 64, 128));
  SWVR_TRY(make_map(&maps.w, p->W, p->compute_dtype, p->hidden, p->vocab, p->ldw * 2, 64, f.BV));
  SWVR_TRY(make_map(&maps.e, p->E, p->compute_dtype, p->embed_dim, p->vocab, p->lde * 2, 64, f.BV));
  char* w = static_cast<char*>(scratch);
  tc::FwdParams prm{};
  prm.N = static_cast<int>(p->n_tokens);
  prm.K = static_cast<int>(p->hidden);
  prm.V = static_cast<int>(p->vocab);
  prm.D = static_cast<int>(p->embed_dim);
  prm.sc2 = static_cast<float>(p->logit_scale * 1.4426950408889634);
  prm.bias = p->bias;
  prm.bias_dt = p->bias_dtype;
  prm.MT = f.MT;
  prm.VT = f.VT;
  prm.splits = f.splits;
  prm.per = f.per;
  prm.units = f.units;
  prm.part_m2 = reinterpret_cast<float*>(w + f.off_m2);
  prm.part_l = reinterpret_cast<float*>(w + f.off_l);
  prm.part_acc = reinterpret_cast<float*>(w + f.off_acc);
  {
    ProfScope ps(kProfFwd, st);
    SWVR_CUDA(tc::launch_fwd_kernel(bf16, f.DP, maps, prm, f.grid, st));
  }
  ProfScope ps_c(kProfCombine, st);
  SWVR_CUDA(small::combine(SWVR_F32, f.splits, p->n_tokens, p->embed_dim, prm.part_m2, prm.part_l, prm.part_acc, 0,
                           f.splits, O, lse, nullptr, nullptr, nullptr, st));
  return SWVR_OK;
}
