// extern "C" entry points of libswvr_b200.so (declared in include/swvr_b200.h): argument
// validation, work planning, TMA descriptor construction and the backward chunk loop.
// No device memory is allocated here; callers pass outputs and workspaces.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "ptx.cuh"
#include "simt.cuh"
#include "small.cuh"
#include "tc.cuh"

namespace swvr {

static thread_local std::string t_err;

static int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

#define SWVR_CUDA(call)                                                                            \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess) return fail(SWVR_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

#define SWVR_TRY(call)          \
  do {                          \
    int rc_ = (call);           \
    if (rc_ != SWVR_OK) return rc_; \
  } while (0)

static int num_sms() {
  int dev = 0, n = kNumSMsB200;
  if (cudaGetDevice(&dev) != cudaSuccess) return kNumSMsB200;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kNumSMsB200;
  return n > 0 ? n : kNumSMsB200;
}


// ---------------------------------------------------------------------------- launch accounting
enum ProfKind { kProfFwd = 0, kProfBwdScores, kProfGemm, kProfCombine, kProfReduce, kProfPrologue, kProfCast,
                kProfMse, kProfSimt, kProfNorm, kProfKinds };
static const char* kProfNames[kProfKinds] = {"fwd_kernel",      "bwd_scores_kernel", "gemm_kernel",
                                             "combine_kernel",  "reduce_de_db_kernel", "prologue_kernel",
                                             "cast_kernel",     "mse_kernel",        "simt_kernels",
                                             "rmsnorm_kernels"};
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static int64_t g_prof_launches[kProfKinds];
struct ProfPending {
  int kind;
  cudaEvent_t e0, e1;
};
static std::vector<ProfPending> g_prof_pending;
static std::vector<cudaEvent_t> g_prof_pool;

static cudaEvent_t prof_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Brackets one kernel launch (or a group, `count` launches) with events when profiling.
struct ProfScope {
  int kind;
  int64_t count;
  cudaStream_t st;
  cudaEvent_t e0 = nullptr;
  ProfScope(int k, cudaStream_t s, int64_t n = 1) : kind(k), count(n), st(s) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on) return;
    e0 = prof_event();
    if (e0) cudaEventRecord(e0, st);
  }
  ~ProfScope() {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    if (!g_prof_on || !e0) return;
    cudaEvent_t e1 = prof_event();
    if (!e1) return;
    cudaEventRecord(e1, st);
    g_prof_launches[kind] += count;
    g_prof_pending.push_back({kind, e0, e1});
  }
};

static bool is_tc(int dt) { return dt == SWVR_BF16 || dt == SWVR_F16; }
static int acc_dtype_of(int cdt) { return cdt == SWVR_F64 ? SWVR_F64 : SWVR_F32; }

// ---------------------------------------------------------------------------- TMA descriptors
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  return fn;
}

// 2-D row-major tensor [outer, inner] with a row pitch of row_bytes; 128-byte swizzle, zero
// fill out of bounds.
static int make_map(CUtensorMap* m, const void* base, int dt, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                    uint32_t box_inner, uint32_t box_outer, int swizzle_bytes = 128) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(SWVR_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_bytes & 15u) != 0)
    return fail(SWVR_ERR_UNSUPPORTED, "TMA operand not 16-byte aligned (base %p, row pitch %llu bytes)", base,
                static_cast<unsigned long long>(row_bytes));
  const CUtensorMapDataType t = dt == SWVR_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : dt == SWVR_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  cuuint64_t dims[2] = {inner > 0 ? inner : 1, outer > 0 ? outer : 1};
  cuuint64_t strides[1] = {row_bytes > 0 ? row_bytes : 16};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = fn(m, t, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SWVR_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled failed (%d): dims {%llu, %llu}, pitch %llu, box {%u, %u}",
                static_cast<int>(r), static_cast<unsigned long long>(inner), static_cast<unsigned long long>(outer),
                static_cast<unsigned long long>(row_bytes), box_inner, box_outer);
  return SWVR_OK;
}

// ---------------------------------------------------------------------------- validation
static int validate(const swvr_problem* p) {
  if (!p) return fail(SWVR_ERR_INVALID_ARGUMENT, "problem is NULL");
  if (p->n_tokens < 0 || p->hidden < 0 || p->vocab < 0 || p->embed_dim < 0)
    return fail(SWVR_ERR_INVALID_ARGUMENT, "negative size");
  if (p->n_tokens >= (1ll << 31) || p->vocab >= (1ll << 31) || p->hidden >= (1ll << 31) || p->embed_dim >= (1ll << 31))
    return fail(SWVR_ERR_UNSUPPORTED, "sizes must be below 2^31");
  if (p->compute_dtype < SWVR_F32 || p->compute_dtype > SWVR_F16)
    return fail(SWVR_ERR_INVALID_ARGUMENT, "unknown compute dtype %d", p->compute_dtype);
  if (p->bias && (p->bias_dtype < SWVR_F32 || p->bias_dtype > SWVR_F16))
    return fail(SWVR_ERR_INVALID_ARGUMENT, "unknown bias dtype %d", p->bias_dtype);
  if (p->chunk <= 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "chunk must be positive, got %lld", (long long)p->chunk);
  if (p->ldh < p->hidden || p->ldw < p->hidden || p->lde < p->embed_dim)
    return fail(SWVR_ERR_INVALID_ARGUMENT, "row stride smaller than the row length");
  if ((p->n_tokens > 0 && p->hidden > 0 && !p->h) || (p->vocab > 0 && p->hidden > 0 && !p->W) ||
      (p->vocab > 0 && p->embed_dim > 0 && !p->E))
    return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL input pointer");
  if (is_tc(p->compute_dtype)) {
    if (p->embed_dim < 1 || p->embed_dim > 256)
      return fail(SWVR_ERR_UNSUPPORTED, "tensor-core path supports 1 <= D <= 256, got %lld", (long long)p->embed_dim);
    if (p->hidden < 8 || (p->hidden % 8) != 0 || (p->ldh % 8) != 0 || (p->ldw % 8) != 0 || (p->lde % 8) != 0)
      return fail(SWVR_ERR_UNSUPPORTED, "tensor-core path needs K and row strides that are multiples of 8 elements");
    if ((reinterpret_cast<uintptr_t>(p->h) | reinterpret_cast<uintptr_t>(p->W) | reinterpret_cast<uintptr_t>(p->E)) & 15u)
      return fail(SWVR_ERR_UNSUPPORTED, "tensor-core path needs 16-byte aligned h, W and E");
  }
  return SWVR_OK;
}

// ---------------------------------------------------------------------------- forward plan
// Token tiles per group of the forward's unit order (tc::fwd_unit).  32 keeps about 74 / 32 =
// 2.3 vocabulary splits streaming at a time on the 74 pairs: measured at c2 (A/B on one B200,
// two rounds) the forward took 9.6-9.7 ms against 10.1-10.2 ms with every split of a token tile
// in a row (1) and 10.8 ms with one split for all token tiles (64); 8 and 16 fell in between.
// SWVR_FWD_GROUP overrides it.
static int fwd_group(int MT) {
  static const int v = [] {
    const char* s = std::getenv("SWVR_FWD_GROUP");
    return s ? std::max(1, std::atoi(s)) : 32;
  }();
  return std::max(1, std::min(v, std::max(MT, 1)));
}

struct FwdPlan {
  int DP, MT, VT, splits, per, units, pairs;
  size_t off_m2, off_l, off_acc, bytes;
};

// Work units are (256-token tile, vocabulary split) pairs run by CTA pairs; the split count
// minimises the rounds over the co-resident pairs times the tiles per unit.  max_splits
// bounds the partial-state slots (units * 256 rows).
static FwdPlan plan_fwd_units(const swvr_problem& p, int max_splits) {
  FwdPlan f{};
  f.pairs = std::max(1, num_sms() / 2);
  f.MT = static_cast<int>(ceil_div(p.n_tokens, tc::kFwdTokenTile));
  f.DP = p.embed_dim <= 64 ? 64 : (p.embed_dim <= 128 ? 128 : 256);
  f.VT = static_cast<int>(ceil_div(p.vocab, tc::fwd_vocab_tile(f.DP)));
  int best_s = 1;
  int64_t best_cost = -1;
  const int smax = std::max(1, std::min(std::min(f.VT, 64), max_splits));
  for (int s = 1; s <= smax; ++s) {
    const int64_t cost = ceil_div(static_cast<int64_t>(f.MT) * s, f.pairs) * ceil_div(f.VT, s);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_s = s;
    }
  }
  f.per = static_cast<int>(ceil_div(std::max(f.VT, 1), best_s));
  f.splits = static_cast<int>(ceil_div(std::max(f.VT, 1), f.per));
  f.units = f.MT * f.splits;
  const size_t rows = static_cast<size_t>(f.units) * tc::kFwdTokenTile;
  f.off_m2 = 0;
  f.off_l = align_up(rows * 4, 256);
  f.off_acc = f.off_l + align_up(rows * 4, 256);
  f.bytes = f.off_acc + align_up(rows * p.embed_dim * 4, 256) + 256;
  return f;
}

static FwdPlan plan_fwd(const swvr_problem& p) { return plan_fwd_units(p, 64); }

// Tensor maps and kernel parameters of the tensor-core forward; the caller provides the
// partial-state scratch (f.bytes).
static int tc_fwd_launch(const swvr_problem& p, const FwdPlan& f, char* scratch, cudaStream_t st,
                         tc::FwdParams* out) {
  const bool bf16 = p.compute_dtype == SWVR_BF16;
  tc::FwdMaps maps;
  SWVR_TRY(make_map(&maps.h, p.h, p.compute_dtype, p.hidden, p.n_tokens, p.ldh * 2, 64, 128));
  const int BV = tc::fwd_vocab_tile(f.DP);
  SWVR_TRY(make_map(&maps.w, p.W, p.compute_dtype, p.hidden, p.vocab, p.ldw * 2, 64, BV / 2));
  SWVR_TRY(make_map(&maps.e, p.E, p.compute_dtype, p.embed_dim, p.vocab, p.lde * 2, 64, BV));
  tc::FwdParams prm{};
  prm.N = static_cast<int>(p.n_tokens);
  prm.K = static_cast<int>(p.hidden);
  prm.V = static_cast<int>(p.vocab);
  prm.D = static_cast<int>(p.embed_dim);
  prm.sc2 = static_cast<float>(p.logit_scale * 1.4426950408889634);
  prm.bias = p.bias;
  prm.bias_dt = p.bias_dtype;
  prm.MT = f.MT;
  prm.VT = f.VT;
  prm.splits = f.splits;
  prm.per = f.per;
  prm.units = f.units;
  prm.gm = fwd_group(f.MT);
  prm.part_m2 = reinterpret_cast<float*>(scratch + f.off_m2);
  prm.part_l = reinterpret_cast<float*>(scratch + f.off_l);
  prm.part_acc = reinterpret_cast<float*>(scratch + f.off_acc);
  {
    ProfScope ps(kProfFwd, st);
    SWVR_CUDA(tc::launch_fwd_kernel(bf16, f.DP, maps, prm, f.pairs, st));
  }
  *out = prm;
  return SWVR_OK;
}

static int tc_fwd(const swvr_problem& p, void* O, void* lse, void* m2o, void* lo, void* acco, void* ws, size_t wsb,
                  cudaStream_t st) {
  const FwdPlan f = plan_fwd(p);
  if (wsb < f.bytes) return fail(SWVR_ERR_WORKSPACE, "forward workspace %zu < required %zu", wsb, f.bytes);
  if (p.n_tokens == 0) return SWVR_OK;
  if (p.vocab == 0) return fail(SWVR_ERR_UNSUPPORTED, "empty vocabulary (callers handle V == 0)");
  tc::FwdParams prm;
  SWVR_TRY(tc_fwd_launch(p, f, static_cast<char*>(ws), st, &prm));
  ProfScope ps_c(kProfCombine, st);
  SWVR_CUDA(small::combine(SWVR_F32, f.splits, p.n_tokens, p.embed_dim, prm.part_m2, prm.part_l, prm.part_acc, 0,
                           f.splits, tc::kFwdTokenTile, O, lse, m2o, lo, acco, /*pdl=*/true, st));
  return SWVR_OK;
}

// ---------------------------------------------------------------------------- backward plan
// gO and E of the score kernel come from their own producer warp (1, the default) or are
// interleaved with the W / h stream (0); SWVR_BWD_AUX_LOADS overrides the default.
static int bwd_aux_loads() {
  const char* s = std::getenv("SWVR_BWD_AUX_LOADS");
  return s ? (std::atoi(s) != 0 ? 1 : 0) : 1;
}

// Unit order of the score kernel: groups of this many vocabulary tiles walk the token splits
// (tc::bwd_unit), so on 74 pairs about four token splits of h and 20 W tiles stream at a
// time.  At c2 (11 token splits per 60-tile chunk) the kernel ran 1.145-1.152 ms per chunk
// against 1.166-1.168 with every split of a vocabulary tile in a row (1), A/B on one box;
// 12 was as good as 20, and 64-wide K stages (6 of them) lost 19 %.  SWVR_BWD_GROUP
// overrides it (read on each call).
static int bwd_group(int VTc) {
  const char* s = std::getenv("SWVR_BWD_GROUP");
  const int v = s ? std::max(1, std::atoi(s)) : 20;
  return std::max(1, std::min(v, std::max(VTc, 1)));
}

// Token splits of the score kernel's units (a 256-row vocabulary tile x a range of token
// tiles): minimise the rounds over the pairs times the tiles per unit.
static void choose_ts(int VTc, int NT, int sms, int* TS, int* per_t) {
  int best = 1;
  int64_t best_cost = -1;
  const int tmax = std::max(1, std::min(NT, 32));
  for (int ts = 1; ts <= tmax; ++ts) {
    const int64_t cost = ceil_div(static_cast<int64_t>(VTc) * ts, sms) * ceil_div(NT, ts);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = ts;
    }
  }
  *per_t = static_cast<int>(ceil_div(std::max(NT, 1), best));
  *TS = static_cast<int>(ceil_div(std::max(NT, 1), *per_t));
}

struct BwdPlan {
  int DP, BN, NT, C, sms;
  int64_t Npad;
  bool need_h, need_W, need_E, need_b, need_ds;
  size_t off_delta, off_goc, off_ds, off_dh, off_de, off_db, bytes;
  int max_units;
};

static BwdPlan plan_bwd(const swvr_problem& p, const swvr_grads& g) {
  BwdPlan b{};
  b.sms = num_sms();
  b.DP = p.embed_dim <= 64 ? 64 : (p.embed_dim <= 128 ? 128 : 256);
  b.BN = tc::bwd_token_tile(b.DP, p.hidden);
  b.NT = static_cast<int>(ceil_div(p.n_tokens, b.BN));
  b.Npad = static_cast<int64_t>(b.NT) * b.BN;  // a multiple of 64 (the GEMMs' token K-blocks)
  // The reference's chunk holds chunk x N fp32 scores; dS here is 16-bit, so the same bytes
  // hold 2 * chunk rows.  A multiple of 256 so that only the last chunk has a partial
  // 256-row pair tile.
  // The chunks are balanced: as many as that bound needs, of equal size, so no small tail
  // chunk runs a mostly idle grid.
  const int64_t cmax = round_up(2 * std::max<int64_t>(p.chunk, 1), 256);
  const int64_t nch = ceil_div(std::max<int64_t>(p.vocab, 1), cmax);
  int64_t C = round_up(ceil_div(std::max<int64_t>(p.vocab, 1), nch), 256);
  b.C = static_cast<int>(C);
  b.need_h = g.grad_h || g.grad_h_acc;
  b.need_W = g.grad_W != nullptr;
  b.need_E = g.grad_E != nullptr;
  b.need_b = g.grad_bias != nullptr && p.bias != nullptr;
  b.need_ds = b.need_h || b.need_W;
  // the largest units count over the full chunk and the tail chunk
  b.max_units = 1;
  for (int64_t rows : {C, p.vocab % C}) {
    if (rows <= 0) continue;
    const int VTc = static_cast<int>(ceil_div(rows, 256));
    int TS, per_t;
    choose_ts(VTc, b.NT, b.sms / 2, &TS, &per_t);
    b.max_units = std::max(b.max_units, VTc * TS);
  }
  size_t off = 0;
  b.off_delta = off;
  off += align_up(static_cast<size_t>(b.Npad) * 4, 256);
  b.off_goc = off;
  off += align_up(static_cast<size_t>(b.Npad) * b.DP * 2, 256);
  b.off_ds = off;
  if (b.need_ds) off += align_up(static_cast<size_t>(C) * b.Npad * 2, 256);
  b.off_dh = off;
  if (b.need_h && !g.grad_h_acc) off += align_up(static_cast<size_t>(p.n_tokens) * p.hidden * 4, 256);
  b.off_de = off;
  if (b.need_E) off += align_up(static_cast<size_t>(b.max_units) * 256 * p.embed_dim * 4, 256);
  b.off_db = off;
  if (b.need_b) off += align_up(static_cast<size_t>(b.max_units) * 256 * 4, 256);
  b.bytes = off + 256;
  return b;
}

// defer_last_dw: leave the dW tiles of the last vocabulary chunk to tc_bwd_finish (dh is final
// when this call's work completes).
static int tc_bwd(const swvr_problem& p, const swvr_grads& g, void* ws, size_t wsb, cudaStream_t st,
                  bool defer_last_dw = false) {
  const BwdPlan b = plan_bwd(p, g);
  if (wsb < b.bytes) return fail(SWVR_ERR_WORKSPACE, "backward workspace %zu < required %zu", wsb, b.bytes);
  const int64_t N = p.n_tokens, K = p.hidden, V = p.vocab, D = p.embed_dim;
  if (g.grad_W && !(g.grad_W_dtype == p.compute_dtype || g.grad_W_dtype == SWVR_F32))
    return fail(SWVR_ERR_UNSUPPORTED, "grad_W must be in the compute dtype or fp32");
  if (g.grad_W && ((reinterpret_cast<uintptr_t>(g.grad_W) & 15u) || (g.ld_grad_W * dtype_size(g.grad_W_dtype)) % 16))
    return fail(SWVR_ERR_UNSUPPORTED, "grad_W must be 16-byte aligned with a 16-byte multiple row pitch");
  if (N == 0 || V == 0) {
    if (g.grad_W) SWVR_CUDA(small::zero_rows(g.grad_W, g.grad_W_dtype, V, K, g.ld_grad_W, st));
    if (g.grad_E) SWVR_CUDA(small::zero_rows(g.grad_E, g.grad_E_dtype, V, D, g.ld_grad_E, st));
    if (g.grad_bias) SWVR_CUDA(small::zero_rows(g.grad_bias, g.grad_bias_dtype, 1, V, V, st));
    if (g.grad_h) SWVR_CUDA(small::zero_rows(g.grad_h, g.grad_h_dtype, N, K, K, st));
    if (g.grad_h_acc && !g.accumulate_grad_h)
      SWVR_CUDA(cudaMemsetAsync(g.grad_h_acc, 0, static_cast<size_t>(N) * K * 4, st));
    return SWVR_OK;
  }
  const bool bf16 = p.compute_dtype == SWVR_BF16;
  char* w = static_cast<char*>(ws);
  float* delta = reinterpret_cast<float*>(w + b.off_delta);
  void* goc = w + b.off_goc;
  void* ds = b.need_ds ? static_cast<void*>(w + b.off_ds) : nullptr;
  float* dh = b.need_h ? (g.grad_h_acc ? static_cast<float*>(g.grad_h_acc) : reinterpret_cast<float*>(w + b.off_dh))
                       : nullptr;
  float* part_de = b.need_E ? reinterpret_cast<float*>(w + b.off_de) : nullptr;
  float* part_db = b.need_b ? reinterpret_cast<float*>(w + b.off_db) : nullptr;

  {
  ProfScope ps(kProfPrologue, st);
  SWVR_CUDA(small::prologue(bf16, static_cast<const float*>(g.O), static_cast<const float*>(g.grad_O),
                            static_cast<const float*>(g.grad_lse), N, static_cast<int>(D), b.DP, delta, goc, st));
  }
  if (dh && !(g.grad_h_acc && g.accumulate_grad_h)) SWVR_CUDA(cudaMemsetAsync(dh, 0, static_cast<size_t>(N) * K * 4, st));

  tc::BwdScoresMaps sm;
  SWVR_TRY(make_map(&sm.w, p.W, p.compute_dtype, K, V, p.ldw * 2, 64, 128));
  SWVR_TRY(make_map(&sm.h, p.h, p.compute_dtype, K, N, p.ldh * 2, 64, b.BN / 2));
  SWVR_TRY(make_map(&sm.e, p.E, p.compute_dtype, D, V, p.lde * 2, 64, 128));
  SWVR_TRY(make_map(&sm.gok, goc, p.compute_dtype, b.DP, N, b.DP * 2, 64, tc::bwd_dp_chunk(b.BN) / 2));
  const int gomw = tc::bwd_gom_width(b.DP);
  SWVR_TRY(make_map(&sm.gom, goc, p.compute_dtype, b.DP, N, b.DP * 2, gomw, b.BN, gomw * 2));
  tc::GemmMaps gm;
  if (b.need_ds) {
    SWVR_TRY(make_map(&gm.h_mn, p.h, p.compute_dtype, K, N, p.ldh * 2, 64, 64));
    SWVR_TRY(make_map(&gm.w_mn, p.W, p.compute_dtype, K, V, p.ldw * 2, 64, 64));
    if (g.grad_W) {
      if (g.grad_W_dtype == SWVR_F32)
        SWVR_TRY(make_map(&gm.gw, g.grad_W, SWVR_F32, K, V, g.ld_grad_W * 4, 32, 128));
      else
        SWVR_TRY(make_map(&gm.gw, g.grad_W, p.compute_dtype, K, V, g.ld_grad_W * 2, 64, 128));
    } else {
      gm.gw = gm.w_mn;  // unused
    }
    if (dh)
      SWVR_TRY(make_map(&gm.dh, dh, SWVR_F32, K, N, K * 4, 32, 128));
    else
      gm.dh = gm.w_mn;  // unused
  }

  for (int64_t v0 = 0; v0 < V; v0 += b.C) {
    const int64_t v1 = std::min<int64_t>(v0 + b.C, V);
    const int rows = static_cast<int>(v1 - v0);
    const int VTc = static_cast<int>(ceil_div(rows, 256));
    int TS, per_t;
    choose_ts(VTc, b.NT, b.sms / 2, &TS, &per_t);
    tc::BwdScoresParams sp{};
    sp.N = static_cast<int>(N);
    sp.K = static_cast<int>(K);
    sp.D = static_cast<int>(D);
    sp.v_begin = static_cast<int>(v0);
    sp.v_end = static_cast<int>(v1);
    sp.scale = static_cast<float>(p.logit_scale);
    sp.sc2 = static_cast<float>(p.logit_scale * 1.4426950408889634);
    sp.bias = p.bias;
    sp.bias_dt = p.bias_dtype;
    sp.lse = static_cast<const float*>(g.lse);
    sp.delta = delta;
    sp.NT = b.NT;
    sp.VT = VTc;
    sp.TS = TS;
    sp.per_t = per_t;
    sp.units = VTc * TS;
    sp.gv = bwd_group(VTc);
    sp.ds = ds;
    sp.ld_ds = b.Npad;
    sp.part_de = part_de;
    sp.part_db = part_db;
    sp.aux_loads = bwd_aux_loads();
    if (b.need_ds) {
      SWVR_TRY(make_map(&gm.ds_k, ds, p.compute_dtype, b.Npad, rows, b.Npad * 2, 64, 128));
      SWVR_TRY(make_map(&gm.ds_mn, ds, p.compute_dtype, b.Npad, rows, b.Npad * 2, 64, 64));
    }
    {
      ProfScope ps(kProfBwdScores, st);
      // after the first chunk the previous kernel in the stream is this loop's own
      SWVR_CUDA(tc::launch_bwd_scores_kernel(bf16, b.DP, b.BN, sm, sp, b.sms / 2, /*pdl=*/v0 > 0, st));
    }
    if (part_de || part_db) {
      void* gE = g.grad_E;
      ProfScope ps(kProfReduce, st);
      SWVR_CUDA(small::reduce_de_db(part_de, part_db, TS, per_t, b.NT, static_cast<int>(v0), rows, 256, D, gE,
                                    g.grad_E_dtype, g.ld_grad_E, g.grad_bias, g.grad_bias_dtype, /*pdl=*/true, st));
    }
    if (b.need_ds) {
      tc::GemmParams gp{};
      const int nt = static_cast<int>(ceil_div(K, 256));
      gp.dw_mt = static_cast<int>(ceil_div(rows, 256));
      gp.dw_nt = nt;
      gp.dw_kb = static_cast<int>(b.Npad / 64);
      gp.dw_tiles = (g.grad_W && !(defer_last_dw && v1 == V)) ? gp.dw_mt * nt : 0;
      gp.dh_mt = static_cast<int>(ceil_div(b.Npad, 256));
      gp.dh_nt = nt;
      gp.dh_kb = static_cast<int>(ceil_div(rows, 64));
      gp.dh_tiles = dh ? gp.dh_mt * nt : 0;
      gp.v_begin = static_cast<int>(v0);
      gp.gw_f32 = g.grad_W_dtype == SWVR_F32 ? 1 : 0;
      const int tiles = gp.dw_tiles + gp.dh_tiles;
      if (tiles > 0) {
        ProfScope ps(kProfGemm, st);
        SWVR_CUDA(tc::launch_gemm_kernel(bf16, gm, gp, b.sms / 2, /*pdl=*/true, st));
      }
    }
  }
  if (g.grad_h) {
    ProfScope ps(kProfCast, st);
    SWVR_CUDA(small::cast_f32(dh, g.grad_h, g.grad_h_dtype, N * K, st));
  }
  return SWVR_OK;
}

// The dW tiles of the last vocabulary chunk that tc_bwd(..., defer_last_dw) left undone, from the
// dS still in the workspace, on at most max_pairs CTA pairs.
static int tc_bwd_finish(const swvr_problem& p, const swvr_grads& g, void* ws, size_t wsb, int max_pairs,
                         cudaStream_t st) {
  const BwdPlan b = plan_bwd(p, g);
  if (wsb < b.bytes) return fail(SWVR_ERR_WORKSPACE, "backward workspace %zu < required %zu", wsb, b.bytes);
  const int64_t N = p.n_tokens, K = p.hidden, V = p.vocab;
  if (N == 0 || V == 0 || !g.grad_W) return SWVR_OK;
  const int64_t v0 = (V - 1) / b.C * b.C;
  const int rows = static_cast<int>(V - v0);
  void* ds = static_cast<char*>(ws) + b.off_ds;
  tc::GemmMaps gm;
  SWVR_TRY(make_map(&gm.ds_k, ds, p.compute_dtype, b.Npad, rows, b.Npad * 2, 64, 128));
  SWVR_TRY(make_map(&gm.ds_mn, ds, p.compute_dtype, b.Npad, rows, b.Npad * 2, 64, 64));
  SWVR_TRY(make_map(&gm.h_mn, p.h, p.compute_dtype, K, N, p.ldh * 2, 64, 64));
  SWVR_TRY(make_map(&gm.w_mn, p.W, p.compute_dtype, K, V, p.ldw * 2, 64, 64));
  if (g.grad_W_dtype == SWVR_F32)
    SWVR_TRY(make_map(&gm.gw, g.grad_W, SWVR_F32, K, V, g.ld_grad_W * 4, 32, 128));
  else
    SWVR_TRY(make_map(&gm.gw, g.grad_W, p.compute_dtype, K, V, g.ld_grad_W * 2, 64, 128));
  gm.dh = gm.w_mn;  // no dh tiles
  tc::GemmParams gp{};
  const int nt = static_cast<int>(ceil_div(K, 256));
  gp.dw_mt = static_cast<int>(ceil_div(rows, 256));
  gp.dw_nt = nt;
  gp.dw_kb = static_cast<int>(b.Npad / 64);
  gp.dw_tiles = gp.dw_mt * nt;
  gp.dh_tiles = 0;
  gp.dh_mt = gp.dh_nt = 1;
  gp.dh_kb = 1;
  gp.v_begin = static_cast<int>(v0);
  gp.gw_f32 = g.grad_W_dtype == SWVR_F32 ? 1 : 0;
  const int pairs = max_pairs > 0 ? std::min(max_pairs, b.sms / 2) : b.sms / 2;
  ProfScope ps(kProfGemm, st);
  SWVR_CUDA(tc::launch_gemm_kernel(p.compute_dtype == SWVR_BF16, gm, gp, pairs, /*pdl=*/false, st));
  return SWVR_OK;
}

}  // namespace swvr

// ================================================================================ extern "C"
using namespace swvr;

extern "C" {

int swvr_abi_version(void) { return SWVR_ABI_VERSION; }

int swvr_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  static_assert((kErrSelftest | 1) == SWVR_SELFTEST_CODE, "self-test code");
  if (limit_ns < 1000000 || limit_ns > 10000000000ll)
    return fail(SWVR_ERR_INVALID_ARGUMENT, "limit_ns must be within 1 ms .. 10 s");
  SWVR_CUDA(small::wait_selftest(static_cast<uint64_t>(limit_ns), static_cast<cudaStream_t>(stream)));
  return SWVR_OK;
}

const char* swvr_last_error(void) { return t_err.c_str(); }

int swvr_device_error(uint32_t* code) {
  if (!code) return fail(SWVR_ERR_INVALID_ARGUMENT, "code is NULL");
  unsigned int v = 0, zero = 0;
  SWVR_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)));
  SWVR_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero)));
  *code = v;
  return SWVR_OK;
}

int swvr_profile_start(void) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (auto& pe : g_prof_pending) {
    g_prof_pool.push_back(pe.e0);
    g_prof_pool.push_back(pe.e1);
  }
  g_prof_pending.clear();
  for (int k = 0; k < kProfKinds; ++k) g_prof_launches[k] = 0;
  g_prof_on = true;
  return SWVR_OK;
}

int swvr_profile_stop(swvr_profile_record* records, int max_records, int* n_records) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  g_prof_on = false;
  double ms[kProfKinds] = {0};
  for (auto& pe : g_prof_pending) {
    float t = 0.f;
    if (cudaEventSynchronize(pe.e1) != cudaSuccess) return fail(SWVR_ERR_CUDA, "profile event wait failed");
    if (cudaEventElapsedTime(&t, pe.e0, pe.e1) == cudaSuccess) ms[pe.kind] += t;
    g_prof_pool.push_back(pe.e0);
    g_prof_pool.push_back(pe.e1);
  }
  g_prof_pending.clear();
  int n = 0;
  for (int k = 0; k < kProfKinds; ++k) {
    if (g_prof_launches[k] == 0) continue;
    if (records && n < max_records) {
      std::memset(records[n].name, 0, sizeof(records[n].name));
      std::strncpy(records[n].name, kProfNames[k], sizeof(records[n].name) - 1);
      records[n].launches = g_prof_launches[k];
      records[n].total_ms = ms[k];
    }
    ++n;
  }
  if (n_records) *n_records = n;
  return SWVR_OK;
}

int swvr_fwd_workspace_size(const swvr_problem* p, size_t* bytes) {
  SWVR_TRY(validate(p));
  if (!bytes) return fail(SWVR_ERR_INVALID_ARGUMENT, "bytes is NULL");
  *bytes = is_tc(p->compute_dtype) ? plan_fwd(*p).bytes : simt::fwd_workspace(*p);
  return SWVR_OK;
}

int swvr_fwd(const swvr_problem* p, void* O, void* lse, void* ws, size_t wsb, void* stream) {
  SWVR_TRY(validate(p));
  if (p->n_tokens > 0 && (!O || !lse)) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (is_tc(p->compute_dtype)) return tc_fwd(*p, O, lse, nullptr, nullptr, nullptr, ws, wsb, st);
  if (wsb < simt::fwd_workspace(*p)) return fail(SWVR_ERR_WORKSPACE, "forward workspace too small");
  ProfScope ps(kProfSimt, st);
  return simt::fwd(*p, O, lse, nullptr, nullptr, nullptr, ws, st) == SWVR_OK
             ? SWVR_OK
             : fail(SWVR_ERR_CUDA, "SIMT forward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
}

int swvr_fwd_partial(const swvr_problem* p, void* m2, void* l, void* acc, void* ws, size_t wsb, void* stream) {
  SWVR_TRY(validate(p));
  if (p->n_tokens > 0 && (!m2 || !l || !acc)) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (is_tc(p->compute_dtype)) return tc_fwd(*p, nullptr, nullptr, m2, l, acc, ws, wsb, st);
  if (wsb < simt::fwd_workspace(*p)) return fail(SWVR_ERR_WORKSPACE, "forward workspace too small");
  ProfScope ps(kProfSimt, st);
  return simt::fwd(*p, nullptr, nullptr, m2, l, acc, ws, st) == SWVR_OK
             ? SWVR_OK
             : fail(SWVR_ERR_CUDA, "SIMT forward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
}

int swvr_combine(int64_t shards, int64_t n_tokens, int64_t embed_dim, int32_t acc_dt, const void* m2, const void* l,
                 const void* acc, void* O, void* lse, void* stream) {
  if (shards <= 0 || n_tokens < 0 || embed_dim < 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "bad combine sizes");
  if (acc_dt != SWVR_F32 && acc_dt != SWVR_F64) return fail(SWVR_ERR_INVALID_ARGUMENT, "combine dtype must be F32/F64");
  if (n_tokens > 0 && (!m2 || !l || !acc || !O || !lse)) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL pointer");
  ProfScope ps(kProfCombine, static_cast<cudaStream_t>(stream));
  SWVR_CUDA(small::combine(acc_dt, static_cast<int>(shards), n_tokens, embed_dim, m2, l, acc, 1, 1, 0, O, lse, nullptr,
                           nullptr, nullptr, /*pdl=*/false, static_cast<cudaStream_t>(stream)));
  return SWVR_OK;
}

int swvr_bwd_workspace_size(const swvr_problem* p, const swvr_grads* g, size_t* bytes) {
  SWVR_TRY(validate(p));
  if (!g || !bytes) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL argument");
  *bytes = is_tc(p->compute_dtype) ? plan_bwd(*p, *g).bytes : simt::bwd_workspace(*p, *g);
  return SWVR_OK;
}

int swvr_bwd(const swvr_problem* p, const swvr_grads* g, void* ws, size_t wsb, void* stream) {
  SWVR_TRY(validate(p));
  if (!g) return fail(SWVR_ERR_INVALID_ARGUMENT, "grads is NULL");
  if (p->n_tokens > 0 && (!g->grad_O || !g->grad_lse || !g->O || !g->lse))
    return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL backward input");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (is_tc(p->compute_dtype)) return tc_bwd(*p, *g, ws, wsb, st);
  if (wsb < simt::bwd_workspace(*p, *g)) return fail(SWVR_ERR_WORKSPACE, "backward workspace too small");
  ProfScope ps(kProfSimt, st);
  return simt::bwd(*p, *g, ws, st) == SWVR_OK
             ? SWVR_OK
             : fail(SWVR_ERR_CUDA, "SIMT backward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
}

int swvr_bwd_split(const swvr_problem* p, const swvr_grads* g, void* ws, size_t wsb, void* stream) {
  SWVR_TRY(validate(p));
  if (!g) return fail(SWVR_ERR_INVALID_ARGUMENT, "grads is NULL");
  if (p->n_tokens > 0 && (!g->grad_O || !g->grad_lse || !g->O || !g->lse))
    return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL backward input");
  if (g->grad_h) return fail(SWVR_ERR_INVALID_ARGUMENT, "swvr_bwd_split leaves dh un-cast: pass grad_h_acc, not grad_h");
  if (!is_tc(p->compute_dtype)) return swvr_bwd(p, g, ws, wsb, stream);  // nothing deferred
  return tc_bwd(*p, *g, ws, wsb, static_cast<cudaStream_t>(stream), /*defer_last_dw=*/true);
}

int swvr_bwd_finish(const swvr_problem* p, const swvr_grads* g, void* ws, size_t wsb, int32_t max_sms,
                    void* stream) {
  SWVR_TRY(validate(p));
  if (!g) return fail(SWVR_ERR_INVALID_ARGUMENT, "grads is NULL");
  if (max_sms < 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "max_sms must be >= 0");
  if (!is_tc(p->compute_dtype)) return SWVR_OK;
  return tc_bwd_finish(*p, *g, ws, wsb, max_sms / 2, static_cast<cudaStream_t>(stream));
}

int swvr_mse_fwd(int64_t n_tokens, int64_t embed_dim, int32_t dtype, const void* O, const void* lse,
                 const void* target, const void* weight, double z, int32_t reduction, void* out, void* stats,
                 void* stream) {
  if (n_tokens < 0 || embed_dim < 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "negative size");
  if (dtype != SWVR_F32 && dtype != SWVR_F64) return fail(SWVR_ERR_INVALID_ARGUMENT, "loss dtype must be F32/F64");
  if (reduction < SWVR_REDUCE_NONE || reduction > SWVR_REDUCE_MEAN)
    return fail(SWVR_ERR_INVALID_ARGUMENT, "unknown reduction %d", reduction);
  if (!out || (n_tokens > 0 && (!O || !lse || !target))) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (reduction != SWVR_REDUCE_NONE && !stats)
    return fail(SWVR_ERR_INVALID_ARGUMENT, "SUM / MEAN need stats (SWVR_MSE_STATS_LEN elements)");
  ProfScope ps(kProfMse, static_cast<cudaStream_t>(stream));
  SWVR_CUDA(small::mse_fwd(dtype, n_tokens, embed_dim, O, lse, target, weight, z, reduction, out, stats,
                           static_cast<cudaStream_t>(stream)));
  return SWVR_OK;
}

int swvr_mse_bwd(int64_t n_tokens, int64_t embed_dim, int32_t dtype, const void* O, const void* lse,
                 const void* target, const void* weight, double z, int32_t reduction, const void* grad_out,
                 const void* stats, void* grad_O, void* grad_lse, void* grad_target, void* grad_weight,
                 void* stream) {
  if (n_tokens < 0 || embed_dim < 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "negative size");
  if (dtype != SWVR_F32 && dtype != SWVR_F64) return fail(SWVR_ERR_INVALID_ARGUMENT, "loss dtype must be F32/F64");
  if (reduction < SWVR_REDUCE_NONE || reduction > SWVR_REDUCE_MEAN)
    return fail(SWVR_ERR_INVALID_ARGUMENT, "unknown reduction %d", reduction);
  if (reduction == SWVR_REDUCE_MEAN && !stats) return fail(SWVR_ERR_INVALID_ARGUMENT, "MEAN needs stats");
  if (n_tokens > 0 && (!O || !lse || !target || !grad_out || !grad_O || !grad_lse))
    return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL pointer");
  ProfScope ps(kProfMse, static_cast<cudaStream_t>(stream));
  SWVR_CUDA(small::mse_bwd(dtype, n_tokens, embed_dim, O, lse, target, weight, z, reduction, grad_out, stats, grad_O,
                           grad_lse, grad_target, grad_weight, static_cast<cudaStream_t>(stream)));
  return SWVR_OK;
}


// ------------------------------------------------------------------ RMSNorm producer of h
static bool norm_dtype_ok(int32_t dt) { return dt == SWVR_F32 || dt == SWVR_F64 || dt == SWVR_BF16 || dt == SWVR_F16; }

int swvr_rmsnorm_fwd(int64_t n_rows, int64_t hidden, const void* x, int32_t x_dtype, int64_t ld_x, const void* weight,
                     int32_t weight_dtype, double eps, void* h, int32_t h_dtype, int64_t ld_h, void* rstd,
                     void* stream) {
  if (n_rows < 0 || hidden <= 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "n_rows must be >= 0 and hidden > 0");
  if (!norm_dtype_ok(x_dtype) || !norm_dtype_ok(h_dtype) || (weight && !norm_dtype_ok(weight_dtype)))
    return fail(SWVR_ERR_INVALID_ARGUMENT, "unknown dtype");
  if (ld_x < hidden || ld_h < hidden) return fail(SWVR_ERR_INVALID_ARGUMENT, "row pitch below hidden");
  if (!(eps >= 0.0)) return fail(SWVR_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (n_rows > 0 && (!x || !h || !rstd)) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  ProfScope ps(kProfNorm, st);
  if (x_dtype == SWVR_F64 || h_dtype == SWVR_F64)
    SWVR_CUDA(norm::fwd<double>(n_rows, hidden, x, x_dtype, ld_x, weight, weight_dtype, eps, h, h_dtype, ld_h, rstd, st));
  else
    SWVR_CUDA(norm::fwd<float>(n_rows, hidden, x, x_dtype, ld_x, weight, weight_dtype, eps, h, h_dtype, ld_h, rstd, st));
  return SWVR_OK;
}

int swvr_rmsnorm_bwd_workspace_size(int64_t n_rows, int64_t hidden, int32_t acc_dtype, int32_t need_grad_weight,
                                    size_t* bytes) {
  if (!bytes) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL pointer");
  if (n_rows < 0 || hidden <= 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "n_rows must be >= 0 and hidden > 0");
  if (acc_dtype != SWVR_F32 && acc_dtype != SWVR_F64) return fail(SWVR_ERR_INVALID_ARGUMENT, "acc dtype must be F32/F64");
  *bytes = norm::bwd_workspace(n_rows, hidden, dtype_size(acc_dtype), need_grad_weight != 0);
  return SWVR_OK;
}

int swvr_rmsnorm_bwd(int64_t n_rows, int64_t hidden, const void* grad_h, int32_t acc_dtype, const void* x,
                     int32_t x_dtype, int64_t ld_x, const void* weight, int32_t weight_dtype, const void* rstd,
                     void* grad_x, int32_t grad_x_dtype, void* grad_weight, int32_t grad_weight_dtype, void* workspace,
                     size_t workspace_bytes, void* stream) {
  if (n_rows < 0 || hidden <= 0) return fail(SWVR_ERR_INVALID_ARGUMENT, "n_rows must be >= 0 and hidden > 0");
  if (acc_dtype != SWVR_F32 && acc_dtype != SWVR_F64) return fail(SWVR_ERR_INVALID_ARGUMENT, "acc dtype must be F32/F64");
  if (!norm_dtype_ok(x_dtype) || (weight && !norm_dtype_ok(weight_dtype)) ||
      (grad_x && !norm_dtype_ok(grad_x_dtype)) || (grad_weight && !norm_dtype_ok(grad_weight_dtype)))
    return fail(SWVR_ERR_INVALID_ARGUMENT, "unknown dtype");
  if (ld_x < hidden) return fail(SWVR_ERR_INVALID_ARGUMENT, "row pitch below hidden");
  if (grad_weight && !weight) return fail(SWVR_ERR_INVALID_ARGUMENT, "grad_weight without weight");
  if (!grad_x && !grad_weight) return SWVR_OK;
  if (n_rows > 0 && (!grad_h || !x || !rstd)) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL pointer");
  const size_t asz = dtype_size(acc_dtype);
  const bool need_w = grad_weight != nullptr;
  if (need_w && norm::bwd_shape(n_rows, hidden, asz, true).nwarps < 1)
    return fail(SWVR_ERR_UNSUPPORTED, "hidden %lld too wide for the weight-gradient sums in shared memory",
                static_cast<long long>(hidden));
  const size_t need = norm::bwd_workspace(n_rows, hidden, asz, need_w);
  if (workspace_bytes < need) return fail(SWVR_ERR_WORKSPACE, "workspace %zu < required %zu", workspace_bytes, need);
  if (need && !workspace) return fail(SWVR_ERR_INVALID_ARGUMENT, "NULL workspace");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  ProfScope ps(kProfNorm, st);
  if (acc_dtype == SWVR_F64)
    SWVR_CUDA(norm::bwd<double>(n_rows, hidden, grad_h, x, x_dtype, ld_x, weight, weight_dtype, rstd, grad_x,
                                grad_x_dtype, grad_weight, grad_weight_dtype, workspace, st));
  else
    SWVR_CUDA(norm::bwd<float>(n_rows, hidden, grad_h, x, x_dtype, ld_x, weight, weight_dtype, rstd, grad_x,
                               grad_x_dtype, grad_weight, grad_weight_dtype, workspace, st));
  return SWVR_OK;
}

}  // extern "C"
