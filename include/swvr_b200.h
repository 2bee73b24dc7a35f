/*
 * swvr_b200 -- C ABI of the B200 (sm_100a) softmax-weighted embedding readout.
 *
 *   S   = logit_scale * h @ W^T + bias          h [N, K], W [V, K], bias [V]
 *   O   = softmax(S) @ E,  LSE = logsumexp(S)   E [V, D], O [N, D], LSE [N]
 *
 * The [N, V] scores are never materialised.  This header is the boundary a host binds
 * (ctypes / cgo / JNI / N-API): plain pointers, sizes and enums, no framework types.
 *
 * Conventions shared by every entry point
 *   - All pointers are device pointers on the current CUDA device unless stated.
 *   - `stream` is a cudaStream_t (may be NULL for the legacy default stream).  All work is
 *     enqueued on it; nothing here synchronises the stream or the device.
 *   - The library never allocates or frees device memory: callers pass every output and a
 *     workspace of at least the size the matching *_workspace_size() call returns.
 *   - Return value: SWVR_OK (0) or a negative SWVR_ERR_* code; swvr_last_error() then holds
 *     a message (per host thread).  Errors raised by a bounded device-side wait surface on
 *     the host through swvr_device_error().
 *   - Reentrant: no call keeps state between calls except a per-device cache of kernel
 *     attributes guarded by a mutex.
 *   - Compute dtypes: SWVR_BF16 / SWVR_F16 run the tcgen05 tensor-core kernels (fp32
 *     accumulation); SWVR_F32 / SWVR_F64 run the exact path (fp32 GEMMs as three-term
 *     split-TF32 tensor-core products with fp32-level error, fp64 on the CUDA cores).  O,
 *     LSE and the softmax state are fp64 for SWVR_F64 compute and fp32 otherwise (the
 *     accumulation dtype).
 */
#ifndef SWVR_B200_H
#define SWVR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SWVR_ABI_VERSION 2

enum swvr_status {
  SWVR_OK = 0,
  SWVR_ERR_INVALID_ARGUMENT = -1, /* bad shape / pointer / value: a ValueError in Python */
  SWVR_ERR_UNSUPPORTED = -2,      /* a dtype, size or alignment the kernels do not cover */
  SWVR_ERR_CUDA = -3,             /* a CUDA runtime / driver call or a launch failed */
  SWVR_ERR_WORKSPACE = -4         /* the workspace passed is smaller than required */
};

enum swvr_dtype { SWVR_F32 = 0, SWVR_F64 = 1, SWVR_BF16 = 2, SWVR_F16 = 3 };

enum swvr_reduction { SWVR_REDUCE_NONE = 0, SWVR_REDUCE_SUM = 1, SWVR_REDUCE_MEAN = 2 };

/*
 * One readout problem.  h, W and E share `compute_dtype`; rows may be padded (ld* is the
 * row stride in elements, the last dimension is contiguous).  On the tensor-core path the
 * base pointers must be 16-byte aligned and ld* * element size a multiple of 16 bytes.
 * `chunk` is the reference's chunk_size, the knob that bounds the backward's working set:
 * the reference stages chunk x N fp32 scores at a time; the tensor-core path stages its
 * 16-bit score gradients for at most 2 * chunk vocabulary rows (the same bytes; the vocab
 * is cut into equal chunks of a multiple of 256 rows), and the fp32 / fp64 path stages
 * chunk rows.
 */
typedef struct swvr_problem {
  int64_t n_tokens;   /* N  (rows of h)             */
  int64_t hidden;     /* K                           */
  int64_t vocab;      /* V  (rows of W, E, bias)     */
  int64_t embed_dim;  /* D                           */
  int32_t compute_dtype;
  int32_t bias_dtype; /* ignored when bias == NULL   */
  const void* h;
  int64_t ldh;
  const void* W;
  int64_t ldw;
  const void* E;
  int64_t lde;
  const void* bias;   /* [V] contiguous, or NULL     */
  double logit_scale;
  int64_t chunk;
} swvr_problem;

/*
 * Forward.  Replaces the reference's custom op swvr::chunked_fwd
 * (swvr/chunked.py:157-161 -> _forward, chunked.py:82-105): writes O [N, D] and LSE [N],
 * contiguous, in the accumulation dtype.
 */
int swvr_fwd_workspace_size(const swvr_problem* p, size_t* bytes);
int swvr_fwd(const swvr_problem* p, void* O, void* lse, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Forward of one vocabulary shard without the final normalisation: the online-softmax state
 * of every row, m2 [N] (running maximum in log2 units, i.e. max of S * log2(e)),
 * l [N] (sum of 2^(S*log2(e) - m2)) and acc [N, D] (sum of those weights times E rows),
 * all in the accumulation dtype.  No counterpart in the reference (which has no vocabulary
 * sharding); it is the per-chunk state of chunked.py:86-104 exposed across devices.
 * Uses the same workspace size as swvr_fwd.
 */
int swvr_fwd_partial(const swvr_problem* p, void* m2, void* l, void* acc, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * Forward without a workspace, for callers that cannot allocate device memory at call
 * time: hosts that plan every byte of device memory up front and give plugins no
 * allocator, or FFI hosts (cgo, JNI, N-API) that forbid their plugins cudaMalloc, which can
 * synchronise the device and fragments a pool the host manages.  No counterpart in the
 * reference.  Same inputs and outputs as swvr_fwd (bf16 / fp16 compute only); the kernel's
 * scratch lives in a static device array of the library, 16 MiB on every GPU that loads the
 * library, held until exit.  Problems whose scratch does not fit (about N * (D + 2) * 4 bytes
 * when the vocabulary is not split, e.g. N = 16384 at D = 64 uses 4.3 MB) return
 * SWVR_ERR_UNSUPPORTED with a message.  The first call on each device looks the array up
 * (with that device current); make it before any stream capture.  All calls on a device
 * share the array: calls that overlap on the GPU race and must be serialised by the caller.
 * Allocates nothing: no cudaMalloc / cudaFree and no allocating library routine.
 */
int swvr_fwd_noalloc(const swvr_problem* p, void* O, void* lse, void* stream);

/*
 * Merge `shards` partial states ([shards, N], [shards, N], [shards, N, D], shard-major,
 * contiguous) in shard order into O [N, D] and LSE [N].  Deterministic.  The same merge as
 * the chunk loop of chunked.py:96-105, applied across shards.
 */
int swvr_combine(int64_t shards, int64_t n_tokens, int64_t embed_dim, int32_t acc_dtype, const void* m2, const void* l,
                 const void* acc, void* O, void* lse, void* stream);

/*
 * Backward inputs and outputs.  grad_O [N, D] and grad_lse [N] are contiguous in the
 * accumulation dtype, as are the saved forward outputs O and lse.  A NULL grad_* pointer
 * means "that input is frozen" (the reference's need_* flags, chunked.py:170-178); frozen
 * inputs skip their GEMMs.  grad_W / grad_E rows may be padded (ld_* in elements).
 * grad_h_acc, when not NULL, is an fp32 (fp64 for F64 compute) [N, K] buffer that receives
 * the un-cast dh accumulator (a vocabulary shard's partial dh, summed across shards by the
 * caller); grad_h may then be NULL.  With accumulate_grad_h non-zero the backward adds into
 * grad_h_acc instead of overwriting it, so a caller can run the vocabulary in pieces (for
 * example to cast fp32 parameters to the compute dtype one piece at a time).
 */
typedef struct swvr_grads {
  const void* grad_O;
  const void* grad_lse;
  const void* O;
  const void* lse;
  void* grad_h;
  int32_t grad_h_dtype;
  void* grad_W;
  int32_t grad_W_dtype;
  int64_t ld_grad_W;
  void* grad_E;
  int32_t grad_E_dtype;
  int64_t ld_grad_E;
  void* grad_bias;
  int32_t grad_bias_dtype;
  void* grad_h_acc;
  int32_t accumulate_grad_h;
} swvr_grads;

/*
 * Backward.  Replaces swvr::chunked_bwd (swvr/chunked.py:170-178 -> _backward, 108-151):
 * recomputes the scores per vocabulary tile and writes dh, dW, dE and db.  dW, dE and db are
 * deterministic (fixed-order reductions, no atomics); dh is accumulated in fp32 across
 * chunks in chunk order.  The workspace size depends on the score kernel's token tile, which
 * the environment variable SWVR_BWD_TOKEN_TILE (128 or 192) can override: keep it unchanged
 * between the size query and the call.
 */
int swvr_bwd_workspace_size(const swvr_problem* p, const swvr_grads* g, size_t* bytes);
int swvr_bwd(const swvr_problem* p, const swvr_grads* g, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The backward in two calls, so that dh can be exchanged while the last dW rows are computed.
 * No counterpart in the reference (which has no vocabulary sharding); used by the
 * vocabulary-sharded path to overlap its cross-device dh reduce-scatter with compute.
 * swvr_bwd_split does the work of swvr_bwd except, on the tensor-core path, the dW rows of the
 * last vocabulary chunk: dh must go to grad_h_acc (grad_h NULL), and it is final once the
 * call's work completes on `stream`.  swvr_bwd_finish then computes those dW rows from the
 * score gradients still in the workspace: same problem, grads and workspace, on a stream
 * ordered after the split call, before the workspace is reused.  max_sms (0: every SM)
 * bounds the SMs its kernel occupies, leaving the rest to a collective running beside it.
 * On the fp32 / fp64 path swvr_bwd_split is swvr_bwd and swvr_bwd_finish does nothing.
 */
int swvr_bwd_split(const swvr_problem* p, const swvr_grads* g, void* workspace, size_t workspace_bytes, void* stream);
int swvr_bwd_finish(const swvr_problem* p, const swvr_grads* g, void* workspace, size_t workspace_bytes,
                    int32_t max_sms, void* stream);

/*
 * MSE / z-loss / per-token-weight epilogue, forward.  Replaces the loss arithmetic of
 * softmax_readout_mse (swvr/api.py:54-66):
 *   per_tok = mean_d (O - target)^2 + z_loss_weight * LSE^2, times weight[n] if weight;
 *   NONE -> out [N]; SUM -> out [1] = sum; MEAN -> out [1] = sum / (sum(weight) or N).
 * O, lse, target, weight (may be NULL), out and stats share `dtype` (F32 or F64).  For SUM and
 * MEAN the reduction runs over a fixed grid in a fixed order (deterministic) and needs
 * `stats`, an array of SWVR_MSE_STATS_LEN elements: on return stats[0] = sum_n weight[n] *
 * per_tok[n] and stats[1] = the denominator (1 for SUM); the rest is scratch.
 */
#define SWVR_MSE_STATS_LEN 514

int swvr_mse_fwd(int64_t n_tokens, int64_t embed_dim, int32_t dtype, const void* O, const void* lse,
                 const void* target, const void* weight, double z_loss_weight, int32_t reduction, void* out,
                 void* stats, void* stream);

/*
 * Gradient of swvr_mse_fwd for upstream grad_out ([1] for SUM/MEAN, [N] for NONE): writes
 * grad_O [N, D], grad_lse [N] and, when not NULL, grad_target [N, D] and grad_weight [N].
 * `stats` is the array swvr_mse_fwd wrote (required for MEAN, ignored otherwise).
 */
int swvr_mse_bwd(int64_t n_tokens, int64_t embed_dim, int32_t dtype, const void* O, const void* lse,
                 const void* target, const void* weight, double z_loss_weight, int32_t reduction,
                 const void* grad_out, const void* stats, void* grad_O, void* grad_lse, void* grad_target,
                 void* grad_weight, void* stream);

/*
 * RMSNorm producer of h, fused at both ends of the readout (no counterpart in the reference,
 * whose callers normalise the trunk's output before swvr.softmax_readout_mse; this is the
 * "final norm feeding the readout" of its model code, kept inside the library).
 *
 * Forward: h[n, k] = x[n, k] * rstd[n] * weight[k] with rstd[n] = 1 / sqrt(mean_k x[n, k]^2 +
 * eps), computed in fp32 (fp64 when x or h is F64) and rounded once into h's dtype (the
 * readout's compute dtype, so the readout reads it as written).  weight may be NULL (1).
 * rstd is fp32 [n_rows] (fp64 when x or h is F64).  x and h rows are ld_x / ld_h elements apart.
 *
 * Backward: grad_h is the readout's un-cast dh accumulator (swvr_grads.grad_h_acc: fp32, or
 * fp64 for F64 compute) [n_rows, hidden], with rstd in the same dtype (acc_dtype).  Writes,
 * where not NULL, grad_x [n_rows, hidden] (contiguous) and grad_weight [hidden]:
 *   grad_x = rstd * (a - xh * mean_k(a * xh)),  a = grad_h * weight,  xh = x * rstd
 *   grad_weight = sum_n grad_h * xh   (fixed-order reduction: deterministic)
 * The workspace (swvr_rmsnorm_bwd_workspace_size) holds per-block partial weight gradients;
 * SWVR_ERR_UNSUPPORTED when hidden is too wide for them (above 51200 fp32 columns).
 */
int swvr_rmsnorm_fwd(int64_t n_rows, int64_t hidden, const void* x, int32_t x_dtype, int64_t ld_x, const void* weight,
                     int32_t weight_dtype, double eps, void* h, int32_t h_dtype, int64_t ld_h, void* rstd,
                     void* stream);
int swvr_rmsnorm_bwd_workspace_size(int64_t n_rows, int64_t hidden, int32_t acc_dtype, int32_t need_grad_weight,
                                    size_t* bytes);
int swvr_rmsnorm_bwd(int64_t n_rows, int64_t hidden, const void* grad_h, int32_t acc_dtype, const void* x,
                     int32_t x_dtype, int64_t ld_x, const void* weight, int32_t weight_dtype, const void* rstd,
                     void* grad_x, int32_t grad_x_dtype, void* grad_weight, int32_t grad_weight_dtype, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * Launch accounting for benchmarks (no counterpart in the reference).  Between
 * swvr_profile_start() and swvr_profile_stop(), every kernel the library launches from any
 * host thread is counted per kind and bracketed by a pair of CUDA events on its stream.
 * swvr_profile_stop() waits for those events and fills up to max_records records (one per
 * kernel kind that ran): launches and summed event time in milliseconds.
 */
typedef struct swvr_profile_record {
  char name[32];
  int64_t launches;
  double total_ms;
} swvr_profile_record;

int swvr_profile_start(void);
int swvr_profile_stop(swvr_profile_record* records, int max_records, int* n_records);

/* Message of the last failed call on this host thread ("" if none). */
const char* swvr_last_error(void);

/*
 * Read and clear the device error word of the current device: *code = 0 when no bounded
 * device-side wait has expired since the last call.  Synchronises with the device.
 */
int swvr_device_error(uint32_t* code);

/*
 * Self test of the device-side failure path (no counterpart in the reference): launches one
 * thread that waits, through the same bounded wait as the tensor-core pipelines, on a
 * barrier that nothing completes, for at most limit_ns (1 ms .. 10 s).  The wait expires, the
 * kernel records SWVR_SELFTEST_CODE in the device error word and returns; no fault, no
 * hang.  swvr_device_error() then reports the code and the device stays usable.
 */
#define SWVR_SELFTEST_CODE 0x7F01u
int swvr_selftest_wait_timeout(int64_t limit_ns, void* stream);

int swvr_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SWVR_B200_H */
