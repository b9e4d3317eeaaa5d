/* moteopt: the B200-native optimizer step of the Mote trainer (Muon + AdamW + global grad-norm clip), as a C ABI.
 *
 * Every entry point takes plain device pointers, element counts, host-side hyperparameters and the CUDA stream to
 * enqueue on; none allocates device memory, none synchronises the host. Scratch memory is the caller's
 * `workspace` (query its size with the matching *_workspace_size function; it must stay allocated until the work
 * enqueued on `stream` has finished; 256-byte aligned). The first 256 bytes of the workspace are a header: the status
 * word and the grad norm and clip coefficient of the last call that uses them (a step, a clip or a Newton-Schulz call
 * resets the header when it starts), which moteopt_read_status() reads back. Entry points that use a workspace only
 * for partial sums (moteopt_muon_apply_ex) leave the header alone.
 *
 * Every function returns MOTEOPT_OK (0) or a negative error code; moteopt_last_error() describes the last failure
 * of the calling thread. References below are to the reference project noahsabaj/mote, path:line.
 */
#ifndef MOTEOPT_H_
#define MOTEOPT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOTEOPT_API __attribute__((visibility("default")))
#else
#define MOTEOPT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* moteopt_stream_t; /* a cudaStream_t; NULL = the legacy default stream */

#define MOTEOPT_OK 0
#define MOTEOPT_ERR_INVALID (-1)   /* bad argument: shape, dtype, null pointer, workspace too small */
#define MOTEOPT_ERR_CUDA (-2)      /* a CUDA runtime call or kernel launch failed */
#define MOTEOPT_ERR_LIMIT (-3)     /* more tensors than one call supports */
#define MOTEOPT_ERR_DEVICE (-4)    /* the current device is not an sm_100 (B200-class) GPU */

#define MOTEOPT_DTYPE_F32 0
#define MOTEOPT_DTYPE_BF16 1

/* status word bits (moteopt_read_status) */
#define MOTEOPT_STATUS_WAIT_TIMEOUT 1   /* a pipeline wait in the Newton-Schulz kernel gave up (a library bug) */
#define MOTEOPT_STATUS_ABORTED 2        /* a kernel unwound early after such a timeout */
#define MOTEOPT_STATUS_NONFINITE 4      /* the global grad norm was NaN or Inf (the step proceeds, as torch's does) */

/* One Muon parameter: a 2-D matrix [rows, cols] or a 3-D stack [batch, rows, cols] of matrices that are
 * orthogonalised one by one (mote/train/muon.py:46-100, the `_muon_stack` case of muon.py:121). */
typedef struct moteopt_muon_param {
  float* param;                 /* fp32, contiguous */
  const void* grad;             /* same shape, fp32 or bf16 (grad_dtype), contiguous */
  float* momentum_buffer;       /* fp32, same shape; zeros before the first step (muon.py:66-67) */
  int64_t batch;                /* 1 for a matrix */
  int64_t rows, cols;
  double lr;                    /* the effective lr: the group's, or its `param_lr` override (muon.py:77) */
  double decay;                 /* the decoupled decay d of muon.py:78 (lr*wd, or lr^2/lr_max*wd for Muon-SW); 0 = none */
  double momentum;              /* muon.py:55 */
  int nesterov;                 /* muon.py:70 */
  int grad_dtype;               /* MOTEOPT_DTYPE_* */
} moteopt_muon_param;

typedef struct moteopt_muon_config {
  int ns_steps;                 /* Newton-Schulz iterations (muon.py:47, default 5) */
  double rms_scale;             /* update scale = rms_scale * sqrt(max(rows, cols)) (muon.py:82, default 0.2) */
  double ns_eps;                /* normalisation epsilon (muon.py:27, 1e-7) */
  int ns_variant;               /* 0 (default): the reference's iteration (muon.py:37-40), bit for bit. 1: the Gram
                                   Newton-Schulz variant the reference's research notes propose
                                   (docs/research/efficiency-campaign-2026-08-23.md:903-911), opt-in and NOT the
                                   reference's iteration, on every matrix whose long side is at least twice its short
                                   one (the others keep the reference iteration): R = X X^T once, the iteration on the
                                   small m x m side, X = Q X at the end, each product rounded once. c1: 28 % fewer
                                   FLOPs. Size its workspace with the *_cfg / *_variant size functions. */
} moteopt_muon_config;

/* One AdamW tensor (torch.optim.AdamW as constructed at mote/train/train.py:98). */
typedef struct moteopt_adamw_tensor {
  float* param;
  const void* grad;
  float* exp_avg;               /* zeros before the first step */
  float* exp_avg_sq;            /* zeros before the first step */
  int64_t numel;
  double lr;
  double weight_decay;
  int64_t step;                 /* the step count including this update (1 on the first step) */
  int grad_dtype;
} moteopt_adamw_tensor;

typedef struct moteopt_adamw_hparams {
  double beta1, beta2, eps;     /* train.py:98: betas=(0.9, beta2), eps=1e-8 */
  float* device_step;           /* NULL: bias corrections from each tensor's host `step`. Else a device fp32 step
                                   counter shared by every tensor: the call adds 1 to it and computes the bias
                                   corrections on the device (the form torch's capturable AdamW keeps), so a captured
                                   CUDA graph of the step stays correct on replay */
} moteopt_adamw_hparams;

/* Gradient pre-processing of mote/train/train.py:944-946. */
typedef struct moteopt_grad_config {
  int clip;                     /* 1: clip_grad_norm_(all params, max_norm) before the updates */
  double max_norm;
  double grad_divisor;          /* train.py:945: grads /= total_n first; 0 or 1 = no division */
  const float* grad_divisor_device; /* or, when non-NULL, total_n as a DEVICE fp32 scalar, read by the kernels (the
                                   trainer's total_n is a GPU tensor: no host round trip, and a captured step reads
                                   each replay's value); overrides grad_divisor */
} moteopt_grad_config;

/* Optional work fused into moteopt_optimizer_step_ex (no counterpart in the reference's step, which does this work
 * in separate passes after it).
 *   ema:        per tensor, in call order (the n_adamw AdamW tensors, then the n_muon Muon params), an fp32 buffer
 *               shaped like the param, or NULL: e = lerp(e, p_new, ema_weight) in the pass that writes p, i.e.
 *               mote/train/train.py:950-953 (_foreach_lerp_(ema, params, 1 - decay)) for the stepped params.
 *               NULL array: no EMA.
 *   muon_norms: n_muon device floats, or NULL: ||p_new||_F of each Muon param (mote/train/elr.py:85-87, the
 *               NormTracker sample), reduced in a fixed order from the apply pass. */
typedef struct {
  float* const* ema;
  double ema_weight;
  float* muon_norms;
  /* lr:          DEVICE array of n_adamw + n_muon doubles, each tensor's lr for this step (AdamW tensors, then Muon
   *              params), read by the kernels instead of the structs' lr: a learning-rate schedule (train.py:177-179
   *              set_lr, elr.py param_lr) then needs no new launch parameters, so a captured step can replay it.
   *              AdamW's decay is lr * weight_decay; a Muon param's decay is lr * muon_wd[i], or
   *              (lr * lr / muon_lr_max[i]) * muon_wd[i] when muon_lr_max[i] > 0 (Muon-SW, muon.py:76-79).
   *              NULL: the structs' lr and decay.
   * muon_wd, muon_lr_max: HOST arrays of n_muon doubles, required with lr when n_muon > 0. */
  const double* lr;
  const double* muon_wd;
  const double* muon_lr_max;
} moteopt_step_extras;

MOTEOPT_API int moteopt_version(void);
MOTEOPT_API const char* moteopt_last_error(void);

/* Measurement hooks (no counterpart in the reference, which has no kernels of its own). The launch count is the
 * number of kernels this library has enqueued since it was loaded. With events set (two cudaEvent_t, or NULL to
 * clear), every later moteopt_optimizer_step / moteopt_muon_step on the calling thread records the first before its
 * first Newton-Schulz launch and the second after its last, on the step's stream. */
MOTEOPT_API unsigned long long moteopt_launch_count(void);
MOTEOPT_API int moteopt_profile_ns_events(void* start_event, void* end_event);

/* Index checks (no counterpart in the reference; the stand-in for a memory checker, which this library's GPUs do not
 * run). Built with -DMOTE_OPT_CHECKS (libmoteopt_checked.so), every kernel checks the tensor, chunk, tile and TMEM
 * indices it derives and counts the failures on the device; the count of the current device is returned (and
 * cleared with `clear`), after synchronising the device. A release build compiles no check and returns 0; -1 means
 * a CUDA error (moteopt_last_error). */
MOTEOPT_API long long moteopt_check_count(int clear);

/* Newton-Schulz launch mode (no counterpart in the reference). 1: all iterations of a step run as one cooperative
 * launch whose tiles wait on per-matrix completion counters; 0: one launch per phase and iteration; -1 (the
 * default): the persistent launch for problems of up to 48 waves of tiles per iteration, per-phase launches above.
 * All compute the same bits. Process-wide; returns the previous mode. */
MOTEOPT_API int moteopt_ns_set_persistent(int mode);
/* Whether a matrix with more rows than columns (both multiples of 8) is iterated as stored (1, the default: A = X^T X,
 * X' = a X + X B, the same products in the same order as the transposed iteration, and no transposing passes) or as
 * its transpose (0). Returns the previous setting; it applies to calls made after it (no counterpart in the
 * reference). */
MOTEOPT_API int moteopt_ns_set_tall(int on);

/* Read (and optionally clear) the workspace's status word and the last [total norm, clip coefficient].
 * Synchronises `stream`. Either output may be NULL. */
MOTEOPT_API int moteopt_read_status(void* workspace, int* status, float* norm_and_coef, int clear, moteopt_stream_t stream);

/* ---- the whole optimizer step of mote/train/train.py:944-947: grads /= total_n; clip_grad_norm_(params, clip);
 *      MultiOpt.step() = AdamW.step() then Muon.step() (train.py:64-66). The clip is folded into the update
 *      kernels: the grads are read, never rewritten. `out_norm` (device, may be NULL) receives the total grad norm
 *      before clipping, which clip_grad_norm_ returns and the trainer logs as grad_norm (train.py:954). */
MOTEOPT_API size_t moteopt_optimizer_step_workspace_size(const moteopt_muon_param* muon, int n_muon, int ns_steps,
                                             const moteopt_adamw_tensor* adamw, int n_adamw);
/* The same for a given Muon config (ns_steps and ns_variant: the Gram variant needs three more m x m buffers per
 * eligible matrix). */
MOTEOPT_API size_t moteopt_optimizer_step_workspace_size_cfg(const moteopt_muon_param* muon, int n_muon,
                                                             const moteopt_muon_config* cfg,
                                                             const moteopt_adamw_tensor* adamw, int n_adamw);
MOTEOPT_API int moteopt_optimizer_step(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* muon_cfg,
                           const moteopt_adamw_tensor* adamw, int n_adamw, const moteopt_adamw_hparams* adamw_hp,
                           const moteopt_grad_config* grad_cfg, float* out_norm, void* workspace,
                           size_t workspace_bytes, moteopt_stream_t stream);
/* moteopt_optimizer_step plus the fused extras above (extras may be NULL). Same workspace size. */
MOTEOPT_API int moteopt_optimizer_step_ex(const moteopt_muon_param* muon, int n_muon,
                                          const moteopt_muon_config* muon_cfg, const moteopt_adamw_tensor* adamw,
                                          int n_adamw, const moteopt_adamw_hparams* adamw_hp,
                                          const moteopt_grad_config* grad_cfg, const moteopt_step_extras* extras,
                                          float* out_norm, void* workspace, size_t workspace_bytes,
                                          moteopt_stream_t stream);

/* ---- the sharded (multi-GPU) step of the same path, which the reference does not have: each rank updates only the
 *      parameters it owns, so the global clip is assembled from per-rank sums of squares.
 *      moteopt_grad_sumsq: out_sum (device fp64) = sum over the listed grads of (g / grad_divisor)^2 (fixed order).
 *      moteopt_clip_coef_from_sums: out_norm_coef (device, 2 floats) = [sqrt(sum of sums[0..n) in order),
 *      min(1, max_norm / (norm + 1e-6)) or 1 when clip == 0].
 *      moteopt_optimizer_step_with_coef: moteopt_optimizer_step with the clip coefficient given (device float; NULL
 *      for none) instead of computed. */
MOTEOPT_API size_t moteopt_grad_sumsq_workspace_size(const int64_t* numels, int n);
MOTEOPT_API int moteopt_grad_sumsq(const void* const* grads, const int64_t* numels, const int* dtypes, int n,
                                   double grad_divisor, double* out_sum, void* workspace, size_t workspace_bytes,
                                   moteopt_stream_t stream);
MOTEOPT_API int moteopt_clip_coef_from_sums(const double* sums, int n, int clip, double max_norm, float* out_norm_coef,
                                            moteopt_stream_t stream);

/*      The clip's norm as the single-GPU step forms it (the norm of the per-tensor norms, torch's get_total_norm), from
 *      per-rank per-tensor sums: every grad tensor has an index t in [0, n_tensors) and a rank holds at most one
 *      piece of it (a ZeRO-1 slice or the whole tensor).
 *      moteopt_grad_sumsq_tensors: out_tensor_sums[tensors[i]] (device fp64, n_tensors) = sum over grad i of
 *      (g / grad_divisor)^2, 0 for indices no grad names.
 *      moteopt_peer_reduce_sumsq: the grad reduce-scatter over peer memory fused with the same sums. Piece p sums its
 *      `world` sources (src[q]: the piece in rank q's grads, mapped into this process, e.g. through
 *      moteopt_ipc_import; src[rank] local) element by element in fp32 in rank order, rounds once to `dtype` and
 *      stores to dst; out_tensor_sums as above over the reduced values. Every source must be complete before the
 *      call's kernels run and must not change until they end (the caller orders that, e.g. with a collective).
 *      moteopt_clip_coef_from_tensor_sums: sums [world][n_tensors] (every rank's out_tensor_sums, e.g. all-gathered)
 *      -> out_norm_coef (device, 2 floats) = [total norm, clip coefficient]: per tensor the ranks' sums added in rank
 *      order, its fp32 norm, then the fp32 norm of those norms and min(1, max_norm / (norm + 1e-6)) (1 when
 *      clip == 0), as moteopt_optimizer_step forms them. */
#define MOTEOPT_MAX_PEERS 8
typedef struct {
  void* dst;                           /* this rank's reduced piece */
  const void* src[MOTEOPT_MAX_PEERS];  /* the piece in rank q's grads, q < world */
  int64_t numel;
  int dtype;                           /* MOTEOPT_DTYPE_*: sources and destination */
  int tensor;                          /* index of the grad tensor the piece belongs to */
} moteopt_peer_piece;
MOTEOPT_API int moteopt_grad_sumsq_tensors(const void* const* grads, const int64_t* numels, const int* dtypes,
                                           const int* tensors, int n, int n_tensors, double grad_divisor,
                                           double* out_tensor_sums, void* workspace, size_t workspace_bytes,
                                           moteopt_stream_t stream);
MOTEOPT_API size_t moteopt_peer_reduce_workspace_size(const moteopt_peer_piece* pieces, int n_pieces);
MOTEOPT_API int moteopt_peer_reduce_sumsq(const moteopt_peer_piece* pieces, int n_pieces, int world, int n_tensors,
                                          double grad_divisor, double* out_tensor_sums, void* workspace,
                                          size_t workspace_bytes, moteopt_stream_t stream);
MOTEOPT_API int moteopt_clip_coef_from_tensor_sums(const double* sums, int world, int n_tensors, int clip,
                                                   double max_norm, float* out_norm_coef, moteopt_stream_t stream);
MOTEOPT_API int moteopt_optimizer_step_with_coef(const moteopt_muon_param* muon, int n_muon,
                                                 const moteopt_muon_config* muon_cfg, const moteopt_adamw_tensor* adamw,
                                                 int n_adamw, const moteopt_adamw_hparams* adamw_hp,
                                                 double grad_divisor, const float* grad_coef, void* workspace,
                                                 size_t workspace_bytes, moteopt_stream_t stream);

/* The sharded step's exchange of Muon updates (no counterpart in the reference, which has no multi-GPU step: owners
 * compute, every rank applies). moteopt_optimizer_step_with_coef_out is moteopt_optimizer_step_with_coef except that
 * each Muon parameter's orthogonalised update O (bf16, the parameter's own shape and orientation, the value the
 * reference casts to fp32 at mote/train/muon.py:99) is written to muon_updates[i] instead of being applied; the
 * momentum buffers are updated as usual. moteopt_muon_apply applies such updates, p = p*(1-decay) (if decay);
 * p += -lr*(O*scale) with scale = rms_scale*sqrt(max(rows, cols)) (muon.py:82, :97-99), to n parameters (grad and
 * momentum_buffer are not read); it needs no workspace. Together they give the same bits as the in-step apply. */
MOTEOPT_API int moteopt_optimizer_step_with_coef_out(const moteopt_muon_param* muon, int n_muon,
                                                     const moteopt_muon_config* muon_cfg,
                                                     const moteopt_adamw_tensor* adamw, int n_adamw,
                                                     const moteopt_adamw_hparams* adamw_hp, double grad_divisor,
                                                     const float* grad_coef, void* const* muon_updates, void* workspace,
                                                     size_t workspace_bytes, moteopt_stream_t stream);
MOTEOPT_API int moteopt_muon_apply(const moteopt_muon_param* muon, int n, const moteopt_muon_config* muon_cfg,
                                   const void* const* updates, moteopt_stream_t stream);
/* moteopt_muon_apply with the trainer's two after-step reads of the weights fused into the same pass:
 * ema[i] (fp32, the param's shape; the array or an entry may be NULL) = lerp(ema[i], p_new, ema_weight), as
 * torch._foreach_lerp_ at mote/train/train.py:950-953; norms (device, n floats, may be NULL) receives ||p_new||_F of
 * each param (mote/train/elr.py:85-87, NormTracker.sample), summed in fp64 in a fixed order. The norms need a
 * workspace of moteopt_muon_apply_workspace_size bytes (256-byte aligned); without norms it may be NULL. */
MOTEOPT_API size_t moteopt_muon_apply_workspace_size(const moteopt_muon_param* muon, int n);
MOTEOPT_API int moteopt_muon_apply_ex(const moteopt_muon_param* muon, int n, const moteopt_muon_config* muon_cfg,
                                      const void* const* updates, float* const* ema, double ema_weight, float* norms,
                                      void* workspace, size_t workspace_bytes, moteopt_stream_t stream);
/* ema[i] = lerp(ema[i], params[i], weight) over n fp32 tensors: torch._foreach_lerp_(ema, params, weight), the EMA
 * update of mote/train/train.py:950-953 (weight = 1 - ema_decay), bit for bit, for params that no fused pass writes. */
MOTEOPT_API int moteopt_ema_lerp(float* const* ema, const float* const* params, const int64_t* numels, int n,
                                 double weight, moteopt_stream_t stream);

/* Peer mappings for the sharded step (no counterpart in the reference). A rank exports the device allocation that
 * holds `ptr` (a CUDA IPC handle of MOTEOPT_IPC_HANDLE_BYTES bytes, plus ptr's byte offset inside it); another process
 * on the same node imports the handle (base pointer of the mapping; add the offset) and may then pass pointers into
 * it, e.g. a peer's Muon updates to moteopt_muon_apply, which reads them over NVLink with plain loads. The exporter's
 * allocation must stay alive until every importer has closed its mapping. */
#define MOTEOPT_IPC_HANDLE_BYTES 64
MOTEOPT_API int moteopt_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out);
MOTEOPT_API int moteopt_ipc_import(const void* handle, void** base_out);
MOTEOPT_API int moteopt_ipc_close(void* base);

/* ---- Muon.step() of one or more param groups (mote/train/muon.py:52-100). Parameters whose grad is NULL are
 *      skipped by the caller (muon.py:61-62). `grad_scale` (device, may be NULL) multiplies every grad first. */
MOTEOPT_API size_t moteopt_muon_step_workspace_size(const moteopt_muon_param* muon, int n_muon, int ns_steps);
MOTEOPT_API size_t moteopt_muon_step_workspace_size_cfg(const moteopt_muon_param* muon, int n_muon,
                                                        const moteopt_muon_config* cfg);
MOTEOPT_API int moteopt_muon_step(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* cfg,
                      const float* grad_scale, void* workspace, size_t workspace_bytes, moteopt_stream_t stream);

/* ---- torch.optim.AdamW.step() (train.py:98; torch's single-tensor update with amsgrad=False). */
MOTEOPT_API int moteopt_adamw_step(const moteopt_adamw_tensor* adamw, int n_adamw, const moteopt_adamw_hparams* hp,
                       const float* grad_scale, moteopt_stream_t stream);

/* ---- torch.nn.utils.clip_grad_norm_(params, max_norm) (train.py:946): the 2-norm of the per-tensor norms, then
 *      grads *= min(1, max_norm / (norm + 1e-6)) in place. `out_norm` (device, may be NULL) receives the norm. */
MOTEOPT_API size_t moteopt_clip_grad_norm_workspace_size(const int64_t* numels, int n);
MOTEOPT_API int moteopt_clip_grad_norm(void* const* grads, const int64_t* numels, const int* dtypes, int n, double max_norm,
                           float* out_norm, void* workspace, size_t workspace_bytes, moteopt_stream_t stream);

/* ---- clip_grad_norm_ for callers that cannot allocate device memory. It has no counterpart in the reference: it
 *      does what moteopt_clip_grad_norm does, but keeps its scratch in a fixed array inside this library instead of
 *      a caller-provided workspace, for callers that may not call cudaMalloc (or any allocating routine) at the
 *      point of the call: a host runtime with its own memory pool that forbids outside allocations, a region where
 *      allocation would break stream ordering, or a C caller without an allocator of its own. Limit: the grads'
 *      element counts, each rounded up to a multiple of 16384, may sum to at most 65536 x 16384 (2^30) elements,
 *      and n <= 4096; beyond that it returns MOTEOPT_ERR_LIMIT and does nothing. The array (512 KB + 256 B) lives on
 *      every device that loads the library until the process exits. The first call on a device looks up the
 *      array's device address; make that first call before any CUDA graph capture on that device. Calls share the
 *      array: calls that can overlap on the GPU (different streams without ordering, or several host threads) race
 *      and must be serialised by the caller. `out_norm` (device, may be NULL) receives the total norm. This call has
 *      no workspace header for moteopt_read_status to read: a NaN or Inf grad shows only as a NaN or Inf *out_norm
 *      (the grads are then scaled by torch's coefficient for that norm, as moteopt_clip_grad_norm does); a caller
 *      that needs the check reads out_norm back. */
MOTEOPT_API int moteopt_clip_grad_norm_noalloc(void* const* grads, const int64_t* numels, const int* dtypes, int n,
                                               double max_norm, float* out_norm, moteopt_stream_t stream);

/* ---- newton_schulz(G, steps, eps) (mote/train/muon.py:26-43): G [batch, rows, cols] fp32 or bf16 -> out bf16 of
 *      the same shape. Every matrix is normalised by its own Frobenius norm; the iteration runs on the transpose
 *      of a matrix with more rows than columns. */
MOTEOPT_API size_t moteopt_newton_schulz_workspace_size(int64_t batch, int64_t rows, int64_t cols);
MOTEOPT_API int moteopt_newton_schulz(const void* G, int g_dtype, void* out, int64_t batch, int64_t rows, int64_t cols,
                          int steps, double eps, void* workspace, size_t workspace_bytes, moteopt_stream_t stream);
/* The same with the Newton-Schulz variant chosen (moteopt_muon_config::ns_variant; 0 is moteopt_newton_schulz). */
MOTEOPT_API size_t moteopt_newton_schulz_workspace_size_variant(int64_t batch, int64_t rows, int64_t cols, int ns_variant);
MOTEOPT_API int moteopt_newton_schulz_variant(const void* G, int g_dtype, void* out, int64_t batch, int64_t rows,
                                              int64_t cols, int steps, double eps, int ns_variant, void* workspace,
                                              size_t workspace_bytes, moteopt_stream_t stream);

/* ---- the lossfree MoE router's bias step after the optimizer step: MoESwiGLU.update_bias
 *      (mote/model/moe.py:147-159), called for every MoE layer at mote/train/train.py:948-949. One launch for all
 *      layers and no host round trip (the reference's `load.sum() <= 0` test reads the sum back on the host).
 *      Per layer: if the loads sum to <= 0 nothing changes; else bias += gamma * (sgn - mean(sgn)) with
 *      sgn = sign((mean(load) - load) / max(mean(load), 1e-9)), and the loads are zeroed. The caller passes only
 *      layers whose router is "lossfree" with gamma > 0 (moe.py:151-152 returns before touching the others). */
typedef struct moteopt_moe_bias {
  float* load_acc;      /* [n_experts] fp32 token counts accumulated since the last step (_load_acc) */
  float* expert_bias;   /* [n_experts] fp32 routing bias (expert_bias), updated in place */
  int n_experts;        /* >= 0; 0 skips the layer */
  float gamma;          /* bias_gamma, rounded to fp32 as torch does for a Python scalar times an fp32 tensor */
} moteopt_moe_bias;
MOTEOPT_API int moteopt_moe_update_bias(const moteopt_moe_bias* layers, int n, moteopt_stream_t stream);

/* ---- self-tests of two device primitives the optimizer's kernels rely on (diagnostics with no counterpart in the
 *      reference; nothing in the optimizer step calls them).
 *      moteopt_selftest_divide: out[i] = a[i] / d[i] (n fp32 device values) computed the way the Newton-Schulz
 *      normalisation divides by a shared norm (a correctly rounded reciprocal, one product, one Markstein
 *      correction), so a caller can hold it against IEEE division.
 *      moteopt_selftest_grad_divide: out[i] = a[i] / d (one divisor for all n values) computed the way the
 *      normalisation divides a matrix by its norm, four entries at a time (groups of four; the tail one by one).
 *      moteopt_selftest_wait_timeout: runs the kernels' bounded waits on something that never completes and returns
 *      once they have given up: mode 0 waits on `counter` (a device int the caller keeps below 1: a persistent
 *      Newton-Schulz tile's input counter that nothing adds to), mode 1 on an mbarrier nothing arrives on (a pipeline
 *      stage whose loads never land). Two CTAs wait; CTA 0 gives up after limit_seconds (1 us .. 0.25 s) and sets
 *      MOTEOPT_STATUS_WAIT_TIMEOUT in *status (device int); CTA 1 waits with four times the limit and, in mode 0,
 *      stops as soon as it sees that bit, as every CTA of a launch does. Each CTA that unwound sets
 *      MOTEOPT_STATUS_ABORTED; elapsed_ns (device, 2 values) receives how long each CTA waited. The GPU context stays
 *      usable afterwards. */
MOTEOPT_API int moteopt_selftest_divide(const float* a, const float* d, float* out, int64_t n, moteopt_stream_t stream);
MOTEOPT_API int moteopt_selftest_grad_divide(const float* a, float d, float* out, int64_t n, moteopt_stream_t stream);
MOTEOPT_API int moteopt_selftest_wait_timeout(int mode, double limit_seconds, int* counter, int* status,
                                              unsigned long long* elapsed_ns, moteopt_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOTEOPT_H_ */
