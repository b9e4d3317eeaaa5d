// Argument blocks of the memory-bound multi-tensor kernels, shared by host and device code. Every block is passed
// by value as a kernel parameter (CUDA 12.1+ allows up to 32 KB), so a step needs no descriptor upload and no
// allocation. Lists longer than one block holds are split into several launches by the host.
#pragma once

#include <cstdint>

namespace moteopt {

// Index checks (-DMOTE_OPT_CHECKS builds only): a failed MO_CHECK counts in g_check_fails and the kernel goes on.
#ifdef MOTE_OPT_CHECKS
__device__ unsigned long long g_check_fails;
#define MO_CHECK(cond)                                     \
  do {                                                     \
    if (!(cond)) atomicAdd(&::moteopt::g_check_fails, 1ull); \
  } while (0)
#else
#define MO_CHECK(cond) \
  do {                 \
  } while (0)
#endif

constexpr int kChunk = 16384;          // elements per work unit of the multi-tensor kernels
constexpr int kMtThreads = 256;
// AdamW's small work unit: two 16-byte vectors per thread, so that a few hundred thousand AdamW elements (a
// trainer's embeddings and norms) still spread over every SM, one load round trip per chunk. Launches with enough
// elements to fill the GPU in kChunk units use those instead (fewer registers, more blocks per SM).
constexpr int kAdamChunk = 8 * kMtThreads;

enum DType : int { kF32 = 0, kBF16 = 1 };

// ---- global grad norm (torch.nn.utils.clip_grad_norm_, called at mote/train/train.py:946)
constexpr int kMaxNormSeg = 512;
struct SumsqSeg {
  const void* g;
  int64_t numel;
  int dtype;
  int pad_;
};
struct SumsqArgs {
  int n;
  int chunk_base;            // index of this launch's first chunk in the partials array
  int has_div;               // divide by `div` first (train.py:945, grads /= total_n)
  float div;
  const float* div_dev;      // or, when non-null, by this device scalar (read once per block)
  double* partials;          // one fp64 sum of squares per chunk
  int chunk_start[kMaxNormSeg + 1];
  SumsqSeg seg[kMaxNormSeg];
};

// The sharded step's grad reduce-scatter over peer memory, fused with the clip's sums of squares: one piece is one
// grad tensor's share of this rank's segment; src[q] is where that share starts in rank q's grad region (mapped into
// this process; src[rank] is local); dst receives the sum over the ranks.
constexpr int kMaxPeers = 8;
constexpr int kMaxPeerSegs = 160;
struct PeerSeg {
  void* dst;
  const void* src[kMaxPeers];
  int64_t numel;
  int dtype;
  int pad_;
};
struct PeerReduceArgs {
  int n;
  int world;
  int chunk_base;            // index of this launch's first chunk in the partials array
  int has_div;
  float div;
  double* partials;          // one fp64 sum of squares per chunk of the reduced grads
  int chunk_start[kMaxPeerSegs + 1];
  PeerSeg seg[kMaxPeerSegs];
};

// Per-tensor sums of squares from chunk partials: out[tensor[p]] = sum of piece p's partials, 0 for tensors without a
// piece here.
constexpr int kMaxPieceSums = 2048;
struct PieceSumArgs {
  int n_pieces;
  int n_tensors;
  const double* partials;
  double* out;
  int chunk_start[kMaxPieceSums + 1];
  int tensor[kMaxPieceSums];
};

constexpr int kMaxFinalTensors = 4096;

// total norm and clip coefficient from every rank's per-tensor sums of squares ([world][n_tensors], fp64)
struct TensorCoefArgs {
  int world;
  int n_tensors;
  int has_clip;
  float max_norm;
  const double* sums;
  float* out;                // out[0] = total norm, out[1] = clip coefficient (1 when no clip)
  int* status;
};
struct FinalizeArgs {
  int n_tensors;
  int has_clip;
  float max_norm;
  const double* partials;
  float* out;                // out[0] = total norm, out[1] = clip coefficient (1 when no clip)
  int* status;
  int tensor_chunk_start[kMaxFinalTensors + 1];
};

// ---- the clip coefficient from per-rank sums of squares (sharded step): total = sqrt(sum in rank order)
struct CoefArgs {
  int n;
  int has_clip;
  float max_norm;
  const double* sums;
  float* out;                // out[0] = total norm, out[1] = clip coefficient
  int* status;
};

// ---- the weights' EMA (mote/train/train.py:950-953: _foreach_lerp_(ema, params, w) after the step), fused into the
// passes that write the params: e = e + w*(p - e) for |w| < 0.5, else p - (p - e)*(1 - w), as torch's lerp
struct EmaConsts {
  float w, omw;              // weight, 1 - weight (fp32, as torch's opmath)
  int small;
  int pad_;
};

// ---- AdamW (torch.optim.AdamW single-tensor update, constructed at mote/train/train.py:98)
constexpr int kMaxAdamSeg = 256;
struct AdamSeg {
  float* p;
  const void* g;
  float* m;
  float* v;
  int64_t numel;
  float decay_mul;           // 1 - lr*wd (fp64 on the host, rounded once)
  float neg_step_size;       // -lr / (1 - beta1^t)
  float bc2_sqrt;            // sqrt(1 - beta2^t)
  int dtype;                 // grad dtype
  int has_decay;
  int pad_;
  double lr, wd;             // for the device-step mode, which recomputes the three scalars above per step
  float* ema;                // EMA of the param, lerped toward the updated param in the same pass, or null
  const double* lr_dev;      // this step's lr read on the device (schedules under graph capture), or null: lr
  double bc1;                // 1 - beta1^t (host step mode), for the device-lr step size
};
struct AdamArgs {
  int n;
  int has_div;
  float div;
  const float* div_dev;
  const float* coef;         // device clip coefficient, or null
  float lerp_w;              // 1 - beta1 (lerp weight)
  int lerp_small;            // weight < 0.5: m + w*(g-m); else g - (g-m)*(1-w)
  float one_minus_w;
  float beta2;
  float one_minus_beta2;
  float eps;
  const float* dstep;        // device step counter (already incremented for this step), or null: host scalars
  double beta1d, beta2d;
  EmaConsts ema;
  int chunk_start[kMaxAdamSeg + 1];
  AdamSeg seg[kMaxAdamSeg];
};

// ---- Muon momentum (mote/train/muon.py:66-70), one segment per matrix (a 3-D stack contributes one per slice)
constexpr int kMaxMomSeg = 512;
struct MomSeg {
  const void* g;
  float* buf;
  int64_t numel;
  float mom;
  int nesterov;
  int dtype;
  int pad_;
};
struct MomArgs {
  int n;
  int chunk_base;
  int has_div;
  float div;
  const float* div_dev;
  const float* coef;
  double* partials;          // per chunk: fp64 sum of u^2 (feeds the Newton-Schulz normalisation)
  int chunk_start[kMaxMomSeg + 1];
  MomSeg seg[kMaxMomSeg];
};

// ---- Newton-Schulz normalisation X0 = bf16(u / (||u||_F + eps)) with the transpose rule (muon.py:32-36)
constexpr int kMaxNormMat = 320;
constexpr int kNormTile = 64;
struct NormMat {
  const void* g;             // source: the grad (momentum mode) or G itself (direct mode)
  const float* buf;          // momentum buffer after this step's update (momentum mode), else null
  void* x;                   // destination [m_pad][n_pad] bf16 (zero padded)
  int rows, cols;            // the source matrix (R x C)
  int m_pad, n_pad;          // destination dims: (C, R) padded if transposed, else (R, C) padded
  int transposed;
  int dtype;
  float mom;
  int nesterov;
  int den_index;             // this matrix's ||u||_F + eps in NormArgs::den
  int pad_;
  int tiles_x;               // destination tiles along n_pad
  int tiles;                 // total destination tiles
};
struct NormArgs {
  int n;
  int has_div;
  float div;
  const float* div_dev;
  const float* coef;
  const float* den;          // per matrix: ||u||_F + eps (mat_denom_kernel)
  NormMat mat[kMaxNormMat];
};

// ---- the same normalisation for matrices that are iterated as they are stored (rows <= cols, no padding): X0 has
// the source's layout, so a matrix is a flat run of chunks and needs no transpose
constexpr int kMaxFlatSeg = 320;
struct FlatNormSeg {
  const void* g;             // grad (momentum mode) or G (direct mode)
  const float* buf;          // momentum buffer after this step's update, or null (direct mode)
  void* x;                   // X0 (bf16), same layout as the source
  int64_t numel;
  float mom;
  int nesterov;
  int dtype;
  int den_index;
};
struct FlatNormArgs {
  int n;
  int has_div;
  float div;
  const float* div_dev;
  const float* coef;
  const float* den;
  int chunk_start[kMaxFlatSeg + 1];
  FlatNormSeg seg[kMaxFlatSeg];
};

// ---- per-matrix Frobenius norm from the sum-of-squares partials: den = fp32(sqrt(sum)) + eps
constexpr int kMaxDenom = 4096;
struct DenomArgs {
  int n;
  int base;                  // den index of this launch's first matrix
  float eps;
  const double* partials;
  float* den;
  int chunk_start[kMaxDenom + 1];
};

// ---- copy the final iterate out of the workspace (standalone newton_schulz), or apply it (ns_steps == 0)
constexpr int kMaxOutMat = 256;
struct OutMat {
  const void* x;             // [m_pad][n_pad] bf16 iterate
  void* out;                 // bf16 [R][C] output, or the fp32 parameter in apply mode
  int rows, cols;            // R x C
  int m_pad, n_pad;
  int transposed;
  int tiles_x, tiles;
  float neg_lr, decay_mul, scale;
  int has_decay;
  float* ema;                // apply mode: EMA of the parameter ([R][C], fp32), or null
  double* partials;          // apply mode: per tile, the fp64 sum of the updated param's squares, or null
  const double* lr_dev;      // apply mode: this step's lr read on the device, or null (neg_lr / decay_mul above)
  double wd, lr_max;         // with lr_dev: decay = lr*wd, or (lr*lr/lr_max)*wd when lr_max > 0 (Muon-SW)
};
struct OutArgs {
  int n;
  int apply;
  EmaConsts ema;
  OutMat mat[kMaxOutMat];
};

// ---- copy-out / apply for matrices iterated as they are stored (the flat counterpart of OutArgs)
struct FlatOutSeg {
  const void* x;             // final iterate (bf16), same layout as the output
  void* out;                 // bf16 output, or the fp32 parameter in apply mode
  int64_t numel;
  float neg_lr, decay_mul, scale;
  int has_decay;
  float* ema;                // apply mode: EMA of the parameter (same layout), or null
  double* partials;          // apply mode: per chunk of the segment, the fp64 sum of the updated param's squares, or null
  const double* lr_dev;      // apply mode: this step's lr read on the device, or null (neg_lr / decay_mul above)
  double wd, lr_max;         // with lr_dev: decay = lr*wd, or (lr*lr/lr_max)*wd when lr_max > 0 (Muon-SW)
};
struct FlatOutArgs {
  int n;
  int apply;
  EmaConsts ema;
  int chunk_start[kMaxFlatSeg + 1];
  FlatOutSeg seg[kMaxFlatSeg];
};

// ---- in-place clip of the grads (standalone clip_grad_norm_)
struct ScaleArgs {
  int n;
  const float* coef;
  int chunk_start[kMaxNormSeg + 1];
  SumsqSeg seg[kMaxNormSeg];
};

// ---- the weights' EMA as a pass of its own (mote/train/train.py:950-953, torch._foreach_lerp_(ema, params, w)),
// for params that no fused pass writes (the sharded step's all-gathered AdamW region)
constexpr int kMaxLerpSeg = 512;
struct LerpSeg {
  float* ema;
  const float* p;
  int64_t numel;
};
struct LerpArgs {
  int n;
  EmaConsts ema;
  int chunk_start[kMaxLerpSeg + 1];
  LerpSeg seg[kMaxLerpSeg];
};

// ---- the lossfree MoE router's bias step after the optimizer step (mote/model/moe.py:147-159), one block per layer
constexpr int kMaxMoeLayers = 512;
struct MoeLayer {
  float* load;               // [experts] token counts since the last step (_load_acc), zeroed by the step
  float* bias;               // [experts] routing bias (expert_bias), updated in place
  int experts;
  float gamma;               // bias_gamma as fp32 (torch multiplies the fp32 tensor by the Python float in fp32)
};
struct MoeBiasArgs {
  int n;
  MoeLayer layer[kMaxMoeLayers];
};

}  // namespace moteopt
