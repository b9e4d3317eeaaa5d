// Launch descriptors of the Newton-Schulz phase kernel, shared by host and device code.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace moteopt {
namespace ns {

constexpr int TM = 256, TN = 256;   // output tile of a CTA pair (cta_group::2 MMA: M = 256, N = 256)
constexpr int HM = 128;             // rows of the tile per CTA (its TMEM lanes), and rows of each operand it loads
constexpr int BK = 64;              // K per pipeline stage: one 128-byte swizzle row of bf16
constexpr int STAGES = 6;
constexpr int A_BYTES = HM * BK * 2;          // 16 KB per CTA and stage
constexpr int B_BYTES = (TN / 2) * BK * 2;    // 16 KB per CTA and stage
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kEpiWarps = 8;   // two epilogue warps per TMEM lane quarter, each owning half of the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;   // warp 0: TMA producer, warp 1: MMA issuer + TMEM owner, 2-9: epilogue
constexpr int EPI_TILE = 32;                                 // epilogue subtile: 32 rows x 32 columns, bf16
constexpr int EPI_BUF_BYTES = EPI_TILE * EPI_TILE * 2;       // 2 KB, 64-byte swizzled
constexpr int EPI_BYTES = kEpiWarps * 2 * EPI_BUF_BYTES;     // two subtiles per epilogue warp (operand in, result out)
constexpr int kSmemBytes = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*alignment slack*/ + 512 /*barriers*/;
constexpr uint32_t kTmemCols = 512;   // two 128 x 256 fp32 accumulators per CTA
constexpr int kArrivalsPerTile = 2 * kEpiWarps;   // completion arrivals of one pair tile (every epilogue warp)

constexpr int kMaxGroups = 8;     // shape groups per launch
constexpr int kMaxChunks = 8;     // runs of matrices an iteration is split into (persistent mode)
constexpr int kMaxApply = 512;    // matrices per shape group

enum Phase : int {
  kGram = 0,     // A = X X^T                         (m x m, K = n)
  kPoly = 1,     // B = b*A + c*(A A)                 (m x m, K = m)
  kUpdate = 2,   // X' = a*X + B X                 (m x n, K = m)
};

// One shape group: `count` matrices that share (m, n) after the transpose rule (m <= n). Buffers are
// [count][m][n] (X) and [count][m][m] (A, B), bf16, row-major, with m and n padded up to multiples of 8 and the
// padding kept at zero (the iteration maps zero rows/columns to zero).
struct alignas(64) Group {
  CUtensorMap xk[2];    // X ping/pong as a K-major operand: dims {n, m, count}, box {64, 128, 1}
  CUtensorMap xmn[2];   // X ping/pong as an MN-major operand: dims {n, m, count}, box {64, 64, 1}
  CUtensorMap ak;       // A: dims {m, m, count}, box {64, 128, 1}
  CUtensorMap bk;       // B: dims {m, m, count}, box {64, 128, 1}
  CUtensorMap amn;      // A as an MN-major operand (a stored upper block read transposed): box {64, 64, 1}
  CUtensorMap bmn;      // B likewise
  CUtensorMap xe[2];    // epilogue views (box {32, 32, 1}, 64-byte swizzle): X ping/pong
  CUtensorMap ae;       //   A
  CUtensorMap be;       //   B
  __nv_bfloat16* x[2];
  __nv_bfloat16* a;
  __nv_bfloat16* b;
  int m, n;             // padded dims of X (m <= n)
  int mv, nv;           // valid dims of X
  int count;            // matrices in the group
  int first;            // index of the group's first matrix in the launch's matrix numbering
  int transposed;       // X = u^T (the parameter has more rows than columns)
  int tall;             // X is a tall matrix as stored: [count][n][m] (n >= m rows); the Gram phase is X^T X with both
                        // operands MN-major, the update X' = a X + X B runs over n x m tiles with B as the right factor
};

// The Muon apply of one matrix (mote/train/muon.py:93-99): p = p*(1-decay) (if decay), p += -lr*(O*scale).
struct MatApply {
  float* p;             // first element of this matrix inside its (2-D or 3-D) parameter
  float neg_lr;
  float decay_mul;
  float scale;
  int has_decay;
};

// A launch walks the tile sequence [iteration][chunk][phase][group][matrix][tile] over [t_begin, t_end): chunk c of
// an iteration holds, in every group, the matrices [ck_b0[c][g], ck_b0[c + 1][g]) (one chunk outside the persistent
// mode, where the phases of an iteration must be contiguous).
struct Launch {
  Group g[kMaxGroups];
  int n_groups;
  int src0;                              // X buffer holding the iterate at iteration 0 (iteration i reads src0 ^ (i & 1))
  int t_begin, t_end;
  int per_iter;                          // tiles of one iteration, all three phases
  int phase_tiles[3];                    // tiles of each phase in one iteration
  int tile_start[3][kMaxGroups + 1];     // per phase: prefix over the groups
  int n_chunks;
  int chunk_start[kMaxChunks + 1];       // per iteration: prefix of tiles over the chunks
  int ck_phase_tiles[kMaxChunks][3];     // tiles of each phase within a chunk
  int ck_tile_start[kMaxChunks][3][kMaxGroups + 1];   // per chunk and phase: prefix over the groups
  int ck_b0[kMaxChunks + 1][kMaxGroups]; // first matrix of each group in each chunk
  int tiles_m[kMaxGroups];               // row blocks of X (= both block counts of A and B)
  int tiles_n[kMaxGroups];               // column blocks of X
  int* done;                             // persistent mode: [matrix][phase] completion arrivals; null: one phase per launch
  int* status;
  float ca, cb, cc;                      // the quintic's coefficients a, b, c (mote/train/muon.py:31); ca = 0 with
                                         // no_aux for a plain product
  int round_once;                        // 0: the reference's rounding of every elementwise op; 1: the product and its
                                         // a*Y (b*A) term summed in fp32 and rounded once (the Gram variant)
  int no_aux;                            // kUpdate without the a*Y term: out = bf16(B X) (the Gram variant's Q X0)
};
// passed by value as a __grid_constant__ kernel parameter: within the 32764-byte parameter limit of sm_70+ launches
static_assert(sizeof(Launch) <= 32764, "Launch exceeds the kernel parameter space");

}  // namespace ns
}  // namespace moteopt
