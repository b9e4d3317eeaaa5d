// Newton-Schulz GEMM kernel for sm_100a: tcgen05.mma on CTA pairs, accumulators in TMEM, operands by TMA.
//
// The quintic iteration of mote/train/muon.py:37-40 for each matrix X (m x n, m <= n after the transpose rule):
//   kGram:   A  = bf16(X X^T)                                   (m x m, K = n)
//   kPoly:   B  = bf16( bf16(b*A) + bf16(c * bf16(A A)) )       (m x m, K = m)
//   kUpdate: X' = bf16( bf16(a*X) + bf16(B X) )                 (m x n, K = m)
// The rounding points are the reference's: every torch op on a bf16 tensor rounds its fp32 result to bf16. A and B
// are symmetric, so kGram and kPoly compute only the 256 x 256 blocks on and above the diagonal; a block below it is
// read as the transpose of its mirror block (an MN-major operand).
//
// Work. A launch walks the tile sequence [iteration][chunk][phase][group][matrix][tile] over [t_begin, t_end) (a
// chunk is a run of every group's matrices; the persistent launch of a large problem has two); CTA pair p
// takes tiles t_begin + p, t_begin + p + P, ... in order (P pairs). Two launch modes share the code:
//   - one launch per phase (`done` null): the kernel boundary orders the phases;
//   - one cooperative launch for all iterations (`done` non-null): before a tile reads a matrix's A, B or X, it waits
//     until every tile that writes it has completed, counted per matrix and phase in `done` (release adds after the
//     TMA stores complete, acquire loads before the reads). Every dependency points to an earlier tile of the
//     sequence, each pair walks its tiles in order and all CTAs are co-resident, so the earliest unfinished tile can
//     always proceed; the phases of different matrices overlap and there is one launch ramp and one tail in all.
//     Overwrites are safe by the same chain: a tile that rewrites A, B or X[s] waits (through its dependency) for the
//     tiles that read the previous contents.
//
// Per CTA pair (a cluster of two): the pair computes a 256 x 256 output tile with tcgen05.mma.cta_group::2 (M = 256,
// N = 256, K = 16). CTA r loads rows [128r, 128r+128) of the A operand and rows [128r, 128r+128) of the B operand
// into its own shared memory; the leader CTA (r = 0) issues the MMAs, which read both CTAs' tiles and accumulate
// output rows [128r, 128r+128) into CTA r's TMEM. A pipeline stage is 32 KB per CTA, so six stages fit beside the
// 32 KB epilogue. Roles per CTA: warp 0 lane 0 is the TMA producer, warp 1 lane 0 the MMA issuer (leader only) and
// TMEM owner, warps 2-9 the epilogue (two accumulators in TMEM: the MMA fills one while the epilogue drains the other).
//
// Synchronisation (every wait is bounded, as in ptx.cuh):
//   full[s]   leader only: the leader's producer arrives with the byte count of both CTAs' loads; both CTAs' TMA
//             loads (".cta_group::2" form) complete their bytes on it.
//   empty[s]  both CTAs: the leader's MMA commit arrives on it in both CTAs once the stage has been read.
//   tfull[a]  both CTAs: the leader's commit after the last k-block of a tile.
//   tempty[a] leader only: one arrival per epilogue warp of both CTAs (the peer's arrive remotely).
#pragma once

#include "mt_types.h"
#include "ns_types.h"
#include "ptx.cuh"

namespace moteopt {
namespace ns {

constexpr float kNsA = 3.4445f, kNsB = -4.7750f, kNsC = 2.0315f;   // mote/train/muon.py:31 (passed in Launch::ca/cb/cc)

// ---------------------------------------------------------------------------------------------------------------
struct Tile {
  int it, phase, src;   // iteration, phase, X buffer read by this iteration
  int gi, b;            // group, matrix within the group
  int i0, j0;           // output tile origin
};

__device__ __forceinline__ int tiles_per_matrix(const Launch& L, int gi, int phase) {
  const int T = L.tiles_m[gi];
  return phase == kUpdate ? T * L.tiles_n[gi] : T * (T + 1) / 2;
}

__device__ __forceinline__ Tile decode_tile(const Launch& L, int t) {
  Tile x;
  x.it = t / L.per_iter;
  int r = t - x.it * L.per_iter;
  int c = 0;
  while (c + 1 < L.n_chunks && r >= L.chunk_start[c + 1]) ++c;
  r -= L.chunk_start[c];
  x.phase = 0;
  while (x.phase < 2 && r >= L.ck_phase_tiles[c][x.phase]) {
    r -= L.ck_phase_tiles[c][x.phase];
    ++x.phase;
  }
  x.src = (L.src0 + x.it) & 1;
  const int* ts = L.ck_tile_start[c][x.phase];
  int gi = 0;
  while (gi + 1 < L.n_groups && r >= ts[gi + 1]) ++gi;
  r -= ts[gi];
  const int T = L.tiles_m[gi];
  int ti, tj;
  if (x.phase == kUpdate) {
    const int per = T * L.tiles_n[gi];
    x.b = r / per;
    r -= x.b * per;
    if (L.g[gi].tall) {   // n x m output: row blocks over the tall side
      ti = r / T;
      tj = r - ti * T;
    } else {
      ti = r / L.tiles_n[gi];
      tj = r - ti * L.tiles_n[gi];
    }
  } else {   // upper-triangle blocks, row-major
    const int per = T * (T + 1) / 2;
    x.b = r / per;
    r -= x.b * per;
    ti = 0;
    while (r >= T - ti) {
      r -= T - ti;
      ++ti;
    }
    tj = ti + r;
  }
  x.b += L.ck_b0[c][gi];
  x.gi = gi;
  x.i0 = ti * TM;
  x.j0 = tj * TN;
  return x;
}

__device__ __forceinline__ int phase_k(int phase, const Group& G) { return phase == kGram ? G.n : G.m; }

// Whether k-block kb of tile x reads its A operand (rows i) and its B operand (rows j, or X for kUpdate) MN-major.
// In kPoly (A A) and kUpdate (B X) the left factor is stored only at and above the diagonal: columns k in a block
// left of row block i come from the mirror block (k, i) as a transposed box. kPoly's right factor is A again (rows
// j); kUpdate's is X, always MN-major. A tall group (X stored n x m): the Gram phase X^T X reads columns i and j of
// X, both MN-major; the update X B reads rows i of X K-major and B's rows j like kPoly's right factor.
__device__ __forceinline__ void operand_mn(const Tile& x, int kb, bool tall, bool& a_mn, bool& b_mn) {
  const int kt = (kb * BK) / TM;
  if (tall && x.phase != kPoly) {
    a_mn = x.phase == kGram;
    b_mn = x.phase == kGram || kt < x.j0 / TN;
    return;
  }
  a_mn = x.phase != kGram && kt < x.i0 / TM;
  b_mn = x.phase == kUpdate || (x.phase == kPoly && kt < x.j0 / TN);
}

// Rows and columns of tile x's output matrix (an n x m update of a tall group, else m x n or m x m).
__device__ __forceinline__ int out_rows(const Tile& x, const Group& G) {
  return (x.phase == kUpdate && G.tall) ? G.n : G.m;
}
__device__ __forceinline__ int out_cols(const Tile& x, const Group& G) {
  return x.phase == kUpdate ? (G.tall ? G.m : G.n) : G.m;
}

// A diagonal block of the symmetric products (kGram X X^T, kPoly A A): its two operands are the same rows, read the
// same way in every k-block (operand_mn gives a_mn == b_mn, from the same tensor maps), and the pair splits them the
// same way (CTA r holds rows 128r..128r+127 of both). They are loaded once and the MMA reads the A stage as B too,
// which saves the block's second operand stream (a quarter to a third of the Gram and polynomial operand bytes).
__device__ __forceinline__ bool on_diagonal(const Tile& x) { return x.phase != kUpdate && x.i0 == x.j0; }

// Persistent mode: the completion counts tile x must see before reading. kGram reads X[src] (written by the previous
// iteration's kUpdate), kPoly reads A (this iteration's kGram), kUpdate reads B (kPoly) and X[src]. kUpdate checks
// only kPoly: this iteration's kPoly tiles of the matrix started after its kGram tiles completed, and those after the
// previous kUpdate completed, so a complete kPoly count already orders X[src] (and the end of every read of X[src^1],
// which kUpdate overwrites) before the tile, through the same release/acquire chain that orders the overwrites.
__device__ __forceinline__ bool wait_inputs(const Launch& L, const Tile& x, const WaitCtx& ctx) {
  const int mat = L.g[x.gi].first + x.b;
  const int* done = L.done + mat * 3;
  if (x.phase != kGram)
    return wait_counter(done + x.phase - 1, (x.it + 1) * tiles_per_matrix(L, x.gi, x.phase - 1) * kArrivalsPerTile,
                        ctx);
  return x.it == 0 || wait_counter(done + kUpdate, x.it * tiles_per_matrix(L, x.gi, kUpdate) * kArrivalsPerTile, ctx);
}

// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void producer(const Launch& L, uint32_t rank, uint8_t* sa, uint8_t* sb, uint64_t* full,
                                         uint64_t* empty, const WaitCtx& ctx) {
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  int stage = 0;
  uint32_t phase = 0;
  long issued = 0;
  bool ok = true;
  for (int t = L.t_begin + pair; t < L.t_end && ok; t += npairs) {
    const Tile x = decode_tile(L, t);
    const Group& G = L.g[x.gi];
    if (L.done != nullptr) {
      if (!wait_inputs(L, x, ctx)) break;
      fence_proxy_async_global();   // the TMA loads below observe the data the counters released
    }
    const int nk = (phase_k(x.phase, G) + BK - 1) / BK;
    MO_CHECK(x.gi >= 0 && x.gi < L.n_groups && x.b >= 0 && x.b < G.count && x.i0 < out_rows(x, G) &&
             x.j0 < out_cols(x, G) && (x.phase == kUpdate || x.i0 <= x.j0) && nk > 0);
    const bool tall = G.tall != 0;
    const CUtensorMap* amap = x.phase == kGram ? &G.xk[x.src] : (x.phase == kPoly ? &G.ak : (tall ? &G.xk[x.src] : &G.bk));
    const CUtensorMap* amap_mn = x.phase == kPoly ? &G.amn : (x.phase == kGram ? &G.xmn[x.src] : &G.bmn);
    const CUtensorMap* bmap = x.phase == kGram ? &G.xk[x.src] : (x.phase == kPoly ? &G.ak : &G.bk);
    const CUtensorMap* bmap_mn = x.phase == kPoly ? &G.amn : (tall && x.phase == kUpdate ? &G.bmn : &G.xmn[x.src]);
    const int ia = x.i0 + HM * static_cast<int>(rank), jb = x.j0 + (TN / 2) * static_cast<int>(rank);
    const bool diag = on_diagonal(x);   // B = A: the stage holds one operand, which the MMA reads as both
    for (int kb = 0; kb < nk; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, ctx)) { ok = false; break; }
      const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
      if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (diag ? A_BYTES : STAGE_BYTES));
      const int k0 = kb * BK;
      bool a_mn, b_mn;
      operand_mn(x, kb, tall, a_mn, b_mn);
      uint8_t* dsta = sa + stage * A_BYTES;
      if (a_mn) {   // rows ia..ia+127 of a block left of the diagonal = columns of the stored mirror block
        tma_load_3d_pair(dsta, amap_mn, bar, ia, k0, x.b);
        tma_load_3d_pair(dsta + BK * 64 * 2, amap_mn, bar, ia + 64, k0, x.b);
      } else {
        tma_load_3d_pair(dsta, amap, bar, k0, ia, x.b);
      }
      uint8_t* dstb = sb + stage * B_BYTES;
      if (!diag) {
        if (b_mn) {   // [k0:k0+64, jb:jb+128] as two 64 x 64 boxes, 128-byte swizzled along j
          tma_load_3d_pair(dstb, bmap_mn, bar, jb, k0, x.b);
          tma_load_3d_pair(dstb + BK * 64 * 2, bmap_mn, bar, jb + 64, k0, x.b);
        } else {
          tma_load_3d_pair(dstb, bmap, bar, k0, jb, x.b);
        }
      }
      ++issued;
      if (++stage == STAGES) { stage = 0; phase ^= 1u; }
    }
  }
  // When unwinding after a timeout, loads already issued complete on the leader's barrier; the cluster-wide barrier at
  // the end of the kernel keeps both CTAs (and their shared memory) alive until every role has returned, and the
  // leader's own drain below waits for its loads.
  if (!ok && rank == 0) {
    for (int s = 0; s < STAGES; ++s) {
      if (issued <= s) break;
      mbar_wait_drain(&full[s], (s < stage) ? phase : (phase ^ 1u));
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma(const Launch& L, uint8_t* sa, uint8_t* sb, uint64_t* full, uint64_t* empty,
                                    uint64_t* tfull, uint64_t* tempty, uint64_t* drain, uint32_t tmem_base,
                                    const WaitCtx& ctx) {
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  int stage = 0;
  uint32_t phase = 0;
  int local = 0;
  bool ok = true;
  for (int t = L.t_begin + pair; t < L.t_end && ok; t += npairs, ++local) {
    const Tile x = decode_tile(L, t);
    const Group& G = L.g[x.gi];
    const int nk = (phase_k(x.phase, G) + BK - 1) / BK;
    const int acc = local & 1;
    const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
    if (!mbar_wait(&tempty[acc], use ^ 1u, ctx)) break;
    tc_fence_after();
    const uint32_t d = tmem_base + static_cast<uint32_t>(acc * TN);
    for (int kb = 0; kb < nk; ++kb) {
      if (!mbar_wait(&full[stage], phase, ctx)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a0 = smem_u32(sa + stage * A_BYTES);
      const uint32_t b0 = on_diagonal(x) ? a0 : smem_u32(sb + stage * B_BYTES);
      bool a_mn, b_mn;
      operand_mn(x, kb, G.tall != 0, a_mn, b_mn);
      const uint32_t idesc = idesc_bf16_f32(TM, TN, a_mn, b_mn);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t adesc = a_mn ? sdesc_sw128(a0 + kk * 16 * 128, BK * 64 * 2, 1024) : sdesc_sw128(a0 + kk * 32, 16, 1024);
        const uint64_t bdesc = b_mn ? sdesc_sw128(b0 + kk * 16 * 128, BK * 64 * 2, 1024) : sdesc_sw128(b0 + kk * 32, 16, 1024);
        umma_bf16_pair(d, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
      }
      umma_commit_pair_both(&empty[stage]);   // both CTAs may refill the stage once these MMAs have read it
      if (++stage == STAGES) { stage = 0; phase ^= 1u; }
    }
    if (ok) umma_commit_pair_both(&tfull[acc]);
  }
  umma_commit_pair_local(drain);
  mbar_wait_drain(drain, 0);
}

// ---------------------------------------------------------------------------------------------------------------
// Round a pair to bf16 and back (one cvt.rn.bf16x2.f32 for two values).
__device__ __forceinline__ void round2(float& a, float& b) {
  const uint32_t p = pack_bf16x2(a, b);
  a = bf16_lo(p);
  b = bf16_hi(p);
}

// Byte offset of 16-byte chunk c (0..3) of row r (0..31) in a 32 x 32 bf16 subtile with the 64-byte TMA swizzle
// (chunk bits [4,5] ^= row bits [7,8] of the address). Row-per-thread accesses are bank-conflict free.
__device__ __forceinline__ uint32_t sw64(int r, int c) {
  return static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// The epilogue on this CTA's 128 rows of the pair tile. Warp (q, half) owns rows row0 = i0 + 128 rank + 32 q and the
// 128 output columns of its half, in four 32 x 32 chunks; lane l owns row row0 + l. Per warp, two 2 KB subtiles
// (64-byte swizzle): the phase's bf16 operand (A for kPoly, X for kUpdate) arrives in one by TMA, each thread combines
// its row with the accumulator's TMEM columns and writes the result in place, one lane TMA-stores it and, once the
// store has read it, refills it with the operand of the chunk two ahead. The accumulator release goes to the leader
// CTA; in persistent mode each warp then waits for its stores to complete and counts the tile done for its matrix and
// phase.
template <bool kRoundOnce>
__device__ __forceinline__ void epilogue(const Launch& L, uint32_t rank, uint64_t* tfull, uint64_t* tempty,
                                         uint8_t* ebuf, uint64_t* ebar, uint32_t tmem_base, const WaitCtx& ctx) {
  constexpr int kChunks = TN / EPI_TILE / 2;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ew = static_cast<int>(warp_id()) - 2;
  const int q = static_cast<int>(warp_id() & 3u);
  const int half = ew >> 2;
  const int lane = static_cast<int>(lane_id());
  uint8_t* buf[2] = {ebuf + (ew * 2) * EPI_BUF_BYTES, ebuf + (ew * 2 + 1) * EPI_BUF_BYTES};
  uint64_t* bar[2] = {&ebar[ew * 2], &ebar[ew * 2 + 1]};
  uint32_t bphase[2] = {0u, 0u};
  bool ok = true;
  int local = 0;
  for (int t = L.t_begin + pair; t < L.t_end && ok; t += npairs, ++local) {
    const Tile x = decode_tile(L, t);
    const Group& G = L.g[x.gi];
    const bool has_aux = x.phase != kGram && !(x.phase == kUpdate && L.no_aux);
    const int acc = local & 1;
    const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
    const int ocols = out_cols(x, G);
    const int row0 = x.i0 + HM * static_cast<int>(rank) + q * 32;
    const bool rows_ok = row0 < out_rows(x, G);
    const int jc0 = x.j0 + half * (kChunks * EPI_TILE);
    const CUtensorMap* omap = x.phase == kGram ? &G.ae : (x.phase == kPoly ? &G.be : &G.xe[x.src ^ 1]);
    const CUtensorMap* amap = x.phase == kPoly ? &G.ae : &G.xe[x.src];
    int nch = 0;
    while (nch < kChunks && jc0 + nch * EPI_TILE < ocols) ++nch;
    const bool work = rows_ok && nch > 0;
    int loaded = 1;
    if (lane == 0 && work) {
      bulk_wait_read<0>();   // the previous tile's stores have left both subtiles
      if (has_aux) {
        if (L.done != nullptr) {   // acquire the operand's producers (complete: the MMA operands waited for them)
          loaded = wait_inputs(L, x, ctx) ? 1 : 0;
          fence_proxy_async_global();
        }
        for (int c = 0; c < 2 && c < nch && loaded; ++c) {
          mbar_arrive_expect_tx(bar[c], EPI_BUF_BYTES);
          tma_load_3d(buf[c], amap, bar[c], jc0 + c * EPI_TILE, row0, x.b);
        }
      }
    }
    if (!__shfl_sync(0xffffffffu, loaded, 0)) break;
    if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], use, ctx) ? 1 : 0)) break;
    tc_fence_after();
    for (int c = 0; c < nch; ++c) {
      const int bi = c & 1;
      uint32_t r[32];
      MO_CHECK(acc * TN + half * (kChunks * EPI_TILE) + (c + 1) * EPI_TILE <= static_cast<int>(kTmemCols));
      tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                    static_cast<uint32_t>(acc * TN + half * (kChunks * EPI_TILE) + c * EPI_TILE), r);
      tmem_ld_wait(r);
      if (!rows_ok) continue;
      uint8_t* row = buf[bi];
      if (has_aux) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar[bi], bphase[bi], ctx) ? 1 : 0)) { ok = false; break; }
        bphase[bi] ^= 1u;
      } else if (c >= 2) {
        if (lane == 0) bulk_wait_read<1>();   // the store of chunk c-2 has left this subtile
        __syncwarp();
      }
      uint32_t out[16];
      if (!has_aux) {   // kGram, or the Gram variant's plain product: bf16 of the accumulator
#pragma unroll
        for (int k = 0; k < 16; ++k) out[k] = pack_bf16x2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
      } else {
        uint32_t in[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const uint4 w = *reinterpret_cast<const uint4*>(row + sw64(lane, cc));
          in[4 * cc] = w.x; in[4 * cc + 1] = w.y; in[4 * cc + 2] = w.z; in[4 * cc + 3] = w.w;
        }
        if (kRoundOnce) {   // the Gram variant: out = bf16(coef * aux + acc'), the fp32 terms as the oracle forms them
          const float ka = x.phase == kPoly ? L.cb : L.ca;
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float p0 = __uint_as_float(r[2 * k]), p1 = __uint_as_float(r[2 * k + 1]);
            if (x.phase == kPoly) { p0 = __fmul_rn(L.cc, p0); p1 = __fmul_rn(L.cc, p1); }            // c * (R @ R)
            out[k] = pack_bf16x2(__fadd_rn(__fmul_rn(ka, bf16_lo(in[k])), p0), __fadd_rn(__fmul_rn(ka, bf16_hi(in[k])), p1));
          }
        } else if (x.phase == kPoly) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float aa0 = __uint_as_float(r[2 * k]), aa1 = __uint_as_float(r[2 * k + 1]);
            round2(aa0, aa1);                                                                   // A @ A
            float t10 = __fmul_rn(L.cb, bf16_lo(in[k])), t11 = __fmul_rn(L.cb, bf16_hi(in[k]));
            round2(t10, t11);                                                                   // b * A
            float t20 = __fmul_rn(L.cc, aa0), t21 = __fmul_rn(L.cc, aa1);
            round2(t20, t21);                                                                   // c * (A @ A)
            out[k] = pack_bf16x2(__fadd_rn(t10, t20), __fadd_rn(t11, t21));
          }
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float bx0 = __uint_as_float(r[2 * k]), bx1 = __uint_as_float(r[2 * k + 1]);
            round2(bx0, bx1);                                                                   // B @ X
            float ax0 = __fmul_rn(L.ca, bf16_lo(in[k])), ax1 = __fmul_rn(L.ca, bf16_hi(in[k]));
            round2(ax0, ax1);                                                                   // a * X
            out[k] = pack_bf16x2(__fadd_rn(ax0, bx0), __fadd_rn(ax1, bx1));
          }
        }
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        *reinterpret_cast<uint4*>(row + sw64(lane, cc)) = make_uint4(out[4 * cc], out[4 * cc + 1], out[4 * cc + 2], out[4 * cc + 3]);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_3d(omap, row, jc0 + c * EPI_TILE, row0, x.b);
        bulk_commit();
        if (has_aux && c + 2 < nch) {   // refill this subtile with the operand of chunk c+2
          bulk_wait_read<0>();
          mbar_arrive_expect_tx(bar[bi], EPI_BUF_BYTES);
          tma_load_3d(row, amap, bar[bi], jc0 + (c + 2) * EPI_TILE, row0, x.b);
        }
      }
      __syncwarp();
    }
    if (!ok) break;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      if (rank == 0) mbar_arrive(&tempty[acc]);   // release the accumulator to the leader's MMA: one arrival per warp
      else mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
      if (L.done != nullptr) {   // this warp's part of the tile is in global memory
        bulk_wait<0>();
        fence_proxy_async_global();
        red_release_gpu_add(L.done + (G.first + x.b) * 3 + x.phase, 1);
      }
    }
    __syncwarp();
  }
  if (lane == 0) {
    bulk_wait<0>();
    if (!ok) {
      for (int k = 0; k < 2; ++k) mbar_wait_drain(bar[k], bphase[k]);
    }
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------------------------------------------
// kRoundOnce: the Gram variant's epilogue (Launch::round_once); the reference iteration's instantiation is false.
template <bool kRoundOnce>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) ns_gemm_kernel(const __grid_constant__ Launch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;
  uint8_t* ebuf = smem + STAGES * STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ebuf + EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* ebar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t rank = cluster_ctarank();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int e = 0; e < 2 * kEpiWarps; ++e) mbar_init(&ebar[e], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane_id() < static_cast<uint32_t>(L.n_groups)) {
    const Group& G = L.g[lane_id()];
    const CUtensorMap* maps[] = {&G.xk[0], &G.xk[1], &G.xmn[0], &G.xmn[1], &G.ak, &G.bk, &G.amn, &G.bmn,
                                 &G.xe[0], &G.xe[1], &G.ae, &G.be};
#pragma unroll
    for (int k = 0; k < 12; ++k) tma_prefetch_desc(maps[k]);
  }
  __syncthreads();
  cluster_sync();   // the pair's barriers exist before either CTA signals the other's
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx ctx{abort_flag, L.status, kWaitLimitNs};
  if (warp == 0) {
    if (lane_id() == 0) producer(L, rank, sa, sb, full, empty, ctx);
    __syncwarp();
  } else if (warp == 1) {
    if (lane_id() == 0 && rank == 0) mma(L, sa, sb, full, empty, tfull, tempty, drain, tmem_base, ctx);
    __syncwarp();
  } else {
    epilogue<kRoundOnce>(L, rank, tfull, tempty, ebuf, ebar, tmem_base, ctx);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // no CTA leaves while its pair still reads its shared memory or signals its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(L.status, kStatusAborted);
}

// ---------------------------------------------------------------------------------------------------------------
// Gram Newton-Schulz helpers (the opt-in variant of docs/research/efficiency-campaign-2026-08-23.md:903-911 in the
// reference project; not the reference's iteration). Both work on bf16 [count][m][m] matrices (m padded to a multiple
// of 8, `mv` valid rows/columns), in 32 x 32 tiles through shared memory, one tile per block: grid (tiles, count).
struct SymArgs {
  __nv_bfloat16* src;   // read (its tiles on and above the 256 x 256 block diagonal)
  __nv_bfloat16* dst;   // written
  int m, mv;
  float a;              // ns_gram_q1_kernel: the coefficient a of a*I
};

// In place (src == dst): every element below the main diagonal gets its mirror above it, R[r][c] = R[c][r] for r > c,
// so R is exactly symmetric. The polynomial phase reads R as its right operand row-wise (R R^T) and shares the
// left operand on diagonal tiles, which is R R only for an exactly symmetric R; the Gram phase's R = X X^T is (its
// upper blocks are written, the rest comes from here), an update's R = a T + B T is not until this runs.
__global__ void __launch_bounds__(256) ns_symmetrize_kernel(const __grid_constant__ SymArgs A) {
  __shared__ __nv_bfloat16 t[32][33];
  const int tiles = (A.m + 31) / 32;
  const int ti = blockIdx.x / tiles, tj = blockIdx.x % tiles;   // destination tile (rows ti, columns tj)
  if (ti < tj) return;                                          // above the diagonal: kept
  const size_t base = static_cast<size_t>(blockIdx.y) * A.m * A.m;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int k = ty; k < 32; k += 8) {   // source tile (rows tj, columns ti), row k
    const int r = tj * 32 + k, c = ti * 32 + tx;
    t[k][tx] = (r < A.m && c < A.m) ? A.src[base + static_cast<size_t>(r) * A.m + c] : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int r = ti * 32 + k, c = tj * 32 + tx;
    if (r < A.m && c < A.m && r > c) A.dst[base + static_cast<size_t>(r) * A.m + c] = t[tx][k];
  }
}

// Q1 = bf16(a*I + B~) for the variant's first iteration (its Q0 = I, so a*Q0 + B Q0 needs no product): B~ is B read
// through its upper blocks (a tile below the block diagonal is the transpose of its mirror); the identity covers the
// valid rows only, so the zero padding stays zero.
__global__ void __launch_bounds__(256) ns_gram_q1_kernel(const __grid_constant__ SymArgs A) {
  __shared__ __nv_bfloat16 t[32][33];
  const int tiles = (A.m + 31) / 32;
  const int ti = blockIdx.x / tiles, tj = blockIdx.x % tiles;
  const bool mirror = (ti * 32) / TM > (tj * 32) / TN;
  const size_t base = static_cast<size_t>(blockIdx.y) * A.m * A.m;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int k = ty; k < 32; k += 8) {
    const int r = (mirror ? tj : ti) * 32 + k, c = (mirror ? ti : tj) * 32 + tx;
    t[k][tx] = (r < A.m && c < A.m) ? A.src[base + static_cast<size_t>(r) * A.m + c] : __float2bfloat16_rn(0.f);
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int r = ti * 32 + k, c = tj * 32 + tx;
    if (r >= A.m || c >= A.m) continue;
    const float b = __bfloat162float(mirror ? t[tx][k] : t[k][tx]);
    const float d = (r == c && r < A.mv) ? A.a : 0.f;
    A.dst[base + static_cast<size_t>(r) * A.m + c] = __float2bfloat16_rn(__fadd_rn(d, b));
  }
}

}  // namespace ns
}  // namespace moteopt
