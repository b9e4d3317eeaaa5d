// Newton-Schulz phase kernel, 2-CTA form: each cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16). CTA r of the pair loads rows [128r, 128r+128) of the A operand and
// rows [128r, 128r+128) of the B operand (its half of N) into its own shared memory; the leader CTA (r = 0) issues the
// MMAs, which read both CTAs' tiles and accumulate rows [128r, 128r+128) of the output into CTA r's TMEM. Per CTA a
// pipeline stage is 32 KB instead of the 48 KB of a 128 x 256 single-CTA tile, so six stages (a 2560-cycle lead over
// the MMA) fit beside the 32 KB epilogue, and each SM pulls a third less operand traffic from L2 for the same tensor
// work.
//
// Synchronisation (all mbarrier waits bounded, as in ptx.cuh):
//   full[s]   leader only: the leader's producer arrives with the byte count of both CTAs' loads; both CTAs' TMA
//             loads (".cta_group::2" form) complete their bytes on it.
//   empty[s]  both CTAs: the leader's MMA commit arrives on it in both CTAs once the stage has been read.
//   tfull[a]  both CTAs: the leader's commit after the last k-block of a tile.
//   tempty[a] leader only: one arrival per epilogue warp of both CTAs (the peer's arrive remotely).
// The epilogue works on this CTA's 128 rows (see epilogue2).
#pragma once

#include "ns_gemm.cuh"

namespace moteopt {
namespace ns2 {

using namespace ns;

constexpr int TM = 256, TN = 256;   // output tile of a CTA pair
constexpr int HM = 128;             // rows (and B rows) per CTA
constexpr int STAGES2 = 6;
constexpr int A2_BYTES = HM * BK * 2;          // 16 KB
constexpr int B2_BYTES = (TN / 2) * BK * 2;    // 16 KB
constexpr int STAGE2_BYTES = A2_BYTES + B2_BYTES;
constexpr int EPI2_BYTES = kEpiWarps * 2 * EPI_BUF_BYTES;   // per warp: two subtiles, operand in and result out
constexpr int kSmem2Bytes = STAGES2 * STAGE2_BYTES + EPI2_BYTES + 1024 + 512;

// Tile t of a launch -> (group, matrix, row block, column block). A = X X^T and B = bA + cA^2 are symmetric, so the
// Gram and polynomial phases compute only the blocks on and above the diagonal (tiles_m (tiles_m + 1) / 2 per
// matrix, row-major over the upper triangle); a block below it is read as the transpose of its mirror (see
// operand_mn).
__device__ __forceinline__ void decode_tile2(const Launch& L, int t, int& gi, int& b, int& i0, int& j0) {
  gi = 0;
  while (gi + 1 < L.n_groups && t >= L.tile_start[gi + 1]) ++gi;
  const int local = t - L.tile_start[gi];
  const int T = L.tiles_m[gi];
  int ti, tj;
  if (L.phase == kUpdate) {
    const int per = T * L.tiles_n[gi];
    b = local / per;
    const int r = local - b * per;
    ti = r / L.tiles_n[gi];
    tj = r - ti * L.tiles_n[gi];
  } else {
    const int per = T * (T + 1) / 2;
    b = local / per;
    int r = local - b * per;
    ti = 0;
    while (r >= T - ti) { r -= T - ti; ++ti; }
    tj = ti + r;
  }
  i0 = ti * TM;
  j0 = tj * TN;
}

// Whether k-block kb of tile (i0, j0) reads its A operand (rows i) and its B operand (rows j, or X for kUpdate) in
// MN-major form. In kPoly (A A) and kUpdate (B X) the row block i of the symmetric left factor is stored only at and
// above the diagonal: columns k in a block left of i are read from the mirror block (k, i) as a transposed box.
// kPoly's right factor is A again (rows j); kUpdate's is X, always MN-major.
__device__ __forceinline__ void operand_mn(const Launch& L, int i0, int j0, int kb, bool& a_mn, bool& b_mn) {
  const int kt = (kb * BK) / TM;
  a_mn = L.phase != kGram && kt < i0 / TM;
  b_mn = L.phase == kUpdate || (L.phase == kPoly && kt < j0 / TN);
}

// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void producer2(const Launch& L, uint32_t rank, uint8_t* sa, uint8_t* sb, uint64_t* full,
                                          uint64_t* empty, const WaitCtx& ctx) {
  const int total = L.tile_start[L.n_groups];
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  int stage = 0;
  uint32_t phase = 0;
  long issued = 0;
  bool ok = true;
  for (int t = pair; t < total && ok; t += npairs) {
    int gi, b, i0, j0;
    decode_tile2(L, t, gi, b, i0, j0);
    const Group& G = L.g[gi];
    const int nk = (phase_k(L, G) + BK - 1) / BK;
    const CUtensorMap* amap = L.phase == kGram ? &G.xk[L.src] : (L.phase == kPoly ? &G.ak : &G.bk);
    const CUtensorMap* amap_mn = L.phase == kPoly ? &G.amn : &G.bmn;
    const CUtensorMap* bmap = L.phase == kGram ? &G.xk[L.src] : (L.phase == kPoly ? &G.ak : &G.xmn[L.src]);
    const CUtensorMap* bmap_mn = L.phase == kPoly ? &G.amn : &G.xmn[L.src];
    const int ia = i0 + HM * static_cast<int>(rank), jb = j0 + (TN / 2) * static_cast<int>(rank);
    for (int kb = 0; kb < nk; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, ctx)) { ok = false; break; }
      const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
      if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * STAGE2_BYTES);
      const int k0 = kb * BK;
      bool a_mn, b_mn;
      operand_mn(L, i0, j0, kb, a_mn, b_mn);
      uint8_t* dsta = sa + stage * A2_BYTES;
      if (a_mn) {   // rows ia..ia+127 of the block left of the diagonal = columns of the stored mirror block
        tma_load_3d_pair(dsta, amap_mn, bar, ia, k0, b);
        tma_load_3d_pair(dsta + BK * 64 * 2, amap_mn, bar, ia + 64, k0, b);
      } else {
        tma_load_3d_pair(dsta, amap, bar, k0, ia, b);
      }
      uint8_t* dst = sb + stage * B2_BYTES;
      if (b_mn) {   // [k0:k0+64, jb:jb+128] as two 64 x 64 boxes, 128-byte swizzled along j
        tma_load_3d_pair(dst, bmap_mn, bar, jb, k0, b);
        tma_load_3d_pair(dst + BK * 64 * 2, bmap_mn, bar, jb + 64, k0, b);
      } else {
        tma_load_3d_pair(dst, bmap, bar, k0, jb, b);
      }
      ++issued;
      if (++stage == STAGES2) { stage = 0; phase ^= 1u; }
    }
  }
  (void)issued;
  // When unwinding after a timeout, loads already issued complete on the leader's barrier; the cluster-wide barrier at
  // the end of the kernel keeps both CTAs (and their shared memory) alive until every role has returned, and the
  // leader's own drain below waits for its loads.
  if (!ok && rank == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      if (issued <= s) break;
      mbar_wait_drain(&full[s], (s < stage) ? phase : (phase ^ 1u));
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mma2(const Launch& L, uint8_t* sa, uint8_t* sb, uint64_t* full, uint64_t* empty,
                                     uint64_t* tfull, uint64_t* tempty, uint64_t* drain, uint32_t tmem_base,
                                     const WaitCtx& ctx) {
  const int total = L.tile_start[L.n_groups];
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  int stage = 0;
  uint32_t phase = 0;
  int local = 0;
  bool ok = true;
  for (int t = pair; t < total && ok; t += npairs, ++local) {
    int gi, b, i0, j0;
    decode_tile2(L, t, gi, b, i0, j0);
    const Group& G = L.g[gi];
    const int nk = (phase_k(L, G) + BK - 1) / BK;
    const int acc = local & 1;
    const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
    if (!mbar_wait(&tempty[acc], use ^ 1u, ctx)) break;
    tc_fence_after();
    const uint32_t d = tmem_base + static_cast<uint32_t>(acc * TN);
    for (int kb = 0; kb < nk; ++kb) {
      if (!mbar_wait(&full[stage], phase, ctx)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a0 = smem_u32(sa + stage * A2_BYTES);
      const uint32_t b0 = smem_u32(sb + stage * B2_BYTES);
      bool a_mn, b_mn;
      operand_mn(L, i0, j0, kb, a_mn, b_mn);
      const uint32_t idesc = idesc_bf16_f32(TM, TN, a_mn, b_mn);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t adesc = a_mn ? sdesc_sw128(a0 + kk * 16 * 128, BK * 64 * 2, 1024) : sdesc_sw128(a0 + kk * 32, 16, 1024);
        const uint64_t bdesc = b_mn ? sdesc_sw128(b0 + kk * 16 * 128, BK * 64 * 2, 1024) : sdesc_sw128(b0 + kk * 32, 16, 1024);
        umma_bf16_pair(d, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
      }
      umma_commit_pair_both(&empty[stage]);   // both CTAs may refill the stage once these MMAs have read it
      if (++stage == STAGES2) { stage = 0; phase ^= 1u; }
    }
    if (ok) umma_commit_pair_both(&tfull[acc]);
  }
  umma_commit_pair_local(drain);
  mbar_wait_drain(drain, 0);
}

// ---------------------------------------------------------------------------------------------------------------
// The epilogue on this CTA's 128 rows of the pair tile. Per warp, two 2 KB subtiles: the phase's bf16 operand (A
// for kPoly, X for kUpdate) arrives in one by TMA, each thread combines its row with the accumulator and writes the
// result in place, one lane TMA-stores it and, once the store has read it, refills it with the chunk two ahead. The
// accumulator release goes to the leader CTA.
__device__ __forceinline__ void epilogue2(const Launch& L, uint32_t rank, uint64_t* tfull, uint64_t* tempty,
                                          uint8_t* ebuf, uint64_t* ebar, uint32_t tmem_base, const WaitCtx& ctx) {
  constexpr int kChunks = BN / EPI_TILE / 2;
  const int total = L.tile_start[L.n_groups];
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ew = static_cast<int>(warp_id()) - 2;
  const int q = static_cast<int>(warp_id() & 3u);
  const int half = ew >> 2;
  const int lane = static_cast<int>(lane_id());
  uint8_t* buf[2] = {ebuf + (ew * 2) * EPI_BUF_BYTES, ebuf + (ew * 2 + 1) * EPI_BUF_BYTES};
  uint64_t* bar[2] = {&ebar[ew * 2], &ebar[ew * 2 + 1]};
  uint32_t bphase[2] = {0u, 0u};
  const bool has_aux = L.phase != kGram;
  bool ok = true;
  int local = 0;
  for (int t = pair; t < total && ok; t += npairs, ++local) {
    int gi, b, i0, j0;
    decode_tile2(L, t, gi, b, i0, j0);
    const Group& G = L.g[gi];
    const int acc = local & 1;
    const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
    const int out_cols = L.phase == kUpdate ? G.n : G.m;
    const int row0 = i0 + HM * static_cast<int>(rank) + q * 32;
    const bool rows_ok = row0 < G.m;
    const int jc0 = j0 + half * (kChunks * EPI_TILE);
    const CUtensorMap* omap = L.phase == kGram ? &G.ae : (L.phase == kPoly ? &G.be : &G.xe[L.src ^ 1]);
    const CUtensorMap* amap = L.phase == kPoly ? &G.ae : &G.xe[L.src];
    int nch = 0;
    while (nch < kChunks && jc0 + nch * EPI_TILE < out_cols) ++nch;
    const bool work = rows_ok && nch > 0;
    if (lane == 0 && work) {
      bulk_wait_read<0>();   // the previous tile's stores have left both subtiles
      if (has_aux) {
        for (int c = 0; c < 2 && c < nch; ++c) {
          mbar_arrive_expect_tx(bar[c], EPI_BUF_BYTES);
          tma_load_3d(buf[c], amap, bar[c], jc0 + c * EPI_TILE, row0, b);
        }
      }
    }
    __syncwarp();
    if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], use, ctx) ? 1 : 0)) break;
    tc_fence_after();
    for (int c = 0; c < nch; ++c) {
      const int bi = c & 1;
      uint32_t r[32];
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
      if (L.phase == kGram) {
#pragma unroll
        for (int k = 0; k < 16; ++k) out[k] = pack_bf16x2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
      } else {
        uint32_t in[16];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const uint4 w = *reinterpret_cast<const uint4*>(row + sw64(lane, cc));
          in[4 * cc] = w.x; in[4 * cc + 1] = w.y; in[4 * cc + 2] = w.z; in[4 * cc + 3] = w.w;
        }
        if (L.phase == kPoly) {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float aa0 = __uint_as_float(r[2 * k]), aa1 = __uint_as_float(r[2 * k + 1]);
            round2(aa0, aa1);                                                                   // A @ A
            float t10 = __fmul_rn(kNsB, bf16_lo(in[k])), t11 = __fmul_rn(kNsB, bf16_hi(in[k]));
            round2(t10, t11);                                                                   // b * A
            float t20 = __fmul_rn(kNsC, aa0), t21 = __fmul_rn(kNsC, aa1);
            round2(t20, t21);                                                                   // c * (A @ A)
            out[k] = pack_bf16x2(__fadd_rn(t10, t20), __fadd_rn(t11, t21));
          }
        } else {
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float bx0 = __uint_as_float(r[2 * k]), bx1 = __uint_as_float(r[2 * k + 1]);
            round2(bx0, bx1);                                                                   // B @ X
            float ax0 = __fmul_rn(kNsA, bf16_lo(in[k])), ax1 = __fmul_rn(kNsA, bf16_hi(in[k]));
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
        tma_store_3d(omap, row, jc0 + c * EPI_TILE, row0, b);
        bulk_commit();
        if (has_aux && c + 2 < nch) {   // refill this subtile with the operand of chunk c+2
          bulk_wait_read<0>();
          mbar_arrive_expect_tx(bar[bi], EPI_BUF_BYTES);
          tma_load_3d(row, amap, bar[bi], jc0 + (c + 2) * EPI_TILE, row0, b);
        }
      }
      __syncwarp();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {   // release the accumulator to the leader's MMA: one arrival per warp
      if (rank == 0) mbar_arrive(&tempty[acc]);
      else mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
    }
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
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) ns_phase_kernel2(const __grid_constant__ Launch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES2 * A2_BYTES;
  uint8_t* ebuf = smem + STAGES2 * STAGE2_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ebuf + EPI2_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES2;
  uint64_t* tfull = bars + 2 * STAGES2;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* ebar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  const uint32_t rank = cluster_ctarank();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
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
  if (warp == 0 && lane_id() == 0) {
    for (int g = 0; g < L.n_groups; ++g) {
      const Group& G = L.g[g];
      if (L.phase == kGram) { tma_prefetch_desc(&G.xk[L.src]); tma_prefetch_desc(&G.ae); }
      if (L.phase == kPoly) { tma_prefetch_desc(&G.ak); tma_prefetch_desc(&G.amn); tma_prefetch_desc(&G.be); }
      if (L.phase == kUpdate) {
        tma_prefetch_desc(&G.bk); tma_prefetch_desc(&G.bmn); tma_prefetch_desc(&G.xmn[L.src]);
        tma_prefetch_desc(&G.xe[0]); tma_prefetch_desc(&G.xe[1]);
      }
    }
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
  const WaitCtx ctx{abort_flag, L.status};

  if (warp == 0) {
    if (lane_id() == 0) producer2(L, rank, sa, sb, full, empty, ctx);
    __syncwarp();
  } else if (warp == 1) {
    if (lane_id() == 0 && rank == 0) mma2(L, sa, sb, full, empty, tfull, tempty, drain, tmem_base, ctx);
    __syncwarp();
  } else {
    epilogue2(L, rank, tfull, tempty, ebuf, ebar, tmem_base, ctx);
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

}  // namespace ns2
}  // namespace moteopt
