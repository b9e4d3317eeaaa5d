// Newton-Schulz phase kernel for sm_100a (tcgen05 + TMEM + TMA).
//
// One launch runs one phase of one Newton-Schulz iteration (mote/train/muon.py:37-40) for every matrix of every
// shape group at once:
//   kGram:   A  = bf16(X X^T)
//   kPoly:   B  = bf16( bf16(b*A) + bf16(c * bf16(A A)) )          (A is symmetric, so A A = A A^T)
//   kUpdate: X' = bf16( bf16(a*X) + bf16(B X) )
// The rounding points are the reference's: every torch op on a bf16 tensor rounds its fp32 result to bf16.
//
// Structure: a persistent grid (one CTA per SM, 197 KB of shared memory) walks a static tile list. Warp 0 streams
// 128x64 A tiles and 256x64 B tiles with TMA into a 4-stage ring; one thread of warp 1 issues tcgen05.mma
// (M=128, N=256, K=16) into one of two TMEM accumulators; warps 2-5 drain the other accumulator (tcgen05.ld),
// apply the phase's polynomial in fp32 with bf16 rounding and store. The B operand of kUpdate (X, indexed [k][j])
// is consumed MN-major straight from the row-major iterate; every other operand is K-major.
#pragma once

#include "ns_types.h"
#include "ptx.cuh"

namespace moteopt {
namespace ns {

constexpr float kNsA = 3.4445f, kNsB = -4.7750f, kNsC = 2.0315f;   // mote/train/muon.py:31

__device__ __forceinline__ void decode_tile(const Launch& L, int t, int& gi, int& b, int& i0, int& j0) {
  gi = 0;
  while (gi + 1 < L.n_groups && t >= L.tile_start[gi + 1]) ++gi;
  const int local = t - L.tile_start[gi];
  const int per = L.tiles_m[gi] * L.tiles_n[gi];
  b = local / per;
  const int r = local - b * per;
  const int ti = r / L.tiles_n[gi];
  const int tj = r - ti * L.tiles_n[gi];
  i0 = ti * BM;
  j0 = tj * BN;
}

__device__ __forceinline__ int phase_k(const Launch& L, const Group& G) { return L.phase == kGram ? G.n : G.m; }

// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void run_producer(const Launch& L, uint8_t* sa, uint8_t* sb, uint64_t* full, uint64_t* empty,
                                             const WaitCtx& ctx) {
  const int total = L.tile_start[L.n_groups];
  int stage = 0;
  uint32_t phase = 0;
  long issued = 0;
  bool ok = true;
  for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
    int gi, b, i0, j0;
    decode_tile(L, t, gi, b, i0, j0);
    const Group& G = L.g[gi];
    const int nk = (phase_k(L, G) + BK - 1) / BK;
    const CUtensorMap* amap = L.phase == kGram ? &G.xk[L.src] : (L.phase == kPoly ? &G.ak : &G.bk);
    const CUtensorMap* bmap = L.phase == kGram ? &G.xk[L.src] : (L.phase == kPoly ? &G.ak : &G.xmn[L.src]);
    for (int kb = 0; kb < nk; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, ctx)) { ok = false; break; }
      mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
      const int k0 = kb * BK;
      tma_load_3d(sa + stage * A_BYTES, amap, &full[stage], k0, i0, b);
      uint8_t* dst = sb + stage * B_BYTES;
      if (L.phase == kUpdate) {
        // X[k0:k0+64, j0:j0+256] as four 64(k) x 64(j) boxes, each 128-byte swizzled along j
#pragma unroll
        for (int q = 0; q < 4; ++q) tma_load_3d(dst + q * (BK * 64 * 2), bmap, &full[stage], j0 + 64 * q, k0, b);
      } else {
        tma_load_3d(dst, bmap, &full[stage], k0, j0, b);
        tma_load_3d(dst + BM * BK * 2, bmap, &full[stage], k0, j0 + BM, b);
      }
      ++issued;
      if (++stage == STAGES) { stage = 0; phase ^= 1u; }
    }
  }
  if (!ok) {
    // unwinding: let the copies already issued land before the CTA's shared memory goes away
    for (int s = 0; s < STAGES; ++s) {
      if (issued <= s) break;
      const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
      mbar_wait_drain(&full[s], par);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void run_mma(const Launch& L, uint8_t* sa, uint8_t* sb, uint64_t* full, uint64_t* empty,
                                        uint64_t* tfull, uint64_t* tempty, uint64_t* drain, uint32_t tmem_base,
                                        const WaitCtx& ctx) {
  const int total = L.tile_start[L.n_groups];
  const bool mn_b = L.phase == kUpdate;
  const uint32_t idesc = idesc_bf16_f32(BM, BN, false, mn_b);
  int stage = 0;
  uint32_t phase = 0;
  int local = 0;
  bool ok = true;
  for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++local) {
    int gi, b, i0, j0;
    decode_tile(L, t, gi, b, i0, j0);
    const Group& G = L.g[gi];
    const int nk = (phase_k(L, G) + BK - 1) / BK;
    const int acc = local & 1;
    const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
    if (!mbar_wait(&tempty[acc], use ^ 1u, ctx)) break;
    tc_fence_after();
    const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
    for (int kb = 0; kb < nk; ++kb) {
      if (!mbar_wait(&full[stage], phase, ctx)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a0 = smem_u32(sa + stage * A_BYTES);
      const uint32_t b0 = smem_u32(sb + stage * B_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t adesc = sdesc_sw128(a0 + kk * 32, 16, 1024);
        const uint64_t bdesc = mn_b ? sdesc_sw128(b0 + kk * 16 * 128, BK * 64 * 2, 1024) : sdesc_sw128(b0 + kk * 32, 16, 1024);
        umma_bf16(d, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
      }
      umma_commit(&empty[stage]);   // frees the stage once these MMAs have read it
      if (++stage == STAGES) { stage = 0; phase ^= 1u; }
    }
    if (ok) umma_commit(&tfull[acc]);   // accumulator complete
  }
  // wait for every MMA this thread issued before TMEM is released
  umma_commit(drain);
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

// Epilogue warps 2..9: warp w reads TMEM lane quarter (w % 4), i.e. tile rows [32q, 32q+32), and owns columns
// [128h, 128h+128) with h = (w - 2) / 4, in four 32-column chunks. Each chunk goes through one of the warp's two
// 2 KB shared-memory subtiles: the phase's bf16 operand (A for kPoly, X for kUpdate) arrives there by TMA, each
// thread combines its row with the accumulator and writes the result back in place, and one lane TMA-stores the
// subtile. No per-thread global access remains, so the epilogue costs no L1 bandwidth.
__device__ __forceinline__ void run_epilogue(const Launch& L, uint64_t* tfull, uint64_t* tempty, uint8_t* ebuf,
                                             uint64_t* ebar, uint32_t tmem_base, const WaitCtx& ctx) {
  constexpr int kChunks = BN / EPI_TILE / 2;
  const int total = L.tile_start[L.n_groups];
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
  for (int t = blockIdx.x; t < total && ok; t += gridDim.x, ++local) {
    int gi, b, i0, j0;
    decode_tile(L, t, gi, b, i0, j0);
    const Group& G = L.g[gi];
    const int acc = local & 1;
    const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
    const int out_cols = L.phase == kUpdate ? G.n : G.m;
    const int row0 = i0 + q * 32;
    const bool rows_ok = row0 < G.m;   // warp-uniform: whole subtile beyond the matrix -> nothing to store
    const int jc0 = j0 + half * (kChunks * EPI_TILE);
    const CUtensorMap* omap = L.phase == kGram ? &G.ae : (L.phase == kPoly ? &G.be : &G.xe[L.src ^ 1]);
    const CUtensorMap* amap = L.phase == kPoly ? &G.ae : &G.xe[L.src];
    int nch = 0;
    while (nch < kChunks && jc0 + nch * EPI_TILE < out_cols) ++nch;
    const bool work = rows_ok && nch > 0;
    // prefetch the operand subtiles of the first two chunks (the previous tile's stores must have left them)
    if (lane == 0 && work) {
      bulk_wait_read<0>();
      if (has_aux) {
        for (int c = 0; c < 2 && c < nch; ++c) {
          mbar_arrive_expect_tx(bar[c], EPI_BUF_BYTES);
          tma_load_3d(buf[c], amap, bar[c], jc0 + c * EPI_TILE, row0, b);
        }
      }
    }
    __syncwarp();
    // warp-uniform outcome: the TMEM loads below are .sync.aligned
    if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], use, ctx) ? 1 : 0)) break;
    tc_fence_after();
    for (int c = 0; c < nch; ++c) {
      const int bi = c & 1;
      uint32_t r[32];
      tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                    static_cast<uint32_t>(acc * BN + half * (kChunks * EPI_TILE) + c * EPI_TILE), r);
      tmem_ld_wait(r);
      if (!rows_ok) continue;
      uint8_t* row = buf[bi];
      if (has_aux) {
        if (!__all_sync(0xffffffffu, mbar_wait(bar[bi], bphase[bi], ctx) ? 1 : 0)) { ok = false; break; }
        bphase[bi] ^= 1u;
      } else if (c >= 2) {
        if (lane == 0) bulk_wait_read<1>();   // the store of chunk c-2 has left this buffer
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
        if (has_aux && c + 2 < nch) {   // refill this buffer with the operand of chunk c+2
          bulk_wait_read<0>();
          mbar_arrive_expect_tx(bar[bi], EPI_BUF_BYTES);
          tma_load_3d(row, amap, bar[bi], jc0 + (c + 2) * EPI_TILE, row0, b);
        }
      }
      __syncwarp();
    }
    tc_fence_before();
    mbar_arrive(&tempty[acc]);
  }
  if (lane == 0) {
    bulk_wait<0>();   // stores complete before the CTA exits
    if (!ok) {        // unwinding: operand loads still in flight land before shared memory goes away
      for (int k = 0; k < 2; ++k) mbar_wait_drain(bar[k], bphase[k]);
    }
  }
  __syncwarp();
}

// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) ns_phase_kernel(const __grid_constant__ Launch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;
  uint8_t* ebuf = smem + STAGES * STAGE_BYTES;                        // 1024-aligned
  uint64_t* bars = reinterpret_cast<uint64_t*>(ebuf + EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* ebar = drain + 1;                                         // 2 per epilogue warp
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const uint32_t warp = warp_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps * 32);
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
      if (L.phase == kPoly) { tma_prefetch_desc(&G.ak); tma_prefetch_desc(&G.be); }
      if (L.phase == kUpdate) {
        tma_prefetch_desc(&G.bk); tma_prefetch_desc(&G.xmn[L.src]);
        tma_prefetch_desc(&G.xe[0]); tma_prefetch_desc(&G.xe[1]);
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx ctx{abort_flag, L.status};

  // Each role warp reconverges (__syncwarp) before the CTA-wide barrier below, which is an aligned barrier.
  if (warp == 0) {
    if (lane_id() == 0) run_producer(L, sa, sb, full, empty, ctx);
    __syncwarp();
  } else if (warp == 1) {
    if (lane_id() == 0) run_mma(L, sa, sb, full, empty, tfull, tempty, drain, tmem_base, ctx);
    __syncwarp();
  } else {
    run_epilogue(L, tfull, tempty, ebuf, ebar, tmem_base, ctx);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(L.status, kStatusAborted);
}

}  // namespace ns
}  // namespace moteopt
