// Newton-Schulz phase kernel for sm_100a (tcgen05 + TMEM + TMA).
//
// One launch runs one phase of one Newton-Schulz iteration (mote/train/muon.py:37-40) for every matrix of every
// shape group at once:
//   kGram:   A  = bf16(X X^T)
//   kPoly:   B  = bf16( bf16(b*A) + bf16(c * bf16(A A)) )          (A is symmetric, so A A = A A^T)
//   kUpdate: X' = bf16( bf16(a*X) + bf16(B X) )                    or, on the last iteration, the Muon apply
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
// Epilogue of one 32-column chunk of one row: v[] holds the fp32 accumulator (or its transform), `cols_left`
// (> 0, a multiple of 8) how many of the 32 columns exist.
__device__ __forceinline__ void store_bf16_row(__nv_bfloat16* dst, const float (&v)[32], int cols_left) {
  uint32_t pk[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) pk[k] = pack_bf16x2(v[2 * k], v[2 * k + 1]);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (k * 8 < cols_left) d4[k] = make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
}

// mote/train/muon.py:93-99 for the 32 columns j..j+31 of row i of the orthogonalised iterate.
__device__ __forceinline__ void apply_row(const Group& G, const MatApply& ma, int i, int j, const float (&o)[32]) {
  if (i >= G.mv) return;
  if (!G.transposed) {
    // p[i][j + k], row stride nv
    float* pr = ma.p + static_cast<size_t>(i) * G.nv + j;
    const int lim = min(32, G.nv - j);
    const bool vec = ((reinterpret_cast<uintptr_t>(pr) & 15u) == 0) && (G.nv % 4 == 0);
    if (vec) {
#pragma unroll
      for (int k = 0; k < 32; k += 4) {
        if (k < lim) {
          float4 pv = *reinterpret_cast<float4*>(pr + k);
          float* pe = reinterpret_cast<float*>(&pv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float x = pe[e];
            if (ma.has_decay) x = __fmul_rn(x, ma.decay_mul);
            pe[e] = fmaf(ma.neg_lr, __fmul_rn(o[k + e], ma.scale), x);
          }
          *reinterpret_cast<float4*>(pr + k) = pv;
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        if (k < lim) {
          float x = pr[k];
          if (ma.has_decay) x = __fmul_rn(x, ma.decay_mul);
          pr[k] = fmaf(ma.neg_lr, __fmul_rn(o[k], ma.scale), x);
        }
      }
    }
  } else {
    // the parameter is the transpose: p[j + k][i], row stride mv (consecutive threads -> consecutive i)
    float* pc = ma.p + static_cast<size_t>(j) * G.mv + i;
    const int lim = min(32, G.nv - j);
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      if (k < lim) {
        float* q = pc + static_cast<size_t>(k) * G.mv;
        float x = *q;
        if (ma.has_decay) x = __fmul_rn(x, ma.decay_mul);
        *q = fmaf(ma.neg_lr, __fmul_rn(o[k], ma.scale), x);
      }
    }
  }
}

// Unpack 8 bf16 (one uint4) into floats.
__device__ __forceinline__ void unpack8(const uint4& w, float* v) {
  v[0] = bf16_lo(w.x); v[1] = bf16_hi(w.x); v[2] = bf16_lo(w.y); v[3] = bf16_hi(w.y);
  v[4] = bf16_lo(w.z); v[5] = bf16_hi(w.z); v[6] = bf16_lo(w.w); v[7] = bf16_hi(w.w);
}

// Round a pair to bf16 and back (one cvt.rn.bf16x2.f32 for two values).
__device__ __forceinline__ void round2(float& a, float& b) {
  const uint32_t p = pack_bf16x2(a, b);
  a = bf16_lo(p);
  b = bf16_hi(p);
}

// Epilogue warps 2..9: warp w reads TMEM lane quarter (w % 4) and owns columns [128*h, 128*h + 128) of the tile,
// h = (w - 2) / 4. The bf16 operand the phase's polynomial needs (A for kPoly, X for kUpdate) is loaded before the
// accumulator is waited for, so its latency hides behind the tile's MMAs.
__device__ __forceinline__ void run_epilogue(const Launch& L, uint64_t* tfull, uint64_t* tempty, uint32_t tmem_base,
                                             const WaitCtx& ctx) {
  constexpr int kChunks = BN / 32 / 2;   // 32-column chunks per epilogue warp
  const int total = L.tile_start[L.n_groups];
  const int q = static_cast<int>(warp_id() & 3u);
  const int half = (static_cast<int>(warp_id()) - 2) >> 2;
  const int row = q * 32 + static_cast<int>(lane_id());
  int local = 0;
  for (int t = blockIdx.x; t < total; t += gridDim.x, ++local) {
    int gi, b, i0, j0;
    decode_tile(L, t, gi, b, i0, j0);
    const Group& G = L.g[gi];
    const int acc = local & 1;
    const uint32_t use = static_cast<uint32_t>(local >> 1) & 1u;
    const int out_cols = L.phase == kUpdate ? G.n : G.m;
    const int i = i0 + row;
    const bool row_ok = i < G.m;
    const int jc0 = j0 + half * (kChunks * 32);   // first column of this warp
    const size_t row_off = L.phase == kUpdate ? (static_cast<size_t>(b) * G.m + i) * G.n
                                              : (static_cast<size_t>(b) * G.m + i) * G.m;
    // prefetch the polynomial's bf16 operand for this warp's columns
    uint4 aux[kChunks][4];
    if (L.phase != kGram) {
      const __nv_bfloat16* src = (L.phase == kPoly ? G.a : G.x[L.src]) + row_off;
#pragma unroll
      for (int c = 0; c < kChunks; ++c)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = jc0 + c * 32 + k * 8;
          aux[c][k] = (row_ok && j < out_cols) ? *reinterpret_cast<const uint4*>(src + j) : make_uint4(0, 0, 0, 0);
        }
    }
    // warp-uniform outcome: the TMEM loads below are .sync.aligned
    if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], use, ctx) ? 1 : 0)) break;
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const int j = jc0 + c * 32;
      if (j >= out_cols) break;   // uniform across the warp
      uint32_t r[32];
      tmem_ld32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                    static_cast<uint32_t>(acc * BN + half * (kChunks * 32) + c * 32), r);
      tmem_ld_wait(r);
      if (!row_ok) continue;
      const int cols_left = out_cols - j;
      float v[32];
      if (L.phase == kGram) {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = __uint_as_float(r[k]);
        store_bf16_row(G.a + row_off + j, v, cols_left);
      } else {
        float a[32];
#pragma unroll
        for (int k = 0; k < 4; ++k) unpack8(aux[c][k], a + 8 * k);
        if (L.phase == kPoly) {
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            float aa0 = __uint_as_float(r[k]), aa1 = __uint_as_float(r[k + 1]);
            round2(aa0, aa1);                                                   // A @ A
            float t10 = __fmul_rn(kNsB, a[k]), t11 = __fmul_rn(kNsB, a[k + 1]);
            round2(t10, t11);                                                   // b * A
            float t20 = __fmul_rn(kNsC, aa0), t21 = __fmul_rn(kNsC, aa1);
            round2(t20, t21);                                                   // c * (A @ A)
            v[k] = __fadd_rn(t10, t20);                                         // rounded by the store
            v[k + 1] = __fadd_rn(t11, t21);
          }
          store_bf16_row(G.b + row_off + j, v, cols_left);
        } else {
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            float bx0 = __uint_as_float(r[k]), bx1 = __uint_as_float(r[k + 1]);
            round2(bx0, bx1);                                                   // B @ X
            float ax0 = __fmul_rn(kNsA, a[k]), ax1 = __fmul_rn(kNsA, a[k + 1]);
            round2(ax0, ax1);                                                   // a * X
            v[k] = __fadd_rn(ax0, bx0);
            v[k + 1] = __fadd_rn(ax1, bx1);
          }
          if (L.apply) {
#pragma unroll
            for (int k = 0; k < 32; k += 2) round2(v[k], v[k + 1]);            // O (bf16)
            apply_row(G, L.mats[G.first + b], i, j, v);
          } else {
            store_bf16_row(G.x[L.src ^ 1] + row_off + j, v, cols_left);
          }
        }
      }
    }
    tc_fence_before();
    mbar_arrive(&tempty[acc]);
  }
}

// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1) ns_phase_kernel(const __grid_constant__ Launch L) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane_id() == 0) {
    for (int g = 0; g < L.n_groups; ++g) {
      const Group& G = L.g[g];
      if (L.phase == kGram) tma_prefetch_desc(&G.xk[L.src]);
      if (L.phase == kPoly) tma_prefetch_desc(&G.ak);
      if (L.phase == kUpdate) { tma_prefetch_desc(&G.bk); tma_prefetch_desc(&G.xmn[L.src]); }
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
    run_epilogue(L, tfull, tempty, tmem_base, ctx);
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
