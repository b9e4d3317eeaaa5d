// Memory-bound kernels of the optimizer step (sm_100a). Each is a grid-stride loop over fixed 16K-element chunks
// (2K for AdamW) of a segment list, with 128-bit loads where the pointers allow. Reductions are deterministic: a
// fixed per-thread order, a fixed warp-shuffle tree and a fixed cross-warp order per chunk, one partial per chunk,
// and a fixed-order second pass, so results are bitwise identical from run to run.
//
// Rounding follows the reference's torch ops one by one (see the per-kernel comments); __fmul_rn / __fadd_rn /
// __fdiv_rn keep the compiler from contracting what torch rounds separately, fmaf is used where torch fuses.
#pragma once

#include "mt_types.h"
#include "ptx.cuh"

namespace moteopt {

__device__ __forceinline__ int find_seg(const int* chunk_start, int n, int chunk) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {   // last segment whose start <= chunk
    const int mid = (lo + hi + 1) >> 1;
    if (chunk_start[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float load_g1(const void* g, int64_t i, int dt) {
  return dt == kBF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(g)[i])
                     : reinterpret_cast<const float*>(g)[i];
}

__device__ __forceinline__ float4 load_g4(const void* g, int64_t i, int dt) {
  if (dt == kBF16) {
    const uint2 w = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(g) + i);
    return make_float4(bf16_lo(w.x), bf16_hi(w.x), bf16_lo(w.y), bf16_hi(w.y));
  }
  return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(g) + i);
}

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
__device__ __forceinline__ bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }
__device__ __forceinline__ bool g_vec_ok(const void* g, int dt) { return dt == kBF16 ? aligned8(g) : aligned16(g); }

// Exact helpers of SharedDivisor's rare path (below).
__device__ __forceinline__ float pow2f(int n) {   // 2^n for n in [-149, 127], exactly
  return n >= -126 ? __uint_as_float(static_cast<uint32_t>(n + 127) << 23) : __uint_as_float(1u << (n + 149));
}
// x (|x| in (0.25, 1]) times 2^n, rounded once
__device__ __forceinline__ float scale_once(float x, int n) {
  if (n > 191) return copysignf(__int_as_float(0x7f800000), x);
  if (n > 127) return __fmul_rn(__fmul_rn(x, 0x1p64f), pow2f(n - 64));
  if (n >= -126) return __fmul_rn(x, pow2f(n));
  if (n >= -152) return __fmul_rn(__fmul_rn(x, pow2f(n + 64)), 0x1p-64f);
  return copysignf(0.f, x);   // |x 2^n| < 2^-152: below half the smallest subnormal
}
// a finite nonzero float as m 2^e with |m| in [0.5, 1) (bias 126) or [1, 2) (bias 127)
__device__ __forceinline__ float split_exp(float a, int bias, int* e) {
  uint32_t u = __float_as_uint(a);
  int shift = 0;
  if (((u >> 23) & 0xffu) == 0u) {   // subnormal: scale into the normal range first (exact)
    u = __float_as_uint(__fmul_rn(a, 0x1p64f));
    shift = 64;
  }
  *e = static_cast<int>((u >> 23) & 0xffu) - bias - shift;
  return __uint_as_float((u & 0x807fffffu) | (static_cast<uint32_t>(bias) << 23));
}
// a / d for one divisor d shared by many numerators (the normalisation's norm, the trainer's total_n), correctly
// rounded, without a reciprocal per element: inside a window of |a| where q = RN(a r) (r = RN(1/d)) plus one
// Markstein correction RN(q + (a - q d) r) is the IEEE quotient (Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", 1990) (|a| >= 2^-80 and 2^-99 <= |a| / d <= 2^125, for 2^-100 <= d < 2^100: the
// residual is exact and nothing under- or overflows; a factor-2 margin on each bound), that quotient, decided by one
// unsigned compare on the bits of |a|. Zeros, infinities and NaN give a r (IEEE's result for them); every other
// numerator takes div_rare, an exact inline path (no call): a = m 2^ea with |m| in [0.5, 1) and d = dm 2^ed with dm
// in [1, 2), so q' = RN(m / dm) by the same correction lies in (0.25, 1); the quotient is q' 2^(ea-ed) scaled back
// with one rounding (overflow gives Inf, underflow a subnormal or zero), and where that rounding falls exactly on a
// midpoint of the subnormal grid the residual's sign picks the neighbour the exact quotient lies toward. A negative
// divisor moves its sign onto the numerator (a / -d = -a / d exactly). tests/test_gpu_selftest.py holds it against
// IEEE division bit for bit: the optimizer's ranges and their edges, tiny and subnormal numerators, divisors across
// the whole exponent range, and special values.
struct SharedDivisor {
  float d, r;          // |divisor| and RN(1 / |divisor|)
  uint32_t lo, span;   // fast path when lo <= bits(|a|) <= lo + span
  uint32_t sgn;        // the divisor's sign bit
  __device__ __forceinline__ float div_rare(float a) const {
    int ed, ea;
    const float dm = split_exp(d, 127, &ed);
    const float rm = __frcp_rn(dm);
    const float m = split_exp(a, 126, &ea);
    const float q1 = __fmul_rn(m, rm);
    const float qm = fmaf(fmaf(-q1, dm, m), rm, q1);   // RN(m / dm), in (0.25, 1)
    const float em = fmaf(-qm, dm, m);                  // exact: m / dm - qm has the sign of em
    const int n = ea - ed;
    float v = scale_once(qm, n);
    // qm 2^n below 2^-126 (tested before the rounding, which can carry it up to 2^-126 itself): the second rounding is
    // to the subnormal grid
    if ((n <= -126 || (n == -125 && qm < 0.5f)) && em != 0.f && n >= -152) {
      const float w = __fmul_rn(qm, pow2f(n + 149));   // the quotient in units of 2^-149, exact
      if (fabsf(w - truncf(w)) == 0.5f) v = __fmul_rn(em > 0.f ? ceilf(w) : floorf(w), 0x1p-149f);
    }
    return v;
  }
  __device__ __forceinline__ float div(float a) const {
    a = __uint_as_float(__float_as_uint(a) ^ sgn);
    const uint32_t ab = __float_as_uint(a) & 0x7fffffffu;
    if (ab - lo <= span) {
      const float q = __fmul_rn(a, r);
      return fmaf(fmaf(-q, d, a), r, q);
    }
    if (ab == 0u || ab >= 0x7f800000u || !(d > 0.f && d <= 0x1.fffffep127f)) return __fmul_rn(a, r);
    return div_rare(a);
  }
  // div4 for numerators known to satisfy |a| <= d with d > 0 (an entry over its matrix's norm plus eps: the norm is
  // the correctly rounded root of the sum of the same entries' squares, so no entry exceeds it, and d finite means
  // every entry is finite): only the window's lower bound can fail, tested on the smallest |a|
  __device__ __forceinline__ float4 div4_bounded(float4 a) const {
    const uint32_t m0 = __float_as_uint(a.x) & 0x7fffffffu, m1 = __float_as_uint(a.y) & 0x7fffffffu;
    const uint32_t m2 = __float_as_uint(a.z) & 0x7fffffffu, m3 = __float_as_uint(a.w) & 0x7fffffffu;
    if (min(min(m0, m1), min(m2, m3)) - lo <= span) {   // lo <= every |a| (and |a| <= d <= the upper bound)
      const float q0 = __fmul_rn(a.x, r), q1 = __fmul_rn(a.y, r), q2 = __fmul_rn(a.z, r), q3 = __fmul_rn(a.w, r);
      return make_float4(fmaf(fmaf(-q0, d, a.x), r, q0), fmaf(fmaf(-q1, d, a.y), r, q1),
                         fmaf(fmaf(-q2, d, a.z), r, q2), fmaf(fmaf(-q3, d, a.w), r, q3));
    }
    float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll 1
    for (int e = 0; e < 4; ++e) v[e] = div(v[e]);   // one copy of the rare path
    return make_float4(v[0], v[1], v[2], v[3]);
  }
  // four quotients: the fast path for all four, one window test on their smallest and largest |a|, and div() for
  // the four when any of them lies outside the window (rare)
  __device__ __forceinline__ float4 div4(float4 a) const {
    const uint32_t b0 = __float_as_uint(a.x) ^ sgn, b1 = __float_as_uint(a.y) ^ sgn;
    const uint32_t b2 = __float_as_uint(a.z) ^ sgn, b3 = __float_as_uint(a.w) ^ sgn;
    const uint32_t m0 = b0 & 0x7fffffffu, m1 = b1 & 0x7fffffffu, m2 = b2 & 0x7fffffffu, m3 = b3 & 0x7fffffffu;
    const uint32_t mn = min(min(m0, m1), min(m2, m3)), mx = max(max(m0, m1), max(m2, m3));
    if (mn >= lo && mx - lo <= span) {
      const float x0 = __uint_as_float(b0), x1 = __uint_as_float(b1), x2 = __uint_as_float(b2), x3 = __uint_as_float(b3);
      const float q0 = __fmul_rn(x0, r), q1 = __fmul_rn(x1, r), q2 = __fmul_rn(x2, r), q3 = __fmul_rn(x3, r);
      return make_float4(fmaf(fmaf(-q0, d, x0), r, q0), fmaf(fmaf(-q1, d, x1), r, q1),
                         fmaf(fmaf(-q2, d, x2), r, q2), fmaf(fmaf(-q3, d, x3), r, q3));
    }
    float v[4] = {a.x, a.y, a.z, a.w};
#pragma unroll 1
    for (int e = 0; e < 4; ++e) v[e] = div(v[e]);   // one copy of the rare path
    return make_float4(v[0], v[1], v[2], v[3]);
  }
};
__device__ __forceinline__ SharedDivisor shared_divisor(float den) {
  SharedDivisor s;
  s.sgn = __float_as_uint(den) & 0x80000000u;
  s.d = fabsf(den);
  s.r = __frcp_rn(s.d);
  if (s.d >= 0x1p-100f && s.d < 0x1p100f) {
    s.lo = __float_as_uint(fmaxf(0x1p-80f, __fmul_rn(s.d, 0x1p-99f)));
    s.span = __float_as_uint(fminf(0x1.fffffep127f, __fmul_rn(s.d, 0x1p125f))) - s.lo;
  } else {   // empty window: bits(|a|) - lo wraps to at least 1
    s.lo = 0xffffffffu;
    s.span = 0u;
  }
  return s;
}

// The divisor of train.py:945 (grads /= total_n): a launch argument, or a device scalar (the trainer's total_n
// tensor, read without a host round trip). Read only by launches that divide.
template <typename Args>
__device__ __forceinline__ float grad_div(const Args& A, bool used) {
  return (used && A.div_dev != nullptr) ? *A.div_dev : A.div;
}

// train.py:945-946: g / total_n (fp32 division, IEEE: __fdiv_rn), then * clip coefficient (fp32 multiply). The grads'
// division stays the IEEE intrinsic: forms with one shared reciprocal (SharedDivisor) measured no faster on the
// dividing passes, and every form that changed this struct slowed the non-dividing AdamW pass by 7 %.
struct GradXform {
  int has_div;
  float div;
  int has_coef;
  float coef;
  __device__ __forceinline__ float operator()(float g) const {
    if (has_div) g = __fdiv_rn(g, div);
    if (has_coef) g = __fmul_rn(g, coef);
    return g;
  }
};

// Sum of a per-thread fp64 value over the block, in a fixed order. Result valid in thread 0.
__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  double s = 0.0;
  if (threadIdx.x == 0) {
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) s += red[k];
  }
  __syncthreads();
  return s;
}

// acc + x^2 in fp64. The square of an fp32 value is exact in fp64 (48 significant bits), so a sum of squares
// accumulated this way is off the exact sum by ~1e-16 relative: sqrt of it, rounded to fp32, is the correctly
// rounded Frobenius norm (a fp64 -> fp32 rounding of a correctly rounded fp64 sqrt is innocuous, 53 >= 2 * 24 + 2).
__device__ __forceinline__ double sqacc(float x, double acc) {
  const double d = static_cast<double>(x);
  return fma(d, d, acc);
}

// ---------------------------------------------------------------------------------------------------------------
// sum of squares of (g / div) per chunk. A full, 16-byte aligned chunk is read with all of a thread's 16-byte loads
// issued before the first is used (128 B in flight per thread); ragged chunks fall back to element loads. The order of
// the per-thread sum is fixed either way.
__device__ __forceinline__ double sq_acc2_bf16(uint32_t w, const GradXform& X, double acc) {
  const float a = X(bf16_lo(w)), b = X(bf16_hi(w));
  acc = sqacc(a, acc);
  return sqacc(b, acc);
}
__device__ __forceinline__ double sq_acc8_bf16(const uint4& v, const GradXform& X, double acc) {
  acc = sq_acc2_bf16(v.x, X, acc);
  acc = sq_acc2_bf16(v.y, X, acc);
  acc = sq_acc2_bf16(v.z, X, acc);
  return sq_acc2_bf16(v.w, X, acc);
}
__device__ __forceinline__ double sq_acc4_f32(const float4& v, const GradXform& X, double acc) {
  const float a = X(v.x), b = X(v.y), d = X(v.z), e = X(v.w);
  acc = sqacc(a, acc); acc = sqacc(b, acc); acc = sqacc(d, acc); acc = sqacc(e, acc);
  return acc;
}

// kDiv: whether the grads are divided first; the division (a call on its slow path) is compiled only where used, so
// the common path keeps all of its loads in registers.
template <bool kDiv>
__device__ __forceinline__ void sumsq_chunks(const SumsqArgs& A, double* red) {
  const int total = A.chunk_start[A.n];
  const GradXform X{kDiv ? 1 : 0, grad_div(A, kDiv), 0, 1.f};
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    const SumsqSeg& S = A.seg[s];
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kChunk;
    const int64_t end = min(begin + kChunk, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel);
    double acc = 0.0;
    if (end - begin == kChunk && aligned16(S.g)) {
      if (S.dtype == kBF16) {   // 2048 16-byte vectors: 8 per thread
        const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(S.g) + begin);
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __ldg(p + threadIdx.x + k * kMtThreads);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc = sq_acc8_bf16(v[k], X, acc);
      } else {                  // 4096 16-byte vectors: 16 per thread, in two batches of 8
        const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(S.g) + begin);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float4 v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) v[k] = __ldg(p + threadIdx.x + (h * 8 + k) * kMtThreads);
#pragma unroll
          for (int k = 0; k < 8; ++k) acc = sq_acc4_f32(v[k], X, acc);
        }
      }
    } else if (g_vec_ok(S.g, S.dtype)) {
      const int64_t vend = begin + ((end - begin) & ~int64_t(3));
      for (int64_t i = begin + 4 * threadIdx.x; i < vend; i += 4 * kMtThreads)
        acc = sq_acc4_f32(load_g4(S.g, i, S.dtype), X, acc);
      for (int64_t i = vend + threadIdx.x; i < end; i += kMtThreads) {
        const float a = X(load_g1(S.g, i, S.dtype));
        acc = sqacc(a, acc);
      }
    } else {
      for (int64_t i = begin + threadIdx.x; i < end; i += kMtThreads) {
        const float a = X(load_g1(S.g, i, S.dtype));
        acc = sqacc(a, acc);
      }
    }
    const double tot = block_sum(acc, red);
    if (threadIdx.x == 0) A.partials[A.chunk_base + c] = tot;
  }
}

// One instantiation per divisor mode (each gets its own register allocation): without the division 48 registers and
// five blocks per SM; the dividing one (its slow path is a call) four blocks, so that nothing spills.
template <bool kDiv>
__global__ void __launch_bounds__(kMtThreads, kDiv ? 4 : 5) sumsq_kernel(const __grid_constant__ SumsqArgs A) {
  __shared__ double red[kMtThreads / 32];
  sumsq_chunks<kDiv>(A, red);
}

// ---------------------------------------------------------------------------------------------------------------
// Sum of partials[begin, end) over a warp in fp64: lane l adds elements l, l+32, ... in that order, then a fixed xor
// tree. Loads go out eight at a time before their adds (out-of-range ones read as 0, and s + 0 = s for the
// non-negative sums here), so a tensor of a few hundred chunks costs one or two load round trips. Result in every lane.
__device__ __forceinline__ double warp_sum_partials(const double* partials, int begin, int end, int lane) {
  double s = 0.0;
  for (int base = begin + lane; base < end; base += 8 * 32) {
    double v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = base + 32 * k < end ? partials[base + 32 * k] : 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += v[k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Warp 0's last stage of the global norm: total = fp32(sqrt(sum of the per-tensor norms' squares)), the squares summed
// in fp64 (lane l takes tensors l, l+32, ... in order, then a fixed xor tree), and the clip coefficient.
__device__ __forceinline__ void finish_total(const float* tnorm, int n_tensors, int has_clip, float max_norm, float* out,
                                             int* status, int lane) {
  double acc = 0.0;
  for (int t = lane; t < n_tensors; t += 32) acc += static_cast<double>(tnorm[t]) * static_cast<double>(tnorm[t]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    const float total = static_cast<float>(sqrt(acc));
    float coef = 1.0f;
    if (has_clip) {
      // clamp(max_norm / (total + 1e-6), max=1) as torch evaluates it: a Python float over a tensor is
      // Tensor.__rdiv__, reciprocal(total + 1e-6) * max_norm (two fp32 roundings); a NaN norm gives NaN, as in torch
      const float c = __fmul_rn(__frcp_rn(__fadd_rn(total, 1e-6f)), max_norm);
      coef = (c > 1.0f) ? 1.0f : c;
    }
    out[0] = total;
    out[1] = coef;
    if (status != nullptr && !isfinite(total)) atomicOr(status, kStatusNonFinite);
  }
}

// per-tensor norms -> total norm (the norm of the per-tensor norms, as torch's get_total_norm) -> clip coefficient.
// One warp per tensor (lanes sum strided chunk partials in fp64, then a fixed xor tree), the per-tensor norms kept in
// shared memory, then warp 0 sums their squares in the same fixed way: deterministic, and no serial chain of loads.
__global__ void __launch_bounds__(1024) norm_finalize_kernel(const __grid_constant__ FinalizeArgs A) {
  __shared__ float tnorm[kMaxFinalTensors];
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int nwarps = static_cast<int>(blockDim.x >> 5);
  // three tensors per warp at a time: the first eight partials per lane of all three are loaded before any is summed
  // (a tensor's sum is the same as warp_sum_partials': lane l adds elements l, l+32, ... in order)
  for (int t0 = warp; t0 < A.n_tensors; t0 += 3 * nwarps) {
    double v[3][8];
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int t = t0 + u * nwarps;
      const int b = t < A.n_tensors ? A.tensor_chunk_start[t] : 0, e = t < A.n_tensors ? A.tensor_chunk_start[t + 1] : 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) v[u][k] = b + lane + 32 * k < e ? A.partials[b + lane + 32 * k] : 0.0;
    }
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int t = t0 + u * nwarps;
      if (t >= A.n_tensors) break;
      const int b = A.tensor_chunk_start[t], e = A.tensor_chunk_start[t + 1];
      MO_CHECK(b <= e);
      double s = 0.0;
#pragma unroll
      for (int k = 0; k < 8; ++k) s += v[u][k];
      for (int base = b + lane + 8 * 32; base < e; base += 8 * 32) {   // tensors of more than 256 chunks
        double w[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = base + 32 * k < e ? A.partials[base + 32 * k] : 0.0;
#pragma unroll
        for (int k = 0; k < 8; ++k) s += w[k];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) tnorm[t] = static_cast<float>(sqrt(s));
    }
  }
  __syncthreads();
  if (warp == 0) finish_total(tnorm, A.n_tensors, A.has_clip, A.max_norm, A.out, A.status, lane);
}

// ---------------------------------------------------------------------------------------------------------------
// Sum of every chunk partial in fixed order, in fp64 (one rank's share of the global sum of squares).
__global__ void __launch_bounds__(1024) partials_total_kernel(const double* partials, int n, double* out) {
  __shared__ double red[32];
  double acc = 0.0;
  const int stride = static_cast<int>(blockDim.x);
  for (int base = threadIdx.x; base < n; base += 8 * stride) {   // thread order c, c + stride, ...; loads batched by 8
    double v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = base + stride * k < n ? partials[base + stride * k] : 0.0;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += v[k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int k = 0; k < static_cast<int>(blockDim.x >> 5); ++k) s += red[k];
    *out = s;
  }
}

// total norm = sqrt(sum of the ranks' sums, in rank order) and the clip coefficient, as norm_finalize_kernel.
__global__ void coef_from_sums_kernel(const __grid_constant__ CoefArgs A) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double s = 0.0;
  for (int r = 0; r < A.n; ++r) s += A.sums[r];
  const float total = static_cast<float>(sqrt(s));
  float coef = 1.0f;
  if (A.has_clip) {
    const float c = __fmul_rn(__frcp_rn(__fadd_rn(total, 1e-6f)), A.max_norm);   // as norm_finalize_kernel
    coef = (c > 1.0f) ? 1.0f : c;
  }
  A.out[0] = total;
  A.out[1] = coef;
  if (A.status != nullptr && !isfinite(total)) atomicOr(A.status, kStatusNonFinite);
}

// ---------------------------------------------------------------------------------------------------------------
// The sharded step's grad reduce-scatter, read from every rank's grad region over NVLink (peer mappings), fused with
// the clip's sums of squares. Element k of a piece: the sum over ranks q = 0, 1, ... of src[q][k] in fp32, in that
// order (the first value taken as it is), rounded once to the grads' type and stored to dst; then (dst[k] / div)^2
// joins the chunk's fp64 partial. A chunk's elements reach a thread in sumsq_chunks' order (full aligned chunks: the
// thread's 16-byte vectors t, t + 256, ...; ragged ones: 4-element vectors, then single elements), so the partials
// of a piece equal sumsq_chunks' partials of the same reduced values.
__device__ __forceinline__ void unpack8_bf16(const uint4& w, float* v) {
  v[0] = bf16_lo(w.x); v[1] = bf16_hi(w.x); v[2] = bf16_lo(w.y); v[3] = bf16_hi(w.y);
  v[4] = bf16_lo(w.z); v[5] = bf16_hi(w.z); v[6] = bf16_lo(w.w); v[7] = bf16_hi(w.w);
}
__device__ __forceinline__ void add8_bf16(const uint4& w, float* v) {
  v[0] = __fadd_rn(v[0], bf16_lo(w.x)); v[1] = __fadd_rn(v[1], bf16_hi(w.x));
  v[2] = __fadd_rn(v[2], bf16_lo(w.y)); v[3] = __fadd_rn(v[3], bf16_hi(w.y));
  v[4] = __fadd_rn(v[4], bf16_lo(w.z)); v[5] = __fadd_rn(v[5], bf16_hi(w.z));
  v[6] = __fadd_rn(v[6], bf16_lo(w.w)); v[7] = __fadd_rn(v[7], bf16_hi(w.w));
}
__device__ __forceinline__ float4 add4(const float4& a, const float4& b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
// v rounded to the grads' type (as floats) and stored at g[i..i+3]
__device__ __forceinline__ float4 store_g4(void* g, int64_t i, int dt, float4 v) {
  if (dt == kBF16) {
    const uint32_t lo = pack_bf16x2(v.x, v.y), hi = pack_bf16x2(v.z, v.w);
    *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(g) + i) = make_uint2(lo, hi);
    return make_float4(bf16_lo(lo), bf16_hi(lo), bf16_lo(hi), bf16_hi(hi));
  }
  *reinterpret_cast<float4*>(reinterpret_cast<float*>(g) + i) = v;
  return v;
}
__device__ __forceinline__ float store_g1(void* g, int64_t i, int dt, float v) {
  if (dt == kBF16) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v);
    reinterpret_cast<__nv_bfloat16*>(g)[i] = b;
    return __bfloat162float(b);
  }
  reinterpret_cast<float*>(g)[i] = v;
  return v;
}

// kW: the largest number of ranks the instantiation sums (1, 2, 4 or 8; world <= kW); each thread keeps 8 / kW of
// its 16-byte vectors of every rank in flight at once (128 bytes), so the latency of peer loads is covered.
template <bool kDiv, int kW>
__device__ __forceinline__ void peer_reduce_chunks(const PeerReduceArgs& A, double* red) {
  constexpr int U = 8 / kW;
  const int total = A.chunk_start[A.n];
  const GradXform X{kDiv ? 1 : 0, A.div, 0, 1.f};
  const int world = A.world;
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    const PeerSeg& S = A.seg[s];
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kChunk;
    const int64_t end = min(begin + kChunk, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel && world >= 1 && world <= kW);
    bool a16 = aligned16(S.dst), vec = g_vec_ok(S.dst, S.dtype);
    for (int q = 0; q < world; ++q) {
      a16 = a16 && aligned16(S.src[q]);
      vec = vec && g_vec_ok(S.src[q], S.dtype);
    }
    double acc = 0.0;
    if (end - begin == kChunk && a16) {
      if (S.dtype == kBF16) {   // 2048 16-byte vectors: thread t takes t + 256 k, k = 0..7
        uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(S.dst) + begin);
        for (int k0 = 0; k0 < 8; k0 += U) {
          uint4 w[kW][U];
#pragma unroll
          for (int q = 0; q < kW; ++q) {   // every rank's vectors in flight before the first add
            if (q < world) {
              const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(S.src[q]) + begin);
#pragma unroll
              for (int j = 0; j < U; ++j) w[q][j] = p[threadIdx.x + (k0 + j) * kMtThreads];
            }
          }
#pragma unroll
          for (int j = 0; j < U; ++j) {
            float v[8];
            unpack8_bf16(w[0][j], v);
#pragma unroll
            for (int q = 1; q < kW; ++q)
              if (q < world) add8_bf16(w[q][j], v);
            const uint4 o = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                                       pack_bf16x2(v[6], v[7]));
            d[threadIdx.x + (k0 + j) * kMtThreads] = o;
            acc = sq_acc8_bf16(o, X, acc);
          }
        }
      } else {                  // 4096 16-byte vectors: thread t takes t + 256 k, k = 0..15
        float4* d = reinterpret_cast<float4*>(reinterpret_cast<float*>(S.dst) + begin);
        for (int k0 = 0; k0 < 16; k0 += U) {
          float4 w[kW][U];
#pragma unroll
          for (int q = 0; q < kW; ++q) {
            if (q < world) {
              const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(S.src[q]) + begin);
#pragma unroll
              for (int j = 0; j < U; ++j) w[q][j] = p[threadIdx.x + (k0 + j) * kMtThreads];
            }
          }
#pragma unroll
          for (int j = 0; j < U; ++j) {
            float4 v = w[0][j];
#pragma unroll
            for (int q = 1; q < kW; ++q)
              if (q < world) v = add4(v, w[q][j]);
            d[threadIdx.x + (k0 + j) * kMtThreads] = v;
            acc = sq_acc4_f32(v, X, acc);
          }
        }
      }
    } else if (vec) {
      const int64_t vend = begin + ((end - begin) & ~int64_t(3));
      for (int64_t i = begin + 4 * threadIdx.x; i < vend; i += 4 * kMtThreads) {
        float4 v = load_g4(S.src[0], i, S.dtype);
        for (int q = 1; q < world; ++q) v = add4(v, load_g4(S.src[q], i, S.dtype));
        acc = sq_acc4_f32(store_g4(S.dst, i, S.dtype, v), X, acc);
      }
      for (int64_t i = vend + threadIdx.x; i < end; i += kMtThreads) {
        float v = load_g1(S.src[0], i, S.dtype);
        for (int q = 1; q < world; ++q) v = __fadd_rn(v, load_g1(S.src[q], i, S.dtype));
        acc = sqacc(X(store_g1(S.dst, i, S.dtype, v)), acc);
      }
    } else {
      for (int64_t i = begin + threadIdx.x; i < end; i += kMtThreads) {
        float v = load_g1(S.src[0], i, S.dtype);
        for (int q = 1; q < world; ++q) v = __fadd_rn(v, load_g1(S.src[q], i, S.dtype));
        acc = sqacc(X(store_g1(S.dst, i, S.dtype, v)), acc);
      }
    }
    const double tot = block_sum(acc, red);
    if (threadIdx.x == 0) A.partials[A.chunk_base + c] = tot;
  }
}

template <bool kDiv, int kW>
__global__ void __launch_bounds__(kMtThreads, 2) peer_reduce_kernel(const __grid_constant__ PeerReduceArgs A) {
  __shared__ double red[kMtThreads / 32];
  peer_reduce_chunks<kDiv, kW>(A, red);
}

// out[tensor[p]] = piece p's sum of squares (its partials summed as warp_sum_partials sums a tensor's), 0 elsewhere
__global__ void __launch_bounds__(1024) piece_sums_kernel(const __grid_constant__ PieceSumArgs A) {
  for (int t = static_cast<int>(threadIdx.x); t < A.n_tensors; t += static_cast<int>(blockDim.x)) A.out[t] = 0.0;
  __syncthreads();
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  for (int p = warp; p < A.n_pieces; p += static_cast<int>(blockDim.x >> 5)) {
    MO_CHECK(A.tensor[p] >= 0 && A.tensor[p] < A.n_tensors && A.chunk_start[p] <= A.chunk_start[p + 1]);
    const double s = warp_sum_partials(A.partials, A.chunk_start[p], A.chunk_start[p + 1], lane);
    if (lane == 0) A.out[A.tensor[p]] = s;
  }
}

// The global norm from every rank's per-tensor sums: per tensor, the ranks' sums added in rank order (a tensor held
// whole by one rank keeps its sum exactly), its norm rounded to fp32, then finish_total as norm_finalize_kernel.
__global__ void __launch_bounds__(1024) tensor_coef_kernel(const __grid_constant__ TensorCoefArgs A) {
  __shared__ float tnorm[kMaxFinalTensors];
  for (int t = static_cast<int>(threadIdx.x); t < A.n_tensors; t += static_cast<int>(blockDim.x)) {
    double s = 0.0;
    for (int r = 0; r < A.world; ++r) s += A.sums[static_cast<size_t>(r) * A.n_tensors + t];
    tnorm[t] = static_cast<float>(sqrt(s));
  }
  __syncthreads();
  if ((threadIdx.x >> 5) == 0) finish_total(tnorm, A.n_tensors, A.has_clip, A.max_norm, A.out, A.status,
                                            static_cast<int>(threadIdx.x & 31));
}

// ---------------------------------------------------------------------------------------------------------------
// AdamW, torch's single-tensor update in torch's rounding order:
//   p *= (1 - lr*wd)                      param.mul_(1 - lr*wd)
//   m  = lerp(m, g, 1-beta1)              exp_avg.lerp_(grad, 1-beta1)            (fused: m + w*(g-m))
//   v  = v*beta2; v = fma((1-b2)*g, g, v) exp_avg_sq.mul_(beta2).addcmul_(g, g, value=1-beta2)
//   d  = sqrt(v)/sqrt(bc2) + eps          (exp_avg_sq.sqrt() / bias_correction2_sqrt).add_(eps)
//   p += ((-step_size)*m) / d             param.addcdiv_(exp_avg, denom, value=-step_size)
struct AdamConsts {
  float lerp_w, one_minus_w, beta2, omb2, eps;
  int lerp_small;
};

// The Muon apply's scalars for this step (mote/train/muon.py:76-79, :97-99) when the lr is read on the device:
// decay = (lr*lr/lr_max if Muon-SW else lr) * wd in fp64, as the reference's Python floats; then fp32 casts of
// -lr and 1 - decay, as torch's scalar arguments.
struct ApplyScalars {
  float neg_lr, decay_mul;
  int has_decay;
};
__device__ __forceinline__ ApplyScalars apply_scalars(const double* lr_dev, double wd, double lr_max, float neg_lr,
                                                      float decay_mul, int has_decay) {
  if (lr_dev == nullptr) return ApplyScalars{neg_lr, decay_mul, has_decay};
  const double e = *lr_dev;
  const double d = wd == 0.0 ? 0.0 : (lr_max > 0.0 ? (e * e / lr_max) * wd : e * wd);
  return ApplyScalars{static_cast<float>(-e), static_cast<float>(1.0 - d), d != 0.0};
}

__device__ __forceinline__ float ema_lerp(float e, float p, const EmaConsts& E) {
  const float d = __fsub_rn(p, e);
  return E.small ? fmaf(E.w, d, e) : fmaf(-E.omw, d, p);
}

__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v, const AdamSeg& S, const AdamConsts& K) {
  if (S.has_decay) p = __fmul_rn(p, S.decay_mul);
  const float d = __fsub_rn(g, m);
  m = K.lerp_small ? fmaf(K.lerp_w, d, m) : fmaf(-K.one_minus_w, d, g);
  v = __fmul_rn(v, K.beta2);
  v = fmaf(__fmul_rn(K.omb2, g), g, v);
  const float den = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), S.bc2_sqrt), K.eps);
  p = __fadd_rn(p, __fdiv_rn(__fmul_rn(S.neg_step_size, m), den));
}

// kSmall: kAdamChunk work units with both of a thread's vectors loaded up front (launches too small to fill the
// GPU in kChunk units); else kChunk units walked one vector per thread at a time, which needs half the registers
// and so runs twice the blocks per SM. A separate instantiation each, so each gets its own register allocation. The
// division is a runtime flag here, not an instantiation: the division-free instantiation measured 7 % slower on 1e8
// elements (0.466 against 0.436 ms) with the same registers.
template <bool kSmall>
__global__ void __launch_bounds__(kMtThreads) adamw_kernel(const __grid_constant__ AdamArgs A) {
  const int total = A.chunk_start[A.n];
  const GradXform X{A.has_div, grad_div(A, A.has_div != 0), A.coef != nullptr, A.coef != nullptr ? *A.coef : 1.f};
  const AdamConsts K{A.lerp_w, A.one_minus_w, A.beta2, A.one_minus_beta2, A.eps, A.lerp_small};
  const double dstep = A.dstep != nullptr ? static_cast<double>(*A.dstep) : 0.0;
  int s_cur = -1;
  AdamSeg S;
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    if (s != s_cur) {   // the segment's scalars, recomputed only when the block moves to another tensor
      s_cur = s;
      S = A.seg[s];
      const double lr = S.lr_dev != nullptr ? *S.lr_dev : S.lr;   // this step's lr (device-read under a schedule)
      if (A.dstep != nullptr) {   // the host computes these in fp64 from its step count; the same formulas here
        const double bc1 = 1.0 - pow(A.beta1d, dstep);
        const double bc2 = 1.0 - pow(A.beta2d, dstep);
        S.neg_step_size = static_cast<float>(-(lr / bc1));
        S.bc2_sqrt = static_cast<float>(pow(bc2, 0.5));
      } else if (S.lr_dev != nullptr) {
        S.neg_step_size = static_cast<float>(-(lr / S.bc1));
      }
      if (S.lr_dev != nullptr) S.decay_mul = static_cast<float>(1.0 - lr * S.wd);
    }
    constexpr int kUnit = kSmall ? kAdamChunk : kChunk;
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kUnit;
    const int64_t end = min(begin + kUnit, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel);
    const bool vec = aligned16(S.p) && aligned16(S.m) && aligned16(S.v) && g_vec_ok(S.g, S.dtype) &&
                     (S.ema == nullptr || aligned16(S.ema));
    int64_t i0 = begin;
    if (kSmall && vec && end - begin == kAdamChunk) {   // a full unit: both vectors' loads go out before the first use
      float4 p[2], m[2], v[2], g[2], e[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int64_t i = begin + 4 * static_cast<int64_t>(threadIdx.x + k * kMtThreads);
        p[k] = *reinterpret_cast<const float4*>(S.p + i);
        m[k] = *reinterpret_cast<const float4*>(S.m + i);
        v[k] = *reinterpret_cast<const float4*>(S.v + i);
        g[k] = load_g4(S.g, i, S.dtype);
        if (S.ema != nullptr) e[k] = *reinterpret_cast<const float4*>(S.ema + i);
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int64_t i = begin + 4 * static_cast<int64_t>(threadIdx.x + k * kMtThreads);
        adam_elem(p[k].x, X(g[k].x), m[k].x, v[k].x, S, K);
        adam_elem(p[k].y, X(g[k].y), m[k].y, v[k].y, S, K);
        adam_elem(p[k].z, X(g[k].z), m[k].z, v[k].z, S, K);
        adam_elem(p[k].w, X(g[k].w), m[k].w, v[k].w, S, K);
        *reinterpret_cast<float4*>(S.p + i) = p[k];
        *reinterpret_cast<float4*>(S.m + i) = m[k];
        *reinterpret_cast<float4*>(S.v + i) = v[k];
        if (S.ema != nullptr) {
          e[k].x = ema_lerp(e[k].x, p[k].x, A.ema); e[k].y = ema_lerp(e[k].y, p[k].y, A.ema);
          e[k].z = ema_lerp(e[k].z, p[k].z, A.ema); e[k].w = ema_lerp(e[k].w, p[k].w, A.ema);
          *reinterpret_cast<float4*>(S.ema + i) = e[k];
        }
      }
      continue;
    }
    if (vec) {
      const int64_t vend = begin + ((end - begin) & ~int64_t(3));
      for (int64_t i = begin + 4 * threadIdx.x; i < vend; i += 4 * kMtThreads) {
        float4 p = *reinterpret_cast<float4*>(S.p + i);
        float4 m = *reinterpret_cast<float4*>(S.m + i);
        float4 v = *reinterpret_cast<float4*>(S.v + i);
        const float4 g = load_g4(S.g, i, S.dtype);
        adam_elem(p.x, X(g.x), m.x, v.x, S, K);
        adam_elem(p.y, X(g.y), m.y, v.y, S, K);
        adam_elem(p.z, X(g.z), m.z, v.z, S, K);
        adam_elem(p.w, X(g.w), m.w, v.w, S, K);
        *reinterpret_cast<float4*>(S.p + i) = p;
        *reinterpret_cast<float4*>(S.m + i) = m;
        *reinterpret_cast<float4*>(S.v + i) = v;
        if (S.ema != nullptr) {
          float4 e = *reinterpret_cast<float4*>(S.ema + i);
          e.x = ema_lerp(e.x, p.x, A.ema); e.y = ema_lerp(e.y, p.y, A.ema);
          e.z = ema_lerp(e.z, p.z, A.ema); e.w = ema_lerp(e.w, p.w, A.ema);
          *reinterpret_cast<float4*>(S.ema + i) = e;
        }
      }
      i0 = vend;
    }
    for (int64_t i = i0 + threadIdx.x; i < end; i += kMtThreads) {
      float p = S.p[i], m = S.m[i], v = S.v[i];
      adam_elem(p, X(load_g1(S.g, i, S.dtype)), m, v, S, K);
      S.p[i] = p; S.m[i] = m; S.v[i] = v;
      if (S.ema != nullptr) S.ema[i] = ema_lerp(S.ema[i], p, A.ema);
    }
  }
}

// torch's `step_t += 1` on a device step counter (fp32, exact for integer counts below 2^24)
__global__ void step_increment_kernel(float* step) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *step = *step + 1.0f;
}

// ---------------------------------------------------------------------------------------------------------------
// Muon momentum (muon.py:69-70): buf = buf*mom + g (two roundings); u = g + mom*buf (fused, torch's add(alpha=)).
// Writes buf and, per chunk, the sum of u^2 for the per-matrix Frobenius norm.
__device__ __forceinline__ float mom_elem(float g, float& buf, float mom, int nesterov) {
  buf = __fadd_rn(__fmul_rn(buf, mom), g);
  return nesterov ? fmaf(mom, buf, g) : buf;
}

// A full chunk with 16-byte aligned buf (and 8/16-byte aligned g) is processed in two halves of 32 elements per
// thread, with every load of a half issued before the first use (192 B in flight per thread for bf16 grads).
// kDiv: whether the grads are divided first. Without the division (and its slow path) the kernel fits four blocks
// per SM and runs at the copy bandwidth (c1: 165 -> 144 us); the dividing instantiation is compute-heavier (205 us).
template <bool kDiv>
__global__ void __launch_bounds__(kMtThreads, kDiv ? 1 : 4) muon_momentum_kernel(const __grid_constant__ MomArgs A) {
  __shared__ double red[kMtThreads / 32];
  const int total = A.chunk_start[A.n];
  const GradXform X{kDiv ? A.has_div : 0, grad_div(A, kDiv && A.has_div), A.coef != nullptr,
                    A.coef != nullptr ? *A.coef : 1.f};
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    const MomSeg& S = A.seg[s];
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kChunk;
    const int64_t end = min(begin + kChunk, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel);
    double acc = 0.0;
    int64_t i0 = begin;
    if (aligned16(S.buf) && g_vec_ok(S.g, S.dtype)) {
      if (end - begin == kChunk) {   // 4096 float4 of buf: 16 per thread, four quarters of 4, software-pipelined:
        float4* bp = reinterpret_cast<float4*>(S.buf + begin);   // quarter q+1's loads go out before quarter q's math
        float4 b[2][4], g[2][4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = threadIdx.x + k * kMtThreads;
          b[0][k] = bp[j];
          g[0][k] = load_g4(S.g, begin + 4 * static_cast<int64_t>(j), S.dtype);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int cur = q & 1;
          if (q + 1 < 4) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int j = threadIdx.x + ((q + 1) * 4 + k) * kMtThreads;
              b[cur ^ 1][k] = bp[j];
              g[cur ^ 1][k] = load_g4(S.g, begin + 4 * static_cast<int64_t>(j), S.dtype);
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float4& bb = b[cur][k];
            const float4& gg = g[cur][k];
            const float u0 = mom_elem(X(gg.x), bb.x, S.mom, S.nesterov);
            const float u1 = mom_elem(X(gg.y), bb.y, S.mom, S.nesterov);
            const float u2 = mom_elem(X(gg.z), bb.z, S.mom, S.nesterov);
            const float u3 = mom_elem(X(gg.w), bb.w, S.mom, S.nesterov);
            bp[threadIdx.x + (q * 4 + k) * kMtThreads] = bb;
            acc = sqacc(u0, acc); acc = sqacc(u1, acc); acc = sqacc(u2, acc); acc = sqacc(u3, acc);
          }
        }
        i0 = end;
      } else {
        const int64_t vend = begin + ((end - begin) & ~int64_t(3));
        for (int64_t i = begin + 4 * threadIdx.x; i < vend; i += 4 * kMtThreads) {
          float4 b = *reinterpret_cast<float4*>(S.buf + i);
          const float4 g = load_g4(S.g, i, S.dtype);
          const float u0 = mom_elem(X(g.x), b.x, S.mom, S.nesterov);
          const float u1 = mom_elem(X(g.y), b.y, S.mom, S.nesterov);
          const float u2 = mom_elem(X(g.z), b.z, S.mom, S.nesterov);
          const float u3 = mom_elem(X(g.w), b.w, S.mom, S.nesterov);
          *reinterpret_cast<float4*>(S.buf + i) = b;
          acc = sqacc(u0, acc); acc = sqacc(u1, acc); acc = sqacc(u2, acc); acc = sqacc(u3, acc);
        }
        i0 = vend;
      }
    }
    for (int64_t i = i0 + threadIdx.x; i < end; i += kMtThreads) {
      float b = S.buf[i];
      const float u = mom_elem(X(load_g1(S.g, i, S.dtype)), b, S.mom, S.nesterov);
      S.buf[i] = b;
      acc = sqacc(u, acc);
    }
    const double tot = block_sum(acc, red);
    if (threadIdx.x == 0) A.partials[A.chunk_base + c] = tot;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// den[m] = fp32(sqrt(sum of matrix m's partials)) + eps (muon.py:33: X.norm() + eps). One warp per matrix; lane l
// sums chunks l, l+32, ... in fp64, then a fixed xor tree: deterministic.
__global__ void __launch_bounds__(256) mat_denom_kernel(const __grid_constant__ DenomArgs A) {
  const int mat = blockIdx.x * 8 + static_cast<int>(threadIdx.x >> 5);
  if (mat >= A.n) return;
  const int lane = threadIdx.x & 31;
  MO_CHECK(A.chunk_start[mat] <= A.chunk_start[mat + 1]);
  const double s = warp_sum_partials(A.partials, A.chunk_start[mat], A.chunk_start[mat + 1], lane);
  if (lane == 0) A.den[A.base + mat] = __fadd_rn(static_cast<float>(sqrt(s)), A.eps);
}

// ---------------------------------------------------------------------------------------------------------------
// X0 = bf16(u / (||u||_F + eps)) for a matrix iterated as it is stored: a flat pass over 16K-element chunks, four
// quarters of 16 elements per thread with every load of a quarter issued before the first use. u is recomputed from
// the grad and the updated momentum buffer exactly as the momentum kernel computed it (direct mode: u = G).
__device__ __forceinline__ float flat_u(float g, float b, const FlatNormSeg& S, bool has_buf) {
  return has_buf ? (S.nesterov ? fmaf(S.mom, b, g) : b) : g;
}

// Four blocks per SM (64 registers) without the grads' division, three with it: the exact quotient's window test
// needs the room (five blocks spill; four measured 8 us faster at c1 than five).
template <bool kDiv>
__global__ void __launch_bounds__(kMtThreads, kDiv ? 3 : 4) ns_normalize_flat_kernel(const __grid_constant__ FlatNormArgs A) {
  const int total = A.chunk_start[A.n];
  const GradXform X{kDiv ? 1 : 0, grad_div(A, kDiv), A.coef != nullptr, A.coef != nullptr ? *A.coef : 1.f};
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    const FlatNormSeg& S = A.seg[s];
    const SharedDivisor den = shared_divisor(A.den[S.den_index]);
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kChunk;
    const int64_t end = min(begin + kChunk, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel);
    const bool has_buf = S.buf != nullptr;
    __nv_bfloat16* x = reinterpret_cast<__nv_bfloat16*>(S.x);
    int64_t i0 = begin;
    if (end - begin == kChunk && g_vec_ok(S.g, S.dtype) && (!has_buf || aligned16(S.buf)) && aligned8(x)) {
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float4 g[4], b[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t i = begin + 4 * static_cast<int64_t>(threadIdx.x + (h * 4 + k) * kMtThreads);
          g[k] = load_g4(S.g, i, S.dtype);
          b[k] = has_buf ? *reinterpret_cast<const float4*>(S.buf + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int64_t i = begin + 4 * static_cast<int64_t>(threadIdx.x + (h * 4 + k) * kMtThreads);
          const float u0 = flat_u(X(g[k].x), b[k].x, S, has_buf), u1 = flat_u(X(g[k].y), b[k].y, S, has_buf);
          const float u2 = flat_u(X(g[k].z), b[k].z, S, has_buf), u3 = flat_u(X(g[k].w), b[k].w, S, has_buf);
          const float4 q = den.div4_bounded(make_float4(u0, u1, u2, u3));   // |u| <= ||u|| < den
          *reinterpret_cast<uint2*>(x + i) = make_uint2(pack_bf16x2(q.x, q.y), pack_bf16x2(q.z, q.w));
        }
      }
      i0 = end;
    }
    for (int64_t i = i0 + threadIdx.x; i < end; i += kMtThreads) {
      const float u = flat_u(X(load_g1(S.g, i, S.dtype)), has_buf ? S.buf[i] : 0.f, S, has_buf);
      x[i] = __float2bfloat16_rn(den.div(u));
    }
  }
}

// The flat counterpart of ns_out_kernel: the Muon apply of muon.py:97-99 (p = p*(1-decay) if decay;
// p += -lr*(O*scale)) into the fp32 parameter, or a copy of the bf16 iterate to the output.
__global__ void __launch_bounds__(kMtThreads) ns_out_flat_kernel(const __grid_constant__ FlatOutArgs A) {
  __shared__ double red[kMtThreads / 32];
  const int total = A.chunk_start[A.n];
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    const FlatOutSeg& S = A.seg[s];
    double sq = 0.0;   // sum of the updated param's squares (norm tracking), fixed per-thread order
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kChunk;
    const int64_t end = min(begin + kChunk, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel);
    const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(S.x);
    int64_t i0 = begin;
    if (A.apply) {
      float* p = reinterpret_cast<float*>(S.out);
      const ApplyScalars K = apply_scalars(S.lr_dev, S.wd, S.lr_max, S.neg_lr, S.decay_mul, S.has_decay);
      if (end - begin == kChunk && aligned8(x) && aligned16(p) && (S.ema == nullptr || aligned16(S.ema))) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint2 w[8];
          float4 q[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int64_t i = begin + 4 * static_cast<int64_t>(threadIdx.x + (h * 8 + k) * kMtThreads);
            w[k] = *reinterpret_cast<const uint2*>(x + i);
            q[k] = *reinterpret_cast<const float4*>(p + i);
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int64_t i = begin + 4 * static_cast<int64_t>(threadIdx.x + (h * 8 + k) * kMtThreads);
            const float o[4] = {bf16_lo(w[k].x), bf16_hi(w[k].x), bf16_lo(w[k].y), bf16_hi(w[k].y)};
            float* qe = reinterpret_cast<float*>(&q[k]);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float v = qe[e];
              if (K.has_decay) v = __fmul_rn(v, K.decay_mul);
              qe[e] = fmaf(K.neg_lr, __fmul_rn(o[e], S.scale), v);
            }
            *reinterpret_cast<float4*>(p + i) = q[k];
            sq = sqacc(q[k].x, sq); sq = sqacc(q[k].y, sq);
            sq = sqacc(q[k].z, sq); sq = sqacc(q[k].w, sq);
            if (S.ema != nullptr) {   // the EMA follows the updated param in the same pass
              float4 e = *reinterpret_cast<float4*>(S.ema + i);
              e.x = ema_lerp(e.x, q[k].x, A.ema); e.y = ema_lerp(e.y, q[k].y, A.ema);
              e.z = ema_lerp(e.z, q[k].z, A.ema); e.w = ema_lerp(e.w, q[k].w, A.ema);
              *reinterpret_cast<float4*>(S.ema + i) = e;
            }
          }
        }
        i0 = end;
      }
      for (int64_t i = i0 + threadIdx.x; i < end; i += kMtThreads) {
        float v = p[i];
        if (K.has_decay) v = __fmul_rn(v, K.decay_mul);
        v = fmaf(K.neg_lr, __fmul_rn(__bfloat162float(x[i]), S.scale), v);
        p[i] = v;
        sq = sqacc(v, sq);
        if (S.ema != nullptr) S.ema[i] = ema_lerp(S.ema[i], v, A.ema);
      }
      if (S.partials != nullptr) {   // block-uniform: every thread of the block works on this chunk
        const double tot = block_sum(sq, red);
        if (threadIdx.x == 0) S.partials[c - A.chunk_start[s]] = tot;
      }
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(S.out);
      if (end - begin == kChunk && aligned16(x) && aligned16(o)) {   // 2048 16-byte vectors: 8 per thread
        const uint4* xs = reinterpret_cast<const uint4*>(x + begin);
        uint4* os = reinterpret_cast<uint4*>(o + begin);
        uint4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = xs[threadIdx.x + k * kMtThreads];
#pragma unroll
        for (int k = 0; k < 8; ++k) os[threadIdx.x + k * kMtThreads] = v[k];
        i0 = end;
      }
      for (int64_t i = i0 + threadIdx.x; i < end; i += kMtThreads) o[i] = x[i];
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// Tiled transpose helpers of the Newton-Schulz normalisation and the final apply: a 64 x 64 tile is read with 4
// consecutive elements per thread along the source's rows and written with 4 consecutive elements along the
// destination's rows; when the two orientations differ, the tile goes through shared memory.
constexpr int kTileRowsPerPass = kMtThreads / (kNormTile / 4);   // 16

// X0 = bf16(u / (||u||_F + eps)), transposed when the matrix has more rows than columns, zero padded.
// grid: (tiles of the largest matrix, matrices). u is recomputed from the grad and the updated momentum buffer
// exactly as the momentum kernel computed it (momentum mode), or read from G (direct mode, buf == null).
// kDiv: whether the grads are divided first (the division's slow path is compiled only where used); without it the
// kernel fits five blocks per SM.
template <bool kDiv>
__global__ void __launch_bounds__(kMtThreads, kDiv ? 1 : 5) ns_normalize_kernel(const __grid_constant__ NormArgs A) {
  __shared__ float tile[kNormTile][kNormTile + 1];
  const NormMat& M = A.mat[blockIdx.y];
  if (static_cast<int>(blockIdx.x) >= M.tiles) return;
  const int ti = blockIdx.x / M.tiles_x, tj = blockIdx.x % M.tiles_x;
  const int i0 = ti * kNormTile, j0 = tj * kNormTile;   // destination tile origin (X rows i, cols j)
  MO_CHECK(i0 < M.m_pad && j0 < M.n_pad);
  const SharedDivisor den = shared_divisor(A.den[M.den_index]);
  const GradXform X{kDiv ? 1 : 0, grad_div(A, kDiv), A.coef != nullptr, A.coef != nullptr ? *A.coef : 1.f};
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;   // 16 x 16 threads, 4 columns each
  const int mv = M.transposed ? M.cols : M.rows;
  const int nv = M.transposed ? M.rows : M.cols;
  const int sr0 = M.transposed ? j0 : i0, sc0 = M.transposed ? i0 : j0;
  const bool vec = (M.cols % 4 == 0) && aligned16(M.buf == nullptr ? M.g : M.buf) && g_vec_ok(M.g, M.dtype);
  float v[4][4];
  if (vec && sr0 + kNormTile <= M.rows && sc0 + kNormTile <= M.cols) {
    // interior tile: all eight 16-byte loads of the thread are issued before the first use
    float4 g4[4], b4[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      g4[k] = load_g4(M.g, static_cast<int64_t>(sr0 + ty + kTileRowsPerPass * k) * M.cols + sc0 + 4 * tx, M.dtype);
    if (M.buf != nullptr) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        b4[k] = *reinterpret_cast<const float4*>(
            M.buf + static_cast<int64_t>(sr0 + ty + kTileRowsPerPass * k) * M.cols + sc0 + 4 * tx);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float* gv = reinterpret_cast<const float*>(&g4[k]);
      const float* bv = reinterpret_cast<const float*>(&b4[k]);
      float u[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        u[e] = X(gv[e]);
        if (M.buf != nullptr) u[e] = M.nesterov ? fmaf(M.mom, bv[e], u[e]) : bv[e];
      }
      const float4 q = den.div4_bounded(make_float4(u[0], u[1], u[2], u[3]));   // |u| <= ||u|| < den
      v[k][0] = bf16_round_f(q.x);
      v[k][1] = bf16_round_f(q.y);
      v[k][2] = bf16_round_f(q.z);
      v[k][3] = bf16_round_f(q.w);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {   // source rows sr0 + ty + 16k, columns sc0 + 4tx .. +3
      const int sr = sr0 + ty + kTileRowsPerPass * k, sc = sc0 + 4 * tx;
      const int64_t idx = static_cast<int64_t>(sr) * M.cols + sc;
      float gv[4] = {0.f, 0.f, 0.f, 0.f}, bv[4] = {0.f, 0.f, 0.f, 0.f};
      if (sr < M.rows) {
        if (vec && sc + 3 < M.cols) {
          const float4 g4 = load_g4(M.g, idx, M.dtype);
          gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
          if (M.buf != nullptr) {
            const float4 b4 = *reinterpret_cast<const float4*>(M.buf + idx);
            bv[0] = b4.x; bv[1] = b4.y; bv[2] = b4.z; bv[3] = b4.w;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (sc + e < M.cols) {
              gv[e] = load_g1(M.g, idx + e, M.dtype);
              if (M.buf != nullptr) bv[e] = M.buf[idx + e];
            }
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float u = X(gv[e]);
        if (M.buf != nullptr) u = M.nesterov ? fmaf(M.mom, bv[e], u) : bv[e];
        const bool ok = sr < M.rows && sc + e < M.cols;
        v[k][e] = ok ? bf16_round_f(den.div(u)) : 0.f;
      }
    }
  }
  __nv_bfloat16* x = reinterpret_cast<__nv_bfloat16*>(M.x);
  if (M.transposed) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) tile[ty + kTileRowsPerPass * k][4 * tx + e] = v[k][e];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) v[k][e] = tile[4 * tx + e][ty + kTileRowsPerPass * k];
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {   // destination rows i0 + ty + 16k, columns j0 + 4tx .. +3 (m_pad, n_pad: x8)
    const int i = i0 + ty + kTileRowsPerPass * k, j = j0 + 4 * tx;
    if (i < M.m_pad && j < M.n_pad) {
      float w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) w[e] = (i < mv && j + e < nv) ? v[k][e] : 0.f;
      uint2 pk = make_uint2(pack_bf16x2(w[0], w[1]), pack_bf16x2(w[2], w[3]));
      *reinterpret_cast<uint2*>(x + static_cast<int64_t>(i) * M.n_pad + j) = pk;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// The final iterate back to the caller's orientation: out[r][c] = X[c][r] (transposed) or X[r][c]; or, in apply mode,
// the Muon apply of muon.py:97-99 into the fp32 parameter: p = p*(1-decay) (if decay); p += -lr*(O*scale).
// kEma: whether any matrix of the launch has an EMA; the instantiation without one needs 43 registers instead of
// 61 and runs five blocks per SM instead of four.
template <bool kEma>
__global__ void __launch_bounds__(kMtThreads, kEma ? 1 : 5) ns_out_kernel(const __grid_constant__ OutArgs A) {
  __shared__ float tile[kNormTile][kNormTile + 1];
  const OutMat& M = A.mat[blockIdx.y];
  float* const ema = kEma ? M.ema : nullptr;
  if (static_cast<int>(blockIdx.x) >= M.tiles) return;
  const int ti = blockIdx.x / M.tiles_x, tj = blockIdx.x % M.tiles_x;
  const int r0 = ti * kNormTile, c0 = tj * kNormTile;      // output tile origin (rows r, cols c of R x C)
  MO_CHECK(r0 < M.rows && c0 < M.cols);
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(M.x);
  const int xr0 = M.transposed ? c0 : r0, xc0 = M.transposed ? r0 : c0;
  const bool vec = (M.cols % 4 == 0) && aligned16(M.out) && (ema == nullptr || aligned16(ema));
  const ApplyScalars K = apply_scalars(A.apply ? M.lr_dev : nullptr, M.wd, M.lr_max, M.neg_lr, M.decay_mul, M.has_decay);
  // interior tile of an apply: the param (and EMA) loads go out first, ahead of the X loads and the transpose
  const bool pre = A.apply && vec && r0 + kNormTile <= M.rows && c0 + kNormTile <= M.cols;
  float4 pp[4], pe[4];
  if (pre) {
    const float* p = reinterpret_cast<const float*>(M.out);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      pp[k] = *reinterpret_cast<const float4*>(p + static_cast<int64_t>(r0 + ty + kTileRowsPerPass * k) * M.cols + c0 + 4 * tx);
    if (ema != nullptr) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        pe[k] = *reinterpret_cast<const float4*>(
            ema + static_cast<int64_t>(r0 + ty + kTileRowsPerPass * k) * M.cols + c0 + 4 * tx);
    }
  }
  float v[4][4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {   // X rows xr0 + ty + 16k, columns xc0 + 4tx .. +3 (n_pad is a multiple of 8)
    const int xr = xr0 + ty + kTileRowsPerPass * k, xc = xc0 + 4 * tx;
    if (xr < M.m_pad && xc < M.n_pad) {
      const uint2 w = *reinterpret_cast<const uint2*>(x + static_cast<int64_t>(xr) * M.n_pad + xc);
      v[k][0] = bf16_lo(w.x); v[k][1] = bf16_hi(w.x); v[k][2] = bf16_lo(w.y); v[k][3] = bf16_hi(w.y);
    } else {
      v[k][0] = v[k][1] = v[k][2] = v[k][3] = 0.f;
    }
  }
  if (M.transposed) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) tile[ty + kTileRowsPerPass * k][4 * tx + e] = v[k][e];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) v[k][e] = tile[4 * tx + e][ty + kTileRowsPerPass * k];
  }
  double sq = 0.0;   // apply mode: sum of the updated param's squares over this thread's elements
#pragma unroll
  for (int k = 0; k < 4; ++k) {   // output rows r0 + ty + 16k, columns c0 + 4tx .. +3
    const int orow = r0 + ty + kTileRowsPerPass * k, ocol = c0 + 4 * tx;
    if (orow >= M.rows || ocol >= M.cols) continue;
    const int64_t idx = static_cast<int64_t>(orow) * M.cols + ocol;
    if (A.apply) {
      float* p = reinterpret_cast<float*>(M.out);
      if (vec) {
        float4 pv = pre ? pp[k] : *reinterpret_cast<float4*>(p + idx);
        float* pf = reinterpret_cast<float*>(&pv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float q = pf[e];
          if (K.has_decay) q = __fmul_rn(q, K.decay_mul);
          pf[e] = fmaf(K.neg_lr, __fmul_rn(v[k][e], M.scale), q);
        }
        *reinterpret_cast<float4*>(p + idx) = pv;
        sq = sqacc(pv.x, sq); sq = sqacc(pv.y, sq); sq = sqacc(pv.z, sq); sq = sqacc(pv.w, sq);
        if (ema != nullptr) {
          float4 ev = pre ? pe[k] : *reinterpret_cast<float4*>(ema + idx);
          ev.x = ema_lerp(ev.x, pv.x, A.ema); ev.y = ema_lerp(ev.y, pv.y, A.ema);
          ev.z = ema_lerp(ev.z, pv.z, A.ema); ev.w = ema_lerp(ev.w, pv.w, A.ema);
          *reinterpret_cast<float4*>(ema + idx) = ev;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (ocol + e < M.cols) {
            float q = p[idx + e];
            if (K.has_decay) q = __fmul_rn(q, K.decay_mul);
            q = fmaf(K.neg_lr, __fmul_rn(v[k][e], M.scale), q);
            p[idx + e] = q;
            sq = sqacc(q, sq);
            if (ema != nullptr) ema[idx + e] = ema_lerp(ema[idx + e], q, A.ema);
          }
      }
    } else {
      __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(M.out);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (ocol + e < M.cols) o[idx + e] = __float2bfloat16_rn(v[k][e]);
    }
  }
  if (A.apply && M.partials != nullptr) {   // block-uniform (one matrix per grid row)
    __shared__ double red[kMtThreads / 32];
    const double tot = block_sum(sq, red);
    if (threadIdx.x == 0) M.partials[blockIdx.x] = tot;
  }
}

// ---------------------------------------------------------------------------------------------------------------
// g *= coef in place (the scaling half of clip_grad_norm_)
__global__ void __launch_bounds__(kMtThreads) clip_scale_kernel(const __grid_constant__ ScaleArgs A) {
  const int total = A.chunk_start[A.n];
  const float coef = *A.coef;
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    const SumsqSeg& S = A.seg[s];
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kChunk;
    const int64_t end = min(begin + kChunk, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel);
    for (int64_t i = begin + threadIdx.x; i < end; i += kMtThreads) {
      if (S.dtype == kBF16) {
        __nv_bfloat16* g = reinterpret_cast<__nv_bfloat16*>(const_cast<void*>(S.g));
        g[i] = __float2bfloat16_rn(__fmul_rn(__bfloat162float(g[i]), coef));
      } else {
        float* g = reinterpret_cast<float*>(const_cast<void*>(S.g));
        g[i] = __fmul_rn(g[i], coef);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// ema = lerp(ema, p, w) over a segment list (torch._foreach_lerp_, train.py:950-953), torch's rounding as ema_lerp.
// A full aligned chunk goes in four quarters of four 16-byte vectors per thread, each quarter's eight loads issued
// before its math.
__global__ void __launch_bounds__(kMtThreads) ema_lerp_kernel(const __grid_constant__ LerpArgs A) {
  const int total = A.chunk_start[A.n];
  for (int c = blockIdx.x; c < total; c += gridDim.x) {
    const int s = find_seg(A.chunk_start, A.n, c);
    const LerpSeg& S = A.seg[s];
    const int64_t begin = static_cast<int64_t>(c - A.chunk_start[s]) * kChunk;
    const int64_t end = min(begin + kChunk, S.numel);
    MO_CHECK(s >= 0 && s < A.n && begin >= 0 && begin < S.numel);
    int64_t i0 = begin;
    if (end - begin == kChunk && aligned16(S.ema) && aligned16(S.p)) {
      float4* ep = reinterpret_cast<float4*>(S.ema + begin);
      const float4* pp = reinterpret_cast<const float4*>(S.p + begin);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 e[4], p[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int j = threadIdx.x + (q * 4 + k) * kMtThreads;
          e[k] = ep[j];
          p[k] = pp[j];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          e[k].x = ema_lerp(e[k].x, p[k].x, A.ema); e[k].y = ema_lerp(e[k].y, p[k].y, A.ema);
          e[k].z = ema_lerp(e[k].z, p[k].z, A.ema); e[k].w = ema_lerp(e[k].w, p[k].w, A.ema);
          ep[threadIdx.x + (q * 4 + k) * kMtThreads] = e[k];
        }
      }
      i0 = end;
    }
    for (int64_t i = i0 + threadIdx.x; i < end; i += kMtThreads) S.ema[i] = ema_lerp(S.ema[i], S.p[i], A.ema);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// MoESwiGLU.update_bias (mote/model/moe.py:147-159) for every MoE layer of the model in one launch, one block per
// layer, fp32 tensor ops as the reference:
//   if load.sum() <= 0: return
//   e = (load.mean() - load) / load.mean().clamp_min(1e-9); sgn = sign(e)   (sign(NaN) = 0, as torch)
//   bias += fp32(gamma) * (sgn - sgn.mean()); load.zero_()
// The loads are token counts (integers), so their sum, formed in fp64 and rounded once, is the reference's fp32 sum
// in any order; the sum of the signs is an exact integer. No host round trip: the reference's `load.sum() <= 0`
// test becomes a per-block branch.
__global__ void __launch_bounds__(kMtThreads) moe_bias_kernel(const __grid_constant__ MoeBiasArgs A) {
  __shared__ double red_d[kMtThreads / 32];
  __shared__ int red_i[kMtThreads / 32];
  __shared__ float sh_mean;
  __shared__ int sh_skip, sh_count;
  const MoeLayer& L = A.layer[blockIdx.x];
  const int E = L.experts;
  MO_CHECK(static_cast<int>(blockIdx.x) < A.n && E > 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double s = 0.0;
  for (int i = threadIdx.x; i < E; i += kMtThreads) s += static_cast<double>(L.load[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o);
  if (lane == 0) red_d[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kMtThreads / 32; ++w) t += red_d[w];
    const float total = static_cast<float>(t);
    sh_skip = total <= 0.f;   // a NaN sum goes on, as `load.sum() <= 0` is false for it
    sh_mean = __fdiv_rn(total, static_cast<float>(E));
  }
  __syncthreads();
  if (sh_skip) return;
  const float mean = sh_mean;
  const float den = mean < 1e-9f ? 1e-9f : mean;   // clamp_min keeps a NaN
  int cnt = 0;
  for (int i = threadIdx.x; i < E; i += kMtThreads) {
    const float e = __fdiv_rn(__fsub_rn(mean, L.load[i]), den);
    cnt += (e > 0.f) - (e < 0.f);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_down_sync(0xffffffffu, cnt, o);
  if (lane == 0) red_i[warp] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < kMtThreads / 32; ++w) t += red_i[w];
    sh_count = t;
  }
  __syncthreads();
  const float sgn_mean = __fdiv_rn(static_cast<float>(sh_count), static_cast<float>(E));
  for (int i = threadIdx.x; i < E; i += kMtThreads) {   // each thread rewrites only the elements it read above
    const float e = __fdiv_rn(__fsub_rn(mean, L.load[i]), den);
    const float sgn = static_cast<float>((e > 0.f) - (e < 0.f));
    L.bias[i] = __fadd_rn(L.bias[i], __fmul_rn(L.gamma, __fsub_rn(sgn, sgn_mean)));
    L.load[i] = 0.f;
  }
}

}  // namespace moteopt
