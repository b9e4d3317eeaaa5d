// C-ABI entry points of the optimizer step (include/moteopt.h): argument checking, workspace layout, tensor-map
// encoding (cached per workspace and shape group) and the launch sequence. No device memory is allocated here.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "moteopt.h"
#include "mt_kernels.cuh"
#include "ns_gemm.cuh"

using namespace moteopt;

namespace {

thread_local std::string t_err;

int fail(int code, const std::string& msg) {
  t_err = msg;
  return code;
}

#define MO_CUDA(expr)                                                                          \
  do {                                                                                         \
    cudaError_t e_ = (expr);                                                                   \
    if (e_ != cudaSuccess) return fail(MOTEOPT_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

std::atomic<unsigned long long> g_launches{0};
// The persistent launch takes an iteration's matrices in two runs (each through all three phases) once an iteration
// is at least kNsChunkWaves waves of tiles: c1 (32 waves) 1.44 -> 1.39 ms, the same bits; three runs gave 1.40 ms,
// four 1.46 ms (the runs' phases get too short to keep every pair busy past their dependency waits), and two runs of
// half of c1 (a 2-GPU rank's share, 16 waves) 0.76 against 0.71 ms for one.
constexpr int kNsChunkWaves = 24;
std::atomic<int> g_ns_persistent{-1};
std::atomic<int> g_ns_tall{1};   // tall matrices iterated as stored (moteopt_ns_set_tall): 1, or 0 = transposed   // Newton-Schulz launch mode (moteopt_ns_set_persistent): 1, 0, or -1 = auto
// Auto mode: one persistent launch while an iteration is at most this many waves of CTA-pair tiles; above it the
// per-phase launches' ramps are amortised and their leaner tiles win (measured: c1 at 32 waves favours the
// persistent launch, c2 at 197 waves the per-phase launches by ~10 %).
constexpr int kPersistentMaxWaves = 48;
thread_local cudaEvent_t t_ns_ev[2] = {nullptr, nullptr};

#define MO_LAUNCHED(what)                                                                      \
  do {                                                                                         \
    g_launches.fetch_add(1, std::memory_order_relaxed);                                       \
    cudaError_t e_ = cudaGetLastError();                                                       \
    if (e_ != cudaSuccess) return fail(MOTEOPT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define MO_TRY(expr)            \
  do {                          \
    int r_ = (expr);            \
    if (r_ != MOTEOPT_OK) return r_; \
  } while (0)

constexpr size_t kHeaderBytes = 256;
struct Header {
  int status;
  float norm;
  float coef;
  int pad;
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------------------------------------------
// per-device setup
struct DeviceState {
  bool ready = false;
  int sms = 0;
  int pairs = 0;   // co-resident CTA pairs of the 2-CTA Newton-Schulz kernel
};
std::mutex g_mu;
DeviceState g_dev[64];

int device_setup(int* sms) {
  int dev = 0;
  MO_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MOTEOPT_ERR_DEVICE, "device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    int major = 0, minor = 0, count = 0;
    MO_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
    MO_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
    MO_CUDA(cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev));
    if (major != 10 || minor != 0)
      return fail(MOTEOPT_ERR_DEVICE, "libmoteopt is built for sm_100a (B200); device " + std::to_string(dev) +
                                          " is sm_" + std::to_string(major) + std::to_string(minor));
    MO_CUDA(cudaFuncSetAttribute(ns::ns_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ns::kSmemBytes));
    MO_CUDA(cudaFuncSetAttribute(ns::ns_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ns::kSmemBytes));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (count / 2), 1, 1);
    cfg.blockDim = dim3(ns::kThreads, 1, 1);
    cfg.dynamicSmemBytes = ns::kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    MO_CUDA(cudaOccupancyMaxActiveClusters(&clusters, ns::ns_gemm_kernel<false>, &cfg));
    int clusters_gram = 0;
    MO_CUDA(cudaOccupancyMaxActiveClusters(&clusters_gram, ns::ns_gemm_kernel<true>, &cfg));
    clusters = std::min(clusters, clusters_gram);
    if (clusters < 1) return fail(MOTEOPT_ERR_DEVICE, "the 2-CTA Newton-Schulz kernel cannot be resident on this device");
    d.sms = count;
    d.pairs = clusters;
    d.ready = true;
  }
  *sms = d.sms;
  return MOTEOPT_OK;
}

int device_pairs() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  return std::max(1, g_dev[dev].pairs);
}

int device_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  return std::max(1, g_dev[dev].sms);
}

// ---------------------------------------------------------------------------------------------------------------
// tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

typedef CUresult (*AddrRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);
AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(p);
  });
  return fn;
}

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 3-D bf16 tensor [depth][outer][inner], row-major, swizzled box {box_inner, box_outer, 1}
int make_map(CUtensorMap* m, void* base, uint64_t inner, uint64_t outer, uint64_t depth, uint32_t box_inner,
             uint32_t box_outer, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(MOTEOPT_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {inner, outer, depth};
  cuuint64_t strides[2] = {inner * 2, inner * outer * 2};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MOTEOPT_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return MOTEOPT_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// Newton-Schulz batch layout
struct MatRef {
  int src;     // Muon param index (step mode) or 0 (direct mode)
  int slice;   // matrix index inside a 3-D stack / the batch
};

struct GroupPlan {
  int rows, cols;          // source matrix dims (R x C)
  int transposed;          // R > C
  int tall = 0;            // R > C iterated as stored: X is [count][R][C] (m = C, n = R), no transposing passes
  int mv, nv, m, n;        // X dims: valid and padded to multiples of 8
  std::vector<MatRef> mats;
  size_t off_x0 = 0, off_x1 = 0, off_a = 0, off_b = 0;
  // The opt-in Gram variant (moteopt_muon_config::ns_variant 1) on a matrix whose long side is at least twice its
  // short one: X0 in, the result in X1; A holds R, B holds B, and the m x m buffers T, Q0, Q1 come in addition.
  bool gram = false;
  size_t off_t = 0, off_q0 = 0, off_q1 = 0;
};

// The X buffer (0: X0, 1: X1) that holds a group's final iterate after `steps` Newton-Schulz iterations.
int out_buffer(const GroupPlan& g, int steps) { return steps == 0 ? 0 : (g.gram ? 1 : (steps & 1)); }

struct Layout {
  std::vector<GroupPlan> groups;          // Newton-Schulz shape groups, in launch order
  std::vector<int> mat_chunk_start;       // per matrix (group-major order): sum-of-squares chunk prefix
  std::vector<int> norm_tensor_chunk_start;
  std::vector<int> param_apply_start;     // per Muon param: its apply-pass partials (norm tracking), in slice order
  size_t off_norm = 0, off_mom = 0, off_den = 0, off_done = 0, off_apply = 0, bytes = 0;
};

constexpr int kMaxMatsPerGroup = ns::kMaxApply;

struct ShapeKey {
  int64_t rows, cols;
  bool operator<(const ShapeKey& o) const { return std::tie(rows, cols) < std::tie(o.rows, o.cols); }
};

// shapes: per source (batch, rows, cols); norm_numels: the tensors of the global grad norm (may be empty)
// Partials one matrix's apply pass writes: one per 16K-element chunk when the matrix is iterated as stored (no
// transpose, no padding: the flat kernel), else one per 64 x 64 tile (the tiled kernel).
int64_t apply_partials_per_slice(int64_t r, int64_t c, bool flat) {
  return flat ? cdiv(r * c, kChunk) : cdiv(c, kNormTile) * cdiv(r, kNormTile);
}

// A matrix is iterated as it is stored when it needs no padding and either has no more rows than columns or is
// iterated tall (its X0 / final iterate then has the parameter's own layout and the normalise / apply are flat
// passes).
bool stored_as_iterated(const GroupPlan& g) {
  return g.tall || (!g.transposed && g.m == g.rows && g.n == g.cols);
}

int build_layout(const std::vector<std::tuple<int64_t, int64_t, int64_t>>& shapes, const std::vector<int64_t>& norm_numels,
                 int ns_steps, Layout* L, int ns_variant = 0) {
  if (ns_variant != 0 && ns_variant != 1) return fail(MOTEOPT_ERR_INVALID, "ns_variant must be 0 or 1");
  L->groups.clear();
  std::map<ShapeKey, std::vector<MatRef>> by_shape;
  std::vector<ShapeKey> order;
  for (size_t s = 0; s < shapes.size(); ++s) {
    const int64_t b = std::get<0>(shapes[s]), r = std::get<1>(shapes[s]), c = std::get<2>(shapes[s]);
    if (b < 1 || r < 1 || c < 1) return fail(MOTEOPT_ERR_INVALID, "Muon matrices must have batch, rows, cols >= 1");
    if (r > (1 << 20) || c > (1 << 20)) return fail(MOTEOPT_ERR_INVALID, "matrix dimension above 2^20");
    const ShapeKey k{r, c};
    if (!by_shape.count(k)) order.push_back(k);
    auto& v = by_shape[k];
    for (int64_t e = 0; e < b; ++e) v.push_back(MatRef{static_cast<int>(s), static_cast<int>(e)});
  }
  for (const ShapeKey& k : order) {
    const auto& all = by_shape[k];
    for (size_t start = 0; start < all.size(); start += kMaxMatsPerGroup) {
      GroupPlan g;
      g.rows = static_cast<int>(k.rows);
      g.cols = static_cast<int>(k.cols);
      g.transposed = k.rows > k.cols;
      g.mv = g.transposed ? g.cols : g.rows;
      g.nv = g.transposed ? g.rows : g.cols;
      g.m = static_cast<int>(align_up(g.mv, 8));
      g.n = static_cast<int>(align_up(g.nv, 8));
      g.gram = ns_variant == 1 && ns_steps > 0 && g.nv >= 2 * g.mv;
      // a tall matrix without padding is iterated as stored (the same products in the same order as its transpose's
      // iteration), except under the Gram variant, whose phases read X row-wise
      g.tall = g.transposed && !g.gram && k.rows % 8 == 0 && k.cols % 8 == 0 &&
               g_ns_tall.load(std::memory_order_relaxed) != 0;
      g.mats.assign(all.begin() + start, all.begin() + std::min(all.size(), start + kMaxMatsPerGroup));
      L->groups.push_back(std::move(g));
    }
  }
  // largest Gram contraction first: a longest-processing-time order for the static tile schedule
  std::stable_sort(L->groups.begin(), L->groups.end(), [](const GroupPlan& a, const GroupPlan& b) {
    return static_cast<int64_t>(a.m) * a.n > static_cast<int64_t>(b.m) * b.n;
  });
  // chunk prefixes
  L->mat_chunk_start.assign(1, 0);
  for (const GroupPlan& g : L->groups)
    for (size_t i = 0; i < g.mats.size(); ++i)
      L->mat_chunk_start.push_back(L->mat_chunk_start.back() +
                                   static_cast<int>(cdiv(static_cast<int64_t>(g.rows) * g.cols, kChunk)));
  L->norm_tensor_chunk_start.assign(1, 0);
  for (int64_t n : norm_numels) {
    if (n < 0) return fail(MOTEOPT_ERR_INVALID, "negative numel");
    L->norm_tensor_chunk_start.push_back(L->norm_tensor_chunk_start.back() + static_cast<int>(cdiv(n, kChunk)));
  }
  size_t off = kHeaderBytes;
  L->off_norm = off;
  off = align_up(off + sizeof(double) * static_cast<size_t>(L->norm_tensor_chunk_start.back()), 256);
  L->off_mom = off;
  off = align_up(off + sizeof(double) * static_cast<size_t>(L->mat_chunk_start.back()), 256);
  L->off_den = off;
  off = align_up(off + 4 * (L->mat_chunk_start.size() - 1), 256);
  L->off_done = off;   // persistent Newton-Schulz: per matrix of a launch set and phase, completion arrivals
  off = align_up(off + 4 * 3 * static_cast<size_t>(ns::kMaxApply), 256);
  std::map<ShapeKey, bool> flat_of;   // every group of a shape is iterated the same way
  for (const GroupPlan& g : L->groups) flat_of[ShapeKey{g.rows, g.cols}] = stored_as_iterated(g);
  L->param_apply_start.assign(1, 0);   // the apply pass's sums of squares, contiguous per Muon param
  for (const auto& sh : shapes) {
    const int64_t b = std::get<0>(sh), r = std::get<1>(sh), c = std::get<2>(sh);
    L->param_apply_start.push_back(L->param_apply_start.back() +
                                   static_cast<int>(b * apply_partials_per_slice(r, c, flat_of[ShapeKey{r, c}])));
  }
  L->off_apply = off;
  off = align_up(off + sizeof(double) * static_cast<size_t>(L->param_apply_start.back()), 1024);
  for (GroupPlan& g : L->groups) {
    const size_t cnt = g.mats.size();
    const size_t xb = cnt * g.m * g.n * 2, ab = cnt * g.m * g.m * 2;
    g.off_x0 = off;
    off = align_up(off + xb, 1024);
    if (ns_steps > 0) {
      g.off_x1 = off;
      off = align_up(off + xb, 1024);
      g.off_a = off;
      off = align_up(off + ab, 1024);
      g.off_b = off;
      off = align_up(off + ab, 1024);
      if (g.gram) {
        g.off_t = off;
        off = align_up(off + ab, 1024);
        g.off_q0 = off;
        off = align_up(off + ab, 1024);
        g.off_q1 = off;
        off = align_up(off + ab, 1024);
      }
    }
  }
  L->bytes = off;
  return MOTEOPT_OK;
}

// cache of encoded tensor maps, keyed by the group's buffers and geometry
struct MapKey {
  uintptr_t x0, x1, a, b;
  int m, n, count, dev, tall;
  bool operator<(const MapKey& o) const {
    return std::tie(x0, x1, a, b, m, n, count, dev, tall) <
           std::tie(o.x0, o.x1, o.a, o.b, o.m, o.n, o.count, o.dev, o.tall);
  }
};
struct MapSet {
  CUtensorMap xk[2], xmn[2], ak, bk, amn, bmn, xe[2], ae, be;
};
std::mutex g_map_mu;
std::map<MapKey, MapSet> g_maps;

int group_maps(char* ws, const GroupPlan& g, MapSet* out) {
  int dev = 0;
  MO_CUDA(cudaGetDevice(&dev));
  const int cnt = static_cast<int>(g.mats.size());
  MapKey key{reinterpret_cast<uintptr_t>(ws + g.off_x0), reinterpret_cast<uintptr_t>(ws + g.off_x1),
             reinterpret_cast<uintptr_t>(ws + g.off_a), reinterpret_cast<uintptr_t>(ws + g.off_b), g.m, g.n, cnt, dev,
             g.tall};
  std::lock_guard<std::mutex> lk(g_map_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return MOTEOPT_OK;
  }
  MapSet s;
  std::memset(&s, 0, sizeof(s));
  void* x[2] = {ws + g.off_x0, ws + g.off_x1};
  const int xin = g.tall ? g.m : g.n, xout = g.tall ? g.n : g.m;   // X is [count][xout][xin]
  for (int k = 0; k < 2; ++k) {
    MO_TRY(make_map(&s.xk[k], x[k], xin, xout, cnt, ns::BK, ns::HM));
    MO_TRY(make_map(&s.xmn[k], x[k], xin, xout, cnt, 64, ns::BK));
  }
  MO_TRY(make_map(&s.ak, ws + g.off_a, g.m, g.m, cnt, ns::BK, ns::HM));
  MO_TRY(make_map(&s.bk, ws + g.off_b, g.m, g.m, cnt, ns::BK, ns::HM));
  MO_TRY(make_map(&s.amn, ws + g.off_a, g.m, g.m, cnt, 64, ns::BK));
  MO_TRY(make_map(&s.bmn, ws + g.off_b, g.m, g.m, cnt, 64, ns::BK));
  for (int k = 0; k < 2; ++k)
    MO_TRY(make_map(&s.xe[k], x[k], xin, xout, cnt, ns::EPI_TILE, ns::EPI_TILE, CU_TENSOR_MAP_SWIZZLE_64B));
  MO_TRY(make_map(&s.ae, ws + g.off_a, g.m, g.m, cnt, ns::EPI_TILE, ns::EPI_TILE, CU_TENSOR_MAP_SWIZZLE_64B));
  MO_TRY(make_map(&s.be, ws + g.off_b, g.m, g.m, cnt, ns::EPI_TILE, ns::EPI_TILE, CU_TENSOR_MAP_SWIZZLE_64B));
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps[key] = s;
  *out = s;
  return MOTEOPT_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// launch helpers
int grid_for(int chunks, int sms) { return std::max(1, std::min(chunks, sms * 8)); }

struct GradSource {          // one tensor of the global grad norm
  const void* g;
  int64_t numel;
  int dtype;
};

int launch_sumsq(const std::vector<GradSource>& src, const std::vector<int>& chunk_start, double* partials, bool has_div,
                 float div, int sms, cudaStream_t st, const float* div_dev = nullptr) {
  SumsqArgs A;
  std::memset(&A, 0, sizeof(A));
  A.partials = partials;
  A.has_div = has_div;
  A.div = div;
  A.div_dev = div_dev;
  for (size_t s0 = 0; s0 < src.size(); s0 += kMaxNormSeg) {
    const size_t n = std::min(src.size() - s0, static_cast<size_t>(kMaxNormSeg));
    A.n = static_cast<int>(n);
    A.chunk_base = chunk_start[s0];
    for (size_t i = 0; i < n; ++i) {
      A.seg[i] = SumsqSeg{src[s0 + i].g, src[s0 + i].numel, src[s0 + i].dtype, 0};
      A.chunk_start[i] = chunk_start[s0 + i] - A.chunk_base;
    }
    A.chunk_start[n] = chunk_start[s0 + n] - A.chunk_base;
    if (A.chunk_start[n] == 0) continue;
    if (A.has_div) sumsq_kernel<true><<<grid_for(A.chunk_start[n], sms), kMtThreads, 0, st>>>(A);
    else sumsq_kernel<false><<<grid_for(A.chunk_start[n], sms), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("sumsq_kernel");
  }
  return MOTEOPT_OK;
}

// per-matrix ||u||_F + eps from the sum-of-squares partials
int launch_denoms(const Layout& L, const double* partials, float* den, float eps, cudaStream_t st) {
  const int nm = static_cast<int>(L.mat_chunk_start.size()) - 1;
  DenomArgs A;
  std::memset(&A, 0, sizeof(A));
  A.eps = eps;
  A.partials = partials;
  A.den = den;
  for (int s0 = 0; s0 < nm; s0 += kMaxDenom) {
    const int cnt = std::min(nm - s0, kMaxDenom);
    A.n = cnt;
    A.base = s0;
    for (int i = 0; i <= cnt; ++i) A.chunk_start[i] = L.mat_chunk_start[s0 + i];
    mat_denom_kernel<<<(cnt + 7) / 8, 256, 0, st>>>(A);
    MO_LAUNCHED("mat_denom_kernel");
  }
  return MOTEOPT_OK;
}

int launch_finalize(const std::vector<int>& tensor_chunk_start, const double* partials, bool clip, double max_norm,
                    float* out, int* status, cudaStream_t st) {
  const int n = static_cast<int>(tensor_chunk_start.size()) - 1;
  if (n > kMaxFinalTensors) return fail(MOTEOPT_ERR_LIMIT, "more than 4096 tensors in one grad-norm call");
  FinalizeArgs A;
  std::memset(&A, 0, sizeof(A));
  A.n_tensors = n;
  A.has_clip = clip;
  A.max_norm = static_cast<float>(max_norm);
  A.partials = partials;
  A.out = out;
  A.status = status;
  for (int i = 0; i <= n; ++i) A.tensor_chunk_start[i] = tensor_chunk_start[i];
  norm_finalize_kernel<<<1, 1024, 0, st>>>(A);
  MO_LAUNCHED("norm_finalize_kernel");
  return MOTEOPT_OK;
}

// torch's lerp constants for a Python-float weight on fp32 tensors: w and 1 - w in fp32, |w| < 0.5 picks the form
EmaConsts ema_consts(double weight) {
  EmaConsts E;
  std::memset(&E, 0, sizeof(E));
  E.w = static_cast<float>(weight);
  E.omw = 1.0f - E.w;
  E.small = std::fabs(E.w) < 0.5f;
  return E;
}

// ema: per AdamW tensor, an EMA buffer or null; lr_dev: device array, one lr per tensor, or null
int launch_adamw(const moteopt_adamw_tensor* t, int n, const moteopt_adamw_hparams* hp, bool has_div, float div,
                 const float* coef, int sms, cudaStream_t st, float* const* ema = nullptr, double ema_weight = 0.0,
                 const double* lr_dev = nullptr, const float* div_dev = nullptr) {
  static thread_local AdamArgs A;
  std::memset(&A, 0, sizeof(A));
  A.ema = ema_consts(ema_weight);
  A.has_div = has_div;
  A.div = div;
  A.div_dev = div_dev;
  A.coef = coef;
  const double w = 1.0 - hp->beta1;
  A.lerp_w = static_cast<float>(w);
  A.lerp_small = std::fabs(static_cast<float>(w)) < 0.5f;
  A.one_minus_w = 1.0f - static_cast<float>(w);
  A.beta2 = static_cast<float>(hp->beta2);
  A.one_minus_beta2 = static_cast<float>(1.0 - hp->beta2);
  A.eps = static_cast<float>(hp->eps);
  A.beta1d = hp->beta1;
  A.beta2d = hp->beta2;
  A.dstep = hp->device_step;
  if (hp->device_step != nullptr && n > 0) {
    step_increment_kernel<<<1, 32, 0, st>>>(hp->device_step);
    MO_LAUNCHED("step_increment_kernel");
  }
  for (int s0 = 0; s0 < n; s0 += kMaxAdamSeg) {
    const int cnt = std::min(n - s0, kMaxAdamSeg);
    A.n = cnt;
    A.chunk_start[0] = 0;
    int64_t elems = 0;
    for (int i = 0; i < cnt; ++i) elems += t[s0 + i].numel;
    const bool small = cdiv(elems, kChunk) < 4 * static_cast<int64_t>(sms);
    const int unit = small ? kAdamChunk : kChunk;
    for (int i = 0; i < cnt; ++i) {
      const moteopt_adamw_tensor& x = t[s0 + i];
      AdamSeg& S = A.seg[i];
      S.p = x.param;
      S.g = x.grad;
      S.m = x.exp_avg;
      S.v = x.exp_avg_sq;
      S.numel = x.numel;
      S.dtype = x.grad_dtype;
      const double step = static_cast<double>(x.step);
      const double bc1 = 1.0 - std::pow(hp->beta1, step);
      const double bc2 = 1.0 - std::pow(hp->beta2, step);
      S.neg_step_size = static_cast<float>(-(x.lr / bc1));
      S.bc2_sqrt = static_cast<float>(std::pow(bc2, 0.5));
      S.has_decay = x.weight_decay != 0.0;
      S.decay_mul = static_cast<float>(1.0 - x.lr * x.weight_decay);
      S.lr = x.lr;
      S.wd = x.weight_decay;
      S.ema = ema != nullptr ? ema[s0 + i] : nullptr;
      S.lr_dev = lr_dev != nullptr ? lr_dev + s0 + i : nullptr;
      S.bc1 = bc1;
      A.chunk_start[i + 1] = A.chunk_start[i] + static_cast<int>(cdiv(x.numel, unit));
    }
    if (A.chunk_start[cnt] == 0) continue;
    if (small) adamw_kernel<true><<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    else adamw_kernel<false><<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("adamw_kernel");
  }
  return MOTEOPT_OK;
}

int check_adamw(const moteopt_adamw_tensor* t, int n, const moteopt_adamw_hparams* hp) {
  if (n < 0 || (n > 0 && (t == nullptr || hp == nullptr))) return fail(MOTEOPT_ERR_INVALID, "bad AdamW tensor list");
  for (int i = 0; i < n; ++i) {
    const moteopt_adamw_tensor& x = t[i];
    if (x.numel < 0) return fail(MOTEOPT_ERR_INVALID, "AdamW tensor " + std::to_string(i) + ": negative numel");
    if (x.numel > 0 && (!x.param || !x.grad || !x.exp_avg || !x.exp_avg_sq))
      return fail(MOTEOPT_ERR_INVALID, "AdamW tensor " + std::to_string(i) + ": null pointer");
    if (x.grad_dtype != kF32 && x.grad_dtype != kBF16)
      return fail(MOTEOPT_ERR_INVALID, "AdamW tensor " + std::to_string(i) + ": grad dtype must be fp32 or bf16");
    if (x.step < 1 && hp->device_step == nullptr)
      return fail(MOTEOPT_ERR_INVALID, "AdamW tensor " + std::to_string(i) + ": step must be >= 1");
    if (cdiv(x.numel, kAdamChunk) > (1 << 30)) return fail(MOTEOPT_ERR_LIMIT, "AdamW tensor too large");
  }
  return MOTEOPT_OK;
}

int check_muon(const moteopt_muon_param* p, int n, const moteopt_muon_config* cfg) {
  if (n < 0 || (n > 0 && (p == nullptr || cfg == nullptr))) return fail(MOTEOPT_ERR_INVALID, "bad Muon param list");
  if (cfg != nullptr && (cfg->ns_steps < 0 || cfg->ns_steps > 100)) return fail(MOTEOPT_ERR_INVALID, "ns_steps out of range");
  if (cfg != nullptr && cfg->ns_variant != 0 && cfg->ns_variant != 1)
    return fail(MOTEOPT_ERR_INVALID, "ns_variant must be 0 (the reference iteration) or 1 (Gram Newton-Schulz)");
  for (int i = 0; i < n; ++i) {
    const moteopt_muon_param& x = p[i];
    if (!x.param || !x.grad || !x.momentum_buffer)
      return fail(MOTEOPT_ERR_INVALID, "Muon param " + std::to_string(i) + ": null pointer");
    if (x.batch < 1 || x.rows < 1 || x.cols < 1)
      return fail(MOTEOPT_ERR_INVALID, "Muon param " + std::to_string(i) + ": batch, rows and cols must be >= 1");
    if (x.grad_dtype != kF32 && x.grad_dtype != kBF16)
      return fail(MOTEOPT_ERR_INVALID, "Muon param " + std::to_string(i) + ": grad dtype must be fp32 or bf16");
  }
  return MOTEOPT_OK;
}

EmaConsts ema_consts(double weight);


int launch_flat_norm(const std::vector<FlatNormSeg>& segs, int has_div, float div, const float* coef,
                     const float* den, int sms, cudaStream_t st, const float* div_dev = nullptr) {
  static thread_local FlatNormArgs A;
  for (size_t s0 = 0; s0 < segs.size(); s0 += kMaxFlatSeg) {
    const int cnt = static_cast<int>(std::min(segs.size() - s0, static_cast<size_t>(kMaxFlatSeg)));
    std::memset(&A, 0, sizeof(A));
    A.n = cnt;
    A.has_div = has_div;
    A.div = div;
    A.div_dev = div_dev;
    A.coef = coef;
    A.den = den;
    for (int i = 0; i < cnt; ++i) {
      A.seg[i] = segs[s0 + i];
      A.chunk_start[i + 1] = A.chunk_start[i] + static_cast<int>(cdiv(A.seg[i].numel, kChunk));
    }
    if (A.has_div) ns_normalize_flat_kernel<true><<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    else ns_normalize_flat_kernel<false><<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("ns_normalize_flat_kernel");
  }
  return MOTEOPT_OK;
}

// Whether any matrix of a tiled copy-out / apply launch lerps an EMA (picks the kernel instantiation).
bool out_has_ema(const OutArgs& A, size_t cnt) {
  for (size_t i = 0; i < cnt; ++i)
    if (A.mat[i].ema != nullptr) return true;
  return false;
}

int launch_flat_out(const std::vector<FlatOutSeg>& segs, int apply, int sms, cudaStream_t st, double ema_weight = 0.0) {
  static thread_local FlatOutArgs A;
  for (size_t s0 = 0; s0 < segs.size(); s0 += kMaxFlatSeg) {
    const int cnt = static_cast<int>(std::min(segs.size() - s0, static_cast<size_t>(kMaxFlatSeg)));
    std::memset(&A, 0, sizeof(A));
    A.n = cnt;
    A.apply = apply;
    A.ema = ema_consts(ema_weight);
    for (int i = 0; i < cnt; ++i) {
      A.seg[i] = segs[s0 + i];
      A.chunk_start[i + 1] = A.chunk_start[i] + static_cast<int>(cdiv(A.seg[i].numel, kChunk));
    }
    ns_out_flat_kernel<<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("ns_out_flat_kernel");
  }
  return MOTEOPT_OK;
}

// The first half of the Muon update of `n` params: momentum and the Newton-Schulz normalisation X0.
int run_muon(const moteopt_muon_param* P, int n, const moteopt_muon_config* cfg, const Layout& L, char* ws,
             bool has_div, float div, const float* coef, int* status, int sms, cudaStream_t st,
             const float* div_dev = nullptr) {
  if (n == 0) return MOTEOPT_OK;
  double* mom_partials = reinterpret_cast<double*>(ws + L.off_mom);
  // flatten the matrices in group-major order
  struct Mat {
    const moteopt_muon_param* p;
    int slice;
    const GroupPlan* g;
    int pos;   // index inside its group
  };
  std::vector<Mat> mats;
  for (const GroupPlan& g : L.groups)
    for (size_t k = 0; k < g.mats.size(); ++k)
      mats.push_back(Mat{&P[g.mats[k].src], g.mats[k].slice, &g, static_cast<int>(k)});
  const int nm = static_cast<int>(mats.size());
  auto elem_off = [](const Mat& m) { return static_cast<int64_t>(m.slice) * m.p->rows * m.p->cols; };
  auto gptr = [&](const Mat& m) -> const void* {
    const int64_t off = elem_off(m);
    return m.p->grad_dtype == kBF16 ? static_cast<const void*>(static_cast<const __nv_bfloat16*>(m.p->grad) + off)
                                    : static_cast<const void*>(static_cast<const float*>(m.p->grad) + off);
  };

  // 1. momentum + per-chunk sum of u^2
  {
    MomArgs A;
    std::memset(&A, 0, sizeof(A));
    A.has_div = has_div;
    A.div = div;
    A.div_dev = div_dev;
    A.coef = coef;
    A.partials = mom_partials;
    for (int s0 = 0; s0 < nm; s0 += kMaxMomSeg) {
      const int cnt = std::min(nm - s0, kMaxMomSeg);
      A.n = cnt;
      A.chunk_base = L.mat_chunk_start[s0];
      for (int i = 0; i < cnt; ++i) {
        const Mat& m = mats[s0 + i];
        MomSeg& S = A.seg[i];
        S.g = gptr(m);
        S.buf = m.p->momentum_buffer + elem_off(m);
        S.numel = m.p->rows * m.p->cols;
        S.mom = static_cast<float>(m.p->momentum);
        S.nesterov = m.p->nesterov != 0;
        S.dtype = m.p->grad_dtype;
        A.chunk_start[i] = L.mat_chunk_start[s0 + i] - A.chunk_base;
      }
      A.chunk_start[cnt] = L.mat_chunk_start[s0 + cnt] - A.chunk_base;
      if (A.has_div) muon_momentum_kernel<true><<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
      else muon_momentum_kernel<false><<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
      MO_LAUNCHED("muon_momentum_kernel");
    }
  }
  // 2. X0 = bf16(u / (||u|| + eps)) into each group's X0 buffer
  {
    float* den = reinterpret_cast<float*>(ws + L.off_den);
    MO_TRY(launch_denoms(L, mom_partials, den, static_cast<float>(cfg->ns_eps), st));
    NormArgs A;
    std::memset(&A, 0, sizeof(A));
    A.has_div = has_div;
    A.div = div;
    A.div_dev = div_dev;
    A.coef = coef;
    A.den = den;
    std::vector<FlatNormSeg> flat;
    std::vector<int> tiled;   // indices into mats of the matrices that need the tiled (transposing) kernel
    for (int i = 0; i < nm; ++i) {
      const Mat& m = mats[i];
      const GroupPlan& g = *m.g;
      if (stored_as_iterated(g)) {
        FlatNormSeg S;
        std::memset(&S, 0, sizeof(S));
        S.g = gptr(m);
        S.buf = m.p->momentum_buffer + elem_off(m);
        S.x = ws + g.off_x0 + static_cast<size_t>(m.pos) * g.m * g.n * 2;
        S.numel = static_cast<int64_t>(g.rows) * g.cols;
        S.mom = static_cast<float>(m.p->momentum);
        S.nesterov = m.p->nesterov != 0;
        S.dtype = m.p->grad_dtype;
        S.den_index = i;
        flat.push_back(S);
      } else {
        tiled.push_back(i);
      }
    }
    MO_TRY(launch_flat_norm(flat, has_div, div, coef, den, sms, st, div_dev));
    const int nt = static_cast<int>(tiled.size());
    for (int s0 = 0; s0 < nt; s0 += kMaxNormMat) {
      const int cnt = std::min(nt - s0, kMaxNormMat);
      A.n = cnt;
      int max_tiles = 0;
      for (int i = 0; i < cnt; ++i) {
        const Mat& m = mats[tiled[s0 + i]];
        const GroupPlan& g = *m.g;
        NormMat& M = A.mat[i];
        M.g = gptr(m);
        M.buf = m.p->momentum_buffer + elem_off(m);
        M.x = ws + g.off_x0 + static_cast<size_t>(m.pos) * g.m * g.n * 2;
        M.rows = g.rows;
        M.cols = g.cols;
        M.m_pad = g.m;
        M.n_pad = g.n;
        M.transposed = g.transposed;
        M.dtype = m.p->grad_dtype;
        M.mom = static_cast<float>(m.p->momentum);
        M.nesterov = m.p->nesterov != 0;
        M.den_index = tiled[s0 + i];
        M.tiles_x = static_cast<int>(cdiv(g.n, kNormTile));
        M.tiles = M.tiles_x * static_cast<int>(cdiv(g.m, kNormTile));
        max_tiles = std::max(max_tiles, M.tiles);
      }
      if (A.has_div) ns_normalize_kernel<true><<<dim3(max_tiles, cnt), kMtThreads, 0, st>>>(A);
      else ns_normalize_kernel<false><<<dim3(max_tiles, cnt), kMtThreads, 0, st>>>(A);
      MO_LAUNCHED("ns_normalize_kernel");
    }
  }
  (void)status;
  return MOTEOPT_OK;
}

// A tensor map of one bf16 [depth][outer][inner] buffer, cached by its address, geometry and box (the Gram
// variant's phases point the launch's operand roles at different buffers).
struct OneMapKey {
  uintptr_t base;
  uint64_t inner, outer, depth;
  uint32_t bi, bo;
  int swz, dev;
  bool operator<(const OneMapKey& o) const {
    return std::tie(base, inner, outer, depth, bi, bo, swz, dev) <
           std::tie(o.base, o.inner, o.outer, o.depth, o.bi, o.bo, o.swz, o.dev);
  }
};
std::map<OneMapKey, CUtensorMap> g_one_maps;

int one_map(void* base, uint64_t inner, uint64_t outer, uint64_t depth, uint32_t bi, uint32_t bo,
            CUtensorMapSwizzle swz, CUtensorMap* out) {
  int dev = 0;
  MO_CUDA(cudaGetDevice(&dev));
  const OneMapKey key{reinterpret_cast<uintptr_t>(base), inner, outer, depth, bi, bo, static_cast<int>(swz), dev};
  std::lock_guard<std::mutex> lk(g_map_mu);
  auto it = g_one_maps.find(key);
  if (it != g_one_maps.end()) {
    *out = it->second;
    return MOTEOPT_OK;
  }
  CUtensorMap m;
  MO_TRY(make_map(&m, base, inner, outer, depth, bi, bo, swz));
  if (g_one_maps.size() > 16384) g_one_maps.clear();
  g_one_maps[key] = m;
  *out = m;
  return MOTEOPT_OK;
}

// The three views the kernel uses of one buffer: K-major operand (box 64 x 128), MN-major operand (box 64 x 64),
// epilogue (32 x 32, 64-byte swizzle).
struct Views {
  CUtensorMap k, mn, e;
};
int buffer_views(void* base, uint64_t inner, uint64_t outer, uint64_t depth, Views* v) {
  MO_TRY(one_map(base, inner, outer, depth, ns::BK, ns::HM, CU_TENSOR_MAP_SWIZZLE_128B, &v->k));
  MO_TRY(one_map(base, inner, outer, depth, 64, ns::BK, CU_TENSOR_MAP_SWIZZLE_128B, &v->mn));
  MO_TRY(one_map(base, inner, outer, depth, ns::EPI_TILE, ns::EPI_TILE, CU_TENSOR_MAP_SWIZZLE_64B, &v->e));
  return MOTEOPT_OK;
}

// Launch sets: runs of at most kMaxGroups groups and kMaxApply matrices.
std::vector<std::vector<const GroupPlan*>> launch_sets(const std::vector<const GroupPlan*>& groups) {
  std::vector<std::vector<const GroupPlan*>> sets;
  size_t mats = 0;
  for (const GroupPlan* g : groups) {
    if (sets.empty() || sets.back().size() >= static_cast<size_t>(ns::kMaxGroups) ||
        mats + g->mats.size() > static_cast<size_t>(ns::kMaxApply)) {
      sets.emplace_back();
      mats = 0;
    }
    sets.back().push_back(g);
    mats += g->mats.size();
  }
  return sets;
}

// The tile tables of a launch over Lh.g[0..n_groups): phase `only` alone (one launch per phase), or all three phases
// of an iteration (only = -1).
// The tile tables of a launch: `only` >= 0 keeps that phase alone; `chunks` > 1 (persistent mode only) splits every
// group's matrices into that many runs, each run taken through its three phases before the next, so that the X, A
// and B a run reads stay in L2 between its phases.
void tile_tables(ns::Launch& Lh, int only, int chunks = 1) {
  chunks = std::max(1, std::min(chunks, ns::kMaxChunks));
  Lh.per_iter = 0;
  for (int ph = ns::kGram; ph <= ns::kUpdate; ++ph) {
    Lh.tile_start[ph][0] = 0;
    for (int gi = 0; gi < Lh.n_groups; ++gi) {
      const ns::Group& G = Lh.g[gi];
      const int T = static_cast<int>(cdiv(G.m, ns::TM));
      Lh.tiles_m[gi] = T;
      Lh.tiles_n[gi] = static_cast<int>(cdiv(G.n, ns::TN));
      const int per = ph == ns::kUpdate ? T * Lh.tiles_n[gi] : T * (T + 1) / 2;
      Lh.tile_start[ph][gi + 1] = Lh.tile_start[ph][gi] + ((only < 0 || only == ph) ? G.count * per : 0);
    }
    Lh.phase_tiles[ph] = Lh.tile_start[ph][Lh.n_groups];
    Lh.per_iter += Lh.phase_tiles[ph];
  }
  Lh.n_chunks = chunks;
  int acc = 0;
  for (int c = 0; c <= chunks; ++c)
    for (int gi = 0; gi < Lh.n_groups; ++gi) Lh.ck_b0[c][gi] = static_cast<int>(int64_t(Lh.g[gi].count) * c / chunks);
  for (int c = 0; c < chunks; ++c) {
    Lh.chunk_start[c] = acc;
    for (int ph = ns::kGram; ph <= ns::kUpdate; ++ph) {
      Lh.ck_tile_start[c][ph][0] = 0;
      for (int gi = 0; gi < Lh.n_groups; ++gi) {
        const int T = Lh.tiles_m[gi];
        const int per = ph == ns::kUpdate ? T * Lh.tiles_n[gi] : T * (T + 1) / 2;
        const int cnt = Lh.ck_b0[c + 1][gi] - Lh.ck_b0[c][gi];
        Lh.ck_tile_start[c][ph][gi + 1] = Lh.ck_tile_start[c][ph][gi] + ((only < 0 || only == ph) ? cnt * per : 0);
      }
      Lh.ck_phase_tiles[c][ph] = Lh.ck_tile_start[c][ph][Lh.n_groups];
      acc += Lh.ck_phase_tiles[c][ph];
    }
  }
  Lh.chunk_start[chunks] = acc;   // == per_iter
}

// The reference iteration (mote/train/muon.py:37-40) over `groups`: one persistent launch per set, or one launch per
// phase and iteration (moteopt_ns_set_persistent).
int run_ns_reference(const std::vector<const GroupPlan*>& groups, const Layout& L, char* ws, int steps, int* status,
                     cudaStream_t st) {
  static thread_local ns::Launch Lh;   // ~20 KB: kept off the stack
  int* done = reinterpret_cast<int*>(ws + L.off_done);
  for (const auto& set : launch_sets(groups)) {
    std::memset(&Lh, 0, sizeof(Lh));
    Lh.n_groups = static_cast<int>(set.size());
    Lh.status = status;
    Lh.ca = ns::kNsA;
    Lh.cb = ns::kNsB;
    Lh.cc = ns::kNsC;
    int first = 0;
    for (size_t gi = 0; gi < set.size(); ++gi) {
      const GroupPlan& g = *set[gi];
      ns::Group& G = Lh.g[gi];
      MapSet ms;
      MO_TRY(group_maps(ws, g, &ms));
      G.xk[0] = ms.xk[0];
      G.xk[1] = ms.xk[1];
      G.xmn[0] = ms.xmn[0];
      G.xmn[1] = ms.xmn[1];
      G.ak = ms.ak;
      G.bk = ms.bk;
      G.amn = ms.amn;
      G.bmn = ms.bmn;
      G.xe[0] = ms.xe[0];
      G.xe[1] = ms.xe[1];
      G.ae = ms.ae;
      G.be = ms.be;
      G.x[0] = reinterpret_cast<__nv_bfloat16*>(ws + g.off_x0);
      G.x[1] = reinterpret_cast<__nv_bfloat16*>(ws + g.off_x1);
      G.a = reinterpret_cast<__nv_bfloat16*>(ws + g.off_a);
      G.b = reinterpret_cast<__nv_bfloat16*>(ws + g.off_b);
      G.m = g.m;
      G.n = g.n;
      G.mv = g.mv;
      G.nv = g.nv;
      G.count = static_cast<int>(g.mats.size());
      G.first = first;
      G.transposed = g.transposed;
      G.tall = g.tall;
      first += G.count;
    }
    // the tile sequence [iteration][chunk][phase][group][matrix][tile]: 256 x 256 tiles, one per CTA pair; A and B are
    // symmetric, so their phases have the upper-triangle blocks only
    Lh.src0 = 0;
    tile_tables(Lh, -1);
    const int pairs = device_pairs();
    const int mode = g_ns_persistent.load(std::memory_order_relaxed);
    if (mode == 1 || (mode < 0 && Lh.per_iter <= kPersistentMaxWaves * pairs)) {
      // one cooperative launch for every iteration; the completion counters start at zero
      tile_tables(Lh, -1, Lh.per_iter >= kNsChunkWaves * pairs ? 2 : 1);
      MO_CUDA(cudaMemsetAsync(done, 0, sizeof(int) * 3 * static_cast<size_t>(first), st));
      Lh.done = done;
      Lh.t_begin = 0;
      Lh.t_end = steps * Lh.per_iter;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * std::min(Lh.t_end, pairs), 1, 1);
      cfg.blockDim = dim3(ns::kThreads, 1, 1);
      cfg.dynamicSmemBytes = ns::kSmemBytes;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      MO_CUDA(cudaLaunchKernelEx(&cfg, ns::ns_gemm_kernel<false>, Lh));
      MO_LAUNCHED("ns_gemm_kernel (persistent)");
    } else {
      Lh.done = nullptr;
      for (int it = 0; it < steps; ++it) {
        int t0 = it * Lh.per_iter;
        for (int ph = ns::kGram; ph <= ns::kUpdate; ++ph) {
          Lh.t_begin = t0;
          Lh.t_end = t0 + Lh.phase_tiles[ph];
          t0 = Lh.t_end;
          ns::ns_gemm_kernel<false><<<2 * std::min(Lh.phase_tiles[ph], pairs), ns::kThreads, ns::kSmemBytes, st>>>(Lh);
          MO_LAUNCHED("ns_gemm_kernel");
        }
      }
    }
  }
  return MOTEOPT_OK;
}

// The opt-in Gram Newton-Schulz variant (the reference's research notes, docs/research/efficiency-campaign-2026-08-23.md
// :903-911; not the reference's iteration) on matrices whose long side is at least twice the short one, X (m x n,
// m <= n) -> X1:
//   R = X X^T; for k < steps: B = b R + c R R; Q = a I + B (k = 0) or a Q + B Q; if k < steps - 1: T = a R + B R,
//   R = a T + B T. Finally X1 = Q X.
// Every product is a phase of the tcgen05 kernel with the launch's operand roles pointed at the variant's buffers,
// one launch per phase (the kernel boundary orders them), and rounds once with its a*Y / b*R term (round_once).
// Storage, which oracle/moteopt_oracle.py::gram_newton_schulz_blocked follows: R is exactly symmetric (the Gram phase
// writes its upper tiles and ns_symmetrize_kernel mirrors every element below the diagonal, again after each R
// update), T and Q are stored whole, B on its upper tiles (the update phases read its tiles below the diagonal through
// their mirrors; B from a symmetric R is symmetric), and the final product reads Q through its upper tiles.
int run_ns_gram(const std::vector<const GroupPlan*>& groups, char* ws, int steps, int* status, cudaStream_t st) {
  static thread_local ns::Launch Lh;
  const int pairs = device_pairs();
  for (const auto& set : launch_sets(groups)) {
    const int ng = static_cast<int>(set.size());
    struct Bufs {
      Views x0, x1, r, b, t, q[2];
    };
    std::vector<Bufs> vb(ng);
    for (int gi = 0; gi < ng; ++gi) {
      const GroupPlan& g = *set[gi];
      const uint64_t c = g.mats.size();
      MO_TRY(buffer_views(ws + g.off_x0, g.n, g.m, c, &vb[gi].x0));
      MO_TRY(buffer_views(ws + g.off_x1, g.n, g.m, c, &vb[gi].x1));
      MO_TRY(buffer_views(ws + g.off_a, g.m, g.m, c, &vb[gi].r));
      MO_TRY(buffer_views(ws + g.off_b, g.m, g.m, c, &vb[gi].b));
      MO_TRY(buffer_views(ws + g.off_t, g.m, g.m, c, &vb[gi].t));
      MO_TRY(buffer_views(ws + g.off_q0, g.m, g.m, c, &vb[gi].q[0]));
      MO_TRY(buffer_views(ws + g.off_q1, g.m, g.m, c, &vb[gi].q[1]));
    }
    // one phase over every group of the set; `roles` points group gi's operand maps at its buffers
    auto phase = [&](int ph, bool wide, float ca, bool no_aux, auto&& roles) -> int {
      std::memset(&Lh, 0, sizeof(Lh));
      Lh.n_groups = ng;
      Lh.status = status;
      Lh.ca = ca;
      Lh.cb = ns::kNsB;
      Lh.cc = ns::kNsC;
      Lh.round_once = 1;
      Lh.no_aux = no_aux ? 1 : 0;
      int first = 0;
      for (int gi = 0; gi < ng; ++gi) {
        const GroupPlan& g = *set[gi];
        ns::Group& G = Lh.g[gi];
        // every map slot holds a valid map (the kernel prefetches all of them); the phase's roles override
        const CUtensorMap& any = vb[gi].r.e;
        G.xk[0] = G.xk[1] = G.xmn[0] = G.xmn[1] = G.ak = G.bk = G.amn = G.bmn = G.xe[0] = G.xe[1] = G.ae = G.be = any;
        roles(gi, G);
        G.m = g.m;
        G.n = wide ? g.n : g.m;   // m x n products (the Gram phase, the final Q X) or m x m ones
        G.mv = g.mv;
        G.nv = wide ? g.nv : g.mv;
        G.count = static_cast<int>(g.mats.size());
        G.first = first;
        G.transposed = g.transposed;
        first += G.count;
      }
      tile_tables(Lh, ph);
      Lh.src0 = 0;
      Lh.done = nullptr;
      Lh.t_begin = 0;
      Lh.t_end = Lh.per_iter;
      ns::ns_gemm_kernel<true><<<2 * std::min(Lh.t_end, pairs), ns::kThreads, ns::kSmemBytes, st>>>(Lh);
      MO_LAUNCHED("ns_gemm_kernel (Gram variant)");
      return MOTEOPT_OK;
    };
    // ns_symmetrize_kernel (q1 false: src = dst = R) or ns_gram_q1_kernel (q1 true: B -> Q0) over every group of the set
    auto elementwise = [&](bool q1) -> int {
      for (int gi = 0; gi < ng; ++gi) {
        const GroupPlan& g = *set[gi];
        ns::SymArgs A;
        A.src = reinterpret_cast<__nv_bfloat16*>(ws + (q1 ? g.off_b : g.off_a));
        A.dst = reinterpret_cast<__nv_bfloat16*>(ws + (q1 ? g.off_q0 : g.off_a));
        A.m = g.m;
        A.mv = g.mv;
        A.a = ns::kNsA;
        const int tiles = static_cast<int>(cdiv(g.m, 32));
        const dim3 grid(static_cast<unsigned>(tiles * tiles), static_cast<unsigned>(g.mats.size()));
        if (q1) ns::ns_gram_q1_kernel<<<grid, 256, 0, st>>>(A);
        else ns::ns_symmetrize_kernel<<<grid, 256, 0, st>>>(A);
        MO_LAUNCHED(q1 ? "ns_gram_q1_kernel" : "ns_symmetrize_kernel");
      }
      return MOTEOPT_OK;
    };
    // R = X X^T (upper tiles), then whole and exactly symmetric
    MO_TRY(phase(ns::kGram, true, 0.f, false, [&](int gi, ns::Group& G) {
      G.xk[0] = vb[gi].x0.k;
      G.ae = vb[gi].r.e;
    }));
    MO_TRY(elementwise(false));
    int q = 0;   // the Q buffer holding the current Q
    for (int k = 0; k < steps; ++k) {
      MO_TRY(phase(ns::kPoly, false, 0.f, false, [&](int gi, ns::Group& G) {   // B = b R + c R R
        G.ak = vb[gi].r.k;
        G.amn = vb[gi].r.mn;
        G.ae = vb[gi].r.e;
        G.be = vb[gi].b.e;
      }));
      if (k == 0) {   // Q = a I + B
        MO_TRY(elementwise(true));
      } else {        // Q' = a Q + B Q
        MO_TRY(phase(ns::kUpdate, false, ns::kNsA, false, [&](int gi, ns::Group& G) {
          G.bk = vb[gi].b.k;
          G.bmn = vb[gi].b.mn;
          G.xmn[0] = vb[gi].q[q].mn;
          G.xe[0] = vb[gi].q[q].e;
          G.xe[1] = vb[gi].q[q ^ 1].e;
        }));
        q ^= 1;
      }
      if (k + 1 < steps) {
        MO_TRY(phase(ns::kUpdate, false, ns::kNsA, false, [&](int gi, ns::Group& G) {   // T = a R + B R
          G.bk = vb[gi].b.k;
          G.bmn = vb[gi].b.mn;
          G.xmn[0] = vb[gi].r.mn;
          G.xe[0] = vb[gi].r.e;
          G.xe[1] = vb[gi].t.e;
        }));
        MO_TRY(phase(ns::kUpdate, false, ns::kNsA, false, [&](int gi, ns::Group& G) {   // R = a T + B T
          G.bk = vb[gi].b.k;
          G.bmn = vb[gi].b.mn;
          G.xmn[0] = vb[gi].t.mn;
          G.xe[0] = vb[gi].t.e;
          G.xe[1] = vb[gi].r.e;
        }));
        MO_TRY(elementwise(false));   // R exactly symmetric again
      }
    }
    MO_TRY(phase(ns::kUpdate, true, 0.f, true, [&](int gi, ns::Group& G) {   // X1 = Q X (Q through its upper tiles)
      G.bk = vb[gi].q[q].k;
      G.bmn = vb[gi].q[q].mn;
      G.xmn[0] = vb[gi].x0.mn;
      G.xe[0] = vb[gi].x0.e;
      G.xe[1] = vb[gi].x1.e;
    }));
  }
  return MOTEOPT_OK;
}

// Newton-Schulz iterations over every group (the final iterate of group g is in X[out_buffer(g, steps)]).
int run_ns(const Layout& L, char* ws, int steps, int* status, cudaStream_t st) {
  if (steps == 0) return MOTEOPT_OK;
  std::vector<const GroupPlan*> ref, gram;
  for (const GroupPlan& g : L.groups) (g.gram ? gram : ref).push_back(&g);
  if (!ref.empty()) MO_TRY(run_ns_reference(ref, L, ws, steps, status, st));
  if (!gram.empty()) MO_TRY(run_ns_gram(gram, ws, steps, status, st));
  return MOTEOPT_OK;
}

std::vector<ns::MatApply> muon_apply_table(const moteopt_muon_param* P, const moteopt_muon_config* cfg, const Layout& L) {
  std::vector<ns::MatApply> out;
  for (const GroupPlan& g : L.groups)
    for (const MatRef& r : g.mats) {
      const moteopt_muon_param& p = P[r.src];
      ns::MatApply a;
      a.p = p.param + static_cast<int64_t>(r.slice) * p.rows * p.cols;
      a.neg_lr = static_cast<float>(-p.lr);
      a.has_decay = p.decay != 0.0;
      a.decay_mul = static_cast<float>(1.0 - p.decay);
      a.scale = static_cast<float>(cfg->rms_scale * std::pow(static_cast<double>(std::max(p.rows, p.cols)), 0.5));
      out.push_back(a);
    }
  return out;
}

// The Muon apply (muon.py:97-99) from the final iterate: X0 when ns_steps == 0, else the last phase's output.
// ema: per Muon param, an EMA buffer or null (null array: none)
// norms: n_muon outputs (||p_new||_F per Muon param), or null; lr_dev: device array of one lr per Muon param, with
// the host arrays wd / lr_max (see moteopt_step_extras), or null
int run_apply(const moteopt_muon_param* P, const moteopt_muon_config* cfg, const Layout& L, char* ws, int steps,
              cudaStream_t st, float* const* ema = nullptr, double ema_weight = 0.0, float* norms = nullptr,
              const double* lr_dev = nullptr, const double* wd = nullptr, const double* lr_max = nullptr) {
  double* apply_partials = reinterpret_cast<double*>(ws + L.off_apply);
  const std::vector<ns::MatApply> tab = muon_apply_table(P, cfg, L);
  static thread_local OutArgs A;
  std::memset(&A, 0, sizeof(A));
  A.apply = 1;
  A.ema = ema_consts(ema_weight);
  std::vector<OutMat> all;
  std::vector<FlatOutSeg> flat;
  size_t k = 0;
  for (const GroupPlan& g : L.groups)
    for (size_t pos = 0; pos < g.mats.size(); ++pos, ++k) {
      const MatRef& ref = g.mats[pos];
      const moteopt_muon_param& pp = P[ref.src];
      float* e = nullptr;   // this matrix's slice of its param's EMA
      if (ema != nullptr && ema[ref.src] != nullptr) e = ema[ref.src] + static_cast<int64_t>(ref.slice) * pp.rows * pp.cols;
      double* part = norms == nullptr ? nullptr
                                     : apply_partials + L.param_apply_start[ref.src] +
                                           static_cast<int64_t>(ref.slice) * apply_partials_per_slice(pp.rows, pp.cols, stored_as_iterated(g));
      if (stored_as_iterated(g)) {
        FlatOutSeg S;
        std::memset(&S, 0, sizeof(S));
        S.x = ws + (out_buffer(g, steps) ? g.off_x1 : g.off_x0) + pos * g.m * g.n * 2;
        S.out = tab[k].p;
        S.numel = static_cast<int64_t>(g.rows) * g.cols;
        S.neg_lr = tab[k].neg_lr;
        S.decay_mul = tab[k].decay_mul;
        S.has_decay = tab[k].has_decay;
        S.scale = tab[k].scale;
        S.ema = e;
        S.partials = part;
        if (lr_dev != nullptr) {
          S.lr_dev = lr_dev + ref.src;
          S.wd = wd[ref.src];
          S.lr_max = lr_max[ref.src];
        }
        flat.push_back(S);
        continue;
      }
      OutMat M;
      std::memset(&M, 0, sizeof(M));
      M.x = ws + (out_buffer(g, steps) ? g.off_x1 : g.off_x0) + pos * g.m * g.n * 2;
      M.out = tab[k].p;
      M.ema = e;
      M.partials = part;
      if (lr_dev != nullptr) {
        M.lr_dev = lr_dev + ref.src;
        M.wd = wd[ref.src];
        M.lr_max = lr_max[ref.src];
      }
      M.rows = g.rows;
      M.cols = g.cols;
      M.m_pad = g.m;
      M.n_pad = g.n;
      M.transposed = g.transposed;
      M.tiles_x = static_cast<int>(cdiv(g.cols, kNormTile));
      M.tiles = M.tiles_x * static_cast<int>(cdiv(g.rows, kNormTile));
      M.neg_lr = tab[k].neg_lr;
      M.decay_mul = tab[k].decay_mul;
      M.has_decay = tab[k].has_decay;
      M.scale = tab[k].scale;
      all.push_back(M);
    }
  MO_TRY(launch_flat_out(flat, 1, device_sms(), st, ema_weight));
  for (size_t s0 = 0; s0 < all.size(); s0 += kMaxOutMat) {
    const size_t cnt = std::min(all.size() - s0, static_cast<size_t>(kMaxOutMat));
    A.n = static_cast<int>(cnt);
    int max_tiles = 0;
    for (size_t i = 0; i < cnt; ++i) {
      A.mat[i] = all[s0 + i];
      max_tiles = std::max(max_tiles, A.mat[i].tiles);
    }
    if (out_has_ema(A, cnt)) ns_out_kernel<true><<<dim3(max_tiles, static_cast<unsigned>(cnt)), kMtThreads, 0, st>>>(A);
    else ns_out_kernel<false><<<dim3(max_tiles, static_cast<unsigned>(cnt)), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("ns_out_kernel");
  }
  if (norms != nullptr) {   // ||p_new||_F per param: fixed-order fp64 sum of its partials (eps 0)
    const int np = static_cast<int>(L.param_apply_start.size()) - 1;
    static thread_local DenomArgs D;
    std::memset(&D, 0, sizeof(D));
    D.eps = 0.f;
    D.partials = apply_partials;
    D.den = norms;
    for (int s0 = 0; s0 < np; s0 += kMaxDenom) {
      const int cnt = std::min(np - s0, kMaxDenom);
      D.n = cnt;
      D.base = s0;
      for (int i = 0; i <= cnt; ++i) D.chunk_start[i] = L.param_apply_start[s0 + i];
      mat_denom_kernel<<<(cnt + 7) / 8, 256, 0, st>>>(D);
      MO_LAUNCHED("mat_denom_kernel");
    }
  }
  return MOTEOPT_OK;
}

// The final iterate of every matrix copied out (bf16, the parameter's orientation) to out[param] at the matrix's
// slice, instead of being applied: the sharded step's owners produce the updates that the ranks all-gather.
int run_copy_out(const moteopt_muon_param* P, const Layout& L, char* ws, int steps, void* const* out, int sms,
                 cudaStream_t st) {
  static thread_local OutArgs A;
  std::memset(&A, 0, sizeof(A));
  A.apply = 0;
  std::vector<OutMat> all;
  std::vector<FlatOutSeg> flat;
  for (const GroupPlan& g : L.groups)
    for (size_t pos = 0; pos < g.mats.size(); ++pos) {
      const MatRef& r = g.mats[pos];
      const moteopt_muon_param& p = P[r.src];
      void* dst = static_cast<char*>(out[r.src]) + static_cast<size_t>(r.slice) * p.rows * p.cols * 2;
      const void* x = ws + (out_buffer(g, steps) ? g.off_x1 : g.off_x0) + pos * g.m * g.n * 2;
      if (stored_as_iterated(g)) {
        FlatOutSeg S;
        std::memset(&S, 0, sizeof(S));
        S.x = x;
        S.out = dst;
        S.numel = static_cast<int64_t>(g.rows) * g.cols;
        flat.push_back(S);
        continue;
      }
      OutMat M;
      std::memset(&M, 0, sizeof(M));
      M.x = x;
      M.out = dst;
      M.rows = g.rows;
      M.cols = g.cols;
      M.m_pad = g.m;
      M.n_pad = g.n;
      M.transposed = g.transposed;
      M.tiles_x = static_cast<int>(cdiv(g.cols, kNormTile));
      M.tiles = M.tiles_x * static_cast<int>(cdiv(g.rows, kNormTile));
      all.push_back(M);
    }
  MO_TRY(launch_flat_out(flat, 0, sms, st));
  for (size_t s0 = 0; s0 < all.size(); s0 += kMaxOutMat) {
    const size_t cnt = std::min(all.size() - s0, static_cast<size_t>(kMaxOutMat));
    A.n = static_cast<int>(cnt);
    int max_tiles = 0;
    for (size_t i = 0; i < cnt; ++i) {
      A.mat[i] = all[s0 + i];
      max_tiles = std::max(max_tiles, A.mat[i].tiles);
    }
    if (out_has_ema(A, cnt)) ns_out_kernel<true><<<dim3(max_tiles, static_cast<unsigned>(cnt)), kMtThreads, 0, st>>>(A);
    else ns_out_kernel<false><<<dim3(max_tiles, static_cast<unsigned>(cnt)), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("ns_out_kernel");
  }
  return MOTEOPT_OK;
}

int check_ws(void* ws, size_t have, size_t need) {
  if (ws == nullptr) return fail(MOTEOPT_ERR_INVALID, "workspace is null");
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail(MOTEOPT_ERR_INVALID, "workspace must be 256-byte aligned");
  if (have < need)
    return fail(MOTEOPT_ERR_INVALID, "workspace too small: " + std::to_string(have) + " < " + std::to_string(need) + " bytes");
  return MOTEOPT_OK;
}

std::vector<std::tuple<int64_t, int64_t, int64_t>> muon_shapes(const moteopt_muon_param* p, int n) {
  std::vector<std::tuple<int64_t, int64_t, int64_t>> s;
  for (int i = 0; i < n; ++i) s.emplace_back(p[i].batch, p[i].rows, p[i].cols);
  return s;
}

// The whole step: (optional) grad norm + clip coefficient, AdamW, Muon.
int run_step(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* mcfg, const moteopt_adamw_tensor* adam,
             int n_adam, const moteopt_adamw_hparams* adamw_hp, const moteopt_grad_config* gcfg, const float* ext_scale,
             float* out_norm, void* workspace, size_t ws_bytes, cudaStream_t st, void* const* muon_out = nullptr,
             const moteopt_step_extras* ex = nullptr) {
  const moteopt_adamw_hparams* ahp = adamw_hp;
  float* const* ema = ex != nullptr ? ex->ema : nullptr;
  const double ema_w = ex != nullptr ? ex->ema_weight : 0.0;
  MO_TRY(check_muon(muon, n_muon, mcfg));
  MO_TRY(check_adamw(adam, n_adam, ahp));
  int sms = 0;
  MO_TRY(device_setup(&sms));
  const bool clip = gcfg != nullptr && gcfg->clip;
  std::vector<int64_t> norm_numels;
  if (clip) {
    for (int i = 0; i < n_adam; ++i) norm_numels.push_back(adam[i].numel);
    for (int i = 0; i < n_muon; ++i) norm_numels.push_back(muon[i].batch * muon[i].rows * muon[i].cols);
  }
  Layout L;
  MO_TRY(build_layout(muon_shapes(muon, n_muon), norm_numels, n_muon > 0 ? mcfg->ns_steps : 0, &L,
                      n_muon > 0 ? mcfg->ns_variant : 0));
  MO_TRY(check_ws(workspace, ws_bytes, L.bytes));
  char* ws = static_cast<char*>(workspace);
  Header* hdr = reinterpret_cast<Header*>(ws);
  int* status = &hdr->status;
  MO_CUDA(cudaMemsetAsync(hdr, 0, sizeof(Header), st));
  // the divisor of train.py:945: a device scalar (grad_divisor_device) or a host value (0 or 1: none)
  const float* div_dev = gcfg != nullptr ? gcfg->grad_divisor_device : nullptr;
  const bool has_div = div_dev != nullptr || (gcfg != nullptr && gcfg->grad_divisor != 0.0 && gcfg->grad_divisor != 1.0);
  const float div = has_div && div_dev == nullptr ? static_cast<float>(gcfg->grad_divisor) : 1.0f;
  const float* coef = ext_scale;
  if (clip) {
    std::vector<GradSource> src;
    for (int i = 0; i < n_adam; ++i) src.push_back(GradSource{adam[i].grad, adam[i].numel, adam[i].grad_dtype});
    for (int i = 0; i < n_muon; ++i)
      src.push_back(GradSource{muon[i].grad, muon[i].batch * muon[i].rows * muon[i].cols, muon[i].grad_dtype});
    double* partials = reinterpret_cast<double*>(ws + L.off_norm);
    MO_TRY(launch_sumsq(src, L.norm_tensor_chunk_start, partials, has_div, div, sms, st, div_dev));
    MO_TRY(launch_finalize(L.norm_tensor_chunk_start, partials, true, gcfg->max_norm, &hdr->norm, status, st));
    coef = &hdr->coef;
    if (out_norm != nullptr) MO_CUDA(cudaMemcpyAsync(out_norm, &hdr->norm, sizeof(float), cudaMemcpyDeviceToDevice, st));
  }
  const double* lr_dev = ex != nullptr ? ex->lr : nullptr;
  if (n_adam > 0) MO_TRY(launch_adamw(adam, n_adam, ahp, has_div, div, coef, sms, st, ema, ema_w, lr_dev, div_dev));
  if (n_muon > 0) {
    MO_TRY(run_muon(muon, n_muon, mcfg, L, ws, has_div, div, coef, status, sms, st, div_dev));
    if (mcfg->ns_steps > 0) {
      if (t_ns_ev[0] != nullptr) MO_CUDA(cudaEventRecord(t_ns_ev[0], st));
      MO_TRY(run_ns(L, ws, mcfg->ns_steps, status, st));
      if (t_ns_ev[1] != nullptr) MO_CUDA(cudaEventRecord(t_ns_ev[1], st));
    }
    if (muon_out != nullptr) MO_TRY(run_copy_out(muon, L, ws, mcfg->ns_steps, muon_out, sms, st));
    else MO_TRY(run_apply(muon, mcfg, L, ws, mcfg->ns_steps, st, ema != nullptr ? ema + n_adam : nullptr, ema_w,
                          ex != nullptr ? ex->muon_norms : nullptr, lr_dev != nullptr ? lr_dev + n_adam : nullptr,
                          ex != nullptr ? ex->muon_wd : nullptr, ex != nullptr ? ex->muon_lr_max : nullptr));
  }
  return MOTEOPT_OK;
}

}  // namespace

// =================================================================================================================
extern "C" {

int moteopt_version(void) { return 1; }

unsigned long long moteopt_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

long long moteopt_check_count(int clear) {
#ifdef MOTE_OPT_CHECKS
  unsigned long long v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_check_fails, sizeof(v));
  if (e == cudaSuccess && clear) {
    const unsigned long long z = 0;
    e = cudaMemcpyToSymbol(g_check_fails, &z, sizeof(z));
  }
  if (e != cudaSuccess) {
    fail(MOTEOPT_ERR_CUDA, std::string("moteopt_check_count: ") + cudaGetErrorString(e));
    return -1;
  }
  return static_cast<long long>(v);
#else
  (void)clear;
  return 0;
#endif
}

int moteopt_profile_ns_events(void* start_event, void* end_event) {
  if ((start_event == nullptr) != (end_event == nullptr))
    return fail(MOTEOPT_ERR_INVALID, "give both events or neither");
  t_ns_ev[0] = static_cast<cudaEvent_t>(start_event);
  t_ns_ev[1] = static_cast<cudaEvent_t>(end_event);
  return MOTEOPT_OK;
}

const char* moteopt_last_error(void) { return t_err.c_str(); }

int moteopt_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(MOTEOPT_ERR_INVALID, "moteopt_ipc_export: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == MOTEOPT_IPC_HANDLE_BYTES, "IPC handle size");
  AddrRangeFn range = addr_range_fn();
  if (range == nullptr) return fail(MOTEOPT_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(MOTEOPT_ERR_CUDA, "cuMemGetAddressRange failed (" + std::to_string(r) + ")");
  cudaIpcMemHandle_t h;
  MO_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return MOTEOPT_OK;
}

int moteopt_ipc_import(const void* handle, void** base_out) {
  if (handle == nullptr || base_out == nullptr) return fail(MOTEOPT_ERR_INVALID, "moteopt_ipc_import: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  MO_CUDA(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess));
  return MOTEOPT_OK;
}

int moteopt_ipc_close(void* base) {
  if (base == nullptr) return fail(MOTEOPT_ERR_INVALID, "moteopt_ipc_close: null argument");
  MO_CUDA(cudaIpcCloseMemHandle(base));
  return MOTEOPT_OK;
}

int moteopt_ns_set_persistent(int mode) { return g_ns_persistent.exchange(mode < 0 ? -1 : (mode ? 1 : 0)); }
int moteopt_ns_set_tall(int on) { return g_ns_tall.exchange(on ? 1 : 0); }

int moteopt_read_status(void* workspace, int* status, float* norm_and_coef, int clear, moteopt_stream_t stream) {
  if (workspace == nullptr) return fail(MOTEOPT_ERR_INVALID, "workspace is null");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Header h;
  MO_CUDA(cudaMemcpyAsync(&h, workspace, sizeof(h), cudaMemcpyDeviceToHost, st));
  MO_CUDA(cudaStreamSynchronize(st));
  if (status) *status = h.status;
  if (norm_and_coef) {
    norm_and_coef[0] = h.norm;
    norm_and_coef[1] = h.coef;
  }
  if (clear) MO_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int), st));
  return MOTEOPT_OK;
}

size_t moteopt_optimizer_step_workspace_size_cfg(const moteopt_muon_param* muon, int n_muon,
                                                 const moteopt_muon_config* cfg, const moteopt_adamw_tensor* adamw,
                                                 int n_adamw) {
  if (n_muon < 0 || n_adamw < 0 || (n_muon > 0 && (!muon || !cfg)) || (n_adamw > 0 && !adamw)) return 0;
  std::vector<int64_t> numels;
  for (int i = 0; i < n_adamw; ++i) numels.push_back(adamw[i].numel);
  for (int i = 0; i < n_muon; ++i) numels.push_back(muon[i].batch * muon[i].rows * muon[i].cols);
  Layout L;
  if (build_layout(muon_shapes(muon, n_muon), numels, cfg ? cfg->ns_steps : 0, &L, cfg ? cfg->ns_variant : 0) !=
      MOTEOPT_OK)
    return 0;
  return L.bytes;
}

size_t moteopt_optimizer_step_workspace_size(const moteopt_muon_param* muon, int n_muon, int ns_steps,
                                             const moteopt_adamw_tensor* adamw, int n_adamw) {
  moteopt_muon_config c;
  std::memset(&c, 0, sizeof(c));
  c.ns_steps = ns_steps;
  return moteopt_optimizer_step_workspace_size_cfg(muon, n_muon, &c, adamw, n_adamw);
}

int moteopt_optimizer_step(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* muon_cfg,
                           const moteopt_adamw_tensor* adamw, int n_adamw, const moteopt_adamw_hparams* adamw_hp,
                           const moteopt_grad_config* grad_cfg, float* out_norm, void* workspace,
                           size_t workspace_bytes, moteopt_stream_t stream) {
  return run_step(muon, n_muon, muon_cfg, adamw, n_adamw, adamw_hp, grad_cfg, nullptr, out_norm, workspace,
                  workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int moteopt_optimizer_step_ex(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* muon_cfg,
                              const moteopt_adamw_tensor* adamw, int n_adamw, const moteopt_adamw_hparams* adamw_hp,
                              const moteopt_grad_config* grad_cfg, const moteopt_step_extras* extras, float* out_norm,
                              void* workspace, size_t workspace_bytes, moteopt_stream_t stream) {
  if (extras != nullptr && extras->lr != nullptr && n_muon > 0 &&
      (extras->muon_wd == nullptr || extras->muon_lr_max == nullptr))
    return fail(MOTEOPT_ERR_INVALID, "extras->lr needs muon_wd and muon_lr_max for the Muon params");
  return run_step(muon, n_muon, muon_cfg, adamw, n_adamw, adamw_hp, grad_cfg, nullptr, out_norm, workspace,
                  workspace_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr, extras);
}

int moteopt_optimizer_step_with_coef(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* muon_cfg,
                                     const moteopt_adamw_tensor* adamw, int n_adamw,
                                     const moteopt_adamw_hparams* adamw_hp, double grad_divisor, const float* grad_coef,
                                     void* workspace, size_t workspace_bytes, moteopt_stream_t stream) {
  moteopt_grad_config gc;
  gc.clip = 0;
  gc.max_norm = 0.0;
  gc.grad_divisor = grad_divisor;
  gc.grad_divisor_device = nullptr;
  return run_step(muon, n_muon, muon_cfg, adamw, n_adamw, adamw_hp, &gc, grad_coef, nullptr, workspace,
                  workspace_bytes, reinterpret_cast<cudaStream_t>(stream));
}

int moteopt_optimizer_step_with_coef_out(const moteopt_muon_param* muon, int n_muon,
                                         const moteopt_muon_config* muon_cfg, const moteopt_adamw_tensor* adamw,
                                         int n_adamw, const moteopt_adamw_hparams* adamw_hp, double grad_divisor,
                                         const float* grad_coef, void* const* muon_updates, void* workspace,
                                         size_t workspace_bytes, moteopt_stream_t stream) {
  if (n_muon > 0 && muon_updates == nullptr) return fail(MOTEOPT_ERR_INVALID, "muon_updates is null");
  for (int i = 0; i < n_muon; ++i)
    if (muon_updates[i] == nullptr) return fail(MOTEOPT_ERR_INVALID, "muon_updates[" + std::to_string(i) + "] is null");
  moteopt_grad_config gc;
  gc.clip = 0;
  gc.max_norm = 0.0;
  gc.grad_divisor = grad_divisor;
  gc.grad_divisor_device = nullptr;
  return run_step(muon, n_muon, muon_cfg, adamw, n_adamw, adamw_hp, &gc, grad_coef, nullptr, workspace,
                  workspace_bytes, reinterpret_cast<cudaStream_t>(stream), muon_updates);
}

size_t moteopt_muon_apply_workspace_size(const moteopt_muon_param* muon, int n) {
  if (n < 0 || (n > 0 && muon == nullptr)) return 0;
  int64_t chunks = 0;
  for (int i = 0; i < n; ++i) chunks += cdiv(std::max<int64_t>(muon[i].batch * muon[i].rows * muon[i].cols, 0), kChunk);
  return sizeof(Header) + static_cast<size_t>(std::max<int64_t>(chunks, 1)) * sizeof(double);   // header, partials
}

int moteopt_muon_apply_ex(const moteopt_muon_param* muon, int n, const moteopt_muon_config* cfg,
                          const void* const* updates, float* const* ema, double ema_weight, float* norms,
                          void* workspace, size_t workspace_bytes, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (muon == nullptr || updates == nullptr)) || cfg == nullptr)
    return fail(MOTEOPT_ERR_INVALID, "moteopt_muon_apply: null argument");
  if (n > kMaxDenom && norms != nullptr)
    return fail(MOTEOPT_ERR_LIMIT, "moteopt_muon_apply: norms of more than 4096 params in one call");
  int sms = 0;
  MO_TRY(device_setup(&sms));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  double* partials = nullptr;
  if (norms != nullptr && n > 0) {
    MO_TRY(check_ws(workspace, workspace_bytes, moteopt_muon_apply_workspace_size(muon, n)));
    partials = reinterpret_cast<double*>(static_cast<char*>(workspace) + sizeof(Header));   // the header stays intact
  }
  std::vector<FlatOutSeg> segs;
  std::vector<int> start(1, 0);
  for (int i = 0; i < n; ++i) {
    const moteopt_muon_param& p = muon[i];
    if (p.param == nullptr || updates[i] == nullptr || p.batch < 1 || p.rows < 1 || p.cols < 1)
      return fail(MOTEOPT_ERR_INVALID, "moteopt_muon_apply: bad entry " + std::to_string(i));
    FlatOutSeg S;   // the same scalars as the in-step apply (muon_apply_table)
    std::memset(&S, 0, sizeof(S));
    S.x = updates[i];
    S.out = p.param;
    S.numel = p.batch * p.rows * p.cols;
    S.neg_lr = static_cast<float>(-p.lr);
    S.has_decay = p.decay != 0.0;
    S.decay_mul = static_cast<float>(1.0 - p.decay);
    S.scale = static_cast<float>(cfg->rms_scale * std::pow(static_cast<double>(std::max(p.rows, p.cols)), 0.5));
    S.ema = ema != nullptr ? ema[i] : nullptr;
    S.partials = partials != nullptr ? partials + start.back() : nullptr;
    start.push_back(start.back() + static_cast<int>(cdiv(S.numel, kChunk)));
    segs.push_back(S);
  }
  MO_TRY(launch_flat_out(segs, 1, sms, st, ema_weight));
  if (partials != nullptr) {   // ||p_new||_F per param: fixed-order fp64 sum of its chunk partials
    static thread_local DenomArgs D;
    std::memset(&D, 0, sizeof(D));
    D.n = n;
    D.base = 0;
    D.eps = 0.f;
    D.partials = partials;
    D.den = norms;
    for (int i = 0; i <= n; ++i) D.chunk_start[i] = start[i];
    mat_denom_kernel<<<(n + 7) / 8, 256, 0, st>>>(D);
    MO_LAUNCHED("mat_denom_kernel");
  }
  return MOTEOPT_OK;
}

int moteopt_muon_apply(const moteopt_muon_param* muon, int n, const moteopt_muon_config* cfg,
                       const void* const* updates, moteopt_stream_t stream) {
  return moteopt_muon_apply_ex(muon, n, cfg, updates, nullptr, 0.0, nullptr, nullptr, 0, stream);
}

int moteopt_ema_lerp(float* const* ema, const float* const* params, const int64_t* numels, int n, double weight,
                     moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (ema == nullptr || params == nullptr || numels == nullptr)))
    return fail(MOTEOPT_ERR_INVALID, "moteopt_ema_lerp: null argument");
  for (int i = 0; i < n; ++i)
    if (numels[i] < 0 || (numels[i] > 0 && (ema[i] == nullptr || params[i] == nullptr)))
      return fail(MOTEOPT_ERR_INVALID, "moteopt_ema_lerp: bad tensor " + std::to_string(i));
  int sms = 0;
  MO_TRY(device_setup(&sms));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  static thread_local LerpArgs A;
  for (int s0 = 0; s0 < n; s0 += kMaxLerpSeg) {
    const int cnt = std::min(n - s0, kMaxLerpSeg);
    std::memset(&A, 0, sizeof(A));
    A.n = cnt;
    A.ema = ema_consts(weight);
    for (int i = 0; i < cnt; ++i) {
      A.seg[i] = LerpSeg{ema[s0 + i], params[s0 + i], numels[s0 + i]};
      if (cdiv(numels[s0 + i], kChunk) > (1 << 30) - A.chunk_start[i])
        return fail(MOTEOPT_ERR_LIMIT, "moteopt_ema_lerp: too many elements in one call");
      A.chunk_start[i + 1] = A.chunk_start[i] + static_cast<int>(cdiv(numels[s0 + i], kChunk));
    }
    if (A.chunk_start[cnt] == 0) continue;
    ema_lerp_kernel<<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("ema_lerp_kernel");
  }
  return MOTEOPT_OK;
}

size_t moteopt_grad_sumsq_workspace_size(const int64_t* numels, int n) {
  return moteopt_clip_grad_norm_workspace_size(numels, n);
}

int moteopt_grad_sumsq(const void* const* grads, const int64_t* numels, const int* dtypes, int n, double grad_divisor,
                       double* out_sum, void* workspace, size_t workspace_bytes, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (!grads || !numels || !dtypes)) || out_sum == nullptr)
    return fail(MOTEOPT_ERR_INVALID, "bad grad list or null output");
  for (int i = 0; i < n; ++i) {
    if (dtypes[i] != kF32 && dtypes[i] != kBF16) return fail(MOTEOPT_ERR_INVALID, "grad dtype must be fp32 or bf16");
    if (numels[i] < 0 || (numels[i] > 0 && grads[i] == nullptr)) return fail(MOTEOPT_ERR_INVALID, "bad grad tensor");
  }
  int sms = 0;
  MO_TRY(device_setup(&sms));
  Layout L;
  MO_TRY(build_layout({}, std::vector<int64_t>(numels, numels + n), 0, &L));
  MO_TRY(check_ws(workspace, workspace_bytes, L.bytes));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  std::vector<GradSource> src;
  for (int i = 0; i < n; ++i) src.push_back(GradSource{grads[i], numels[i], dtypes[i]});
  double* partials = reinterpret_cast<double*>(ws + L.off_norm);
  const bool has_div = grad_divisor != 0.0 && grad_divisor != 1.0;
  MO_TRY(launch_sumsq(src, L.norm_tensor_chunk_start, partials, has_div, has_div ? static_cast<float>(grad_divisor) : 1.f,
                      sms, st));
  partials_total_kernel<<<1, 1024, 0, st>>>(partials, L.norm_tensor_chunk_start.back(), out_sum);
  MO_LAUNCHED("partials_total_kernel");
  return MOTEOPT_OK;
}

int moteopt_clip_coef_from_sums(const double* sums, int n, int clip, double max_norm, float* out_norm_coef,
                                moteopt_stream_t stream) {
  if (n < 1 || sums == nullptr || out_norm_coef == nullptr) return fail(MOTEOPT_ERR_INVALID, "bad sums");
  int sms = 0;
  MO_TRY(device_setup(&sms));
  CoefArgs A;
  A.n = n;
  A.has_clip = clip != 0;
  A.max_norm = static_cast<float>(max_norm);
  A.sums = sums;
  A.out = out_norm_coef;
  A.status = nullptr;
  coef_from_sums_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(A);
  MO_LAUNCHED("coef_from_sums_kernel");
  return MOTEOPT_OK;
}

// piece_sums_kernel over pieces [0, n) whose chunk partials start at chunk_start[p] (a prefix array of n + 1)
static int launch_piece_sums(const std::vector<int>& chunk_start, const int* tensors, int n, int n_tensors,
                             const double* partials, double* out, cudaStream_t st) {
  if (n > kMaxPieceSums) return fail(MOTEOPT_ERR_LIMIT, "more than 2048 grad pieces in one call");
  static thread_local PieceSumArgs A;
  std::memset(&A, 0, sizeof(A));
  A.n_pieces = n;
  A.n_tensors = n_tensors;
  A.partials = partials;
  A.out = out;
  for (int p = 0; p <= n; ++p) A.chunk_start[p] = chunk_start[p];
  for (int p = 0; p < n; ++p) A.tensor[p] = tensors[p];
  piece_sums_kernel<<<1, 1024, 0, st>>>(A);
  MO_LAUNCHED("piece_sums_kernel");
  return MOTEOPT_OK;
}

static int check_tensor_ids(const int* tensors, int n, int n_tensors) {
  if (n_tensors < 1 || n_tensors > kMaxFinalTensors) return fail(MOTEOPT_ERR_LIMIT, "n_tensors must be 1..4096");
  std::vector<char> seen(static_cast<size_t>(n_tensors), 0);
  for (int p = 0; p < n; ++p) {
    if (tensors[p] < 0 || tensors[p] >= n_tensors) return fail(MOTEOPT_ERR_INVALID, "tensor index out of range");
    if (seen[tensors[p]]) return fail(MOTEOPT_ERR_INVALID, "two pieces of one tensor in one call");
    seen[tensors[p]] = 1;
  }
  return MOTEOPT_OK;
}

int moteopt_grad_sumsq_tensors(const void* const* grads, const int64_t* numels, const int* dtypes, const int* tensors,
                               int n, int n_tensors, double grad_divisor, double* out_tensor_sums, void* workspace,
                               size_t workspace_bytes, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (!grads || !numels || !dtypes || !tensors)) || out_tensor_sums == nullptr)
    return fail(MOTEOPT_ERR_INVALID, "bad grad list or null output");
  for (int i = 0; i < n; ++i) {
    if (dtypes[i] != kF32 && dtypes[i] != kBF16) return fail(MOTEOPT_ERR_INVALID, "grad dtype must be fp32 or bf16");
    if (numels[i] < 0 || (numels[i] > 0 && grads[i] == nullptr)) return fail(MOTEOPT_ERR_INVALID, "bad grad tensor");
  }
  MO_TRY(check_tensor_ids(tensors, n, n_tensors));
  int sms = 0;
  MO_TRY(device_setup(&sms));
  Layout L;
  MO_TRY(build_layout({}, std::vector<int64_t>(numels, numels + n), 0, &L));
  MO_TRY(check_ws(workspace, workspace_bytes, L.bytes));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  std::vector<GradSource> src;
  for (int i = 0; i < n; ++i) src.push_back(GradSource{grads[i], numels[i], dtypes[i]});
  double* partials = reinterpret_cast<double*>(ws + L.off_norm);
  const bool has_div = grad_divisor != 0.0 && grad_divisor != 1.0;
  MO_TRY(launch_sumsq(src, L.norm_tensor_chunk_start, partials, has_div, has_div ? static_cast<float>(grad_divisor) : 1.f,
                      sms, st));
  return launch_piece_sums(L.norm_tensor_chunk_start, tensors, n, n_tensors, partials, out_tensor_sums, st);
}

size_t moteopt_peer_reduce_workspace_size(const moteopt_peer_piece* pieces, int n_pieces) {
  if (n_pieces < 0 || (n_pieces > 0 && pieces == nullptr)) return 0;
  std::vector<int64_t> numels;
  for (int p = 0; p < n_pieces; ++p) numels.push_back(pieces[p].numel);
  return moteopt_grad_sumsq_workspace_size(numels.data(), n_pieces);
}

int moteopt_peer_reduce_sumsq(const moteopt_peer_piece* pieces, int n_pieces, int world, int n_tensors,
                              double grad_divisor, double* out_tensor_sums, void* workspace, size_t workspace_bytes,
                              moteopt_stream_t stream) {
  static_assert(MOTEOPT_MAX_PEERS == kMaxPeers, "peer count");
  if (n_pieces < 0 || (n_pieces > 0 && pieces == nullptr) || out_tensor_sums == nullptr)
    return fail(MOTEOPT_ERR_INVALID, "bad piece list or null output");
  if (world < 1 || world > kMaxPeers) return fail(MOTEOPT_ERR_LIMIT, "world must be 1..8");
  std::vector<int64_t> numels;
  std::vector<int> tensors;
  for (int p = 0; p < n_pieces; ++p) {
    const moteopt_peer_piece& P = pieces[p];
    if (P.dtype != kF32 && P.dtype != kBF16) return fail(MOTEOPT_ERR_INVALID, "grad dtype must be fp32 or bf16");
    if (P.numel < 0) return fail(MOTEOPT_ERR_INVALID, "negative piece size");
    if (P.numel > 0) {
      if (P.dst == nullptr) return fail(MOTEOPT_ERR_INVALID, "null piece destination");
      for (int q = 0; q < world; ++q)
        if (P.src[q] == nullptr) return fail(MOTEOPT_ERR_INVALID, "null piece source");
    }
    numels.push_back(P.numel);
    tensors.push_back(P.tensor);
  }
  MO_TRY(check_tensor_ids(tensors.data(), n_pieces, n_tensors));
  int sms = 0;
  MO_TRY(device_setup(&sms));
  Layout L;
  MO_TRY(build_layout({}, numels, 0, &L));
  MO_TRY(check_ws(workspace, workspace_bytes, L.bytes));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  double* partials = reinterpret_cast<double*>(static_cast<char*>(workspace) + L.off_norm);
  const std::vector<int>& cs = L.norm_tensor_chunk_start;
  static thread_local PeerReduceArgs A;
  const bool has_div = grad_divisor != 0.0 && grad_divisor != 1.0;
  for (int s0 = 0; s0 < n_pieces; s0 += kMaxPeerSegs) {
    const int n = std::min(n_pieces - s0, kMaxPeerSegs);
    std::memset(&A, 0, sizeof(A));
    A.n = n;
    A.world = world;
    A.has_div = has_div;
    A.div = has_div ? static_cast<float>(grad_divisor) : 1.f;
    A.partials = partials;
    A.chunk_base = cs[s0];
    for (int i = 0; i < n; ++i) {
      const moteopt_peer_piece& P = pieces[s0 + i];
      A.seg[i].dst = P.dst;
      for (int q = 0; q < world; ++q) A.seg[i].src[q] = P.src[q];
      A.seg[i].numel = P.numel;
      A.seg[i].dtype = P.dtype;
      A.chunk_start[i] = cs[s0 + i] - A.chunk_base;
    }
    A.chunk_start[n] = cs[s0 + n] - A.chunk_base;
    if (A.chunk_start[n] == 0) continue;
    // two blocks of 256 threads per SM, each thread with 128 bytes of loads in flight
    const int grid = std::max(1, std::min(A.chunk_start[n], sms * 2));
    const int kw = world <= 1 ? 1 : world <= 2 ? 2 : world <= 4 ? 4 : 8;
    auto go = [&](auto div_tag) {
      constexpr bool kDiv = decltype(div_tag)::value;
      switch (kw) {
        case 1: peer_reduce_kernel<kDiv, 1><<<grid, kMtThreads, 0, st>>>(A); break;
        case 2: peer_reduce_kernel<kDiv, 2><<<grid, kMtThreads, 0, st>>>(A); break;
        case 4: peer_reduce_kernel<kDiv, 4><<<grid, kMtThreads, 0, st>>>(A); break;
        default: peer_reduce_kernel<kDiv, 8><<<grid, kMtThreads, 0, st>>>(A); break;
      }
    };
    if (has_div) go(std::true_type{});
    else go(std::false_type{});
    MO_LAUNCHED("peer_reduce_kernel");
  }
  return launch_piece_sums(cs, tensors.data(), n_pieces, n_tensors, partials, out_tensor_sums, st);
}

int moteopt_clip_coef_from_tensor_sums(const double* sums, int world, int n_tensors, int clip, double max_norm,
                                       float* out_norm_coef, moteopt_stream_t stream) {
  if (world < 1 || sums == nullptr || out_norm_coef == nullptr) return fail(MOTEOPT_ERR_INVALID, "bad sums");
  if (n_tensors < 1 || n_tensors > kMaxFinalTensors) return fail(MOTEOPT_ERR_LIMIT, "n_tensors must be 1..4096");
  int sms = 0;
  MO_TRY(device_setup(&sms));
  TensorCoefArgs A;
  A.world = world;
  A.n_tensors = n_tensors;
  A.has_clip = clip != 0;
  A.max_norm = static_cast<float>(max_norm);
  A.sums = sums;
  A.out = out_norm_coef;
  A.status = nullptr;
  tensor_coef_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(A);
  MO_LAUNCHED("tensor_coef_kernel");
  return MOTEOPT_OK;
}

size_t moteopt_muon_step_workspace_size_cfg(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* cfg) {
  if (n_muon < 0 || (n_muon > 0 && (!muon || !cfg))) return 0;
  Layout L;
  if (build_layout(muon_shapes(muon, n_muon), {}, cfg ? cfg->ns_steps : 0, &L, cfg ? cfg->ns_variant : 0) != MOTEOPT_OK)
    return 0;
  return L.bytes;
}

size_t moteopt_muon_step_workspace_size(const moteopt_muon_param* muon, int n_muon, int ns_steps) {
  moteopt_muon_config c;
  std::memset(&c, 0, sizeof(c));
  c.ns_steps = ns_steps;
  return moteopt_muon_step_workspace_size_cfg(muon, n_muon, &c);
}

int moteopt_muon_step(const moteopt_muon_param* muon, int n_muon, const moteopt_muon_config* cfg,
                      const float* grad_scale, void* workspace, size_t workspace_bytes, moteopt_stream_t stream) {
  return run_step(muon, n_muon, cfg, nullptr, 0, nullptr, nullptr, grad_scale, nullptr, workspace, workspace_bytes,
                  reinterpret_cast<cudaStream_t>(stream));
}

int moteopt_adamw_step(const moteopt_adamw_tensor* adamw, int n_adamw, const moteopt_adamw_hparams* hp,
                       const float* grad_scale, moteopt_stream_t stream) {
  int r = check_adamw(adamw, n_adamw, hp);
  if (r != MOTEOPT_OK) return r;
  int sms = 0;
  r = device_setup(&sms);
  if (r != MOTEOPT_OK) return r;
  return launch_adamw(adamw, n_adamw, hp, false, 1.0f, grad_scale, sms, reinterpret_cast<cudaStream_t>(stream));
}

int moteopt_moe_update_bias(const moteopt_moe_bias* layers, int n, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && layers == nullptr)) return fail(MOTEOPT_ERR_INVALID, "bad MoE layer list");
  for (int i = 0; i < n; ++i) {
    const moteopt_moe_bias& x = layers[i];
    if (x.n_experts < 0) return fail(MOTEOPT_ERR_INVALID, "MoE layer " + std::to_string(i) + ": negative n_experts");
    if (x.n_experts > 0 && (x.load_acc == nullptr || x.expert_bias == nullptr))
      return fail(MOTEOPT_ERR_INVALID, "MoE layer " + std::to_string(i) + ": null pointer");
  }
  int sms = 0;
  int r = device_setup(&sms);
  if (r != MOTEOPT_OK) return r;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  static thread_local MoeBiasArgs A;
  A.n = 0;
  for (int i = 0; i <= n; ++i) {
    if (i == n || A.n == kMaxMoeLayers) {   // flush a full argument block, and the last one
      if (A.n > 0) {
        moe_bias_kernel<<<A.n, kMtThreads, 0, st>>>(A);
        MO_LAUNCHED("moe_bias_kernel");
      }
      A.n = 0;
    }
    if (i < n && layers[i].n_experts > 0)
      A.layer[A.n++] = MoeLayer{layers[i].load_acc, layers[i].expert_bias, layers[i].n_experts, layers[i].gamma};
  }
  return MOTEOPT_OK;
}

size_t moteopt_clip_grad_norm_workspace_size(const int64_t* numels, int n) {
  if (n < 0 || (n > 0 && !numels)) return 0;
  Layout L;
  if (build_layout({}, std::vector<int64_t>(numels, numels + n), 0, &L) != MOTEOPT_OK) return 0;
  return L.bytes;
}

int moteopt_clip_grad_norm(void* const* grads, const int64_t* numels, const int* dtypes, int n, double max_norm,
                           float* out_norm, void* workspace, size_t workspace_bytes, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (!grads || !numels || !dtypes))) return fail(MOTEOPT_ERR_INVALID, "bad grad list");
  if (n > kMaxFinalTensors) return fail(MOTEOPT_ERR_LIMIT, "more than 4096 tensors in one clip_grad_norm call");
  for (int i = 0; i < n; ++i) {
    if (dtypes[i] != kF32 && dtypes[i] != kBF16) return fail(MOTEOPT_ERR_INVALID, "grad dtype must be fp32 or bf16");
    if (numels[i] < 0 || (numels[i] > 0 && grads[i] == nullptr)) return fail(MOTEOPT_ERR_INVALID, "bad grad tensor");
  }
  int sms = 0;
  int r = device_setup(&sms);
  if (r != MOTEOPT_OK) return r;
  Layout L;
  r = build_layout({}, std::vector<int64_t>(numels, numels + n), 0, &L);
  if (r != MOTEOPT_OK) return r;
  r = check_ws(workspace, workspace_bytes, L.bytes);
  if (r != MOTEOPT_OK) return r;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  Header* hdr = reinterpret_cast<Header*>(ws);
  MO_CUDA(cudaMemsetAsync(hdr, 0, sizeof(Header), st));
  std::vector<GradSource> src;
  for (int i = 0; i < n; ++i) src.push_back(GradSource{grads[i], numels[i], dtypes[i]});
  double* partials = reinterpret_cast<double*>(ws + L.off_norm);
  r = launch_sumsq(src, L.norm_tensor_chunk_start, partials, false, 1.0f, sms, st);
  if (r != MOTEOPT_OK) return r;
  r = launch_finalize(L.norm_tensor_chunk_start, partials, true, max_norm, &hdr->norm, &hdr->status, st);
  if (r != MOTEOPT_OK) return r;
  ScaleArgs A;
  std::memset(&A, 0, sizeof(A));
  A.coef = &hdr->coef;
  for (int s0 = 0; s0 < n; s0 += kMaxNormSeg) {
    const int cnt = std::min(n - s0, kMaxNormSeg);
    A.n = cnt;
    A.chunk_start[0] = 0;
    for (int i = 0; i < cnt; ++i) {
      A.seg[i] = SumsqSeg{grads[s0 + i], numels[s0 + i], dtypes[s0 + i], 0};
      A.chunk_start[i + 1] = A.chunk_start[i] + static_cast<int>(cdiv(numels[s0 + i], kChunk));
    }
    if (A.chunk_start[cnt] == 0) continue;
    clip_scale_kernel<<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("clip_scale_kernel");
  }
  if (out_norm != nullptr) MO_CUDA(cudaMemcpyAsync(out_norm, &hdr->norm, sizeof(float), cudaMemcpyDeviceToDevice, st));
  return MOTEOPT_OK;
}

// ---- clip_grad_norm_ without a caller-provided workspace ------------------------------------------------------
// Scratch of moteopt_clip_grad_norm_noalloc: one fp64 sum of squares per 16K-element chunk plus a 256-byte header
// (status, norm, clip coefficient), in a file-scope device array. Every device that loads this library holds it
// (512 KB + 256 B) until the process exits; all calls on a device share it.
}  // extern "C"

namespace {
constexpr int kNoAllocMaxChunks = 65536;   // 65536 x 16384 = 2^30 grad elements per call
constexpr size_t kNoAllocBytes = kHeaderBytes + sizeof(double) * static_cast<size_t>(kNoAllocMaxChunks);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// The device address of the scratch array for the current device (host code cannot use the symbol itself).
int noalloc_scratch(void** out) {
  int dev = 0;
  MO_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MOTEOPT_ERR_DEVICE, "device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    MO_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return MOTEOPT_OK;
}
}  // namespace

extern "C" {

int moteopt_clip_grad_norm_noalloc(void* const* grads, const int64_t* numels, const int* dtypes, int n,
                                   double max_norm, float* out_norm, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (!grads || !numels || !dtypes))) return fail(MOTEOPT_ERR_INVALID, "bad grad list");
  if (n > kMaxFinalTensors) return fail(MOTEOPT_ERR_LIMIT, "more than 4096 tensors in one clip_grad_norm call");
  int64_t chunks = 0;
  for (int i = 0; i < n; ++i) {
    if (dtypes[i] != kF32 && dtypes[i] != kBF16) return fail(MOTEOPT_ERR_INVALID, "grad dtype must be fp32 or bf16");
    if (numels[i] < 0 || (numels[i] > 0 && grads[i] == nullptr)) return fail(MOTEOPT_ERR_INVALID, "bad grad tensor");
    chunks += cdiv(numels[i], kChunk);
  }
  if (chunks > kNoAllocMaxChunks)
    return fail(MOTEOPT_ERR_LIMIT, "moteopt_clip_grad_norm_noalloc: " + std::to_string(chunks) +
                                       " chunks of 16384 elements (the per-tensor element counts rounded up) exceed "
                                       "its fixed scratch of " + std::to_string(kNoAllocMaxChunks) +
                                       "; use moteopt_clip_grad_norm with a workspace");
  int sms = 0;
  int r = device_setup(&sms);
  if (r != MOTEOPT_OK) return r;
  void* scratch = nullptr;
  r = noalloc_scratch(&scratch);
  if (r != MOTEOPT_OK) return r;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(scratch);
  Header* hdr = reinterpret_cast<Header*>(ws);
  double* partials = reinterpret_cast<double*>(ws + kHeaderBytes);
  // the header carries the previous call's status bits: clear it (every partial is overwritten)
  MO_CUDA(cudaMemsetAsync(hdr, 0, sizeof(Header), st));
  // fixed-size argument blocks on the stack: no host or device allocation on this path
  SumsqArgs S;
  FinalizeArgs F;
  ScaleArgs A;
  F.n_tensors = n;
  F.has_clip = 1;
  F.max_norm = static_cast<float>(max_norm);
  F.partials = partials;
  F.out = &hdr->norm;
  F.status = &hdr->status;
  F.tensor_chunk_start[0] = 0;
  for (int i = 0; i < n; ++i)
    F.tensor_chunk_start[i + 1] = F.tensor_chunk_start[i] + static_cast<int>(cdiv(numels[i], kChunk));
  S.partials = partials;
  S.has_div = 0;
  S.div = 1.0f;
  S.div_dev = nullptr;
  A.coef = &hdr->coef;
  for (int s0 = 0; s0 < n; s0 += kMaxNormSeg) {
    const int cnt = std::min(n - s0, kMaxNormSeg);
    S.n = cnt;
    S.chunk_base = F.tensor_chunk_start[s0];
    for (int i = 0; i < cnt; ++i) {
      S.seg[i] = SumsqSeg{grads[s0 + i], numels[s0 + i], dtypes[s0 + i], 0};
      S.chunk_start[i] = F.tensor_chunk_start[s0 + i] - S.chunk_base;
    }
    S.chunk_start[cnt] = F.tensor_chunk_start[s0 + cnt] - S.chunk_base;
    if (S.chunk_start[cnt] == 0) continue;
    if (S.has_div) sumsq_kernel<true><<<grid_for(S.chunk_start[cnt], sms), kMtThreads, 0, st>>>(S);
    else sumsq_kernel<false><<<grid_for(S.chunk_start[cnt], sms), kMtThreads, 0, st>>>(S);
    MO_LAUNCHED("sumsq_kernel");
  }
  norm_finalize_kernel<<<1, 1024, 0, st>>>(F);
  MO_LAUNCHED("norm_finalize_kernel");
  for (int s0 = 0; s0 < n; s0 += kMaxNormSeg) {
    const int cnt = std::min(n - s0, kMaxNormSeg);
    A.n = cnt;
    for (int i = 0; i < cnt; ++i) {
      A.seg[i] = SumsqSeg{grads[s0 + i], numels[s0 + i], dtypes[s0 + i], 0};
      A.chunk_start[i] = F.tensor_chunk_start[s0 + i] - F.tensor_chunk_start[s0];
    }
    A.chunk_start[cnt] = F.tensor_chunk_start[s0 + cnt] - F.tensor_chunk_start[s0];
    if (A.chunk_start[cnt] == 0) continue;
    clip_scale_kernel<<<grid_for(A.chunk_start[cnt], sms), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("clip_scale_kernel");
  }
  if (out_norm != nullptr) MO_CUDA(cudaMemcpyAsync(out_norm, &hdr->norm, sizeof(float), cudaMemcpyDeviceToDevice, st));
  return MOTEOPT_OK;
}

size_t moteopt_newton_schulz_workspace_size_variant(int64_t batch, int64_t rows, int64_t cols, int ns_variant) {
  Layout L;
  if (build_layout({std::make_tuple(batch, rows, cols)}, {}, 1, &L, ns_variant) != MOTEOPT_OK) return 0;
  return L.bytes;
}

size_t moteopt_newton_schulz_workspace_size(int64_t batch, int64_t rows, int64_t cols) {
  return moteopt_newton_schulz_workspace_size_variant(batch, rows, cols, 0);
}

int moteopt_newton_schulz(const void* G, int g_dtype, void* out, int64_t batch, int64_t rows, int64_t cols, int steps,
                          double eps, void* workspace, size_t workspace_bytes, moteopt_stream_t stream) {
  return moteopt_newton_schulz_variant(G, g_dtype, out, batch, rows, cols, steps, eps, 0, workspace, workspace_bytes,
                                       stream);
}

int moteopt_newton_schulz_variant(const void* G, int g_dtype, void* out, int64_t batch, int64_t rows, int64_t cols,
                                  int steps, double eps, int ns_variant, void* workspace, size_t workspace_bytes,
                                  moteopt_stream_t stream) {
  if (!G || !out) return fail(MOTEOPT_ERR_INVALID, "null input or output");
  if (g_dtype != kF32 && g_dtype != kBF16) return fail(MOTEOPT_ERR_INVALID, "G must be fp32 or bf16");
  if (steps < 0 || steps > 100) return fail(MOTEOPT_ERR_INVALID, "steps out of range");
  int sms = 0;
  int r = device_setup(&sms);
  if (r != MOTEOPT_OK) return r;
  Layout L;
  r = build_layout({std::make_tuple(batch, rows, cols)}, {}, 1, &L, ns_variant);
  if (r != MOTEOPT_OK) return r;
  r = check_ws(workspace, workspace_bytes, L.bytes);
  if (r != MOTEOPT_OK) return r;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  Header* hdr = reinterpret_cast<Header*>(ws);
  MO_CUDA(cudaMemsetAsync(hdr, 0, sizeof(Header), st));
  const size_t esz = g_dtype == kBF16 ? 2 : 4;
  const int64_t per = rows * cols;
  // per-matrix sum of squares, in the layout's matrix order
  std::vector<GradSource> src;
  std::vector<const GroupPlan*> gofm;
  std::vector<int> posm;
  for (const GroupPlan& g : L.groups)
    for (size_t k = 0; k < g.mats.size(); ++k) {
      src.push_back(GradSource{static_cast<const char*>(G) + static_cast<size_t>(g.mats[k].slice) * per * esz, per, g_dtype});
      gofm.push_back(&g);
      posm.push_back(static_cast<int>(k));
    }
  double* partials = reinterpret_cast<double*>(ws + L.off_mom);
  r = launch_sumsq(src, L.mat_chunk_start, partials, false, 1.0f, sms, st);
  if (r != MOTEOPT_OK) return r;
  float* den = reinterpret_cast<float*>(ws + L.off_den);
  r = launch_denoms(L, partials, den, static_cast<float>(eps), st);
  if (r != MOTEOPT_OK) return r;
  NormArgs A;
  std::memset(&A, 0, sizeof(A));
  A.den = den;
  const int nm = static_cast<int>(src.size());
  for (int s0 = 0; s0 < nm; s0 += kMaxNormMat) {
    const int cnt = std::min(nm - s0, kMaxNormMat);
    A.n = cnt;
    int max_tiles = 0;
    for (int i = 0; i < cnt; ++i) {
      const GroupPlan& g = *gofm[s0 + i];
      NormMat& M = A.mat[i];
      M.g = src[s0 + i].g;
      M.buf = nullptr;
      M.x = ws + g.off_x0 + static_cast<size_t>(posm[s0 + i]) * g.m * g.n * 2;
      M.rows = g.rows;
      M.cols = g.cols;
      M.m_pad = g.tall ? g.n : g.m;   // X's rows and columns (a tall X has the matrix's own layout)
      M.n_pad = g.tall ? g.m : g.n;
      M.transposed = g.tall ? 0 : g.transposed;
      M.dtype = g_dtype;
      M.den_index = s0 + i;
      M.tiles_x = static_cast<int>(cdiv(M.n_pad, kNormTile));
      M.tiles = M.tiles_x * static_cast<int>(cdiv(M.m_pad, kNormTile));
      max_tiles = std::max(max_tiles, M.tiles);
    }
    if (A.has_div) ns_normalize_kernel<true><<<dim3(max_tiles, cnt), kMtThreads, 0, st>>>(A);
    else ns_normalize_kernel<false><<<dim3(max_tiles, cnt), kMtThreads, 0, st>>>(A);
    MO_LAUNCHED("ns_normalize_kernel");
  }
  r = run_ns(L, ws, steps, &hdr->status, st);
  if (r != MOTEOPT_OK) return r;
  // copy out (transpose back)
  OutArgs O;
  std::memset(&O, 0, sizeof(O));
  O.apply = 0;
  int k = 0;
  std::vector<OutMat> all;
  for (const GroupPlan& g : L.groups)
    for (size_t pos = 0; pos < g.mats.size(); ++pos, ++k) {
      OutMat M;
      std::memset(&M, 0, sizeof(M));
      M.x = ws + (out_buffer(g, steps) ? g.off_x1 : g.off_x0) + pos * g.m * g.n * 2;
      M.out = static_cast<char*>(out) + static_cast<size_t>(g.mats[pos].slice) * per * 2;
      M.rows = g.rows;
      M.cols = g.cols;
      M.m_pad = g.tall ? g.n : g.m;
      M.n_pad = g.tall ? g.m : g.n;
      M.transposed = g.tall ? 0 : g.transposed;
      M.tiles_x = static_cast<int>(cdiv(g.cols, kNormTile));
      M.tiles = M.tiles_x * static_cast<int>(cdiv(g.rows, kNormTile));
      all.push_back(M);
    }
  for (size_t s0 = 0; s0 < all.size(); s0 += kMaxOutMat) {
    const size_t cnt = std::min(all.size() - s0, static_cast<size_t>(kMaxOutMat));
    O.n = static_cast<int>(cnt);
    int max_tiles = 0;
    for (size_t i = 0; i < cnt; ++i) {
      O.mat[i] = all[s0 + i];
      max_tiles = std::max(max_tiles, O.mat[i].tiles);
    }
    if (out_has_ema(O, cnt)) ns_out_kernel<true><<<dim3(max_tiles, static_cast<unsigned>(cnt)), kMtThreads, 0, st>>>(O);
    else ns_out_kernel<false><<<dim3(max_tiles, static_cast<unsigned>(cnt)), kMtThreads, 0, st>>>(O);
    MO_LAUNCHED("ns_out_kernel");
  }
  return MOTEOPT_OK;
}

}  // extern "C"

// ---- self-tests of two device primitives (diagnostics; no counterpart in the reference) ---------------------------
namespace {

// out[i] = a[i] / d[i] by SharedDivisor (the normalisation's quotient: reciprocal + one Markstein correction)
__global__ void selftest_divide_kernel(const float* a, const float* d, float* out, int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = shared_divisor(d[i]).div(a[i]);
}

// out[i] = a[i] / d with one SharedDivisor for the whole pass, as the normalisation divides a matrix by its norm:
// groups of four through div4, the tail through div
__global__ void selftest_grad_divide_kernel(const float* a, float d, float* out, int64_t n) {
  const SharedDivisor g = shared_divisor(d);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; 4 * j < n; j += stride) {
    const int64_t i = 4 * j;
    if (i + 3 < n) {
      const float4 q = g.div4(make_float4(a[i], a[i + 1], a[i + 2], a[i + 3]));
      out[i] = q.x;
      out[i + 1] = q.y;
      out[i + 2] = q.z;
      out[i + 3] = q.w;
    } else {
      for (int64_t k = i; k < n; ++k) out[k] = g.div(a[k]);
    }
  }
}

// Two CTAs, one waiting thread each, on something that never completes: mode 0 a completion counter nothing adds to
// (wait_counter, as a persistent Newton-Schulz tile waits for its inputs), mode 1 an mbarrier nothing arrives on
// (mbar_wait, as a pipeline stage waits for its loads). CTA 0 gives up after limit_ns and records the timeout; CTA 1
// waits with four times the limit and, in mode 0, must give up as soon as it sees CTA 0's timeout in the status
// word, as the other CTAs of a launch do. Each CTA records how long it waited (elapsed_ns[blockIdx.x]) and, like the
// Newton-Schulz kernel at its exit, MOTEOPT_STATUS_ABORTED when it unwound.
__global__ void selftest_wait_kernel(int* counter, int* status, int mode, unsigned long long limit_ns,
                                     unsigned long long* elapsed_ns) {
  __shared__ uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const WaitCtx ctx{&abort_flag, status, blockIdx.x == 0 ? limit_ns : 4 * limit_ns};
    const unsigned long long t0 = globaltimer_ns();
    const bool ok = mode == 0 ? wait_counter(counter, 1, ctx) : mbar_wait(&bar, 0, ctx);
    elapsed_ns[blockIdx.x] = globaltimer_ns() - t0;
    if (!ok) atomicOr(status, kStatusAborted);
  }
}

}  // namespace

extern "C" {

int moteopt_selftest_divide(const float* a, const float* d, float* out, int64_t n, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (!a || !d || !out))) return fail(MOTEOPT_ERR_INVALID, "moteopt_selftest_divide: bad arguments");
  int sms = 0;
  MO_TRY(device_setup(&sms));
  if (n == 0) return MOTEOPT_OK;
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(n, 256), 8 * sms));
  selftest_divide_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a, d, out, n);
  MO_LAUNCHED("selftest_divide_kernel");
  return MOTEOPT_OK;
}

int moteopt_selftest_grad_divide(const float* a, float d, float* out, int64_t n, moteopt_stream_t stream) {
  if (n < 0 || (n > 0 && (!a || !out))) return fail(MOTEOPT_ERR_INVALID, "moteopt_selftest_grad_divide: bad arguments");
  int sms = 0;
  MO_TRY(device_setup(&sms));
  if (n == 0) return MOTEOPT_OK;
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(cdiv(n, 4), 256), 8 * sms));
  selftest_grad_divide_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a, d, out, n);
  MO_LAUNCHED("selftest_grad_divide_kernel");
  return MOTEOPT_OK;
}

int moteopt_selftest_wait_timeout(int mode, double limit_seconds, int* counter, int* status,
                                  unsigned long long* elapsed_ns, moteopt_stream_t stream) {
  if ((mode != 0 && mode != 1) || !counter || !status || !elapsed_ns)
    return fail(MOTEOPT_ERR_INVALID, "moteopt_selftest_wait_timeout: bad arguments");
  if (!(limit_seconds >= 1e-6 && limit_seconds <= 0.25))
    return fail(MOTEOPT_ERR_INVALID, "moteopt_selftest_wait_timeout: the limit must lie in [1 us, 0.25 s]");
  int sms = 0;
  MO_TRY(device_setup(&sms));
  selftest_wait_kernel<<<2, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      counter, status, mode, static_cast<unsigned long long>(limit_seconds * 1e9), elapsed_ns);
  MO_LAUNCHED("selftest_wait_kernel");
  return MOTEOPT_OK;
}

}  // extern "C"
