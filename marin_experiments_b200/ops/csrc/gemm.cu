// Host side of the sm_100a GEMM: TMA tensor-map encoding, argument validation and the
// (BN, operand majors, epilogue) dispatch table.
#include <cuda.h>
#include <cuda_runtime.h>

#include <dlfcn.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <utility>
#include <vector>

#include "gemm_sm100.cuh"
#include "kernels.h"
#include "launch.h"

namespace mxk {

static bool trace_on() {
  static int on = -1;
  if (on < 0) on = std::getenv("MXK_TRACE") ? 1 : 0;
  return on == 1;
}
#define MXK_TRACE(msg) \
  do { if (trace_on()) { std::fprintf(stderr, "[mxk] %s\n", msg); std::fflush(stderr); } } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The driver's cuTensorMapEncodeTiled and cuCtxGetCurrent, resolved with dlsym from libcuda.so.1
// (already loaded by the CUDA runtime).
static void* driver_sym(const char* name) {
  void* lib = dlopen("libcuda.so.1", RTLD_NOW | RTLD_NOLOAD);
  if (!lib) lib = dlopen("libcuda.so.1", RTLD_NOW);
  return lib ? dlsym(lib, name) : nullptr;
}

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] { fn = reinterpret_cast<EncodeTiledFn>(driver_sym("cuTensorMapEncodeTiled")); });
  return fn;
}

// The runtime binds its primary context to a thread lazily, on the first runtime call that needs
// it. Threads that only queried state so far (autograd's device threads run backward on their
// own) have no current driver context, and encoding a tensor map there faulted inside the driver.
// Bind the context of the runtime's current device first.
static void ensure_current_context() {
  static CtxGetCurrentFn get = nullptr;
  static std::once_flag once;
  std::call_once(once, [] { get = reinterpret_cast<CtxGetCurrentFn>(driver_sym("cuCtxGetCurrent")); });
  CUcontext ctx = nullptr;
  if (get && get(&ctx) == CUDA_SUCCESS && ctx != nullptr) return;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaSetDevice(dev);
  cudaFree(nullptr);
}

// 2-D bf16 tensor map over a row-major matrix [outer, inner] with row stride `ld` elements,
// 128-byte swizzle, box {box_inner, box_outer}. Out-of-bounds elements read as zero.
bool make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                       int box_outer) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  ensure_current_context();
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The same with a 64-byte swizzle: box_inner * 2 must be 64 (a 32-column bf16 chunk whose rows are
// one 64-byte swizzle row each).
bool make_tmap_bf16_2d_sw64(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld,
                            int box_inner, int box_outer) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc || box_inner * 2 != 64) return false;
  ensure_current_context();
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D tensor map for an epilogue output: 64-byte-wide boxes of 32 rows (16 fp32 or 32 bf16
// columns), 64-byte swizzle (matches the staging layout in gemm_sm100.cuh).
bool make_tmap_epi(CUtensorMap* m, const void* ptr, bool f32, int64_t cols, int64_t rows, int64_t ld) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  ensure_current_context();
  const int es = f32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {(cuuint32_t)(64 / es), 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr),
                   dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// Per-stream SM budgets: a persistent GEMM launched on a stream with a budget runs at most that
// many CTAs (one per SM), leaving the other SMs to kernels of other streams -- e.g. the token
// exchange of expert parallelism beside a side-stream GEMM.
static std::mutex g_budget_mu;
static std::vector<std::pair<cudaStream_t, int>> g_budget;

void set_stream_sm_budget(cudaStream_t s, int sms) {
  std::lock_guard<std::mutex> lock(g_budget_mu);
  for (auto it = g_budget.begin(); it != g_budget.end(); ++it)
    if (it->first == s) {
      g_budget.erase(it);
      break;
    }
  if (sms > 0) g_budget.emplace_back(s, sms);
}

static int stream_sm_budget(cudaStream_t s) {
  std::lock_guard<std::mutex> lock(g_budget_mu);
  for (const auto& e : g_budget)
    if (e.first == s) return e.second;
  return 0;
}

// CTA-pair (cta_group::2) tiles are used for BN = 256 problems whose row tiles of 256 stay
// inside each group; MXK_GEMM_PAIR=0 turns them off.
static bool pair_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = std::getenv("MXK_GEMM_PAIR");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Operand stages of the CTA-pair weight-gradient GEMM (MXK_GEMM_DW_STAGES: 6, the default, or 4).
static int dw_stages() {
  static int n = -1;
  if (n < 0) {
    const char* e = std::getenv("MXK_GEMM_DW_STAGES");
    n = (e && e[0] == '4') ? 4 : 6;
  }
  return n;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, bool PAIR>
static int launch_impl(const GemmLaunch& L, cudaStream_t stream) {
  MXK_TRACE("launch_impl enter");
  constexpr int TM = PAIR ? 2 * kBM : kBM;
  constexpr int BNL = PAIR ? BN / 2 : BN;
  CUtensorMap ta, tb, tc, tc2;
  // A tile: K-major -> box {64 (K), 128 rows}; MN-major -> box {64 (M), 64 (K rows)}.
  // B tile (this CTA's BNL rows): K-major -> box {64 (K), BNL rows}; MN-major -> {64 (N), 64}.
  if (!make_tmap_bf16_2d(&ta, L.a, L.a_inner, L.a_outer, L.lda, 64, A_MN ? 64 : kBM)) return kErrBadArgs;
  if (!make_tmap_bf16_2d(&tb, L.b, L.b_inner, L.b_outer, L.ldb, 64, B_MN ? 64 : BNL)) return kErrBadArgs;
  if (!make_tmap_epi(&tc, L.p.C, L.p.c_f32 != 0, L.c_cols, L.c_rows, L.p.ldc)) return kErrBadArgs;
  if constexpr (EPI == EPI_SWIGLU_BWD) {
    // second map = the SwiGLU pre-activations H, loaded by the epilogue in the store boxes' layout
    if (!make_tmap_epi(&tc2, L.p.R, false, L.c_cols, L.c_rows, L.p.ldr)) return kErrBadArgs;
  } else if (L.p.C2 != nullptr && EPI != EPI_CE) {
    if (!make_tmap_epi(&tc2, L.p.C2, L.c2_f32 != 0, L.c2_cols, L.c2_rows, L.p.ldc2)) return kErrBadArgs;
  } else {
    tc2 = tc;
  }
  MXK_TRACE("tmaps");
  auto kern = gemm_sm100_kernel<BN, STAGES, A_MN, B_MN, EPI, PAIR>;
  constexpr int smem = gemm_smem_bytes<BN, STAGES, PAIR, EPI>();
  static_assert(smem <= 232448, "shared memory budget exceeded");
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return kErrBadArgs;
    attr_set = true;
  }
  GemmParams p = L.p;
  const int n_tiles = (p.N + BN - 1) / BN;
  const int m_tiles = (p.M + TM - 1) / TM;
  int sms = num_sms();
  const int budget = stream_sm_budget(stream);
  if (budget > 0 && budget < sms) sms = budget;
  const int units = PAIR ? (sms / 2 > 0 ? sms / 2 : 1) : sms;  // concurrently running tile workers
  long long tiles = (long long)p.G * m_tiles * n_tiles;
  // Split K over workers when a non-grouped fp32 accumulation has too few output tiles for the
  // GPU; the partial sums are combined by the element-wise atomic TMA reduce-add.
  // The split count is the smallest whose work units fill the last wave to >= 90 % (each split
  // adds one fp32 reduce-add pass over C).
  p.ksplit = 1;
  p.raster_n = n_tiles <= 16 ? 1 : 0;
  if (p.G == 1 && p.ragged == 0 && p.c_f32 && p.c_accum && tiles < 2 * units) {
    const int nkb = (p.K + kBK - 1) / kBK;
    int ks = 1;
    for (int c = 1; c <= 16 && c <= nkb; ++c) {
      const long long w = tiles * c;
      const long long waves = (w + units - 1) / units;
      ks = c;
      if (w >= (units * 9) / 10 && w * 10 >= waves * units * 9) break;
    }
    if (ks > 1) {
      const int per = (nkb + ks - 1) / ks;
      ks = (nkb + per - 1) / per;  // no empty splits
      p.ksplit = ks;
      tiles *= ks;
    }
  }
  const int workers = (int)(tiles < units ? tiles : units);
  if (workers <= 0) return 0;
  MXK_TRACE("launch");
  count_launch();
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * workers, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, tc2, p) != cudaSuccess) return kErrBadArgs;
  } else {
    kern<<<workers, kGemmThreads, smem, stream>>>(ta, tb, tc, tc2, p);
  }
  MXK_TRACE("launched");
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgs;
}

#define MXK_CASE(BN_, ST_, AMN_, BMN_, EPI_)                                                     \
  if (L.bn == BN_ && L.a_mn == AMN_ && L.b_mn == BMN_ && L.epi == EPI_)                        \
    return launch_impl<BN_, ST_, AMN_, BMN_, EPI_, false>(L, stream);

// BN = 256 cases: CTA-pair tiles (6 stages of 32 KB per CTA) when the problem allows them.
#define MXK_CASE2(ST_, AMN_, BMN_, EPI_)                                                         \
  if (L.bn == 256 && L.a_mn == AMN_ && L.b_mn == BMN_ && L.epi == EPI_)                        \
    return pair ? launch_impl<256, 6, AMN_, BMN_, EPI_, true>(L, stream)                       \
                : launch_impl<256, ST_, AMN_, BMN_, EPI_, false>(L, stream);

int launch_gemm(const GemmLaunch& L, cudaStream_t stream) {
  MXK_TRACE("launch_gemm");
  if (L.p.G > 1 && L.p.M % kBM != 0) return kErrBadArgs;  // grouped outputs are stored in whole tiles
  if (L.p.G <= 0 || L.p.G > kMaxGroups || L.p.K <= 0 || L.p.N <= 0 || L.p.M <= 0) return kErrBadArgs;
  if (L.p.K % kBK != 0 && L.p.ragged != 2) return kErrBadArgs;
  if ((reinterpret_cast<uintptr_t>(L.a) | reinterpret_cast<uintptr_t>(L.b)) & 15) return kErrBadArgs;
  if ((L.lda * 2) % 16 || (L.ldb * 2) % 16) return kErrBadArgs;
  // 256-row tiles: a single problem of at least 256 rows, or groups whose row extent is a
  // multiple of 256 (grouped outputs are written in whole tiles)
  const bool pair = pair_enabled() && L.bn == 256 && L.p.M >= 2 * kBM && (L.p.G == 1 || L.p.M % (2 * kBM) == 0);
  // plain stores / accumulation
  MXK_CASE2(4, false, false, EPI_STORE)
  MXK_CASE(128, 6, false, false, EPI_STORE)
  MXK_CASE(64, 8, false, false, EPI_STORE)
  MXK_CASE2(4, false, true, EPI_STORE)
  MXK_CASE(128, 6, false, true, EPI_STORE)
  MXK_CASE(64, 8, false, true, EPI_STORE)
  // weight gradients (both operands MN-major; fp32 reduce-add into the gradient): CTA pairs with 6
  // operand stages and a 2-deep store ring per epilogue warp, measured 7-14 % faster on the model's
  // dW shapes than 4 operand stages with a 6-deep ring (MXK_GEMM_DW_STAGES=4)
  if (L.bn == 256 && L.a_mn && L.b_mn && L.epi == EPI_STORE) {
    if (!pair) return launch_impl<256, 4, true, true, EPI_STORE, false>(L, stream);
    return dw_stages() == 6 ? launch_impl<256, 6, true, true, EPI_STORE, true>(L, stream)
                            : launch_impl<256, 4, true, true, EPI_STORE, true>(L, stream);
  }
  MXK_CASE(128, 6, true, true, EPI_STORE)
  MXK_CASE(64, 8, true, true, EPI_STORE)
  // input-gradient GEMMs that add a second gradient term in the epilogue
  MXK_CASE2(4, false, true, EPI_RESID)
  MXK_CASE(128, 6, false, true, EPI_RESID)
  // activation-gradient GEMM with the SwiGLU backward in the epilogue
  // (fewer operand stages: the epilogue stages its H chunks in shared memory)
  if (L.bn == 256 && !L.a_mn && L.b_mn && L.epi == EPI_SWIGLU_BWD)
    return pair ? launch_impl<256, 4, false, true, EPI_SWIGLU_BWD, true>(L, stream)
                : launch_impl<256, 3, false, true, EPI_SWIGLU_BWD, false>(L, stream);
  // fused epilogues (forward, K-major x K-major)
  MXK_CASE2(4, false, false, EPI_SWIGLU)
  MXK_CASE2(4, false, false, EPI_RESID)
  MXK_CASE(128, 6, false, false, EPI_RESID)
  MXK_CASE2(4, false, false, EPI_GATE_MUL)
  MXK_CASE(128, 6, false, false, EPI_GATE_MUL)
  MXK_CASE(128, 6, false, false, EPI_SILU)
  MXK_CASE2(4, false, false, EPI_ACT)
  MXK_CASE(128, 6, false, false, EPI_ACT)
  MXK_CASE2(4, false, false, EPI_ROWSCALE)
  MXK_CASE(128, 6, false, false, EPI_ROWSCALE)
  MXK_CASE2(4, false, false, EPI_CE)
  return kErrBadArgs;
}

}  // namespace mxk
