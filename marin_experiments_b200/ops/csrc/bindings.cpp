// Torch bindings of the sm_100a kernels. Every op validates shapes, dtypes, devices and
// alignment on the host and raises on a bad argument instead of launching.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "launch.h"
#include "kernels.h"

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_code(int code, const char* what) { TORCH_CHECK(code == 0, what, ": launch failed (code ", code, ")"); }

void check_2d_bf16(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must be contiguous in its last dimension");
}

template <class T>
T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

// C[g] = A'[g] B'[g]^T with A' = A (K-major, A is [rows, K]) or A^T (MN-major, A is [K, rows]),
// likewise B'. See gemm_sm100.cuh for the grouping and ragged semantics.
void gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, const at::Tensor& C, int64_t G,
          int64_t M, int64_t N, int64_t K, const c10::optional<at::Tensor>& counts, int64_t ragged, int64_t a_grp,
          int64_t b_grp, int64_t c_grp, int64_t epi, int64_t bn, int64_t accum, double alpha,
          const c10::optional<at::Tensor>& C2, const c10::optional<at::Tensor>& R,
          const c10::optional<at::Tensor>& row_scale, int64_t act_kind, const at::Tensor& err, int64_t b_mod,
          int64_t c_mod, const c10::optional<at::Tensor>& peer_maps, int64_t peer_epl, int64_t peer_my,
          int64_t peer_cap) {
  if (std::getenv("MXK_TRACE")) { std::fprintf(stderr, "[mxk] gemm binding enter\n"); std::fflush(stderr); }
  check_2d_bf16(A, "A");
  check_2d_bf16(B, "B");
  TORCH_CHECK(C.is_cuda() && C.dim() == 2 && C.stride(1) == 1, "C must be a 2-D CUDA tensor, contiguous rows");
  TORCH_CHECK(C.scalar_type() == at::kBFloat16 || C.scalar_type() == at::kFloat, "C must be bf16 or f32");
  TORCH_CHECK(!accum || C.scalar_type() == at::kFloat, "accumulation requires an f32 C");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == at::kInt, "err must be a CUDA int32 tensor");
  if (counts.has_value()) {
    TORCH_CHECK(counts->is_cuda() && counts->scalar_type() == at::kInt && counts->numel() >= G,
                "counts must be a CUDA int32 tensor with G entries");
  }
  if (R.has_value()) check_2d_bf16(*R, "R");
  if (peer_maps.has_value()) {
    // peer-store epilogue: plain bf16 stores of whole groups, one tensor map per destination rank
    TORCH_CHECK(epi == 0 && C.scalar_type() == at::kBFloat16 && !accum && G > 1 && c_mod == 0 && ragged == 1,
                "peer stores: grouped ragged-M bf16 store epilogue only");
    TORCH_CHECK(peer_epl > 0 && G % peer_epl == 0 && peer_my >= 0 && peer_cap >= M,
                "peer stores: groups must be whole (rank, local expert) blocks");
    TORCH_CHECK(peer_maps->is_cuda() && peer_maps->scalar_type() == at::kByte &&
                    peer_maps->numel() >= (int64_t)sizeof(CUtensorMap) * (G / peer_epl) &&
                    reinterpret_cast<uintptr_t>(peer_maps->data_ptr()) % 64 == 0,
                "peer stores: peer_maps must hold one 64-byte-aligned CUtensorMap per rank on the GPU");
  }
  TORCH_CHECK(reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "C must be 16-byte aligned");
  TORCH_CHECK((C.stride(0) * C.element_size()) % 16 == 0, "C row stride must be a multiple of 16 bytes");
  // Epilogues store 32-column chunks: C must be wide enough for N rounded up to 32.
  TORCH_CHECK(C.size(1) >= ((N + 31) / 32) * 32 || epi == 1, "C must have at least round_up(N, 32) columns");
  TORCH_CHECK(epi != 8 || (N % 128 == 0 && C.size(1) >= 2 * N && R.has_value() && R->size(1) >= 2 * N),
              "SwiGLU backward: N a multiple of 128, C and R with 2N columns");
  // the SwiGLU backward epilogue loads R (the pre-activations) with TMA: 16-byte aligned rows
  TORCH_CHECK(epi != 8 || (reinterpret_cast<uintptr_t>(R->data_ptr()) % 16 == 0 && (R->stride(0) * 2) % 16 == 0 &&
                           R->stride(1) == 1 && R->size(0) >= (G == 1 ? std::min<int64_t>(M, C.size(0)) : C.size(0))),
              "SwiGLU backward: R must be row-major with 16-byte aligned rows and cover C's rows");
  const c10::cuda::CUDAGuard guard(A.device());
  mxk::GemmLaunch L{};
  L.a = A.data_ptr();
  L.lda = A.stride(0);
  L.a_inner = A.size(1);
  L.a_outer = A.size(0);
  L.a_mn = a_mn ? 1 : 0;
  L.b = B.data_ptr();
  L.ldb = B.stride(0);
  L.b_inner = B.size(1);
  L.b_outer = B.size(0);
  L.b_mn = b_mn ? 1 : 0;
  L.bn = (int)bn;
  L.epi = (int)epi;
  mxk::GemmParams& p = L.p;
  p.G = (int)G;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.counts = counts.has_value() ? reinterpret_cast<const int*>(counts->data_ptr()) : nullptr;
  p.ragged = (int)ragged;
  p.a_grp = (int)a_grp;
  p.b_grp = (int)b_grp;
  p.c_grp = (int)c_grp;
  p.C = C.data_ptr();
  p.ldc = (int)C.stride(0);
  p.c_f32 = C.scalar_type() == at::kFloat ? 1 : 0;
  p.c_accum = (int)accum;
  p.b_mod = (int)b_mod;
  p.c_mod = (int)c_mod;
  p.C2 = opt_ptr<void>(C2);
  p.ldc2 = C2.has_value() ? (int)C2->stride(0) : 0;
  p.R = opt_ptr<const void>(R);
  p.ldr = R.has_value() ? (int)R->stride(0) : 0;
  p.row_scale = opt_ptr<const float>(row_scale);
  p.alpha = (float)alpha;
  p.act_kind = (int)act_kind;
  p.err = reinterpret_cast<int*>(err.data_ptr());
  p.ksplit = 1;
  p.raster_n = 0;
  p.peer_maps = peer_maps.has_value() ? peer_maps->data_ptr() : nullptr;
  p.peer_epl = (int)peer_epl;
  p.peer_my = (int)peer_my;
  p.peer_cap = (int)peer_cap;
  // Output extents for the TMA stores: columns clip at N; rows clip at M for a single problem,
  // at the buffer end for grouped problems.
  L.c_cols = epi == 8 ? 2 * N : N;  // SwiGLU backward writes gate and up gradients: 2N columns
  L.c_rows = G == 1 ? std::min<int64_t>(M, C.size(0)) : C.size(0);
  if (C2.has_value()) {
    L.c2_f32 = C2->scalar_type() == at::kFloat ? 1 : 0;
    L.c2_cols = epi == 1 ? N / 2 : std::min<int64_t>(N, C2->size(1));
    L.c2_rows = G == 1 ? std::min<int64_t>(M, C2->size(0)) : C2->size(0);
    TORCH_CHECK(reinterpret_cast<uintptr_t>(C2->data_ptr()) % 16 == 0, "C2 must be 16-byte aligned");
    // CE statistics: two (max, sumexp) float pairs per 256-column tile and row
    TORCH_CHECK(epi != 6 || (L.c2_f32 && C2->size(1) >= 4 * ((N + 255) / 256)),
                "CE stats must be f32 with 4 floats per 256-column tile");
  }
  if (std::getenv("MXK_TRACE")) { std::fprintf(stderr, "[mxk] binding -> launch_gemm\n"); std::fflush(stderr); }
  check_code(mxk::launch_gemm(L, cur_stream()), "gemm");
}

int64_t num_sms() { return mxk::num_sms(); }

// Tensor maps for the peer-store epilogue: one per rank, over the bf16 [rows, cols] buffer at byte
// offset `off` of that rank's heap (peers[r] = its base as mapped in this process). Returned as
// host bytes; the caller copies them to the GPU.
at::Tensor peer_store_maps(const std::vector<int64_t>& peers, int64_t off, int64_t cols, int64_t rows) {
  TORCH_CHECK(!peers.empty() && cols > 0 && rows > 0 && (cols * 2) % 16 == 0 && off % 16 == 0,
              "peer_store_maps: bad arguments");
  auto out = at::zeros({(int64_t)(peers.size() * sizeof(CUtensorMap))}, at::kByte);
  for (size_t r = 0; r < peers.size(); ++r) {
    CUtensorMap m;
    const char* base = reinterpret_cast<const char*>(peers[r]) + off;
    TORCH_CHECK(mxk::make_tmap_epi(&m, base, false, cols, rows, cols), "peer_store_maps: encoding failed");
    std::memcpy(out.data_ptr<uint8_t>() + r * sizeof(CUtensorMap), &m, sizeof(CUtensorMap));
  }
  return out;
}

void set_stream_sm_budget(int64_t stream, int64_t sms) {
  mxk::set_stream_sm_budget(reinterpret_cast<cudaStream_t>(stream), (int)sms);
}

}  // namespace

void register_ops(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm", &gemm, "sm_100a tcgen05 GEMM (grouped / ragged, fused epilogues)");
  m.def("num_sms", &num_sms);
  m.def("peer_store_maps", &peer_store_maps);
  m.def("set_stream_sm_budget", &set_stream_sm_budget, "cap the CTAs of persistent GEMMs on a stream");
  register_ops(m);
}
