// Torch bindings of the row-wise, attention, MoE and optimizer kernels.
#include <algorithm>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "kernels.h"

namespace {

using at::Tensor;
using OptT = c10::optional<Tensor>;

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void need(bool c, const char* msg) { TORCH_CHECK(c, msg); }

void cuda_bf16(const Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16, n, " must be a CUDA bf16 tensor");
}
void cuda_f32(const Tensor& t, const char* n) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat, n, " must be a CUDA fp32 tensor");
}
void contig(const Tensor& t, const char* n) { TORCH_CHECK(t.is_contiguous(), n, " must be contiguous"); }
void aligned16(const Tensor& t, const char* n) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, n, " must be 16-byte aligned");
}
template <class T>
T* ptr(const OptT& t) {
  return t.has_value() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
void ok(int code, const char* what) { TORCH_CHECK(code == 0, what, " failed (", code, ")"); }

// ------------------------------------------------------------------------------------ rows
void rmsnorm_fwd(const Tensor& x, const Tensor& w, const Tensor& y, const Tensor& rstd, double eps) {
  cuda_bf16(x, "x"); cuda_f32(w, "w"); cuda_bf16(y, "y"); cuda_f32(rstd, "rstd");
  contig(x, "x"); contig(y, "y");
  const int D = x.size(-1), T = x.numel() / D;
  need(D % 8 == 0, "D must be a multiple of 8");
  aligned16(x, "x"); aligned16(y, "y"); aligned16(w, "w");
  c10::cuda::CUDAGuard g(x.device());
  mxk::launch_rmsnorm_fwd(x.data_ptr(), w.data_ptr<float>(), y.data_ptr(), rstd.data_ptr<float>(), T, D, (float)eps,
                          stream());
}

void rmsnorm_bwd(const Tensor& dy, const Tensor& x, const Tensor& w, const Tensor& rstd, const OptT& dres,
                 const Tensor& dx, const Tensor& dw) {
  cuda_bf16(dy, "dy"); cuda_bf16(x, "x"); cuda_bf16(dx, "dx"); cuda_f32(dw, "dw");
  contig(dy, "dy"); contig(x, "x"); contig(dx, "dx");
  if (dres.has_value()) { cuda_bf16(*dres, "dres"); contig(*dres, "dres"); }
  const int D = x.size(-1), T = x.numel() / D;
  need(D % 8 == 0 && D <= 4096, "D must be a multiple of 8 and <= 4096");
  c10::cuda::CUDAGuard g(x.device());
  mxk::launch_rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr<float>(), rstd.data_ptr<float>(),
                          ptr<const void>(dres), dx.data_ptr(), dw.data_ptr<float>(), T, D, stream());
}

void embed_fwd(const Tensor& ids, const Tensor& table, const Tensor& out) {
  need(ids.is_cuda() && ids.scalar_type() == at::kLong, "ids must be CUDA int64");
  cuda_bf16(table, "table"); cuda_bf16(out, "out"); contig(table, "table"); contig(out, "out"); contig(ids, "ids");
  const int D = table.size(1);
  need(D % 8 == 0, "embedding dim must be a multiple of 8");
  c10::cuda::CUDAGuard g(ids.device());
  mxk::launch_embed_fwd(ids.data_ptr<int64_t>(), table.data_ptr(), out.data_ptr(), ids.numel(), D, table.size(0),
                        stream());
}

void embed_bwd(const Tensor& ids, const Tensor& dout, const Tensor& dtable) {
  cuda_bf16(dout, "dout"); cuda_f32(dtable, "dtable"); contig(dout, "dout"); contig(dtable, "dtable");
  const int D = dtable.size(1);
  c10::cuda::CUDAGuard g(ids.device());
  mxk::launch_embed_bwd(ids.data_ptr<int64_t>(), dout.data_ptr(), dtable.data_ptr<float>(), ids.numel(), D,
                        dtable.size(0), stream());
}

void gate_mul_bwd(const Tensor& dout, const Tensor& y, const Tensor& z, const Tensor& dy, const Tensor& dz) {
  for (auto* t : {&dout, &y, &z, &dy, &dz}) { cuda_bf16(*t, "gate_mul_bwd arg"); contig(*t, "gate_mul_bwd arg"); }
  need(dout.numel() % 8 == 0, "numel must be a multiple of 8");
  c10::cuda::CUDAGuard g(dout.device());
  mxk::launch_gate_mul_bwd(dout.data_ptr(), y.data_ptr(), z.data_ptr(), dy.data_ptr(), dz.data_ptr(), dout.numel(),
                           stream());
}

void act_bwd(const Tensor& da, const Tensor& h, const Tensor& dh, int64_t kind) {
  for (auto* t : {&da, &h, &dh}) { cuda_bf16(*t, "act_bwd arg"); contig(*t, "act_bwd arg"); }
  need(da.numel() % 8 == 0, "numel must be a multiple of 8");
  c10::cuda::CUDAGuard g(da.device());
  mxk::launch_act_bwd(da.data_ptr(), h.data_ptr(), dh.data_ptr(), da.numel(), (int)kind, stream());
}

void swiglu_bwd(const Tensor& dact, const Tensor& H, const Tensor& dH, int64_t kind, const OptT& counts,
                int64_t cap) {
  for (auto* t : {&dact, &H, &dH}) { cuda_bf16(*t, "swiglu_bwd arg"); contig(*t, "swiglu_bwd arg"); }
  const int I = dact.size(-1);
  need(I % 128 == 0 && H.size(-1) == 2 * I, "blocked SwiGLU needs I % 128 == 0 and H = [rows, 2I]");
  c10::cuda::CUDAGuard g(dact.device());
  mxk::launch_swiglu_bwd(dact.data_ptr(), H.data_ptr(), dH.data_ptr(), dact.numel() / I, I, (int)kind,
                         ptr<const int>(counts), (int)cap, stream());
}

void qk_norm_rope_fwd(const Tensor& qkv, const Tensor& qn, const Tensor& kn, const Tensor& rstd, const Tensor& cos,
                      const Tensor& sin, int64_t S, int64_t H, int64_t Hkv, int64_t hd, bool qk_norm, double qk_mult) {
  cuda_bf16(qkv, "qkv"); cuda_bf16(qn, "qn"); cuda_bf16(kn, "kn"); contig(qn, "qn"); contig(kn, "kn");
  need(qkv.stride(1) == 1, "qkv rows must be contiguous");
  need(hd % 2 == 0 && hd <= 256, "head_dim must be even and <= 256");
  c10::cuda::CUDAGuard g(qkv.device());
  mxk::launch_qk_norm_rope_fwd(qkv.data_ptr(), qkv.stride(0), qn.data_ptr(), kn.data_ptr(), rstd.data_ptr<float>(),
                               cos.data_ptr<float>(), sin.data_ptr<float>(), qkv.size(0), S, H, Hkv, hd, qk_norm,
                               (float)qk_mult, stream());
}

void qk_norm_rope_bwd(const Tensor& dqn, const Tensor& dkn, const Tensor& qkv, const Tensor& rstd, const Tensor& cos,
                      const Tensor& sin, const Tensor& dqkv, int64_t S, int64_t H, int64_t Hkv, int64_t hd,
                      bool qk_norm, double qk_mult) {
  need(dqkv.stride(0) == qkv.stride(0), "dqkv and qkv must share the row stride");
  c10::cuda::CUDAGuard g(qkv.device());
  mxk::launch_qk_norm_rope_bwd(dqn.data_ptr(), dkn.data_ptr(), qkv.data_ptr(), qkv.stride(0), rstd.data_ptr<float>(),
                               cos.data_ptr<float>(), sin.data_ptr<float>(), dqkv.data_ptr(), qkv.size(0), S, H, Hkv,
                               hd, qk_norm, (float)qk_mult, stream());
}

void xsa_gate_fwd(const Tensor& y, const Tensor& qkv, int64_t voff, int64_t goff, const Tensor& out, int64_t H,
                  int64_t Hkv, int64_t hd, bool xsa, bool gate) {
  cuda_bf16(y, "y"); cuda_bf16(out, "out"); contig(y, "y"); contig(out, "out");
  need(hd <= 128, "head_dim must be <= 128");
  c10::cuda::CUDAGuard g(y.device());
  mxk::launch_xsa_gate_fwd(y.data_ptr(), qkv.data_ptr(), qkv.stride(0), voff, goff, out.data_ptr(), qkv.size(0), H,
                           Hkv, hd, xsa, gate, stream());
}

void xsa_gate_bwd(const Tensor& dout, const Tensor& y, const Tensor& qkv, int64_t voff, int64_t goff, const Tensor& dy,
                  const Tensor& dqkv, int64_t H, int64_t Hkv, int64_t hd, bool xsa, bool gate) {
  need(dqkv.stride(0) == qkv.stride(0), "dqkv and qkv must share the row stride");
  c10::cuda::CUDAGuard g(y.device());
  mxk::launch_xsa_gate_bwd(dout.data_ptr(), y.data_ptr(), qkv.data_ptr(), qkv.stride(0), voff, goff, dy.data_ptr(),
                           dqkv.data_ptr(), qkv.size(0), H, Hkv, hd, xsa, gate, stream());
}

void ce_grad(const Tensor& logits, const Tensor& stats, const Tensor& labels, const Tensor& weights, const Tensor& wsum,
             const Tensor& loss, const OptT& lse, int64_t V, double z_weight, double scale) {
  cuda_bf16(logits, "logits"); cuda_f32(stats, "stats");
  need(logits.stride(1) == 1 && logits.size(1) % 8 == 0, "logits rows must be contiguous, width % 8 == 0");
  need(labels.scalar_type() == at::kLong, "labels must be int64");
  c10::cuda::CUDAGuard g(logits.device());
  mxk::launch_ce_grad(logits.data_ptr(), logits.stride(0), stats.data_ptr<float>(), stats.size(1) / 2,
                      labels.data_ptr<int64_t>(), weights.data_ptr<float>(), wsum.data_ptr<float>(),
                      loss.data_ptr<float>(), ptr<float>(lse), logits.size(0), V, (float)z_weight, (float)scale,
                      stream());
}

// ------------------------------------------------------------------------------- attention
mxk::AttnLaunch attn_args(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse,
                          const OptT& seg, int64_t B, int64_t S, int64_t window, double scale) {
  cuda_bf16(q, "q"); cuda_bf16(k, "k"); cuda_bf16(v, "v"); cuda_bf16(o, "o"); cuda_f32(lse, "lse");
  need(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "q, k, v must be [T, heads, hd] (strided views allowed)");
  need(q.stride(2) == 1 && k.stride(2) == 1 && v.stride(2) == 1, "head_dim must be contiguous");
  need(o.is_contiguous(), "o must be contiguous");
  const int hd = q.size(2);
  need(q.stride(0) % 8 == 0 && k.stride(0) % 8 == 0 && v.stride(0) % 8 == 0 && q.stride(1) % 8 == 0 &&
           k.stride(1) % 8 == 0 && v.stride(1) % 8 == 0,
       "q/k/v strides must be multiples of 8 elements");
  need(q.size(1) % k.size(1) == 0, "heads must be a multiple of kv heads");
  need(q.size(0) == B * S, "q rows must equal B*S");
  mxk::AttnLaunch L{};
  L.q = q.data_ptr(); L.k = k.data_ptr(); L.v = v.data_ptr();
  L.q_tok = q.stride(0); L.q_head = q.stride(1);
  L.k_tok = k.stride(0); L.k_head = k.stride(1);
  L.v_tok = v.stride(0); L.v_head = v.stride(1);
  L.o = o.data_ptr(); L.lse = lse.data_ptr<float>();
  L.seg = seg.has_value() ? seg->data_ptr<int>() : nullptr;
  L.B = B; L.S = S; L.H = q.size(1); L.Hkv = k.size(1); L.hd = hd; L.window = window; L.scale = scale;
  return L;
}

void flash_fwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse, const OptT& seg,
               int64_t B, int64_t S, int64_t window, double scale) {
  auto L = attn_args(q, k, v, o, lse, seg, B, S, window, scale);
  c10::cuda::CUDAGuard g(q.device());
  ok(mxk::launch_flash_fwd(L, stream()), "flash_fwd");
}

void flash_fwd_sm100(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse,
                     const OptT& seg, int64_t B, int64_t S, int64_t window, double scale, const Tensor& err,
                     const OptT& prof) {
  auto L = attn_args(q, k, v, o, lse, seg, B, S, window, scale);
  L.prof = prof.has_value() ? prof->data_ptr() : nullptr;
  c10::cuda::CUDAGuard g(q.device());
  ok(mxk::launch_flash_fwd_sm100(L, err.data_ptr<int>(), stream()), "flash_fwd_sm100");
}

void flash_bwd(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse, const OptT& seg,
               int64_t B, int64_t S, int64_t window, double scale, const Tensor& dout, const Tensor& dsum,
               const Tensor& dq_acc, const Tensor& dq, const Tensor& dk, const Tensor& dv, bool dv_accumulate) {
  auto L = attn_args(q, k, v, o, lse, seg, B, S, window, scale);
  need(dout.is_contiguous() && dq.is_contiguous() && dq_acc.is_contiguous(), "dout/dq/dq_acc must be contiguous");
  need(dk.stride(2) == 1 && dv.stride(2) == 1, "dk/dv head_dim must be contiguous");
  L.dout = dout.data_ptr(); L.dsum = dsum.data_ptr<float>(); L.dq_acc = dq_acc.data_ptr<float>();
  L.dq = dq.data_ptr(); L.dk = dk.data_ptr(); L.dk_tok = dk.stride(0); L.dk_head = dk.stride(1);
  L.dv = dv.data_ptr(); L.dv_tok = dv.stride(0); L.dv_head = dv.stride(1); L.dv_accumulate = dv_accumulate;
  c10::cuda::CUDAGuard g(q.device());
  ok(mxk::launch_flash_bwd(L, stream()), "flash_bwd");
}

// Phase counters for the tcgen05 attention backward (int64 CUDA tensor of >= 8 entries; layout in
// attention_bwd_sm100.cu), or none. Debug instrumentation.
static void* g_attn_bwd_prof = nullptr;
void set_attn_bwd_prof(const OptT& prof) {
  if (prof.has_value()) need(prof->is_cuda() && prof->numel() >= 8 && prof->element_size() == 8, "prof: 8 x int64");
  g_attn_bwd_prof = prof.has_value() ? prof->data_ptr() : nullptr;
}

void flash_bwd_sm100(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& o, const Tensor& lse,
                     const OptT& seg, int64_t B, int64_t S, int64_t window, double scale, const Tensor& dout,
                     const Tensor& dsum, const Tensor& dq_acc, const Tensor& dq, const Tensor& dk, const Tensor& dv,
                     bool dv_accumulate, const Tensor& err) {
  auto L = attn_args(q, k, v, o, lse, seg, B, S, window, scale);
  need(dout.is_contiguous() && dq.is_contiguous() && dq_acc.is_contiguous() && o.is_contiguous(),
       "dout/o/dq/dq_acc must be contiguous");
  need(dk.stride(2) == 1 && dv.stride(2) == 1, "dk/dv head_dim must be contiguous");
  L.dout = dout.data_ptr(); L.dsum = dsum.data_ptr<float>(); L.dq_acc = dq_acc.data_ptr<float>();
  L.dq = dq.data_ptr(); L.dk = dk.data_ptr(); L.dk_tok = dk.stride(0); L.dk_head = dk.stride(1);
  L.dv = dv.data_ptr(); L.dv_tok = dv.stride(0); L.dv_head = dv.stride(1); L.dv_accumulate = dv_accumulate;
  L.prof = g_attn_bwd_prof;
  c10::cuda::CUDAGuard g(q.device());
  ok(mxk::launch_flash_bwd_sm100(L, err.data_ptr<int>(), stream()), "flash_bwd_sm100");
}

// ------------------------------------------------------------------------------------- MoE
void router_fwd(const Tensor& logits, const Tensor& bias, int64_t E, int64_t K, bool adaptive, const Tensor& theta,
                int64_t k_min, double temp, const Tensor& sel, const Tensor& comb, const Tensor& topb,
                const Tensor& alpha, const Tensor& lse, const Tensor& keep, const Tensor& counts, const Tensor& psum,
                const Tensor& scalars) {
  cuda_f32(logits, "logits");
  need(logits.stride(1) == 1, "logits rows must be contiguous");
  need(sel.scalar_type() == at::kInt && keep.scalar_type() == at::kByte, "sel int32, keep uint8");
  c10::cuda::CUDAGuard g(logits.device());
  ok(mxk::launch_router_fwd(logits.data_ptr<float>(), logits.stride(0), bias.data_ptr<float>(), logits.size(0), E, K,
                            adaptive, theta.data_ptr<float>(), k_min, (float)temp, sel.data_ptr<int>(),
                            comb.data_ptr<float>(), topb.data_ptr<float>(), alpha.data_ptr<float>(),
                            lse.data_ptr<float>(), keep.data_ptr<uint8_t>(), counts.data_ptr<float>(),
                            psum.data_ptr<float>(), scalars.data_ptr<float>(), stream()),
     "router_fwd");
}

void router_bwd(const Tensor& logits, const Tensor& lse, const Tensor& sel, const Tensor& topb, const Tensor& keep,
                const Tensor& dcomb, const Tensor& counts, const Tensor& dscal, int64_t E, int64_t K, bool adaptive,
                const Tensor& theta, int64_t k_min, double temp, const Tensor& dlog, const Tensor& dtheta) {
  cuda_bf16(dlog, "dlog");
  need(dlog.stride(1) == 1, "dlog rows must be contiguous");
  c10::cuda::CUDAGuard g(logits.device());
  ok(mxk::launch_router_bwd(logits.data_ptr<float>(), logits.stride(0), lse.data_ptr<float>(), sel.data_ptr<int>(),
                            topb.data_ptr<float>(), keep.data_ptr<uint8_t>(), dcomb.data_ptr<float>(),
                            counts.data_ptr<float>(), dscal.data_ptr<float>(), logits.size(0), E, K, adaptive,
                            theta.data_ptr<float>(), k_min, (float)temp, dlog.data_ptr(), dlog.stride(0),
                            dtheta.data_ptr<float>(), stream()),
     "router_bwd");
}

void qb_beta(const Tensor& logits, const Tensor& alpha, int64_t E, int64_t qb_count, const Tensor& beta) {
  c10::cuda::CUDAGuard g(logits.device());
  mxk::launch_qb_beta(logits.data_ptr<float>(), logits.stride(0), alpha.data_ptr<float>(), logits.size(0), E, qb_count,
                      beta.data_ptr<float>(), stream());
}

int64_t plan_workspace(int64_t n, int64_t E) { return mxk::plan_workspace_ints(n, E); }

void dispatch_plan(const Tensor& sel, const OptT& keep, const Tensor& comb, int64_t E, int64_t cap,
                   const Tensor& blk_counts, const Tensor& slot, const Tensor& perm, const Tensor& wperm,
                   const Tensor& counts) {
  need(sel.scalar_type() == at::kInt && sel.is_contiguous(), "sel must be contiguous int32 [T, K]");
  need(blk_counts.numel() >= mxk::plan_workspace_ints(sel.numel(), E), "plan workspace too small");
  need(E >= 1 && E <= mxk::plan_max_experts(), "expert count out of range for the dispatch plan (1..plan_max_experts)");
  c10::cuda::CUDAGuard g(sel.device());
  ok(mxk::launch_dispatch_plan(sel.data_ptr<int>(), ptr<const uint8_t>(keep), comb.data_ptr<float>(), sel.numel(),
                               sel.size(1), E, cap, blk_counts.data_ptr<int>(), slot.data_ptr<int>(),
                               perm.data_ptr<int>(), wperm.data_ptr<float>(), counts.data_ptr<int>(), stream()),
     "dispatch_plan");
}

void permute(const Tensor& x, const Tensor& perm, const Tensor& counts, int64_t cap, const Tensor& xp) {
  cuda_bf16(x, "x"); cuda_bf16(xp, "xp"); contig(x, "x"); contig(xp, "xp");
  need(x.size(1) % 8 == 0, "D must be a multiple of 8");
  c10::cuda::CUDAGuard g(x.device());
  mxk::launch_permute(x.data_ptr(), perm.data_ptr<int>(), counts.data_ptr<int>(), cap, counts.numel(), x.size(1),
                      xp.data_ptr(), stream());
}

void combine(const Tensor& Y, const Tensor& sel, const Tensor& slot, const Tensor& comb, const OptT& residual,
             const Tensor& out, int64_t cap) {
  cuda_bf16(Y, "Y"); cuda_bf16(out, "out"); contig(Y, "Y"); contig(out, "out");
  if (residual.has_value()) { cuda_bf16(*residual, "residual"); contig(*residual, "residual"); }
  c10::cuda::CUDAGuard g(Y.device());
  mxk::launch_combine(Y.data_ptr(), sel.data_ptr<int>(), slot.data_ptr<int>(), comb.data_ptr<float>(),
                      ptr<const void>(residual), out.data_ptr(), sel.size(0), sel.size(1), cap, out.size(1), stream());
}

void combine_bwd(const Tensor& dout, const Tensor& Y, const Tensor& sel, const Tensor& slot, const Tensor& perm,
                 const Tensor& wperm, const Tensor& counts, int64_t cap, const OptT& dY, const Tensor& dcomb) {
  contig(dout, "dout");
  if (dY.has_value()) contig(*dY, "dY");
  c10::cuda::CUDAGuard g(Y.device());
  mxk::launch_combine_bwd(dout.data_ptr(), Y.data_ptr(), sel.data_ptr<int>(), slot.data_ptr<int>(), perm.data_ptr<int>(),
                          wperm.data_ptr<float>(), counts.data_ptr<int>(), sel.size(0), sel.size(1), cap,
                          counts.numel(), dout.size(1), ptr<void>(dY), dcomb.data_ptr<float>(), stream());
}

void unpermute_add(const Tensor& dxp, const Tensor& sel, const Tensor& slot, const OptT& dx_in, const Tensor& dx,
                   int64_t cap) {
  contig(dxp, "dxp"); contig(dx, "dx");
  c10::cuda::CUDAGuard g(dx.device());
  mxk::launch_unpermute_add(dxp.data_ptr(), sel.data_ptr<int>(), slot.data_ptr<int>(), ptr<const void>(dx_in),
                            dx.data_ptr(), sel.size(0), sel.size(1), cap, dx.size(1), stream());
}

// ------------------------------------------------------------------------------- optimizer
void opt_sqnorm(const Tensor& chunks, int64_t nchunks, const Tensor& grad, double scale, const Tensor& out) {
  c10::cuda::CUDAGuard g(grad.device());
  mxk::launch_opt_sqnorm(chunks.data_ptr(), nchunks, grad.data_ptr<float>(), (float)scale, out.data_ptr<double>(),
                         stream());
}

void opt_step(const Tensor& chunks, int64_t nchunks, const Tensor& hp, const OptT& gnorm2, double gscale,
              const Tensor& grad, const Tensor& m, const Tensor& v, const Tensor& p, const OptT& pb,
              const Tensor& mat_sums, bool has_adamh, int64_t mv_offset, int64_t phase) {
  // m and v may hold only the flat range [mv_offset, mv_offset + numel) of a sharded optimizer; the
  // chunk table addresses global offsets inside that range.
  cuda_f32(grad, "grad"); cuda_f32(m, "m"); cuda_f32(v, "v"); cuda_f32(p, "p");
  need(m.numel() == v.numel() && mv_offset >= 0 && mv_offset + m.numel() <= p.numel(), "bad moment shard");
  c10::cuda::CUDAGuard g(grad.device());
  mxk::launch_opt_step(chunks.data_ptr(), nchunks, hp.data_ptr<float>(), ptr<const double>(gnorm2), (float)gscale,
                       grad.data_ptr<float>(), m.data_ptr<float>() - mv_offset, v.data_ptr<float>() - mv_offset,
                       p.data_ptr<float>(), ptr<void>(pb), mat_sums.data_ptr<double>(), has_adamh, (int)phase,
                       stream());
}

void delayed_prep(const Tensor& chunks, int64_t nchunks, const Tensor& grad, const Tensor& master,
                  const OptT& grad_ring, const OptT& param_ring, const OptT& v_ema, const OptT& m_raw,
                  const Tensor& before, int64_t t, int64_t tau_max, int64_t corrector, double dc_lambda,
                  double dc_beta2, double pred_beta, double grad_scale) {
  cuda_f32(grad, "grad"); cuda_f32(master, "master"); cuda_f32(before, "before");
  const int64_t n = grad.numel();
  need(master.numel() == n && before.numel() == n, "delayed_prep: buffer sizes differ");
  need(tau_max == 0 || (grad_ring.has_value() && grad_ring->numel() == tau_max * n), "delayed_prep: gradient ring");
  need(corrector == 0 || (param_ring.has_value() && param_ring->numel() == tau_max * n), "delayed_prep: weight ring");
  need(corrector != 2 || (v_ema.has_value() && v_ema->numel() == n), "delayed_prep: curvature EMA");
  need(!m_raw.has_value() || m_raw->numel() == n, "delayed_prep: raw momentum");
  c10::cuda::CUDAGuard g(grad.device());
  mxk::DelayArgs a{};
  a.grad = grad.data_ptr<float>();
  a.master = master.data_ptr<float>();
  a.grad_ring = ptr<float>(grad_ring);
  a.param_ring = ptr<float>(param_ring);
  a.v_ema = ptr<float>(v_ema);
  a.m_raw = ptr<float>(m_raw);
  a.before = before.data_ptr<float>();
  a.n = n;
  a.t = t;
  a.tau_max = (int)std::max<int64_t>(tau_max, 1);
  a.corrector = (int)corrector;
  a.dc_lambda = (float)dc_lambda; a.dc_beta2 = (float)dc_beta2; a.pred_beta = (float)pred_beta;
  a.grad_scale = (float)grad_scale;
  mxk::launch_delayed_prep(chunks.data_ptr(), nchunks, a, stream());
}

void delayed_finish(const Tensor& master, const Tensor& before_upd, const OptT& compute, double damp) {
  cuda_f32(master, "master"); cuda_f32(before_upd, "before_upd");
  need(master.numel() == before_upd.numel(), "delayed_finish: buffer sizes differ");
  c10::cuda::CUDAGuard g(master.device());
  mxk::launch_delayed_finish(master.data_ptr<float>(), before_upd.data_ptr<float>(), ptr<void>(compute),
                             master.numel(), (float)damp, stream());
}

void ema(const Tensor& dst, const Tensor& src, double beta) {
  c10::cuda::CUDAGuard g(dst.device());
  mxk::launch_ema(dst.data_ptr<float>(), src.data_ptr<float>(), dst.numel(), (float)beta, stream());
}

void cast_bf16(const Tensor& src, const Tensor& dst) {
  need(src.numel() == dst.numel(), "size mismatch");
  c10::cuda::CUDAGuard g(src.device());
  mxk::launch_cast_bf16(src.data_ptr<float>(), dst.data_ptr(), src.numel(), stream());
}

// ---------------------------------------------------------------- expert-parallel peer exchange
mxk::EpArgs ep_args(const std::vector<int64_t>& peers, int64_t my, int64_t e_loc, int64_t cap, int64_t D,
                    int64_t buf_off, int64_t counts_off, int64_t flags_off, int64_t purpose, int64_t epoch,
                    const OptT& counter) {
  need((int64_t)peers.size() <= mxk::kMaxPeers && my < (int64_t)peers.size(), "bad peer table");
  need(D % 8 == 0, "row width must be a multiple of 8 elements");
  mxk::EpArgs a{};
  for (size_t i = 0; i < peers.size(); ++i) a.peers.base[i] = reinterpret_cast<void*>(peers[i]);
  a.world = (int)peers.size();
  a.my = (int)my;
  a.e_loc = (int)e_loc;
  a.cap = (int)cap;
  a.D = (int)D;
  a.buf_off = (size_t)buf_off;
  a.counts_off = (size_t)counts_off;
  a.flags_off = (size_t)flags_off;
  a.purpose = (int)purpose;
  a.epoch = (int)epoch;
  a.counter = counter.has_value() ? reinterpret_cast<unsigned int*>(counter->data_ptr()) : nullptr;
  return a;
}

std::tuple<int64_t, Tensor> ipc_alloc(int64_t bytes) {
  void* p = nullptr;
  Tensor h = torch::empty({64}, torch::dtype(torch::kUInt8));
  need(sizeof(cudaIpcMemHandle_t) <= 64, "ipc handle size");
  const int rc = mxk::ipc_alloc((size_t)bytes, &p, h.data_ptr());
  need(rc == 0, "ipc_alloc failed");
  return {reinterpret_cast<int64_t>(p), h};
}

int64_t ipc_open(const Tensor& h) {
  void* p = nullptr;
  need(mxk::ipc_open(h.contiguous().data_ptr(), &p) == 0, "cudaIpcOpenMemHandle failed");
  return reinterpret_cast<int64_t>(p);
}

Tensor heap_tensor(int64_t base, int64_t offset, std::vector<int64_t> shape, int64_t dtype_code, int64_t device) {
  // dtype_code: 0 bf16, 1 f32, 2 i32
  const auto dt = dtype_code == 0 ? torch::kBFloat16 : dtype_code == 1 ? torch::kFloat32 : torch::kInt32;
  void* p = reinterpret_cast<char*>(base) + offset;
  need(reinterpret_cast<uintptr_t>(p) % 16 == 0, "heap tensor must be 16-byte aligned");
  return torch::from_blob(p, shape, [](void*) {}, torch::dtype(dt).device(torch::kCUDA, device));
}

void ep_dispatch_push(const Tensor& x, const Tensor& perm, const Tensor& counts, const std::vector<int64_t>& peers,
                      int64_t my, int64_t e_loc, int64_t cap, int64_t buf_off, int64_t counts_off, int64_t flags_off,
                      int64_t purpose, int64_t epoch, const Tensor& counter, int64_t s_lo, int64_t s_hi,
                      int64_t max_blocks) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = ep_args(peers, my, e_loc, cap, x.size(1), buf_off, counts_off, flags_off, purpose, epoch, counter);
  a.s_lo = (int)s_lo;
  a.s_hi = (int)s_hi;
  a.max_blocks = (int)max_blocks;
  mxk::launch_ep_dispatch_push(x.data_ptr(), perm.data_ptr<int>(), counts.data_ptr<int>(), a, stream());
}

void ep_combine_bwd_push(const Tensor& dout, const Tensor& perm, const Tensor& wperm, const Tensor& counts,
                         const std::vector<int64_t>& peers, int64_t my, int64_t e_loc, int64_t cap, int64_t buf_off,
                         int64_t flags_off, int64_t purpose, int64_t epoch, const Tensor& counter, int64_t s_lo,
                         int64_t s_hi, int64_t max_blocks) {
  c10::cuda::CUDAGuard g(dout.device());
  auto a = ep_args(peers, my, e_loc, cap, dout.size(1), buf_off, 0, flags_off, purpose, epoch, counter);
  a.s_lo = (int)s_lo;
  a.s_hi = (int)s_hi;
  a.max_blocks = (int)max_blocks;
  mxk::launch_ep_combine_bwd_push(dout.data_ptr(), perm.data_ptr<int>(), wperm.data_ptr<float>(),
                                  counts.data_ptr<int>(), a, stream());
}

void ep_combine_pull(const Tensor& sel, const Tensor& slot, const Tensor& comb, const OptT& residual, const Tensor& out,
                     const OptT& y_local, const std::vector<int64_t>& peers, int64_t my, int64_t e_loc, int64_t cap,
                     int64_t buf_off) {
  c10::cuda::CUDAGuard g(out.device());
  auto a = ep_args(peers, my, e_loc, cap, out.size(1), buf_off, 0, 0, 0, 0, c10::nullopt);
  mxk::launch_ep_combine_pull(sel.data_ptr<int>(), slot.data_ptr<int>(), comb.data_ptr<float>(), ptr<void>(residual),
                              out.data_ptr(), ptr<void>(y_local), (int)sel.size(0), (int)sel.size(1), a, stream());
}

void ep_unpermute_pull(const Tensor& sel, const Tensor& slot, const Tensor& dx, const std::vector<int64_t>& peers,
                       int64_t my, int64_t e_loc, int64_t cap, int64_t buf_off) {
  c10::cuda::CUDAGuard g(dx.device());
  auto a = ep_args(peers, my, e_loc, cap, dx.size(1), buf_off, 0, 0, 0, 0, c10::nullopt);
  mxk::launch_ep_unpermute_pull(sel.data_ptr<int>(), slot.data_ptr<int>(), dx.data_ptr(), (int)sel.size(0),
                                (int)sel.size(1), a, stream());
}

void ep_signal(const std::vector<int64_t>& peers, int64_t my, int64_t flags_off, int64_t purpose, int64_t epoch) {
  auto a = ep_args(peers, my, 1, 1, 8, 0, 0, flags_off, purpose, epoch, c10::nullopt);
  mxk::launch_ep_signal(a, stream());
}

mxk::PeerTable peer_table(const std::vector<int64_t>& peers) {
  need(!peers.empty() && (int64_t)peers.size() <= mxk::kMaxPeers, "bad peer table");
  mxk::PeerTable t{};
  for (size_t i = 0; i < peers.size(); ++i) t.base[i] = reinterpret_cast<void*>(peers[i]);
  return t;
}

void zero_rs(const std::vector<int64_t>& peers, int64_t grad_off, int64_t lo, int64_t hi, const Tensor& out,
             double scale) {
  cuda_f32(out, "out");
  need(lo % 4 == 0 && hi % 4 == 0 && hi >= lo && grad_off % 16 == 0, "zero_rs: 16-byte aligned range");
  need(out.numel() >= hi && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "zero_rs: output buffer");
  c10::cuda::CUDAGuard g(out.device());
  mxk::launch_zero_rs(peer_table(peers), (int)peers.size(), (size_t)grad_off, lo, hi, out.data_ptr<float>(),
                      (float)scale, stream());
}

void zero_ag(const std::vector<int64_t>& peers, int64_t my, int64_t master_off, int64_t per, int64_t end,
             const Tensor& master, const Tensor& compute) {
  cuda_f32(master, "master");
  need(per % 4 == 0 && end % 4 == 0 && master_off % 16 == 0 && master.numel() >= end && compute.numel() >= end,
       "zero_ag: 16-byte aligned shards");
  c10::cuda::CUDAGuard g(master.device());
  mxk::launch_zero_ag(peer_table(peers), (int)peers.size(), (int)my, (size_t)master_off, per, end,
                      master.data_ptr<float>(), compute.data_ptr(), stream());
}

void ep_wait(const std::vector<int64_t>& peers, int64_t my, int64_t flags_off, int64_t purpose, int64_t epoch,
             const Tensor& err, int64_t limit_ns) {
  auto a = ep_args(peers, my, 1, 1, 8, 0, 0, flags_off, purpose, epoch, c10::nullopt);
  mxk::launch_ep_wait(a, err.data_ptr<int>(), limit_ns, stream());
}

// ------------------------------------------------------------------------------- decode path
void head_norm_rope(const Tensor& x, int64_t nh, int64_t hd, const OptT& w, double eps, const Tensor& pos,
                    const Tensor& cos_t, const Tensor& sin_t, const Tensor& out) {
  need(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "x must be CUDA bf16 rows");
  need(out.is_contiguous() && pos.scalar_type() == at::kInt, "out contiguous, pos int32");
  c10::cuda::CUDAGuard g(x.device());
  ok(mxk::launch_head_norm_rope(x.data_ptr(), x.stride(0), (int)nh, (int)hd, ptr<const float>(w), (float)eps,
                                pos.data_ptr<int>(), cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), (int)x.size(0),
                                out.data_ptr(), stream()),
     "head_norm_rope");
}

// Rows r of k / v ([rows, Hkv, hd], row stride shared) go to cache[row_seq[r] (or r), pos[r]].
void kv_append(const Tensor& k, const Tensor& v, const Tensor& ck, const Tensor& cv, const Tensor& pos,
               const OptT& row_seq) {
  need(ck.is_contiguous() && cv.is_contiguous() && k.stride(-1) == 1 && v.stride(-1) == 1, "kv_append layout");
  need(k.size(1) * k.size(2) == k.stride(1) * k.size(1) && v.stride(1) == v.size(2), "kv_append head rows");
  need(pos.numel() == k.size(0), "one position per row");
  c10::cuda::CUDAGuard g(k.device());
  ok(mxk::launch_kv_append(k.data_ptr(), v.data_ptr(), k.stride(0), v.stride(0), ck.data_ptr(), cv.data_ptr(),
                           pos.data_ptr<int>(),
                           ptr<const int>(row_seq), (int)k.size(0), (int)ck.size(1), (int)ck.size(2), (int)ck.size(3),
                           stream()),
     "kv_append");
}

void decode_attention(const Tensor& q, const Tensor& ck, const Tensor& cv, const Tensor& lens, double scale,
                      int64_t nsplit, const Tensor& part_ml, const Tensor& part_acc, const Tensor& out) {
  need(q.is_contiguous() && ck.is_contiguous() && cv.is_contiguous() && out.is_contiguous(), "decode layout");
  c10::cuda::CUDAGuard g(q.device());
  ok(mxk::launch_decode_attention(q.data_ptr(), ck.data_ptr(), cv.data_ptr(), lens.data_ptr<int>(), (int)q.size(0),
                                  (int)q.size(1), (int)ck.size(2), (int)q.size(2), (int)ck.size(1), (float)scale,
                                  (int)nsplit, part_ml.data_ptr<float>(), part_acc.data_ptr<float>(), out.data_ptr(),
                                  stream()),
     "decode_attention");
}

// -------------------------------------------------------------------- hashed n-gram embedding
void ngram_fwd(const Tensor& ids, const Tensor& orders, int64_t n_hash, int64_t buckets, const Tensor& table,
               const Tensor& out) {
  need(ids.dim() == 2 && ids.scalar_type() == at::kLong && ids.is_contiguous(), "ids must be [B, S] int64");
  need(orders.scalar_type() == at::kInt && orders.is_cuda(), "orders must be CUDA int32");
  need(table.dim() == 3 && table.is_contiguous() && out.is_contiguous(), "table [orders, buckets, rank]");
  c10::cuda::CUDAGuard g(ids.device());
  ok(mxk::launch_ngram_fwd(ids.data_ptr<int64_t>(), ids.size(0), ids.size(1), orders.data_ptr<int>(), orders.numel(),
                           (int)n_hash, (long)buckets, table.data_ptr(), table.size(2), out.data_ptr(), stream()),
     "ngram_fwd");
}

void ngram_bwd(const Tensor& ids, const Tensor& orders, int64_t n_hash, int64_t buckets, const Tensor& dout,
               const Tensor& dtable) {
  cuda_f32(dtable, "dtable");
  c10::cuda::CUDAGuard g(ids.device());
  ok(mxk::launch_ngram_bwd(ids.data_ptr<int64_t>(), ids.size(0), ids.size(1), orders.data_ptr<int>(), orders.numel(),
                           (int)n_hash, (long)buckets, dout.data_ptr(), dtable.size(2), dtable.data_ptr<float>(),
                           stream()),
     "ngram_bwd");
}

}  // namespace

void register_ops(pybind11::module& m) {
  m.def("launch_count", []() { return (int64_t)mxk::launch_counter().load(); });
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("embed_fwd", &embed_fwd);
  m.def("embed_bwd", &embed_bwd);
  m.def("gate_mul_bwd", &gate_mul_bwd);
  m.def("act_bwd", &act_bwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("qk_norm_rope_fwd", &qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &qk_norm_rope_bwd);
  m.def("xsa_gate_fwd", &xsa_gate_fwd);
  m.def("xsa_gate_bwd", &xsa_gate_bwd);
  m.def("ce_grad", &ce_grad);
  m.def("flash_fwd", &flash_fwd);
  m.def("flash_bwd", &flash_bwd);
  m.def("flash_fwd_sm100", &flash_fwd_sm100);
  m.def("router_fwd", &router_fwd);
  m.def("router_bwd", &router_bwd);
  m.def("qb_beta", &qb_beta);
  m.def("plan_workspace", &plan_workspace);
  m.def("dispatch_plan", &dispatch_plan);
  m.def("permute", &permute);
  m.def("combine", &combine);
  m.def("combine_bwd", &combine_bwd);
  m.def("unpermute_add", &unpermute_add);
  m.def("opt_sqnorm", &opt_sqnorm);
  m.def("opt_step", &opt_step);
  m.def("ema", &ema);
  m.def("delayed_prep", &delayed_prep);
  m.def("delayed_finish", &delayed_finish);
  m.def("cast_bf16", &cast_bf16);
  m.def("flash_bwd_sm100", &flash_bwd_sm100);
  m.def("set_attn_bwd_prof", &set_attn_bwd_prof);
  m.def("head_norm_rope", &head_norm_rope);
  m.def("ngram_fwd", &ngram_fwd);
  m.def("ngram_bwd", &ngram_bwd);
  m.def("kv_append", &kv_append);
  m.def("decode_attention", &decode_attention);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", [](int64_t p) { return mxk::ipc_close(reinterpret_cast<void*>(p)); });
  m.def("ipc_free", [](int64_t p) { return mxk::ipc_free(reinterpret_cast<void*>(p)); });
  m.def("heap_tensor", &heap_tensor);
  m.def("zero_rs", &zero_rs);
  m.def("zero_ag", &zero_ag);
  m.def("ep_dispatch_push", &ep_dispatch_push, py::arg("x"), py::arg("perm"), py::arg("counts"), py::arg("peers"),
        py::arg("my"), py::arg("e_loc"), py::arg("cap"), py::arg("buf_off"), py::arg("counts_off"),
        py::arg("flags_off"), py::arg("purpose"), py::arg("epoch"), py::arg("counter"), py::arg("s_lo") = 0,
        py::arg("s_hi") = 1 << 30, py::arg("max_blocks") = 0);
  m.def("ep_combine_bwd_push", &ep_combine_bwd_push, py::arg("dout"), py::arg("perm"), py::arg("wperm"),
        py::arg("counts"), py::arg("peers"), py::arg("my"), py::arg("e_loc"), py::arg("cap"), py::arg("buf_off"),
        py::arg("flags_off"), py::arg("purpose"), py::arg("epoch"), py::arg("counter"), py::arg("s_lo") = 0,
        py::arg("s_hi") = 1 << 30, py::arg("max_blocks") = 0);
  m.def("ep_combine_pull", &ep_combine_pull);
  m.def("ep_unpermute_pull", &ep_unpermute_pull);
  m.def("ep_signal", &ep_signal);
  m.def("ep_wait", &ep_wait, py::arg("peers"), py::arg("my"), py::arg("flags_off"), py::arg("purpose"),
        py::arg("epoch"), py::arg("err"), py::arg("limit_ns") = 0);
}
