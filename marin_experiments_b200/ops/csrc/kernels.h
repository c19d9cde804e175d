// Plain C++ launch interfaces of the non-GEMM sm_100a kernels (no torch types).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace mxk {

constexpr int kErrBadArgsHost = 5;

// Number of kernels this library launched (read by benchmarks to report their launch count).
inline std::atomic<long long>& launch_counter() {
  static std::atomic<long long> c{0};
  return c;
}
inline void count_launch(int n = 1) { launch_counter().fetch_add(n, std::memory_order_relaxed); }

// elementwise.cu
void launch_rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int T, int D, float eps, cudaStream_t st);
void launch_rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, const void* dres, void* dx,
                        float* dw, int T, int D, cudaStream_t st);
void launch_embed_fwd(const int64_t* ids, const void* table, void* out, int T, int D, int V, cudaStream_t st);
void launch_embed_bwd(const int64_t* ids, const void* dout, float* dtable, int T, int D, int V, cudaStream_t st);
void launch_gate_mul_bwd(const void* dout, const void* y, const void* z, void* dy, void* dz, long n, cudaStream_t st);
void launch_act_bwd(const void* da, const void* h, void* dh, long n, int kind, cudaStream_t st);
void launch_swiglu_bwd(const void* dact, const void* H, void* dH, long rows, int I, int kind, const int* counts,
                       int cap, cudaStream_t st);
void launch_qk_norm_rope_fwd(const void* qkv, int ld, void* qn, void* kn, float* rstd, const float* cos_t,
                             const float* sin_t, int T, int S, int H, int Hkv, int hd, int qk_norm, float qk_mult,
                             cudaStream_t st);
void launch_qk_norm_rope_bwd(const void* dqn, const void* dkn, const void* qkv, int ld, const float* rstd,
                             const float* cos_t, const float* sin_t, void* dqkv, int T, int S, int H, int Hkv, int hd,
                             int qk_norm, float qk_mult, cudaStream_t st);
void launch_xsa_gate_fwd(const void* y, const void* qkv, int ld, int voff, int goff, void* out, int T, int H, int Hkv,
                         int hd, int xsa, int gate, cudaStream_t st);
void launch_xsa_gate_bwd(const void* dout, const void* y, const void* qkv, int ld, int voff, int goff, void* dy,
                         void* dqkv, int T, int H, int Hkv, int hd, int xsa, int gate, cudaStream_t st);
void launch_ce_grad(void* logits, int ldl, const float* stats, int nt, const int64_t* labels, const float* weights,
                    const float* wsum, float* loss_out, float* lse_out, int rows, int V, float z_weight, float scale,
                    cudaStream_t st);

// moe.cu
int launch_router_fwd(const float* logits, int ldl, const float* bias, int T, int E, int K, int adaptive,
                      const float* theta, int k_min, float temp, int* sel, float* comb, float* topb, float* alpha,
                      float* lse, uint8_t* keep, float* counts, float* psum, float* scalars, cudaStream_t st);
int launch_router_bwd(const float* logits, int ldl, const float* lse, const int* sel, const float* topb,
                      const uint8_t* keep, const float* dcomb, const float* counts, const float* dscal, int T, int E,
                      int K, int adaptive, const float* theta, int k_min, float temp, void* dlog, int ldd,
                      float* dtheta, cudaStream_t st);
void launch_qb_beta(const float* logits, int ldl, const float* alpha, int T, int E, int qb_count, float* beta,
                    cudaStream_t st);
int plan_workspace_ints(long n, int E);
// Largest expert count the dispatch plan accepts (bounded by one block's shared memory).
int plan_max_experts();
int launch_dispatch_plan(const int* sel, const uint8_t* keep, const float* comb, long n, int K, int E, int cap,
                          int* blk_counts, int* slot, int* perm, float* wperm, int* counts, cudaStream_t st);
void launch_permute(const void* x, const int* perm, const int* counts, int cap, int E, int D, void* xp,
                    cudaStream_t st);
void launch_combine(const void* Y, const int* sel, const int* slot, const float* comb, const void* residual, void* out,
                    int T, int K, int cap, int D, cudaStream_t st);
void launch_combine_bwd(const void* dout, const void* Y, const int* sel, const int* slot, const int* perm,
                        const float* wperm, const int* counts, int T, int K, int cap, int E, int D, void* dY,
                        float* dcomb, cudaStream_t st);
void launch_unpermute_add(const void* dxp, const int* sel, const int* slot, const void* dx_in, void* dx, int T, int K,
                          int cap, int D, cudaStream_t st);

// optim.cu
void launch_opt_sqnorm(const void* chunks, int nchunks, const float* grad, float scale, double* out, cudaStream_t st);
void launch_opt_step(const void* chunks, int nchunks, const float* hp, const double* gnorm2, float gscale,
                     const float* grad, float* m, float* v, float* p, void* pb, double* mat_sums, int has_adamh, int phase,
                     cudaStream_t st);
void launch_ema(float* dst, const float* src, long n, float beta, cudaStream_t st);

// Delayed-gradient optimizer passes (delayed.cu). Rings are [tau_max, n] (null when tau_max == 0).
struct DelayArgs {
  float* grad;
  const float* master;
  float* grad_ring;
  float* param_ring;  // DC-ASGD correctors only
  float* v_ema;       // dc_asgd_ema only
  float* m_raw;       // raw momentum of the forward predictors, or null
  float* before;      // snapshot of the masters (the update is measured against it)
  long long n;
  long long t;
  int tau_max;
  int corrector;  // 0 none, 1 dc_asgd, 2 dc_asgd_ema
  float dc_lambda, dc_beta2, pred_beta, grad_scale;
};
void launch_delayed_prep(const void* chunks, int nchunks, const DelayArgs& a, cudaStream_t st);
void launch_delayed_finish(float* master, float* before_upd, void* compute, long long n, float damp,
                           cudaStream_t st);
void launch_cast_bf16(const float* src, void* dst, long n, cudaStream_t st);

// attention.cu
struct AttnLaunch {
  const void* q;
  const void* k;
  const void* v;
  long q_tok, q_head, k_tok, k_head, v_tok, v_head;
  void* o;
  float* lse;
  const int* seg;
  int B, S, H, Hkv, hd, window;
  float scale;
  const void* dout;
  float* dsum;
  float* dq_acc;
  void* dq;
  void* dk;
  long dk_tok, dk_head;
  void* dv;
  long dv_tok, dv_head;
  int dv_accumulate;
  void* prof;  // optional phase-timing counters (debug)
};
int launch_flash_fwd(const AttnLaunch& L, cudaStream_t st);
int launch_flash_bwd(const AttnLaunch& L, cudaStream_t st);
// tcgen05 forward (attention_sm100.cu); q/k/v heads contiguous (head stride == hd)
int launch_flash_fwd_sm100(const AttnLaunch& L, int* err, cudaStream_t st);
// tcgen05 backward (attention_bwd_sm100.cu) and the passes it shares with the mma.sync one
int launch_flash_bwd_sm100(const AttnLaunch& L, int* err, cudaStream_t st);
int launch_flash_bwd_prep(const AttnLaunch& L, cudaStream_t st);
int launch_dq_convert(const AttnLaunch& L, cudaStream_t st);

// ------------------------------------------------------------ expert-parallel peer exchange (comm.cu)
constexpr int kMaxPeers = 16;
struct PeerTable {
  void* base[kMaxPeers];  // every rank's heap base as mapped in this process (own rank included)
};
struct EpArgs {
  PeerTable peers;
  int world, my, e_loc, cap, D;
  size_t buf_off;     // heap offset of the exchanged row buffer ([W][E_loc][cap][D] on the owner)
  size_t counts_off;  // heap offset of the received counts ([W][E_loc] ints; dispatch only)
  size_t flags_off;   // heap offset of the flag area ([purpose][kMaxPeers] ints)
  int purpose, epoch;
  unsigned int* counter;  // local completion counter of the producer kernel
  // push kernels: only capacity slots [s_lo, s_hi) of each expert (the received counts travel with
  // the chunk that starts at slot 0), on at most max_blocks CTAs (0: the default grid)
  int s_lo = 0, s_hi = 1 << 30, max_blocks = 0;
};
void launch_ep_dispatch_push(const void* x, const int* perm, const int* counts, const EpArgs& a, cudaStream_t st);
void launch_ep_combine_bwd_push(const void* dout, const int* perm, const float* wperm, const int* counts,
                                const EpArgs& a, cudaStream_t st);
void launch_ep_combine_pull(const int* sel, const int* slot, const float* comb, const void* residual, void* out,
                            void* y_local, int T, int K, const EpArgs& a, cudaStream_t st);
void launch_ep_unpermute_pull(const int* sel, const int* slot, void* dx, int T, int K, const EpArgs& a,
                              cudaStream_t st);
void launch_ep_signal(const EpArgs& a, cudaStream_t st);
// ZeRO over peer memory (comm.cu): reduce-scatter fused with the mean; all-gather fused with the
// bf16 cast.
void launch_zero_rs(const PeerTable& peers, int world, size_t grad_off, long long lo, long long hi, float* out,
                    float scale, cudaStream_t st);
void launch_zero_ag(const PeerTable& peers, int world, int my, size_t master_off, long long per, long long end,
                    float* master, void* compute, cudaStream_t st);
// Bounded wait (limit_ns of wall time; <= 0 selects the 20 s default) for every peer's flag.
void launch_ep_wait(const EpArgs& a, int* err, long long limit_ns, cudaStream_t st);
int ipc_alloc(size_t bytes, void** ptr, void* handle_out);
int ipc_open(const void* handle, void** ptr);
int ipc_close(void* ptr);
int ipc_free(void* ptr);

// ------------------------------------------------------------------------- decode path (decode.cu)
int launch_head_norm_rope(const void* x, long x_tok, int nh, int hd, const float* w, float eps, const int* pos,
                          const float* cos_t, const float* sin_t, int T, void* out, cudaStream_t st);
int launch_kv_append(const void* k, const void* v, long k_tok, long v_tok, void* ck, void* cv, const int* pos,
                     const int* row_seq, int rows, int Lmax, int hkv, int hd, cudaStream_t st);
int launch_decode_attention(const void* q, const void* ck, const void* cv, const int* lens, int B, int H, int hkv,
                            int hd, int Lmax, float scale, int nsplit, float* part_ml, float* part_acc, void* out,
                            cudaStream_t st);

// ------------------------------------------------------------------- hashed n-gram embedding (ngram.cu)
int launch_ngram_fwd(const int64_t* ids, int B, int S, const int* orders, int n_orders, int n_hash, long buckets,
                     const void* table, int rank, void* out, cudaStream_t st);
int launch_ngram_bwd(const int64_t* ids, int B, int S, const int* orders, int n_orders, int n_hash, long buckets,
                     const void* dout, int rank, float* dtable, cudaStream_t st);

}  // namespace mxk
