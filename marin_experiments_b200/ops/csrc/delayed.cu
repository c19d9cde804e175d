// Delayed-gradient optimizer step (pipeline staleness) as two passes over the flat buffers.
//
// The wrapper delays every parameter's gradient by its own tau through a ring of the last tau_max
// gradients, optionally corrects the stale gradient (DC-ASGD with a fixed or an EMA curvature),
// keeps a raw momentum for the forward predictors, and records the update the inner optimizer
// applied (delayed-gradient-pp/delay_optim.py:103-262). Unfused, that is a clone of the gradient,
// a per-parameter loop of small kernels, ring writes and a clone plus difference of the master
// weights around the inner step. Here:
//
//   prep   (before the inner step), per element k of a chunk with delay tau:
//            g = grad[k]; ring[t % tau_max][k] = g after reading the entry of step t - tau (zero
//            while the ring fills); DC-ASGD: g_s + lambda * c * (w - w_stale) with c = g_s^2 or the
//            EMA of g_s^2 (and the weight ring written the same way); grad[k] = corrected stale
//            gradient; raw momentum m_raw = beta m_raw + (1 - beta) grad_scale grad[k];
//            before[k] = w (the snapshot the update is measured against);
//   finish (after the inner step): u = w - before; lr damping w = before + damp u (and its bf16
//            copy); last_update = damp u, written over the snapshot.
//
// tau == 0 chunks keep their gradient (bit-identical to the inner optimizer) and only snapshot.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace mxk {
namespace {

struct DelayChunk {
  long long start;
  int len;
  int tau;
};

__global__ void __launch_bounds__(256) delayed_prep_kernel(const DelayChunk* __restrict__ chunks, DelayArgs a) {
  const DelayChunk c = chunks[blockIdx.x];
  const long long n = a.n;
  const int cur = (int)(a.t % a.tau_max);
  const bool have = c.tau > 0 && a.t >= c.tau;
  const int old = c.tau > 0 ? (int)((a.t - c.tau) % a.tau_max) : 0;
  for (long long k = c.start + threadIdx.x; k < c.start + c.len; k += blockDim.x) {
    const float w = a.master[k];
    float g = a.grad[k];
    if (c.tau > 0) {
      float* gr_cur = a.grad_ring + (long long)cur * n;
      const float stale = have ? a.grad_ring[(long long)old * n + k] : 0.f;
      gr_cur[k] = g;  // after the read: tau == tau_max reads and replaces the same entry
      float out = stale;
      if (a.corrector == 1 || a.corrector == 2) {
        const float w_stale = a.param_ring[(long long)old * n + k];
        a.param_ring[(long long)cur * n + k] = w;
        float curv = stale * stale;
        if (a.corrector == 2) {
          curv = a.dc_beta2 * a.v_ema[k] + (1.f - a.dc_beta2) * stale * stale;
          a.v_ema[k] = curv;
        }
        out = stale + a.dc_lambda * curv * (w - w_stale);
      }
      g = out;
      a.grad[k] = g;
    }
    if (a.m_raw) a.m_raw[k] = a.pred_beta * a.m_raw[k] + (1.f - a.pred_beta) * a.grad_scale * g;
    a.before[k] = w;
  }
}

__global__ void delayed_finish_kernel(float* __restrict__ master, float* __restrict__ before_upd,
                                      __nv_bfloat16* __restrict__ compute, long long n, float damp) {
  for (long long k = blockIdx.x * (long long)blockDim.x + threadIdx.x; k < n; k += (long long)gridDim.x * blockDim.x) {
    const float b = before_upd[k];
    const float u = master[k] - b;
    if (damp != 1.f) {
      const float w = b + damp * u;
      master[k] = w;
      if (compute) compute[k] = __float2bfloat16(w);
    }
    before_upd[k] = damp * u;
  }
}

}  // namespace

void launch_delayed_prep(const void* chunks, int nchunks, const DelayArgs& a, cudaStream_t st) {
  if (nchunks <= 0) return;
  count_launch();
  delayed_prep_kernel<<<nchunks, 256, 0, st>>>((const DelayChunk*)chunks, a);
}

void launch_delayed_finish(float* master, float* before_upd, void* compute, long long n, float damp, cudaStream_t st) {
  count_launch();
  delayed_finish_kernel<<<148 * 8, 256, 0, st>>>(master, before_upd, (__nv_bfloat16*)compute, n, damp);
}

}  // namespace mxk
