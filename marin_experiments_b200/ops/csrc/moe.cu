// MoE routing and dispatch kernels (single GPU; the expert-parallel exchange lives in comm.cu).
//
//  router_fwd   : fp32 logits [T, E] -> softmax stats, top-(K+1) on biased logits, sigmoid combine
//                 weights, adaptive keep gate, per-expert counts / prob sums, z-loss partials.
//  router_bwd   : d(combine), d(z-loss), d(LBL), d(sparsity) -> d(logits) (bf16) and d(threshold).
//  qb_beta      : per expert, the qb_count-th largest (logit - alpha) over tokens (radix select).
//  dispatch_plan: capacity-layout slots in first-come-first-served token-major order.
//  permute / combine / combine_bwd / unpermute_add: gathers between token order and the
//                 [E, C, D] capacity layout (rows past an expert's count stay zero up to 128).
#include <algorithm>

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace mxk {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// ------------------------------------------------------------------------------------- router
// One warp per token; EPL = experts per lane (expert e lives in lane e % 32, slot e / 32).
template <int EPL>
__global__ void router_fwd_kernel(const float* __restrict__ logits, int ldl, const float* __restrict__ bias,
                                  int T, int E, int K, int adaptive, const float* __restrict__ theta_p, int k_min,
                                  float temp, int* __restrict__ sel, float* __restrict__ comb,
                                  float* __restrict__ topb, float* __restrict__ alpha, float* __restrict__ lse_out,
                                  uint8_t* __restrict__ keep, float* __restrict__ counts, float* __restrict__ psum,
                                  float* __restrict__ scalars /* [zsum, expected, realized] */) {
  extern __shared__ float sm[];  // [E] counts, [E] psum, [3] block scalars
  float* s_cnt = sm;
  float* s_ps = sm + E;
  float* s_sc = sm + 2 * E;
  for (int i = threadIdx.x; i < 2 * E + 3; i += blockDim.x) sm[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const float theta = adaptive ? *theta_p : 0.f;
  float z_acc = 0.f, exp_acc = 0.f, real_acc = 0.f;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    float l[EPL], b[EPL];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      l[j] = e < E ? logits[(long)t * ldl + e] : -INFINITY;
      b[j] = e < E ? l[j] + bias[e] : -INFINITY;
      m = fmaxf(m, l[j]);
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) s += (lane + 32 * j < E) ? __expf(l[j] - m) : 0.f;
    s = warp_sum(s);
    const float lse = m + __logf(s);
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (e < E) atomicAdd(&s_ps[e], __expf(l[j] - lse));
    }
    if (lane == 0) {
      lse_out[t] = lse;
      z_acc += lse * lse;
    }
    // top-(K+1) on biased logits: repeated warp argmax (lowest index wins ties)
    const int KK = min(K + 1, E);
    for (int k = 0; k < KK; ++k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const int e = lane + 32 * j;
        if (e < E && (b[j] > bv || (b[j] == bv && e < bi))) {
          bv = b[j];
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (lane + 32 * j == bi) b[j] = -INFINITY;
      if (k == K) {
        if (lane == 0) alpha[t] = bv;
        break;
      }
      // unbiased logit of the selected expert
      float lsel = 0.f;
#pragma unroll
      for (int j = 0; j < EPL; ++j)
        if (lane + 32 * j == bi) lsel = l[j];
      lsel = __shfl_sync(0xffffffffu, lsel, bi & 31);
      if (lane == 0) {
        float cw = sigm(lsel);
        uint8_t kp = 1;
        if (adaptive) {
          const bool floor_on = k < k_min;
          const bool hard = floor_on || bv > theta;
          const float soft = floor_on ? 1.f : sigm((bv - theta) / temp);
          kp = hard ? 1 : 0;
          cw *= hard ? 1.f : 0.f;
          exp_acc += soft;
          real_acc += hard ? 1.f : 0.f;
        } else {
          exp_acc += 1.f;
          real_acc += 1.f;
        }
        sel[(long)t * K + k] = bi;
        comb[(long)t * K + k] = cw;
        topb[(long)t * K + k] = bv;
        keep[(long)t * K + k] = kp;
        atomicAdd(&s_cnt[bi], 1.f);
      }
    }
    if (KK <= K && lane == 0) alpha[t] = -INFINITY;
  }
  // block totals first: one global atomic per block and scalar (same-address global atomics
  // from every warp serialise in L2)
  if (lane == 0) {
    atomicAdd(&s_sc[0], z_acc);
    atomicAdd(&s_sc[1], exp_acc);
    atomicAdd(&s_sc[2], real_acc);
  }
  __syncthreads();
  if (threadIdx.x < 3) atomicAdd(&scalars[threadIdx.x], s_sc[threadIdx.x]);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    atomicAdd(&counts[e], s_cnt[e]);
    atomicAdd(&psum[e], s_ps[e]);
  }
}

// d_logits[t, e] (bf16, row stride ldd, columns >= E zeroed) from
//   combine: dc_k * keep_k * sigma'(l_sel) and, adaptive, through the soft keep gate;
//   z-loss  : dz * 2 lse p_e / T ;   LBL: softmax^T of dlbl * E * f_e / T ; sparsity via soft gate.
template <int EPL>
__global__ void router_bwd_kernel(const float* __restrict__ logits, int ldl, const float* __restrict__ lse_in,
                                  const int* __restrict__ sel, const float* __restrict__ topb,
                                  const uint8_t* __restrict__ keep, const float* __restrict__ dcomb,
                                  const float* __restrict__ counts, const float* __restrict__ dscal,
                                  /* [dz, dlbl, dsparsity] */ int T, int E, int K, int adaptive,
                                  const float* __restrict__ theta_p, int k_min, float temp,
                                  __nv_bfloat16* __restrict__ dlog, int ldd, float* __restrict__ dtheta) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const float dz = dscal[0], dlbl = dscal[1], dsp = dscal[2];
  const float theta = adaptive ? *theta_p : 0.f;
  float dth_acc = 0.f;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const float lse = lse_in[t];
    float p[EPL], d[EPL];
    float pdp = 0.f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      p[j] = e < E ? __expf(logits[(long)t * ldl + e] - lse) : 0.f;
      // LBL: d p_{t,e} = dlbl * E * (counts_e / T) / T
      const float dp = e < E ? dlbl * E * (counts[e] / T) / T : 0.f;
      pdp += p[j] * dp;
      d[j] = dp;
    }
    pdp = warp_sum(pdp);
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      d[j] = p[j] * (d[j] - pdp);             // softmax backward of the LBL term
      d[j] += dz * 2.f * lse * p[j] / T;      // z-loss = mean_t lse^2
    }
    for (int k = 0; k < K; ++k) {
      const int e = sel[(long)t * K + k];
      const float dc = dcomb[(long)t * K + k];
      const float l = logits[(long)t * ldl + e];
      const float sg = sigm(l);
      const float kp = keep[(long)t * K + k] ? 1.f : 0.f;
      float de = dc * kp * sg * (1.f - sg);
      if (adaptive && k >= k_min) {
        const float bv = topb[(long)t * K + k];
        const float soft = sigm((bv - theta) / temp);
        const float dsoft = dc * sg + dsp / ((float)T * E);
        const float g = dsoft * soft * (1.f - soft) / temp;
        de += g;  // through the biased top-k value (the bias itself is stop-gradient)
        dth_acc -= g;
      }
      if ((e & 31) == lane) {
#pragma unroll
        for (int j = 0; j < EPL; ++j)
          if (lane + 32 * j == e) d[j] += de;
      }
    }
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
      const int e = lane + 32 * j;
      if (e < ldd) dlog[(long)t * ldd + e] = __float2bfloat16(e < E ? d[j] : 0.f);
    }
    for (int e = 32 * EPL + lane; e < ldd; e += 32) dlog[(long)t * ldd + e] = __float2bfloat16(0.f);
  }
  // every lane walked the same tokens' slots, so lane 0 alone holds the warp's contribution
  if (adaptive && lane == 0) atomicAdd(dtheta, dth_acc);
}

// ----------------------------------------------------------------------------------- QB beta
__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// Shared-memory variant (T <= kQbSmemKeys): one strided pass stages the expert's keys
// (logit - alpha, order-preserving uint32) in shared memory; the 4 radix passes then read shared
// memory, and each digit is chosen by a parallel suffix scan of the 256-bin histogram.
constexpr int kQbSmemKeys = 49152;  // 192 KB of keys

__global__ void __launch_bounds__(1024) qb_beta_smem_kernel(const float* __restrict__ logits, int ldl,
                                                            const float* __restrict__ alpha, int T, int E,
                                                            int qb_count, float* __restrict__ beta) {
  extern __shared__ uint32_t keys[];  // [T]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t warp_tot[8];
  __shared__ uint32_t s_prefix, s_mask, s_k;
  const int e = blockIdx.x;
  for (int t = threadIdx.x; t < T; t += blockDim.x) keys[t] = f2key(logits[(long)t * ldl + e] - alpha[t]);
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_k = (uint32_t)min(max(qb_count, 1), T);
  }
  __syncthreads();
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    if (threadIdx.x < 256) hist[threadIdx.x] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask, k = s_k;  // written again only after the next barrier
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      const uint32_t key = keys[t];
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    // thread i < 256 holds bin 255 - i; inclusive scan over i = counts of the i+1 largest bins
    const int i = threadIdx.x, lane = i & 31, w = i >> 5;
    uint32_t v = i < 256 ? hist[255 - i] : 0u;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (i < 256 && lane == 31) warp_tot[w] = incl;
    __syncthreads();
    if (i < 256) {
      uint32_t before = 0;
      for (int q = 0; q < w; ++q) before += warp_tot[q];
      incl += before;
      const uint32_t excl = incl - v;
      // the digit is the first bin (from the top) where the running count reaches k
      if (incl >= k && excl < k) {
        const int b = 255 - i;
        s_k = k - excl;
        s_prefix = prefix | ((uint32_t)b << shift);
        s_mask = mask | (255u << shift);
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) beta[e] = key2f(s_prefix);
}

// One block per expert: exact qb_count-th largest of (logit[t, e] - alpha[t]) via 4 radix passes.
__global__ void qb_beta_kernel(const float* __restrict__ logits, int ldl, const float* __restrict__ alpha, int T,
                               int E, int qb_count, float* __restrict__ beta) {
  const int e = blockIdx.x;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_mask, s_k;
  if (threadIdx.x == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_k = (uint32_t)min(max(qb_count, 1), T);
  }
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
      const uint32_t key = f2key(logits[(long)t * ldl + e] - alpha[t]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t k = s_k, acc = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (acc + hist[b] >= k) break;
        acc += hist[b];
      }
      s_k = k - acc;
      s_prefix = prefix | ((uint32_t)b << shift);
      s_mask = mask | (255u << shift);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) beta[e] = key2f(s_prefix);
}

// ------------------------------------------------------------------------------ dispatch plan
constexpr int kPlanChunk = 4096;  // assignments per block
constexpr int kPlanMaxSmem = 227 * 1024;  // opt-in dynamic shared memory limit of one block

// Per-block per-expert counts of kept assignments.
__global__ void plan_count_kernel(const int* __restrict__ sel, const uint8_t* __restrict__ keep, long n, int E,
                                  int* __restrict__ blk_counts) {
  extern __shared__ int cnt[];
  for (int i = threadIdx.x; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const long base = (long)blockIdx.x * kPlanChunk;
  for (long i = base + threadIdx.x; i < min(base + kPlanChunk, n); i += blockDim.x)
    if (!keep || keep[i]) atomicAdd(&cnt[sel[i]], 1);
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x) blk_counts[(long)blockIdx.x * E + i] = cnt[i];
}

// Slot assignment in flattened order. blockDim = 1024 (32 warps).
__global__ void plan_assign_kernel(const int* __restrict__ sel, const uint8_t* __restrict__ keep,
                                   const float* __restrict__ comb, long n, int K, int E, int cap,
                                   const int* __restrict__ blk_counts, int nblk, int* __restrict__ slot,
                                   int* __restrict__ perm, float* __restrict__ wperm, int* __restrict__ counts) {
  extern __shared__ int sh[];
  int* base = sh;              // [E]
  int* wcnt = sh + E;          // [32][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0, tot = 0;
    for (int b = 0; b < nblk; ++b) {
      const int c = blk_counts[(long)b * E + e];
      if (b < (int)blockIdx.x) s += c;
      tot += c;
    }
    base[e] = s;
    if (blockIdx.x == 0) counts[e] = min(tot, cap);
  }
  __syncthreads();
  const long start = (long)blockIdx.x * kPlanChunk;
  const long end = min(start + kPlanChunk, n);
  for (long r0 = start; r0 < end; r0 += blockDim.x) {
    for (int i = threadIdx.x; i < 32 * E; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    const long i = r0 + threadIdx.x;
    const bool valid = i < end && (!keep || keep[i]);
    const int e = valid ? sel[i] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(same & ((1u << lane) - 1u));
    if (valid && rank == 0) wcnt[warp * E + e] = __popc(same);
    __syncthreads();
    if (i < end) {
      if (valid) {
        int off = base[e] + rank;
        for (int w = 0; w < warp; ++w) off += wcnt[w * E + e];
        if (off < cap) {
          slot[i] = off;
          const long r = (long)e * cap + off;
          perm[r] = (int)(i / K);
          wperm[r] = comb[i];
        } else {
          slot[i] = -1;
        }
      } else {
        slot[i] = -1;
      }
    }
    __syncthreads();
    for (int ee = threadIdx.x; ee < E; ee += blockDim.x) {
      int s = 0;
      for (int w = 0; w < 32; ++w) s += wcnt[w * E + ee];
      base[ee] += s;
    }
    __syncthreads();
  }
}

__device__ __forceinline__ int round128(int c) { return (c + 127) & ~127; }

// Xp[e*C + s] = x[perm] for s < count_e; zeros for count_e <= s < round128(count_e).
__global__ void permute_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ perm,
                               const int* __restrict__ counts, int cap, int E, int D,
                               __nv_bfloat16* __restrict__ xp) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long r = blockIdx.x * (long)warps + (threadIdx.x >> 5); r < (long)E * cap; r += (long)gridDim.x * warps) {
    const int e = (int)(r / cap), s = (int)(r % cap);
    const int c = counts[e];
    if (s >= round128(c)) continue;
    uint4* dst = reinterpret_cast<uint4*>(xp + r * D);
    if (s < c) {
      const uint4* src = reinterpret_cast<const uint4*>(x + (long)perm[r] * D);
      for (int i = lane; i < D / 8; i += 32) dst[i] = src[i];
    } else {
      for (int i = lane; i < D / 8; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
}

__device__ __forceinline__ void acc8(float (&a)[8], uint4 u, float w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    a[2 * i] += w * f.x;
    a[2 * i + 1] += w * f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&a)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
  return u;
}

// out[t] = residual[t] + sum_k w[t,k] * Y[sel*C + slot] (fp32 accumulation).
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ Y, const int* __restrict__ sel,
                               const int* __restrict__ slot, const float* __restrict__ comb,
                               const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out, int T,
                               int K, int cap, int D) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    for (int c = lane; c < D / 8; c += 32) {
      float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (residual) acc8(a, reinterpret_cast<const uint4*>(residual + (long)t * D)[c], 1.f);
      for (int k = 0; k < K; ++k) {
        const int s = slot[(long)t * K + k];
        if (s < 0) continue;
        const long r = (long)sel[(long)t * K + k] * cap + s;
        acc8(a, reinterpret_cast<const uint4*>(Y + r * D)[c], comb[(long)t * K + k]);
      }
      reinterpret_cast<uint4*>(out + (long)t * D)[c] = pack8(a);
    }
  }
}

// The same two gathers with all of a token's K rows in flight: lanes 0..K-1 read the token's
// (slot, expert, weight) once and broadcast them, and each 16-byte chunk issues its K loads before
// accumulating (the loops above wait for one row's load at a time). W = nullptr: unit weights.
template <int KMAX>
__global__ void gather_k_kernel(const __nv_bfloat16* __restrict__ Y, const int* __restrict__ sel,
                                const int* __restrict__ slot, const float* __restrict__ W,
                                const __nv_bfloat16* __restrict__ add, __nv_bfloat16* __restrict__ out, int T, int K,
                                int cap, int D) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    int s = -1, e = 0;
    float wk = 1.f;
    if (lane < K) {
      s = slot[(long)t * K + lane];
      e = sel[(long)t * K + lane];
      if (W) wk = W[(long)t * K + lane];
    }
    const uint4* src[KMAX];
    float w[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      const int sk = __shfl_sync(0xffffffffu, s, k), ek = __shfl_sync(0xffffffffu, e, k);
      w[k] = __shfl_sync(0xffffffffu, wk, k);
      src[k] = (k < K && sk >= 0) ? reinterpret_cast<const uint4*>(Y + ((long)ek * cap + sk) * D) : nullptr;
    }
    for (int c = lane; c < D / 8; c += 32) {
      uint4 v[KMAX];
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (src[k]) v[k] = src[k][c];
      float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (add) acc8(a, reinterpret_cast<const uint4*>(add + (long)t * D)[c], 1.f);
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (src[k]) acc8(a, v[k], w[k]);
      reinterpret_cast<uint4*>(out + (long)t * D)[c] = pack8(a);
    }
  }
}

// dY[e*C+s] = wperm * dout[perm] (zeros on pad rows up to round128(count)).
__global__ void combine_bwd_rows_kernel(const __nv_bfloat16* __restrict__ dout, const int* __restrict__ perm,
                                        const float* __restrict__ wperm, const int* __restrict__ counts, int cap,
                                        int E, int D, __nv_bfloat16* __restrict__ dY) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long r = blockIdx.x * (long)warps + (threadIdx.x >> 5); r < (long)E * cap; r += (long)gridDim.x * warps) {
    const int e = (int)(r / cap), s = (int)(r % cap);
    const int c = counts[e];
    if (s >= round128(c)) continue;
    uint4* dst = reinterpret_cast<uint4*>(dY + r * D);
    if (s < c) {
      const float w = wperm[r];
      const uint4* src = reinterpret_cast<const uint4*>(dout + (long)perm[r] * D);
      for (int i = lane; i < D / 8; i += 32) {
        float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        acc8(a, src[i], w);
        dst[i] = pack8(a);
      }
    } else {
      for (int i = lane; i < D / 8; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
}

// dcomb[t,k] = <dout[t], Y[sel*C + slot]> (0 for dropped assignments).
__global__ void combine_bwd_weights_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ Y,
                                           const int* __restrict__ sel, const int* __restrict__ slot, int T, int K,
                                           int cap, int D, float* __restrict__ dcomb) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long i = blockIdx.x * (long)warps + (threadIdx.x >> 5); i < (long)T * K; i += (long)gridDim.x * warps) {
    const long t = i / K;
    const int s = slot[i];
    float acc = 0.f;
    if (s >= 0) {
      const long r = (long)sel[i] * cap + s;
      const uint4* a = reinterpret_cast<const uint4*>(dout + t * D);
      const uint4* b = reinterpret_cast<const uint4*>(Y + r * D);
      for (int c = lane; c < D / 8; c += 32) {
        uint4 ua = a[c], ub = b[c];
        const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&ua);
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&ub);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 fa = __bfloat1622float2(ha[j]), fb = __bfloat1622float2(hb[j]);
          acc += fa.x * fb.x + fa.y * fb.y;
        }
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) dcomb[i] = acc;
  }
}

// dx[t] = sum_k dXp[sel*C + slot] (+ dx_in[t] if given).
__global__ void unpermute_add_kernel(const __nv_bfloat16* __restrict__ dxp, const int* __restrict__ sel,
                                     const int* __restrict__ slot, const __nv_bfloat16* __restrict__ dx_in,
                                     __nv_bfloat16* __restrict__ dx, int T, int K, int cap, int D) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    for (int c = lane; c < D / 8; c += 32) {
      float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (dx_in) acc8(a, reinterpret_cast<const uint4*>(dx_in + (long)t * D)[c], 1.f);
      for (int k = 0; k < K; ++k) {
        const int s = slot[(long)t * K + k];
        if (s < 0) continue;
        const long r = (long)sel[(long)t * K + k] * cap + s;
        acc8(a, reinterpret_cast<const uint4*>(dxp + r * D)[c], 1.f);
      }
      reinterpret_cast<uint4*>(dx + (long)t * D)[c] = pack8(a);
    }
  }
}

inline int grid_for(long work, int per_block) {
  long g = (work + per_block - 1) / per_block;
  if (g > 148 * 16) g = 148 * 16;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

// -------------------------------------------------------------------------------- launchers
int launch_router_fwd(const float* logits, int ldl, const float* bias, int T, int E, int K, int adaptive,
                      const float* theta, int k_min, float temp, int* sel, float* comb, float* topb, float* alpha,
                      float* lse, uint8_t* keep, float* counts, float* psum, float* scalars, cudaStream_t st) {
  // a few warps' worth of tokens per block keeps the per-block flush of 2E + 3 atomics small
  const int grid = std::min(grid_for(T, 8), 148 * 4);
  const size_t sm = (2 * E + 3) * sizeof(float);
#define RF(EPL) router_fwd_kernel<EPL><<<grid, 256, sm, st>>>(logits, ldl, bias, T, E, K, adaptive, theta, k_min, \
                                                             temp, sel, comb, topb, alpha, lse, keep, counts, psum, scalars)
  count_launch();
  if (E <= 32) RF(1);
  else if (E <= 64) RF(2);
  else if (E <= 128) RF(4);
  else if (E <= 256) RF(8);
  else if (E <= 512) RF(16);
  else if (E <= 1024) RF(32);
  else return kErrBadArgsHost;
#undef RF
  return 0;
}

int launch_router_bwd(const float* logits, int ldl, const float* lse, const int* sel, const float* topb,
                      const uint8_t* keep, const float* dcomb, const float* counts, const float* dscal, int T, int E,
                      int K, int adaptive, const float* theta, int k_min, float temp, void* dlog, int ldd,
                      float* dtheta, cudaStream_t st) {
  const int grid = grid_for(T, 8);
#define RB(EPL) router_bwd_kernel<EPL><<<grid, 256, 0, st>>>(logits, ldl, lse, sel, topb, keep, dcomb, counts, dscal, \
                                                            T, E, K, adaptive, theta, k_min, temp,               \
                                                            (__nv_bfloat16*)dlog, ldd, dtheta)
  count_launch();
  if (E <= 32) RB(1);
  else if (E <= 64) RB(2);
  else if (E <= 128) RB(4);
  else if (E <= 256) RB(8);
  else if (E <= 512) RB(16);
  else if (E <= 1024) RB(32);
  else return kErrBadArgsHost;
#undef RB
  return 0;
}

void launch_qb_beta(const float* logits, int ldl, const float* alpha, int T, int E, int qb_count, float* beta,
                    cudaStream_t st) {
  count_launch();
  if (T <= kQbSmemKeys) {
    const size_t sm = (size_t)T * sizeof(uint32_t);
    static bool attr = false;
    if (!attr) {
      cudaFuncSetAttribute(qb_beta_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kQbSmemKeys * (int)sizeof(uint32_t));
      attr = true;
    }
    qb_beta_smem_kernel<<<E, 1024, sm, st>>>(logits, ldl, alpha, T, E, qb_count, beta);
    return;
  }
  qb_beta_kernel<<<E, 1024, 0, st>>>(logits, ldl, alpha, T, E, qb_count, beta);
}

int plan_workspace_ints(long n, int E) { return (int)(((n + kPlanChunk - 1) / kPlanChunk) * E); }

int plan_max_experts() { return kPlanMaxSmem / (33 * (int)sizeof(int)); }

int launch_dispatch_plan(const int* sel, const uint8_t* keep, const float* comb, long n, int K, int E, int cap,
                         int* blk_counts, int* slot, int* perm, float* wperm, int* counts, cudaStream_t st) {
  if (E <= 0 || E > plan_max_experts()) return kErrBadArgsHost;
  // The assign kernel keeps a running offset and 32 per-warp counts per expert in shared memory
  // (33 E ints): past 48 KB (E > 372) the launch needs the dynamic shared-memory opt-in, set once
  // per device for the largest size this launcher accepts.
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if (cudaFuncSetAttribute(plan_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPlanMaxSmem) !=
        cudaSuccess)
      return kErrBadArgsHost;
    attr_set[dev] = true;
  }
  const int nblk = (int)((n + kPlanChunk - 1) / kPlanChunk);
  count_launch();
  plan_count_kernel<<<nblk, 1024, E * sizeof(int), st>>>(sel, keep, n, E, blk_counts);
  count_launch();
  plan_assign_kernel<<<nblk, 1024, (33 * E) * sizeof(int), st>>>(sel, keep, comb, n, K, E, cap, blk_counts, nblk,
                                                                  slot, perm, wperm, counts);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

void launch_permute(const void* x, const int* perm, const int* counts, int cap, int E, int D, void* xp,
                    cudaStream_t st) {
  count_launch();
  permute_kernel<<<grid_for((long)E * cap, 8), 256, 0, st>>>((const __nv_bfloat16*)x, perm, counts, cap, E, D,
                                                             (__nv_bfloat16*)xp);
}

static bool gather_k(const void* Y, const int* sel, const int* slot, const float* W, const void* add, void* out,
                     int T, int K, int cap, int D, cudaStream_t st) {
  const auto* y = (const __nv_bfloat16*)Y;
  const auto* ad = (const __nv_bfloat16*)add;
  auto* o = (__nv_bfloat16*)out;
  if (K <= 4) {
    gather_k_kernel<4><<<grid_for(T, 8), 256, 0, st>>>(y, sel, slot, W, ad, o, T, K, cap, D);
    return true;
  }
  if (K <= 8) {
    gather_k_kernel<8><<<grid_for(T, 8), 256, 0, st>>>(y, sel, slot, W, ad, o, T, K, cap, D);
    return true;
  }
  return false;
}

void launch_combine(const void* Y, const int* sel, const int* slot, const float* comb, const void* residual,
                    void* out, int T, int K, int cap, int D, cudaStream_t st) {
  count_launch();
  if (gather_k(Y, sel, slot, comb, residual, out, T, K, cap, D, st)) return;
  combine_kernel<<<grid_for(T, 8), 256, 0, st>>>((const __nv_bfloat16*)Y, sel, slot, comb,
                                                 (const __nv_bfloat16*)residual, (__nv_bfloat16*)out, T, K, cap, D);
}

void launch_combine_bwd(const void* dout, const void* Y, const int* sel, const int* slot, const int* perm,
                        const float* wperm, const int* counts, int T, int K, int cap, int E, int D, void* dY,
                        float* dcomb, cudaStream_t st) {
  if (dY) {  // the expert-parallel path pushes these rows to the owners itself
    count_launch();
    combine_bwd_rows_kernel<<<grid_for((long)E * cap, 8), 256, 0, st>>>((const __nv_bfloat16*)dout, perm, wperm,
                                                                        counts, cap, E, D, (__nv_bfloat16*)dY);
  }
  count_launch();
  combine_bwd_weights_kernel<<<grid_for((long)T * K, 8), 256, 0, st>>>(
      (const __nv_bfloat16*)dout, (const __nv_bfloat16*)Y, sel, slot, T, K, cap, D, dcomb);
}

void launch_unpermute_add(const void* dxp, const int* sel, const int* slot, const void* dx_in, void* dx, int T, int K,
                          int cap, int D, cudaStream_t st) {
  count_launch();
  if (gather_k(dxp, sel, slot, nullptr, dx_in, dx, T, K, cap, D, st)) return;
  unpermute_add_kernel<<<grid_for(T, 8), 256, 0, st>>>((const __nv_bfloat16*)dxp, sel, slot,
                                                       (const __nv_bfloat16*)dx_in, (__nv_bfloat16*)dx, T, K, cap, D);
}

}  // namespace mxk
