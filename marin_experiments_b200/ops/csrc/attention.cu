// Causal flash attention, forward and backward, for bf16 q/k/v with fp32 softmax statistics.
// Supports grouped-query attention, a sliding window (key j visible to query i iff
// 0 <= i - j < window) and packed-document segment ids (visible iff same segment).
//
// Forward: one CTA per (128-query block, head, batch), 8 warps x 16 query rows, 64-key blocks
// double-buffered with cp.async; online softmax in registers (exp2 domain); P is fed back to the
// PV product straight from the score accumulators. Writes O and lse (natural log).
// Backward: one CTA per (128-key block, kv head, batch), 8 warps x 16 key rows; loops over the q
// heads of the kv group and over 64-query blocks. dK/dV accumulate in registers; dQ is
// accumulated in an fp32 buffer with vector atomics and converted at the end.
// Tensor-core math: mma.sync m16n8k16 bf16 -> fp32, operands staged with ldmatrix.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace mxk {
namespace {

struct AttnParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long q_tok, q_head;  // element strides
  long k_tok, k_head;
  long v_tok, v_head;
  __nv_bfloat16* o;  // [T, H, hd]
  float* lse;        // [T, H]
  const int* seg;    // [T] or null
  int B, S, H, Hkv;
  int window;
  float scale;
  // backward
  const __nv_bfloat16* dout;  // [T, H, hd]
  const float* dsum;          // [T, H]  rowsum(dO * O)
  float* dq_acc;              // [T, H, hd] fp32
  __nv_bfloat16* dk;
  long dk_tok, dk_head;
  __nv_bfloat16* dv;  // added into (dv += ...)
  long dv_tok, dv_head;
  int dv_accumulate;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ bool visible(int qi, int kj, int S, int window, const int* seg, int base) {
  if (kj > qi || kj >= S || qi >= S) return false;
  if (window > 0 && qi - kj >= window) return false;
  if (seg && seg[base + qi] != seg[base + kj]) return false;
  return true;
}

// Load `rows` rows of a [tokens, heads, hd]-strided tensor into smem (row stride LDS elements).
template <int HD, int LDS>
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, long tok_stride, int row0,
                                          int rows, int S, int tid, int nthreads) {
  constexpr int CH = HD / 8;
  for (int i = tid; i < rows * CH; i += nthreads) {
    const int r = i / CH, c = i % CH;
    const int tok = row0 + r;
    const bool ok = tok < S;
    const __nv_bfloat16* s = src + (long)(ok ? tok : 0) * tok_stride + c * 8;
    cp_async16(dst + r * LDS + c * 8, s, ok);
  }
}

// ------------------------------------------------------------------------------------ forward
template <int HD>
__global__ void __launch_bounds__(256) flash_fwd_kernel(const AttnParams p) {
  constexpr int BM = 128, BN = 64, LDS = HD + 8, KS = HD / 16, NT = HD / 8;
  extern __shared__ __align__(16) __nv_bfloat16 smem[];
  __nv_bfloat16* sQ = smem;
  __nv_bfloat16* sK = sQ + BM * LDS;
  __nv_bfloat16* sV = sK + 2 * BN * LDS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int q0 = blockIdx.x * BM, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (p.H / p.Hkv);
  const int base = b * p.S;
  const __nv_bfloat16* Qg = p.q + (long)base * p.q_tok + (long)h * p.q_head;
  const __nv_bfloat16* Kg = p.k + (long)base * p.k_tok + (long)kh * p.k_head;
  const __nv_bfloat16* Vg = p.v + (long)base * p.v_tok + (long)kh * p.v_head;

  int kb_lo = 0;
  if (p.window > 0) kb_lo = max(0, q0 - p.window + 1) / BN;
  const int kb_hi = (min(p.S, q0 + BM) + BN - 1) / BN;  // exclusive

  load_tile<HD, LDS>(sQ, Qg, p.q_tok, q0, BM, p.S, tid, 256);
  if (kb_lo < kb_hi) {
    load_tile<HD, LDS>(sK, Kg, p.k_tok, kb_lo * BN, BN, p.S, tid, 256);
    load_tile<HD, LDS>(sV, Vg, p.v_tok, kb_lo * BN, BN, p.S, tid, 256);
  }
  cp_async_commit();

  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = p.scale * 1.4426950408889634f;
  const int qr0 = q0 + warp * 16 + g, qr1 = qr0 + 8;
  uint32_t qa[KS][4];

  for (int kb = kb_lo; kb < kb_hi; ++kb) {
    const int buf = (kb - kb_lo) & 1;
    if (kb + 1 < kb_hi) {
      load_tile<HD, LDS>(sK + (buf ^ 1) * BN * LDS, Kg, p.k_tok, (kb + 1) * BN, BN, p.S, tid, 256);
      load_tile<HD, LDS>(sV + (buf ^ 1) * BN * LDS, Vg, p.v_tok, (kb + 1) * BN, BN, p.S, tid, 256);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == kb_lo) {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
        ldsm_x4(qa[ks], sQ + (warp * 16 + (lane & 15)) * LDS + ks * 16 + (lane >> 4) * 8);
    }
    const __nv_bfloat16* cK = sK + buf * BN * LDS;
    const __nv_bfloat16* cV = sV + buf * BN * LDS;
    // S = Q K^T : 16 x 64 per warp
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t kb4[4];
        // rows n0..n0+15 (two n-tiles), cols ks*16 .. +15
        const int n_row = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int k_col = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(kb4, cK + n_row * LDS + k_col);
        mma16816(s[2 * jp], qa[ks], kb4[0], kb4[1]);
        mma16816(s[2 * jp + 1], qa[ks], kb4[2], kb4[3]);
      }
    }
    // mask + scale (log2 domain)
    const int k0 = kb * BN;
    const bool need_mask = (k0 + BN - 1 > q0) || (p.window > 0 && k0 < q0 + BM - p.window) || p.seg != nullptr ||
                           (k0 + BN > p.S);
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = (e < 2) ? qr0 : qr1;
        const int kj = k0 + j * 8 + 2 * c4 + (e & 1);
        float v = s[j][e] * sl2;
        if (need_mask && !visible(qi, kj, p.S, p.window, p.seg, base)) v = -INFINITY;
        s[j][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float b0 = nm0 == -INFINITY ? 0.f : nm0, b1 = nm1 == -INFINITY ? 0.f : nm1;
    const float a0 = exp2f(m0 - b0), a1 = exp2f(m1 - b1);
    m0 = nm0;
    m1 = nm1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = exp2f(s[j][0] - b0);
      s[j][1] = exp2f(s[j][1] - b0);
      s[j][2] = exp2f(s[j][2] - b1);
      s[j][3] = exp2f(s[j][3] - b1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a0;
      o[i][2] *= a1;
      o[i][3] *= a1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
      uint32_t pa[4];
      pa[0] = pack2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t vb[4];
        // V rows (keys) kk*16 .. +15, cols (d) np*16 .. +15, transposed fragments
        const int k_row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int d_col = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(vb, cV + k_row * LDS + d_col);
        mma16816(o[2 * np], pa, vb[0], vb[1]);
        mma16816(o[2 * np + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();
  }
  // finalize
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const float ln2 = 0.6931471805599453f;
  if (qr0 < p.S) {
    __nv_bfloat16* orow = p.o + ((long)(base + qr0) * p.H + h) * HD;
#pragma unroll
    for (int i = 0; i < NT; ++i)
      *reinterpret_cast<uint32_t*>(orow + i * 8 + 2 * c4) = pack2(o[i][0] * inv0, o[i][1] * inv0);
    if (c4 == 0) p.lse[(long)(base + qr0) * p.H + h] = l0 > 0.f ? (m0 + log2f(l0)) * ln2 : INFINITY;
  }
  if (qr1 < p.S) {
    __nv_bfloat16* orow = p.o + ((long)(base + qr1) * p.H + h) * HD;
#pragma unroll
    for (int i = 0; i < NT; ++i)
      *reinterpret_cast<uint32_t*>(orow + i * 8 + 2 * c4) = pack2(o[i][2] * inv1, o[i][3] * inv1);
    if (c4 == 0) p.lse[(long)(base + qr1) * p.H + h] = l1 > 0.f ? (m1 + log2f(l1)) * ln2 : INFINITY;
  }
}

// ------------------------------------------------------------------------------ backward prep
// dsum[t,h] = sum_d dO * O ; zero dq_acc.
template <int HD>
__global__ void flash_bwd_prep_kernel(const AttnParams p, long T) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long i = blockIdx.x * (long)warps + (threadIdx.x >> 5); i < T * p.H; i += (long)gridDim.x * warps) {
    const __nv_bfloat16* a = p.dout + i * HD;
    const __nv_bfloat16* o = p.o + i * HD;
    float acc = 0.f;
    for (int d = lane; d < HD; d += 32) acc += __bfloat162float(a[d]) * __bfloat162float(o[d]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) const_cast<float*>(p.dsum)[i] = acc;
    if (p.dq_acc)
      for (int d = lane; d < HD; d += 32) p.dq_acc[i * HD + d] = 0.f;
  }
}

// ----------------------------------------------------------------------------------- backward
template <int HD>
__global__ void __launch_bounds__(256) flash_bwd_kernel(const AttnParams p) {
  constexpr int BN = 128, BM = 64, LDS = HD + 8, KS = HD / 16, NT = HD / 8;
  constexpr int LDP = BN + 8;  // dS tile row stride ([query][key])
  extern __shared__ __align__(16) __nv_bfloat16 smem[];
  __nv_bfloat16* sK = smem;                  // BN x LDS
  __nv_bfloat16* sV = sK + BN * LDS;         // BN x LDS
  __nv_bfloat16* sQ = sV + BN * LDS;         // 2 x BM x LDS
  __nv_bfloat16* sO = sQ + 2 * BM * LDS;     // 2 x BM x LDS  (dO)
  __nv_bfloat16* sS = sO + 2 * BM * LDS;     // BM x LDP      (dS, [query][key])
  float* sL = reinterpret_cast<float*>(sS + BM * LDP);  // 2 x BM lse
  float* sD = sL + 2 * BM;                               // 2 x BM dsum
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int k0 = blockIdx.x * BN, kh = blockIdx.y, b = blockIdx.z;
  const int rep = p.H / p.Hkv;
  const int base = b * p.S;
  const __nv_bfloat16* Kg = p.k + (long)base * p.k_tok + (long)kh * p.k_head;
  const __nv_bfloat16* Vg = p.v + (long)base * p.v_tok + (long)kh * p.v_head;
  load_tile<HD, LDS>(sK, Kg, p.k_tok, k0, BN, p.S, tid, 256);
  load_tile<HD, LDS>(sV, Vg, p.v_tok, k0, BN, p.S, tid, 256);
  cp_async_commit();

  float dk[NT][4], dv[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  const int qb_lo = k0 / BM;
  int qb_hi = (p.S + BM - 1) / BM;
  if (p.window > 0) qb_hi = min(qb_hi, (k0 + BN - 1 + p.window - 1) / BM + 1);
  const int nq = qb_hi - qb_lo;
  const int total = nq * rep;
  const float sl2 = p.scale * 1.4426950408889634f;
  const int kr = k0 + warp * 16 + g;  // this thread's key rows: kr, kr + 8

  auto issue = [&](int it, int buf) {
    const int hq = kh * rep + it / nq;
    const int qb = qb_lo + it % nq;
    const __nv_bfloat16* Qg = p.q + (long)base * p.q_tok + (long)hq * p.q_head;
    const __nv_bfloat16* Og = p.dout + ((long)base * p.H + hq) * HD;
    load_tile<HD, LDS>(sQ + buf * BM * LDS, Qg, p.q_tok, qb * BM, BM, p.S, tid, 256);
    load_tile<HD, LDS>(sO + buf * BM * LDS, Og, (long)p.H * HD, qb * BM, BM, p.S, tid, 256);
    if (tid < BM) {
      const int qi = qb * BM + tid;
      sL[buf * BM + tid] = qi < p.S ? p.lse[(long)(base + qi) * p.H + hq] : INFINITY;
      sD[buf * BM + tid] = qi < p.S ? p.dsum[(long)(base + qi) * p.H + hq] : 0.f;
    }
  };
  if (total > 0) issue(0, 0);
  cp_async_commit();

  for (int it = 0; it < total; ++it) {
    const int buf = it & 1;
    const int hq = kh * rep + it / nq;
    const int q0 = (qb_lo + it % nq) * BM;
    if (it + 1 < total) issue(it + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const __nv_bfloat16* cQ = sQ + buf * BM * LDS;
    const __nv_bfloat16* cO = sO + buf * BM * LDS;
    const float* cL = sL + buf * BM;
    const float* cD = sD + buf * BM;
    // S^T = K Q^T  (16 keys x 64 queries per warp)
    float st[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) st[j][0] = st[j][1] = st[j][2] = st[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t ka[4];
      ldsm_x4(ka, sK + (warp * 16 + (lane & 15)) * LDS + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t qb4[4];
        const int n_row = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int k_col = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(qb4, cQ + n_row * LDS + k_col);
        mma16816(st[2 * jp], ka, qb4[0], qb4[1]);
        mma16816(st[2 * jp + 1], ka, qb4[2], qb4[3]);
      }
    }
    // P^T = exp(S^T * scale - lse[q])
    const bool need_mask = (q0 < k0 + BN - 1) || (p.window > 0 && q0 + BM - 1 - k0 >= p.window) ||
                           p.seg != nullptr || (q0 + BM > p.S) || (k0 + BN > p.S);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = (e < 2) ? kr : kr + 8;
        const int ql = j * 8 + 2 * c4 + (e & 1);
        const int qi = q0 + ql;
        float v = exp2f(st[j][e] * sl2 - cL[ql] * 1.4426950408889634f);
        if (need_mask && !visible(qi, kj, p.S, p.window, p.seg, base)) v = 0.f;
        st[j][e] = v;
      }
    }
    // dV += P^T dO
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack2(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t ob[4];
        const int q_row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int d_col = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(ob, cO + q_row * LDS + d_col);
        mma16816(dv[2 * np], pa, ob[0], ob[1]);
        mma16816(dv[2 * np + 1], pa, ob[2], ob[3]);
      }
    }
    // dP^T = V dO^T
    float dp[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) dp[j][0] = dp[j][1] = dp[j][2] = dp[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t va[4];
      ldsm_x4(va, sV + (warp * 16 + (lane & 15)) * LDS + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        uint32_t ob4[4];
        const int n_row = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int k_col = ks * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(ob4, cO + n_row * LDS + k_col);
        mma16816(dp[2 * jp], va, ob4[0], ob4[1]);
        mma16816(dp[2 * jp + 1], va, ob4[2], ob4[3]);
      }
    }
    // dS^T = P^T * (dP^T - D[q]) ; store dS ([query][key]) to smem for the dQ product
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = j * 8 + 2 * c4 + (e & 1);
        st[j][e] = st[j][e] * (dp[j][e] - cD[ql]);
      }
      const int kl0 = warp * 16 + g, kl1 = kl0 + 8;
      const int ql0 = j * 8 + 2 * c4;
      sS[ql0 * LDP + kl0] = __float2bfloat16(st[j][0]);
      sS[(ql0 + 1) * LDP + kl0] = __float2bfloat16(st[j][1]);
      sS[ql0 * LDP + kl1] = __float2bfloat16(st[j][2]);
      sS[(ql0 + 1) * LDP + kl1] = __float2bfloat16(st[j][3]);
    }
    // dK += dS^T Q (scale applied at the end)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack2(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack2(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack2(st[2 * kk + 1][2], st[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t qb[4];
        const int q_row = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int d_col = np * 16 + (lane >> 4) * 8;
        ldsm_x4_t(qb, cQ + q_row * LDS + d_col);
        mma16816(dk[2 * np], pa, qb[0], qb[1]);
        mma16816(dk[2 * np + 1], pa, qb[2], qb[3]);
      }
    }
    __syncthreads();
    // dQ[64 x HD] = dS [64 x 128] K [128 x HD]; warps: 4 row groups x 2 column halves
    {
      const int rg = warp & 3, ch = warp >> 2;
      constexpr int NTH = NT / 2;  // n-tiles per half
      static_assert(NTH % 2 == 0, "head_dim must be a multiple of 32");
      float acc[NTH][4];
#pragma unroll
      for (int i = 0; i < NTH; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < BN / 16; ++ks) {
        uint32_t sa[4];
        ldsm_x4(sa, sS + (rg * 16 + (lane & 15)) * LDP + ks * 16 + (lane >> 4) * 8);
#pragma unroll
        for (int np = 0; np < NTH / 2; ++np) {
          uint32_t kb4[4];
          const int k_row = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int d_col = ch * (HD / 2) + np * 16 + (lane >> 4) * 8;
          ldsm_x4_t(kb4, sK + k_row * LDS + d_col);
          mma16816(acc[2 * np], sa, kb4[0], kb4[1]);
          mma16816(acc[2 * np + 1], sa, kb4[2], kb4[3]);
        }
      }
      const int qa0 = q0 + rg * 16 + g, qa1 = qa0 + 8;
#pragma unroll
      for (int i = 0; i < NTH; ++i) {
        const int d = ch * (HD / 2) + i * 8 + 2 * c4;
        if (qa0 < p.S)
          atomicAdd(reinterpret_cast<float2*>(p.dq_acc + ((long)(base + qa0) * p.H + hq) * HD + d),
                    make_float2(acc[i][0] * p.scale, acc[i][1] * p.scale));
        if (qa1 < p.S)
          atomicAdd(reinterpret_cast<float2*>(p.dq_acc + ((long)(base + qa1) * p.H + hq) * HD + d),
                    make_float2(acc[i][2] * p.scale, acc[i][3] * p.scale));
      }
    }
    __syncthreads();
  }
  // write dK (scaled) and dV (optionally accumulated into existing values)
  const int kr1 = kr + 8;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int d = i * 8 + 2 * c4;
    if (kr < p.S) {
      *reinterpret_cast<uint32_t*>(p.dk + (long)(base + kr) * p.dk_tok + (long)kh * p.dk_head + d) =
          pack2(dk[i][0] * p.scale, dk[i][1] * p.scale);
      __nv_bfloat16* dvp = p.dv + (long)(base + kr) * p.dv_tok + (long)kh * p.dv_head + d;
      float a = dv[i][0], bb = dv[i][1];
      if (p.dv_accumulate) {
        __nv_bfloat162 old = *reinterpret_cast<__nv_bfloat162*>(dvp);
        a += __bfloat162float(old.x);
        bb += __bfloat162float(old.y);
      }
      *reinterpret_cast<uint32_t*>(dvp) = pack2(a, bb);
    }
    if (kr1 < p.S) {
      *reinterpret_cast<uint32_t*>(p.dk + (long)(base + kr1) * p.dk_tok + (long)kh * p.dk_head + d) =
          pack2(dk[i][2] * p.scale, dk[i][3] * p.scale);
      __nv_bfloat16* dvp = p.dv + (long)(base + kr1) * p.dv_tok + (long)kh * p.dv_head + d;
      float a = dv[i][2], bb = dv[i][3];
      if (p.dv_accumulate) {
        __nv_bfloat162 old = *reinterpret_cast<__nv_bfloat162*>(dvp);
        a += __bfloat162float(old.x);
        bb += __bfloat162float(old.y);
      }
      *reinterpret_cast<uint32_t*>(dvp) = pack2(a, bb);
    }
  }
}

__global__ void dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n / 2; i += (long)gridDim.x * blockDim.x) {
    float2 v = reinterpret_cast<const float2*>(acc)[i];
    reinterpret_cast<__nv_bfloat162*>(dq)[i] = __floats2bfloat162_rn(v.x, v.y);
  }
}

template <int HD>
size_t fwd_smem() {
  return (size_t)(128 + 4 * 64) * (HD + 8) * 2;
}
template <int HD>
size_t bwd_smem() {
  return (size_t)(2 * 128 + 4 * 64) * (HD + 8) * 2 + 64 * (128 + 8) * 2 + 4 * 64 * 4;
}

template <int HD>
int run_fwd(const AttnParams& p, cudaStream_t st) {
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(flash_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_smem<HD>());
    init = true;
  }
  dim3 grid((p.S + 127) / 128, p.H, p.B);
  count_launch();
  flash_fwd_kernel<HD><<<grid, 256, fwd_smem<HD>(), st>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

template <int HD>
int run_bwd(const AttnParams& p, cudaStream_t st) {
  static bool init = false;
  if (!init) {
    cudaFuncSetAttribute(flash_bwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bwd_smem<HD>());
    init = true;
  }
  const long T = (long)p.B * p.S;
  count_launch();
  flash_bwd_prep_kernel<HD><<<148 * 8, 256, 0, st>>>(p, T);
  dim3 grid((p.S + 127) / 128, p.Hkv, p.B);
  count_launch();
  flash_bwd_kernel<HD><<<grid, 256, bwd_smem<HD>(), st>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

}  // namespace

int launch_flash_fwd(const AttnLaunch& L, cudaStream_t st) {
  AttnParams p{};
  p.q = (const __nv_bfloat16*)L.q;
  p.k = (const __nv_bfloat16*)L.k;
  p.v = (const __nv_bfloat16*)L.v;
  p.q_tok = L.q_tok; p.q_head = L.q_head;
  p.k_tok = L.k_tok; p.k_head = L.k_head;
  p.v_tok = L.v_tok; p.v_head = L.v_head;
  p.o = (__nv_bfloat16*)L.o;
  p.lse = L.lse;
  p.seg = L.seg;
  p.B = L.B; p.S = L.S; p.H = L.H; p.Hkv = L.Hkv;
  p.window = L.window;
  p.scale = L.scale;
  switch (L.hd) {
    case 64: return run_fwd<64>(p, st);
    case 96: return run_fwd<96>(p, st);
    case 128: return run_fwd<128>(p, st);
    default: return kErrBadArgsHost;
  }
}

// dsum = rowsum(dO * O) and dq_acc = 0 for the tcgen05 backward (attention_bwd_sm100.cu).
int launch_flash_bwd_prep(const AttnLaunch& L, cudaStream_t st) {
  AttnParams p{};
  p.o = (__nv_bfloat16*)L.o;
  p.H = L.H;
  p.dout = (const __nv_bfloat16*)L.dout;
  p.dsum = L.dsum;
  p.dq_acc = L.dq_acc;
  const long T = (long)L.B * L.S;
  count_launch();
  switch (L.hd) {
    case 64: flash_bwd_prep_kernel<64><<<148 * 8, 256, 0, st>>>(p, T); break;
    case 96: flash_bwd_prep_kernel<96><<<148 * 8, 256, 0, st>>>(p, T); break;
    case 128: flash_bwd_prep_kernel<128><<<148 * 8, 256, 0, st>>>(p, T); break;
    default: return kErrBadArgsHost;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

int launch_dq_convert(const AttnLaunch& L, cudaStream_t st) {
  const long n = (long)L.B * L.S * L.H * L.hd;
  count_launch();
  dq_convert_kernel<<<148 * 8, 256, 0, st>>>(L.dq_acc, (__nv_bfloat16*)L.dq, n);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

int launch_flash_bwd(const AttnLaunch& L, cudaStream_t st) {
  AttnParams p{};
  p.q = (const __nv_bfloat16*)L.q;
  p.k = (const __nv_bfloat16*)L.k;
  p.v = (const __nv_bfloat16*)L.v;
  p.q_tok = L.q_tok; p.q_head = L.q_head;
  p.k_tok = L.k_tok; p.k_head = L.k_head;
  p.v_tok = L.v_tok; p.v_head = L.v_head;
  p.o = (__nv_bfloat16*)L.o;
  p.lse = L.lse;
  p.seg = L.seg;
  p.B = L.B; p.S = L.S; p.H = L.H; p.Hkv = L.Hkv;
  p.window = L.window;
  p.scale = L.scale;
  p.dout = (const __nv_bfloat16*)L.dout;
  p.dsum = L.dsum;
  p.dq_acc = L.dq_acc;
  p.dk = (__nv_bfloat16*)L.dk;
  p.dk_tok = L.dk_tok; p.dk_head = L.dk_head;
  p.dv = (__nv_bfloat16*)L.dv;
  p.dv_tok = L.dv_tok; p.dv_head = L.dv_head;
  p.dv_accumulate = L.dv_accumulate;
  int r;
  switch (L.hd) {
    case 64: r = run_bwd<64>(p, st); break;
    case 96: r = run_bwd<96>(p, st); break;
    case 128: r = run_bwd<128>(p, st); break;
    default: return kErrBadArgsHost;
  }
  if (r) return r;
  const long n = (long)L.B * L.S * L.H * L.hd;
  count_launch();
  dq_convert_kernel<<<148 * 8, 256, 0, st>>>(L.dq_acc, (__nv_bfloat16*)L.dq, n);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

}  // namespace mxk
