// Row-wise and elementwise sm_100a kernels: RMSNorm, embedding gather / scatter-add,
// QK-norm + RoPE, exclusive self-attention + head gate, activation backward passes and the
// cross-entropy gradient. All are bandwidth-bound; rows are processed one warp each with
// 16-byte vector accesses.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <initializer_list>

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

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ void load8f(const float* p, float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ float2 unpack2(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}

__device__ __forceinline__ float sigm(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// ------------------------------------------------------------------------------------ RMSNorm
// y = x * rsqrt(mean(x^2) + eps) * w ; one warp per row, D a multiple of 8.
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd, int T, int D,
                                   float eps) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < T; row += gridDim.x * warps) {
    const __nv_bfloat16* xr = x + (long)row * D;
    float ss = 0.f;
    for (int c = lane * 8; c < D; c += 256) {
      float f[8];
      load8(xr + c, f);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += f[i] * f[i];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
    if (lane == 0) rstd[row] = r;
    for (int c = lane * 8; c < D; c += 256) {
      float f[8];
      load8(xr + c, f);
      float4 w0 = *reinterpret_cast<const float4*>(w + c);
      float4 w1 = *reinterpret_cast<const float4*>(w + c + 4);
      float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = f[i] * r * wv[i];
      store8(y + (long)row * D + c, f);
    }
  }
}

// dx = r * (g - xhat * mean(g * xhat)), g = dy * w, xhat = x * r ; dw += sum_rows dy * xhat.
// One warp per row; a row's dy and x vectors stay in registers between the two passes and w is
// staged once per block in shared memory. dw partials are kept per lane in registers (column
// slots fixed per lane) and flushed with one atomicAdd per column per block. Optional dres is
// added to dx (residual-stream gradient).
template <int MAXV>
__global__ void __launch_bounds__(256, 2)
    rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                       const float* __restrict__ w, const float* __restrict__ rstd,
                       const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                       float* __restrict__ dw, int T, int D) {
  extern __shared__ float sm_rms[];  // [D] dw partials, [D] w
  float* sdw = sm_rms;
  float* sw = sm_rms + D;
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    sdw[c] = 0.f;
    sw[c] = w[c];
  }
  __syncthreads();
  float acc[MAXV][8];
#pragma unroll
  for (int v = 0; v < MAXV; ++v)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[v][i] = 0.f;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < T; row += gridDim.x * warps) {
    const float r = rstd[row];
    uint4 gu[MAXV], xu[MAXV];
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int c = lane * 8 + v * 256;
      if (c < D) {
        gu[v] = *reinterpret_cast<const uint4*>(dy + (long)row * D + c);
        xu[v] = *reinterpret_cast<const uint4*>(x + (long)row * D + c);
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int c = lane * 8 + v * 256;
      if (c < D) {
        float wv[8];
        load8f(sw + c, wv);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 g = unpack2(reinterpret_cast<const uint32_t*>(&gu[v])[k]);
          const float2 xv = unpack2(reinterpret_cast<const uint32_t*>(&xu[v])[k]);
          const float xh0 = xv.x * r, xh1 = xv.y * r;
          acc[v][2 * k] += g.x * xh0;
          acc[v][2 * k + 1] += g.y * xh1;
          dot += g.x * wv[2 * k] * xh0 + g.y * wv[2 * k + 1] * xh1;
        }
      }
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int c = lane * 8 + v * 256;
      if (c < D) {
        float wv[8], o[8], rr[8];
        load8f(sw + c, wv);
        if (dres) load8(dres + (long)row * D + c, rr);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 g = unpack2(reinterpret_cast<const uint32_t*>(&gu[v])[k]);
          const float2 xv = unpack2(reinterpret_cast<const uint32_t*>(&xu[v])[k]);
          o[2 * k] = r * (g.x * wv[2 * k] - xv.x * r * dot);
          o[2 * k + 1] = r * (g.y * wv[2 * k + 1] - xv.y * r * dot);
        }
        if (dres) {
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] += rr[i];
        }
        store8(dx + (long)row * D + c, o);
      }
    }
  }
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int c = lane * 8 + v * 256;
    if (c < D)
#pragma unroll
      for (int i = 0; i < 8; ++i) atomicAdd(&sdw[c + i], acc[v][i]);
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) atomicAdd(&dw[c], sdw[c]);
}

// The same backward with the weight-gradient partials in shared memory: each warp owns a private
// [MAXV * 8][32] float region (conflict-free: lane = fastest index) instead of MAXV * 8 registers per
// thread, so three 8-warp blocks fit an SM (24 warps against 16) and more rows' loads are in flight.
template <int MAXV>
__global__ void __launch_bounds__(256, 3)
    rmsnorm_bwd_smem_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                            const float* __restrict__ w, const float* __restrict__ rstd,
                            const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx,
                            float* __restrict__ dw, int T, int D) {
  extern __shared__ float sm_rms2[];
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* sw = sm_rms2;                                  // [D]
  float* pacc = sm_rms2 + D + warp * (MAXV * 8 * 32);  // this warp's [MAXV * 8][32] partials
  for (int c = threadIdx.x; c < D; c += blockDim.x) sw[c] = w[c];
#pragma unroll
  for (int i = 0; i < MAXV * 8; ++i) pacc[i * 32 + lane] = 0.f;
  __syncthreads();
  for (int row = blockIdx.x * warps + warp; row < T; row += gridDim.x * warps) {
    const float r = rstd[row];
    uint4 gu[MAXV], xu[MAXV];
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int c = lane * 8 + v * 256;
      if (c < D) {
        gu[v] = *reinterpret_cast<const uint4*>(dy + (long)row * D + c);
        xu[v] = *reinterpret_cast<const uint4*>(x + (long)row * D + c);
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int c = lane * 8 + v * 256;
      if (c < D) {
        float wv[8];
        load8f(sw + c, wv);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 g = unpack2(reinterpret_cast<const uint32_t*>(&gu[v])[k]);
          const float2 xv = unpack2(reinterpret_cast<const uint32_t*>(&xu[v])[k]);
          const float xh0 = xv.x * r, xh1 = xv.y * r;
          pacc[(v * 8 + 2 * k) * 32 + lane] += g.x * xh0;
          pacc[(v * 8 + 2 * k + 1) * 32 + lane] += g.y * xh1;
          dot += g.x * wv[2 * k] * xh0 + g.y * wv[2 * k + 1] * xh1;
        }
      }
    }
    dot = warp_sum(dot) / D;
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int c = lane * 8 + v * 256;
      if (c < D) {
        float wv[8], o[8], rr[8];
        load8f(sw + c, wv);
        if (dres) load8(dres + (long)row * D + c, rr);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 g = unpack2(reinterpret_cast<const uint32_t*>(&gu[v])[k]);
          const float2 xv = unpack2(reinterpret_cast<const uint32_t*>(&xu[v])[k]);
          o[2 * k] = r * (g.x * wv[2 * k] - xv.x * r * dot);
          o[2 * k + 1] = r * (g.y * wv[2 * k + 1] - xv.y * r * dot);
        }
        if (dres) {
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] += rr[i];
        }
        store8(dx + (long)row * D + c, o);
      }
    }
  }
  __syncthreads();
  // column c = 256 v + 8 lane + i lives at [(8 v + i) * 32 + lane] of every warp's region
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    const int v = c >> 8, ln = (c & 255) >> 3, i = c & 7;
    float sum = 0.f;
    for (int wp = 0; wp < warps; ++wp) sum += sm_rms2[D + wp * (MAXV * 8 * 32) + (v * 8 + i) * 32 + ln];
    atomicAdd(&dw[c], sum);
  }
}

// ----------------------------------------------------------------------------------- embedding
__global__ void embed_fwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int T, int D, int V) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < T; row += gridDim.x * warps) {
    long id = ids[row];
    if (id < 0 || id >= V) id = 0;
    const uint4* src = reinterpret_cast<const uint4*>(table + id * (long)D);
    uint4* dst = reinterpret_cast<uint4*>(out + (long)row * D);
    for (int c = lane; c < D / 8; c += 32) dst[c] = src[c];
  }
}

__global__ void embed_bwd_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dout,
                                 float* __restrict__ dtable, int T, int D, int V) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  for (int row = blockIdx.x * warps + (threadIdx.x >> 5); row < T; row += gridDim.x * warps) {
    long id = ids[row];
    if (id < 0 || id >= V) continue;
    float* dst = dtable + id * (long)D;
    for (int c = lane * 8; c < D; c += 256) {
      float f[8];
      load8(dout + (long)row * D + c, f);
      atomicAdd(reinterpret_cast<float4*>(dst + c), make_float4(f[0], f[1], f[2], f[3]));
      atomicAdd(reinterpret_cast<float4*>(dst + c + 4), make_float4(f[4], f[5], f[6], f[7]));
    }
  }
}

// ---------------------------------------------------------------------------- GatedNorm / acts
// out = y * sigmoid(z):  dy_direct = dout * s ; dz = dout * y * s * (1 - s)
__global__ void gate_mul_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                                    const __nv_bfloat16* __restrict__ z, __nv_bfloat16* __restrict__ dy,
                                    __nv_bfloat16* __restrict__ dz, long n8) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float d[8], yv[8], zv[8], a[8], b[8];
    load8(dout + i * 8, d);
    load8(y + i * 8, yv);
    load8(z + i * 8, zv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float s = sigm(zv[k]);
      a[k] = d[k] * s;
      b[k] = d[k] * yv[k] * s * (1.f - s);
    }
    store8(dy + i * 8, a);
    store8(dz + i * 8, b);
  }
}

__device__ __forceinline__ float act_f(float x, int kind) {
  if (kind == 1) return fmaxf(x, 0.f);
  if (kind == 2) {
    const float u = 0.7978845608f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.f + tanhf(u));
  }
  return x * sigm(x);
}

__device__ __forceinline__ float act_grad(float x, int kind) {
  if (kind == 1) return x > 0.f ? 1.f : 0.f;
  if (kind == 2) {
    const float u = 0.7978845608f * (x + 0.044715f * x * x * x);
    const float t = tanhf(u);
    const float du = 0.7978845608f * (1.f + 3.f * 0.044715f * x * x);
    return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * du;
  }
  const float s = sigm(x);
  return s * (1.f + x * (1.f - s));
}

// dh = dact * act'(h)
__global__ void act_bwd_kernel(const __nv_bfloat16* __restrict__ da, const __nv_bfloat16* __restrict__ h,
                               __nv_bfloat16* __restrict__ dh, long n8, int kind) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    float d[8], hv[8], o[8];
    load8(da + i * 8, d);
    load8(h + i * 8, hv);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = d[k] * act_grad(hv[k], kind);
    store8(dh + i * 8, o);
  }
}

// Blocked SwiGLU backward: H row = [g(128) u(128)] x I/128 ; dact row = I.
// dg = dact * u * act'(g) ; du = dact * act(g)
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dact, const __nv_bfloat16* __restrict__ H,
                                  __nv_bfloat16* __restrict__ dH, long rows, int I, int kind,
                                  const int* __restrict__ counts, int cap) {
  const long per_row = I / 8;
  const long n = rows * per_row;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long row = i / per_row;
    if (counts) {  // capacity layout: skip rows past the expert's rounded-up count
      const int e = (int)(row / cap), r = (int)(row % cap);
      const int lim = ((counts[e] + 127) / 128) * 128;
      if (r >= lim) continue;
    }
    const int c = (int)(i % per_row) * 8;
    const int blk = c / 128, off = c % 128;
    const long gcol = (long)blk * 256 + off;
    float d[8], g[8], u[8], dg[8], du[8];
    load8(dact + row * I + c, d);
    load8(H + row * 2 * I + gcol, g);
    load8(H + row * 2 * I + gcol + 128, u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      dg[k] = d[k] * u[k] * act_grad(g[k], kind);
      du[k] = d[k] * act_f(g[k], kind);
    }
    store8(dH + row * 2 * I + gcol, dg);
    store8(dH + row * 2 * I + gcol + 128, du);
  }
}

// ------------------------------------------------------------------------------ QK-norm + RoPE
// qkv row: [q (H*hd) | k (Hkv*hd) | ...] with row stride ld. Writes qn [T, H, hd], kn [T, Hkv, hd].
// One warp per (token, head); positions = token % S. hd even, hd/2 <= 128.
__global__ void qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, int ld, __nv_bfloat16* __restrict__ qn,
                                        __nv_bfloat16* __restrict__ kn, float* __restrict__ rstd,
                                        const float* __restrict__ cos_t, const float* __restrict__ sin_t, int T,
                                        int S, int H, int Hkv, int hd, int qk_norm, float qk_mult, float eps) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NH = H + Hkv;
  const int half = hd / 2;
  for (long item = blockIdx.x * (long)warps + (threadIdx.x >> 5); item < (long)T * NH;
       item += (long)gridDim.x * warps) {
    const int t = (int)(item / NH), h = (int)(item % NH);
    const __nv_bfloat16* src = qkv + (long)t * ld + h * hd;
    float x1[4], x2[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      x1[j] = x2[j] = 0.f;
      if (i < half) {
        x1[j] = __bfloat162float(src[i]);
        x2[j] = __bfloat162float(src[i + half]);
        ss += x1[j] * x1[j] + x2[j] * x2[j];
      }
    }
    float r = 1.f;
    if (qk_norm) {
      r = rsqrtf(warp_sum(ss) / hd + eps);
      if (lane == 0) rstd[(long)t * NH + h] = r;
    }
    const float mult = h < H ? qk_mult : 1.f;
    __nv_bfloat16* dst = h < H ? qn + ((long)t * H + h) * hd : kn + ((long)t * Hkv + (h - H)) * hd;
    const int pos = t % S;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      if (i < half) {
        // the normalised value is rounded to the activation dtype before RoPE, as in the oracle
        const float a = __bfloat162float(__float2bfloat16(x1[j] * r));
        const float b = __bfloat162float(__float2bfloat16(x2[j] * r));
        const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
        const float o1 = __bfloat162float(__float2bfloat16(a * c - b * s));
        const float o2 = __bfloat162float(__float2bfloat16(b * c + a * s));
        dst[i] = __float2bfloat16(o1 * mult);
        dst[i + half] = __float2bfloat16(o2 * mult);
      }
    }
  }
}

// Backward: dqn/dkn -> d(raw q/k) written into dqkv (row stride ld) at the q/k columns.
__global__ void qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dqn, const __nv_bfloat16* __restrict__ dkn,
                                        const __nv_bfloat16* __restrict__ qkv, int ld, const float* __restrict__ rstd,
                                        const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                        __nv_bfloat16* __restrict__ dqkv, int T, int S, int H, int Hkv, int hd,
                                        int qk_norm, float qk_mult) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int NH = H + Hkv;
  const int half = hd / 2;
  for (long item = blockIdx.x * (long)warps + (threadIdx.x >> 5); item < (long)T * NH;
       item += (long)gridDim.x * warps) {
    const int t = (int)(item / NH), h = (int)(item % NH);
    const __nv_bfloat16* g = h < H ? dqn + ((long)t * H + h) * hd : dkn + ((long)t * Hkv + (h - H)) * hd;
    const __nv_bfloat16* src = qkv + (long)t * ld + h * hd;
    const float mult = h < H ? qk_mult : 1.f;
    const float r = qk_norm ? rstd[(long)t * NH + h] : 1.f;
    const int pos = t % S;
    float dn1[4], dn2[4], n1[4], n2[4];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      dn1[j] = dn2[j] = n1[j] = n2[j] = 0.f;
      if (i < half) {
        const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
        const float g1 = __bfloat162float(g[i]) * mult, g2 = __bfloat162float(g[i + half]) * mult;
        // RoPE^T
        dn1[j] = g1 * c + g2 * s;
        dn2[j] = -g1 * s + g2 * c;
        n1[j] = __bfloat162float(src[i]) * r;
        n2[j] = __bfloat162float(src[i + half]) * r;
        dot += dn1[j] * n1[j] + dn2[j] * n2[j];
      }
    }
    if (qk_norm) dot = warp_sum(dot) / hd;
    __nv_bfloat16* dst = dqkv + (long)t * ld + h * hd;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      if (i < half) {
        float a = dn1[j], b = dn2[j];
        if (qk_norm) {
          a = r * (dn1[j] - n1[j] * dot);
          b = r * (dn2[j] - n2[j] * dot);
        }
        dst[i] = __float2bfloat16(a);
        dst[i + half] = __float2bfloat16(b);
      }
    }
  }
}

// ----------------------------------------------------------------------------- XSA + head gate
// y: [T, H, hd] attention output; v at qkv[t, voff + (h/rep)*hd]; gate logit at qkv[t, goff + h].
// out[t, h*hd + i] = gate * (y - (y.v)/(v.v + 1e-6) v), gate = 2*sigmoid(logit).
__global__ void xsa_gate_fwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ qkv,
                                    int ld, int voff, int goff, __nv_bfloat16* __restrict__ out, int T, int H,
                                    int Hkv, int hd, int xsa, int gate) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rep = H / Hkv;
  for (long item = blockIdx.x * (long)warps + (threadIdx.x >> 5); item < (long)T * H;
       item += (long)gridDim.x * warps) {
    const int t = (int)(item / H), h = (int)(item % H);
    const __nv_bfloat16* yr = y + ((long)t * H + h) * hd;
    const __nv_bfloat16* vr = qkv + (long)t * ld + voff + (h / rep) * hd;
    float yv[4], vv[4];
    float dot = 0.f, vn = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      yv[j] = vv[j] = 0.f;
      if (i < hd) {
        yv[j] = __bfloat162float(yr[i]);
        vv[j] = __bfloat162float(vr[i]);
        dot += yv[j] * vv[j];
        vn += vv[j] * vv[j];
      }
    }
    float c = 0.f;
    if (xsa) c = warp_sum(dot) / (warp_sum(vn) + 1e-6f);
    const float gmul = gate ? 2.f * sigm(__bfloat162float(qkv[(long)t * ld + goff + h])) : 1.f;
    __nv_bfloat16* o = out + (long)t * H * hd + h * hd;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      if (i < hd) o[i] = __float2bfloat16(gmul * (yv[j] - c * vv[j]));
    }
  }
}

// Backward. dout [T, H*hd]. Writes dy [T, H, hd]; dv contribution into dqkv v-columns
// (summed over the q heads of a kv group, one warp per (token, kv head)); dgate into dqkv.
__global__ void xsa_gate_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                                    const __nv_bfloat16* __restrict__ qkv, int ld, int voff, int goff,
                                    __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dqkv, int T, int H,
                                    int Hkv, int hd, int xsa, int gate) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rep = H / Hkv;
  for (long item = blockIdx.x * (long)warps + (threadIdx.x >> 5); item < (long)T * Hkv;
       item += (long)gridDim.x * warps) {
    const int t = (int)(item / Hkv), kh = (int)(item % Hkv);
    const __nv_bfloat16* vr = qkv + (long)t * ld + voff + kh * hd;
    float vv[4], dv[4];
    float vn = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      vv[j] = 0.f;
      dv[j] = 0.f;
      if (i < hd) vv[j] = __bfloat162float(vr[i]);
      vn += vv[j] * vv[j];
    }
    const float n = warp_sum(vn) + 1e-6f;
    for (int h = kh * rep; h < (kh + 1) * rep; ++h) {
      const __nv_bfloat16* yr = y + ((long)t * H + h) * hd;
      const __nv_bfloat16* dr = dout + (long)t * H * hd + h * hd;
      float yv[4], dz[4];
      float yd = 0.f, zd = 0.f;
      const float lg = gate ? __bfloat162float(qkv[(long)t * ld + goff + h]) : 0.f;
      const float s = sigm(lg);
      const float gmul = gate ? 2.f * s : 1.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = lane + 32 * j;
        yv[j] = dz[j] = 0.f;
        if (i < hd) {
          yv[j] = __bfloat162float(yr[i]);
          dz[j] = __bfloat162float(dr[i]);
        }
        yd += yv[j] * vv[j];
      }
      const float c = xsa ? warp_sum(yd) / n : 0.f;
      // dgate: d(out)/d(logit) = z * 2 s (1 - s)
      float gd = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) gd += dz[j] * (yv[j] - c * vv[j]);
      gd = warp_sum(gd);
      if (gate && lane == 0) dqkv[(long)t * ld + goff + h] = __float2bfloat16(gd * 2.f * s * (1.f - s));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dz[j] *= gmul;
        zd += dz[j] * vv[j];
      }
      const float a = xsa ? warp_sum(zd) / n : 0.f;
      __nv_bfloat16* dyr = dy + ((long)t * H + h) * hd;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = lane + 32 * j;
        if (i < hd) dyr[i] = __float2bfloat16(dz[j] - a * vv[j]);
        if (xsa) dv[j] += -a * yv[j] - c * dz[j] + 2.f * c * a * vv[j];
      }
    }
    __nv_bfloat16* dvr = dqkv + (long)t * ld + voff + kh * hd;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      if (i < hd) dvr[i] = __float2bfloat16(dv[j]);
    }
  }
}

// ------------------------------------------------------- vectorised head kernels (hd % 16 == 0)
// G lanes per (token, head): lane c < hd/16 of the group owns the 8-element chunks c and
// c + hd/16 (for RoPE these hold the element pairs (i, i + hd/2)), so every global access is one
// 16-byte vector and a per-head reduction is log2(G) xor-shuffles inside an aligned lane group.
// Lanes past hd/16 (and past the last item) only take part in the shuffles.
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}


__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

template <int G>
__global__ void __launch_bounds__(256)
    qk_norm_rope_fwd_vec(const __nv_bfloat16* __restrict__ qkv, int ld, __nv_bfloat16* __restrict__ qn,
                         __nv_bfloat16* __restrict__ kn, float* __restrict__ rstd, const float* __restrict__ cos_t,
                         const float* __restrict__ sin_t, int T, int S, int H, int Hkv, int hd, int qk_norm,
                         float qk_mult, float eps) {
  const int NH = H + Hkv, half = hd >> 1, nc = hd >> 4;
  // block (G x heads, positions); grid (position blocks, sequences, head blocks)
  const int pos = blockIdx.x * blockDim.y + threadIdx.y;
  const long tl = (long)blockIdx.y * S + pos;
  const int hh = blockIdx.z * (blockDim.x / G) + threadIdx.x / G;
  const int c = threadIdx.x & (G - 1);
  const bool valid = pos < S && tl < T && hh < NH;
  const bool act = valid && c < nc;
  const long t = valid ? tl : 0;
  const int h = valid ? hh : 0;
  float a[8], b[8];
  float ss = 0.f;
  const __nv_bfloat16* src = qkv + (long)t * ld + h * hd + 8 * c;
  if (act) {
    load8(src, a);
    load8(src + half, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += a[i] * a[i] + b[i] * b[i];
  }
  float r = 1.f;
  if (qk_norm) {
    r = rsqrtf(group_sum<G>(ss) / hd + eps);
    if (valid && c == 0) rstd[(long)t * NH + h] = r;
  }
  if (!act) return;
  float cs[8], sn[8];
  load8f(cos_t + (long)pos * half + 8 * c, cs);
  load8f(sin_t + (long)pos * half + 8 * c, sn);
  const float mult = h < H ? qk_mult : 1.f;
  float o1[8], o2[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // the normalised value is rounded to the activation dtype before RoPE, as in the oracle
    const float x1 = bf16r(a[i] * r), x2 = bf16r(b[i] * r);
    o1[i] = bf16r(x1 * cs[i] - x2 * sn[i]) * mult;
    o2[i] = bf16r(x2 * cs[i] + x1 * sn[i]) * mult;
  }
  __nv_bfloat16* dst = (h < H ? qn + ((long)t * H + h) * hd : kn + ((long)t * Hkv + (h - H)) * hd) + 8 * c;
  store8(dst, o1);
  store8(dst + half, o2);
}

template <int G>
__global__ void __launch_bounds__(256)
    qk_norm_rope_bwd_vec(const __nv_bfloat16* __restrict__ dqn, const __nv_bfloat16* __restrict__ dkn,
                         const __nv_bfloat16* __restrict__ qkv, int ld, const float* __restrict__ rstd,
                         const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                         __nv_bfloat16* __restrict__ dqkv, int T, int S, int H, int Hkv, int hd, int qk_norm,
                         float qk_mult) {
  const int NH = H + Hkv, half = hd >> 1, nc = hd >> 4;
  // block (G x heads, positions); grid (position blocks, sequences, head blocks)
  const int pos = blockIdx.x * blockDim.y + threadIdx.y;
  const long tl = (long)blockIdx.y * S + pos;
  const int hh = blockIdx.z * (blockDim.x / G) + threadIdx.x / G;
  const int c = threadIdx.x & (G - 1);
  const bool valid = pos < S && tl < T && hh < NH;
  const bool act = valid && c < nc;
  const long t = valid ? tl : 0;
  const int h = valid ? hh : 0;
  float dn1[8], dn2[8], n1[8], n2[8];
  float dot = 0.f, r = 1.f;
  if (act) {
    const __nv_bfloat16* g = (h < H ? dqn + ((long)t * H + h) * hd : dkn + ((long)t * Hkv + (h - H)) * hd) + 8 * c;
    const __nv_bfloat16* src = qkv + (long)t * ld + h * hd + 8 * c;
    float g1[8], g2[8], cs[8], sn[8];
    load8(g, g1);
    load8(g + half, g2);
    load8(src, n1);
    load8(src + half, n2);
    load8f(cos_t + (long)pos * half + 8 * c, cs);
    load8f(sin_t + (long)pos * half + 8 * c, sn);
    const float mult = h < H ? qk_mult : 1.f;
    if (qk_norm) r = rstd[(long)t * NH + h];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = g1[i] * mult, b = g2[i] * mult;
      dn1[i] = a * cs[i] + b * sn[i];  // RoPE^T
      dn2[i] = b * cs[i] - a * sn[i];
      n1[i] *= r;
      n2[i] *= r;
      dot += dn1[i] * n1[i] + dn2[i] * n2[i];
    }
  }
  if (qk_norm) dot = group_sum<G>(dot) / hd;
  if (!act) return;
  if (qk_norm) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dn1[i] = r * (dn1[i] - n1[i] * dot);
      dn2[i] = r * (dn2[i] - n2[i] * dot);
    }
  }
  __nv_bfloat16* dst = dqkv + (long)t * ld + h * hd + 8 * c;
  store8(dst, dn1);
  store8(dst + half, dn2);
}

template <int G>
__global__ void __launch_bounds__(256)
    xsa_gate_fwd_vec(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ qkv, int ld, int voff,
                     int goff, __nv_bfloat16* __restrict__ out, int T, int H, int Hkv, int hd, int xsa, int gate) {
  const int rep = H / Hkv, nc = hd >> 4;
  // block (G x heads, tokens); grid (token blocks, 1, head blocks)
  const long tl = (long)blockIdx.x * blockDim.y + threadIdx.y;
  const int hh = blockIdx.z * (blockDim.x / G) + threadIdx.x / G;
  const int c = threadIdx.x & (G - 1);
  const bool valid = tl < T && hh < H;
  const bool act = valid && c < nc;
  const long t = valid ? tl : 0;
  const int h = valid ? hh : 0;
  float y0[8], y1[8], v0[8], v1[8];
  float dot = 0.f, vn = 0.f;
  if (act) {
    const __nv_bfloat16* yr = y + ((long)t * H + h) * hd + 8 * c;
    const __nv_bfloat16* vr = qkv + (long)t * ld + voff + (h / rep) * hd + 8 * c;
    load8(yr, y0);
    load8(yr + 8 * nc, y1);
    load8(vr, v0);
    load8(vr + 8 * nc, v1);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dot += y0[i] * v0[i] + y1[i] * v1[i];
      vn += v0[i] * v0[i] + v1[i] * v1[i];
    }
  }
  float cc = 0.f;
  if (xsa) cc = group_sum<G>(dot) / (group_sum<G>(vn) + 1e-6f);
  if (!act) return;
  const float gmul = gate ? 2.f * sigm(__bfloat162float(qkv[(long)t * ld + goff + h])) : 1.f;
  float o0[8], o1[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    o0[i] = gmul * (y0[i] - cc * v0[i]);
    o1[i] = gmul * (y1[i] - cc * v1[i]);
  }
  __nv_bfloat16* o = out + ((long)t * H + h) * hd + 8 * c;
  store8(o, o0);
  store8(o + 8 * nc, o1);
}

// Operands stay packed (bf16 pairs) in registers and are unpacked at each use, which keeps the
// kernel at 3 resident blocks per SM without spills.
__device__ __forceinline__ float pk_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float pk_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float pk_at(const uint4 (&u)[2], int i) {
  const uint32_t w = reinterpret_cast<const uint32_t*>(&u[i >> 3])[(i & 7) >> 1];
  return (i & 1) ? pk_hi(w) : pk_lo(w);
}

template <int G>
__global__ void __launch_bounds__(256, 3)
    xsa_gate_bwd_vec(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ y,
                     const __nv_bfloat16* __restrict__ qkv, int ld, int voff, int goff, __nv_bfloat16* __restrict__ dy,
                     __nv_bfloat16* __restrict__ dqkv, int T, int H, int Hkv, int hd, int xsa, int gate) {
  const int rep = H / Hkv, nc = hd >> 4;
  // block (G x kv heads, tokens); grid (token blocks, 1, kv-head blocks)
  const long tl = (long)blockIdx.x * blockDim.y + threadIdx.y;
  const int hh = blockIdx.z * (blockDim.x / G) + threadIdx.x / G;
  const int c = threadIdx.x & (G - 1);
  const bool valid = tl < T && hh < Hkv;
  const bool act = valid && c < nc;
  const long t = valid ? tl : 0;
  const int kh = valid ? hh : 0;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  uint4 vp[2] = {zero, zero};
  float dv[16];
  float vn = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) dv[i] = 0.f;
  if (act) {
    const __nv_bfloat16* vr = qkv + t * ld + voff + kh * hd + 8 * c;
    vp[0] = *reinterpret_cast<const uint4*>(vr);
    vp[1] = *reinterpret_cast<const uint4*>(vr + 8 * nc);
#pragma unroll
    for (int i = 0; i < 16; ++i) vn += pk_at(vp, i) * pk_at(vp, i);
  }
  const float n = group_sum<G>(vn) + 1e-6f;
  for (int h = kh * rep; h < (kh + 1) * rep; ++h) {
    uint4 yp[2] = {zero, zero}, zp[2] = {zero, zero};
    float yd = 0.f;
    if (act) {
      const __nv_bfloat16* yr = y + (t * H + h) * hd + 8 * c;
      const __nv_bfloat16* dr = dout + (t * H + h) * hd + 8 * c;
      yp[0] = *reinterpret_cast<const uint4*>(yr);
      yp[1] = *reinterpret_cast<const uint4*>(yr + 8 * nc);
      zp[0] = *reinterpret_cast<const uint4*>(dr);
      zp[1] = *reinterpret_cast<const uint4*>(dr + 8 * nc);
#pragma unroll
      for (int i = 0; i < 16; ++i) yd += pk_at(yp, i) * pk_at(vp, i);
    }
    const float lg = (gate && valid) ? __bfloat162float(qkv[t * ld + goff + h]) : 0.f;
    const float s = sigm(lg);
    const float gmul = gate ? 2.f * s : 1.f;
    const float cc = xsa ? group_sum<G>(yd) / n : 0.f;
    // dgate: d(out)/d(logit) = z * 2 s (1 - s); zd = (gmul z) . v
    float gd = 0.f, zd = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float z = pk_at(zp, i), vv = pk_at(vp, i);
      gd += z * (pk_at(yp, i) - cc * vv);
      zd += z * vv;
    }
    zd *= gmul;
    if (gate) {
      gd = group_sum<G>(gd);
      if (valid && c == 0) dqkv[t * ld + goff + h] = __float2bfloat16(gd * 2.f * s * (1.f - s));
    }
    const float a = xsa ? group_sum<G>(zd) / n : 0.f;
    if (act) {
      float d[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float z = gmul * pk_at(zp, i), vv = pk_at(vp, i);
        d[i] = z - a * vv;
        if (xsa) dv[i] += -a * pk_at(yp, i) - cc * z + 2.f * cc * a * vv;
      }
      __nv_bfloat16* dyr = dy + (t * H + h) * hd + 8 * c;
      store8(dyr, *reinterpret_cast<const float(*)[8]>(d));
      store8(dyr + 8 * nc, *reinterpret_cast<const float(*)[8]>(d + 8));
    }
  }
  if (act) {
    __nv_bfloat16* dvr = dqkv + t * ld + voff + kh * hd + 8 * c;
    store8(dvr, *reinterpret_cast<const float(*)[8]>(dv));
    store8(dvr + 8 * nc, *reinterpret_cast<const float(*)[8]>(dv + 8));
  }
}

// ------------------------------------------------------------------------- cross-entropy grad
// One block per row of a logits chunk [rows, ldl] (bf16, V valid columns) with per-tile stats
// (max, sumexp) [rows, nt]. Computes lse, the weighted loss term, and overwrites the logits with
// dlogits = coef * ((1 + 2 z lse) softmax - onehot(label)), coef = scale * w / wsum. Columns
// in [V, ldl) are zeroed.
__global__ void ce_grad_kernel(__nv_bfloat16* __restrict__ logits, int ldl, const float2* __restrict__ stats,
                               int nt, const int64_t* __restrict__ labels, const float* __restrict__ weights,
                               const float* __restrict__ wsum, float* __restrict__ loss_out,
                               float* __restrict__ lse_out, int V, float z_weight, float scale) {
  const int row = blockIdx.x;
  __shared__ float s_red[32];
  __shared__ float s_lse;
  // combine per-tile stats
  float m = -INFINITY;
  for (int i = threadIdx.x; i < nt; i += blockDim.x) m = fmaxf(m, stats[(long)row * nt + i].x);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : -INFINITY;
    v = warp_max(v);
    if (threadIdx.x == 0) s_red[0] = v;
  }
  __syncthreads();
  m = s_red[0];
  __syncthreads();
  float se = 0.f;
  for (int i = threadIdx.x; i < nt; i += blockDim.x) {
    float2 st = stats[(long)row * nt + i];
    if (st.x > -INFINITY) se += st.y * __expf(st.x - m);
  }
  se = warp_sum(se);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = se;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? s_red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) s_lse = m + __logf(v);
  }
  __syncthreads();
  const float lse = s_lse;
  const float w = weights[row];
  const long lab = labels[row];
  __nv_bfloat16* lr = logits + (long)row * ldl;
  if (threadIdx.x == 0) {
    const float xl = (lab >= 0 && lab < V) ? __bfloat162float(lr[lab]) : 0.f;
    const float nll = lse - xl + z_weight * lse * lse;
    atomicAdd(loss_out, w * nll);
    if (lse_out) lse_out[row] = lse;
  }
  __syncthreads();
  const float coef = scale * w / fmaxf(*wsum, 1.f);
  const float pmul = coef * (1.f + 2.f * z_weight * lse);
  for (int c = threadIdx.x * 8; c < ldl; c += blockDim.x * 8) {
    float f[8];
    load8(lr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int col = c + i;
      float d = 0.f;
      if (col < V) {
        d = pmul * __expf(f[i] - lse);
        if (col == lab) d -= coef;
      }
      f[i] = d;
    }
    store8(lr + c, f);
  }
}

inline int grid_for(long work, int per_block) {
  long g = (work + per_block - 1) / per_block;
  if (g > 148 * 16) g = 148 * 16;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

// ------------------------------------------------------------------------------ launchers
void launch_rmsnorm_fwd(const void* x, const float* w, void* y, float* rstd, int T, int D, float eps,
                        cudaStream_t st) {
  count_launch();
  rmsnorm_fwd_kernel<<<grid_for(T, 8), 256, 0, st>>>((const __nv_bfloat16*)x, w, (__nv_bfloat16*)y, rstd, T, D, eps);
}

void launch_rmsnorm_bwd(const void* dy, const void* x, const float* w, const float* rstd, const void* dres, void* dx,
                        float* dw, int T, int D, cudaStream_t st) {
  const int blocks = T < 148 * 8 * 2 ? (T + 7) / 8 : 148 * 2;
  const size_t sm = 2 * (size_t)D * sizeof(float);
#define RB(V) rmsnorm_bwd_kernel<V><<<blocks, 256, sm, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, w, rstd, \
                                                            (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, dw, T, D)
  count_launch();
  if (D % 256 == 0 && D <= 1536) {
    // shared-memory partials: [D] weights + 8 warps x [D / 256 * 8][32] floats
    const size_t sm2 = (size_t)D * sizeof(float) + 8 * (size_t)(D / 256) * 8 * 32 * sizeof(float);
    const int blocks2 = T < 148 * 8 * 3 ? (T + 7) / 8 : 148 * 3;
#define RB2(V)                                                                                                  \
  do {                                                                                                          \
    static bool attr = false;                                                                                   \
    if (!attr) {                                                                                                \
      cudaFuncSetAttribute(rmsnorm_bwd_smem_kernel<V>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2); \
      attr = true;                                                                                              \
    }                                                                                                           \
    rmsnorm_bwd_smem_kernel<V><<<blocks2, 256, sm2, st>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, w, \
                                                          rstd, (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, \
                                                          dw, T, D);                                            \
  } while (0)
    switch (D / 256) {
      case 1: RB2(1); return;
      case 2: RB2(2); return;
      case 3: RB2(3); return;
      case 4: RB2(4); return;
      case 5: RB2(5); return;
      case 6: RB2(6); return;
    }
#undef RB2
  }
  if (D <= 256) RB(1);
  else if (D <= 512) RB(2);
  else if (D <= 1024) RB(4);
  else if (D <= 1536) RB(6);
  else if (D <= 2048) RB(8);
  else RB(16);
#undef RB
}

void launch_embed_fwd(const int64_t* ids, const void* table, void* out, int T, int D, int V, cudaStream_t st) {
  count_launch();
  embed_fwd_kernel<<<grid_for(T, 8), 256, 0, st>>>(ids, (const __nv_bfloat16*)table, (__nv_bfloat16*)out, T, D, V);
}

void launch_embed_bwd(const int64_t* ids, const void* dout, float* dtable, int T, int D, int V, cudaStream_t st) {
  count_launch();
  embed_bwd_kernel<<<grid_for(T, 8), 256, 0, st>>>(ids, (const __nv_bfloat16*)dout, dtable, T, D, V);
}

void launch_gate_mul_bwd(const void* dout, const void* y, const void* z, void* dy, void* dz, long n,
                         cudaStream_t st) {
  count_launch();
  gate_mul_bwd_kernel<<<grid_for(n / 8, 256), 256, 0, st>>>((const __nv_bfloat16*)dout, (const __nv_bfloat16*)y,
                                                            (const __nv_bfloat16*)z, (__nv_bfloat16*)dy,
                                                            (__nv_bfloat16*)dz, n / 8);
}

void launch_act_bwd(const void* da, const void* h, void* dh, long n, int kind, cudaStream_t st) {
  count_launch();
  act_bwd_kernel<<<grid_for(n / 8, 256), 256, 0, st>>>((const __nv_bfloat16*)da, (const __nv_bfloat16*)h,
                                                       (__nv_bfloat16*)dh, n / 8, kind);
}

void launch_swiglu_bwd(const void* dact, const void* H, void* dH, long rows, int I, int kind, const int* counts,
                       int cap, cudaStream_t st) {
  count_launch();
  swiglu_bwd_kernel<<<grid_for(rows * I / 8, 256), 256, 0, st>>>(
      (const __nv_bfloat16*)dact, (const __nv_bfloat16*)H, (__nv_bfloat16*)dH, rows, I, kind, counts, cap);
}

namespace {
// The vectorised head kernels need hd a multiple of 16 (two 16-byte chunks per lane), hd <= 256,
// 16-byte aligned rows and offsets; anything else takes the warp-per-head kernels.
inline int head_group(int hd) { return hd <= 64 ? 4 : hd <= 128 ? 8 : 16; }
inline bool vec_ok(int hd, long ld, std::initializer_list<const void*> ptrs) {
  if (hd % 16 || hd > 256 || ld % 8) return false;
  for (const void* q : ptrs)
    if (reinterpret_cast<uintptr_t>(q) & 15) return false;
  return true;
}
// Launch shape of the vectorised head kernels: heads_per_block heads of G lanes along x, rows
// (positions or tokens) along y up to 256 threads, head blocks along z.
struct HeadLaunch {
  dim3 grid, block;
};
inline HeadLaunch head_launch(int g, int heads, long rows_x, int rows_y) {
  const int hb = std::min(heads, 256 / g);
  const int tpb = std::max(1, 256 / (g * hb));
  HeadLaunch L;
  L.block = dim3(g * hb, tpb, 1);
  L.grid = dim3((unsigned)((rows_x + tpb - 1) / tpb), (unsigned)rows_y, (unsigned)((heads + hb - 1) / hb));
  return L;
}
}  // namespace

#define MXK_HEAD_VEC(KERNEL, HEADS, ROWS_X, ROWS_Y, ...)                               \
  do {                                                                                 \
    const int g_ = head_group(hd);                                                     \
    const HeadLaunch L_ = head_launch(g_, HEADS, ROWS_X, ROWS_Y);                      \
    if (g_ == 4) KERNEL<4><<<L_.grid, L_.block, 0, st>>>(__VA_ARGS__);                 \
    else if (g_ == 8) KERNEL<8><<<L_.grid, L_.block, 0, st>>>(__VA_ARGS__);            \
    else KERNEL<16><<<L_.grid, L_.block, 0, st>>>(__VA_ARGS__);                        \
  } while (0)

void launch_qk_norm_rope_fwd(const void* qkv, int ld, void* qn, void* kn, float* rstd, const float* cos_t,
                             const float* sin_t, int T, int S, int H, int Hkv, int hd, int qk_norm, float qk_mult,
                             cudaStream_t st) {
  count_launch();
  if (vec_ok(hd, ld, {qkv, qn, kn, cos_t, sin_t})) {
    MXK_HEAD_VEC(qk_norm_rope_fwd_vec, H + Hkv, S, (T + S - 1) / S, (const __nv_bfloat16*)qkv, ld,
                 (__nv_bfloat16*)qn, (__nv_bfloat16*)kn, rstd, cos_t, sin_t, T, S, H, Hkv, hd, qk_norm, qk_mult,
                 1e-6f);
    return;
  }
  qk_norm_rope_fwd_kernel<<<grid_for((long)T * (H + Hkv), 8), 256, 0, st>>>(
      (const __nv_bfloat16*)qkv, ld, (__nv_bfloat16*)qn, (__nv_bfloat16*)kn, rstd, cos_t, sin_t, T, S, H, Hkv, hd,
      qk_norm, qk_mult, 1e-6f);
}

void launch_qk_norm_rope_bwd(const void* dqn, const void* dkn, const void* qkv, int ld, const float* rstd,
                             const float* cos_t, const float* sin_t, void* dqkv, int T, int S, int H, int Hkv,
                             int hd, int qk_norm, float qk_mult, cudaStream_t st) {
  count_launch();
  if (vec_ok(hd, ld, {dqn, dkn, qkv, dqkv, cos_t, sin_t})) {
    MXK_HEAD_VEC(qk_norm_rope_bwd_vec, H + Hkv, S, (T + S - 1) / S, (const __nv_bfloat16*)dqn,
                 (const __nv_bfloat16*)dkn, (const __nv_bfloat16*)qkv, ld, rstd, cos_t, sin_t, (__nv_bfloat16*)dqkv,
                 T, S, H, Hkv, hd, qk_norm, qk_mult);
    return;
  }
  qk_norm_rope_bwd_kernel<<<grid_for((long)T * (H + Hkv), 8), 256, 0, st>>>(
      (const __nv_bfloat16*)dqn, (const __nv_bfloat16*)dkn, (const __nv_bfloat16*)qkv, ld, rstd, cos_t, sin_t,
      (__nv_bfloat16*)dqkv, T, S, H, Hkv, hd, qk_norm, qk_mult);
}

void launch_xsa_gate_fwd(const void* y, const void* qkv, int ld, int voff, int goff, void* out, int T, int H,
                         int Hkv, int hd, int xsa, int gate, cudaStream_t st) {
  count_launch();
  if (voff % 8 == 0 && vec_ok(hd, ld, {y, qkv, out})) {
    MXK_HEAD_VEC(xsa_gate_fwd_vec, H, T, 1, (const __nv_bfloat16*)y, (const __nv_bfloat16*)qkv, ld, voff, goff,
                 (__nv_bfloat16*)out, T, H, Hkv, hd, xsa, gate);
    return;
  }
  xsa_gate_fwd_kernel<<<grid_for((long)T * H, 8), 256, 0, st>>>((const __nv_bfloat16*)y, (const __nv_bfloat16*)qkv,
                                                                ld, voff, goff, (__nv_bfloat16*)out, T, H, Hkv, hd,
                                                                xsa, gate);
}

void launch_xsa_gate_bwd(const void* dout, const void* y, const void* qkv, int ld, int voff, int goff, void* dy,
                         void* dqkv, int T, int H, int Hkv, int hd, int xsa, int gate, cudaStream_t st) {
  count_launch();
  if (voff % 8 == 0 && vec_ok(hd, ld, {dout, y, qkv, dy, dqkv})) {
    MXK_HEAD_VEC(xsa_gate_bwd_vec, Hkv, T, 1, (const __nv_bfloat16*)dout, (const __nv_bfloat16*)y,
                 (const __nv_bfloat16*)qkv, ld, voff, goff, (__nv_bfloat16*)dy, (__nv_bfloat16*)dqkv, T, H, Hkv, hd,
                 xsa, gate);
    return;
  }
  xsa_gate_bwd_kernel<<<grid_for((long)T * Hkv, 8), 256, 0, st>>>(
      (const __nv_bfloat16*)dout, (const __nv_bfloat16*)y, (const __nv_bfloat16*)qkv, ld, voff, goff,
      (__nv_bfloat16*)dy, (__nv_bfloat16*)dqkv, T, H, Hkv, hd, xsa, gate);
}
#undef MXK_HEAD_VEC

void launch_ce_grad(void* logits, int ldl, const float* stats, int nt, const int64_t* labels, const float* weights,
                    const float* wsum, float* loss_out, float* lse_out, int rows, int V, float z_weight, float scale,
                    cudaStream_t st) {
  count_launch();
  ce_grad_kernel<<<rows, 256, 0, st>>>((__nv_bfloat16*)logits, ldl, (const float2*)stats, nt, labels, weights, wsum,
                                       loss_out, lse_out, V, z_weight, scale);
}

}  // namespace mxk
