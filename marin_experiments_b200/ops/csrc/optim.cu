// Fused multi-tensor optimizers over flat fp32 master / moment / gradient buffers.
//
// Work is described by a chunk table: chunk i covers flat elements [start, start+len) of matrix
// `mat` in parameter group `group`. Per-group hyper-parameters live in device memory (so a
// captured CUDA graph picks up each step's learning rate and bias corrections):
//   hp[g] = {kind (0 adam, 1 adamh), lr, b1, b2, eps, wd, bc1 = 1-b1^t, bc2 = 1-b2^t,
//            max_grad_norm (<= 0: no clipping)}
//
// AdamH (megagpt-speedrun/adamh.py:36-73): u = mhat / (sqrt(vhat) + eps) per element, then per
// matrix  new = p - lr * u * |p| / max(|u|, 1e-10) ;  p <- new * |p| / |new| .
// |new| is evaluated from the three sums S_uu, S_pp, S_pu gathered in the moment pass:
//   |new|^2 = S_pp - 2 a S_pu + a^2 S_uu,   a = lr * sqrt(S_pp) / max(sqrt(S_uu), 1e-10)
// so the update needs one pass for the moments and one for the parameters.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace mxk {
namespace {

constexpr int kHp = 9;

// One work unit: `len` elements from flat offset `start` (parameter / gradient index k) of matrix
// `mat` in group `group`. The moments of element k live at m[k - moff]: a sharded optimizer keeps
// moments only for its ranges, packed back to back, and each chunk names its range's shift.
struct Chunk {
  long long start;
  int len;
  int mat;
  int group;
  int pad;
  long long moff;
};

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  v = (threadIdx.x < (blockDim.x >> 5)) ? sh[threadIdx.x] : 0.f;
  if (w == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  }
  return v;  // valid in thread 0
}

// Vector (float4) body over [start, start+len) with a scalar head/tail so any alignment works.
template <class F>
__device__ __forceinline__ void for_chunk(long long start, int len, F&& f4, int tid, int nthr) {
  const int head = (int)((4 - (start & 3)) & 3) < len ? (int)((4 - (start & 3)) & 3) : len;
  for (int i = tid; i < head; i += nthr) f4.scalar(start + i);
  const long long vs = start + head;
  const int nv = (len - head) / 4;
  for (int i = tid; i < nv; i += nthr) f4.vec(vs + 4ll * i);
  for (int i = head + nv * 4 + tid; i < len; i += nthr) f4.scalar(start + i);
}

struct SqNorm {
  const float* g;
  float scale;
  float acc;
  __device__ void scalar(long long k) {
    const float x = g[k] * scale;
    acc += x * x;
  }
  __device__ void vec(long long k) {
    const float4 x = *reinterpret_cast<const float4*>(g + k);
    acc += scale * scale * (x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w);
  }
};

__global__ void __launch_bounds__(256) sqnorm_kernel(const Chunk* __restrict__ chunks, const float* __restrict__ g,
                                                     float scale, double* __restrict__ out) {
  __shared__ float sh[32];
  const Chunk c = chunks[blockIdx.x];
  SqNorm f{g, scale, 0.f};
  for_chunk(c.start, c.len, f, threadIdx.x, blockDim.x);
  const float acc = block_sum(f.acc, sh);
  if (threadIdx.x == 0) atomicAdd(&out[c.group], (double)acc);
}

__device__ __forceinline__ float clip_scale(const float* hp, const double* gnorm2, int group, float gscale) {
  const float mx = hp[group * kHp + 8];
  if (mx <= 0.f || gnorm2 == nullptr) return gscale;
  const float n = (float)sqrt(gnorm2[group]);
  return n < mx ? gscale : gscale * mx / n;
}

struct Moments {
  const float* grad;
  float *m, *v, *p;
  __nv_bfloat16* pb;
  float s, lr, b1, b2, eps, wd, ibc1, ibc2;
  int kind;
  float suu, spp, spu;
  __device__ __forceinline__ float one(float gg, float& mm, float& vv, float pv, float& np) {
    gg *= s;
    mm = b1 * mm + (1.f - b1) * gg;
    vv = b2 * vv + (1.f - b2) * gg * gg;
    const float u = (mm * ibc1) / (sqrtf(vv * ibc2) + eps);
    if (kind == 0) {
      np = pv - lr * (u + wd * pv);
    } else {
      suu += u * u;
      spp += pv * pv;
      spu += pv * u;
      np = pv;
    }
    return u;
  }
  __device__ void scalar(long long k) {
    float mm = m[k], vv = v[k], np;
    one(grad[k], mm, vv, p[k], np);
    m[k] = mm;
    v[k] = vv;
    if (kind == 0) {
      p[k] = np;
      if (pb) pb[k] = __float2bfloat16(np);
    }
  }
  __device__ void vec(long long k) {
    float4 g4 = *reinterpret_cast<const float4*>(grad + k);
    float4 m4 = *reinterpret_cast<float4*>(m + k);
    float4 v4 = *reinterpret_cast<float4*>(v + k);
    float4 p4 = *reinterpret_cast<float4*>(p + k);
    float4 n4;
    one(g4.x, m4.x, v4.x, p4.x, n4.x);
    one(g4.y, m4.y, v4.y, p4.y, n4.y);
    one(g4.z, m4.z, v4.z, p4.z, n4.z);
    one(g4.w, m4.w, v4.w, p4.w, n4.w);
    *reinterpret_cast<float4*>(m + k) = m4;
    *reinterpret_cast<float4*>(v + k) = v4;
    if (kind == 0) {
      *reinterpret_cast<float4*>(p + k) = n4;
      if (pb) {
        __nv_bfloat162 a = __floats2bfloat162_rn(n4.x, n4.y), b = __floats2bfloat162_rn(n4.z, n4.w);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(pb + k) = u;
      }
    }
  }
};

// Moments for all groups; Adam groups are finished here, AdamH groups accumulate S_uu/S_pp/S_pu.
__global__ void __launch_bounds__(256) moments_kernel(const Chunk* __restrict__ chunks, const float* __restrict__ hp,
                                                      const double* __restrict__ gnorm2, float gscale,
                                                      const float* __restrict__ grad, float* __restrict__ m,
                                                      float* __restrict__ v, float* __restrict__ p,
                                                      __nv_bfloat16* __restrict__ pb, double* __restrict__ mat_sums) {
  __shared__ float sh[32];
  const Chunk c = chunks[blockIdx.x];
  const float* h = hp + c.group * kHp;
  Moments f;
  f.grad = grad; f.m = m - c.moff; f.v = v - c.moff; f.p = p; f.pb = pb;
  f.kind = (int)h[0];
  f.lr = h[1]; f.b1 = h[2]; f.b2 = h[3]; f.eps = h[4]; f.wd = h[5];
  f.ibc1 = 1.f / h[6]; f.ibc2 = 1.f / h[7];
  f.s = clip_scale(hp, gnorm2, c.group, gscale);
  f.suu = f.spp = f.spu = 0.f;
  for_chunk(c.start, c.len, f, threadIdx.x, blockDim.x);
  if (f.kind == 1) {
    const float suu = block_sum(f.suu, sh);
    const float spp = block_sum(f.spp, sh);
    const float spu = block_sum(f.spu, sh);
    if (threadIdx.x == 0) {
      atomicAdd(&mat_sums[3 * c.mat + 0], (double)suu);
      atomicAdd(&mat_sums[3 * c.mat + 1], (double)spp);
      atomicAdd(&mat_sums[3 * c.mat + 2], (double)spu);
    }
  }
}

struct Apply {
  const float *m, *v;
  float* p;
  __nv_bfloat16* pb;
  float ibc1, ibc2, eps, step, rescale;
  __device__ __forceinline__ float one(float mm, float vv, float pv) {
    const float u = (mm * ibc1) / (sqrtf(vv * ibc2) + eps);
    return (pv - step * u) * rescale;
  }
  __device__ void scalar(long long k) {
    const float np = one(m[k], v[k], p[k]);
    p[k] = np;
    if (pb) pb[k] = __float2bfloat16(np);
  }
  __device__ void vec(long long k) {
    const float4 m4 = *reinterpret_cast<const float4*>(m + k);
    const float4 v4 = *reinterpret_cast<const float4*>(v + k);
    float4 p4 = *reinterpret_cast<float4*>(p + k);
    p4.x = one(m4.x, v4.x, p4.x);
    p4.y = one(m4.y, v4.y, p4.y);
    p4.z = one(m4.z, v4.z, p4.z);
    p4.w = one(m4.w, v4.w, p4.w);
    *reinterpret_cast<float4*>(p + k) = p4;
    if (pb) {
      __nv_bfloat162 a = __floats2bfloat162_rn(p4.x, p4.y), b = __floats2bfloat162_rn(p4.z, p4.w);
      uint2 u;
      u.x = *reinterpret_cast<uint32_t*>(&a);
      u.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(pb + k) = u;
    }
  }
};

__global__ void __launch_bounds__(256) adamh_apply_kernel(const Chunk* __restrict__ chunks,
                                                          const float* __restrict__ hp, const float* __restrict__ m,
                                                          const float* __restrict__ v, float* __restrict__ p,
                                                          __nv_bfloat16* __restrict__ pb,
                                                          const double* __restrict__ mat_sums) {
  const Chunk c = chunks[blockIdx.x];
  const float* h = hp + c.group * kHp;
  if ((int)h[0] != 1) return;
  const double suu = mat_sums[3 * c.mat + 0], spp = mat_sums[3 * c.mat + 1], spu = mat_sums[3 * c.mat + 2];
  const double pn = sqrt(spp), un = fmax(sqrt(suu), 1e-10);
  const double a = (double)h[1] * pn / un;
  const double nn2 = spp - 2.0 * a * spu + a * a * suu;
  Apply f;
  f.m = m - c.moff; f.v = v - c.moff; f.p = p; f.pb = pb;
  f.ibc1 = 1.f / h[6]; f.ibc2 = 1.f / h[7]; f.eps = h[4];
  f.step = (float)a;
  f.rescale = nn2 > 0.0 ? (float)(pn / sqrt(nn2)) : 1.f;
  for_chunk(c.start, c.len, f, threadIdx.x, blockDim.x);
}

// dst = beta * dst + (1 - beta) * src  (EMA of parameters)
__global__ void ema_kernel(float* __restrict__ dst, const float* __restrict__ src, long n, float beta) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = beta * dst[i] + (1.f - beta) * src[i];
}

// fp32 -> bf16 copy (compute weights from masters)
__global__ void cast_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16(src[i]);
}

}  // namespace

void launch_opt_sqnorm(const void* chunks, int nchunks, const float* grad, float scale, double* out,
                       cudaStream_t st) {
  count_launch();
  if (nchunks > 0) sqnorm_kernel<<<nchunks, 256, 0, st>>>((const Chunk*)chunks, grad, scale, out);
}

void launch_opt_step(const void* chunks, int nchunks, const float* hp, const double* gnorm2, float gscale,
                     const float* grad, float* m, float* v, float* p, void* pb, double* mat_sums, int has_adamh,
                     int phase, cudaStream_t st) {
  // phase 0: moments + AdamH apply; 1: moments (and Adam updates, AdamH matrix sums) only; 2: AdamH
  // apply only -- a sharded optimizer all-reduces the matrix sums between phases 1 and 2.
  if (nchunks <= 0) return;
  if (phase != 2) {
    count_launch();
    moments_kernel<<<nchunks, 256, 0, st>>>((const Chunk*)chunks, hp, gnorm2, gscale, grad, m, v, p,
                                            (__nv_bfloat16*)pb, mat_sums);
  }
  if (has_adamh && phase != 1) {
    count_launch();
    adamh_apply_kernel<<<nchunks, 256, 0, st>>>((const Chunk*)chunks, hp, m, v, p, (__nv_bfloat16*)pb, mat_sums);
  }
}

void launch_ema(float* dst, const float* src, long n, float beta, cudaStream_t st) {
  count_launch();
  ema_kernel<<<148 * 8, 256, 0, st>>>(dst, src, n, beta);
}

void launch_cast_bf16(const float* src, void* dst, long n, cudaStream_t st) {
  count_launch();
  cast_bf16_kernel<<<148 * 8, 256, 0, st>>>(src, (__nv_bfloat16*)dst, n);
}

}  // namespace mxk
