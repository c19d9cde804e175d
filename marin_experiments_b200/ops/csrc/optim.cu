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

struct Chunk {
  long long start;
  int len;
  int mat;
  int group;
  int pad;
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

__global__ void sqnorm_kernel(const Chunk* __restrict__ chunks, const float* __restrict__ g, float scale,
                              double* __restrict__ out) {
  __shared__ float sh[32];
  const Chunk c = chunks[blockIdx.x];
  float acc = 0.f;
  const float* p = g + c.start;
  for (int i = threadIdx.x; i < c.len; i += blockDim.x) {
    const float x = p[i] * scale;
    acc += x * x;
  }
  acc = block_sum(acc, sh);
  if (threadIdx.x == 0) atomicAdd(&out[c.group], (double)acc);
}

__device__ __forceinline__ float clip_scale(const float* hp, const double* gnorm2, int group, float gscale) {
  const float mx = hp[group * kHp + 8];
  if (mx <= 0.f || gnorm2 == nullptr) return gscale;
  const float n = (float)sqrt(gnorm2[group]);
  return n < mx ? gscale : gscale * mx / n;
}

// Moments for all groups; Adam groups are finished here, AdamH groups accumulate S_uu/S_pp/S_pu.
__global__ void moments_kernel(const Chunk* __restrict__ chunks, const float* __restrict__ hp,
                               const double* __restrict__ gnorm2, float gscale, const float* __restrict__ grad,
                               float* __restrict__ m, float* __restrict__ v, float* __restrict__ p,
                               __nv_bfloat16* __restrict__ pb, double* __restrict__ mat_sums) {
  __shared__ float sh[32];
  const Chunk c = chunks[blockIdx.x];
  const float* h = hp + c.group * kHp;
  const int kind = (int)h[0];
  const float lr = h[1], b1 = h[2], b2 = h[3], eps = h[4], wd = h[5], bc1 = h[6], bc2 = h[7];
  const float s = clip_scale(hp, gnorm2, c.group, gscale);
  float suu = 0.f, spp = 0.f, spu = 0.f;
  for (int i = threadIdx.x; i < c.len; i += blockDim.x) {
    const long long k = c.start + i;
    const float gg = grad[k] * s;
    const float mm = b1 * m[k] + (1.f - b1) * gg;
    const float vv = b2 * v[k] + (1.f - b2) * gg * gg;
    m[k] = mm;
    v[k] = vv;
    const float u = (mm / bc1) / (sqrtf(vv / bc2) + eps);
    const float pv = p[k];
    if (kind == 0) {
      const float np = pv - lr * (u + wd * pv);
      p[k] = np;
      if (pb) pb[k] = __float2bfloat16(np);
    } else {
      suu += u * u;
      spp += pv * pv;
      spu += pv * u;
    }
  }
  if (kind == 1) {
    suu = block_sum(suu, sh);
    spp = block_sum(spp, sh);
    spu = block_sum(spu, sh);
    if (threadIdx.x == 0) {
      atomicAdd(&mat_sums[3 * c.mat + 0], (double)suu);
      atomicAdd(&mat_sums[3 * c.mat + 1], (double)spp);
      atomicAdd(&mat_sums[3 * c.mat + 2], (double)spu);
    }
  }
}

__global__ void adamh_apply_kernel(const Chunk* __restrict__ chunks, const float* __restrict__ hp,
                                   const float* __restrict__ m, const float* __restrict__ v, float* __restrict__ p,
                                   __nv_bfloat16* __restrict__ pb, const double* __restrict__ mat_sums) {
  const Chunk c = chunks[blockIdx.x];
  const float* h = hp + c.group * kHp;
  if ((int)h[0] != 1) return;
  const float lr = h[1], eps = h[4], bc1 = h[6], bc2 = h[7];
  const double suu = mat_sums[3 * c.mat + 0], spp = mat_sums[3 * c.mat + 1], spu = mat_sums[3 * c.mat + 2];
  const double pn = sqrt(spp), un = fmax(sqrt(suu), 1e-10);
  const double a = (double)lr * pn / un;
  const double nn2 = spp - 2.0 * a * spu + a * a * suu;
  const float step = (float)a;
  const float rescale = nn2 > 0.0 ? (float)(pn / sqrt(nn2)) : 1.f;
  for (int i = threadIdx.x; i < c.len; i += blockDim.x) {
    const long long k = c.start + i;
    const float u = (m[k] / bc1) / (sqrtf(v[k] / bc2) + eps);
    const float np = (p[k] - step * u) * rescale;
    p[k] = np;
    if (pb) pb[k] = __float2bfloat16(np);
  }
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
                     cudaStream_t st) {
  if (nchunks <= 0) return;
  count_launch();
  moments_kernel<<<nchunks, 256, 0, st>>>((const Chunk*)chunks, hp, gnorm2, gscale, grad, m, v, p,
                                          (__nv_bfloat16*)pb, mat_sums);
  if (has_adamh) {
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
