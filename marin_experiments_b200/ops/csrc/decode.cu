// Kernels of the autoregressive decode path (serving): per-head RMS norm + RoPE at explicit
// positions, KV-cache append, and split-K decode attention (one new query token per sequence
// attending to its cached keys) with a combine pass. Decode is bound by reading the KV cache, so
// these are plain CUDA-core kernels with 16-byte loads, not tensor-core kernels.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "kernels.h"

namespace mxk {
namespace {

__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// out[t, h, :] = rope(norm(x[t, h, :]) * w) at position pos[t] (rotate-half convention). One warp
// per (token, head); hd <= 256.
__global__ void head_norm_rope_kernel(const __nv_bfloat16* __restrict__ x, long x_tok, int nh, int hd,
                                      const float* __restrict__ w, float eps, const int* __restrict__ pos,
                                      const float* __restrict__ cos_t, const float* __restrict__ sin_t, int T,
                                      __nv_bfloat16* __restrict__ out) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int half = hd / 2;
  for (long r = blockIdx.x * (long)warps + (threadIdx.x >> 5); r < (long)T * nh; r += (long)gridDim.x * warps) {
    const long t = r / nh;
    const int h = (int)(r % nh);
    const __nv_bfloat16* xr = x + t * x_tok + (long)h * hd;
    float v[8];  // hd / 32 <= 8
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      v[i] = d < hd ? __bfloat162float(xr[d]) : 0.f;
      ss += v[i] * v[i];
    }
    float inv = 1.f;
    if (eps >= 0.f) inv = rsqrtf(warp_sum32(ss) / hd + eps);  // eps < 0: no normalisation
    const int p = pos[t];
    __nv_bfloat16* o = out + (r * hd);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d >= hd) continue;
      float a = v[i] * inv * (w ? w[d] : 1.f);
      // partner element of the rotate-half pair lives in another lane / register
      const int dp = d < half ? d + half : d - half;
      const int ip = dp / 32, lp = dp % 32;
      float b = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float cand = __shfl_sync(0xffffffffu, v[j], lp);
        if (j == ip) b = cand;
      }
      b = b * inv * (w ? w[dp] : 1.f);
      const int f = d < half ? d : d - half;
      const float c = cos_t[(long)p * half + f], s = sin_t[(long)p * half + f];
      o[d] = __float2bfloat16(d < half ? a * c - b * s : a * c + b * s);
    }
  }
}

// cache[seq(r), pos[r], h, :] = src[r, h, :] for keys and values; seq(r) = row_seq[r] (or r).
__global__ void kv_append_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v, long k_tok,
                                 long v_tok,
                                 __nv_bfloat16* __restrict__ ck, __nv_bfloat16* __restrict__ cv, const int* __restrict__ pos,
                                 const int* __restrict__ row_seq, int rows, int Lmax, int hkv, int hd) {
  const long per = (long)hkv * hd / 8;  // uint4 per token row
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < (long)rows * per; i += (long)gridDim.x * blockDim.x) {
    const long b = i / per, c = i % per;
    const long sq = row_seq ? row_seq[b] : b;
    const long dst = ((sq * Lmax + pos[b]) * hkv * hd) / 8 + c;
    reinterpret_cast<uint4*>(ck)[dst] = reinterpret_cast<const uint4*>(k + b * k_tok)[c];
    reinterpret_cast<uint4*>(cv)[dst] = reinterpret_cast<const uint4*>(v + b * v_tok)[c];
  }
}

constexpr int kMaxRep = 8;

// grid (nsplit, Hkv, B), 128 threads. Each warp walks keys j = split_start + warp, +4, ...; lane l
// holds elements [l * E, (l + 1) * E) of q, k, v (E = hd / 32). Partial (max, sum, acc) per query
// head of the group are merged across warps in shared memory and written per split.
template <int HD>
__global__ void __launch_bounds__(128) decode_attn_kernel(const __nv_bfloat16* __restrict__ q,
                                                          const __nv_bfloat16* __restrict__ ck,
                                                          const __nv_bfloat16* __restrict__ cv,
                                                          const int* __restrict__ lens, int H, int hkv, int Lmax,
                                                          int chunk, float scale_log2, float* __restrict__ part_ml,
                                                          float* __restrict__ part_acc) {
  constexpr int E = HD / 32;
  const int split = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int nsplit = gridDim.x;
  const int rep = H / hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = lens[b];
  const int j0 = split * chunk, j1 = min(len, j0 + chunk);
  float qv[kMaxRep][E];
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r)
#pragma unroll
    for (int e = 0; e < E; ++e)
      qv[r][e] = r < rep ? __bfloat162float(q[((long)b * H + kh * rep + r) * HD + lane * E + e]) * scale_log2 : 0.f;
  float m[kMaxRep], l[kMaxRep], acc[kMaxRep][E];
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[r][e] = 0.f;
  }
  for (int j = j0 + warp; j < j1; j += 4) {
    const long row = (((long)b * Lmax + j) * hkv + kh) * HD + lane * E;
    float kf[E], vf[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      kf[e] = __bfloat162float(ck[row + e]);
      vf[e] = __bfloat162float(cv[row + e]);
    }
#pragma unroll
    for (int r = 0; r < kMaxRep; ++r) {
      if (r >= rep) break;
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) s += qv[r][e] * kf[e];
      s = warp_sum32(s);
      const float mn = fmaxf(m[r], s);
      const float alpha = exp2f(m[r] - mn), p = exp2f(s - mn);
      l[r] = l[r] * alpha + p;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[r][e] = acc[r][e] * alpha + p * vf[e];
      m[r] = mn;
    }
  }
  // merge the four warps
  __shared__ float sm[4][kMaxRep], sl[4][kMaxRep];
  __shared__ float sacc[4][kMaxRep][HD];
  if (lane == 0)
    for (int r = 0; r < kMaxRep; ++r) {
      sm[warp][r] = m[r];
      sl[warp][r] = l[r];
    }
#pragma unroll
  for (int r = 0; r < kMaxRep; ++r)
#pragma unroll
    for (int e = 0; e < E; ++e) sacc[warp][r][lane * E + e] = acc[r][e];
  __syncthreads();
  for (int idx = threadIdx.x; idx < rep * HD; idx += blockDim.x) {
    const int r = idx / HD, d = idx % HD;
    float mx = -INFINITY;
    for (int w = 0; w < 4; ++w) mx = fmaxf(mx, sm[w][r]);
    float lt = 0.f, at = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float f = sm[w][r] == -INFINITY ? 0.f : exp2f(sm[w][r] - mx);
      lt += sl[w][r] * f;
      at += sacc[w][r][d] * f;
    }
    const long hq = (long)b * H + kh * rep + r;
    part_acc[(hq * nsplit + split) * HD + d] = at;
    if (d == 0) {
      part_ml[(hq * nsplit + split) * 2 + 0] = mx;
      part_ml[(hq * nsplit + split) * 2 + 1] = lt;
    }
  }
}

// out[b, h, :] = merge of the splits. One block of HD threads per (b, h).
__global__ void decode_combine_kernel(const float* __restrict__ part_ml, const float* __restrict__ part_acc,
                                      int nsplit, int hd, __nv_bfloat16* __restrict__ out) {
  const long hq = blockIdx.x;
  const int d = threadIdx.x;
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, part_ml[(hq * nsplit + s) * 2]);
  float lt = 0.f, at = 0.f;
  for (int s = 0; s < nsplit; ++s) {
    const float ms = part_ml[(hq * nsplit + s) * 2];
    const float f = ms == -INFINITY ? 0.f : exp2f(ms - mx);
    lt += part_ml[(hq * nsplit + s) * 2 + 1] * f;
    if (d < hd) at += part_acc[(hq * nsplit + s) * hd + d] * f;
  }
  if (d < hd) out[hq * hd + d] = __float2bfloat16(lt > 0.f ? at / lt : 0.f);
}

}  // namespace

int launch_head_norm_rope(const void* x, long x_tok, int nh, int hd, const float* w, float eps, const int* pos,
                          const float* cos_t, const float* sin_t, int T, void* out, cudaStream_t st) {
  if (hd > 256 || hd % 32) return kErrBadArgsHost;  // warp-uniform register layout
  long work = (long)T * nh;
  int grid = (int)((work + 7) / 8);
  if (grid > 148 * 16) grid = 148 * 16;
  if (grid < 1) grid = 1;
  count_launch();
  head_norm_rope_kernel<<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, x_tok, nh, hd, w, eps, pos, cos_t, sin_t, T,
                                              (__nv_bfloat16*)out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

int launch_kv_append(const void* k, const void* v, long k_tok, long v_tok, void* ck, void* cv, const int* pos,
                     const int* row_seq, int rows, int Lmax, int hkv, int hd, cudaStream_t st) {
  if ((hkv * hd) % 8 || k_tok % 8 || v_tok % 8) return kErrBadArgsHost;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15) return kErrBadArgsHost;
  count_launch();
  kv_append_kernel<<<148, 256, 0, st>>>((const __nv_bfloat16*)k, (const __nv_bfloat16*)v, k_tok, v_tok,
                                        (__nv_bfloat16*)ck, (__nv_bfloat16*)cv, pos, row_seq, rows, Lmax, hkv, hd);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

int launch_decode_attention(const void* q, const void* ck, const void* cv, const int* lens, int B, int H, int hkv,
                            int hd, int Lmax, float scale, int nsplit, float* part_ml, float* part_acc, void* out,
                            cudaStream_t st) {
  if (H % hkv || H / hkv > kMaxRep || nsplit < 1) return kErrBadArgsHost;
  const int chunk = (Lmax + nsplit - 1) / nsplit;
  dim3 grid(nsplit, hkv, B);
  const float sl2 = scale * 1.4426950408889634f;
  count_launch();
  switch (hd) {
    case 64:
      decode_attn_kernel<64><<<grid, 128, 0, st>>>((const __nv_bfloat16*)q, (const __nv_bfloat16*)ck,
                                                   (const __nv_bfloat16*)cv, lens, H, hkv, Lmax, chunk, sl2, part_ml,
                                                   part_acc);
      break;
    case 128:
      decode_attn_kernel<128><<<grid, 128, 0, st>>>((const __nv_bfloat16*)q, (const __nv_bfloat16*)ck,
                                                    (const __nv_bfloat16*)cv, lens, H, hkv, Lmax, chunk, sl2, part_ml,
                                                    part_acc);
      break;
    default:
      return kErrBadArgsHost;
  }
  count_launch();
  decode_combine_kernel<<<B * H, hd, 0, st>>>(part_ml, part_acc, nsplit, hd, (__nv_bfloat16*)out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

}  // namespace mxk
