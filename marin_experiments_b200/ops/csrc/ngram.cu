// Hashed n-gram input embedding (Over-Encoding style): for every token position and every
// (order n, hash function h) the n-gram ending at the position is hashed into a shared per-order
// table; the looked-up rows are averaged. Forward gathers, backward scatter-adds (fp32 atomics into
// the table gradient). The hash is an FNV-1a-style 64-bit mix of the n token ids, salted by (n, h);
// positions before the start of a sequence contribute the id -1.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace mxk {

__host__ __device__ __forceinline__ uint64_t ngram_hash(const int64_t* ids, int t, int n, int h) {
  uint64_t x = 0xcbf29ce484222325ull ^ ((uint64_t)(n * 131 + h + 1) * 0x9E3779B97F4A7C15ull);
  for (int i = 0; i < n; ++i) {
    const int64_t v = t - i >= 0 ? ids[t - i] : -1;
    x ^= (uint64_t)v;
    x *= 0x100000001B3ull;
    x ^= x >> 29;
  }
  return x;
}

namespace {

// out[b*S + t, :] = mean over (order, hash) of table[order][bucket(order, hash, t)] ; one warp per row.
__global__ void ngram_fwd_kernel(const int64_t* __restrict__ ids, int B, int S, const int* __restrict__ orders,
                                 int n_orders, int n_hash, long buckets, const __nv_bfloat16* __restrict__ table,
                                 int rank, __nv_bfloat16* __restrict__ out) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const float inv = 1.f / (float)(n_orders * n_hash);
  for (long r = blockIdx.x * (long)warps + (threadIdx.x >> 5); r < (long)B * S; r += (long)gridDim.x * warps) {
    const long b = r / S;
    const int t = (int)(r % S);
    const int64_t* seq = ids + b * S;
    for (int c = lane; c < rank; c += 32) {
      float acc = 0.f;
      for (int o = 0; o < n_orders; ++o)
        for (int h = 0; h < n_hash; ++h) {
          const long bk = (long)(ngram_hash(seq, t, orders[o], h) % (uint64_t)buckets);
          acc += __bfloat162float(table[((long)o * buckets + bk) * rank + c]);
        }
      out[r * rank + c] = __float2bfloat16(acc * inv);
    }
  }
}

__global__ void ngram_bwd_kernel(const int64_t* __restrict__ ids, int B, int S, const int* __restrict__ orders,
                                 int n_orders, int n_hash, long buckets, const __nv_bfloat16* __restrict__ dout,
                                 int rank, float* __restrict__ dtable) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const float inv = 1.f / (float)(n_orders * n_hash);
  for (long r = blockIdx.x * (long)warps + (threadIdx.x >> 5); r < (long)B * S; r += (long)gridDim.x * warps) {
    const long b = r / S;
    const int t = (int)(r % S);
    const int64_t* seq = ids + b * S;
    for (int o = 0; o < n_orders; ++o)
      for (int h = 0; h < n_hash; ++h) {
        const long bk = (long)(ngram_hash(seq, t, orders[o], h) % (uint64_t)buckets);
        float* row = dtable + ((long)o * buckets + bk) * rank;
        for (int c = lane; c < rank; c += 32) atomicAdd(row + c, __bfloat162float(dout[r * rank + c]) * inv);
      }
  }
}

inline int grid_rows(long rows) {
  long g = (rows + 7) / 8;
  if (g > 148 * 16) g = 148 * 16;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

int launch_ngram_fwd(const int64_t* ids, int B, int S, const int* orders, int n_orders, int n_hash, long buckets,
                     const void* table, int rank, void* out, cudaStream_t st) {
  count_launch();
  ngram_fwd_kernel<<<grid_rows((long)B * S), 256, 0, st>>>(ids, B, S, orders, n_orders, n_hash, buckets,
                                                           (const __nv_bfloat16*)table, rank, (__nv_bfloat16*)out);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

int launch_ngram_bwd(const int64_t* ids, int B, int S, const int* orders, int n_orders, int n_hash, long buckets,
                     const void* dout, int rank, float* dtable, cudaStream_t st) {
  count_launch();
  ngram_bwd_kernel<<<grid_rows((long)B * S), 256, 0, st>>>(ids, B, S, orders, n_orders, n_hash, buckets,
                                                           (const __nv_bfloat16*)dout, rank, dtable);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

}  // namespace mxk
