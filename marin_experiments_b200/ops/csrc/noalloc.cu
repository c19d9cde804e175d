// Allocation-free variant of the MoE capacity dispatch plan (see noalloc.h for the contract).
// No counterpart in the reference project.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "kernels.h"
#include "noalloc.h"

namespace {

constexpr int kChunk = 4096;   // assignments per block (same split as the regular plan)
constexpr int kMaxDevices = 64;
// The assign kernel's shared memory: a running offset plus 32 per-warp counts per expert.
constexpr int kAssignSmem = 33 * MXK_NOALLOC_MAX_EXPERTS * (int)sizeof(int);

// Scratch for the per-block per-expert counts. Host code must not use this name as a device
// address: it is a host-side stand-in; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) int g_plan_scratch[MXK_NOALLOC_SCRATCH_INTS];

// Per-device set-up result, published with release / read with acquire so that a host thread
// that sees the pointer also sees the kernel attribute set before it.
std::atomic<int*> g_scratch_ptr[kMaxDevices];
std::mutex g_setup_mutex;

__global__ void noalloc_count_kernel(const int* __restrict__ sel, const uint8_t* __restrict__ keep, long n, int E,
                                     int* __restrict__ blk_counts) {
  extern __shared__ int cnt[];
  for (int i = threadIdx.x; i < E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const long base = (long)blockIdx.x * kChunk;
  const long end = min(base + kChunk, n);
  for (long i = base + threadIdx.x; i < end; i += blockDim.x)
    if (!keep || keep[i]) atomicAdd(&cnt[sel[i]], 1);
  __syncthreads();
  for (int i = threadIdx.x; i < E; i += blockDim.x) blk_counts[(long)blockIdx.x * E + i] = cnt[i];
}

// First-come-first-served slots in flattened (token, k) order; blockDim = 1024.
__global__ void noalloc_assign_kernel(const int* __restrict__ sel, const uint8_t* __restrict__ keep,
                                      const float* __restrict__ comb, long n, int K, int E, int cap,
                                      const int* __restrict__ blk_counts, int nblk, int* __restrict__ slot,
                                      int* __restrict__ perm, float* __restrict__ wperm, int* __restrict__ counts) {
  extern __shared__ int sh[];
  int* base = sh;        // [E] running offset of this block per expert
  int* wcnt = sh + E;    // [32 warps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int before = 0, total = 0;
    for (int b = 0; b < nblk; ++b) {
      const int c = blk_counts[(long)b * E + e];
      if (b < (int)blockIdx.x) before += c;
      total += c;
    }
    base[e] = before;
    if (blockIdx.x == 0) counts[e] = min(total, cap);
  }
  __syncthreads();
  const long start = (long)blockIdx.x * kChunk;
  const long end = min(start + kChunk, n);
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
      int s = -1;
      if (valid) {
        int off = base[e] + rank;
        for (int w = 0; w < warp; ++w) off += wcnt[w * E + e];
        if (off < cap) {
          s = off;
          const long r = (long)e * cap + off;
          perm[r] = (int)(i / K);
          wperm[r] = comb[i];
        }
      }
      slot[i] = s;
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

// Device address of the scratch array on the current device, looked up once per device. The same
// set-up raises the assign kernel's dynamic shared-memory limit on that device (its table needs
// more than the 48 KB default above 372 experts).
int scratch_for_current_device(int** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return MXK_NOALLOC_CUDA_ERROR + (int)err;
  if (dev < 0 || dev >= kMaxDevices) return MXK_NOALLOC_BAD_ARGS;
  int* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      err = cudaFuncSetAttribute(noalloc_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAssignSmem);
      if (err != cudaSuccess) return MXK_NOALLOC_CUDA_ERROR + (int)err;
      void* addr = nullptr;
      err = cudaGetSymbolAddress(&addr, g_plan_scratch);
      if (err != cudaSuccess) return MXK_NOALLOC_CUDA_ERROR + (int)err;
      p = static_cast<int*>(addr);
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return 0;
}

}  // namespace

extern "C" int mxk_dispatch_plan_noalloc_scratch_ints(void) { return MXK_NOALLOC_SCRATCH_INTS; }

extern "C" int mxk_dispatch_plan_noalloc(const int32_t* selected, const uint8_t* keep, const float* combine,
                                         int64_t num_tokens, int32_t k, int32_t num_experts, int32_t capacity,
                                         int32_t* slot, int32_t* perm, float* wperm, int32_t* counts,
                                         cudaStream_t stream) {
  if (!selected || !combine || !slot || !perm || !wperm || !counts) return MXK_NOALLOC_BAD_ARGS;
  if (num_tokens <= 0 || k <= 0 || num_experts <= 0 || capacity <= 0) return MXK_NOALLOC_BAD_ARGS;
  if (num_experts > MXK_NOALLOC_MAX_EXPERTS) return MXK_NOALLOC_TOO_LARGE;
  // An error left pending by earlier, unrelated work is the caller's: report it without clearing
  // it and launch nothing, so it is not mistaken for (or hidden by) this call's result.
  const cudaError_t pending = cudaPeekAtLastError();
  if (pending != cudaSuccess) return MXK_NOALLOC_PENDING_ERROR;
  const long n = (long)num_tokens * k;
  const long nblk = (n + kChunk - 1) / kChunk;
  if (nblk * (long)num_experts > MXK_NOALLOC_SCRATCH_INTS) return MXK_NOALLOC_TOO_LARGE;
  int* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  mxk::count_launch(2);
  noalloc_count_kernel<<<(int)nblk, 1024, num_experts * sizeof(int), stream>>>(selected, keep, n, num_experts, scratch);
  noalloc_assign_kernel<<<(int)nblk, 1024, 33 * num_experts * sizeof(int), stream>>>(
      selected, keep, combine, n, k, num_experts, capacity, scratch, (int)nblk, slot, perm, wperm, counts);
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? 0 : MXK_NOALLOC_CUDA_ERROR + (int)err;
}
