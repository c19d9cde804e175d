// Allocation-free C entry point for the MoE capacity dispatch plan.
//
// This entry point has no counterpart in the reference project. It exists for callers that
// cannot call cudaMalloc (or any allocator) at the time they dispatch: code running inside a
// region where allocation is forbidden (for example a serving engine that reserves all device
// memory up front, or a host runtime that must not touch the allocator from its dispatch
// thread), and plain C callers that have no tensor allocator at all.
//
// mxk_dispatch_plan_noalloc computes the same plan as the regular dispatch-plan op: for every
// (token, k) assignment its slot in the expert's capacity buffer (-1 if dropped), the token and
// combine weight held by every slot, and the kept count per expert. The caller passes all inputs
// and outputs. The kernels' scratch (per-block per-expert counts) lives in one file-scope
// device array of MXK_NOALLOC_SCRATCH_INTS ints (256 KiB), which every GPU that loads this
// library holds until the process exits.
//
// Limits: num_experts <= MXK_NOALLOC_MAX_EXPERTS (1024) and
// ceil(n_assign / 4096) * num_experts <= MXK_NOALLOC_SCRATCH_INTS; larger problems are rejected
// with MXK_NOALLOC_TOO_LARGE before anything is launched.
//
// Set-up: the first call on a device (with that device current) looks up the device address of
// the scratch array with cudaGetSymbolAddress, raises the assign kernel's dynamic shared-memory
// limit (132 KB at 1024 experts), and caches both for that device. Make that first call before any
// stream capture begins.
//
// Concurrency: all calls share the one scratch array and it keeps the last call's contents.
// Every scratch entry a call reads is written earlier in the same call, so nothing needs
// clearing, but calls whose kernels overlap on the GPU (different streams, no ordering between
// them) race on the scratch and must not be issued.
//
// Returns 0 on success, MXK_NOALLOC_TOO_LARGE, MXK_NOALLOC_BAD_ARGS, MXK_NOALLOC_PENDING_ERROR
// (a CUDA error was already pending when the call began: nothing was launched and the error is
// left for the caller to read), or a cudaError_t value (offset by MXK_NOALLOC_CUDA_ERROR) if a
// CUDA call made here failed.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define MXK_NOALLOC_SCRATCH_INTS (64 * 1024)
#define MXK_NOALLOC_TOO_LARGE 1
#define MXK_NOALLOC_BAD_ARGS 2
#define MXK_NOALLOC_PENDING_ERROR 3
#define MXK_NOALLOC_MAX_EXPERTS 1024
#define MXK_NOALLOC_CUDA_ERROR 1000

#ifdef __cplusplus
extern "C" {
#endif

int mxk_dispatch_plan_noalloc(const int32_t* selected, const uint8_t* keep, const float* combine, int64_t num_tokens,
                              int32_t k, int32_t num_experts, int32_t capacity, int32_t* slot, int32_t* perm,
                              float* wperm, int32_t* counts, cudaStream_t stream);

int mxk_dispatch_plan_noalloc_scratch_ints(void);

#ifdef __cplusplus
}
#endif
