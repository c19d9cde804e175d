// Plain C++ launch interface of the sm_100a kernels (no torch types), shared by the torch
// bindings and by the C entry points.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm_params.h"

namespace mxk {

struct GemmLaunch {
  const void* a;
  int64_t lda, a_inner, a_outer;
  int a_mn;
  const void* b;
  int64_t ldb, b_inner, b_outer;
  int b_mn;
  int bn;
  int epi;
  GemmParams p;
};

int launch_gemm(const GemmLaunch& L, cudaStream_t stream);
int num_sms();

}  // namespace mxk
