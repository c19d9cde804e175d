// Plain C++ launch interface of the sm_100a kernels (no torch types), shared by the torch
// bindings and by the C entry points.
#pragma once
#include <cuda.h>
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
  // output tensor maps: C [c_rows, c_cols] (row stride p.ldc), C2 [c2_rows, c2_cols] (p.ldc2)
  int64_t c_rows, c_cols, c2_rows, c2_cols;
  int c2_f32;
  GemmParams p;
};

int launch_gemm(const GemmLaunch& L, cudaStream_t stream);
int num_sms();
// Epilogue-store tensor map (64-byte boxes of 32 rows, 64-byte swizzle) over [rows, cols], row stride ld.
bool make_tmap_epi(CUtensorMap* m, const void* ptr, bool f32, int64_t cols, int64_t rows, int64_t ld);
// At most `sms` CTAs for persistent GEMMs launched on stream `s` (<= 0: no limit).
void set_stream_sm_budget(cudaStream_t s, int sms);

}  // namespace mxk
