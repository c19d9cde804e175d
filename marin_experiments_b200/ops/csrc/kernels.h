// Plain C++ launch interfaces of the non-GEMM sm_100a kernels (no torch types).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
