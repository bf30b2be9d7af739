// Launchers for the non-GEMM sm_100a kernels (norms, RoPE, SwiGLU, MoE routing and
// dispatch/combine, optimizer, loss). Each takes raw device pointers and a stream.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
