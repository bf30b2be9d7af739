// Host-facing description of the tcgen05 grouped GEMM (see grouped_gemm.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "opt_hyper.h"

namespace sepx {

enum : int {
  kEpiBf16 = 0,       // D -> bf16 [rows, ldo]
  kEpiSwigluFwd = 1,  // D = [gate | up] -> h = silu(g) * u (out), pre-activation gu (aux)
  kEpiSwigluBwd = 2,  // D = dh (unweighted) -> dgu (out), w*h (aux2), dw += <dh, h> (row_dw)
  kEpiF32 = 3,        // D -> fp32 [G, M, ldo] (weight gradients)
  kEpiAdamW = 4,      // D = weight gradient -> AdamW update of W[G, M, N] in place (fp32 state)
  kEpiAdamW8 = 5,     // same, 8-bit state, with the state streamed through a TMA ring
};

struct GemmParams {
  const int* group_off = nullptr;  // [G+1] device offsets of the ragged dimension
  int G = 1;
  int M = 0;                 // ragged-K: output rows per group
  int N = 0;                 // output columns
  int K = 0;                 // ragged-M: reduction length
  int b_rows_per_group = 0;  // rows of B's 2-D view that belong to one group
  int n_tiles = 0;           // set by the launcher
  int I = 0;                 // SwiGLU intermediate size (gate and up halves)
  void* out = nullptr;
  int64_t ldo = 0;
  void* aux = nullptr;
  int64_t ld_aux = 0;
  void* aux2 = nullptr;
  int64_t ld_aux2 = 0;
  const float* row_w = nullptr;
  float* row_dw = nullptr;
  int* status = nullptr;
  unsigned long long timeout_ns = 2000000000ull;
  OptHyper opt;  // kEpiAdamW
};

struct GemmCall {
  GemmParams p;
  int epi = kEpiBf16;
  const void* A = nullptr;
  int64_t a_rows = 0;
  int64_t lda = 0;
  const void* B = nullptr;
  int64_t b_rows = 0;
  int64_t ldb = 0;
  bool b_kmajor = true;
};

void grouped_gemm_ragged_m(const GemmCall& c, cudaStream_t stream);
void grouped_gemm_ragged_k(const GemmCall& c, cudaStream_t stream);
// weight gradient with the AdamW update fused into the epilogue (c.p.opt describes W)
void grouped_gemm_wgrad_adamw(const GemmCall& c, cudaStream_t stream);
// Whether 256-column tiles run on CTA pairs (tcgen05.mma.cta_group::2); returns the
// previous setting.
bool gemm_set_pairs(bool on);

}  // namespace sepx
