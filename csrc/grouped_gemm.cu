// Grouped (per-expert) GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One persistent, warp-specialised kernel template covers every expert GEMM of the
// MoE layer, forward and backward:
//
//   mode        A (rows x K)            B                         D
//   fwd         X_perm  K-major         W[e] [N,K] K-major        [rows, N]   ragged M
//   dgrad       dY_perm K-major         W[e] [K,N] MN-major       [rows, N]   ragged M
//   wgrad       dY^T    MN-major        Z^T      MN-major         [G, M, N]   ragged K
//
// Ragged dimension = rows of each expert group, taken from device-side offsets
// (`group_off`, 64-row aligned, zero-filled padding) so that no host sync is needed.
//
// Warp roles (192 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer (one elected lane): A/B tiles, 128B swizzle, STAGES deep.
//   warp 1      TMEM allocator + MMA issuer (one lane): tcgen05.mma M=128, N=BN, K=16.
//   warps 2..5  epilogue: tcgen05.ld of the fp32 accumulator, fused SwiGLU fwd/bwd,
//               bf16/fp32 stores. Two TMEM accumulators so the epilogue of tile i
//               overlaps the MMAs of tile i+1.
//
// All pipeline waits are bounded (see sm100.cuh); a timeout aborts the CTA cleanly and
// leaves an error code in `status`.
//
// Reference parity: the reference runs experts through a user callback
// (`expert(rows, expert_ids)`, src/rbd.py:485) and, in its model path, DeepSpeed's
// grouped_mm (configs/qwen_ep8.json:7). This kernel is that expert computation.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "adamw_math.cuh"
#include "sm100.cuh"
#include "grouped_gemm.h"
#include "kernels.h"

namespace sepx {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;                 // two warps per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer + MMA + epilogue
// Epilogue warps of the fused 8-bit optimizer. Twelve (three per TMEM lane quarter, 128
// registers, two-job rings) measured slower than eight (168 registers, three-job rings):
// 1.10 vs 0.96 ms for the 128 x 1536 x 2048 gate|up update at 256 rows per expert.
constexpr int kOptEpiWarps = 8;
__host__ __device__ constexpr int epi_warps(int epi) { return epi == kEpiAdamW8 ? kOptEpiWarps : kEpiWarps; }
__host__ __device__ constexpr int threads_for(int epi) { return 64 + 32 * epi_warps(epi); }
// fused 8-bit optimizer epilogue: one job = 32 rows x 32 columns of W (bf16, 64B-swizzled)
// + m codes + v codes (uint8, 32B-swizzled), streamed by TMA a few jobs deep per warp
constexpr int kOptJob = 4096;  // w 2048 B @0, m 1024 B @2048, v 1024 B @3072
// ring depth per epilogue warp: what fits next to the mainloop stages. With two stages
// the three-job ring measured fastest for the 128 x 1536 x 2048 gate|up update at 256
// rows per expert: 0.956 ms, against 1.088 (two jobs) and 1.201 (four jobs, which leaves
// the SM 28 KB of L1 instead of 60 KB). Three stages (long reductions, or group tables
// too large for two) leave room for two jobs.
__host__ __device__ constexpr int opt_ring(int bn, int stages) { return bn == 256 ? (stages >= 3 ? 2 : 3) : 5; }
constexpr size_t kMaxSmem = 232448;  // dynamic shared memory per block (opt-in)

struct OptMaps {  // kEpiAdamW8 state tensor maps over [G * M, N]
  CUtensorMap w, m, v;
};

// Output tensor maps of the TMA-store epilogues (bf16, box 32 columns x 32 rows, 64-byte
// swizzle): out, aux, aux2 as in GemmParams.
struct EpiMaps {
  CUtensorMap out, aux, aux2;
};
// Per epilogue warp: three 32 x 32 bf16 staging blocks (2 KB each) for TMA stores.
constexpr int kEpiStoreBytes = 3 * 2048;

template <int BN, int STAGES, int EPI>
struct GemmSmem {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // epilogues that transpose 32x32 accumulator blocks through shared memory
  static constexpr int EPI_STAGE_OFF = STAGES * STAGE_BYTES;
  // kEpiAdamW8: per epilogue warp, a ring of kOptRing jobs (32x32 weights + m + v codes)
  // followed by one mbarrier per ring slot
  static constexpr int EPI_STAGE_BYTES =
      (EPI == kEpiAdamW || EPI == kEpiF32)
          ? kEpiWarps * 32 * 33 * 4
          : (EPI == kEpiAdamW8 ? epi_warps(EPI) * opt_ring(BN, STAGES) * (kOptJob + 8) : 0);
  static constexpr int BAR_OFF = EPI_STAGE_OFF + EPI_STAGE_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1;  // full, empty, tfull[2], tempty[2], drain
  static constexpr int MISC_OFF = BAR_OFF + NUM_BARS * 8;
  static constexpr int PREFIX_OFF = MISC_OFF + 16;
  static size_t bytes(int G) { return 1024 + PREFIX_OFF + 4 * (size_t)(G + 1); }
};

struct TileInfo {
  int g;        // group
  int row0;     // ragged-M: first row of the tile; ragged-K: m0
  int row_end;  // ragged-M: end of the group's rows
  int n0;       // first output column (in units of accumulator columns)
  int k0;       // ragged-K: first reduction row of the group
  int num_kb;   // k-blocks
};

// TM: output rows per tile (128 for one CTA, 256 for a CTA pair).
template <bool RAGGED_K, int BN, int TM = kBM>
__device__ __forceinline__ TileInfo decode_tile(int t, const GemmParams& p, const int* s_prefix) {
  TileInfo ti;
  if (!RAGGED_K) {
    // binary search: largest g with prefix[g] <= t
    int lo = 0, hi = p.G;  // prefix[G] = total > t
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (s_prefix[mid] <= t) lo = mid; else hi = mid;
    }
    int g = lo;
    int local = t - s_prefix[g];
    int m_tile = local / p.n_tiles;
    int n_tile = local - m_tile * p.n_tiles;
    int off0 = __ldg(p.group_off + g);
    ti.g = g;
    ti.row0 = off0 + m_tile * TM;
    ti.row_end = __ldg(p.group_off + g + 1);
    ti.n0 = n_tile * BN;
    ti.k0 = 0;
    ti.num_kb = p.K / kBK;
  } else {
    int m_tiles = p.M / TM;
    int per_group = m_tiles * p.n_tiles;
    int gi = t / per_group;
    int local = t - gi * per_group;
    const int g = s_prefix[gi];  // ragged K: groups in order of decreasing rows (group_order)
    int m_tile = local / p.n_tiles;
    int n_tile = local - m_tile * p.n_tiles;
    int off0 = __ldg(p.group_off + g);
    int off1 = __ldg(p.group_off + g + 1);
    ti.g = g;
    ti.row0 = m_tile * TM;
    ti.row_end = p.M;
    ti.n0 = n_tile * BN;
    ti.k0 = off0;
    ti.num_kb = (off1 - off0) / kBK;
  }
  return ti;
}

// Ragged K (weight gradients): a tile's MMA time grows with its group's rows, so the
// persistent CTAs take tiles in order of decreasing group rows (ties by group index):
// the long tiles are dealt out first, one per CTA, and the short ones even out the end
// (longest-processing-time order for the static round-robin assignment). order[r] = group
// of rank r. Every thread of the CTA calls it; scratch holds G ints and is free until the
// first TMA load; the caller synchronises before order is read.
__device__ __forceinline__ void group_order(const GemmParams& p, int* order, int* scratch) {
  for (int i = threadIdx.x; i < p.G; i += blockDim.x) scratch[i] = __ldg(p.group_off + i + 1) - __ldg(p.group_off + i);
  __syncthreads();
  for (int i = threadIdx.x; i < p.G; i += blockDim.x) {
    const int si = scratch[i];
    int rank = 0;
    for (int j = 0; j < p.G; ++j) {
      const int sj = scratch[j];
      rank += (sj > si) || (sj == si && j < i);
    }
    order[rank] = i;
  }
}

// SiLU and the logistic function with the fast division intrinsic (for exp(-x) beyond
// 2^126 it returns 0, which is the limit of both); epilogues round the results to bf16
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }

// One accumulator tile (128 rows x BN fp32 columns in TMEM at t_acc) through the
// epilogue EPI by the 8 epilogue warps (warps 2..9): rows ti.row0 .. ti.row0 + 127 of the
// output, valid below ti.row_end. Shared by the single-CTA and the CTA-pair kernels
// (each CTA of a pair owns 128 rows of the 256-row tile). epi_smem: the CTA's epilogue
// staging area (32 x 33 fp32 per warp for the transposing epilogues).
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile(const GemmParams& p, const TileInfo& ti, uint32_t t_acc, int warp,
                                              int lane, uint8_t* epi_smem) {
  const int q = warp & 3;            // TMEM lane quarter this warp may access
  const int half = (warp - 2) >> 2;  // which of the two warps on this quarter
  constexpr int kCStep = kEpiWarps / 4;
  const int r = ti.row0 + q * 32 + lane;
  const bool valid = r < ti.row_end;
  const uint32_t t_row = t_acc + ((uint32_t)(q * 32) << 16);
  const bool zero = ti.num_kb == 0;

  if (EPI == kEpiBf16) {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);
#pragma unroll 1
    for (int c = half; c < BN / 32; c += kCStep) {
      float v[32];
      tmem_ld32(t_row + c * 32, v);
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(out + (size_t)r * p.ldo + ti.n0 + c * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 w;
          w.x = pack_bf16x2(zero ? 0.f : v[8 * j + 0], zero ? 0.f : v[8 * j + 1]);
          w.y = pack_bf16x2(zero ? 0.f : v[8 * j + 2], zero ? 0.f : v[8 * j + 3]);
          w.z = pack_bf16x2(zero ? 0.f : v[8 * j + 4], zero ? 0.f : v[8 * j + 5]);
          w.w = pack_bf16x2(zero ? 0.f : v[8 * j + 6], zero ? 0.f : v[8 * j + 7]);
          dst[j] = w;
        }
      }
    }
  } else if (EPI == kEpiF32) {
    // Transpose each 32x32 fp32 block through shared memory so every store is one
    // row's 32 contiguous floats (128 bytes per warp instruction).
    float* out = reinterpret_cast<float*>(p.out);
    float* tile = reinterpret_cast<float*>(epi_smem) + (warp - 2) * 32 * 33;
    const size_t row_base = ((size_t)ti.g * p.M + ti.row0 + q * 32) * (size_t)p.ldo;
#pragma unroll 1
    for (int c = half; c < BN / 32; c += kCStep) {
      float v[32];
      tmem_ld32(t_row + c * 32, v);
#pragma unroll
      for (int e = 0; e < 32; ++e) tile[lane * 33 + e] = zero ? 0.f : v[e];
      __syncwarp();
      float* dst = out + row_base + ti.n0 + c * 32 + lane;
#pragma unroll 8
      for (int i = 0; i < 32; ++i) dst[(size_t)i * p.ldo] = tile[i * 33 + lane];
      __syncwarp();
    }
  } else if (EPI == kEpiSwigluFwd) {
    // accumulator columns [0,128) = gate, [128,256) = up, for I-range [i0, i0+128)
    const int i0 = ti.n0 / 2;
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.out);
    __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(p.aux);
#pragma unroll 1
    for (int c = half; c < 4; c += kCStep) {
      float g[32], u[32];
      tmem_ld32(t_row + c * 32, g);
      tmem_ld32(t_row + 128 + c * 32, u);
      if (valid) {
        uint4* dh = reinterpret_cast<uint4*>(h + (size_t)r * p.ldo + i0 + c * 32);
        uint4* dg = reinterpret_cast<uint4*>(gu + (size_t)r * p.ld_aux + i0 + c * 32);
        uint4* du = reinterpret_cast<uint4*>(gu + (size_t)r * p.ld_aux + p.I + i0 + c * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float gg[8], uu[8], hh[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            // round g/u to bf16 first so h is consistent with the stored pre-activation
            gg[e] = __bfloat162float(__float2bfloat16(g[8 * j + e]));
            uu[e] = __bfloat162float(__float2bfloat16(u[8 * j + e]));
            hh[e] = silu_f(gg[e]) * uu[e];
          }
          dg[j] = make_uint4(pack_bf16x2(gg[0], gg[1]), pack_bf16x2(gg[2], gg[3]),
                             pack_bf16x2(gg[4], gg[5]), pack_bf16x2(gg[6], gg[7]));
          du[j] = make_uint4(pack_bf16x2(uu[0], uu[1]), pack_bf16x2(uu[2], uu[3]),
                             pack_bf16x2(uu[4], uu[5]), pack_bf16x2(uu[6], uu[7]));
          dh[j] = make_uint4(pack_bf16x2(hh[0], hh[1]), pack_bf16x2(hh[2], hh[3]),
                             pack_bf16x2(hh[4], hh[5]), pack_bf16x2(hh[6], hh[7]));
        }
      }
    }
  } else if (EPI == kEpiSwigluBwd) {
    // accumulator = dh_unweighted[r, i0 : i0+BN]; gate weight w = row_w[r]
    const int i0 = ti.n0;
    const __nv_bfloat16* gu = reinterpret_cast<const __nv_bfloat16*>(p.aux);
    __nv_bfloat16* dgu = reinterpret_cast<__nv_bfloat16*>(p.out);
    __nv_bfloat16* hw = reinterpret_cast<__nv_bfloat16*>(p.aux2);
    const float w = valid ? __ldg(p.row_w + r) : 0.f;
    float dw_part = 0.f;
#pragma unroll 1
    for (int c = half; c < BN / 32; c += kCStep) {
      float d[32];
      tmem_ld32(t_row + c * 32, d);
      if (valid) {
        const uint4* sg = reinterpret_cast<const uint4*>(gu + (size_t)r * p.ld_aux + i0 + c * 32);
        const uint4* su =
            reinterpret_cast<const uint4*>(gu + (size_t)r * p.ld_aux + p.I + i0 + c * 32);
        uint4* og = reinterpret_cast<uint4*>(dgu + (size_t)r * p.ldo + i0 + c * 32);
        uint4* ou = reinterpret_cast<uint4*>(dgu + (size_t)r * p.ldo + p.I + i0 + c * 32);
        uint4* oh = reinterpret_cast<uint4*>(hw + (size_t)r * p.ld_aux2 + i0 + c * 32);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 gv = sg[j], uv = su[j];
          uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
          uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
          uint32_t rg[4], ru[4], rh[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 g2 = unpack_bf16x2(gw[e]);
            float2 u2 = unpack_bf16x2(uw[e]);
            float dd0 = d[8 * j + 2 * e], dd1 = d[8 * j + 2 * e + 1];
            float s0 = sigmoid_f(g2.x), s1 = sigmoid_f(g2.y);
            float si0 = g2.x * s0, si1 = g2.y * s1;
            float h0 = si0 * u2.x, h1 = si1 * u2.y;
            dw_part += dd0 * h0 + dd1 * h1;
            float wd0 = w * dd0, wd1 = w * dd1;
            float dg0 = wd0 * u2.x * s0 * (1.f + g2.x * (1.f - s0));
            float dg1 = wd1 * u2.y * s1 * (1.f + g2.y * (1.f - s1));
            rg[e] = pack_bf16x2(dg0, dg1);
            ru[e] = pack_bf16x2(wd0 * si0, wd1 * si1);
            rh[e] = pack_bf16x2(w * h0, w * h1);
          }
          og[j] = make_uint4(rg[0], rg[1], rg[2], rg[3]);
          ou[j] = make_uint4(ru[0], ru[1], ru[2], ru[3]);
          oh[j] = make_uint4(rh[0], rh[1], rh[2], rh[3]);
        }
      }
    }
    if (valid && p.row_dw) atomicAdd(p.row_dw + r, dw_part);
  } else if (EPI == kEpiAdamW) {
    // fp32 state. The weight gradient never leaves the SM. Each 32x32 fp32 block (32
    // rows of this warp's lane quarter x 32 columns) is transposed through shared
    // memory so that the warp then updates one row's 32 contiguous weights per step,
    // one per lane (coalesced).
    float* tile = reinterpret_cast<float*>(epi_smem) + (warp - 2) * 32 * 33;
    const size_t row_base = ((size_t)ti.g * p.M + ti.row0 + q * 32) * (size_t)p.N;
#pragma unroll 1
    for (int c = half; c < BN / 32; c += kCStep) {
      float v[32];
      tmem_ld32(t_row + c * 32, v);
#pragma unroll
      for (int e = 0; e < 32; ++e) tile[lane * 33 + e] = zero ? 0.f : v[e];
      __syncwarp();
      const size_t col = (size_t)ti.n0 + c * 32 + lane;
#pragma unroll 1
      for (int i = 0; i < 32; i += 4) {
        float g4[4];
        size_t idx[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          g4[u] = tile[(i + u) * 33 + lane];
          idx[u] = row_base + (size_t)(i + u) * p.N + col;
        }
        adamw_fp32_lanes<4>(g4, idx, p.opt);
      }
      __syncwarp();
    }
  }
}

template <int BN, int STAGES, bool A_MN, bool B_MN, bool RAGGED_K, int EPI>
__global__ void __launch_bounds__(threads_for(EPI), 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const GemmParams p,
                        const __grid_constant__ OptMaps om) {
  using L = GemmSmem<BN, STAGES, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  int* s_prefix = reinterpret_cast<int*>(smem + L::PREFIX_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- tile prefix (ragged M): tiles of group g = ceil(rows_g / BM) * n_tiles ----
  int total_tiles;
  if (RAGGED_K) group_order(p, s_prefix, reinterpret_cast<int*>(smem));
  if (!RAGGED_K) {
    if (threadIdx.x == 0) {
      int acc = 0;
      for (int g = 0; g < p.G; ++g) {
        s_prefix[g] = acc;
        int rows = __ldg(p.group_off + g + 1) - __ldg(p.group_off + g);
        acc += ((rows + kBM - 1) / kBM) * p.n_tiles;
      }
      s_prefix[p.G] = acc;
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], epi_warps(EPI));
    }
    mbar_init(drain_bar, 1);
    if (EPI == kEpiAdamW8) {
      uint64_t* obars =
          reinterpret_cast<uint64_t*>(smem + L::EPI_STAGE_OFF + epi_warps(EPI) * opt_ring(BN, STAGES) * kOptJob);
      for (int i = 0; i < epi_warps(EPI) * opt_ring(BN, STAGES); ++i) mbar_init(&obars[i], 1);
    }
    *s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI == kEpiAdamW8) {
      tma_prefetch_desc(&om.w);
      tma_prefetch_desc(&om.m);
      tma_prefetch_desc(&om.v);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (!RAGGED_K) {
    total_tiles = s_prefix[p.G];
  } else {
    total_tiles = p.G * (p.M / kBM) * p.n_tiles;
  }

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        TileInfo ti = decode_tile<RAGGED_K, BN>(t, p, s_prefix);
        for (int kb = 0; kb < ti.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, s_abort, p.status, p.timeout_ns)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * L::STAGE_BYTES;
          uint8_t* sB = sA + L::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], L::STAGE_BYTES);
          if (!A_MN) {
            tma_load_2d(sA, &tmA, &full_bar[stage], kb * kBK, ti.row0);
          } else {
            // A[m, k] stored as [k rows, m contiguous]: two 64-wide MN chunks
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j)
              tma_load_2d(sA + j * 8192, &tmA, &full_bar[stage], ti.row0 + j * 64,
                          ti.k0 + kb * kBK);
          }
          if (!B_MN) {
            if (EPI == kEpiSwigluFwd) {
              // gate rows [i0, i0+128) and up rows [I + i0, ...) of expert g
              const int i0 = ti.n0 / 2;
              const int base = ti.g * p.b_rows_per_group;
              tma_load_2d(sB, &tmB, &full_bar[stage], kb * kBK, base + i0);
              tma_load_2d(sB + 128 * 128, &tmB, &full_bar[stage], kb * kBK, base + p.I + i0);
            } else {
              const int base = ti.g * p.b_rows_per_group + ti.n0;
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                tma_load_2d(sB + j * 128 * 128, &tmB, &full_bar[stage], kb * kBK, base + j * 128);
            }
          } else {
            const int krow = RAGGED_K ? (ti.k0 + kb * kBK) : (ti.g * p.b_rows_per_group + kb * kBK);
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sB + j * 8192, &tmB, &full_bar[stage], ti.n0 + j * 64, krow);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer --------------------------------
    constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      TileInfo ti = decode_tile<RAGGED_K, BN>(t, p, s_prefix);
      if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, s_abort, p.status, p.timeout_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < ti.num_kb; ++kb) {
        if (!mbar_wait_bounded(&full_bar[stage], phase, s_abort, p.status, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t b_addr = a_addr + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            uint64_t adesc, bdesc;
            if (!A_MN) adesc = make_smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            else adesc = make_smem_desc_sw128(a_addr + kk * 2048, 8192, 1024);
            if (!B_MN) bdesc = make_smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            else bdesc = make_smem_desc_sw128(b_addr + kk * 2048, 8192, 1024);
            umma_bf16(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&tfull_bar[acc]);
      __syncwarp();
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  } else if constexpr (EPI == kEpiAdamW8) {
    // -------------------- epilogue: weight gradient -> 8-bit AdamW --------------------
    // Thread = one accumulator row (TMEM lane); one 32-column TMEM load = one 8-bit
    // quantisation block of W, so the update needs no shuffles. W, m and v of each
    // 32x32 job arrive by TMA (swizzled, so the per-row 16-byte reads are bank-conflict
    // free) several jobs ahead of the one being computed, the block scales a job ahead, and
    // the updated W / m / v leave by TMA stores. The gradient never reaches HBM.
    // Jobs: each tile has NJ = BN / 32 column blocks per TMEM lane quarter, shared by the
    // NWQ warps of the quarter. Column block c of the CTA's tile tt goes to warp
    // (tt * NJ + c) % NWQ, so over NWQ tiles every warp gets NJ jobs even when NWQ does not
    // divide NJ; every warp has at least one job in every tile (NJ >= NWQ).
    constexpr int NWQ = epi_warps(EPI) / 4;
    constexpr int NJ = BN / 32;
    static_assert(NJ >= NWQ, "every epilogue warp needs a job in every tile");
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // warp within its lane quarter
    constexpr int kOptRing = opt_ring(BN, STAGES);
    const int ew = warp - 2;
    uint8_t* ring = smem + L::EPI_STAGE_OFF + ew * kOptRing * kOptJob;
    uint64_t* obar =
        reinterpret_cast<uint64_t*>(smem + L::EPI_STAGE_OFF + epi_warps(EPI) * kOptRing * kOptJob) + ew * kOptRing;
    const int my_tiles = total_tiles > (int)blockIdx.x ? (total_tiles - (int)blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const int njobs = my_tiles * NJ > half ? (my_tiles * NJ - half + NWQ - 1) / NWQ : 0;
    // tile (in this CTA's sequence) and column block of this warp's job j
    auto job_tc = [&](int j, int& tt, int& c) {
      const int x = (j / NJ) * (NWQ * NJ) + (j % NJ) * NWQ + half;
      tt = x / NJ;
      c = x - tt * NJ;
    };
    auto job_tile = [&](int j) {
      int tt, c;
      job_tc(j, tt, c);
      return tt;
    };
    const AdamCoef kc = adam_coef(p.opt);
    const int nb_row = p.N / 32;
    // Tile decoding (integer divisions, group offsets) happens once per tile and stream of
    // jobs: the TMA issue, the scale prefetch and the update each walk the jobs in order,
    // so each keeps the last tile it decoded.
    struct TileMemo {
      int tt = -1;
      TileInfo ti;
    };
    auto job_pos = [&](int j, int& grow, int& col0, int& c, TileInfo& ti, TileMemo& memo) {
      int tt;
      job_tc(j, tt, c);
      if (tt != memo.tt) {
        memo.ti = decode_tile<RAGGED_K, BN>((int)blockIdx.x + tt * (int)gridDim.x, p, s_prefix);
        memo.tt = tt;
      }
      ti = memo.ti;
      grow = ti.g * p.M + ti.row0 + q * 32;
      col0 = ti.n0 + c * 32;
    };
    TileMemo memo_issue, memo_scale, memo_main;
    auto issue = [&](int j) {  // lane 0
      int grow, col0, c;
      TileInfo ti;
      job_pos(j, grow, col0, c, ti, memo_issue);
      const int s = j % kOptRing;
      uint8_t* b = ring + s * kOptJob;
      mbar_arrive_expect_tx(&obar[s], kOptJob);
      tma_load_2d(b, &om.w, &obar[s], col0, grow);
      tma_load_2d(b + 2048, &om.m, &obar[s], col0, grow);
      tma_load_2d(b + 3072, &om.v, &obar[s], col0, grow);
    };
    auto load_scales = [&](int j, float& ms, float& vs) {
      ms = vs = 0.f;
      if (j >= njobs) return;
      int grow, col0, c;
      TileInfo ti;
      job_pos(j, grow, col0, c, ti, memo_scale);
      const size_t bi = (size_t)(grow + lane) * nb_row + col0 / 32;
      ms = p.opt.m_scale[bi];
      vs = p.opt.v_scale[bi];
    };
    int issued = 0, consumed = 0;
    if (lane == 0)
      for (; issued < kOptRing - 1 && issued < njobs; ++issued) issue(issued);
    int acc = 0;
    uint32_t acc_phase = 0;
    float msc, vsc;
    load_scales(0, msc, vsc);
    const int sw = (lane >> 1) & 3, sc = (lane >> 2) & 1;  // swizzled 16-byte chunk of this row
    int cur_tile = -1;
    for (int j = 0; j < njobs; ++j) {
      int grow, col0, c;
      TileInfo ti;
      job_pos(j, grow, col0, c, ti, memo_main);
      const bool first_of_tile = memo_main.tt != cur_tile;
      cur_tile = memo_main.tt;
      const bool last_of_tile = j + 1 == njobs || job_tile(j + 1) != cur_tile;
      float nms, nvs;
      load_scales(j + 1, nms, nvs);
      if (first_of_tile) {
        if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, s_abort, p.status, p.timeout_ns)) break;
        tc_fence_after();
      }
      const int s = j % kOptRing;
      if (!mbar_wait_bounded(&obar[s], (uint32_t)(j / kOptRing) & 1u, s_abort, p.status, p.timeout_ns)) break;
      ++consumed;
      uint8_t* b = ring + s * kOptJob;
      float g[32];
      tmem_ld32(tmem_base + acc * BN + ((uint32_t)(q * 32) << 16) + c * 32, g);
      if (ti.num_kb == 0) {
#pragma unroll
        for (int e = 0; e < 32; ++e) g[e] = 0.f;
      }
      uint8_t* wrow = b + lane * 64;
      uint8_t* mrow = b + 2048 + lane * 32;
      uint8_t* vrow = b + 3072 + lane * 32;
      uint2 w[8];
      uint32_t mq[8], vq[8];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const uint4 x = *reinterpret_cast<const uint4*>(wrow + ((cc ^ sw) << 4));
        w[2 * cc] = make_uint2(x.x, x.y);
        w[2 * cc + 1] = make_uint2(x.z, x.w);
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const uint4 x = *reinterpret_cast<const uint4*>(mrow + ((cc ^ sc) << 4));
        const uint4 y = *reinterpret_cast<const uint4*>(vrow + ((cc ^ sc) << 4));
        mq[4 * cc] = x.x; mq[4 * cc + 1] = x.y; mq[4 * cc + 2] = x.z; mq[4 * cc + 3] = x.w;
        vq[4 * cc] = y.x; vq[4 * cc + 1] = y.y; vq[4 * cc + 2] = y.z; vq[4 * cc + 3] = y.w;
      }
      adamw_8bit_units<8>(g, w, mq, vq, msc, vsc, (uint64_t)(grow + lane) * p.N + col0, 0, kc, p.opt);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        *reinterpret_cast<uint4*>(wrow + ((cc ^ sw) << 4)) = make_uint4(w[2 * cc].x, w[2 * cc].y, w[2 * cc + 1].x, w[2 * cc + 1].y);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        *reinterpret_cast<uint4*>(mrow + ((cc ^ sc) << 4)) = make_uint4(mq[4 * cc], mq[4 * cc + 1], mq[4 * cc + 2], mq[4 * cc + 3]);
        *reinterpret_cast<uint4*>(vrow + ((cc ^ sc) << 4)) = make_uint4(vq[4 * cc], vq[4 * cc + 1], vq[4 * cc + 2], vq[4 * cc + 3]);
      }
      const size_t bi = (size_t)(grow + lane) * nb_row + col0 / 32;
      p.opt.m_scale[bi] = msc;
      p.opt.v_scale[bi] = vsc;
      fence_proxy_async_smem();  // shared-memory writes -> the TMA stores
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&om.w, b, col0, grow);
        tma_store_2d(&om.m, b + 2048, col0, grow);
        tma_store_2d(&om.v, b + 3072, col0, grow);
        bulk_commit();
        if (issued < njobs) {  // refill the slot of job j - 1 (its stores are the older group)
          bulk_wait_read<1>();
          issue(issued);
          ++issued;
        }
      }
      __syncwarp();
      if (last_of_tile) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      msc = nms;
      vsc = nvs;
    }
    if (lane == 0) {
      // after an abort: let every issued load land (bounded) before the CTA exits
      for (int j = consumed; j < issued; ++j) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&obar[j % kOptRing], (uint32_t)(j / kOptRing) & 1u) &&
               globaltimer_ns() - t0 < p.timeout_ns) {
        }
      }
      bulk_wait_all();
    }
    __syncwarp();
  } else {
    // --------------------------------- epilogue --------------------------------
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      TileInfo ti = decode_tile<RAGGED_K, BN>(t, p, s_prefix);
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, s_abort, p.status, p.timeout_ns)) break;
      tc_fence_after();
      epilogue_tile<BN, EPI>(p, ti, tmem_base + acc * BN, warp, lane, smem + L::EPI_STAGE_OFF);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  __syncthreads();
  if (warp == 1) {
    if (*s_abort) {
      // drain: wait (bounded) for any MMA this thread issued before releasing TMEM
      if (lane == 0) umma_commit(drain_bar);
      __syncwarp();
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain_bar, 0) && globaltimer_ns() - t0 < p.timeout_ns) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// Writes one 32 x 32 bf16 block (this thread's row: 32 floats, scaled to bf16) into a
// 64-byte-swizzled staging block: thread = row, 16-byte chunk c lands at chunk c ^ ((row >>
// 1) & 3), which is the layout a SWIZZLE_64B tensor map stores from, and which spreads the
// warp's 16-byte writes over all banks.
__device__ __forceinline__ void stage_row_bf16(uint8_t* blk, int lane, const uint32_t (&w)[16]) {
  const int sw = (lane >> 1) & 3;
  uint8_t* row = blk + lane * 64;
#pragma unroll
  for (int cc = 0; cc < 4; ++cc)
    *reinterpret_cast<uint4*>(row + ((cc ^ sw) << 4)) = make_uint4(w[4 * cc], w[4 * cc + 1], w[4 * cc + 2], w[4 * cc + 3]);
}

// One accumulator tile through a bf16-output epilogue whose rows leave by TMA stores:
// each warp converts a 32-row x 32-column block, stages it in shared memory and one lane
// stores it with cp.async.bulk.tensor (one 2 KB request instead of 32 rows of scattered
// 16-byte stores). A warp's 32 rows go out by TMA only when they all lie inside the group;
// the ragged end of a group takes the per-thread stores of epilogue_tile.
template <int BN, int EPI>
__device__ __forceinline__ void epilogue_tile_tma(const GemmParams& p, const EpiMaps& em, const TileInfo& ti,
                                                  uint32_t t_acc, int warp, int lane, uint8_t* stage) {
  static_assert(EPI == kEpiBf16 || EPI == kEpiSwigluFwd || EPI == kEpiSwigluBwd, "bf16-output epilogues only");
  const int q = warp & 3;
  const int half = (warp - 2) >> 2;
  constexpr int kCStep = kEpiWarps / 4;
  const int r0w = ti.row0 + q * 32;  // first row of this warp's slab
  if (r0w >= ti.row_end) return;     // nothing of this warp's rows is in the group
  if (r0w + 32 > ti.row_end) {       // ragged end of the group: per-thread stores
    epilogue_tile<BN, EPI>(p, ti, t_acc, warp, lane, nullptr);
    return;
  }
  const int r = r0w + lane;
  const uint32_t t_row = t_acc + ((uint32_t)(q * 32) << 16);
  const bool zero = ti.num_kb == 0;
  auto wait_stage_free = [&]() {  // the previous block's TMA stores have read the staging area
    if (lane == 0) bulk_wait_read<0>();
    __syncwarp();
  };
  auto store_blocks = [&](int n, const CUtensorMap* const* maps, const int* cols) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      for (int i = 0; i < n; ++i) tma_store_2d(maps[i], stage + i * 2048, cols[i], r0w);
      bulk_commit();
    }
  };
  if (EPI == kEpiBf16) {
#pragma unroll 1
    for (int c = half; c < BN / 32; c += kCStep) {
      float v[32];
      tmem_ld32(t_row + c * 32, v);
      uint32_t w[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(zero ? 0.f : v[2 * j], zero ? 0.f : v[2 * j + 1]);
      wait_stage_free();
      stage_row_bf16(stage, lane, w);
      const CUtensorMap* maps[1] = {&em.out};
      const int cols[1] = {ti.n0 + c * 32};
      store_blocks(1, maps, cols);
    }
  } else if (EPI == kEpiSwigluFwd) {
    // accumulator columns [0,128) = gate, [128,256) = up, for I-range [i0, i0+128)
    const int i0 = ti.n0 / 2;
#pragma unroll 1
    for (int c = half; c < 4; c += kCStep) {
      float g[32], u[32];
      tmem_ld32(t_row + c * 32, g);
      tmem_ld32(t_row + 128 + c * 32, u);
      uint32_t wg[16], wu[16], wh[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        // round g/u to bf16 first so h is consistent with the stored pre-activation
        const float g0 = __bfloat162float(__float2bfloat16(g[2 * j])), g1 = __bfloat162float(__float2bfloat16(g[2 * j + 1]));
        const float u0 = __bfloat162float(__float2bfloat16(u[2 * j])), u1 = __bfloat162float(__float2bfloat16(u[2 * j + 1]));
        wg[j] = pack_bf16x2(g0, g1);
        wu[j] = pack_bf16x2(u0, u1);
        wh[j] = pack_bf16x2(silu_f(g0) * u0, silu_f(g1) * u1);
      }
      wait_stage_free();
      stage_row_bf16(stage, lane, wg);
      stage_row_bf16(stage + 2048, lane, wu);
      stage_row_bf16(stage + 4096, lane, wh);
      const CUtensorMap* maps[3] = {&em.aux, &em.aux, &em.out};
      const int cols[3] = {i0 + c * 32, p.I + i0 + c * 32, i0 + c * 32};
      store_blocks(3, maps, cols);
    }
  } else {
    // SwiGLU backward: accumulator = dh_unweighted[r, i0 : i0+BN]; gate weight w = row_w[r]
    const int i0 = ti.n0;
    const __nv_bfloat16* gu = reinterpret_cast<const __nv_bfloat16*>(p.aux);
    const float wr = __ldg(p.row_w + r);
    float dw_part = 0.f;
    // gate|up of this row's next 32 columns are loaded one job ahead, so their latency
    // overlaps the current job's TMEM load, math and stores (two jobs ahead spills: ten
    // warps leave 168 registers a thread)
    const __nv_bfloat16* grow = gu + (size_t)r * p.ld_aux + i0;
    uint4 gn[4], un[4];
    auto load_gu = [&](int c) {
      const uint4* sg = reinterpret_cast<const uint4*>(grow + c * 32);
      const uint4* su = reinterpret_cast<const uint4*>(grow + p.I + c * 32);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        gn[j] = __ldg(sg + j);
        un[j] = __ldg(su + j);
      }
    };
    load_gu(half);
#pragma unroll 1
    for (int c = half; c < BN / 32; c += kCStep) {
      uint4 gv[4], uv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        gv[j] = gn[j];
        uv[j] = un[j];
      }
      if (c + kCStep < BN / 32) load_gu(c + kCStep);
      float d[32];
      tmem_ld32(t_row + c * 32, d);
      uint32_t rg[16], ru[16], rh[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t gw[4] = {gv[j].x, gv[j].y, gv[j].z, gv[j].w};
        const uint32_t uw[4] = {uv[j].x, uv[j].y, uv[j].z, uv[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 g2 = unpack_bf16x2(gw[e]);
          const float2 u2 = unpack_bf16x2(uw[e]);
          const float dd0 = zero ? 0.f : d[8 * j + 2 * e], dd1 = zero ? 0.f : d[8 * j + 2 * e + 1];
          const float s0 = sigmoid_f(g2.x), s1 = sigmoid_f(g2.y);
          const float si0 = g2.x * s0, si1 = g2.y * s1;
          const float h0 = si0 * u2.x, h1 = si1 * u2.y;
          dw_part += dd0 * h0 + dd1 * h1;
          const float wd0 = wr * dd0, wd1 = wr * dd1;
          rg[4 * j + e] = pack_bf16x2(wd0 * u2.x * s0 * (1.f + g2.x * (1.f - s0)),
                                      wd1 * u2.y * s1 * (1.f + g2.y * (1.f - s1)));
          ru[4 * j + e] = pack_bf16x2(wd0 * si0, wd1 * si1);
          rh[4 * j + e] = pack_bf16x2(wr * h0, wr * h1);
        }
      }
      wait_stage_free();
      stage_row_bf16(stage, lane, rg);
      stage_row_bf16(stage + 2048, lane, ru);
      stage_row_bf16(stage + 4096, lane, rh);
      const CUtensorMap* maps[3] = {&em.out, &em.out, &em.aux2};
      const int cols[3] = {i0 + c * 32, p.I + i0 + c * 32, i0 + c * 32};
      store_blocks(3, maps, cols);
    }
    if (p.row_dw) atomicAdd(p.row_dw + r, dw_part);
  }
}

// =====================================================================================
// CTA-pair kernel: one tcgen05.mma.cta_group::2 per k-step over a 256-row x BN tile.
//
// A cluster of two CTAs on two SMs shares each MMA: every CTA TMA-loads its own 128 rows
// of A and its own BN/2 rows (columns of the product) of B from this GPU's memory into
// its own shared memory, and receives its 128 accumulator rows in its own TMEM. Per SM
// the tensor core then streams half of the B tile a single-CTA MMA of the same output
// width would, which is what keeps shared-memory bandwidth below the tensor-core rate at
// N = 256 (a single CTA at M = 128, N = 256 needs 96 B/clk of operand reads plus the TMA
// writes, beyond the SM's shared-memory bandwidth).
//
// Roles per CTA as in the single-CTA kernel (warp 0 TMA, warp 1 MMA, warps 2..9
// epilogue), except that only the leader CTA (cluster rank 0) issues MMAs:
//   full[s]   leader only; the leader's producer expects both CTAs' bytes, both CTAs'
//             loads complete on it
//   empty[s]  per CTA; the leader's MMA thread commits to both after the stage's MMAs
//   tfull[a]  per CTA; committed to both when a tile's MMAs are done
//   tempty[a] leader only; both CTAs' epilogue warps arrive (2 x 8 arrivals)
// Every load fills only its own CTA's shared memory; the only cross-CTA traffic is mbarrier arrivals and the MMA's
// own reads of the peer's operand tiles.
// =====================================================================================
template <int BN, int STAGES, int EPI>
struct PairSmem {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = (BN / 2) * kBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_STAGE_OFF = STAGES * STAGE_BYTES;
  // fp32 epilogues transpose through 32 x 33 floats per warp; bf16 epilogues stage their
  // TMA stores (kEpiStoreBytes per warp)
  static constexpr int EPI_STAGE_BYTES =
      (EPI == kEpiAdamW || EPI == kEpiF32) ? kEpiWarps * 32 * 33 * 4 : kEpiWarps * kEpiStoreBytes;
  static constexpr int BAR_OFF = EPI_STAGE_OFF + EPI_STAGE_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 4 + 1;  // full, empty, tfull[2], tempty[2], drain
  static constexpr int MISC_OFF = BAR_OFF + NUM_BARS * 8;
  static constexpr int PREFIX_OFF = MISC_OFF + 16;
  static size_t bytes(int G) { return 1024 + PREFIX_OFF + 4 * (size_t)(G + 1); }
};

constexpr int kPairM = 2 * kBM;
constexpr bool epi_tma_store(int epi) { return epi == kEpiBf16 || epi == kEpiSwigluFwd || epi == kEpiSwigluBwd; }

template <int BN, int STAGES, bool A_MN, bool B_MN, bool RAGGED_K, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const GemmParams p, const __grid_constant__ EpiMaps em) {
  static_assert(BN == 256, "the pair kernel covers 256 output columns per tile");
  static_assert(EPI != kEpiAdamW8, "the 8-bit optimizer epilogue runs in the single-CTA kernel");
  using L = PairSmem<BN, STAGES, EPI>;
  constexpr int BH = BN / 2;  // B rows (product columns) held by each CTA
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  int* s_prefix = reinterpret_cast<int*>(smem + L::PREFIX_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_ctarank();
  const bool leader = cta == 0;
  const int cluster = (int)cluster_id_x();
  const int nclusters = (int)num_clusters_x();

  if (RAGGED_K) group_order(p, s_prefix, reinterpret_cast<int*>(smem));
  if (!RAGGED_K && threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < p.G; ++g) {
      s_prefix[g] = acc;
      const int rows = __ldg(p.group_off + g + 1) - __ldg(p.group_off + g);
      acc += ((rows + kPairM - 1) / kPairM) * p.n_tiles;
    }
    s_prefix[p.G] = acc;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (epi_tma_store(EPI) && warp >= 2 && lane == 0) {
    tma_prefetch_desc(&em.out);
    if (EPI != kEpiBf16) tma_prefetch_desc(EPI == kEpiSwigluFwd ? &em.aux : &em.aux2);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 2 * BN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = RAGGED_K ? p.G * (p.M / kPairM) * p.n_tiles : s_prefix[p.G];

  if (warp == 0) {
    // ------------------------------- TMA producer -------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; t < total_tiles && ok; t += nclusters) {
        const TileInfo ti = decode_tile<RAGGED_K, BN, kPairM>(t, p, s_prefix);
        const int my_row0 = ti.row0 + (int)cta * kBM;  // this CTA's rows (ragged M) / m columns (ragged K)
        for (int kb = 0; kb < ti.num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1, s_abort, p.status, p.timeout_ns)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * L::STAGE_BYTES;
          uint8_t* sB = sA + L::A_BYTES;
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * L::STAGE_BYTES);
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
          if (!A_MN) {
            tma_load_2d_pair(sA, &tmA, fb, kb * kBK, my_row0);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j)
              tma_load_2d_pair(sA + j * 8192, &tmA, fb, my_row0 + j * 64, ti.k0 + kb * kBK);
          }
          if (!B_MN) {
            int brow;
            if (EPI == kEpiSwigluFwd) {  // leader: gate rows, peer: up rows of the same I range
              brow = ti.g * p.b_rows_per_group + (int)cta * p.I + ti.n0 / 2;
            } else {
              brow = ti.g * p.b_rows_per_group + ti.n0 + (int)cta * BH;
            }
            tma_load_2d_pair(sB, &tmB, fb, kb * kBK, brow);
          } else {
            const int krow = RAGGED_K ? (ti.k0 + kb * kBK) : (ti.g * p.b_rows_per_group + kb * kBK);
#pragma unroll
            for (int j = 0; j < BH / 64; ++j)
              tma_load_2d_pair(sB + j * 8192, &tmB, fb, ti.n0 + (int)cta * BH + j * 64, krow);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------- MMA issuer (leader CTA only) -------------------------
    if (leader) {
      constexpr uint32_t idesc = make_idesc_bf16(kPairM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = cluster; t < total_tiles && ok; t += nclusters) {
        const TileInfo ti = decode_tile<RAGGED_K, BN, kPairM>(t, p, s_prefix);
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1, s_abort, p.status, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < ti.num_kb; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase, s_abort, p.status, p.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(smem + stage * L::STAGE_BYTES);
            const uint32_t b_addr = a_addr + L::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              uint64_t adesc, bdesc;
              if (!A_MN) adesc = make_smem_desc_sw128(a_addr + kk * 32, 16, 1024);
              else adesc = make_smem_desc_sw128(a_addr + kk * 2048, 8192, 1024);
              if (!B_MN) bdesc = make_smem_desc_sw128(b_addr + kk * 32, 16, 1024);
              else bdesc = make_smem_desc_sw128(b_addr + kk * 2048, 8192, 1024);
              umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            const uint32_t eb = smem_u32(&empty_bar[stage]);
            umma_commit_pair(mapa_shared(eb, 0));
            umma_commit_pair(mapa_shared(eb, 1));
          }
          __syncwarp();
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (lane == 0) {
          const uint32_t tb = smem_u32(&tfull_bar[acc]);
          umma_commit_pair(mapa_shared(tb, 0));
          umma_commit_pair(mapa_shared(tb, 1));
        }
        __syncwarp();
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else {
    // ----------------------------- epilogue (both CTAs) -----------------------------
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = cluster; t < total_tiles; t += nclusters) {
      TileInfo ti = decode_tile<RAGGED_K, BN, kPairM>(t, p, s_prefix);
      ti.row0 += (int)cta * kBM;
      if (!mbar_wait_bounded(&tfull_bar[acc], acc_phase, s_abort, p.status, p.timeout_ns)) break;
      tc_fence_after();
      if constexpr (epi_tma_store(EPI)) {
        epilogue_tile_tma<BN, EPI>(p, em, ti, tmem_base + acc * BN, warp, lane,
                                   smem + L::EPI_STAGE_OFF + (warp - 2) * kEpiStoreBytes);
      } else {
        epilogue_tile<BN, EPI>(p, ti, tmem_base + acc * BN, warp, lane, smem + L::EPI_STAGE_OFF);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty_bar[acc]), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (epi_tma_store(EPI) && lane == 0) bulk_wait_all();  // this warp's stores are done
    __syncwarp();
  }

  __syncthreads();
  if (warp == 1 && leader && *s_abort) {
    // drain: wait (bounded) for any MMA this thread issued before the TMEM is released
    if (lane == 0) umma_commit_pair(mapa_shared(smem_u32(drain_bar), 0));
    __syncwarp();
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(drain_bar, 0) && globaltimer_ns() - t0 < p.timeout_ns) {
    }
  }
  tc_fence_before();
  cluster_sync();  // no CTA leaves while its peer may still read its operands or TMEM
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, 2 * BN);
}

// =====================================================================================
// Host side
// =====================================================================================

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  // The encoder is a driver call and needs the device's context current on this thread.
  // A thread that has only selected the device (e.g. autograd's backward worker on device
  // 0) may not have bound it yet; a no-op runtime call binds the primary context.
  static thread_local bool bound = false;
  if (!bound) {
    cudaFree(nullptr);
    bound = true;
  }
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !ptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix with a {64, box_rows} box and
// 128-byte swizzle. `cols` is the contiguous dimension.
static CUtensorMap make_tmap_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld_elems,
                                  int box_rows) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld_elems * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld_elems * 2) & 15))
    throw std::runtime_error("TMA operand must be 16-byte aligned with 16-byte row stride");
  CUresult r = get_encode_fn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return tm;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, bool RAGGED_K, int EPI>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p,
                   int max_tiles, cudaStream_t stream, const OptMaps& om = OptMaps{}) {
  using L = GemmSmem<BN, STAGES, EPI>;
  auto kern = grouped_gemm_kernel<BN, STAGES, A_MN, B_MN, RAGGED_K, EPI>;
  size_t smem = L::bytes(p.G);
  if (smem > kMaxSmem) throw std::runtime_error("grouped_gemm: too many groups for this kernel's shared memory");
  static unsigned long long smem_devices = 0;
  smem_optin_once(kern, kMaxSmem, smem_devices);
  int grid = num_sms();
  if (max_tiles > 0 && max_tiles < grid) grid = max_tiles;
  if (grid < 1) grid = 1;
  kern<<<grid, threads_for(EPI), smem, stream>>>(ta, tb, p, om);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("grouped_gemm launch: ") + cudaGetErrorString(e));
}

// Tensor map of a bf16 output [rows, cols] (row stride ld elements) for the TMA-store
// epilogues: 32 x 32 boxes, 64-byte swizzle (matching stage_row_bf16).
static CUtensorMap make_tmap_out(const void* base, int64_t rows, int64_t cols, int64_t ld) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || (cols % 32))
    throw std::runtime_error("TMA-store output must be 16-byte aligned, 16-byte row stride, 32-column multiple");
  CUresult r = get_encode_fn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return tm;
}

// Output maps of a call's bf16 epilogue: rows = the call's A rows (ragged M) or, for a
// one-group weight gradient, M.
static EpiMaps make_epi_maps(const GemmCall& c, int epi, int64_t rows = -1) {
  EpiMaps em{};
  const GemmParams& p = c.p;
  if (rows < 0) rows = c.a_rows;
  if (epi == kEpiBf16) {
    em.out = make_tmap_out(p.out, rows, p.N, p.ldo);
  } else if (epi == kEpiSwigluFwd) {
    em.out = make_tmap_out(p.out, c.a_rows, p.I, p.ldo);
    em.aux = make_tmap_out(p.aux, c.a_rows, 2 * p.I, p.ld_aux);
  } else if (epi == kEpiSwigluBwd) {
    em.out = make_tmap_out(p.out, c.a_rows, 2 * p.I, p.ldo);
    em.aux2 = make_tmap_out(p.aux2, c.a_rows, p.I, p.ld_aux2);
  }
  return em;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, bool RAGGED_K, int EPI>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int max_tiles,
                        cudaStream_t stream, const EpiMaps& em = EpiMaps{}) {
  using L = PairSmem<BN, STAGES, EPI>;
  auto kern = grouped_gemm_pair_kernel<BN, STAGES, A_MN, B_MN, RAGGED_K, EPI>;
  const size_t smem = L::bytes(p.G);
  static unsigned long long smem_devices = 0;
  smem_optin_once(kern, 232448, smem_devices);
  int clusters = num_sms() / 2;
  if (max_tiles > 0 && max_tiles < clusters) clusters = max_tiles;
  if (clusters < 1) clusters = 1;
  kern<<<2 * clusters, kThreads, smem, stream>>>(ta, tb, p, em);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("grouped_gemm (pair) launch: ") + cudaGetErrorString(e));
}

// CTA pairs for the 256-column tiles: on unless SEPX_GEMM_PAIR=0 or gemm_set_pairs(false)
// (single-CTA tiles, for comparison).
static int g_pairs = -1;
static bool use_pairs() {
  if (g_pairs < 0) {
    const char* v = std::getenv("SEPX_GEMM_PAIR");
    g_pairs = (v && v[0] == '0') ? 0 : 1;
  }
  return g_pairs == 1;
}
bool gemm_set_pairs(bool on) {
  const bool prev = use_pairs();
  g_pairs = on ? 1 : 0;
  return prev;
}

// ---------------------------------------------------------------------------------
// Forward / dgrad: D[rows, N] = A[rows, K] . B_g   (ragged M)
//   b_kmajor: B stored [G * N_b, K] (weights as [out, in]);  else B stored [G * K, N].
// ---------------------------------------------------------------------------------
void grouped_gemm_ragged_m(const GemmCall& c, cudaStream_t stream) {
  GemmParams p = c.p;
  if (p.K % kBK) throw std::runtime_error("K must be a multiple of 64");
  CUtensorMap ta = make_tmap_bf16(c.A, c.a_rows, p.K, c.lda, 128);
  // upper bound on tiles, used only to size the grid
  int max_tiles = 0;
  if (c.epi == kEpiSwigluFwd) {
    if (!c.b_kmajor) throw std::runtime_error("swiglu fwd expects K-major weights");
    if (p.I % 128) throw std::runtime_error("SwiGLU intermediate must be a multiple of 128");
    p.n_tiles = p.I / 128;
    CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.K, c.ldb, 128);
    if (use_pairs()) {
      launch_pair<256, 5, false, false, false, kEpiSwigluFwd>(ta, tb, p, (int)((c.a_rows + 255) / 256 + p.G) * p.n_tiles,
                                                              stream, make_epi_maps(c, kEpiSwigluFwd));
      return;
    }
    max_tiles = (int)((c.a_rows + 127) / 128 + p.G) * p.n_tiles;
    launch<256, 4, false, false, false, kEpiSwigluFwd>(ta, tb, p, max_tiles, stream);
    return;
  }
  if (c.epi == kEpiSwigluBwd) {
    if (c.b_kmajor) throw std::runtime_error("swiglu bwd expects MN-major weights");
    if (p.N % 256) throw std::runtime_error("N must be a multiple of 256");
    p.n_tiles = p.N / 256;
    CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.N, c.ldb, 64);
    if (use_pairs()) {
      launch_pair<256, 5, false, true, false, kEpiSwigluBwd>(ta, tb, p, (int)((c.a_rows + 255) / 256 + p.G) * p.n_tiles,
                                                             stream, make_epi_maps(c, kEpiSwigluBwd));
      return;
    }
    max_tiles = (int)((c.a_rows + 127) / 128 + p.G) * p.n_tiles;
    launch<256, 4, false, true, false, kEpiSwigluBwd>(ta, tb, p, max_tiles, stream);
    return;
  }
  if (c.epi != kEpiBf16) throw std::runtime_error("unsupported epilogue for ragged-M GEMM");
  if (p.N % 256 != 0 && p.N % 32 == 0 && p.N > 256 && p.G == 1 && use_pairs() && c.b_kmajor) {
    // one group (a dense projection) whose last 256-column tile is partial: B rows past N
    // load as zeros and the TMA stores clip the output at N (e.g. a vocabulary)
    p.n_tiles = (p.N + 255) / 256;
    CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.K, c.ldb, 128);
    launch_pair<256, 5, false, false, false, kEpiBf16>(ta, tb, p, (int)((c.a_rows + 255) / 256 + p.G) * p.n_tiles,
                                                       stream, make_epi_maps(c, kEpiBf16));
    return;
  }
  if (p.N % 256 == 0) {
    p.n_tiles = p.N / 256;
    max_tiles = (int)((c.a_rows + 127) / 128 + p.G) * p.n_tiles;
    const int pair_tiles = (int)((c.a_rows + 255) / 256 + p.G) * p.n_tiles;
    if (c.b_kmajor) {
      CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.K, c.ldb, 128);
      if (use_pairs()) launch_pair<256, 5, false, false, false, kEpiBf16>(ta, tb, p, pair_tiles, stream, make_epi_maps(c, kEpiBf16));
      else launch<256, 4, false, false, false, kEpiBf16>(ta, tb, p, max_tiles, stream);
    } else {
      CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.N, c.ldb, 64);
      if (use_pairs()) launch_pair<256, 5, false, true, false, kEpiBf16>(ta, tb, p, pair_tiles, stream, make_epi_maps(c, kEpiBf16));
      else launch<256, 4, false, true, false, kEpiBf16>(ta, tb, p, max_tiles, stream);
    }
  } else if (p.N % 128 == 0) {
    p.n_tiles = p.N / 128;
    max_tiles = (int)((c.a_rows + 127) / 128 + p.G) * p.n_tiles;
    if (c.b_kmajor) {
      CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.K, c.ldb, 128);
      launch<128, 6, false, false, false, kEpiBf16>(ta, tb, p, max_tiles, stream);
    } else {
      CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.N, c.ldb, 64);
      launch<128, 6, false, true, false, kEpiBf16>(ta, tb, p, max_tiles, stream);
    }
  } else {
    throw std::runtime_error("N must be a multiple of 128");
  }
}

// ---------------------------------------------------------------------------------
// Weight gradient: D[g][M, N] = sum_{r in group g} A[r, m] * B[r, n]   (ragged K)
//   A stored [rows, M], B stored [rows, N] (both row-major, so MN-major operands).
// ---------------------------------------------------------------------------------
void grouped_gemm_ragged_k(const GemmCall& c, cudaStream_t stream) {
  GemmParams p = c.p;
  if (p.M % 128) throw std::runtime_error("M must be a multiple of 128");
  CUtensorMap ta = make_tmap_bf16(c.A, c.a_rows, p.M, c.lda, 64);
  CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.N, c.ldb, 64);
  if (c.epi == kEpiBf16) {  // one group (a dense weight gradient), bf16 [M, N]
    if (p.G != 1) throw std::runtime_error("bf16 weight gradients take a single group");
    if (p.N % 256 == 0) {
      p.n_tiles = p.N / 256;
      if (use_pairs() && p.M % 256 == 0) {
        launch_pair<256, 5, true, true, true, kEpiBf16>(ta, tb, p, (p.M / 256) * p.n_tiles, stream,
                                                        make_epi_maps(c, kEpiBf16, p.M));
        return;
      }
      launch<256, 3, true, true, true, kEpiBf16>(ta, tb, p, (p.M / 128) * p.n_tiles, stream);
    } else if (p.N % 128 == 0) {
      p.n_tiles = p.N / 128;
      launch<128, 5, true, true, true, kEpiBf16>(ta, tb, p, (p.M / 128) * p.n_tiles, stream);
    } else {
      throw std::runtime_error("N must be a multiple of 128");
    }
    return;
  }
  if (p.N % 256 == 0) {
    p.n_tiles = p.N / 256;
    // pairs pay off when each group reduces over enough rows (per-tile fixed costs)
    if (use_pairs() && p.M % 256 == 0 && c.a_rows >= 1024LL * p.G) {
      launch_pair<256, 5, true, true, true, kEpiF32>(ta, tb, p, p.G * (p.M / 256) * p.n_tiles, stream);
      return;
    }
    int max_tiles = p.G * (p.M / 128) * p.n_tiles;
    launch<256, 3, true, true, true, kEpiF32>(ta, tb, p, max_tiles, stream);
  } else if (p.N % 128 == 0) {
    p.n_tiles = p.N / 128;
    int max_tiles = p.G * (p.M / 128) * p.n_tiles;
    launch<128, 5, true, true, true, kEpiF32>(ta, tb, p, max_tiles, stream);
  } else {
    throw std::runtime_error("N must be a multiple of 128");
  }
}

// ---------------------------------------------------------------------------------
// Weight gradient + AdamW: W[g] <- AdamW(W[g], sum_{r in group g} A[r, :]^T B[r, :]).
// The fp32 gradient tile goes from TMEM straight into the optimizer update.
// ---------------------------------------------------------------------------------
static CUtensorMap make_tmap_state(const void* base, CUtensorMapDataType dt, int esize, int64_t rows, int64_t cols,
                                   CUtensorMapSwizzle sw) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * esize)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((cols * esize) & 15))
    throw std::runtime_error("optimizer state must be 16-byte aligned with 16-byte row stride");
  CUresult r = get_encode_fn()(&tm, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return tm;
}

void grouped_gemm_wgrad_adamw(const GemmCall& c, cudaStream_t stream) {
  GemmParams p = c.p;
  if (p.M % 128) throw std::runtime_error("M must be a multiple of 128");
  if (p.opt.kind != kOptFp32 && p.opt.kind != kOpt8bit) throw std::runtime_error("bad optimizer kind");
  CUtensorMap ta = make_tmap_bf16(c.A, c.a_rows, p.M, c.lda, 64);
  CUtensorMap tb = make_tmap_bf16(c.B, c.b_rows, p.N, c.ldb, 64);
  if (p.opt.kind == kOpt8bit) {
    if (p.N % 32) throw std::runtime_error("8-bit fused optimizer needs N % 32 == 0");
    const int64_t rows = (int64_t)p.G * p.M;
    OptMaps om;
    om.w = make_tmap_state(p.opt.param, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, p.N, CU_TENSOR_MAP_SWIZZLE_64B);
    om.m = make_tmap_state(p.opt.m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, p.N, CU_TENSOR_MAP_SWIZZLE_32B);
    om.v = make_tmap_state(p.opt.v, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, p.N, CU_TENSOR_MAP_SWIZZLE_32B);
    if (p.N % 256 == 0) {
      p.n_tiles = p.N / 256;
      // long reductions (many rows per expert: the MMA bounds the tile) take a third
      // mainloop stage; short ones (the optimizer stream bounds it) a deeper state ring
      if (c.a_rows >= 512LL * p.G || GemmSmem<256, 2, kEpiAdamW8>::bytes(p.G) > kMaxSmem)
        launch<256, 3, true, true, true, kEpiAdamW8>(ta, tb, p, p.G * (p.M / 128) * p.n_tiles, stream, om);
      else
        launch<256, 2, true, true, true, kEpiAdamW8>(ta, tb, p, p.G * (p.M / 128) * p.n_tiles, stream, om);
    } else if (p.N % 128 == 0) {
      p.n_tiles = p.N / 128;
      launch<128, 2, true, true, true, kEpiAdamW8>(ta, tb, p, p.G * (p.M / 128) * p.n_tiles, stream, om);
    } else {
      throw std::runtime_error("N must be a multiple of 128");
    }
    return;
  }
  if (p.N % 256 == 0) {
    p.n_tiles = p.N / 256;
    launch<256, 3, true, true, true, kEpiAdamW>(ta, tb, p, p.G * (p.M / 128) * p.n_tiles, stream);
  } else if (p.N % 128 == 0) {
    p.n_tiles = p.N / 128;
    launch<128, 5, true, true, true, kEpiAdamW>(ta, tb, p, p.G * (p.M / 128) * p.n_tiles, stream);
  } else {
    throw std::runtime_error("N must be a multiple of 128");
  }
}

}  // namespace sepx
