// Causal grouped-query attention (head_dim 128) on tcgen05 / TMEM, forward.
//
// One CTA per (128-query block, query head); the heaviest (latest) query blocks start
// first. Warp roles (192 threads):
//   warp 0      TMA: Q once, then K/V blocks through a 2-stage ring (local memory only)
//   warp 1      TMEM allocation + tcgen05.mma issue (one thread):
//                 S_j = Q K_j^T  (M=128 queries, N=128 keys, K=128) into one of two TMEM
//                 S buffers, and O += P_{j-1} V_{j-1} (V as an MN-major operand)
//   warps 2..5  online softmax, one query row per thread: S from TMEM, exp2 with the
//               running max, P (bf16) into shared memory in the 128B-swizzled K-major
//               layout the MMA reads; O in TMEM is rescaled only when a row's max grows
//               by more than 2^8 (lazy rescaling), and at the end O / l goes to global
//               memory with the row's log-sum-exp (natural log) for the backward pass.
//
// Inputs are token-major as written by the q/k-norm+RoPE kernel: q [T, Hq*128],
// k/v [T, Hkv*128]; output o [T, Hq*128]; lse [Hq, T] fp32.
// Every wait is bounded (sm100.cuh); a timeout aborts the CTA and records an error.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <stdexcept>
#include <string>

#include "attention.h"
#include "kernels.h"
#include "sm100.cuh"

namespace sepx {

namespace attn {
constexpr int BQ = 128, BKV = 128, D = 128;
constexpr int kThreads = 192;
constexpr int TILE = BQ * D * 2;  // 32 KB: a 128x128 bf16 tile
// shared memory map (1024-byte aligned base)
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + TILE;       // 2 stages
constexpr int OFF_V = OFF_K + 2 * TILE;   // 2 stages
constexpr int OFF_P = OFF_V + 2 * TILE;   // P (bf16), two 64-key halves
constexpr int OFF_BAR = OFF_P + TILE;
// barriers: q_full, kv_full[2], kv_empty[2], s_full[2], s_free[2], p_full, pv_done, drain
constexpr int NBAR = 12;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM = 1024 + OFF_MISC + 16;
}  // namespace attn

__global__ void __launch_bounds__(attn::kThreads, 1)
    attention_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  using namespace attn;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* pv_done = bars + 10;
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.T / BQ;
  const int qb = nqb - 1 - (int)(blockIdx.x / p.Hq);  // heavy (late) blocks first
  const int h = blockIdx.x % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int nkv = qb + 1;  // causal: key blocks 0..qb

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_o = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, TILE);
      tma_load_2d(smem + OFF_Q, &tmQ, q_full, h * D, qb * BQ);
      tma_load_2d(smem + OFF_Q + TILE / 2, &tmQ, q_full, h * D + 64, qb * BQ);
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        if (!mbar_wait_bounded(&kv_empty[st], ((j >> 1) & 1) ^ 1, s_abort, p.status, p.timeout_ns)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE);
        uint8_t* sk = smem + OFF_K + st * TILE;
        uint8_t* sv = smem + OFF_V + st * TILE;
        tma_load_2d(sk, &tmK, &kv_full[st], hk * D, j * BKV);
        tma_load_2d(sk + TILE / 2, &tmK, &kv_full[st], hk * D + 64, j * BKV);
        // V as the MN-major B operand: boxes {64 dims, 64 keys}; key half kc, dim half dc
#pragma unroll
        for (int kc = 0; kc < 2; ++kc)
#pragma unroll
          for (int dc = 0; dc < 2; ++dc)
            tma_load_2d(sv + kc * (TILE / 2) + dc * 8192, &tmV, &kv_full[st], hk * D + dc * 64, j * BKV + kc * 64);
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BKV, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16(BQ, D, false, true);
    bool ok = mbar_wait_bounded(q_full, 0, s_abort, p.status, p.timeout_ns);
    const uint32_t sq = smem_u32(smem + OFF_Q);
    const uint32_t sp = smem_u32(smem + OFF_P);
    auto issue_pv = [&](int jj) -> bool {
      // O += P_jj V_jj once the softmax has written P_jj
      if (!mbar_wait_bounded(p_full, jj & 1, s_abort, p.status, p.timeout_ns)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t sv = smem_u32(smem + OFF_V + (jj & 1) * TILE);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = make_smem_desc_sw128(sp + kb * (TILE / 2) + kk * 32, 16, 1024);
            const uint64_t bd = make_smem_desc_sw128(sv + kb * (TILE / 2) + kk * 2048, 8192, 1024);
            umma_bf16(t_o, ad, bd, idesc_o, (jj > 0 || kb > 0 || kk > 0) ? 1u : 0u);
          }
        umma_commit(pv_done);
        umma_commit(&kv_empty[jj & 1]);
      }
      __syncwarp();
      return true;
    };
    for (int j = 0; j < nkv && ok; ++j) {
      const int st = j & 1, sb = j & 1;
      if (!mbar_wait_bounded(&kv_full[st], (j >> 1) & 1, s_abort, p.status, p.timeout_ns)) break;
      if (!mbar_wait_bounded(&s_free[sb], ((j >> 1) & 1) ^ 1, s_abort, p.status, p.timeout_ns)) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t sk = smem_u32(smem + OFF_K + st * TILE);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = make_smem_desc_sw128(sq + kb * (TILE / 2) + kk * 32, 16, 1024);
            const uint64_t bd = make_smem_desc_sw128(sk + kb * (TILE / 2) + kk * 32, 16, 1024);
            umma_bf16(sb ? tmem + 128 : tmem, ad, bd, idesc_s, (kb > 0 || kk > 0) ? 1u : 0u);
          }
        umma_commit(&s_full[sb]);
      }
      __syncwarp();
      if (j > 0 && !issue_pv(j - 1)) break;
      if (j == nkv - 1 && !issue_pv(j)) break;
    }
  } else {
    // --------------------------- softmax (one row per thread) ---------------------------
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // row within the block (TMEM lane)
    const int qrow = qb * BQ + r;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float c = p.scale_log2;  // softmax scale * log2(e)
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait_bounded(&s_full[sb], (j >> 1) & 1, s_abort, p.status, p.timeout_ns)) { ok = false; break; }
      tc_fence_after();
      float x[128];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32((sb ? tmem + 128 : tmem) + lane_off + cc * 32, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) x[cc * 32 + e] = v[e] * c;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      if (j == qb) {  // diagonal block: keys after the query are masked
#pragma unroll
        for (int e = 0; e < 128; ++e)
          if (e > r) x[e] = -INFINITY;
      }
      float mb = -INFINITY;
#pragma unroll
      for (int e = 0; e < 128; ++e) mb = fmaxf(mb, x[e]);
      const bool need = (j == 0) || (mb > m + 8.f);
      const bool warp_need = __any_sync(0xffffffffu, need) && j > 0;
      float m_new = m;
      if (j == 0) m_new = mb;
      else if (warp_need) m_new = fmaxf(m, mb);
      // P_{j-1} V_{j-1} must be done before O is touched or P is overwritten
      if (j > 0 && !mbar_wait_bounded(pv_done, (j - 1) & 1, s_abort, p.status, p.timeout_ns)) { ok = false; break; }
      if (warp_need) {
        const float alpha = exp2f(m - m_new);
        l *= alpha;
        tc_fence_after();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float v[32];
          tmem_ld32(t_o + lane_off + cc * 32, v);
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] *= alpha;
          tmem_st32(t_o + lane_off + cc * 32, v);
        }
      }
      m = m_new;
      float rs = 0.f;
      uint8_t* sp = smem + OFF_P;
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {  // 16 chunks of 8 keys
        float pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          pv[e] = exp2f(x[ch * 8 + e] - m);
          rs += pv[e];
        }
        const int half = ch >> 3, c8 = ch & 7;
        uint4 w = make_uint4(pack_bf16x2(pv[0], pv[1]), pack_bf16x2(pv[2], pv[3]), pack_bf16x2(pv[4], pv[5]),
                             pack_bf16x2(pv[6], pv[7]));
        *reinterpret_cast<uint4*>(sp + half * (TILE / 2) + r * 128 + ((c8 ^ (r & 7)) * 16)) = w;
      }
      l += rs;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && mbar_wait_bounded(pv_done, (nkv - 1) & 1, s_abort, p.status, p.timeout_ns)) {
      tc_fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.o) + (size_t)qrow * p.Hq * D + h * D;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(t_o + lane_off + cc * 32, v);
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf16x2(v[8 * q] * inv, v[8 * q + 1] * inv), pack_bf16x2(v[8 * q + 2] * inv, v[8 * q + 3] * inv),
                              pack_bf16x2(v[8 * q + 4] * inv, v[8 * q + 5] * inv), pack_bf16x2(v[8 * q + 6] * inv, v[8 * q + 7] * inv));
      }
      // natural-log LSE of the scaled logits: m is in log2 units
      p.lse[(size_t)h * p.T + qrow] = (m + log2f(l)) * 0.69314718055994531f;
    }
  }

  __syncthreads();
  if (warp == 1) {
    if (*s_abort) {
      if (lane == 0) umma_commit(drain);
      __syncwarp();
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < p.timeout_ns) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =====================================================================================
// Forward, two query tiles per CTA ("ping-pong"). One CTA per (pair of 128-query tiles
// A = 2m, B = 2m + 1, query head); both tiles share every K/V block load. Warp roles
// (320 threads):
//   warp 0      TMA: Q_A and Q_B once, then K/V blocks through a 2-stage ring
//   warp 1      TMEM allocation (512 columns) + tcgen05.mma issue (one thread):
//                 S_t = Q_t K_j^T into S_t (128 fp32 columns per tile t in {A, B});
//                 O_t += P_t V_j with P_t read from TMEM (the A operand in TMEM)
//   warps 2..5  softmax of tile A, warps 6..9 softmax of tile B (one row per thread):
//               P packed to bf16 and stored back over S_t's first 64 columns.
// S_t of block j + 1 overwrites P_t of block j, so it is issued once P_t V_j completed;
// the MMA warp issues, per block, tile A's P V and next S, then tile B's, so one tile's
// P V and next S run while the other tile's softmax works.
// =====================================================================================
namespace attn2 {
constexpr int BQ = 128, BKV = 128, D = 128;
constexpr int kThreads = 320;
constexpr int TILE = BQ * D * 2;
constexpr int OFF_Q = 0;                 // Q_A, Q_B
constexpr int OFF_K = OFF_Q + 2 * TILE;  // 2 stages
constexpr int OFF_V = OFF_K + 2 * TILE;  // 2 stages
constexpr int OFF_BAR = OFF_V + 2 * TILE;
// q_full, kv_full[2], kv_empty[2], s_full[2], p_full[2], pv_done[2], drain
constexpr int NBAR = 12;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM = 1024 + OFF_MISC + 16;
}  // namespace attn2

// 2^x with the hardware approximation (one MUFU.EX2; denormal results flush to 0,
// which softmax probabilities can afford).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One 128-key block of one row: P = 2^(s c - mref) packed to bf16 pairs in pk, row sum
// in rs; with TRACK also the raw row max; DIAG masks keys > r.
template <bool DIAG, bool TRACK>
__device__ __forceinline__ void attn_exp_pass(uint32_t taddr, float c, float mref, int r, uint32_t (&pk)[64],
                                              float& rs, float& mraw) {
  const float nm = -mref;
  float acc = 0.f, mx = mraw;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    uint32_t u[64];
    tmem_ld64(taddr + hh * 64, u);
#pragma unroll
    for (int e2 = 0; e2 < 32; ++e2) {
      float s0 = __uint_as_float(u[2 * e2]), s1 = __uint_as_float(u[2 * e2 + 1]);
      if (DIAG) {
        const int e = hh * 64 + 2 * e2;
        s0 = e <= r ? s0 : -INFINITY;
        s1 = e + 1 <= r ? s1 : -INFINITY;
      }
      if (TRACK) mx = fmaxf(mx, fmaxf(s0, s1));
      const float p0 = ex2_ftz(fmaf(s0, c, nm)), p1 = ex2_ftz(fmaf(s1, c, nm));
      acc += p0 + p1;
      pk[hh * 32 + e2] = pack_bf16x2(p0, p1);
    }
  }
  rs = acc;
  mraw = mx;
}

// Raw row max of one 128-key block (keys > r masked when DIAG).
template <bool DIAG>
__device__ __forceinline__ float attn_row_max(uint32_t taddr, int r) {
  float mx = -INFINITY;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    uint32_t u[64];
    tmem_ld64(taddr + hh * 64, u);
#pragma unroll
    for (int e = 0; e < 64; ++e)
      if (!DIAG || hh * 64 + e <= r) mx = fmaxf(mx, __uint_as_float(u[e]));
  }
  return mx;
}

__global__ void __launch_bounds__(attn2::kThreads, 1)
    attention_fwd_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, AttnParams p) {
  using namespace attn2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [tile]
  uint64_t* p_full = bars + 7;    // [tile]
  uint64_t* pv_done = bars + 9;   // [tile]
  uint64_t* drain = bars + 11;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.T / BQ;
  const int npairs = (nqb + 1) / 2;
  const int m = npairs - 1 - (int)(blockIdx.x / p.Hq);  // heavy (late) pairs first
  const int h = blockIdx.x % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int qbA = 2 * m, qbB = 2 * m + 1;
  const bool hasB = qbB < nqb;
  const int nkvA = qbA + 1, nkvB = hasB ? qbB + 1 : 0;  // causal: key blocks 0..qb
  const int nkv_all = hasB ? nkvB : nkvA;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  long long* const trace = (blockIdx.x == 0) ? p.trace : nullptr;
  auto stamp = [&](int role, int j, int ev) {
    if (trace && lane == 0 && j < 64) trace[(role * 64 + j) * 4 + ev] = clock64();
  };
  // TMEM columns: S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512); P_t = S_t's first 64

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, hasB ? 2 * TILE : TILE);
      tma_load_2d(smem + OFF_Q, &tmQ, q_full, h * D, qbA * BQ);
      tma_load_2d(smem + OFF_Q + TILE / 2, &tmQ, q_full, h * D + 64, qbA * BQ);
      if (hasB) {
        tma_load_2d(smem + OFF_Q + TILE, &tmQ, q_full, h * D, qbB * BQ);
        tma_load_2d(smem + OFF_Q + TILE + TILE / 2, &tmQ, q_full, h * D + 64, qbB * BQ);
      }
      for (int j = 0; j < nkv_all; ++j) {
        const int st = j & 1;
        if (!mbar_wait_bounded(&kv_empty[st], ((j >> 1) & 1) ^ 1, s_abort, p.status, p.timeout_ns)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * TILE);
        uint8_t* sk = smem + OFF_K + st * TILE;
        uint8_t* sv = smem + OFF_V + st * TILE;
        tma_load_2d(sk, &tmK, &kv_full[st], hk * D, j * BKV);
        tma_load_2d(sk + TILE / 2, &tmK, &kv_full[st], hk * D + 64, j * BKV);
        // V as the MN-major B operand: boxes {64 dims, 64 keys}; key half kc, dim half dc
#pragma unroll
        for (int kc = 0; kc < 2; ++kc)
#pragma unroll
          for (int dc = 0; dc < 2; ++dc)
            tma_load_2d(sv + kc * (TILE / 2) + dc * 8192, &tmV, &kv_full[st], hk * D + dc * 64, j * BKV + kc * 64);
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t idesc_s = make_idesc_bf16(BQ, BKV, false, false);
    constexpr uint32_t idesc_o = make_idesc_bf16(BQ, D, false, true);
    const int nkv[2] = {nkvA, nkvB};
    auto issue_s = [&](int t, int j) {  // S_t = Q_t K_j^T
      const uint32_t sq = smem_u32(smem + OFF_Q + t * TILE);
      const uint32_t sk = smem_u32(smem + OFF_K + (j & 1) * TILE);
      if (lane == 0) {
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + t * 128, make_smem_desc_sw128(sq + kb * (TILE / 2) + kk * 32, 16, 1024),
                      make_smem_desc_sw128(sk + kb * (TILE / 2) + kk * 32, 16, 1024), idesc_s,
                      (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&s_full[t]);
      }
      __syncwarp();
    };
    auto issue_pv = [&](int t, int j) {  // O_t += P_t V_j, P_t read from TMEM
      const uint32_t sv = smem_u32(smem + OFF_V + (j & 1) * TILE);
      if (lane == 0) {
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_ts(tmem + 256 + t * 128, tmem + t * 128 + (uint32_t)((kb * 4 + kk) * 8),
                         make_smem_desc_sw128(sv + kb * (TILE / 2) + kk * 2048, 8192, 1024), idesc_o,
                         (j > 0 || kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[t]);
      }
      __syncwarp();
    };
    bool ok = mbar_wait_bounded(q_full, 0, s_abort, p.status, p.timeout_ns) &&
              mbar_wait_bounded(&kv_full[0], 0, s_abort, p.status, p.timeout_ns);
    if (ok) {
      tc_fence_after();
      issue_s(0, 0);
      if (hasB) issue_s(1, 0);
    }
    // Fixed issue order with blocking waits: for each block j, tile A's P V then its next
    // S (which overwrites P_A, so it waits for that P V to complete), then tile B's.
    for (int j = 0; j < nkv_all && ok; ++j) {
      const int nx = j + 1;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (!ok || j >= nkv[t]) continue;
        if (!mbar_wait_bounded(&p_full[t], j & 1, s_abort, p.status, p.timeout_ns)) { ok = false; break; }
        stamp(t, j, 0);
        tc_fence_after();
        issue_pv(t, j);
        stamp(t, j, 1);
        if (nx < nkv[t]) {
          if (!mbar_wait_bounded(&kv_full[nx & 1], (nx >> 1) & 1, s_abort, p.status, p.timeout_ns) ||
              !mbar_wait_bounded(&pv_done[t], j & 1, s_abort, p.status, p.timeout_ns)) {
            ok = false;
            break;
          }
          stamp(t, j, 2);
          tc_fence_after();
          issue_s(t, nx);
          stamp(t, j, 3);
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&kv_empty[j & 1]);  // K_j / V_j free once these MMAs finish
      __syncwarp();
    }
  } else {
    const int t = (warp - 2) >> 2;  // tile
    const int q4 = warp & 3;        // TMEM lane quarter
    const int r = q4 * 32 + lane;   // row within the tile (TMEM lane)
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const uint32_t ts = tmem + t * 128 + lane_off, to = tmem + 256 + t * 128 + lane_off;
    const float c = p.scale_log2;  // softmax scale * log2(e)
    const int qb = t ? qbB : qbA;
    const int nk = t ? nkvB : nkvA;
    float mrow = -INFINITY, l = 0.f;
    bool ok = nk > 0;
    for (int j = 0; j < nk && ok; ++j) {
      if (!mbar_wait_bounded(&s_full[t], j & 1, s_abort, p.status, p.timeout_ns)) { ok = false; break; }
      if (q4 == 2) stamp(2 + t, j, 0);
      tc_fence_after();
      // One pass: P = 2^(s c - m_ref) against the running max, tracking the block max on
      // the way. Only when some row's max grows by more than 2^8 (lazy rescaling) does the
      // warp rescale O and recompute P from S, still intact until P is stored over it.
      const bool diag = (j == qb);
      uint32_t pk[64];
      float rs = 0.f, mraw = -INFINITY;
      if (j == 0) {  // first block: the row max comes first
        mraw = diag ? attn_row_max<true>(ts, r) : attn_row_max<false>(ts, r);
        mrow = mraw * c;
        if (diag) attn_exp_pass<true, false>(ts, c, mrow, r, pk, rs, mraw);
        else attn_exp_pass<false, false>(ts, c, mrow, r, pk, rs, mraw);
      } else {
        if (diag) attn_exp_pass<true, true>(ts, c, mrow, r, pk, rs, mraw);
        else attn_exp_pass<false, true>(ts, c, mrow, r, pk, rs, mraw);
        const float mb = mraw * c;
        if (__any_sync(0xffffffffu, mb > mrow + 8.f)) {
          const float m_new = fmaxf(mrow, mb);
          const float alpha = exp2f(mrow - m_new);
          l *= alpha;
          // O_t is idle here: P_t V_{j-1} completed before S_t of block j was issued
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            float v[32];
            tmem_ld32(to + cc * 32, v);
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= alpha;
            tmem_st32(to + cc * 32, v);
          }
          mrow = m_new;
          if (diag) attn_exp_pass<true, false>(ts, c, mrow, r, pk, rs, mraw);
          else attn_exp_pass<false, false>(ts, c, mrow, r, pk, rs, mraw);
        }
      }
      {
        uint32_t lo[32], hi[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          lo[e] = pk[e];
          hi[e] = pk[32 + e];
        }
        if (q4 == 2) stamp(2 + t, j, 1);
        tmem_st32_u(ts, lo);
        tmem_st32_u(ts + 32, hi);
      }
      l += rs;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      if (q4 == 2) stamp(2 + t, j, 2);
    }
    if (ok && mbar_wait_bounded(&pv_done[t], (nk - 1) & 1, s_abort, p.status, p.timeout_ns)) {
      tc_fence_after();
      const int qrow = qb * BQ + r;
      const float inv = 1.f / l;
      __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(p.o) + (size_t)qrow * p.Hq * D + h * D;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(to + cc * 32, v);
        uint4* dst = reinterpret_cast<uint4*>(orow + cc * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf16x2(v[8 * q] * inv, v[8 * q + 1] * inv),
                              pack_bf16x2(v[8 * q + 2] * inv, v[8 * q + 3] * inv),
                              pack_bf16x2(v[8 * q + 4] * inv, v[8 * q + 5] * inv),
                              pack_bf16x2(v[8 * q + 6] * inv, v[8 * q + 7] * inv));
      }
      // natural-log LSE of the scaled logits: mrow is in log2 units
      p.lse[(size_t)h * p.T + qrow] = (mrow + log2f(l)) * 0.69314718055994531f;
    }
  }

  __syncthreads();
  if (warp == 1) {
    if (*s_abort) {
      if (lane == 0) umma_commit(drain);
      __syncwarp();
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < p.timeout_ns) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =====================================================================================
// Backward. One CTA per (128-key block j, query head h); it walks the query blocks
// i = j .. T/128-1 (causal). Per query block:
//   MMA:      S = Q_i K_j^T,  dP = dO_i V_j^T                        (TMEM)
//   compute:  P = exp2(S*c - lse*log2e) (diagonal masked), dS = P * (dP - Dsum)
//             -> P, dS (bf16) into shared memory, 128B-swizzled
//   MMA:      dV += P^T dO_i, dK += dS^T Q_i (TMEM accumulators kept across i),
//             dQ_i = dS K_j (TMEM)
//   compute:  dQ_i * scale atomically added into the fp32 dQ accumulator
// The same swizzled tiles serve as K-major operands (rows x 64 along K) and, read the
// other way, as MN-major operands (64-wide MN chunks 16 KB apart), so no transposes.
// dK / dV of the key block are accumulated over query heads with fp32 atomics.
// =====================================================================================
namespace attnb {
constexpr int TILE = 128 * 128 * 2;
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + TILE;
constexpr int OFF_Q = OFF_V + TILE;
constexpr int OFF_DO = OFF_Q + TILE;
constexpr int OFF_P = OFF_DO + TILE;
constexpr int OFF_DS = OFF_P + TILE;
constexpr int OFF_BAR = OFF_DS + TILE;
// kv_full, qo_full, qo_empty, sdp_full, pds_full, dq_full, s_free, done, drain
constexpr int NBAR = 9;
constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
constexpr int SMEM = 1024 + OFF_MISC + 16;
}  // namespace attnb

__global__ void __launch_bounds__(192, 1)
    attention_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                         AttnBwdParams p) {
  using namespace attnb;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qo_full = bars + 1;
  uint64_t* qo_empty = bars + 2;
  uint64_t* sdp_full = bars + 3;
  uint64_t* pds_full = bars + 4;
  uint64_t* dq_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* done = bars + 7;
  uint64_t* drain = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = p.T / 128;
  const int j = (int)(blockIdx.x / p.Hq);  // small j = most query blocks: launched first
  const int h = blockIdx.x % p.Hq;
  const int hk = h / (p.Hq / p.Hkv);
  const int nit = nqb - j;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(qo_full, 1);
    mbar_init(qo_empty, 1);
    mbar_init(sdp_full, 1);
    mbar_init(pds_full, 4);
    mbar_init(dq_full, 1);
    mbar_init(s_free, 4);
    mbar_init(done, 1);
    mbar_init(drain, 1);
    *s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_dv = tmem, t_dk = tmem + 128, t_s = tmem + 256, t_dp = tmem + 384;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      tma_prefetch_desc(&tmDO);
      mbar_arrive_expect_tx(kv_full, 2 * TILE);
      tma_load_2d(smem + OFF_K, &tmK, kv_full, hk * 128, j * 128);
      tma_load_2d(smem + OFF_K + TILE / 2, &tmK, kv_full, hk * 128 + 64, j * 128);
      tma_load_2d(smem + OFF_V, &tmV, kv_full, hk * 128, j * 128);
      tma_load_2d(smem + OFF_V + TILE / 2, &tmV, kv_full, hk * 128 + 64, j * 128);
      for (int it = 0; it < nit; ++it) {
        const int i = j + it;
        if (!mbar_wait_bounded(qo_empty, (it & 1) ^ 1, s_abort, p.status, p.timeout_ns)) break;
        mbar_arrive_expect_tx(qo_full, 2 * TILE);
        tma_load_2d(smem + OFF_Q, &tmQ, qo_full, h * 128, i * 128);
        tma_load_2d(smem + OFF_Q + TILE / 2, &tmQ, qo_full, h * 128 + 64, i * 128);
        tma_load_2d(smem + OFF_DO, &tmDO, qo_full, h * 128, i * 128);
        tma_load_2d(smem + OFF_DO + TILE / 2, &tmDO, qo_full, h * 128 + 64, i * 128);
      }
    }
  } else if (warp == 1) {
    constexpr uint32_t id_kk = make_idesc_bf16(128, 128, false, false);  // K-major A and B
    constexpr uint32_t id_mm = make_idesc_bf16(128, 128, true, true);    // MN-major A and B
    constexpr uint32_t id_km = make_idesc_bf16(128, 128, false, true);   // K-major A, MN-major B
    const uint32_t sk = smem_u32(smem + OFF_K), sv = smem_u32(smem + OFF_V);
    const uint32_t sq = smem_u32(smem + OFF_Q), sdo = smem_u32(smem + OFF_DO);
    const uint32_t sp = smem_u32(smem + OFF_P), sds = smem_u32(smem + OFF_DS);
    bool ok = mbar_wait_bounded(kv_full, 0, s_abort, p.status, p.timeout_ns);
    for (int it = 0; it < nit && ok; ++it) {
      if (!mbar_wait_bounded(qo_full, it & 1, s_abort, p.status, p.timeout_ns)) break;
      if (!mbar_wait_bounded(s_free, (it & 1) ^ 1, s_abort, p.status, p.timeout_ns)) break;
      tc_fence_after();
      if (lane == 0) {
        // S = Q K^T and dP = dO V^T (K-major operands, K = head dim in two 64-wide halves)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t o = kb * (TILE / 2) + kk * 32;
            const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
            umma_bf16(t_s, make_smem_desc_sw128(sq + o, 16, 1024), make_smem_desc_sw128(sk + o, 16, 1024), id_kk, acc);
            umma_bf16(t_dp, make_smem_desc_sw128(sdo + o, 16, 1024), make_smem_desc_sw128(sv + o, 16, 1024), id_kk,
                      acc);
          }
        umma_commit(sdp_full);
      }
      __syncwarp();
      if (!mbar_wait_bounded(pds_full, it & 1, s_abort, p.status, p.timeout_ns)) break;
      tc_fence_after();
      if (lane == 0) {
        // dV += P^T dO, dK += dS^T Q: MN-major (K = 128 query rows, 16 per instruction)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          umma_bf16(t_dv, make_smem_desc_sw128(sp + kk * 2048, TILE / 2, 1024),
                    make_smem_desc_sw128(sdo + kk * 2048, TILE / 2, 1024), id_mm, acc);
          umma_bf16(t_dk, make_smem_desc_sw128(sds + kk * 2048, TILE / 2, 1024),
                    make_smem_desc_sw128(sq + kk * 2048, TILE / 2, 1024), id_mm, acc);
        }
        // dQ = dS K: K-major dS (K = keys), MN-major K tile (N = head dim)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(t_s, make_smem_desc_sw128(sds + kb * (TILE / 2) + kk * 32, 16, 1024),
                      make_smem_desc_sw128(sk + (kb * 4 + kk) * 2048, TILE / 2, 1024), id_km,
                      (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(dq_full);
        umma_commit(qo_empty);
        if (it == nit - 1) umma_commit(done);
      }
      __syncwarp();
    }
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q4 * 32) << 16;
    const float c = p.scale_log2;
    bool ok = true;
    for (int it = 0; it < nit && ok; ++it) {
      const int i = j + it;
      const int qrow = i * 128 + r;
      const float lse2 = p.lse[(size_t)h * p.T + qrow] * 1.4426950408889634f;
      const float dsum = p.dsum[(size_t)h * p.T + qrow];
      if (!mbar_wait_bounded(sdp_full, it & 1, s_abort, p.status, p.timeout_ns)) { ok = false; break; }
      tc_fence_after();
      uint8_t* spp = smem + OFF_P;
      uint8_t* sdd = smem + OFF_DS;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {  // 32 keys at a time
        float sv[32], dp[32];
        tmem_ld32(t_s + lane_off + cc * 32, sv);
        tmem_ld32(t_dp + lane_off + cc * 32, dp);
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {
          float pp[8], ds[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int key = cc * 32 + q8 * 8 + e;
            const bool masked = (i == j) && (key > r);
            pp[e] = masked ? 0.f : exp2f(sv[q8 * 8 + e] * c - lse2);
            ds[e] = pp[e] * (dp[q8 * 8 + e] - dsum);
          }
          const int ch = cc * 4 + q8;
          const int half = ch >> 3, c8 = ch & 7;
          const int off = half * (TILE / 2) + r * 128 + ((c8 ^ (r & 7)) * 16);
          *reinterpret_cast<uint4*>(spp + off) = make_uint4(pack_bf16x2(pp[0], pp[1]), pack_bf16x2(pp[2], pp[3]),
                                                            pack_bf16x2(pp[4], pp[5]), pack_bf16x2(pp[6], pp[7]));
          *reinterpret_cast<uint4*>(sdd + off) = make_uint4(pack_bf16x2(ds[0], ds[1]), pack_bf16x2(ds[2], ds[3]),
                                                            pack_bf16x2(ds[4], ds[5]), pack_bf16x2(ds[6], ds[7]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_full);
      if (!mbar_wait_bounded(dq_full, it & 1, s_abort, p.status, p.timeout_ns)) { ok = false; break; }
      tc_fence_after();
      float4* dq = reinterpret_cast<float4*>(p.dq_acc + ((size_t)qrow * p.Hq + h) * 128);
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(t_s + lane_off + cc * 32, v);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          atomicAdd(dq + cc * 8 + q, make_float4(v[4 * q] * p.scale, v[4 * q + 1] * p.scale, v[4 * q + 2] * p.scale,
                                                 v[4 * q + 3] * p.scale));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
    }
    // dK (scaled) and dV of this key block: TMEM lanes are keys here
    if (ok && mbar_wait_bounded(done, 0, s_abort, p.status, p.timeout_ns)) {
      tc_fence_after();
      const int krow = j * 128 + r;
      float4* dk = reinterpret_cast<float4*>(p.dk_acc + ((size_t)krow * p.Hkv + hk) * 128);
      float4* dv = reinterpret_cast<float4*>(p.dv_acc + ((size_t)krow * p.Hkv + hk) * 128);
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        float a[32], b[32];
        tmem_ld32(t_dk + lane_off + cc * 32, a);
        tmem_ld32(t_dv + lane_off + cc * 32, b);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          atomicAdd(dk + cc * 8 + q, make_float4(a[4 * q] * p.scale, a[4 * q + 1] * p.scale, a[4 * q + 2] * p.scale,
                                                 a[4 * q + 3] * p.scale));
          atomicAdd(dv + cc * 8 + q, make_float4(b[4 * q], b[4 * q + 1], b[4 * q + 2], b[4 * q + 3]));
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    if (*s_abort) {
      if (lane == 0) umma_commit(drain);
      __syncwarp();
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(drain, 0) && globaltimer_ns() - t0 < p.timeout_ns) {
      }
    }
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Dsum[h][t] = sum_d dO[t, h, d] * O[t, h, d]  (one warp per (t, h))
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                    float* __restrict__ dsum, int T, int Hq) {
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (gw >= T * Hq) return;
  const int t = gw / Hq, h = gw % Hq;
  const size_t base = ((size_t)t * Hq + h) * 128 + lane * 4;
  const uint2 a = *reinterpret_cast<const uint2*>(o + base);
  const uint2 b = *reinterpret_cast<const uint2*>(dout + base);
  const float2 a0 = unpack_bf16x2(a.x), a1 = unpack_bf16x2(a.y), b0 = unpack_bf16x2(b.x), b1 = unpack_bf16x2(b.y);
  float s = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) dsum[(size_t)h * T + t] = s;
}

// fp32 accumulators -> bf16 gradients
__global__ void f32_to_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(in)[i];
    reinterpret_cast<uint2*>(out)[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

// =====================================================================================
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  // driver call: bind the device's primary context on this thread first (see grouped_gemm.cu)
  static thread_local bool bound = false;
  if (!bound) {
    cudaFree(nullptr);
    bound = true;
  }
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !ptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

static CUtensorMap tmap_2d(const void* base, int64_t rows, int64_t cols, int box_rows) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((cols * 2) & 15))
    throw std::runtime_error("attention operands must be 16-byte aligned");
  CUresult r = encode_fn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return tm;
}

void attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int T, int Hq, int Hkv,
                   float scale, int* status, cudaStream_t st) {
  using namespace attn;
  if (T % BQ) throw std::runtime_error("attention: sequence length must be a multiple of 128");
  if (Hq % Hkv) throw std::runtime_error("attention: query heads must be a multiple of kv heads");
  CUtensorMap tq = tmap_2d(q, T, (int64_t)Hq * D, BQ);
  CUtensorMap tk = tmap_2d(k, T, (int64_t)Hkv * D, BKV);
  CUtensorMap tv = tmap_2d(v, T, (int64_t)Hkv * D, 64);
  AttnParams p;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.lse = lse;
  p.status = status;
  static unsigned long long smem_devices = 0;
  smem_optin_once(attention_fwd_kernel, SMEM, smem_devices);
  attention_fwd_kernel<<<(T / BQ) * Hq, kThreads, SMEM, st>>>(tq, tk, tv, p);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("attention_fwd launch: ") + cudaGetErrorString(e));
}

void attention_fwd_pp(const void* q, const void* k, const void* v, void* o, float* lse, int T, int Hq, int Hkv,
                      float scale, int* status, cudaStream_t st, long long* trace) {
  using namespace attn2;
  if (T % BQ) throw std::runtime_error("attention: sequence length must be a multiple of 128");
  if (Hq % Hkv) throw std::runtime_error("attention: query heads must be a multiple of kv heads");
  CUtensorMap tq = tmap_2d(q, T, (int64_t)Hq * D, BQ);
  CUtensorMap tk = tmap_2d(k, T, (int64_t)Hkv * D, BKV);
  CUtensorMap tv = tmap_2d(v, T, (int64_t)Hkv * D, 64);
  AttnParams p;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = o;
  p.lse = lse;
  p.status = status;
  p.trace = trace;
  static unsigned long long smem_devices = 0;
  smem_optin_once(attention_fwd_pp_kernel, SMEM, smem_devices);
  attention_fwd_pp_kernel<<<((T / BQ + 1) / 2) * Hq, kThreads, SMEM, st>>>(tq, tk, tv, p);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("attention_fwd_pp launch: ") + cudaGetErrorString(e));
}

void attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
                   float* dsum, float* dq_acc, float* dk_acc, float* dv_acc, void* dq, void* dk, void* dv, int T,
                   int Hq, int Hkv, float scale, int* status, cudaStream_t st) {
  using namespace attnb;
  if (T % 128) throw std::runtime_error("attention: sequence length must be a multiple of 128");
  if (Hq % Hkv) throw std::runtime_error("attention: query heads must be a multiple of kv heads");
  const size_t nq = (size_t)T * Hq * 128, nk = (size_t)T * Hkv * 128;
  cudaMemsetAsync(dq_acc, 0, nq * 4, st);
  cudaMemsetAsync(dk_acc, 0, nk * 4, st);
  cudaMemsetAsync(dv_acc, 0, nk * 4, st);
  const int warps = T * Hq;
  attn_bwd_pre_kernel<<<(warps + 7) / 8, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(o),
                                                       reinterpret_cast<const __nv_bfloat16*>(dout), dsum, T, Hq);
  note_launch();
  CUtensorMap tq = tmap_2d(q, T, (int64_t)Hq * 128, 128);
  CUtensorMap tk = tmap_2d(k, T, (int64_t)Hkv * 128, 128);
  CUtensorMap tv = tmap_2d(v, T, (int64_t)Hkv * 128, 128);
  CUtensorMap tdo = tmap_2d(dout, T, (int64_t)Hq * 128, 128);
  AttnBwdParams p;
  p.T = T;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse = lse;
  p.dsum = dsum;
  p.dq_acc = dq_acc;
  p.dk_acc = dk_acc;
  p.dv_acc = dv_acc;
  p.status = status;
  static unsigned long long smem_devices = 0;
  smem_optin_once(attention_bwd_kernel, SMEM, smem_devices);
  attention_bwd_kernel<<<(T / 128) * Hq, 192, SMEM, st>>>(tq, tk, tv, tdo, p);
  note_launch();
  f32_to_bf16_kernel<<<1184, 256, 0, st>>>(dq_acc, reinterpret_cast<__nv_bfloat16*>(dq), nq / 4);
  f32_to_bf16_kernel<<<1184, 256, 0, st>>>(dk_acc, reinterpret_cast<__nv_bfloat16*>(dk), nk / 4);
  f32_to_bf16_kernel<<<1184, 256, 0, st>>>(dv_acc, reinterpret_cast<__nv_bfloat16*>(dv), nk / 4);
  note_launch();
  note_launch();
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("attention_bwd launch: ") + cudaGetErrorString(e));
}

}  // namespace sepx
