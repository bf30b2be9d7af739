// AdamW update of 32-element blocks (one warp, one element per lane), shared by the standalone optimizer kernels
// (elementwise.cu) and the fused weight-gradient + optimizer GEMM epilogue
// (grouped_gemm.cu), so both paths produce the same parameters.
//
// State kinds:
//   kOptFp32: fp32 master weight, fp32 first/second moments; bf16 weight = round(master).
//   kOpt8bit: block-wise 8-bit moments, one block = 32 consecutive elements with its own
//             fp32 absmax scale per moment (block-wise quantisation, Dettmers et al.,
//             ICLR 2022): m as int8 (linear, +-127), v as uint8 of sqrt(v) (0..255).
//             No master copy: the bf16 weight is updated with stochastic rounding.
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "opt_hyper.h"
#include "sm100.cuh"

namespace sepx {

__device__ __forceinline__ uint32_t opt_hash32(uint32_t x) {
  // integer finaliser of MurmurHash3 (fmix32)
  x ^= x >> 16;
  x *= 0x85ebca6bu;
  x ^= x >> 13;
  x *= 0xc2b2ae35u;
  x ^= x >> 16;
  return x;
}

// Stochastic rounding to bf16: add uniform random bits below the kept mantissa, truncate.
__device__ __forceinline__ uint32_t bf16_bits_stochastic(float x, uint32_t rnd) {
  uint32_t u = __float_as_uint(x);
  u += (rnd & 0xFFFFu);
  return u >> 16;
}

// sqrt through the hardware reciprocal square root (rsqrtf); exact 0 for x <= 0.
__device__ __forceinline__ float opt_sqrt(float x) { return x > 0.f ? __fmul_rn(x, rsqrtf(x)) : 0.f; }

// All arithmetic below uses explicitly rounded operations and fixed intrinsics (never
// contracted into FMAs), so every kernel that applies this update gives bit-identical
// results. h.bc2 holds sqrt(1 / (1 - beta2^step)).
__device__ __forceinline__ float adamw_step_elem(float w, float g, float& m, float& v, float& sq, const OptHyper& h) {
  m = __fadd_rn(__fmul_rn(h.beta1, m), __fmul_rn(1.f - h.beta1, g));
  v = __fadd_rn(__fmul_rn(h.beta2, v), __fmul_rn(__fmul_rn(1.f - h.beta2, g), g));
  sq = opt_sqrt(v);
  const float denom = __fadd_rn(__fmul_rn(sq, h.bc2), h.eps);
  const float upd = __fdividef(__fmul_rn(m, h.bc1), denom);
  return __fsub_rn(__fmul_rn(w, 1.f - h.lr * h.weight_decay), __fmul_rn(h.lr, upd));
}

__device__ __forceinline__ uint32_t opt_rand(uint64_t gi, const OptHyper& h) {
  return opt_hash32((uint32_t)gi ^ ((uint32_t)(gi >> 32) * 0x27d4eb2du) ^ (h.step * 0x9E3779B9u) ^ h.seed);
}

// 8-bit block codec: m in [-127, 127] * mmax / 127, sqrt(v) in [0, 255] * vmax / 255.
__device__ __forceinline__ float dec_m(int q, float scale) { return __fmul_rn((float)q, __fdividef(scale, 127.f)); }
__device__ __forceinline__ float dec_v(int q, float scale) {
  const float s = __fmul_rn((float)q, __fdividef(scale, 255.f));
  return __fmul_rn(s, s);
}
// sqrt(v) is rounded up: a non-zero second moment never decodes to 0 (which would turn
// the next update into m / eps); the error only ever shrinks the step.
__device__ __forceinline__ int enc_m(float m, float mmax) {
  return mmax > 0.f ? __float2int_rn(__fmul_rn(m, __fdividef(127.f, mmax))) : 0;
}
__device__ __forceinline__ int enc_v(float sq, float vmax) {
  return vmax > 0.f ? min(255, __float2int_ru(__fmul_rn(sq, __fdividef(255.f, vmax)))) : 0;
}

__device__ __forceinline__ float opt_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

// One thread updates one block of 32 consecutive elements [idx, idx + 32), idx % 32 == 0.
__device__ __forceinline__ void adamw_block32(const float (&g)[32], size_t idx, const OptHyper& h) {
  __nv_bfloat16* p = h.param + idx;
  if (h.kind == kOptFp32) {
    float* ms = h.master + idx;
    float* mm = reinterpret_cast<float*>(h.m) + idx;
    float* vv = reinterpret_cast<float*>(h.v) + idx;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 w4 = reinterpret_cast<const float4*>(ms)[q];
      float4 m4 = reinterpret_cast<const float4*>(mm)[q];
      float4 v4 = reinterpret_cast<const float4*>(vv)[q];
      float w[4] = {w4.x, w4.y, w4.z, w4.w}, m[4] = {m4.x, m4.y, m4.z, m4.w}, v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float sq;
        w[e] = adamw_step_elem(w[e], __fmul_rn(g[4 * q + e], h.grad_scale), m[e], v[e], sq, h);
      }
      reinterpret_cast<float4*>(ms)[q] = make_float4(w[0], w[1], w[2], w[3]);
      reinterpret_cast<float4*>(mm)[q] = make_float4(m[0], m[1], m[2], m[3]);
      reinterpret_cast<float4*>(vv)[q] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<uint2*>(p)[q] = make_uint2(pack_bf16x2(w[0], w[1]), pack_bf16x2(w[2], w[3]));
    }
    return;
  }
  int8_t* mq = reinterpret_cast<int8_t*>(h.m) + idx;
  uint8_t* vq = reinterpret_cast<uint8_t*>(h.v) + idx;
  const size_t blk = idx >> 5;
  // issue every load of the block before any arithmetic
  const float msc = h.m_scale[blk], vsc = h.v_scale[blk];
  uint4 mraw[2] = {reinterpret_cast<const uint4*>(mq)[0], reinterpret_cast<const uint4*>(mq)[1]};
  uint4 vraw[2] = {reinterpret_cast<const uint4*>(vq)[0], reinterpret_cast<const uint4*>(vq)[1]};
  uint4 praw[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) praw[q] = reinterpret_cast<const uint4*>(p)[q];
  const int8_t* mb = reinterpret_cast<const int8_t*>(mraw);
  const uint8_t* vb = reinterpret_cast<const uint8_t*>(vraw);
  float m[32], sq[32];
  float mmax = 0.f, vmax = 0.f;
  uint32_t pbits[16];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t pw4[4] = {praw[q].x, praw[q].y, praw[q].z, praw[q].w};
#pragma unroll
    for (int e2 = 0; e2 < 4; ++e2) {
      float2 w2 = unpack_bf16x2(pw4[e2]);
      const float wv[2] = {w2.x, w2.y};
      uint32_t outb[2];
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int e = 8 * q + 2 * e2 + s;
        m[e] = dec_m(mb[e], msc);
        float v = dec_v(vb[e], vsc);
        const float w = adamw_step_elem(wv[s], __fmul_rn(g[e], h.grad_scale), m[e], v, sq[e], h);
        outb[s] = bf16_bits_stochastic(w, opt_rand(idx + e, h));
        mmax = fmaxf(mmax, fabsf(m[e]));
        vmax = fmaxf(vmax, sq[e]);
      }
      pbits[4 * q + e2] = (outb[0] & 0xFFFFu) | (outb[1] << 16);
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
    reinterpret_cast<uint4*>(p)[q] = make_uint4(pbits[4 * q], pbits[4 * q + 1], pbits[4 * q + 2], pbits[4 * q + 3]);
  uint32_t mo[8], vo[8];
#pragma unroll
  for (int w4 = 0; w4 < 8; ++w4) {
    uint32_t a = 0, b = 0;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int e = 4 * w4 + s;
      a |= ((uint32_t)(enc_m(m[e], mmax) & 0xFF)) << (8 * s);
      b |= ((uint32_t)enc_v(sq[e], vmax)) << (8 * s);
    }
    mo[w4] = a;
    vo[w4] = b;
  }
  reinterpret_cast<uint4*>(mq)[0] = make_uint4(mo[0], mo[1], mo[2], mo[3]);
  reinterpret_cast<uint4*>(mq)[1] = make_uint4(mo[4], mo[5], mo[6], mo[7]);
  reinterpret_cast<uint4*>(vq)[0] = make_uint4(vo[0], vo[1], vo[2], vo[3]);
  reinterpret_cast<uint4*>(vq)[1] = make_uint4(vo[4], vo[5], vo[6], vo[7]);
  h.m_scale[blk] = mmax;
  h.v_scale[blk] = vmax;
}

// One warp updates U blocks of 32 consecutive elements; lane l owns element idx[u], and
// the 32 lanes of one u cover one whole quantisation block (idx[u] - lane is a multiple
// of 32). Every lane of the warp must call this (it uses warp shuffles). Same results as
// adamw_block32.
template <int U>
__device__ __forceinline__ void adamw_warp_blocks(const float (&g)[U], const size_t (&idx)[U], const OptHyper& h) {
  const int lane = threadIdx.x & 31;
  if (h.kind == kOptFp32) {
    float* mm = reinterpret_cast<float*>(h.m);
    float* vv = reinterpret_cast<float*>(h.v);
    float w[U], m[U], v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      w[u] = h.master[idx[u]];
      m[u] = mm[idx[u]];
      v[u] = vv[idx[u]];
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float sq;
      w[u] = adamw_step_elem(w[u], __fmul_rn(g[u], h.grad_scale), m[u], v[u], sq, h);
      h.master[idx[u]] = w[u];
      mm[idx[u]] = m[u];
      vv[idx[u]] = v[u];
      h.param[idx[u]] = __float2bfloat16(w[u]);
    }
    return;
  }
  int8_t* mq = reinterpret_cast<int8_t*>(h.m);
  uint8_t* vq = reinterpret_cast<uint8_t*>(h.v);
  float msc[U], vsc[U], wv[U];
  int mi[U], vi[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const size_t blk = idx[u] >> 5;
    msc[u] = h.m_scale[blk];
    vsc[u] = h.v_scale[blk];
    mi[u] = mq[idx[u]];
    vi[u] = vq[idx[u]];
    wv[u] = __bfloat162float(h.param[idx[u]]);
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    float m = dec_m(mi[u], msc[u]);
    float v = dec_v(vi[u], vsc[u]);
    float sq;
    const float w = adamw_step_elem(wv[u], __fmul_rn(g[u], h.grad_scale), m, v, sq, h);
    h.param[idx[u]] = __ushort_as_bfloat16((unsigned short)bf16_bits_stochastic(w, opt_rand(idx[u], h)));
    const float mmax = opt_warp_max(fabsf(m));
    const float vmax = opt_warp_max(sq);
    mq[idx[u]] = (int8_t)enc_m(m, mmax);
    vq[idx[u]] = (uint8_t)enc_v(sq, vmax);
    if (lane == 0) {
      h.m_scale[idx[u] >> 5] = mmax;
      h.v_scale[idx[u] >> 5] = vmax;
    }
  }
}

}  // namespace sepx
