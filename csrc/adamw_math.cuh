// AdamW element math shared by the standalone optimizer kernels (elementwise.cu) and the
// fused weight-gradient + optimizer GEMM epilogue (grouped_gemm.cu), so both paths produce
// the same parameters bit for bit.
//
// State kinds:
//   kOptFp32: fp32 master weight, fp32 first/second moments; bf16 weight = round(master).
//   kOpt8bit: block-wise 8-bit moments, one block = 32 consecutive elements with its own
//             fp32 absmax scale per moment (block-wise quantisation, Dettmers et al.,
//             ICLR 2022): m as int8 (linear, +-127), v as uint8 of sqrt(v) (0..255).
//             No master copy: the bf16 weight is updated with stochastic rounding.
//
// Every operation is an explicitly rounded intrinsic or a fixed hardware approximation
// (sqrt.approx.ftz / rcp.approx.ftz), never left to compiler contraction, so any kernel that
// applies the update gets the same bits.
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

// Stochastic rounding to bf16: add 16 uniform random bits below the kept mantissa, truncate.
__device__ __forceinline__ uint32_t bf16_bits_stochastic(float x, uint32_t rnd16) {
  return (__float_as_uint(x) + rnd16) >> 16;
}

// One 32-bit hash per element pair (2p, 2p + 1): the even element takes the low 16 bits,
// the odd element the high 16 bits.
__device__ __forceinline__ uint32_t opt_rand_pair(uint64_t pair, const OptHyper& h) {
  return opt_hash32((uint32_t)pair ^ ((uint32_t)(pair >> 32) * 0x27d4eb2du) ^ (h.step * 0x9E3779B9u) ^ h.seed);
}
__device__ __forceinline__ uint32_t opt_rand16(uint64_t gi, const OptHyper& h) {
  const uint32_t r = opt_rand_pair(gi >> 1, h);
  return (gi & 1) ? (r >> 16) : (r & 0xFFFFu);
}

__device__ __forceinline__ float sqrt_approx(float x) {
  float y;
  asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Per-launch constants of one AdamW step. bc1 = 1 / (1 - beta1^t),
// bc2 = sqrt(1 / (1 - beta2^t)); grad_scale is folded into the moment coefficients.
struct AdamCoef {
  float b1, c1, b2, c2, bc2, eps, lr_bc1, decay;
};

__device__ __forceinline__ AdamCoef adam_coef(const OptHyper& h) {
  AdamCoef k;
  k.b1 = h.beta1;
  k.c1 = __fmul_rn(__fsub_rn(1.f, h.beta1), h.grad_scale);
  k.b2 = h.beta2;
  k.c2 = __fmul_rn(__fmul_rn(__fsub_rn(1.f, h.beta2), h.grad_scale), h.grad_scale);
  k.bc2 = h.bc2;
  k.eps = h.eps;
  k.lr_bc1 = __fmul_rn(h.lr, h.bc1);
  k.decay = __fsub_rn(1.f, __fmul_rn(h.lr, h.weight_decay));
  return k;
}

// w <- w (1 - lr wd) - lr m_hat / (sqrt(v_hat) + eps), with m, v updated in place and
// sq = sqrt(v) returned for the 8-bit encoder.
__device__ __forceinline__ float adamw_step_elem(float w, float g, float& m, float& v, float& sq, const AdamCoef& k) {
  m = __fmaf_rn(k.b1, m, __fmul_rn(k.c1, g));
  v = __fmaf_rn(k.b2, v, __fmul_rn(__fmul_rn(k.c2, g), g));
  sq = sqrt_approx(v);
  const float r = rcp_approx(__fmaf_rn(sq, k.bc2, k.eps));
  return __fmaf_rn(-k.lr_bc1, __fmul_rn(m, r), __fmul_rn(w, k.decay));
}

// ---------------------------------------------------------------------------------------
// 8-bit block codec: m = q_m * mmax / 127, sqrt(v) = q_v * vmax / 255. Integer <-> float
// conversions use the exponent-bias trick (2^23 + n has integer n in its low mantissa
// bits), which keeps them on the FMA/ALU pipes; results equal (float)n and
// __float2int_rn / __float2int_ru exactly.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float dec_scale_m(float mmax) { return __fdividef(mmax, 127.f); }
__device__ __forceinline__ float dec_scale_v(float vmax) { return __fdividef(vmax, 255.f); }
// byte e of a word of int8 codes, pre-flipped by 0x80808080 (so the byte is q + 128)
__device__ __forceinline__ float m_code_to_float(uint32_t word_x80, int e) {
  return __fsub_rn(__uint_as_float(__byte_perm(word_x80, 0x4Bu, 0x4550 | e)), 8388736.f);  // 2^23 + 128
}
__device__ __forceinline__ float v_code_to_float(uint32_t word, int e) {
  return __fsub_rn(__uint_as_float(__byte_perm(word, 0x4Bu, 0x4550 | e)), 8388608.f);  // 2^23
}
__device__ __forceinline__ float dec_m(float code, float dm) { return __fmul_rn(code, dm); }
__device__ __forceinline__ float dec_v(float code, float dv) {
  const float s = __fmul_rn(code, dv);
  return __fmul_rn(s, s);
}
// Encoder factors: 0 for an all-zero block (every code is then 0).
__device__ __forceinline__ float enc_scale_m(float mmax) { return mmax > 0.f ? __fdividef(127.f, mmax) : 0.f; }
__device__ __forceinline__ float enc_scale_v(float vmax) { return vmax > 0.f ? __fdividef(255.f, vmax) : 0.f; }
// round-to-nearest-even int8 code in the low byte (two's complement)
__device__ __forceinline__ uint32_t enc_m_bits(float m, float em) {
  return __float_as_uint(__fadd_rn(__fmul_rn(m, em), 12582912.f));  // 1.5 * 2^23
}
// sqrt(v) is rounded up, so a non-zero second moment never decodes to 0 (which would turn
// the next update into m / eps); the error only ever shrinks the step. Code in low byte.
__device__ __forceinline__ uint32_t enc_v_bits(float sq, float ev) {
  return __float_as_uint(__fadd_ru(fminf(__fmul_rn(sq, ev), 255.f), 8388608.f));
}

__device__ __forceinline__ float opt_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

// Two lanes update one 8-bit block of 32 consecutive elements: lane pair (2b, 2b + 1)
// holds block b, each lane 16 consecutive elements (4 units of 4) in registers; register
// slot q holds unit u = (q + rot) & 3 (elements 4u .. 4u+3 of the lane's half), so callers
// can read shared memory in a lane-rotated order without dynamic register indexing.
// g: gradients; w: bf16 pairs; mq / vq: 4 codes per word; msc / vsc: the block's scales
// (the same value on both lanes). Updated in place (new scales on both lanes);
// i0 = index of the lane's first element. Every lane of the warp must call this.
__device__ __forceinline__ void adamw_8bit_half(const float (&g)[16], uint2 (&w)[4], uint32_t (&mq)[4],
                                                uint32_t (&vq)[4], float& msc, float& vsc, uint64_t i0, int rot,
                                                const AdamCoef& k, const OptHyper& h) {
  const float dm = dec_scale_m(msc), dv = dec_scale_v(vsc);
  const uint64_t pair0 = i0 >> 1;
  float m[16], sq[16];
  float mmax = 0.f, vmax = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t u = (uint32_t)(q + rot) & 3u;
    const uint32_t mx = mq[q] ^ 0x80808080u;
    const uint32_t r0 = opt_rand_pair(pair0 + 2 * u, h), r1 = opt_rand_pair(pair0 + 2 * u + 1, h);
    const uint32_t rnd[4] = {r0 & 0xFFFFu, r0 >> 16, r1 & 0xFFFFu, r1 >> 16};
    const uint32_t wb[2] = {w[q].x, w[q].y};
    uint32_t ob[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = 4 * q + e;
      const float wv = __uint_as_float((e & 1) ? (wb[e >> 1] & 0xFFFF0000u) : (wb[e >> 1] << 16));
      m[j] = dec_m(m_code_to_float(mx, e), dm);
      float v = dec_v(v_code_to_float(vq[q], e), dv);
      const float nw = adamw_step_elem(wv, g[j], m[j], v, sq[j], k);
      ob[e] = bf16_bits_stochastic(nw, rnd[e]);
      mmax = fmaxf(mmax, fabsf(m[j]));
      vmax = fmaxf(vmax, sq[j]);
    }
    w[q] = make_uint2(__byte_perm(ob[0], ob[1], 0x5410), __byte_perm(ob[2], ob[3], 0x5410));
  }
  mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, 1));
  vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
  const float em = enc_scale_m(mmax), ev = enc_scale_v(vmax);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t a = __byte_perm(enc_m_bits(m[4 * q], em), enc_m_bits(m[4 * q + 1], em), 0x0040);
    const uint32_t b = __byte_perm(enc_m_bits(m[4 * q + 2], em), enc_m_bits(m[4 * q + 3], em), 0x0040);
    mq[q] = __byte_perm(a, b, 0x5410);
    const uint32_t c = __byte_perm(enc_v_bits(sq[4 * q], ev), enc_v_bits(sq[4 * q + 1], ev), 0x0040);
    const uint32_t d = __byte_perm(enc_v_bits(sq[4 * q + 2], ev), enc_v_bits(sq[4 * q + 3], ev), 0x0040);
    vq[q] = __byte_perm(c, d, 0x5410);
  }
  msc = mmax;
  vsc = vmax;
}

// One warp updates U blocks of 32 consecutive elements; lane l owns element idx[u], and
// the 32 lanes of one u cover one whole quantisation block (idx[u] - lane is a multiple
// of 32). Every lane of the warp must call this (it uses warp shuffles). Same results as
// adamw_8bit_half and the fp32 kernel in elementwise.cu.
template <int U>
__device__ __forceinline__ void adamw_warp_blocks(const float (&g)[U], const size_t (&idx)[U], const OptHyper& h) {
  const int lane = threadIdx.x & 31;
  const AdamCoef k = adam_coef(h);
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
      w[u] = adamw_step_elem(w[u], g[u], m[u], v[u], sq, k);
      h.master[idx[u]] = w[u];
      mm[idx[u]] = m[u];
      vv[idx[u]] = v[u];
      h.param[idx[u]] = __float2bfloat16(w[u]);
    }
    return;
  }
  uint8_t* mq = reinterpret_cast<uint8_t*>(h.m);
  uint8_t* vq = reinterpret_cast<uint8_t*>(h.v);
  float msc[U], vsc[U], wv[U];
  uint32_t mi[U], vi[U];
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
    float m = dec_m(m_code_to_float(mi[u] ^ 0x80u, 0), dec_scale_m(msc[u]));
    float v = dec_v(v_code_to_float(vi[u], 0), dec_scale_v(vsc[u]));
    float sq;
    const float w = adamw_step_elem(wv[u], g[u], m, v, sq, k);
    h.param[idx[u]] = __ushort_as_bfloat16((unsigned short)bf16_bits_stochastic(w, opt_rand16(idx[u], h)));
    const float mmax = opt_warp_max(fabsf(m));
    const float vmax = opt_warp_max(sq);
    mq[idx[u]] = (uint8_t)(enc_m_bits(m, enc_scale_m(mmax)) & 0xFFu);
    vq[idx[u]] = (uint8_t)(enc_v_bits(sq, enc_scale_v(vmax)) & 0xFFu);
    if (lane == 0) {
      h.m_scale[idx[u] >> 5] = mmax;
      h.v_scale[idx[u] >> 5] = vmax;
    }
  }
}

}  // namespace sepx
