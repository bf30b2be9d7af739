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

// Stochastic-rounding noise of the 8-bit path: one seed per 32-element block (a full hash
// of the block index, step and seed), then for pair k of the block one multiply-xorshift
// round of the Weyl sequence seed + k * golden; the even element of the pair takes the low
// 16 bits, the odd one the high 16 bits. A pure function of the element index.
__device__ __forceinline__ uint32_t opt_block_seed(uint64_t blk, const OptHyper& h) {
  return opt_hash32((uint32_t)blk ^ ((uint32_t)(blk >> 32) * 0x27d4eb2du) ^ (h.step * 0x9E3779B9u) ^ h.seed);
}
__device__ __forceinline__ uint32_t opt_pair_noise(uint32_t seed, uint32_t k) {
  const uint32_t x = seed + k * 0x9E3779B9u;
  return (x ^ (x >> 16)) * 0x85EBCA6Bu;
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
// conversions use the exponent-bias trick (2^23 + n holds the integer n in its low
// mantissa bits), which keeps them on the FMA/ALU pipes; they equal (float)n,
// __float2int_rn and __float2int_ru exactly. sqrt(v) is rounded up, so a non-zero second
// moment never decodes to 0 (which would turn the next update into m / eps); that error
// only ever shrinks the step.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float dec_scale_m(float mmax) { return __fdividef(mmax, 127.f); }
__device__ __forceinline__ float dec_scale_v(float vmax) { return __fdividef(vmax, 255.f); }
// Encoder factors: 0 for an all-zero block (every code is then 0).
__device__ __forceinline__ float enc_scale_m(float mmax) { return mmax > 0.f ? __fdividef(127.f, mmax) : 0.f; }
__device__ __forceinline__ float enc_scale_v(float vmax) { return vmax > 0.f ? __fdividef(255.f, vmax) : 0.f; }

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Moment updates of two elements (packed fp32x2): m, v in place, sq = sqrt(v).
__device__ __forceinline__ void adam_moments2(float2 g, float2& m, float2& v, float2& sq, const AdamCoef& k) {
  m = __ffma2_rn(f2(k.b1), m, __fmul2_rn(f2(k.c1), g));
  v = __ffma2_rn(f2(k.b2), v, __fmul2_rn(__fmul2_rn(f2(k.c2), g), g));
  sq = make_float2(sqrt_approx(v.x), sqrt_approx(v.y));
}

// Two elements of one AdamW step in packed fp32x2 arithmetic (sm_100 FFMA2/FMUL2).
__device__ __forceinline__ float2 adamw_step2(float2 w, float2 g, float2& m, float2& v, float2& sq,
                                              const AdamCoef& k) {
  adam_moments2(g, m, v, sq, k);
  const float2 den = __ffma2_rn(sq, f2(k.bc2), f2(k.eps));
  const float2 r = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  return __ffma2_rn(f2(-k.lr_bc1), __fmul2_rn(m, r), __fmul2_rn(w, f2(k.decay)));
}

// codes e and e+1 of a word as floats: (byte | 0x4B000000) - bias; exact
__device__ __forceinline__ float2 codes2(uint32_t word, int e, float bias) {
  return __fadd2_rn(make_float2(__uint_as_float(__byte_perm(word, 0x4Bu, 0x4550 | e)),
                                __uint_as_float(__byte_perm(word, 0x4Bu, 0x4550 | (e + 1)))),
                    f2(-bias));
}

// 8-bit update of NU units of 4 consecutive elements held in registers.
//   NU = 8: one thread holds a whole block of 32 consecutive elements.
//   NU = 4: lane pair (2b, 2b + 1) holds block b, each lane 16 consecutive elements; the
//           block maxima are combined over the pair (every lane of the warp must call).
// Register slot q holds unit u = (q + rot) & (NU - 1) (elements 4u .. 4u+3 of the
// thread's range), so callers can read shared memory in a lane-rotated order without
// dynamic register indexing. g: gradients; w: bf16 pairs; mq / vq: 4 codes per word;
// msc / vsc: the block's scales (same value on both lanes of a pair). Everything is
// updated in place; i0 = global index of the thread's first element (i0 % 16 == 0).
// Arithmetic runs on element pairs (FFMA2 / FMUL2 / FADD2), so any caller layout gives
// the same bits.
template <int NU>
__device__ __forceinline__ void adamw_8bit_units(const float (&g)[4 * NU], uint2 (&w)[NU], uint32_t (&mq)[NU],
                                                 uint32_t (&vq)[NU], float& msc, float& vsc, uint64_t i0, int rot,
                                                 const AdamCoef& k, const OptHyper& h) {
  static_assert(NU == 4 || NU == 8, "a thread holds half or all of a 32-element block");
  const float dm = dec_scale_m(msc), dv = dec_scale_v(vsc);
  const uint32_t seed = opt_block_seed(i0 >> 5, h);
  const uint32_t k0 = (uint32_t)(i0 & 31) >> 1;  // first pair of this thread within the block
  float2 m[2 * NU], sq[2 * NU];
  float mmax = 0.f, vmax = 0.f;
#pragma unroll
  for (int q = 0; q < NU; ++q) {
    const uint32_t u = (uint32_t)(q + rot) & (uint32_t)(NU - 1);
    const uint32_t mx = mq[q] ^ 0x80808080u;
    const uint32_t wb[2] = {w[q].x, w[q].y};
    uint32_t ob[2];
#pragma unroll
    for (int e2 = 0; e2 < 2; ++e2) {
      const int j = 2 * q + e2;
      const float2 wv = make_float2(__uint_as_float(wb[e2] << 16), __uint_as_float(wb[e2] & 0xFFFF0000u));
      const float2 g2 = make_float2(g[2 * j], g[2 * j + 1]);
      m[j] = __fmul2_rn(codes2(mx, 2 * e2, 8388736.f), f2(dm));  // 2^23 + 128
      const float2 s = __fmul2_rn(codes2(vq[q], 2 * e2, 8388608.f), f2(dv));
      float2 v = __fmul2_rn(s, s);
      const float2 nw = adamw_step2(wv, g2, m[j], v, sq[j], k);
      const uint32_t r = opt_pair_noise(seed, k0 + 2 * u + e2);
      ob[e2] = __byte_perm(__float_as_uint(nw.x) + (r & 0xFFFFu), __float_as_uint(nw.y) + (r >> 16), 0x7632);
      mmax = fmaxf(mmax, fmaxf(fabsf(m[j].x), fabsf(m[j].y)));
      vmax = fmaxf(vmax, fmaxf(sq[j].x, sq[j].y));
    }
    w[q] = make_uint2(ob[0], ob[1]);
  }
  if (NU == 4) {
    mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffffu, mmax, 1));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
  }
  const float em = enc_scale_m(mmax), ev = enc_scale_v(vmax);
#pragma unroll
  for (int q = 0; q < NU; ++q) {
    uint32_t mb[2], vb[2];
#pragma unroll
    for (int e2 = 0; e2 < 2; ++e2) {
      const int j = 2 * q + e2;
      // m: round to nearest even in the low byte; sqrt(v): rounded up, capped at 255
      const float2 tm = __fadd2_rn(__fmul2_rn(m[j], f2(em)), f2(12582912.f));  // 1.5 * 2^23
      float2 y = __fmul2_rn(sq[j], f2(ev));
      y = make_float2(fminf(y.x, 255.f), fminf(y.y, 255.f));
      const float2 tv = __fadd2_ru(y, f2(8388608.f));
      mb[e2] = __byte_perm(__float_as_uint(tm.x), __float_as_uint(tm.y), 0x0040);
      vb[e2] = __byte_perm(__float_as_uint(tv.x), __float_as_uint(tv.y), 0x0040);
    }
    mq[q] = __byte_perm(mb[0], mb[1], 0x5410);
    vq[q] = __byte_perm(vb[0], vb[1], 0x5410);
  }
  msc = mmax;
  vsc = vmax;
}

// fp32 state: one warp updates U rows of 32 consecutive elements, lane l owning element
// idx[u] (the fused weight-gradient epilogue's layout). Same results as the standalone
// fp32 kernel in elementwise.cu.
template <int U>
__device__ __forceinline__ void adamw_fp32_lanes(const float (&g)[U], const size_t (&idx)[U], const OptHyper& h) {
  const AdamCoef k = adam_coef(h);
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
}

}  // namespace sepx
