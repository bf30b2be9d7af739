// Memory-bound hot ops of the Qwen3-MoE block, written for sm_100a:
//   RMSNorm fwd/bwd, fused per-head q/k RMSNorm + RoPE fwd/bwd, SwiGLU fwd/bwd,
//   router softmax/top-k/renorm fwd/bwd, fused AdamW (fp32 or block-wise 8-bit state),
//   fused cross-entropy (loss + dlogits in one pass pair).
// All use 16-byte vector accesses and fp32 math; transcendental functions are CUDA's
// own intrinsics (__expf, rsqrtf, __logf).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "adamw_math.cuh"
#include "elementwise.h"
#include "kernels.h"
#include "sm100.cuh"

namespace sepx {

static void check(const char* what) {
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), c = unpack_bf16x2(v.z), d = unpack_bf16x2(v.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  unpack8(*reinterpret_cast<const uint4*>(p), f);
}
// An empty asm that claims to rewrite the registers: the compiler must unpack them again
// afterwards instead of keeping the earlier unpacked floats live (values are unchanged).
__device__ __forceinline__ void opaque(uint4& v) {
  asm volatile("" : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w));
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
  return v;
}

// =====================================================================================
// RMSNorm: y = w * x * rsqrt(mean(x^2) + eps). One warp per row; D % 256 == 0, D <= 8192.
// =====================================================================================
// With `add` (and `sum`): the input is s = x + add, rounded to bf16 as a bf16 tensor add
// rounds it, and s is written to `sum` (the residual stream) before it is normalised.
template <int VPL>  // 8-element vectors per lane
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          __nv_bfloat16* __restrict__ y, float* __restrict__ rstd,
                                                          int N, int D, float eps,
                                                          const __nv_bfloat16* __restrict__ add = nullptr,
                                                          __nv_bfloat16* __restrict__ sum = nullptr) {
  const int lane = threadIdx.x & 31;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= N) return;
  float v[VPL][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const size_t off = (size_t)row * D + (i * 32 + lane) * 8;
    load8(x + off, v[i]);
    if (add) {
      float a[8];
      load8(add + off, a);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = __bfloat162float(__float2bfloat16(v[i][e] + a[e]));
      store8(sum + off, v[i]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += v[i][e] * v[i][e];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / D + eps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    float wv[8], o[8];
    load8(w + (i * 32 + lane) * 8, wv);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = v[i][e] * r * wv[e];
    store8(y + (size_t)row * D + (i * 32 + lane) * 8, o);
  }
}

// dx = r * (w*dy - xhat * mean(xhat * w*dy)); dw += sum_rows dy * xhat (fp32, per-block
// reduction in shared memory then one atomicAdd per element per block).
template <int VPL>
__global__ void __launch_bounds__(256, 2) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const float* __restrict__ rstd,
                                                          const __nv_bfloat16* __restrict__ dy,
                                                          __nv_bfloat16* __restrict__ dx, float* __restrict__ dw,
                                                          int N, int D,
                                                          const __nv_bfloat16* __restrict__ dres = nullptr) {
  extern __shared__ float s_dw[];  // [D]
  for (int i = threadIdx.x; i < D; i += blockDim.x) s_dw[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nw = gridDim.x * (blockDim.x >> 5);
  float acc[VPL][8];
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
  // Only the dw accumulators stay in registers across rows: the second pass over a row
  // reads x and dy again (L1 / L2 hits: the warp read them a moment before) and w comes
  // from L1, so a thread needs about half the registers of holding the row, and twice the
  // warps fit on an SM to hide the loads.
  for (int row = blockIdx.x * (blockDim.x >> 5) + warp; row < N; row += nw) {
    const float r = rstd[row];
    const __nv_bfloat16* xrow = x + (size_t)row * D;
    const __nv_bfloat16* grow = dy + (size_t)row * D;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      float xv[8], g[8], wv[8];
      unpack8(*reinterpret_cast<const uint4*>(xrow + (i * 32 + lane) * 8), xv);
      unpack8(*reinterpret_cast<const uint4*>(grow + (i * 32 + lane) * 8), g);
      unpack8(__ldg(reinterpret_cast<const uint4*>(w + (i * 32 + lane) * 8)), wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xh = xv[e] * r;
        acc[i][e] += g[e] * xh;
        dot += xh * (g[e] * wv[e]);
      }
    }
    dot = warp_sum(dot) / D;
    // opaque pointers: the compiler must read the row again instead of keeping the first
    // pass's values live in registers
    asm volatile("" : "+l"(xrow), "+l"(grow));
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      float xv[8], g[8], wv[8], o[8];
      unpack8(*reinterpret_cast<const uint4*>(xrow + (i * 32 + lane) * 8), xv);
      unpack8(*reinterpret_cast<const uint4*>(grow + (i * 32 + lane) * 8), g);
      unpack8(__ldg(reinterpret_cast<const uint4*>(w + (i * 32 + lane) * 8)), wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = r * (g[e] * wv[e] - (xv[e] * r) * dot);
      if (dres) {  // the input's other gradient, added as a bf16 tensor add would
        float d[8];
        load8(dres + (size_t)row * D + (i * 32 + lane) * 8, d);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = __bfloat162float(__float2bfloat16(o[e])) + d[e];
      }
      store8(dx + (size_t)row * D + (i * 32 + lane) * 8, o);
    }
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i)
#pragma unroll
    for (int e = 0; e < 8; ++e) atomicAdd(&s_dw[(i * 32 + lane) * 8 + e], acc[i][e]);
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) atomicAdd(dw + i, s_dw[i]);
}

void rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int N, int D, float eps, cudaStream_t st,
                 const void* add, void* sum) {
  if (D % 256 || D > 8192) throw std::runtime_error("rmsnorm: D must be a multiple of 256, <= 8192");
  if ((add == nullptr) != (sum == nullptr)) throw std::runtime_error("rmsnorm: add and sum go together");
  const int blocks = (N + 7) / 8;
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto Wt = reinterpret_cast<const __nv_bfloat16*>(w);
  auto Y = reinterpret_cast<__nv_bfloat16*>(y);
  auto A = reinterpret_cast<const __nv_bfloat16*>(add);
  auto S = reinterpret_cast<__nv_bfloat16*>(sum);
  switch (D / 256) {
    case 1: rmsnorm_fwd_kernel<1><<<blocks, 256, 0, st>>>(X, Wt, Y, rstd, N, D, eps, A, S); break;
    case 2: rmsnorm_fwd_kernel<2><<<blocks, 256, 0, st>>>(X, Wt, Y, rstd, N, D, eps, A, S); break;
    case 4: rmsnorm_fwd_kernel<4><<<blocks, 256, 0, st>>>(X, Wt, Y, rstd, N, D, eps, A, S); break;
    case 8: rmsnorm_fwd_kernel<8><<<blocks, 256, 0, st>>>(X, Wt, Y, rstd, N, D, eps, A, S); break;
    case 16: rmsnorm_fwd_kernel<16><<<blocks, 256, 0, st>>>(X, Wt, Y, rstd, N, D, eps, A, S); break;
    case 32: rmsnorm_fwd_kernel<32><<<blocks, 256, 0, st>>>(X, Wt, Y, rstd, N, D, eps, A, S); break;
    default: throw std::runtime_error("rmsnorm: unsupported D");
  }
  check("rmsnorm_fwd");
}

void rmsnorm_bwd(const void* x, const void* w, const float* rstd, const void* dy, void* dx, float* dw, int N, int D,
                 int num_sms, cudaStream_t st, const void* dres) {
  if (D % 256 || D > 8192) throw std::runtime_error("rmsnorm: D must be a multiple of 256, <= 8192");
  const int blocks = std::min((N + 7) / 8, num_sms * 2);
  auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto Wt = reinterpret_cast<const __nv_bfloat16*>(w);
  auto DY = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto DX = reinterpret_cast<__nv_bfloat16*>(dx);
  auto DR = reinterpret_cast<const __nv_bfloat16*>(dres);
  const size_t sm = D * sizeof(float);
  switch (D / 256) {
    case 1: rmsnorm_bwd_kernel<1><<<blocks, 256, sm, st>>>(X, Wt, rstd, DY, DX, dw, N, D, DR); break;
    case 2: rmsnorm_bwd_kernel<2><<<blocks, 256, sm, st>>>(X, Wt, rstd, DY, DX, dw, N, D, DR); break;
    case 4: rmsnorm_bwd_kernel<4><<<blocks, 256, sm, st>>>(X, Wt, rstd, DY, DX, dw, N, D, DR); break;
    case 8: rmsnorm_bwd_kernel<8><<<blocks, 256, sm, st>>>(X, Wt, rstd, DY, DX, dw, N, D, DR); break;
    default: throw std::runtime_error("rmsnorm_bwd: unsupported D");
  }
  check("rmsnorm_bwd");
}

// =====================================================================================
// Fused per-head RMSNorm + rotary embedding (rotate-half convention, Qwen3):
//   in  qkv [T, (Hq + 2*Hkv) * 128]  (output of the fused QKV projection)
//   out q [T, Hq, 128], k [T, Hkv, 128] normalised and rotated; v [T, Hkv, 128] copied.
// One warp per token: lane l owns elements i = 2l, 2l+1 and their rotate-half partners
// i + 64, so the lane's two rotation angles are computed once per token and reused by
// every q / k head; heads go in batches of kRopeBatch with all their loads issued first.
// =====================================================================================
constexpr int kRopeBatch = 4;

__device__ __forceinline__ void rope_cs(int pos, int i, float log2_theta, float* c, float* s) {
  // inv_freq_i = theta^(-2i/128), angle = pos * inv_freq
  const float inv = exp2f(-(2.f * i / 128.f) * log2_theta);
  const float ang = (float)pos * inv;
  sincosf(ang, s, c);
}

__global__ void __launch_bounds__(256) qk_norm_rope_fwd_kernel(
    const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ wq, const __nv_bfloat16* __restrict__ wk,
    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v,
    float* __restrict__ rstd_q, float* __restrict__ rstd_k, const int* __restrict__ pos_ids, int T, int Hq, int Hkv,
    float eps, float log2_theta) {
  const int lane = threadIdx.x & 31;
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  const int Ht = Hq + 2 * Hkv;
  const int pos = pos_ids ? pos_ids[t] : t;
  float c0, s0, c1, s1;
  rope_cs(pos, 2 * lane, log2_theta, &c0, &s0);
  rope_cs(pos, 2 * lane + 1, log2_theta, &c1, &s1);
  const float2 wql = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wq)[lane]);
  const float2 wqh = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wq + 64)[lane]);
  const float2 wkl = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wk)[lane]);
  const float2 wkh = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wk + 64)[lane]);
  const __nv_bfloat162* row = reinterpret_cast<const __nv_bfloat162*>(qkv + (size_t)t * Ht * 128);
  for (int h0 = 0; h0 < Ht; h0 += kRopeBatch) {
    __nv_bfloat162 lo[kRopeBatch], hi[kRopeBatch];
#pragma unroll
    for (int b = 0; b < kRopeBatch; ++b) {
      const int h = min(h0 + b, Ht - 1);
      lo[b] = row[h * 64 + lane];
      hi[b] = row[h * 64 + 32 + lane];
    }
#pragma unroll
    for (int b = 0; b < kRopeBatch; ++b) {
      const int h = h0 + b;
      if (h >= Ht) break;
      const float2 l = __bfloat1622float2(lo[b]), u = __bfloat1622float2(hi[b]);
      if (h >= Hq + Hkv) {  // value head: plain copy
        __nv_bfloat162* dst = reinterpret_cast<__nv_bfloat162*>(v + ((size_t)t * Hkv + (h - Hq - Hkv)) * 128);
        dst[lane] = lo[b];
        dst[32 + lane] = hi[b];
        continue;
      }
      const bool is_q = h < Hq;
      const float2 wl = is_q ? wql : wkl, wh = is_q ? wqh : wkh;
      const float r = rsqrtf(warp_sum(l.x * l.x + l.y * l.y + u.x * u.x + u.y * u.y) / 128.f + eps);
      const float a0 = l.x * r * wl.x, a1 = l.y * r * wl.y, b0 = u.x * r * wh.x, b1 = u.y * r * wh.y;
      // out_lo = a*cos - b*sin ; out_hi = b*cos + a*sin
      const float o0 = a0 * c0 - b0 * s0, o1 = a1 * c1 - b1 * s1;
      const float p0 = b0 * c0 + a0 * s0, p1 = b1 * c1 + a1 * s1;
      __nv_bfloat162* dst;
      if (is_q) {
        dst = reinterpret_cast<__nv_bfloat162*>(q + ((size_t)t * Hq + h) * 128);
        if (lane == 0) rstd_q[(size_t)t * Hq + h] = r;
      } else {
        dst = reinterpret_cast<__nv_bfloat162*>(k + ((size_t)t * Hkv + (h - Hq)) * 128);
        if (lane == 0) rstd_k[(size_t)t * Hkv + (h - Hq)] = r;
      }
      dst[lane] = __floats2bfloat162_rn(o0, o1);
      dst[32 + lane] = __floats2bfloat162_rn(p0, p1);
    }
  }
}

// Backward: dq/dk (post-rotation) -> un-rotate -> RMSNorm backward -> dqkv; dv copied.
// dwq/dwk accumulate per-element weight gradients (fp32). One warp per token (grid-stride
// over tokens), heads in batches as in the forward.
__global__ void __launch_bounds__(256) qk_norm_rope_bwd_kernel(
    const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ wq, const __nv_bfloat16* __restrict__ wk,
    const float* __restrict__ rstd_q, const float* __restrict__ rstd_k, const __nv_bfloat16* __restrict__ dq,
    const __nv_bfloat16* __restrict__ dk, const __nv_bfloat16* __restrict__ dv, __nv_bfloat16* __restrict__ dqkv,
    float* __restrict__ dwq, float* __restrict__ dwk, const int* __restrict__ pos_ids, int T, int Hq, int Hkv,
    float log2_theta) {
  __shared__ float s_dw[2][128];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) (&s_dw[0][0])[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int Ht = Hq + 2 * Hkv;
  const int nw = gridDim.x * (blockDim.x >> 5);
  const float2 wql = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wq)[lane]);
  const float2 wqh = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wq + 64)[lane]);
  const float2 wkl = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wk)[lane]);
  const float2 wkh = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(wk + 64)[lane]);
  float aq[4] = {0, 0, 0, 0}, ak[4] = {0, 0, 0, 0};
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T; t += nw) {
    const int pos = pos_ids ? pos_ids[t] : t;
    float c0, s0, c1, s1;
    rope_cs(pos, 2 * lane, log2_theta, &c0, &s0);
    rope_cs(pos, 2 * lane + 1, log2_theta, &c1, &s1);
    const __nv_bfloat162* xrow = reinterpret_cast<const __nv_bfloat162*>(qkv + (size_t)t * Ht * 128);
    __nv_bfloat162* orow = reinterpret_cast<__nv_bfloat162*>(dqkv + (size_t)t * Ht * 128);
    for (int h0 = 0; h0 < Ht; h0 += kRopeBatch) {
      __nv_bfloat162 glo[kRopeBatch], ghi[kRopeBatch], xlo[kRopeBatch], xhi[kRopeBatch];
      float rr[kRopeBatch];
#pragma unroll
      for (int b = 0; b < kRopeBatch; ++b) {
        const int h = min(h0 + b, Ht - 1);
        const __nv_bfloat162* g;
        if (h < Hq) {
          g = reinterpret_cast<const __nv_bfloat162*>(dq + ((size_t)t * Hq + h) * 128);
          rr[b] = rstd_q[(size_t)t * Hq + h];
        } else if (h < Hq + Hkv) {
          g = reinterpret_cast<const __nv_bfloat162*>(dk + ((size_t)t * Hkv + (h - Hq)) * 128);
          rr[b] = rstd_k[(size_t)t * Hkv + (h - Hq)];
        } else {
          g = reinterpret_cast<const __nv_bfloat162*>(dv + ((size_t)t * Hkv + (h - Hq - Hkv)) * 128);
          rr[b] = 0.f;
        }
        glo[b] = g[lane];
        ghi[b] = g[32 + lane];
        if (h < Hq + Hkv) {
          xlo[b] = xrow[h * 64 + lane];
          xhi[b] = xrow[h * 64 + 32 + lane];
        }
      }
#pragma unroll
      for (int b = 0; b < kRopeBatch; ++b) {
        const int h = h0 + b;
        if (h >= Ht) break;
        if (h >= Hq + Hkv) {  // value head: the gradient is copied
          orow[h * 64 + lane] = glo[b];
          orow[h * 64 + 32 + lane] = ghi[b];
          continue;
        }
        const bool is_q = h < Hq;
        const float2 gl = __bfloat1622float2(glo[b]), gh = __bfloat1622float2(ghi[b]);
        const float2 lo = __bfloat1622float2(xlo[b]), hi = __bfloat1622float2(xhi[b]);
        const float r = rr[b];
        // inverse rotation: da = glo*cos + ghi*sin ; db = ghi*cos - glo*sin
        float gy[4] = {gl.x * c0 + gh.x * s0, gl.y * c1 + gh.y * s1, gh.x * c0 - gl.x * s0, gh.y * c1 - gl.y * s1};
        const float xh[4] = {lo.x * r, lo.y * r, hi.x * r, hi.y * r};
        const float2 wl = is_q ? wql : wkl, wh = is_q ? wqh : wkh;
        const float wv[4] = {wl.x, wl.y, wh.x, wh.y};
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (is_q) aq[e] += gy[e] * xh[e]; else ak[e] += gy[e] * xh[e];
          gy[e] *= wv[e];
          dot += gy[e] * xh[e];
        }
        dot = warp_sum(dot) / 128.f;
        orow[h * 64 + lane] = __floats2bfloat162_rn(r * (gy[0] - xh[0] * dot), r * (gy[1] - xh[1] * dot));
        orow[h * 64 + 32 + lane] = __floats2bfloat162_rn(r * (gy[2] - xh[2] * dot), r * (gy[3] - xh[3] * dot));
      }
    }
  }
  atomicAdd(&s_dw[0][2 * lane], aq[0]);
  atomicAdd(&s_dw[0][2 * lane + 1], aq[1]);
  atomicAdd(&s_dw[0][64 + 2 * lane], aq[2]);
  atomicAdd(&s_dw[0][64 + 2 * lane + 1], aq[3]);
  atomicAdd(&s_dw[1][2 * lane], ak[0]);
  atomicAdd(&s_dw[1][2 * lane + 1], ak[1]);
  atomicAdd(&s_dw[1][64 + 2 * lane], ak[2]);
  atomicAdd(&s_dw[1][64 + 2 * lane + 1], ak[3]);
  __syncthreads();
  for (int i = threadIdx.x; i < 128; i += blockDim.x) {
    atomicAdd(dwq + i, s_dw[0][i]);
    atomicAdd(dwk + i, s_dw[1][i]);
  }
}

void qk_norm_rope_fwd(const void* qkv, const void* wq, const void* wk, void* q, void* k, void* v, float* rstd_q,
                      float* rstd_k, const int* pos_ids, int T, int Hq, int Hkv, float eps, float theta,
                      cudaStream_t st) {
  qk_norm_rope_fwd_kernel<<<(T + 7) / 8, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), reinterpret_cast<const __nv_bfloat16*>(wq),
      reinterpret_cast<const __nv_bfloat16*>(wk), reinterpret_cast<__nv_bfloat16*>(q),
      reinterpret_cast<__nv_bfloat16*>(k), reinterpret_cast<__nv_bfloat16*>(v), rstd_q, rstd_k, pos_ids, T, Hq, Hkv,
      eps, log2f(theta));
  check("qk_norm_rope_fwd");
}

void qk_norm_rope_bwd(const void* qkv, const void* wq, const void* wk, const float* rstd_q, const float* rstd_k,
                      const void* dq, const void* dk, const void* dv, void* dqkv, float* dwq, float* dwk,
                      const int* pos_ids, int T, int Hq, int Hkv, float theta, int num_sms, cudaStream_t st) {
  const int blocks = std::max(1, std::min((T + 7) / 8, num_sms * 4));
  qk_norm_rope_bwd_kernel<<<blocks, 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv), reinterpret_cast<const __nv_bfloat16*>(wq),
      reinterpret_cast<const __nv_bfloat16*>(wk), rstd_q, rstd_k, reinterpret_cast<const __nv_bfloat16*>(dq),
      reinterpret_cast<const __nv_bfloat16*>(dk), reinterpret_cast<const __nv_bfloat16*>(dv),
      reinterpret_cast<__nv_bfloat16*>(dqkv), dwq, dwk, pos_ids, T, Hq, Hkv, log2f(theta));
  check("qk_norm_rope_bwd");
}

// =====================================================================================
// SwiGLU on a [N, 2I] gate|up tensor: h = silu(g) * u; backward gives d[g|u].
// =====================================================================================
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, int N, int I) {
  const size_t total = (size_t)N * I / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / (I / 8), c = (i % (I / 8)) * 8;
    float g[8], u[8], o[8];
    load8(gu + row * 2 * I + c, g);
    load8(gu + row * 2 * I + I + c, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __fdividef(g[e], 1.f + __expf(-g[e])) * u[e];
    store8(h + row * I + c, o);
  }
}
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                  __nv_bfloat16* __restrict__ dgu, int N, int I) {
  const size_t total = (size_t)N * I / 8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const size_t row = i / (I / 8), c = (i % (I / 8)) * 8;
    float g[8], u[8], d[8], og[8], ou[8];
    load8(gu + row * 2 * I + c, g);
    load8(gu + row * 2 * I + I + c, u);
    load8(dh + row * I + c, d);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float s = __fdividef(1.f, 1.f + __expf(-g[e]));
      og[e] = d[e] * u[e] * s * (1.f + g[e] * (1.f - s));
      ou[e] = d[e] * g[e] * s;
    }
    store8(dgu + row * 2 * I + c, og);
    store8(dgu + row * 2 * I + I + c, ou);
  }
}
void swiglu_fwd(const void* gu, void* h, int N, int I, int num_sms, cudaStream_t st) {
  if (I % 8) throw std::runtime_error("swiglu: I must be a multiple of 8");
  swiglu_fwd_kernel<<<num_sms * 8, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(gu),
                                                 reinterpret_cast<__nv_bfloat16*>(h), N, I);
  check("swiglu_fwd");
}
void swiglu_bwd(const void* gu, const void* dh, void* dgu, int N, int I, int num_sms, cudaStream_t st) {
  if (I % 8) throw std::runtime_error("swiglu: I must be a multiple of 8");
  swiglu_bwd_kernel<<<num_sms * 8, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(gu),
                                                 reinterpret_cast<const __nv_bfloat16*>(dh),
                                                 reinterpret_cast<__nv_bfloat16*>(dgu), N, I);
  check("swiglu_bwd");
}

// =====================================================================================
// Router: p = softmax(logits) (fp32), top-k, optional renormalisation over the top-k.
// One warp per token; E <= 1024 (E/32 values per lane in registers).
// =====================================================================================
template <int EPL>
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits,
                                                          const float* __restrict__ bias, int T, int E, int k,
                                                          int renorm, int* __restrict__ topk_e,
                                                          float* __restrict__ topk_w, float* __restrict__ probs) {
  const int lane = threadIdx.x & 31;
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float p[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    p[i] = e < E ? logits[(size_t)t * E + e] : -INFINITY;
    mx = fmaxf(mx, p[i]);
  }
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    p[i] = (i * 32 + lane) < E ? __expf(p[i] - mx) : 0.f;
    s += p[i];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    p[i] *= inv;
    if (probs && (i * 32 + lane) < E) probs[(size_t)t * E + i * 32 + lane] = p[i];
  }
  // selection score = p (+ optional per-expert bias, used for skewed synthetic routing)
  float sc[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    sc[i] = e < E ? p[i] + (bias ? bias[e] : 0.f) : -INFINITY;
  }
  float sel_sum = 0.f;
  int my_e = -1;
  float my_w = 0.f;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      if (sc[i] > best || (sc[i] == best && e < bi)) { best = sc[i]; bi = e; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ob = __shfl_xor_sync(0xffffffff, best, o);
      int oi = __shfl_xor_sync(0xffffffff, bi, o);
      if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    // owner lane removes it and reports its probability
    float pw = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      if (i * 32 + lane == bi) { pw = p[i]; sc[i] = -INFINITY; }
    }
    pw = warp_sum(pw);
    sel_sum += pw;
    if (lane == j) { my_e = bi; my_w = pw; }
  }
  if (lane < k) {
    topk_e[(size_t)t * k + lane] = my_e;
    topk_w[(size_t)t * k + lane] = renorm ? my_w / sel_sum : my_w;
  }
}

// Backward through renorm + softmax: dlogits[t, :] given dw[t, j] for the chosen experts.
template <int EPL>
__global__ void __launch_bounds__(256) router_bwd_kernel(const float* __restrict__ probs, const int* __restrict__ topk_e,
                                                         const float* __restrict__ dw, int T, int E, int k, int renorm,
                                                         float* __restrict__ dlogits) {
  const int lane = threadIdx.x & 31;
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  // dp_i for chosen experts
  float S = 0.f, gw = 0.f;
  int e_l = -1;
  float g_l = 0.f, p_l = 0.f;
  if (lane < k) {
    e_l = topk_e[(size_t)t * k + lane];
    g_l = dw[(size_t)t * k + lane];
    p_l = probs[(size_t)t * E + e_l];
  }
  S = warp_sum(lane < k ? p_l : 0.f);
  // with renorm: w_j = p_j / S; dL/dp_i = (g_i - sum_j g_j w_j) / S for chosen i
  gw = warp_sum(lane < k ? g_l * p_l : 0.f) / S;
  float dp_l = lane < k ? (renorm ? (g_l - gw) / S : g_l) : 0.f;
  // softmax backward: dlogit_i = p_i * (dp_i - sum_j p_j dp_j)
  float pdp = warp_sum(lane < k ? p_l * dp_l : 0.f);
  float p[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    p[i] = e < E ? probs[(size_t)t * E + e] : 0.f;
  }
  float dpv[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) dpv[i] = 0.f;
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffff, e_l, j);
    const float dj = __shfl_sync(0xffffffff, dp_l, j);
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (i * 32 + lane == ej) dpv[i] += dj;
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    if (e < E) dlogits[(size_t)t * E + e] = p[i] * (dpv[i] - pdp);
  }
}

void router_topk(const float* logits, const float* bias, int T, int E, int k, bool renorm, int* topk_e, float* topk_w,
                 float* probs, cudaStream_t st) {
  if (k > 32) throw std::runtime_error("router: top-k above 32");
  const int blocks = (T + 7) / 8;
  const int epl = (E + 31) / 32;
  if (epl <= 2) router_topk_kernel<2><<<blocks, 256, 0, st>>>(logits, bias, T, E, k, renorm, topk_e, topk_w, probs);
  else if (epl <= 4) router_topk_kernel<4><<<blocks, 256, 0, st>>>(logits, bias, T, E, k, renorm, topk_e, topk_w, probs);
  else if (epl <= 8) router_topk_kernel<8><<<blocks, 256, 0, st>>>(logits, bias, T, E, k, renorm, topk_e, topk_w, probs);
  else if (epl <= 16) router_topk_kernel<16><<<blocks, 256, 0, st>>>(logits, bias, T, E, k, renorm, topk_e, topk_w, probs);
  else throw std::runtime_error("router: at most 512 experts");
  check("router_topk");
}

void router_bwd(const float* probs, const int* topk_e, const float* dw, int T, int E, int k, bool renorm,
                float* dlogits, cudaStream_t st) {
  const int blocks = (T + 7) / 8;
  const int epl = (E + 31) / 32;
  if (epl <= 2) router_bwd_kernel<2><<<blocks, 256, 0, st>>>(probs, topk_e, dw, T, E, k, renorm, dlogits);
  else if (epl <= 4) router_bwd_kernel<4><<<blocks, 256, 0, st>>>(probs, topk_e, dw, T, E, k, renorm, dlogits);
  else if (epl <= 8) router_bwd_kernel<8><<<blocks, 256, 0, st>>>(probs, topk_e, dw, T, E, k, renorm, dlogits);
  else if (epl <= 16) router_bwd_kernel<16><<<blocks, 256, 0, st>>>(probs, topk_e, dw, T, E, k, renorm, dlogits);
  else throw std::runtime_error("router: at most 512 experts");
  check("router_bwd");
}

// =====================================================================================
// Fused AdamW (standalone). The per-element math is adamw_math.cuh, shared with the
// weight-gradient GEMM epilogue that applies the same update in place, so both give the
// same bits.
//  * fp32 state: 4 consecutive elements per thread and step (16-byte accesses, coalesced
//    across the warp), any size (scalar tail). Streams at the HBM limit.
//  * 8-bit state (size % 32 == 0): persistent, one CTA of 16 independent warps per SM.
//    Each warp streams 512-element chunks (16 quantisation blocks) through a 3-stage
//    shared-memory ring with bulk copies (cp.async.bulk, completion on an mbarrier),
//    two chunks ahead of the one it computes; a lane pair updates one block from shared
//    memory in a lane-rotated unit order (conflict-free for 4/8/16-byte accesses), the
//    block scales are prefetched a chunk ahead, and the new weights and codes go back
//    with bulk stores, so the arithmetic overlaps the streaming instead of waiting for it.
// =====================================================================================
template <typename G>
__device__ __forceinline__ float grad_at(const G* g, size_t i);
template <>
__device__ __forceinline__ float grad_at<float>(const float* g, size_t i) { return g[i]; }
template <>
__device__ __forceinline__ float grad_at<__nv_bfloat16>(const __nv_bfloat16* g, size_t i) {
  return __bfloat162float(g[i]);
}

template <typename G>
__device__ __forceinline__ void load_grad4(const G* g, size_t i, float (&out)[4]) {
  if constexpr (sizeof(G) == 4) {
    const float4 g4 = *reinterpret_cast<const float4*>(g + i);
    out[0] = g4.x; out[1] = g4.y; out[2] = g4.z; out[3] = g4.w;
  } else {
    const uint2 r = *reinterpret_cast<const uint2*>(g + i);
    const float2 a = unpack_bf16x2(r.x), b = unpack_bf16x2(r.y);
    out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
  }
}

template <typename G>
__global__ void __launch_bounds__(256) adamw_fp32_kernel(const G* __restrict__ g, size_t n, OptHyper h) {
  const AdamCoef k = adam_coef(h);
  const size_t n4 = n / 4, stride = (size_t)gridDim.x * blockDim.x;
  float4* ms = reinterpret_cast<float4*>(h.master);
  float4* mm = reinterpret_cast<float4*>(h.m);
  float4* vv = reinterpret_cast<float4*>(h.v);
  uint2* pp = reinterpret_cast<uint2*>(h.param);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float gg[4];
    load_grad4(g, i * 4, gg);
    const float4 w4 = ms[i], m4 = mm[i], v4 = vv[i];
    float w[4] = {w4.x, w4.y, w4.z, w4.w}, m[4] = {m4.x, m4.y, m4.z, m4.w}, v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float sq;
      w[e] = adamw_step_elem(w[e], gg[e], m[e], v[e], sq, k);
    }
    ms[i] = make_float4(w[0], w[1], w[2], w[3]);
    mm[i] = make_float4(m[0], m[1], m[2], m[3]);
    vv[i] = make_float4(v[0], v[1], v[2], v[3]);
    pp[i] = make_uint2(pack_bf16x2(w[0], w[1]), pack_bf16x2(w[2], w[3]));
  }
  float* mms = reinterpret_cast<float*>(h.m);
  float* vvs = reinterpret_cast<float*>(h.v);
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    float m = mms[i], v = vvs[i], sq;
    const float w = adamw_step_elem(h.master[i], grad_at(g, i), m, v, sq, k);
    h.master[i] = w;
    mms[i] = m;
    vvs[i] = v;
    h.param[i] = __float2bfloat16(w);
  }
}

namespace opt8 {
constexpr int kWarps = 16, kStages = 3, kChunk = 512;  // 16 quantisation blocks per chunk
template <typename G>
struct Lay {  // one stage of one warp (bytes)
  static constexpr int OFF_W = kChunk * (int)sizeof(G);
  static constexpr int OFF_M = OFF_W + kChunk * 2;
  static constexpr int OFF_V = OFF_M + kChunk;
  static constexpr int BYTES = OFF_V + kChunk;
  static constexpr int SMEM = kWarps * kStages * BYTES + kWarps * kStages * 8;
};
}  // namespace opt8

template <typename G>
__global__ void __launch_bounds__(opt8::kWarps * 32, 1)
    adamw_8bit_kernel(const G* __restrict__ g, size_t n, OptHyper h, int* status, uint64_t timeout_ns) {
  using namespace opt8;
  using L = Lay<G>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * kStages * L::BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * kStages * L::BYTES) + warp * kStages;
  uint8_t* mq8 = reinterpret_cast<uint8_t*>(h.m);
  uint8_t* vq8 = reinterpret_cast<uint8_t*>(h.v);
  const AdamCoef k = adam_coef(h);
  const size_t nchunks = (n + kChunk - 1) / kChunk;
  const size_t nw = (size_t)gridDim.x * kWarps;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  auto issue = [&](int s, size_t c) {  // lane 0
    const size_t e0 = c * kChunk;
    const uint32_t ne = (uint32_t)(n - e0 < (size_t)kChunk ? n - e0 : (size_t)kChunk);
    uint8_t* b = ring + s * L::BYTES;
    mbar_arrive_expect_tx(&bars[s], ne * (uint32_t)(sizeof(G) + 4));
    bulk_load(b, g + e0, ne * (uint32_t)sizeof(G), &bars[s]);
    bulk_load(b + L::OFF_W, h.param + e0, ne * 2, &bars[s]);
    bulk_load(b + L::OFF_M, mq8 + e0, ne, &bars[s]);
    bulk_load(b + L::OFF_V, vq8 + e0, ne, &bars[s]);
  };
  size_t c = (size_t)blockIdx.x * kWarps + warp;
  if (lane == 0) {
    if (c < nchunks) issue(0, c);
    if (c + nw < nchunks) issue(1, c + nw);
  }
  volatile int abort_flag = 0;
  // lane l holds elements [16 l, 16 l + 16) of the chunk (block l / 2); unit rotation
  // (l >> 1) + (l >> 3) keeps 16-, 8- and 4-byte shared-memory accesses conflict-free
  const int rot = (lane >> 1) + (lane >> 3);
  auto scales = [&](size_t cc, float& ms, float& vs) {
    const size_t e = cc * kChunk + (size_t)lane * 16;
    const bool ok = cc < nchunks && e < n;
    ms = ok ? h.m_scale[e / 32] : 0.f;
    vs = ok ? h.v_scale[e / 32] : 0.f;
  };
  float msc, vsc;
  scales(c, msc, vsc);
  for (int it = 0; c < nchunks; ++it, c += nw) {
    const int s = it % kStages;
    const size_t e0 = c * kChunk;
    const size_t i0 = e0 + (size_t)lane * 16;
    const bool valid = i0 < n;
    float nmsc, nvsc;  // next chunk's scales, in flight during this chunk's arithmetic
    scales(c + nw, nmsc, nvsc);
    if (!mbar_wait_bounded(&bars[s], (uint32_t)(it / kStages) & 1u, &abort_flag, status, timeout_ns)) break;
    uint8_t* b = ring + s * L::BYTES;
    float gg[16];
    uint2 w[4];
    uint32_t mq[4], vq[4];
    const uint8_t* grow = b + lane * 16 * (int)sizeof(G);
    uint8_t* wrow = b + L::OFF_W + lane * 32;
    uint8_t* mrow = b + L::OFF_M + lane * 16;
    uint8_t* vrow = b + L::OFF_V + lane * 16;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int u = (q + rot) & 3;
      if (valid) {
        if constexpr (sizeof(G) == 4) {
          const float4 g4 = *reinterpret_cast<const float4*>(grow + 16 * u);
          gg[4 * q] = g4.x; gg[4 * q + 1] = g4.y; gg[4 * q + 2] = g4.z; gg[4 * q + 3] = g4.w;
        } else {
          const uint2 r = *reinterpret_cast<const uint2*>(grow + 8 * u);
          const float2 a = unpack_bf16x2(r.x), bb = unpack_bf16x2(r.y);
          gg[4 * q] = a.x; gg[4 * q + 1] = a.y; gg[4 * q + 2] = bb.x; gg[4 * q + 3] = bb.y;
        }
        w[q] = *reinterpret_cast<const uint2*>(wrow + 8 * u);
        mq[q] = *reinterpret_cast<const uint32_t*>(mrow + 4 * u);
        vq[q] = *reinterpret_cast<const uint32_t*>(vrow + 4 * u);
      } else {
        gg[4 * q] = gg[4 * q + 1] = gg[4 * q + 2] = gg[4 * q + 3] = 0.f;
        w[q] = make_uint2(0u, 0u);
        mq[q] = vq[q] = 0u;
      }
    }
    adamw_8bit_units<4>(gg, w, mq, vq, msc, vsc, i0, rot, k, h);
    if (valid) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int u = (q + rot) & 3;
        *reinterpret_cast<uint2*>(wrow + 8 * u) = w[q];
        *reinterpret_cast<uint32_t*>(mrow + 4 * u) = mq[q];
        *reinterpret_cast<uint32_t*>(vrow + 4 * u) = vq[q];
      }
      if ((lane & 1) == 0) {
        h.m_scale[i0 / 32] = msc;
        h.v_scale[i0 / 32] = vsc;
      }
    }
    fence_proxy_async_smem();  // this thread's shared-memory writes -> the bulk stores
    __syncwarp();
    if (lane == 0) {
      const uint32_t ne = (uint32_t)(n - e0 < (size_t)kChunk ? n - e0 : (size_t)kChunk);
      bulk_store(h.param + e0, b + L::OFF_W, ne * 2);
      bulk_store(mq8 + e0, b + L::OFF_M, ne);
      bulk_store(vq8 + e0, b + L::OFF_V, ne);
      bulk_commit();
      // refill the stage of iteration it-1 (its stores are the older pending group)
      if (c + 2 * nw < nchunks) {
        bulk_wait_read<1>();
        issue((it + 2) % kStages, c + 2 * nw);
      }
    }
    __syncwarp();
    msc = nmsc;
    vsc = nvsc;
  }
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

void adamw_update(const OptHyper& h, const void* g, bool g_bf16, size_t n, int num_sms, cudaStream_t st) {
  if (h.kind != kOptFp32 && h.kind != kOpt8bit) throw std::runtime_error("unknown optimizer state kind");
  if (h.kind == kOpt8bit) {
    if (n % 32) throw std::runtime_error("8-bit AdamW needs a multiple of 32 elements");
    const uintptr_t al = reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(h.param) |
                         reinterpret_cast<uintptr_t>(h.m) | reinterpret_cast<uintptr_t>(h.v);
    if (al & 15) throw std::runtime_error("8-bit AdamW needs 16-byte aligned gradient, weight and state");
    const size_t chunks = (n + opt8::kChunk - 1) / opt8::kChunk;
    const int grid = (int)std::max<size_t>(1, std::min<size_t>((chunks + opt8::kWarps - 1) / opt8::kWarps, num_sms));
    if (g_bf16) {
      using L = opt8::Lay<__nv_bfloat16>;
      static unsigned long long smem_devices = 0;
      smem_optin_once(adamw_8bit_kernel<__nv_bfloat16>, L::SMEM, smem_devices);
      adamw_8bit_kernel<__nv_bfloat16><<<grid, opt8::kWarps * 32, L::SMEM, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(g), n, h, nullptr, 2000000000ull);
    } else {
      using L = opt8::Lay<float>;
      static unsigned long long smem_devices = 0;
      smem_optin_once(adamw_8bit_kernel<float>, L::SMEM, smem_devices);
      adamw_8bit_kernel<float><<<grid, opt8::kWarps * 32, L::SMEM, st>>>(reinterpret_cast<const float*>(g), n, h,
                                                                         nullptr, 2000000000ull);
    }
  } else {
    if ((reinterpret_cast<uintptr_t>(h.master) | reinterpret_cast<uintptr_t>(h.m) | reinterpret_cast<uintptr_t>(h.v) |
         reinterpret_cast<uintptr_t>(h.param) | reinterpret_cast<uintptr_t>(g)) & 15)
      throw std::runtime_error("AdamW needs 16-byte aligned gradient, weight and state");
    const int grid = (int)std::max<size_t>(1, std::min<size_t>(((n + 3) / 4 + 255) / 256, (size_t)num_sms * 8));
    if (g_bf16) adamw_fp32_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(g), n, h);
    else adamw_fp32_kernel<float><<<grid, 256, 0, st>>>(reinterpret_cast<const float*>(g), n, h);
  }
  check("adamw");
}

// =====================================================================================
// Cross-entropy (mean over valid labels) fused with its gradient:
//   loss[t] = logsumexp(z_t) - z_t[y_t];  dz_t = (softmax(z_t) - onehot(y_t)) * scale,
// written in place over the bf16 logits. One block per row; labels < 0 are ignored.
// =====================================================================================
__global__ void __launch_bounds__(512) xent_fwd_bwd_kernel(__nv_bfloat16* __restrict__ logits, const int* __restrict__ labels,
                                                           int V, float scale, float* __restrict__ loss) {
  const int t = blockIdx.x;
  __nv_bfloat16* z = logits + (size_t)t * V;
  const int y = labels[t];
  __shared__ float s_m[16], s_s[16];
  float m = -INFINITY, s = 0.f;
  const int nvec = V / 8;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float f[8];
    load8(z + i * 8, f);
    float lm = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) lm = fmaxf(lm, f[e]);
    const float nm = fmaxf(m, lm);
    float acc = s * __expf(m - nm);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc += __expf(f[e] - nm);
    m = nm;
    s = acc;
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    const float f = __bfloat162float(z[i]);
    const float nm = fmaxf(m, f);
    s = s * __expf(m - nm) + __expf(f - nm);
    m = nm;
  }
  // block reduce (m, s)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffff, m, o);
    const float os = __shfl_xor_sync(0xffffffff, s, o);
    const float nm = fmaxf(m, om);
    s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    m = nm;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_m[warp] = m;
    s_s[warp] = s;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? s_m[lane] : -INFINITY;
    s = lane < nw ? s_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffff, m, o);
      const float os = __shfl_xor_sync(0xffffffff, s, o);
      const float nm = fmaxf(m, om);
      s = (m == -INFINITY ? 0.f : s * __expf(m - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      m = nm;
    }
    if (lane == 0) {
      s_m[0] = m;
      s_s[0] = s;
    }
  }
  __syncthreads();
  m = s_m[0];
  s = s_s[0];
  const float lse = m + __logf(s);
  const float zy = (y >= 0) ? __bfloat162float(z[y]) : 0.f;
  __syncthreads();
  if (threadIdx.x == 0) loss[t] = (y >= 0) ? (lse - zy) : 0.f;
  const float sc = (y >= 0) ? scale : 0.f;
  for (int i = threadIdx.x; i < nvec; i += blockDim.x) {
    float f[8], o[8];
    load8(z + i * 8, f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int col = i * 8 + e;
      o[e] = (__expf(f[e] - lse) - (col == y ? 1.f : 0.f)) * sc;
    }
    store8(z + i * 8, o);
  }
  for (int i = nvec * 8 + threadIdx.x; i < V; i += blockDim.x) {
    const float f = __bfloat162float(z[i]);
    z[i] = __float2bfloat16((__expf(f - lse) - (i == y ? 1.f : 0.f)) * sc);
  }
}

void xent_fwd_bwd(void* logits, const int* labels, int T, int V, float scale, float* loss, cudaStream_t st) {
  xent_fwd_bwd_kernel<<<T, 512, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(logits), labels, V, scale, loss);
  check("xent_fwd_bwd");
}

}  // namespace sepx
