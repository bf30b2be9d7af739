// Expert-parallel dispatch / combine over NVLink peer memory (one process per GPU).
//
// Data plane: every rank owns the same symmetric layout (see symm_heap.cpp) and the
// kernels write straight into peers' buffers with 16-byte stores, then publish an
// epoch-tagged header with a system-scope release store. Receivers acquire-poll the
// headers with a deadline; on timeout they record kErrTimeoutPeer and return.
//
// Per-rank deduplication: a token is sent to a destination rank at most once, whatever
// number of its top-k experts live there (the reference sends one row per (token,
// expert) inside a node, src/rbd.py:229-236, and one pilot per (token, node) between
// nodes, src/rbd.py:238-252). The receiving rank fans the row out to its local experts
// in HBM (permute kernel), applies the gate weights, reduces a token's co-resident
// experts and returns ONE partial row per (token, rank).
//
// Symmetric slabs (per rank, indexed [src][slot]):
//   recv_x   [W][cap][H] bf16   rows received from each source
//   recv_e   [W][cap][k] int16  local expert slot of each of the row's k choices (-1: other rank)
//   recv_w   [W][cap][k] f32    gate weight of each choice
//   ret_x    [W][cap][H] bf16   partial outputs returned by each expert rank
//   ret_w    [W][cap][k] f32    per-choice router-weight gradients (backward)
//   hdr      [4][W]      u64    (epoch << 32 | rows) per phase: 0 dispatch, 1 combine
//
// Rows a rank sends to itself never cross the slab: the permute reads x directly and
// the slot->token map for self rows is kept locally.
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>

#include <stdexcept>
#include <string>

#include "kernels.h"
#include "sm100.cuh"

namespace sepx {

constexpr int kMaxW = 64;

__device__ __forceinline__ bool wait_header(const uint64_t* hdr, uint32_t epoch, uint32_t* rows,
                                            int* status, uint64_t timeout_ns) {
  uint64_t v = ld_acquire_sys_u64(hdr);
  if ((uint32_t)(v >> 32) == epoch) {
    *rows = (uint32_t)v;
    return true;
  }
  uint64_t t0 = globaltimer_ns();
  while (true) {
    v = ld_acquire_sys_u64(hdr);
    if ((uint32_t)(v >> 32) == epoch) {
      *rows = (uint32_t)v;
      return true;
    }
    if (globaltimer_ns() - t0 > timeout_ns) {
      record_error(status, kErrTimeoutPeer);
      return false;
    }
    __nanosleep(64);
  }
}

// ------------------------------------------------------------------------------------
// K1: route plan. slot[t][d] = ordinal of token t among tokens sent to rank d (-1 if
// none of t's choices goes to d). dst_tk[t][j] is the destination rank of choice j (-1:
// not sent). Single block; T up to a few 10^4 tokens.
// ------------------------------------------------------------------------------------
// Inclusive scan of one int per lane of a full warp.
__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Destination mask of token t: bit d set when any choice goes to rank d. KV > 0: k == KV
// is known at compile time and each row is read with KV / 4 16-byte loads.
template <int KV>
__device__ __forceinline__ unsigned long long token_mask(const int* __restrict__ dst_tk, int t, int T, int k) {
  unsigned long long m = 0;
  if (t >= T) return 0;
  if constexpr (KV > 0) {
    const int4* p = reinterpret_cast<const int4*>(dst_tk + (size_t)t * KV);
#pragma unroll
    for (int q = 0; q < KV / 4; ++q) {
      const int4 v = __ldg(p + q);
      m |= (v.x >= 0 ? 1ull << v.x : 0ull) | (v.y >= 0 ? 1ull << v.y : 0ull) |
           (v.z >= 0 ? 1ull << v.z : 0ull) | (v.w >= 0 ? 1ull << v.w : 0ull);
    }
  } else {
    for (int j = 0; j < k; ++j) {
      const int d = __ldg(dst_tk + (size_t)t * k + j);
      if (d >= 0) m |= 1ull << d;
    }
  }
  return m;
}

constexpr int kPlanRounds = 4;  // rounds of 1024 tokens whose loads are issued together

// self_tok (optional): also writes self_tok[slot[t][rank]] = t for the tokens that stay on
// this rank (the receive side's map of its own rows), which at world size 1 is all the
// dispatch kernel would do.
template <int KV>
__global__ void __launch_bounds__(1024) route_plan_kernel(const int* __restrict__ dst_tk, int T,
                                                          int k, int W, int* __restrict__ slot,
                                                          int* __restrict__ send_count,
                                                          int* __restrict__ self_tok = nullptr, int rank = 0) {
  // Tokens in passes of kPlanRounds x 1024 (one per thread per round, every load of a pass
  // in flight at once). Per destination, a warp ballot gives each token its rank among the
  // warp's senders; the 128 per-warp totals of a pass (round-major, so token order) are
  // scanned by one warp per destination, and a running base per destination carries
  // across passes. Slots follow token order (deterministic).
  __shared__ int s_warp[kPlanRounds * 32][kMaxW];
  __shared__ int s_base[kMaxW];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  if (tid < W) s_base[tid] = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += blockDim.x * kPlanRounds) {
    unsigned long long m[kPlanRounds];
#pragma unroll
    for (int r = 0; r < kPlanRounds; ++r) m[r] = token_mask<KV>(dst_tk, t0 + r * blockDim.x + tid, T, k);
#pragma unroll
    for (int r = 0; r < kPlanRounds; ++r)
      for (int d = 0; d < W; ++d) {
        const unsigned b = __ballot_sync(0xffffffffu, (m[r] >> d) & 1ull);
        if (lane == 0) s_warp[r * nwarps + warp][d] = __popc(b);
      }
    __syncthreads();
    // exclusive scan of the kPlanRounds * nwarps totals of destination d, one warp each
    const int n = kPlanRounds * nwarps, per = (n + 31) / 32;
    for (int d = warp; d < W; d += nwarps) {
      int v[kPlanRounds];
      int sum = 0;
#pragma unroll
      for (int i = 0; i < kPlanRounds; ++i) {
        const int e = lane * per + i;
        v[i] = (i < per && e < n) ? s_warp[e][d] : 0;
        sum += v[i];
      }
      const int incl = warp_incl_scan(sum, lane);
      int acc = s_base[d] + incl - sum;
      const int total = __shfl_sync(0xffffffffu, incl, 31);
#pragma unroll
      for (int i = 0; i < kPlanRounds; ++i) {
        const int e = lane * per + i;
        if (i < per && e < n) s_warp[e][d] = acc;
        acc += v[i];
      }
      __syncwarp();
      if (lane == 0) s_base[d] += total;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kPlanRounds; ++r) {
      const int t = t0 + r * blockDim.x + tid;
      for (int d = 0; d < W; ++d) {  // every lane takes part in the ballot; only real tokens store
        const unsigned b = __ballot_sync(0xffffffffu, (m[r] >> d) & 1ull);
        const int before = __popc(b & ((1u << lane) - 1u));
        const bool sent = (m[r] >> d) & 1ull;
        const int sl = s_warp[r * nwarps + warp][d] + before;
        if (t < T) slot[(size_t)t * W + d] = sent ? sl : -1;
        if (self_tok && d == rank && sent && t < T) self_tok[sl] = t;
      }
    }
    __syncthreads();
  }
  if (tid < W) send_count[tid] = s_base[tid];
}

// Per-(token, choice) routing tables from expert ids: dst = e2r[e], meta = e2l[e] (-1 for e < 0).
__global__ void route_tables_kernel(const int* __restrict__ topk_e, const int* __restrict__ e2r,
                                    const int* __restrict__ e2l, int n, int* __restrict__ dst, int* __restrict__ meta) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = topk_e[i];
    dst[i] = e >= 0 ? __ldg(e2r + e) : -1;
    meta[i] = e >= 0 ? __ldg(e2l + e) : -1;
  }
}

// Bit mask of W ranks rotated right by r: bit i of the result is bit (i + r) % W of m.
__device__ __forceinline__ unsigned long long rotr_mask(unsigned long long m, int r, int W) {
  if (r == 0) return m;
  const unsigned long long full = W >= 64 ? ~0ull : ((1ull << W) - 1ull);
  return ((m >> r) | (m << (W - r))) & full;
}

// Epoch of this call: the host value plus the device counter when one is given.
__device__ __forceinline__ uint32_t ep_epoch(const EpArgs& a) {
  return a.epoch_dev ? a.epoch + *a.epoch_dev : a.epoch;
}

// Publish helper: the last CTA to finish writes the headers (release, system scope).
__device__ __forceinline__ void publish_last_cta(unsigned int* done_counter, const EpArgs& a,
                                                 int phase, const int* counts_per_dst,
                                                 bool counts_are_per_src) {
  __syncthreads();
  __shared__ bool s_last;
  if (threadIdx.x == 0) {
    __threadfence_system();
    unsigned int prev = atomicAdd(done_counter, 1u);
    s_last = ((prev + 1) % gridDim.x) == 0;
  }
  __syncthreads();
  if (s_last && threadIdx.x < a.W) {
    __threadfence_system();
    const int d = threadIdx.x;
    char* base = reinterpret_cast<char*>(a.peer_base[d]);
    uint64_t* hdr = reinterpret_cast<uint64_t*>(base + a.off_hdr) + (size_t)phase * a.W + a.rank;
    uint32_t rows = (uint32_t)counts_per_dst[d];
    (void)counts_are_per_src;
    st_release_sys_u64(hdr, ((uint64_t)ep_epoch(a) << 32) | rows);
  }
}

// ------------------------------------------------------------------------------------
// K3: dispatch. One warp per (token): loads the row once, stores it to every remote
// destination's recv_x[rank][slot], with the k (local expert, weight) entries.
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) dispatch_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x,
                                                       const int* __restrict__ dst_tk,
                                                       const int* __restrict__ meta_tk,
                                                       const float* __restrict__ topk_w,
                                                       const int* __restrict__ slot,
                                                       int* __restrict__ self_tok,
                                                       const int* __restrict__ send_count,
                                                       int with_meta, int fp8) {
  const int lane = threadIdx.x & 31;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  const int vec = a.H / 8;  // uint4 per row
  for (int t = gwarp; t < a.T; t += nwarps) {
    const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)t * a.H);
    // destinations of this token
    unsigned long long m = 0;
    for (int j = 0; j < a.k; ++j) {
      const int d = __ldg(dst_tk + t * a.k + j);
      if (d >= 0) m |= 1ull << d;
    }
    if ((m >> a.rank) & 1) {
      if (lane == 0) self_tok[__ldg(slot + (size_t)t * a.W + a.rank)] = t;
    }
    unsigned long long remote = m & ~(1ull << a.rank);
    if (!remote) continue;
    // destinations are visited starting at a token-dependent rank (a rotation of the
    // bit mask), so concurrent warps spread their stores over every peer's ingress
    const int rot = (t + a.rank) % a.W;
    for (int c0 = 0; c0 < vec; c0 += 32 * 8) {
      uint4 r[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int c = c0 + i * 32 + lane;
        if (c < vec) r[i] = __ldg(src + c);
      }
      if (fp8) {
        // e4m3 payload, one fp32 scale per 128 values (= 16 lanes x 8 values)
        uint2 q[8];
        float sc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = c0 + i * 32 + lane;
          float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          if (c < vec) {
            float2 a0 = unpack_bf16x2(r[i].x), a1 = unpack_bf16x2(r[i].y), a2 = unpack_bf16x2(r[i].z),
                   a3 = unpack_bf16x2(r[i].w);
            f[0] = a0.x; f[1] = a0.y; f[2] = a1.x; f[3] = a1.y; f[4] = a2.x; f[5] = a2.y; f[6] = a3.x; f[7] = a3.y;
          }
          float amax = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
#pragma unroll
          for (int o = 1; o < 16; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffff, amax, o));
          sc[i] = amax > 0.f ? amax / 448.f : 1.f;
          const float inv = 1.f / sc[i];
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_fp8x2_storage_t p2 =
                __nv_cvt_float2_to_fp8x2(make_float2(f[2 * e] * inv, f[2 * e + 1] * inv), __NV_SATFINITE, __NV_E4M3);
            w[e] = (uint32_t)p2;
          }
          q[i] = make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
        }
        unsigned long long rm = rotr_mask(remote, rot, a.W);
        while (rm) {
          int d = __ffsll(rm) - 1;
          rm &= rm - 1;
          d += rot;
          if (d >= a.W) d -= a.W;
          int s = __ldg(slot + (size_t)t * a.W + d);
          char* base = reinterpret_cast<char*>(a.peer_base[d]);
          uint2* dq = reinterpret_cast<uint2*>(base + a.off_recv_q) + ((size_t)a.rank * a.cap + s) * vec;
          float* ds = reinterpret_cast<float*>(base + a.off_recv_s) + ((size_t)a.rank * a.cap + s) * (a.H / 128);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            int c = c0 + i * 32 + lane;
            if (c < vec) {
              dq[c] = q[i];
              if ((lane & 15) == 0) ds[c / 16] = sc[i];
            }
          }
        }
        continue;
      }
      unsigned long long rm = rotr_mask(remote, rot, a.W);
      while (rm) {
        int d = __ffsll(rm) - 1;
        rm &= rm - 1;
        d += rot;
        if (d >= a.W) d -= a.W;
        int s = __ldg(slot + (size_t)t * a.W + d);
        char* base = reinterpret_cast<char*>(a.peer_base[d]);
        uint4* dst = reinterpret_cast<uint4*>(base + a.off_recv_x) +
                     ((size_t)a.rank * a.cap + s) * vec;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          int c = c0 + i * 32 + lane;
          if (c < vec) dst[c] = r[i];
        }
      }
    }
    if (with_meta && a.k == 8) {
      // top-8: the 8 expert ids (16 B) and 8 weights (32 B) of each (token, destination)
      // go out as three 16-byte stores gathered by warp shuffles (one NVLink write each)
      const int j = lane < 8 ? lane : 0;
      const int owner = __ldg(dst_tk + t * 8 + j);
      const int meta = __ldg(meta_tk + t * 8 + j);
      const float w = __ldg(topk_w + t * 8 + j);
      float wf[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) wf[q] = __shfl_sync(0xffffffffu, w, q);
      unsigned long long rm = rotr_mask(remote, rot, a.W);
      while (rm) {
        int d = __ffsll(rm) - 1;
        rm &= rm - 1;
        d += rot;
        if (d >= a.W) d -= a.W;
        const int e = (owner == d) ? meta : -1;
        const uint32_t pair = ((uint32_t)e & 0xFFFFu) | ((uint32_t)__shfl_down_sync(0xffffffffu, e, 1) << 16);
        const uint32_t p1 = __shfl_sync(0xffffffffu, pair, 2), p2 = __shfl_sync(0xffffffffu, pair, 4),
                       p3 = __shfl_sync(0xffffffffu, pair, 6);
        if (lane == 0) {
          const int s = __ldg(slot + (size_t)t * a.W + d);
          char* base = reinterpret_cast<char*>(a.peer_base[d]);
          const size_t row = (size_t)a.rank * a.cap + s;
          *reinterpret_cast<uint4*>(reinterpret_cast<int16_t*>(base + a.off_recv_e) + row * 8) =
              make_uint4(pair, p1, p2, p3);
          float4* rw = reinterpret_cast<float4*>(reinterpret_cast<float*>(base + a.off_recv_w) + row * 8);
          rw[0] = make_float4(wf[0], wf[1], wf[2], wf[3]);
          rw[1] = make_float4(wf[4], wf[5], wf[6], wf[7]);
        }
      }
    } else if (with_meta && lane < a.k) {
      const int j = lane;
      const int owner = __ldg(dst_tk + t * a.k + j);
      const int meta = __ldg(meta_tk + t * a.k + j);
      const float w = __ldg(topk_w + t * a.k + j);
      unsigned long long rm = rotr_mask(remote, rot, a.W);
      while (rm) {
        int d = __ffsll(rm) - 1;
        rm &= rm - 1;
        d += rot;
        if (d >= a.W) d -= a.W;
        int s = __ldg(slot + (size_t)t * a.W + d);
        char* base = reinterpret_cast<char*>(a.peer_base[d]);
        int16_t* re = reinterpret_cast<int16_t*>(base + a.off_recv_e) + ((size_t)a.rank * a.cap + s) * a.k;
        float* rw = reinterpret_cast<float*>(base + a.off_recv_w) + ((size_t)a.rank * a.cap + s) * a.k;
        re[j] = (owner == d) ? (int16_t)meta : (int16_t)-1;
        rw[j] = w;
      }
    }
  }
  publish_last_cta(a.done_counter, a, a.phase, send_count, false);
}

// ------------------------------------------------------------------------------------
// Receive side. Rows are enumerated src-major: (src, slot) for slot < rows_from[src].
// ------------------------------------------------------------------------------------
// All k (local expert, weight) entries of received row (src, s), loaded at once (the
// permute kernel's passes over the choices then wait on no memory). k <= 8.
__device__ __forceinline__ void row_meta_all(const EpArgs& a, const int* dst_tk, const float* topk_w,
                                             const int* self_tok, const int* meta_tk, int src, int s,
                                             int (&le)[8], float (&w)[8]) {
  if (src == a.rank) {
    const int t = self_tok[s];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < a.k) {
        le[j] = (__ldg(dst_tk + t * a.k + j) == a.rank) ? __ldg(meta_tk + t * a.k + j) : -1;
        w[j] = __ldg(topk_w + t * a.k + j);
      }
    }
  } else {
    const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
    const int16_t* re = reinterpret_cast<const int16_t*>(base + a.off_recv_e) + ((size_t)src * a.cap + s) * a.k;
    const float* rw = reinterpret_cast<const float*>(base + a.off_recv_w) + ((size_t)src * a.cap + s) * a.k;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < a.k) {
        le[j] = re[j];
        w[j] = rw[j];
      }
    }
  }
}

constexpr int kChunk = 128;

// Chunk counts the scan stages in shared memory (dynamic, with the kernel's static
// shared memory under 48 KB); larger layouts are scanned in place in global memory.
constexpr int kScanSmemEntries = 8192;
__host__ __device__ constexpr int scan_smem_words(int n) { return n + (n >> 5) + 1; }

// K4a count: per chunk of 128 rows, rows per local expert -> chunk_cnt[g][chunk].
__global__ void __launch_bounds__(kChunk) recv_count_kernel(EpArgs a, const int* __restrict__ dst_tk,
                                                            const float* __restrict__ topk_w,
                                                            const int* __restrict__ self_tok,
                                                            const int* __restrict__ meta_tk,
                                                            const int* __restrict__ send_count,
                                                            int* __restrict__ rows_from,
                                                            int* __restrict__ chunk_cnt, int G) {
  // blockIdx.x = src * chunks_per_src + chunk
  const int chunks_per_src = (a.cap + kChunk - 1) / kChunk;
  const int src = blockIdx.x / chunks_per_src;
  const int chunk = blockIdx.x % chunks_per_src;
  __shared__ int s_rows;
  __shared__ int s_cnt[1024];
  for (int g = threadIdx.x; g < G; g += blockDim.x) s_cnt[g] = 0;
  if (threadIdx.x == 0) {
    uint32_t rows = 0;
    if (src == a.rank) {
      rows = (uint32_t)send_count[a.rank];
    } else {
      const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
      const uint64_t* hdr = reinterpret_cast<const uint64_t*>(base + a.off_hdr) + (size_t)a.phase * a.W + src;
      if (!wait_header(hdr, ep_epoch(a), &rows, a.status, a.timeout_ns)) rows = 0;
    }
    if (rows > (uint32_t)a.cap) {
      record_error(a.status, kErrOverflow);
      rows = a.cap;
    }
    s_rows = (int)rows;
    if (chunk == 0) rows_from[src] = (int)rows;
  }
  __syncthreads();
  const int s = chunk * kChunk + threadIdx.x;
  if (s < s_rows) {
    int le_all[8];
    float w_all[8];
    row_meta_all(a, dst_tk, topk_w, self_tok, meta_tk, src, s, le_all, w_all);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= a.k) break;
      const int le = le_all[j];
      if (le >= G || le < -1) {
        record_error(a.status, kErrCorrupt);  // corrupted metadata: the entry is dropped
      } else if (le >= 0) {
        atomicAdd(&s_cnt[le], 1);
      }
    }
  }
  __syncthreads();
  for (int g = threadIdx.x; g < G; g += blockDim.x)
    chunk_cnt[(size_t)g * gridDim.x + blockIdx.x] = s_cnt[g];
}

// Block-wide exclusive scan of one int per thread; *total (shared) gets the sum.
__device__ __forceinline__ int block_excl_scan(int v, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int incl = warp_incl_scan(v, lane);
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int x = lane < nw ? s_warp[lane] : 0;
    const int sx = warp_incl_scan(x, lane);
    if (lane < nw) s_warp[lane] = sx - x;
    if (lane == 31) *total = sx;
  }
  __syncthreads();
  const int r = s_warp[warp] + incl - v;
  __syncthreads();
  return r;
}

// Segmented-scan operator on (segment started, value) pairs, a before b.
__device__ __forceinline__ void seg_combine(bool fa, int va, bool& fb, int& vb) {
  if (!fb) vb += va;
  fb = fb || fa;
}

// K4b scan. chunk_cnt is laid out [G][nchunks] (each group's chunk counts contiguous).
// Per group: exclusive scan over chunks and the group's total; then an exclusive scan of
// the 64-row-padded group totals gives group_off / pad_off, and the chunk entries become
// absolute row offsets. With s_cc (shared memory for scan_smem_words(G * nchunks) words)
// the counts are staged and scanned as one segmented scan, each thread a contiguous run;
// without it, one warp per group scans in place in global memory. Any block size that is
// a multiple of 32.
__device__ void scan_groups(const EpArgs& a, int* __restrict__ chunk_cnt, int nchunks, int G,
                            int* __restrict__ group_off, int* __restrict__ group_cnt, int* __restrict__ pad_off,
                            int cap_rows, int* __restrict__ need, int* __restrict__ miss, int* s_cc) {
  __shared__ int s_tot[1024];
  __shared__ int s_off[1024];
  __shared__ int s_warp[32];
  __shared__ int s_wv[32];
  __shared__ bool s_wf[32];
  __shared__ int s_sum[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int n = nchunks * G;
  auto P = [](int i) { return i + (i >> 5); };  // one pad word per 32: conflict-free runs
  if (s_cc) {
    // 1) staged: load all counts (written by other blocks: read from L2), then one
    //    segmented exclusive scan over the flattened [G][nchunks] array, each thread a
    //    contiguous run of it, a segment per group
#pragma unroll 8
    for (int i = threadIdx.x; i < n; i += blockDim.x) s_cc[P(i)] = __ldcg(chunk_cnt + i);
    __syncthreads();
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int i0 = min(n, (int)threadIdx.x * per), i1 = min(n, i0 + per);
    bool f = false;
    int v = 0;
    for (int i = i0; i < i1; ++i) {
      if (i % nchunks == 0) {
        v = 0;
        f = true;
      }
      v += s_cc[P(i)];
    }
    // inclusive warp scan of (f, v), then exclusive per thread
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const bool nf = __shfl_up_sync(0xffffffffu, f, o);
      const int nv = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) seg_combine(nf, nv, f, v);
    }
    bool ef = __shfl_up_sync(0xffffffffu, f, 1);
    int ev = __shfl_up_sync(0xffffffffu, v, 1);
    if (lane == 0) {
      ef = false;
      ev = 0;
    }
    if (lane == 31) {
      s_wf[warp] = f;
      s_wv[warp] = v;
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the warp aggregates
      bool wf = lane < nw ? s_wf[lane] : false;
      int wv = lane < nw ? s_wv[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const bool nf = __shfl_up_sync(0xffffffffu, wf, o);
        const int nv = __shfl_up_sync(0xffffffffu, wv, o);
        if (lane >= o) seg_combine(nf, nv, wf, wv);
      }
      const bool xf = __shfl_up_sync(0xffffffffu, wf, 1);
      const int xv = __shfl_up_sync(0xffffffffu, wv, 1);
      if (lane < nw) {
        s_wf[lane] = lane == 0 ? false : xf;
        s_wv[lane] = lane == 0 ? 0 : xv;
      }
    }
    __syncthreads();
    bool cf = s_wf[warp];
    int carry = s_wv[warp];
    seg_combine(cf, carry, ef, ev);  // prefix of the warp, then of the lanes before
    int run = ev;
    for (int i = i0; i < i1; ++i) {
      if (i % nchunks == 0) run = 0;
      const int x = s_cc[P(i)];
      s_cc[P(i)] = run;
      run += x;
      if ((i + 1) % nchunks == 0) s_tot[i / nchunks] = run;
    }
  } else {
    // 1) in place in global memory: per group (one warp each, coalesced over its
    //    contiguous chunk counts)
    for (int g = warp; g < G; g += nw) {
      int carry = 0;
      int* row = chunk_cnt + (size_t)g * nchunks;
      for (int c0 = 0; c0 < nchunks; c0 += 32) {
        const int c = c0 + lane;
        const int v = c < nchunks ? __ldcg(row + c) : 0;  // written by other blocks: read from L2
        const int incl = warp_incl_scan(v, lane);
        if (c < nchunks) row[c] = carry + incl - v;
        carry += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) s_tot[g] = carry;
    }
  }
  __syncthreads();
  // 2) padded totals and padding counts, scanned over groups: each thread takes a
  //    contiguous run of groups
  const int per = (G + blockDim.x - 1) / blockDim.x;
  const int g0 = min(G, (int)threadIdx.x * per), g1 = min(G, g0 + per);
  int sp = 0, sq = 0;
  for (int g = g0; g < g1; ++g) {
    const int padded = (s_tot[g] + 63) & ~63;
    sp += padded;
    sq += padded - s_tot[g];
  }
  int base_p = block_excl_scan(sp, s_warp, &s_sum[0]);
  int base_q = block_excl_scan(sq, s_warp, &s_sum[1]);
  for (int g = g0; g < g1; ++g) {
    const int padded = (s_tot[g] + 63) & ~63;
    s_off[g] = base_p;
    group_cnt[g] = s_tot[g];
    pad_off[g] = base_q;
    base_p += padded;
    base_q += padded - s_tot[g];
  }
  __syncthreads();
  const int total = s_sum[0], ptotal = s_sum[1];
  if (threadIdx.x == 0 && need) *need = total;
  if (total > cap_rows) {
    // with the worst-case capacity this cannot happen (a guard); with a row budget it
    // asks the caller for a larger one: the layout is emptied
    if (threadIdx.x == 0) {
      if (miss) atomicExch(miss, 1);
      else record_error(a.status, kErrOverflow);
    }
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      group_off[g] = 0;
      group_cnt[g] = 0;
      pad_off[g] = 0;
    }
    if (threadIdx.x == 0) {
      group_off[G] = 0;
      pad_off[G] = 0;
    }
    return;
  }
  for (int g = threadIdx.x; g < G; g += blockDim.x) group_off[g] = s_off[g];
  if (threadIdx.x == 0) {
    group_off[G] = total;
    pad_off[G] = ptotal;
  }
  // 3) chunk bases become absolute row offsets
  if (s_cc) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) chunk_cnt[i] = s_cc[P(i)] + s_off[i / nchunks];
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) chunk_cnt[i] += s_off[i / nchunks];
  }
}

// cap_rows bounds the receive buffers. With `miss` given, cap_rows is the caller's row
// budget for this call (buffers sized before the count is known, so the host never waits
// for it): a total above it sets *miss = 1 instead of an error, the layout is emptied
// (every later kernel of the call moves nothing) and the caller runs the pass again with
// a larger budget. `need`, when given, receives the total rows the layout needs.
__global__ void __launch_bounds__(1024) recv_scan_kernel(EpArgs a, int* __restrict__ chunk_cnt,
                                                         int nchunks, int G,
                                                         int* __restrict__ group_off,
                                                         int* __restrict__ group_cnt,
                                                         int* __restrict__ pad_off,
                                                         int cap_rows, int* __restrict__ need = nullptr,
                                                         int* __restrict__ miss = nullptr, int smem = 0) {
  extern __shared__ int s_dyn[];
  scan_groups(a, chunk_cnt, nchunks, G, group_off, group_cnt, pad_off, cap_rows, need, miss,
              smem ? s_dyn : nullptr);
}

// K4c permute: place every (row, local choice) at its deterministic position inside its
// expert group, copy the row (from the slab or, for self rows, from x), record maps.
// Also zero-fills the group padding rows.
__global__ void __launch_bounds__(kChunk) recv_permute_kernel(
    EpArgs a, const __nv_bfloat16* __restrict__ x, const int* __restrict__ dst_tk,
    const float* __restrict__ topk_w, const int* __restrict__ self_tok, const int* __restrict__ meta_tk,
    const int* __restrict__ rows_from, const int* __restrict__ chunk_base,
    int G, const int* __restrict__ group_off, const int* __restrict__ group_cnt,
    const int* __restrict__ pad_off, __nv_bfloat16* __restrict__ xp, float* __restrict__ row_w,
    int* __restrict__ row_src, int* __restrict__ inv_rows) {
  const int chunks_per_src = (a.cap + kChunk - 1) / kChunk;
  const int src = blockIdx.x / chunks_per_src;
  const int chunk = blockIdx.x % chunks_per_src;
  const int s = chunk * kChunk + threadIdx.x;
  const int rows = rows_from[src];
  __shared__ int s_base[1024];
  for (int g = threadIdx.x; g < G; g += blockDim.x) s_base[g] = chunk_base[(size_t)g * gridDim.x + blockIdx.x];
  __syncthreads();
  // per-warp entry counts of each group in the current pass (zero between passes)
  constexpr int kWarpsPerChunk = kChunk / 32;
  __shared__ int s_wcnt[kWarpsPerChunk * 1024];
  for (int i = threadIdx.x; i < kWarpsPerChunk * G; i += blockDim.x) s_wcnt[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned lanes_below = (1u << lane) - 1u;
  // Positions are deterministic: within an expert group, entries of this chunk are
  // ordered by (choice j, slot). Each pass j ranks the block's threads sharing a group:
  // within a warp by __match_any_sync, across warps by per-warp group counts.
  int le_all[8];
  float w_all[8];
  if (s < rows) row_meta_all(a, dst_tk, topk_w, self_tok, meta_tk, src, s, le_all, w_all);
  for (int j = 0; j < a.k; ++j) {
    int le = -1;
    float w = 0.f;
    if (s < rows) {
      // registers indexed by the loop counter: the loop is unrolled over k <= 8
      switch (j) {
        case 0: le = le_all[0]; w = w_all[0]; break;
        case 1: le = le_all[1]; w = w_all[1]; break;
        case 2: le = le_all[2]; w = w_all[2]; break;
        case 3: le = le_all[3]; w = w_all[3]; break;
        case 4: le = le_all[4]; w = w_all[4]; break;
        case 5: le = le_all[5]; w = w_all[5]; break;
        case 6: le = le_all[6]; w = w_all[6]; break;
        default: le = le_all[7]; w = w_all[7]; break;
      }
    }
    if (le >= G || le < -1) le = -1;  // corrupted entry (recorded by the count kernel)
    const unsigned peers = __match_any_sync(0xffffffffu, le);
    const bool leader = (__ffs(peers) - 1) == lane;
    if (le >= 0 && leader) s_wcnt[warp * G + le] = __popc(peers);
    __syncthreads();
    int pos = -1, before = 0, total = 0;
    if (le >= 0) {
      before = __popc(peers & lanes_below);
#pragma unroll
      for (int w2 = 0; w2 < kWarpsPerChunk; ++w2) {
        const int c = s_wcnt[w2 * G + le];
        before += (w2 < warp) ? c : 0;
        total += c;
      }
      pos = s_base[le] + before;
      if (pos - group_off[le] < group_cnt[le]) {
        row_w[pos] = w;
        row_src[pos] = src * a.cap + s;
      } else {
        pos = -1;  // beyond capacity: dropped (overflow already recorded)
      }
    }
    __syncthreads();  // every thread has read s_base and s_wcnt for this pass
    if (le >= 0 && leader) s_wcnt[warp * G + le] = 0;
    if (le >= 0 && before == total - 1) s_base[le] += total;  // last of its group advances
    if (s < rows) inv_rows[((size_t)src * a.cap + s) * a.k + j] = pos;
    __syncthreads();
  }
  // padding rows: weight 0, no source (the gather kernel zero-fills their data)
  const int npad = pad_off[G];
  for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < npad; q += gridDim.x * blockDim.x) {
    int lo = 0, hi = G;  // largest g with pad_off[g] <= q
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (pad_off[mid] <= q) lo = mid; else hi = mid;
    }
    const int r = group_off[lo] + group_cnt[lo] + (q - pad_off[lo]);
    row_w[r] = 0.f;
    row_src[r] = -1;
  }
}

// ------------------------------------------------------------------------------------
// Plain gather for the backward: xp[p] = slab row (or dy[self]) for p in every group;
// padding rows zero.
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) recv_gather_kernel(EpArgs a, const __nv_bfloat16* __restrict__ x,
                                                          const int* __restrict__ self_tok,
                                                          const int* __restrict__ row_src,
                                                          const int* __restrict__ total_rows,
                                                          const int* __restrict__ send_count,
                                                          __nv_bfloat16* __restrict__ xp, int fp8 = 0) {
  // every block first waits for all peers' headers of this phase
  if (threadIdx.x < a.W) {
    const int src = threadIdx.x;
    if (src != a.rank) {
      const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
      const uint64_t* hdr = reinterpret_cast<const uint64_t*>(base + a.off_hdr) + (size_t)a.phase * a.W + src;
      uint32_t rows;
      wait_header(hdr, ep_epoch(a), &rows, a.status, a.timeout_ns);
    }
  }
  __syncthreads();
  (void)send_count;
  const int vec = a.H / 8;
  const int lane = threadIdx.x & 31;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int R = *total_rows;
  for (int p = gwarp; p < R; p += nw) {
    const int code = row_src[p];
    uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)p * a.H);
    if (code < 0) {
      for (int c = lane; c < vec; c += 32) dst[c] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const int src = code / a.cap, s = code % a.cap;
    if (fp8 && src != a.rank) {
      const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
      const uint2* q = reinterpret_cast<const uint2*>(base + a.off_recv_q) + ((size_t)src * a.cap + s) * vec;
      const float* sc = reinterpret_cast<const float*>(base + a.off_recv_s) + ((size_t)src * a.cap + s) * (a.H / 128);
      for (int c = lane; c < vec; c += 32) {
        const uint2 w = q[c];
        const float scale = sc[c / 16];
        const uint32_t ww[2] = {w.x, w.y};
        uint32_t o[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)((ww[h] >> (16 * e)) & 0xFFFF), __NV_E4M3);
            float2 f = __half22float2(*reinterpret_cast<__half2*>(&hr));
            o[2 * h + e] = pack_bf16x2(f.x * scale, f.y * scale);
          }
        }
        dst[c] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      continue;
    }
    const uint4* srow;
    if (src == a.rank) {
      srow = reinterpret_cast<const uint4*>(x + (size_t)self_tok[s] * a.H);
    } else {
      const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
      srow = reinterpret_cast<const uint4*>(base + a.off_recv_x) + ((size_t)src * a.cap + s) * vec;
    }
    for (int c = lane; c < vec; c += 32) dst[c] = srow[c];
  }
}

// ------------------------------------------------------------------------------------
// K6: combine. For each received (src, slot): out = sum_j scale_j * y[inv_rows[j]]
// (scale_j = gate weight in the forward, 1 in the backward), one bf16 partial row
// returned to the source's ret_x[rank][slot]; optional per-choice values (router-weight
// gradients) returned to ret_w.
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) combine_kernel(EpArgs a, const __nv_bfloat16* __restrict__ y,
                                                      const int* __restrict__ inv_rows,
                                                      const float* __restrict__ row_w,
                                                      const int* __restrict__ rows_from,
                                                      int weighted, const float* __restrict__ row_val,
                                                      int* __restrict__ done_rows) {
  const int lane = threadIdx.x & 31;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int vec = a.H / 8;
  // Work items (src, slot) run slot-major, and each warp visits the sources in an order
  // rotated by its own index and this rank: at any moment the warps of every rank write to
  // all destinations at once, instead of every rank streaming into the same peer (which
  // would leave one NVLink ingress saturated and the others idle).
  int max_rows = 0;
  for (int src = 0; src < a.W; ++src) max_rows = max(max_rows, rows_from[src]);
  for (int s = gwarp; s < max_rows; s += nw) {
    for (int i = 0; i < a.W; ++i) {
      const int src = (a.rank + 1 + i + gwarp) % a.W;
      if (s >= rows_from[src]) continue;
      char* dbase = reinterpret_cast<char*>(a.peer_base[src]);
      uint4* ret = reinterpret_cast<uint4*>(dbase + a.off_ret_x) + (size_t)a.rank * a.cap * vec;
      const int* inv = inv_rows + ((size_t)src * a.cap + s) * a.k;
      int plist[8];
      float wl[8];
      int np = 0;
      for (int j = 0; j < a.k && j < 8; ++j) {
        int p = inv[j];
        if (p >= 0) {
          plist[np] = p;
          wl[np] = weighted ? row_w[p] : 1.f;
          ++np;
        }
      }
      if (row_val && lane < a.k) {
        int p = inv[lane];
        float* rw = reinterpret_cast<float*>(dbase + a.off_ret_w) + ((size_t)a.rank * a.cap + s) * a.k;
        rw[lane] = p >= 0 ? row_val[p] : 0.f;
      }
      // all of a slot's expert rows are loaded before any accumulation (up to 8 x 16 B in
      // flight per lane per chunk)
      for (int c = lane; c < vec; c += 32) {
        uint4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (q < np) v[q] = reinterpret_cast<const uint4*>(y + (size_t)plist[q] * a.H)[c];
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (q >= np) break;
          float2 f0 = unpack_bf16x2(v[q].x), f1 = unpack_bf16x2(v[q].y), f2 = unpack_bf16x2(v[q].z),
                 f3 = unpack_bf16x2(v[q].w);
          const float w = wl[q];
          acc[0] += w * f0.x; acc[1] += w * f0.y; acc[2] += w * f1.x; acc[3] += w * f1.y;
          acc[4] += w * f2.x; acc[5] += w * f2.y; acc[6] += w * f3.x; acc[7] += w * f3.y;
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]);
        o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]);
        o.w = pack_bf16x2(acc[6], acc[7]);
        ret[(size_t)s * vec + c] = o;
      }
    }
  }
  publish_last_cta(a.done_counter, a, a.phase, rows_from, true);
  (void)done_rows;
}

// ------------------------------------------------------------------------------------
// K7: source reduce. out[t] = sum_d ret_x[d][slot[t][d]] over the ranks t was sent to,
// in rank order (deterministic), plus optional residual; per-choice values gathered
// back into val[t][j] from the rank that owns choice j.
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) source_reduce_kernel(EpArgs a, const int* __restrict__ slot,
                                                            const int* __restrict__ dst_tk,
                                                            const __nv_bfloat16* __restrict__ residual,
                                                            __nv_bfloat16* __restrict__ out,
                                                            float* __restrict__ val) {
  if (threadIdx.x < a.W) {
    const int d = threadIdx.x;
    const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
    const uint64_t* hdr = reinterpret_cast<const uint64_t*>(base + a.off_hdr) + (size_t)a.phase * a.W + d;
    uint32_t rows;
    wait_header(hdr, ep_epoch(a), &rows, a.status, a.timeout_ns);
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int vec = a.H / 8;
  const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
  const uint4* ret = reinterpret_cast<const uint4*>(base + a.off_ret_x);
  const float* retw = reinterpret_cast<const float*>(base + a.off_ret_w);
  for (int t = gwarp; t < a.T; t += nw) {
    int sl[kMaxW];
    for (int d = 0; d < a.W; ++d) sl[d] = __ldg(slot + (size_t)t * a.W + d);
    if (val && lane < a.k) {
      const int j = lane;
      const int d = __ldg(dst_tk + t * a.k + j);
      val[t * a.k + j] = d >= 0 ? retw[((size_t)d * a.cap + sl[d]) * a.k + j] : 0.f;
    }
    for (int c = lane; c < vec; c += 32) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (residual) {
        uint4 v = reinterpret_cast<const uint4*>(residual + (size_t)t * a.H)[c];
        float2 f0 = unpack_bf16x2(v.x), f1 = unpack_bf16x2(v.y), f2 = unpack_bf16x2(v.z), f3 = unpack_bf16x2(v.w);
        acc[0] = f0.x; acc[1] = f0.y; acc[2] = f1.x; acc[3] = f1.y;
        acc[4] = f2.x; acc[5] = f2.y; acc[6] = f3.x; acc[7] = f3.y;
      }
      for (int d = 0; d < a.W; ++d) {
        if (sl[d] < 0) continue;
        uint4 v = ret[((size_t)d * a.cap + sl[d]) * vec + c];
        float2 f0 = unpack_bf16x2(v.x), f1 = unpack_bf16x2(v.y), f2 = unpack_bf16x2(v.z), f3 = unpack_bf16x2(v.w);
        acc[0] += f0.x; acc[1] += f0.y; acc[2] += f1.x; acc[3] += f1.y;
        acc[4] += f2.x; acc[5] += f2.y; acc[6] += f3.x; acc[7] += f3.y;
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      reinterpret_cast<uint4*>(out + (size_t)t * a.H)[c] = o;
    }
  }
}

// ------------------------------------------------------------------------------------
// K5 + K7 on one rank (W == 1): every expert row is local, so each token's gate-weighted
// sum goes straight to out, plus the residual, with no return slab, no header and no
// second kernel. The sum is rounded to bf16 before the residual is added, as the combine
// and source-reduce kernels do, so the result has the same bits as that pair.
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) local_combine_kernel(EpArgs a, const __nv_bfloat16* __restrict__ y,
                                                            const int* __restrict__ inv_rows,
                                                            const float* __restrict__ row_w,
                                                            const int* __restrict__ slot,
                                                            const int* __restrict__ dst_tk, int weighted,
                                                            const float* __restrict__ row_val,
                                                            const __nv_bfloat16* __restrict__ residual,
                                                            __nv_bfloat16* __restrict__ out,
                                                            float* __restrict__ val) {
  const int lane = threadIdx.x & 31;
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int vec = a.H / 8;
  for (int t = gwarp; t < a.T; t += nw) {
    const int s = __ldg(slot + t);
    const int* inv = inv_rows + (size_t)(s < 0 ? 0 : s) * a.k;
    int plist[8];
    float wl[8];
    int np = 0;
    if (s >= 0) {
      for (int j = 0; j < a.k && j < 8; ++j) {
        const int p = inv[j];
        if (p >= 0) {
          plist[np] = p;
          wl[np] = weighted ? row_w[p] : 1.f;
          ++np;
        }
      }
    }
    if (val && lane < a.k) {
      const int j = lane;
      const int p = (s >= 0 && __ldg(dst_tk + t * a.k + j) >= 0) ? inv[j] : -1;
      val[t * a.k + j] = p >= 0 ? row_val[p] : 0.f;
    }
    for (int c = lane; c < vec; c += 32) {
      uint4 v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q < np) v[q] = reinterpret_cast<const uint4*>(y + (size_t)plist[q] * a.H)[c];
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (q >= np) break;
        float2 f0 = unpack_bf16x2(v[q].x), f1 = unpack_bf16x2(v[q].y), f2 = unpack_bf16x2(v[q].z),
               f3 = unpack_bf16x2(v[q].w);
        const float w = wl[q];
        acc[0] += w * f0.x; acc[1] += w * f0.y; acc[2] += w * f1.x; acc[3] += w * f1.y;
        acc[4] += w * f2.x; acc[5] += w * f2.y; acc[6] += w * f3.x; acc[7] += w * f3.y;
      }
      float r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (residual) {
        const uint4 x = reinterpret_cast<const uint4*>(residual + (size_t)t * a.H)[c];
        float2 f0 = unpack_bf16x2(x.x), f1 = unpack_bf16x2(x.y), f2 = unpack_bf16x2(x.z), f3 = unpack_bf16x2(x.w);
        r[0] = f0.x; r[1] = f0.y; r[2] = f1.x; r[3] = f1.y;
        r[4] = f2.x; r[5] = f2.y; r[6] = f3.x; r[7] = f3.y;
      }
      if (s >= 0) {  // the partial as the two-kernel path stores it (bf16), then the sum
        const uint32_t pk[4] = {pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7])};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(pk[e]);
          r[2 * e] += f.x;
          r[2 * e + 1] += f.y;
        }
      }
      uint4 o;
      o.x = pack_bf16x2(r[0], r[1]);
      o.y = pack_bf16x2(r[2], r[3]);
      o.z = pack_bf16x2(r[4], r[5]);
      o.w = pack_bf16x2(r[6], r[7]);
      reinterpret_cast<uint4*>(out + (size_t)t * a.H)[c] = o;
    }
  }
}

// =====================================================================================
// launchers
// =====================================================================================
static void check_launch(const char* what) {
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

void ep_route_plan(const int* dst_tk, int T, int k, int W, int* slot, int* send_count, cudaStream_t st,
                   int* self_tok, int rank) {
  if (W > kMaxW) throw std::runtime_error("EP world size above 64 is not supported");
  if (k == 8 && (reinterpret_cast<uintptr_t>(dst_tk) & 15) == 0)
    route_plan_kernel<8><<<1, 1024, 0, st>>>(dst_tk, T, k, W, slot, send_count, self_tok, rank);
  else
    route_plan_kernel<0><<<1, 1024, 0, st>>>(dst_tk, T, k, W, slot, send_count, self_tok, rank);
  check_launch("route_plan");
}

void ep_route_tables(const int* topk_e, const int* e2r, const int* e2l, int n, int* dst, int* meta, cudaStream_t st) {
  route_tables_kernel<<<std::min((n + 255) / 256, 1024), 256, 0, st>>>(topk_e, e2r, e2l, n, dst, meta);
  check_launch("route_tables");
}

// Grid of the warp-per-token / warp-per-slot kernels: one warp per slot of the
// communicator's capacity (8 per CTA), at most two CTAs per SM. It depends only on the
// capacity, never on a call's token count, because the last-CTA publish counts
// completions modulo the grid size on a counter that persists across calls.
static int ep_grid(const EpArgs& a) {
  const int want = (a.cap + 7) / 8;
  return std::max(1, std::min(sm_count() * 2, want));
}

void ep_dispatch(const EpArgs& a, const void* x, const int* dst_tk, const int* meta_tk, const float* topk_w,
                 const int* slot, int* self_tok, const int* send_count, bool with_meta, cudaStream_t st, bool fp8) {
  if (fp8 && (a.H % 128 || a.off_recv_q == 0)) throw std::runtime_error("fp8 dispatch needs H % 128 == 0 and fp8 slabs");
  if (a.H % 8) throw std::runtime_error("hidden size must be a multiple of 8");
  if (a.k > 32) throw std::runtime_error("top-k above 32 is not supported");
  const int blocks = ep_grid(a);
  dispatch_kernel<<<blocks, 256, 0, st>>>(a, reinterpret_cast<const __nv_bfloat16*>(x), dst_tk, meta_tk, topk_w,
                                          slot, self_tok, send_count, with_meta ? 1 : 0, fp8 ? 1 : 0);
  check_launch("dispatch");
}

void ep_recv_count_scan(const EpArgs& a, const int* dst_tk, const int* meta_tk, const float* topk_w,
                        const int* self_tok, const int* send_count, int G, int cap_rows, int* rows_from,
                        int* chunk_cnt, int* group_off, int* group_cnt, int* pad_off, cudaStream_t st,
                        int* need, int* miss) {
  if (G > 1024) throw std::runtime_error("at most 1024 local experts");
  if (a.k > 8) throw std::runtime_error("top-k above 8 is not supported by the permute kernel");
  const int nchunks = ((a.cap + kChunk - 1) / kChunk) * a.W;
  const bool staged = nchunks * G <= kScanSmemEntries;
  recv_count_kernel<<<nchunks, kChunk, 0, st>>>(a, dst_tk, topk_w, self_tok, meta_tk, send_count, rows_from,
                                                chunk_cnt, G);
  check_launch("recv_count");
  recv_scan_kernel<<<1, 1024, staged ? scan_smem_words(nchunks * G) * sizeof(int) : 0, st>>>(
      a, chunk_cnt, nchunks, G, group_off, group_cnt, pad_off, cap_rows, need, miss, staged ? 1 : 0);
  check_launch("recv_scan");
}

void ep_recv_permute_gather(const EpArgs& a, const void* x, const int* dst_tk, const int* meta_tk,
                            const float* topk_w, const int* self_tok, const int* send_count, int G,
                            const int* rows_from, const int* chunk_cnt, const int* group_off, const int* group_cnt,
                            const int* pad_off, void* xp, float* row_w, int* row_src, int* inv_rows,
                            cudaStream_t st, bool fp8) {
  const int nchunks = ((a.cap + kChunk - 1) / kChunk) * a.W;
  recv_permute_kernel<<<nchunks, kChunk, 0, st>>>(a, reinterpret_cast<const __nv_bfloat16*>(x), dst_tk, topk_w,
                                                  self_tok, meta_tk, rows_from, chunk_cnt, G, group_off, group_cnt,
                                                  pad_off, reinterpret_cast<__nv_bfloat16*>(xp), row_w, row_src,
                                                  inv_rows);
  check_launch("recv_permute");
  recv_gather_kernel<<<sm_count() * 4, 256, 0, st>>>(a, reinterpret_cast<const __nv_bfloat16*>(x), self_tok, row_src,
                                                     group_off + G, send_count, reinterpret_cast<__nv_bfloat16*>(xp),
                                                     fp8 ? 1 : 0);
  check_launch("recv_gather");
}

void ep_recv_gather(const EpArgs& a, const void* x, const int* self_tok, const int* row_src, const int* total_rows,
                    const int* send_count, void* xp, int cap_rows, cudaStream_t st) {
  int blocks = sm_count() * 4;
  (void)cap_rows;
  recv_gather_kernel<<<blocks, 256, 0, st>>>(a, reinterpret_cast<const __nv_bfloat16*>(x), self_tok, row_src,
                                             total_rows, send_count, reinterpret_cast<__nv_bfloat16*>(xp));
  check_launch("recv_gather");
}

// Waits for every source's header of this phase; rows_from[src] = rows it sent.
__global__ void wait_rows_kernel(EpArgs a, const int* __restrict__ send_count, int* __restrict__ rows_from) {
  const int src = threadIdx.x;
  if (src >= a.W) return;
  uint32_t rows = 0;
  if (src == a.rank) {
    rows = (uint32_t)send_count[a.rank];
  } else {
    const char* base = reinterpret_cast<const char*>(a.peer_base[a.rank]);
    const uint64_t* hdr = reinterpret_cast<const uint64_t*>(base + a.off_hdr) + (size_t)a.phase * a.W + src;
    if (!wait_header(hdr, ep_epoch(a), &rows, a.status, a.timeout_ns)) rows = 0;
  }
  rows_from[src] = (int)min(rows, (uint32_t)a.cap);
}

void ep_wait_rows(const EpArgs& a, const int* send_count, int* rows_from, cudaStream_t st) {
  wait_rows_kernel<<<1, 64, 0, st>>>(a, send_count, rows_from);
  check_launch("wait_rows");
}

void ep_combine(const EpArgs& a, const void* y, const int* inv_rows, const float* row_w, const int* rows_from,
                bool weighted, const float* row_val, cudaStream_t st) {
  const int blocks = ep_grid(a);
  combine_kernel<<<blocks, 256, 0, st>>>(a, reinterpret_cast<const __nv_bfloat16*>(y), inv_rows, row_w, rows_from,
                                         weighted ? 1 : 0, row_val, nullptr);
  check_launch("combine");
}

void ep_combine_local(const EpArgs& a, const void* y, const int* inv_rows, const float* row_w, const int* slot,
                      const int* dst_tk, bool weighted, const float* row_val, const void* residual, void* out,
                      float* val, cudaStream_t st) {
  if (a.W != 1) throw std::runtime_error("the local combine is for world size 1");
  if (a.k > 8) throw std::runtime_error("top-k above 8 is not supported by the combine");
  if (a.T == 0) return;
  const int blocks = std::max(1, std::min(sm_count() * 2, (a.T + 7) / 8));
  local_combine_kernel<<<blocks, 256, 0, st>>>(a, reinterpret_cast<const __nv_bfloat16*>(y), inv_rows, row_w, slot,
                                               dst_tk, weighted ? 1 : 0, row_val,
                                               reinterpret_cast<const __nv_bfloat16*>(residual),
                                               reinterpret_cast<__nv_bfloat16*>(out), val);
  check_launch("local_combine");
}

void ep_source_reduce(const EpArgs& a, const int* slot, const int* dst_tk, const void* residual, void* out,
                      float* val, cudaStream_t st) {
  const int blocks = ep_grid(a);
  source_reduce_kernel<<<blocks, 256, 0, st>>>(a, slot, dst_tk, reinterpret_cast<const __nv_bfloat16*>(residual),
                                               reinterpret_cast<__nv_bfloat16*>(out), val);
  check_launch("source_reduce");
}

}  // namespace sepx

// =====================================================================================
// Allocation-free variant of the world-size-1 dispatch (declared in moe_noalloc.h; it has
// no counterpart in the reference). Every temporary lives in one static device array;
// the entry point calls no allocator. See moe_noalloc.h for limits and semantics.
// =====================================================================================
#include <cstdio>
#include <mutex>

#include "moe_noalloc.h"

namespace {

constexpr int kNaMaxT = 8192;
constexpr int kNaMaxE = 256;
constexpr int kNaMaxChunks = kNaMaxT / sepx::kChunk;
// word offsets inside the scratch array
constexpr int kNaSlot = 0;                              // [T]   slot of each token (all go to rank 0)
constexpr int kNaSelfTok = kNaSlot + kNaMaxT;           // [T]   slot -> token
constexpr int kNaSendCount = kNaSelfTok + kNaMaxT;      // [1]
constexpr int kNaRowsFrom = kNaSendCount + 64;          // [1]
constexpr int kNaGroupCnt = kNaRowsFrom + 64;           // [E]
constexpr int kNaPadOff = kNaGroupCnt + kNaMaxE;        // [E + 1]
constexpr int kNaDst = kNaPadOff + kNaMaxE + 64;        // [T * 8] destination of each choice (all 0)
constexpr int kNaChunkCnt = kNaDst + kNaMaxT * 8;       // [chunks * E]
constexpr int kNaWords = kNaChunkCnt + kNaMaxChunks * kNaMaxE;  // 98,944 words = 395,776 bytes

}  // namespace

static __device__ __align__(256) int g_sepx_noalloc_scratch[kNaWords];

namespace {

__global__ void noalloc_init_kernel(int* scratch, int T, int k) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kNaMaxT * 8; i += gridDim.x * blockDim.x) {
    if (i < T) scratch[kNaSelfTok + i] = i;  // world size 1: token t has slot t
    if (i < T * k) scratch[kNaDst + i] = 0;   // every choice stays on this GPU
  }
}

// The scratch array's device address on the current device. The address is looked up
// once per device and primary context: a cudaDeviceReset destroys the context (and the
// module holding the array), so the cache also remembers which context the address
// belongs to and looks it up again when the current context is a different one.
int* noalloc_scratch_for_current_device(int* dev_out) {
  static int* ptrs[64] = {nullptr};
  static CUcontext ctxs[64] = {nullptr};
  static std::mutex mu;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  *dev_out = dev;
  std::lock_guard<std::mutex> lock(mu);
  // cudaFree(0) makes the runtime create (or bind) this device's primary context, so the
  // driver call below sees it
  using CtxGetCurrent = CUresult (*)(CUcontext*);
  static CtxGetCurrent get_ctx = nullptr;
  if (!get_ctx) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return nullptr;
    get_ctx = reinterpret_cast<CtxGetCurrent>(fn);
  }
  CUcontext ctx = nullptr;
  if (cudaFree(nullptr) != cudaSuccess || get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return nullptr;
  if (!ptrs[dev] || ctxs[dev] != ctx) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_sepx_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
    ctxs[dev] = ctx;
  }
  return ptrs[dev];
}

int noalloc_fail(int code, const char* msg) {
  std::fprintf(stderr, "sepx_moe_permute_noalloc: %s (code %d)\n", msg, code);
  return code;
}

}  // namespace

extern "C" int sepx_moe_permute_noalloc(const void* x, const int* topk_e, const float* topk_w, int T, int k,
                                        int H, int E, void* xp, int cap_rows, int* group_off, float* row_w,
                                        int* row_src, int* inv_rows, int* status, cudaStream_t stream) {
  using namespace sepx;
  if (T < 1 || T > kNaMaxT) return noalloc_fail(1, "T must be in [1, 8192]");
  if (k < 1 || k > 8) return noalloc_fail(2, "k must be in [1, 8]");
  if (E < 1 || E > kNaMaxE) return noalloc_fail(3, "E must be in [1, 256]");
  if (H < 8 || H % 8) return noalloc_fail(4, "H must be a positive multiple of 8");
  if ((long long)cap_rows < (long long)T * k + 64LL * E) return noalloc_fail(5, "cap_rows must be >= T*k + 64*E");
  if (!x || !topk_e || !topk_w || !xp || !group_off || !row_w || !row_src || !inv_rows || !status)
    return noalloc_fail(6, "null pointer argument");
  // rows of x and xp are read and written as 16-byte vectors
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(xp)) & 15)
    return noalloc_fail(8, "x and xp must be 16-byte aligned");
  // an error left by earlier work on this thread is not ours: report it without clearing it
  if (cudaPeekAtLastError() != cudaSuccess)
    return noalloc_fail(9, "a CUDA error from earlier work is pending on this thread");
  int dev = -1;
  int* s = noalloc_scratch_for_current_device(&dev);
  if (!s) return noalloc_fail(7, "cudaGetSymbolAddress failed for the scratch array on the current device");

  const int nchunks = (T + kChunk - 1) / kChunk;
  EpArgs a;
  for (int i = 0; i < 64; ++i) a.peer_base[i] = nullptr;
  a.W = 1;
  a.rank = 0;
  a.cap = T;
  a.k = k;
  a.H = H;
  a.T = T;
  a.phase = 0;
  a.epoch = 0;
  a.status = status;

  cudaMemsetAsync(status, 0, sizeof(int), stream);
  noalloc_init_kernel<<<(kNaMaxT * 8 + 255) / 256, 256, 0, stream>>>(s, T, k);
  route_plan_kernel<0><<<1, 1024, 0, stream>>>(s + kNaDst, T, k, 1, s + kNaSlot, s + kNaSendCount);
  // local slot of each choice = its expert id (all experts on this GPU)
  recv_count_kernel<<<nchunks, kChunk, 0, stream>>>(a, s + kNaDst, topk_w, s + kNaSelfTok, topk_e,
                                                    s + kNaSendCount, s + kNaRowsFrom, s + kNaChunkCnt, E);
  recv_scan_kernel<<<1, 1024, 0, stream>>>(a, s + kNaChunkCnt, nchunks, E, group_off, s + kNaGroupCnt,
                                           s + kNaPadOff, cap_rows);
  recv_permute_kernel<<<nchunks, kChunk, 0, stream>>>(
      a, reinterpret_cast<const __nv_bfloat16*>(x), s + kNaDst, topk_w, s + kNaSelfTok, topk_e,
      s + kNaRowsFrom, s + kNaChunkCnt, E, group_off, s + kNaGroupCnt, s + kNaPadOff,
      reinterpret_cast<__nv_bfloat16*>(xp), row_w, row_src, inv_rows);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  recv_gather_kernel<<<(sms > 0 ? sms : 148) * 4, 256, 0, stream>>>(
      a, reinterpret_cast<const __nv_bfloat16*>(x), s + kNaSelfTok, row_src, group_off + E, s + kNaSendCount,
      reinterpret_cast<__nv_bfloat16*>(xp));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::fprintf(stderr, "sepx_moe_permute_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return 100 + (int)e;
  }
  return 0;
}
