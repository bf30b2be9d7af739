// Speculative expert replication: a per-rank LRU cache of non-local experts, refilled
// from the experts' primary copies in peer memory, driven by a routing prediction.
//
// The reference only describes the scheme (docs/plan.md:3-21): predict which experts the
// next layer's tokens will use by applying its router to earlier activations, load the
// predicted experts onto the node, evict others LRU-first, and keep one copy of every
// expert that is never evicted. Here, per MoE layer and rank:
//
//   * primaries (and any static replicas) occupy local slots [0, P) and are never
//     evicted: they are the copies every other rank may fetch from;
//   * S cache slots [P, P + S) hold replicas of other ranks' experts;
//   * spec_policy_kernel (one block) turns predicted top-k expert ids into a want set
//     (the S most-predicted non-local experts with at least min_count predicted rows),
//     keeps cached experts that are wanted (hits), assigns each missing wanted expert
//     to the least recently used unwanted slot, and rewrites this rank's routing tables
//     so every cached expert is served by the local copy;
//   * spec_fetch_kernel copies the newly assigned experts' weights from their primary
//     rank's symmetric buffer (plain 16-byte peer loads over NVLink, no TMA) into the
//     cache slots.
//
// Everything stays on the device (no host sync); the only state is the cache map, its
// LRU stamps and a step counter, all device tensors. Replica slots are only ever read by
// this rank, primaries only ever written at load time, so a fetch needs no cross-rank
// synchronisation.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sepx {

namespace {
constexpr int kPolicyThreads = 1024;
constexpr int kMaxPolicyE = 1024;
constexpr int kMaxSlots = 256;
}  // namespace

// One block. Shared: per-expert predicted counts, want ranks, cache reverse map; per
// slot: hit flags, free order. Deterministic: ties break by expert id / slot index.
__global__ void __launch_bounds__(kPolicyThreads) spec_policy_kernel(SpecPolicyArgs a) {
  __shared__ int cnt[kMaxPolicyE];
  __shared__ int want_rank[kMaxPolicyE];  // rank among candidates, or INT_MAX
  __shared__ int cached_at[kMaxPolicyE];  // cache slot holding the expert, or -1
  __shared__ int miss_idx[kMaxPolicyE];   // order among missing wanted experts, or -1
  __shared__ unsigned char is_cand[kMaxPolicyE];  // not local in the base tables, enough rows
  __shared__ int slot_hit[kMaxSlots];
  __shared__ int slot_by_free[kMaxSlots];
  __shared__ int new_expert[kMaxSlots];
  __shared__ int s_hits, s_fetches, s_cand_rows, s_local_rows, s_free;
  const int E = a.E, S = a.S, tid = threadIdx.x;
  for (int e = tid; e < E; e += blockDim.x) {
    cnt[e] = 0;
    cached_at[e] = -1;
  }
  for (int s = tid; s < S; s += blockDim.x) new_expert[s] = -1;
  if (tid == 0) s_hits = s_fetches = s_cand_rows = s_local_rows = s_free = 0;
  __syncthreads();
  const int n = a.T * a.k;
  for (int i = tid; i < n; i += blockDim.x) {
    int e = a.pred_e[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  for (int s = tid; s < S; s += blockDim.x) {
    int e = a.slot_expert[s];
    if (e >= 0 && e < E) cached_at[e] = s;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x)
    is_cand[e] = (a.base_e2r[e] != a.rank && cnt[e] >= a.min_count && cnt[e] > 0) ? 1 : 0;
  __syncthreads();
  // want set: the S candidates (experts not local in the base tables) with the most
  // predicted rows, at least min_count of them
  for (int e = tid; e < E; e += blockDim.x) {
    int r = 0x7fffffff;
    const int c = cnt[e];
    if (is_cand[e]) {
      r = 0;
      for (int o = 0; o < E; ++o) {
        const int co = cnt[o];
        if (is_cand[o] && (co > c || (co == c && o < e))) ++r;
      }
      if (r >= S) r = 0x7fffffff;
    }
    want_rank[e] = r;
  }
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x) {
    int e = a.slot_expert[s];
    slot_hit[s] = (e >= 0 && e < E && want_rank[e] != 0x7fffffff) ? 1 : 0;
  }
  for (int e = tid; e < E; e += blockDim.x) {
    int m = -1;
    if (want_rank[e] != 0x7fffffff && cached_at[e] < 0) {
      m = 0;
      for (int o = 0; o < E; ++o)
        if (want_rank[o] != 0x7fffffff && cached_at[o] < 0 && want_rank[o] < want_rank[e]) ++m;
    }
    miss_idx[e] = m;
  }
  __syncthreads();
  // unwanted slots, least recently used first (never-used slots carry stamp -1)
  for (int s = tid; s < S; s += blockDim.x) {
    if (slot_hit[s]) continue;
    const int st = a.slot_stamp[s];
    int f = 0;
    for (int o = 0; o < S; ++o) {
      if (slot_hit[o]) continue;
      const int so = a.slot_stamp[o];
      if (so < st || (so == st && o < s)) ++f;
    }
    slot_by_free[f] = s;
    atomicAdd(&s_free, 1);
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    const int m = miss_idx[e];
    // #misses <= #unwanted slots whenever no expert is cached twice; a corrupted cache
    // map (an expert in two slots) only loses the surplus misses
    if (m >= 0 && m < s_free) new_expert[slot_by_free[m]] = e;
  }
  __syncthreads();
  const int now = a.step[0] + 1;
  for (int s = tid; s < S; s += blockDim.x) {
    const int e = new_expert[s];
    if (e >= 0) {
      a.fetch_rank[s] = a.owner[e];
      a.fetch_slot[s] = a.owner_slot[e];
      a.slot_expert[s] = e;
      a.slot_stamp[s] = now;
      atomicAdd(&s_fetches, 1);
    } else {
      a.fetch_rank[s] = -1;
      a.fetch_slot[s] = -1;
      if (slot_hit[s]) {
        a.slot_stamp[s] = now;
        atomicAdd(&s_hits, 1);
      }
    }
  }
  for (int e = tid; e < E; e += blockDim.x) {
    a.e2r[e] = a.base_e2r[e];
    a.e2l[e] = a.base_e2l[e];
  }
  __syncthreads();
  for (int s = tid; s < S; s += blockDim.x) {
    const int e = a.slot_expert[s];
    if (e >= 0 && e < E) {
      a.e2r[e] = a.rank;
      a.e2l[e] = a.P + s;
    }
  }
  __syncthreads();
  // predicted rows that the updated tables serve locally vs. all predicted rows of
  // experts that are not local in the base tables
  for (int e = tid; e < E; e += blockDim.x) {
    if (a.base_e2r[e] == a.rank) continue;
    atomicAdd(&s_cand_rows, cnt[e]);
    if (a.e2r[e] == a.rank) atomicAdd(&s_local_rows, cnt[e]);
  }
  __syncthreads();
  if (tid == 0) {
    a.step[0] = now;
    if (a.stats) {
      a.stats[0] += s_hits;
      a.stats[1] += s_fetches;
      a.stats[2] += s_cand_rows;
      a.stats[3] += s_local_rows;
    }
  }
}

// Grid (blocks_per_slot, S). Block (b, s) copies its share of every region of the
// expert assigned to slot s, or returns at once when the slot needs no fetch.
__global__ void __launch_bounds__(512) spec_fetch_kernel(SpecFetchArgs a) {
  const int s = blockIdx.y;
  const int src_rank = a.fetch_rank[s];
  if (src_rank < 0 || src_rank >= a.W) return;
  const int src_slot = a.fetch_slot[s];
  if (src_slot < 0 || src_slot >= a.src_limit) return;  // pinned slots only, within every peer's buffer
  const char* peer = reinterpret_cast<const char*>(a.peer_base[src_rank]);
  char* mine = reinterpret_cast<char*>(a.local_base);
  constexpr int kUnroll = 8;
  for (int r = 0; r < a.nreg; ++r) {
    const size_t stride = a.reg_stride[r];
    const uint4* src = reinterpret_cast<const uint4*>(peer + a.reg_off[r] + (size_t)src_slot * stride);
    uint4* dst = reinterpret_cast<uint4*>(mine + a.reg_off[r] + (size_t)(a.P + s) * stride);
    const size_t nvec = stride / 16;
    const size_t step = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + (kUnroll - 1) * step < nvec; i += kUnroll * step) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) v[u] = src[i + u * step];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) dst[i + u * step] = v[u];
    }
    for (; i < nvec; i += step) dst[i] = src[i];
  }
}

void spec_policy(const SpecPolicyArgs& a, cudaStream_t st) {
  if (a.E > kMaxPolicyE) throw std::runtime_error("speculative policy: at most 1024 experts");
  if (a.S < 1 || a.S > kMaxSlots) throw std::runtime_error("speculative policy: cache slots must be in [1, 256]");
  spec_policy_kernel<<<1, kPolicyThreads, 0, st>>>(a);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("spec_policy: ") + cudaGetErrorString(e));
}

void spec_fetch(const SpecFetchArgs& a, int blocks_per_slot, cudaStream_t st) {
  if (a.S < 1 || a.S > 65535) throw std::runtime_error("speculative fetch: bad slot count");
  if (a.nreg < 1 || a.nreg > 4) throw std::runtime_error("speculative fetch: 1 to 4 regions");
  for (int r = 0; r < a.nreg; ++r)
    if (a.reg_stride[r] % 16 || a.reg_off[r] % 16)
      throw std::runtime_error("speculative fetch: region offsets and strides must be multiples of 16 bytes");
  dim3 grid(blocks_per_slot < 1 ? 1 : blocks_per_slot, a.S);
  spec_fetch_kernel<<<grid, 512, 0, st>>>(a);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("spec_fetch: ") + cudaGetErrorString(e));
}

}  // namespace sepx
