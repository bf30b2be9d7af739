// All-to-all peer write bandwidth over NVLink: the two ways a kernel can push rows into
// other GPUs' memory, measured on the same pattern as the expert-parallel dispatch (every
// rank writes its share to every other rank at once, 4 KB rows, destinations interleaved).
//   mode 0  SM stores: each lane loads 16-byte vectors of the row and stores them to the
//           peer address (what dispatch_kernel / combine_kernel do)
//   mode 1  TMA bulk copies: one lane per warp loads the row into shared memory with
//           cp.async.bulk and stores it to the peer with cp.async.bulk (4 rows in flight
//           per warp); no vector registers hold the data
// Used by benchmarks/p2p_store.py to choose the store path of the EP kernels.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "kernels.h"
#include "sm100.cuh"

namespace sepx {

constexpr int kRow = 4096;       // bytes per row
constexpr int kBulkSlots = 4;    // rows in flight per warp (mode 1)

__global__ void __launch_bounds__(256) p2p_write_kernel(P2PBenchArgs a) {
  extern __shared__ __align__(128) uint8_t p2p_smem[];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int peers = a.W - 1;
  const long long rows_per_peer = a.bytes_per_peer / kRow;
  const long long total = rows_per_peer * peers;
  if (a.mode == 0) {
    for (long long c = gw; c < total; c += nw) {
      const int d = (a.rank + 1 + (int)(c % peers)) % a.W;
      const long long row = c / peers;
      const uint4* src = reinterpret_cast<const uint4*>(a.src + row * kRow);
      uint4* dst = reinterpret_cast<uint4*>(a.dst[d] + (long long)a.rank * a.bytes_per_peer + row * kRow);
      uint4 v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __ldg(src + i * 32 + lane);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i * 32 + lane] = v[i];
    }
  } else {
    uint8_t* slots = p2p_smem + wib * kBulkSlots * kRow;
    uint64_t* bars = reinterpret_cast<uint64_t*>(p2p_smem + (blockDim.x >> 5) * kBulkSlots * kRow) + wib * kBulkSlots;
    if (lane == 0)
      for (int s = 0; s < kBulkSlots; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    __syncwarp();
    if (lane == 0) {
      int it = 0;
      for (long long c = gw; c < total; c += nw, ++it) {
        const int s = it % kBulkSlots;
        const int d = (a.rank + 1 + (int)(c % peers)) % a.W;
        const long long row = c / peers;
        if (it >= kBulkSlots) bulk_wait_read<kBulkSlots - 1>();  // slot s free again
        mbar_arrive_expect_tx(&bars[s], kRow);
        bulk_load(slots + s * kRow, a.src + row * kRow, kRow, &bars[s]);
        const uint32_t parity = (uint32_t)(it / kBulkSlots) & 1u;
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&bars[s], parity)) {
          if (globaltimer_ns() - t0 > 2000000000ull) {  // bounded: report and stop
            record_error(a.status, kErrTimeoutMbar);
            bulk_wait_all();
            return;
          }
        }
        bulk_store(a.dst[d] + (long long)a.rank * a.bytes_per_peer + row * kRow, slots + s * kRow, kRow);
        bulk_commit();
      }
      bulk_wait_all();
    }
    __syncwarp();
  }
}

void p2p_write_bench(const P2PBenchArgs& a, int blocks, cudaStream_t st) {
  if (a.W < 2) throw std::runtime_error("p2p_write_bench needs at least 2 ranks");
  if (a.bytes_per_peer % kRow) throw std::runtime_error("bytes_per_peer must be a multiple of 4096");
  const size_t smem = a.mode == 1 ? (size_t)8 * kBulkSlots * kRow + 8 * kBulkSlots * 8 : 0;
  if (smem > 48 * 1024) {
    static unsigned long long done = 0;
    smem_optin_once(p2p_write_kernel, (int)smem, done);
  }
  p2p_write_kernel<<<blocks, 256, smem, st>>>(a);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("p2p_write_bench: ") + cudaGetErrorString(e));
}

}  // namespace sepx
