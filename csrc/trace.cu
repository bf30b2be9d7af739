// Device-side stage timeline: a one-thread kernel appends (tag, %globaltimer ns) to a
// per-rank ring buffer at stage boundaries on the launching stream, so stage durations
// and overlaps come from the device clock without events or host round trips.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "kernels.h"
#include "sm100.cuh"

namespace sepx {

__global__ void trace_stamp_kernel(unsigned long long* ring, unsigned int* counter, int cap, int tag) {
  const unsigned int i = atomicAdd(counter, 1u) % (unsigned int)cap;
  ring[2 * (size_t)i] = (unsigned long long)(unsigned int)tag;
  ring[2 * (size_t)i + 1] = globaltimer_ns();
}

void trace_stamp(unsigned long long* ring, unsigned int* counter, int cap, int tag, cudaStream_t st) {
  if (cap < 1) throw std::runtime_error("trace ring needs at least one entry");
  trace_stamp_kernel<<<1, 1, 0, st>>>(ring, counter, cap, tag);
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("trace_stamp: ") + cudaGetErrorString(e));
}

}  // namespace sepx
