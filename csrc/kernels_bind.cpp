// Registration of the non-GEMM kernels and native runtime classes with the Python module.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <atomic>

#include "kernels.h"

namespace sepx {
static std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }
}  // namespace sepx

void register_ep_comm(pybind11::module& m);
void register_elementwise(pybind11::module& m);

namespace {
void trace_stamp(at::Tensor& ring, at::Tensor& counter, int64_t tag) {
  TORCH_CHECK(ring.is_cuda() && ring.scalar_type() == at::kLong && ring.is_contiguous() && ring.dim() == 2 &&
                  ring.size(1) == 2,
              "ring must be a contiguous [cap, 2] int64 CUDA tensor");
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt && counter.numel() == 1,
              "counter must be one int32 on the GPU");
  const c10::cuda::CUDAGuard g(ring.device());
  sepx::trace_stamp(reinterpret_cast<unsigned long long*>(ring.data_ptr<int64_t>()),
                    reinterpret_cast<unsigned int*>(counter.data_ptr<int>()), (int)ring.size(0), (int)tag,
                    at::cuda::getCurrentCUDAStream().stream());
}
}  // namespace

void register_kernels(pybind11::module& m) {
  m.def("launch_count", &sepx::launch_count, "kernels launched by this library so far");
  m.def("trace_stamp", &trace_stamp, "append (tag, device time) to a device timeline ring");
  register_ep_comm(m);
  register_elementwise(m);
}
