// Registration of the non-GEMM kernels and native runtime classes with the Python module.
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

void register_kernels(pybind11::module& m) {
  m.def("launch_count", &sepx::launch_count, "kernels launched by this library so far");
  register_ep_comm(m);
  register_elementwise(m);
}
