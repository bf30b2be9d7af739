// Registration of the non-GEMM kernels and native runtime classes with the Python module.
#include <torch/extension.h>

#include "kernels.h"

void register_ep_comm(pybind11::module& m);
void register_elementwise(pybind11::module& m);

void register_kernels(pybind11::module& m) {
  register_ep_comm(m);
  register_elementwise(m);
}
