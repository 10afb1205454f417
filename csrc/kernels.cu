// Registration of every non-GEMM kernel family with the Python module.
#include "kernels.cuh"

namespace bw {

void register_projector(pybind11::module& m);

void register_kernels(pybind11::module& m) { register_projector(m); }

}  // namespace bw
