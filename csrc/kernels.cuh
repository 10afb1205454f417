// Registration hook for the non-GEMM kernels (random projections, fused
// reductions, top-k, norm / embedding per-sample gradients, optimizer maps).
#pragma once

#include <torch/extension.h>

namespace bw {
void register_kernels(pybind11::module& m);
}
