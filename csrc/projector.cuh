// Registration of the counter-based projection generator (projector.cu).
#pragma once

#include <torch/extension.h>

namespace bw {
void register_projector(pybind11::module& m);
}
