// Bindings of the SIMT kernels (filled per op family below).
#include <torch/extension.h>
#include "kernels_api.h"

void register_kernels(pybind11::module& m) {}
