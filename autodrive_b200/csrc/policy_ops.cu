// Training-side kernels: registered into the same extension module.
#include <torch/extension.h>

namespace py = pybind11;

void register_policy_ops(py::module& m) { (void)m; }
