// torch-tensor entry points of the peer-memory collective kernels.
#include <pybind11/pybind11.h>
#include <torch/extension.h>

namespace py = pybind11;

void register_comm_ops(py::module_& m) { (void)m; }
