// Python binding for the reference's own rms_norm, compiled from the reference's sources where
// they lie (see oracle/build.py). TEST INFRASTRUCTURE: loaded only by the tests, the smoke check
// and the CPU-baseline leg of bench.py, as the reference implementation to compare against.
#include <torch/extension.h>

#include "ops/rms_norm.h"

PYBIND11_MODULE(svllm_ref_ops, m) {
  m.def("rms_norm", &svllm::ops::rms_norm, pybind11::arg("x"), pybind11::arg("weight"),
        pybind11::arg("eps"));
}
