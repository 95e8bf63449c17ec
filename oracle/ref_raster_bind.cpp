// Python binding of the reference's own binning/blend launchers (csrc/forward/rasterize.h and
// csrc/backward/rasterize_backward.h), which compile without GLM. TEST INFRASTRUCTURE ONLY:
// build_ref.py compiles this file together with the unmodified reference sources into
// oracle/_ref, and the parity tests use the module to pin the oracle and the CUDA path.
#include <torch/extension.h>

#include "backward/rasterize_backward.h"
#include "forward/rasterize.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("rasterize", &launch_rasterization, "reference tile binning + sort + alpha blend");
  m.def("backwards_rasterization", &launch_backward_rasterization, "reference blend backward");
}
