// Python bindings for the native extension syntropy_b200._C.
#include <torch/extension.h>

#include "ops.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "syntropy_b200 native runtime and sm_100a kernels";
  syn::register_all(m);
}
