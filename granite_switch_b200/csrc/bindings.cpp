// Python bindings of the native extension granite_switch_b200._C.
// Every op launches on the current PyTorch CUDA stream of its inputs' device.
#include <torch/extension.h>

#include <vector>

#include "ops.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "granite_switch_b200 sm_100a kernels";
  m.def("switched_gemm", &gsb_switched_gemm, "tcgen05 GEMM with fused switched-LoRA expand");
}
