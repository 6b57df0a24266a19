// Test-only binding of the reference's own sparse-conv CUDA kernels.
//
// oracle/build_ref.py compiles this file together with the reference's unmodified
// BK/ops/libsparse/conv.cu, read in place from the reference checkout, into
// oracle/_ref/vdit_ref_libsparse.so.  The GPU parity tests use it as a checker (and print
// its timings beside ours); nothing in the product loads it.  The three entry points
// are the functions the reference's libsparse module binds as conv_indices, conv_fwd
// and dense_conv_fwd (BK/ops/libsparse/libsparse.cpp:626-633); their argument checks
// are the callers' job here.
#include <torch/extension.h>

#include <vector>

std::vector<torch::Tensor> conv_indices_cuda(torch::Tensor pos);
torch::Tensor conv_fwd_cuda(torch::Tensor feat, torch::Tensor weight, torch::Tensor bias,
                            std::vector<torch::Tensor> indices);
torch::Tensor dense_conv_fwd_cuda(torch::Tensor feat, torch::Tensor weight, torch::Tensor bias,
                                  std::vector<torch::Tensor> indices);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.def("conv_indices", &conv_indices_cuda, "27-neighbour indices (reference kernel)");
    m.def("conv_fwd", &conv_fwd_cuda, "depthwise 27-tap conv (reference kernel)");
    m.def("dense_conv_fwd", &dense_conv_fwd_cuda, "dense 27-tap conv (reference kernel)");
}
