// Python binding of the reference's CUDA kernels for use as a checker.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/build_ref.py together with the
// reference's own kernel sources (read in place from the reference checkout,
// never copied) into oracle/_ref/.  The declarations below restate the
// signatures of the reference's headers (quantization_new/gemm/gemm_cuda.h,
// quantization_new/gemv/gemv_cuda.h, w8a8/*.h, rope_new/fused_rope_with_pos.h);
// the reference's own pybind.cpp cannot be used because it includes headers
// the reference does not ship.
#include <torch/extension.h>

torch::Tensor gemm_forward_cuda_new(torch::Tensor in_feats, torch::Tensor kernel, torch::Tensor scales,
                                    torch::Tensor zeros);
torch::Tensor gemv_forward_cuda_new(torch::Tensor in_feats, torch::Tensor kernel, torch::Tensor scaling_factors,
                                    torch::Tensor zeros, int m, int n, int k, int group_size);
void w8a8_gemm_forward_cuda(torch::Tensor in_feats, torch::Tensor kernel, torch::Tensor wscales,
                            torch::Tensor ascales, torch::Tensor out_feats);
void w8a8_gemm_fuse_bias_forward_cuda(torch::Tensor in_feats, torch::Tensor kernel, torch::Tensor wscales,
                                      torch::Tensor ascales, torch::Tensor out_feats, torch::Tensor bias);
void invoke_quant(torch::Tensor& out, torch::Tensor& input, torch::Tensor& scale);
void rms_norm_general(torch::Tensor& out, torch::Tensor& input, torch::Tensor& weight, torch::Tensor& bias,
                      torch::Tensor& scaling, float epsilon, bool use_per_token_quant);
void gelu_and_quant(torch::Tensor& out, torch::Tensor& input, torch::Tensor& scale_out, torch::Tensor& tmp);
at::Tensor fused_rope_with_pos_forward_func(const at::Tensor& input, const at::Tensor& freqs,
                                            const bool transpose_output_memory);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm_forward_cuda_new", &gemm_forward_cuda_new);
  m.def("gemv_forward_cuda_new", &gemv_forward_cuda_new);
  m.def("w8a8_gemm_forward_cuda", &w8a8_gemm_forward_cuda);
  m.def("w8a8_gemm_fuse_bias_forward_cuda", &w8a8_gemm_fuse_bias_forward_cuda);
  m.def("invoke_quant", &invoke_quant);
  m.def("rms_norm_general", &rms_norm_general, py::arg("out"), py::arg("input"), py::arg("weight"),
        py::arg("bias"), py::arg("scaling"), py::arg("epsilon"), py::arg("use_per_token_quant") = true);
  m.def("gelu_and_quant", &gelu_and_quant);
  m.def("fused_rope_with_pos_forward_func", &fused_rope_with_pos_forward_func);
}
