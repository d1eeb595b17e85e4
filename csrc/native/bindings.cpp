// Python bindings of the host-side C++ runtime (module swarm_inference_lab_b200._native):
// CPU SwiGLU / fp8 oracle, SWRING01 codec, paged-KV page allocator.
#include <torch/extension.h>

at::Tensor swiglu_f32(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&);
at::Tensor swiglu_bf16(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&);
at::Tensor swiglu_int4_g32(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                           const at::Tensor&, const at::Tensor&, const at::Tensor&,
                           const at::Tensor&);
at::Tensor fp8_block_gemm(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                          const at::Tensor&);
std::vector<at::Tensor> quant_fp8_1x128(const at::Tensor&);
at::Tensor e4m3_decode(const at::Tensor&);
pybind11::bytes ring_encode(int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                            const std::string&, const std::string&);
pybind11::tuple ring_decode(const std::string&);
void bind_page_allocator(pybind11::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "host-side runtime: CPU oracle kernels, SWRING01 codec, page allocator";
  m.def("swiglu_f32", &swiglu_f32);
  m.def("swiglu_bf16", &swiglu_bf16);
  m.def("swiglu_int4_g32", &swiglu_int4_g32);
  m.def("fp8_block_gemm", &fp8_block_gemm);
  m.def("quant_fp8_1x128", &quant_fp8_1x128);
  m.def("e4m3_decode", &e4m3_decode);
  m.def("ring_encode", &ring_encode);
  m.def("ring_decode", &ring_decode);
  bind_page_allocator(m);
}
