// Python binding for the reference's kt_moe_a8_vec_multi torch op, compiled together with the
// reference's own hot/kt_gguf_moe_multi/kt_gguf_moe_multi.cu by oracle/build_ref.py.
// TEST INFRASTRUCTURE ONLY: the GPU parity tests use the resulting module as the reference.
#include <torch/extension.h>

torch::Tensor kt_moe_a8_vec_multi(torch::Tensor X, torch::Tensor W, torch::Tensor topk_ids, int64_t top_k, int64_t type,
                                  int64_t row, int64_t tokens);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) { m.def("kt_moe_a8_vec_multi", &kt_moe_a8_vec_multi); }
