// PyTorch extension `cuda_attn._C`: the reference's pybind entry points (csrc/bindings.cpp:40-54) with
// the same names, argument names and defaults, and the same input checks and error texts
// (bindings.cpp:12-22). Each entry allocates O with empty_like(q), as the reference wrappers did
// (csrc/attn_fused_tc.cu:15), and calls the C ABI of libphantom_attn on the current CUDA stream.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "../../include/phantom_attn.h"

namespace {

using CFn = int (*)(const void*, const void*, const void*, void*, int, int, int, int, int, void*);

int dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return PHANTOM_ATTN_F32;
    case at::kHalf: return PHANTOM_ATTN_F16;
    case at::kBFloat16: return PHANTOM_ATTN_BF16;
    default: return -1;
  }
}

void check_inputs(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v) {
  for (const auto* t : {&q, &k, &v}) {
    TORCH_CHECK(t->is_cuda(), "inputs must be CUDA tensors");
    TORCH_CHECK(t->is_contiguous(), "inputs must be contiguous");
    TORCH_CHECK(t->dim() == 4, "inputs must be shaped (B, H, N, d)");
    TORCH_CHECK(t->scalar_type() == q.scalar_type(), "q, k, v must share a dtype");
  }
  TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(), "q, k, v must have the same shape");
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device(), "q, k, v must be on the same device");
  TORCH_CHECK(q.numel() > 0, "inputs must be non-empty");
  TORCH_CHECK(dtype_code(q) >= 0, "inputs must be float32, float16 or bfloat16 (got ", q.scalar_type(), ")");
}

torch::Tensor call(CFn fn, const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, bool causal) {
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty_like(q);
  const int B = (int)q.size(0), H = (int)q.size(1), N = (int)q.size(2), d = (int)q.size(3);
  const int rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B * H, N, d, dtype_code(q),
                    causal ? 1 : 0, at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == PHANTOM_ATTN_OK, phantom_attn_last_error());
  return o;
}

template <CFn F>
torch::Tensor checked(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal) {
  check_inputs(q, k, v);
  return call(F, q, k, v, causal);
}

torch::Tensor checked_tuned(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal, bool double_buffer,
                            int64_t br, int64_t bc) {
  check_inputs(q, k, v);
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = torch::empty_like(q);
  const int B = (int)q.size(0), H = (int)q.size(1), N = (int)q.size(2), d = (int)q.size(3);
  const int rc = phantom_attn_fused_tuned(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), B * H, N, d,
                                          dtype_code(q), causal ? 1 : 0, double_buffer ? 1 : 0, (int)br, (int)bc,
                                          at::cuda::getCurrentCUDAStream().stream());
  TORCH_CHECK(rc == PHANTOM_ATTN_OK, phantom_attn_last_error());
  return o;
}

int device_status() {
  int status = 0;
  const int rc = phantom_attn_device_status(&status);
  TORCH_CHECK(rc == PHANTOM_ATTN_OK || rc == PHANTOM_ATTN_ERR_DEVICE, phantom_attn_last_error());
  return status;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) attention kernels: naive, tiled, fused, fused_tuned, fused_tc";
  m.def("naive", &checked<phantom_attn_naive>, "v1 entry point (fp32 CUDA-core fused kernel on sm_100a)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal") = false);
  m.def("tiled", &checked<phantom_attn_tiled>, "v2 entry point (fp32 CUDA-core fused kernel on sm_100a)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal") = false);
  m.def("fused", &checked<phantom_attn_fused>, "v3 fused online-softmax attention (fp32 CUDA cores)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal") = false);
  m.def("fused_tuned", &checked_tuned,
        "v3.1/v3.2 entry point; (br, bc) validated, runs on the tcgen05 tensor-core kernel (fp16/bf16)",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal") = false, py::arg("double_buffer") = true,
        py::arg("br") = 64, py::arg("bc") = 32);
  m.def("fused_tc", &checked<phantom_attn_fused_tc>,
        "v4 fused attention on tcgen05 tensor cores with TMEM accumulators (fp16/bf16, d 64/128)", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("causal") = false);
  m.def("device_status", &device_status, "read and clear the device status word (0 = no wait expired)");
}
