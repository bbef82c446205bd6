// sf_torch_ext.cpp -- the thin PyTorch binding of the C ABI (include/sf_q4.h).
//
// Q4Linear.__call__ (siliconfer/model/q4_linear.py:49-68) reaches its kernel
// through the reference's pybind module (siliconfer/kernels/neon/
// bindings.cpp:97-150), which checks shapes, allocates the output and throws
// std::runtime_error on a mismatch.  This module is the same layer for torch
// tensors on the GPU: it checks devices, shapes and dtypes, allocates Y with
// torch, runs the library's entry point on torch's current CUDA stream and
// turns a status code into RuntimeError with the library's message.  No
// computation happens here.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <stdexcept>
#include <string>

#include "sf_q4.h"

namespace {

int dtype_code(const at::ScalarType t) {
  switch (t) {
    case at::kFloat: return SF_F32;
    case at::kHalf: return SF_F16;
    case at::kBFloat16: return SF_BF16;
    default: throw std::runtime_error("unsupported activation dtype (fp32, fp16 or bf16)");
  }
}

void check(int rc) {
  if (rc != SF_OK) throw std::runtime_error(std::string(sf_last_error()));
}

const void* ptr_or_null(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? t->data_ptr() : nullptr;
}

void check_weights(const at::Tensor& W, const at::Tensor& S, const c10::optional<at::Tensor>& Z,
                   const c10::optional<at::Tensor>& bias, const at::Tensor& X) {
  TORCH_CHECK(W.is_cuda() && S.is_cuda() && X.is_cuda(), "W, scales and X must be CUDA tensors");
  TORCH_CHECK(W.dim() == 2 && S.dim() == 2 && X.dim() == 2, "W, scales and X must be 2-D");
  TORCH_CHECK(W.scalar_type() == at::kByte && S.scalar_type() == at::kFloat, "W must be uint8, scales fp32");
  TORCH_CHECK(W.is_contiguous() && S.is_contiguous() && X.is_contiguous(), "tensors must be contiguous");
  TORCH_CHECK(W.get_device() == X.get_device() && S.get_device() == X.get_device(), "tensors on one device");
  if (Z.has_value() && Z->defined())
    TORCH_CHECK(Z->is_cuda() && Z->scalar_type() == at::kFloat && Z->is_contiguous() && Z->sizes() == S.sizes(),
                "zeros must be a contiguous fp32 CUDA tensor shaped like scales");
  if (bias.has_value() && bias->defined())
    TORCH_CHECK(bias->is_cuda() && bias->scalar_type() == at::kFloat && bias->is_contiguous(),
                "bias must be a contiguous fp32 CUDA tensor");
}

// Y[T, N] = X[T, K] @ dequant(W)^T (+ bias): sf_q4_linear (4 bits) or sf_q2_linear (2 bits).
at::Tensor linear(const at::Tensor& W, const at::Tensor& S, const c10::optional<at::Tensor>& Z,
                  const c10::optional<at::Tensor>& bias, const at::Tensor& X, int64_t group_size,
                  at::ScalarType out_dtype, int64_t bits, bool pdl) {
  check_weights(W, S, Z, bias, X);
  TORCH_CHECK(bits == 4 || bits == 2, "bits must be 4 or 2");
  const c10::cuda::CUDAGuard guard(X.device());
  const int64_t T = X.size(0), K = X.size(1), N = W.size(0);
  TORCH_CHECK(W.size(1) * (8 / bits) == K, "X/W in_features mismatch");
  at::Tensor Y = at::empty({T, N}, X.options().dtype(out_dtype));
  void* st = at::cuda::getCurrentCUDAStream(X.get_device()).stream();
  const auto* w = static_cast<const uint8_t*>(W.data_ptr());
  const auto* s = static_cast<const float*>(S.data_ptr());
  const auto* z = static_cast<const float*>(ptr_or_null(Z));
  const auto* b = static_cast<const float*>(ptr_or_null(bias));
  if (bits == 2)
    check(sf_q2_linear(w, s, z, b, X.data_ptr(), dtype_code(X.scalar_type()), Y.data_ptr(), dtype_code(out_dtype),
                       (int)N, (int)K, (int)T, (int)group_size, st));
  else
    check(sf_q4_linear(w, s, z, b, X.data_ptr(), dtype_code(X.scalar_type()), Y.data_ptr(), dtype_code(out_dtype),
                       (int)N, (int)K, (int)T, (int)group_size, pdl ? SF_FLAG_PDL : 0, st));
  return Y;
}

// silu(gate) * up over interleaved gate/up rows (sf_q4_linear_swiglu); W has 2N rows.
at::Tensor linear_swiglu(const at::Tensor& W, const at::Tensor& S, const c10::optional<at::Tensor>& Z,
                         const c10::optional<at::Tensor>& bias, const at::Tensor& X, int64_t group_size,
                         at::ScalarType out_dtype) {
  check_weights(W, S, Z, bias, X);
  const c10::cuda::CUDAGuard guard(X.device());
  const int64_t T = X.size(0), K = X.size(1), N = W.size(0) / 2;
  TORCH_CHECK(W.size(1) * 2 == K, "X/W in_features mismatch");
  at::Tensor Y = at::empty({T, N}, X.options().dtype(out_dtype));
  check(sf_q4_linear_swiglu(static_cast<const uint8_t*>(W.data_ptr()), static_cast<const float*>(S.data_ptr()),
                            static_cast<const float*>(ptr_or_null(Z)), static_cast<const float*>(ptr_or_null(bias)),
                            X.data_ptr(), dtype_code(X.scalar_type()), Y.data_ptr(), dtype_code(out_dtype), (int)N,
                            (int)K, (int)T, (int)group_size, at::cuda::getCurrentCUDAStream(X.get_device()).stream()));
  return Y;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "torch binding of libsf_q4 (include/sf_q4.h)";
  m.def("linear", &linear, "Y = X @ dequant(W)^T (+ bias) on the GPU", py::arg("W"), py::arg("scales"),
        py::arg("zeros"), py::arg("bias"), py::arg("X"), py::arg("group_size"), py::arg("out_dtype"),
        py::arg("bits") = 4, py::arg("pdl") = false);
  m.def("linear_swiglu", &linear_swiglu, "silu(gate) * up over interleaved gate/up rows", py::arg("W"),
        py::arg("scales"), py::arg("zeros"), py::arg("bias"), py::arg("X"), py::arg("group_size"),
        py::arg("out_dtype"));
}
