// PyTorch operators over the C ABI of libgemm.so (built as
// lib/libgemm_torch_op.so; load it with torch.ops.load_library).
//
// trtllm_gemm_sample::gemm(Tensor a, Tensor b) -> Tensor
//   Drop-in for the reference's TRT-LLM sample operator
//   (samples/trtllm_gemm/binding.cpp:17-60): same namespace, schema, argument
//   checks and messages, CUDA and Meta registrations, and the same
//   launchGemmSample call on the current PyTorch stream. The reference's
//   adapter (samples/trtllm_gemm/adapter.py:32-34, which loads
//   GEMM_SAMPLE_LIBRARY and calls torch.ops.trtllm_gemm_sample.gemm) runs on
//   this library unchanged.
// gemm_b200::gemm(Tensor a, Tensor b, Tensor? c=None, float alpha=1, float beta=0) -> Tensor
//   Any shape: alpha * a[M,K] @ b[K,N] + beta * c[M,N] (c required when
//   beta != 0; it is not modified), through gemm_launcher_ex's automatic path.
// gemm_b200::linear(Tensor x, Tensor w) -> Tensor
//   x[..., K] @ w[N, K]^T with the weight in its stored layout (the TN kernels:
//   no transposed copy of w, unlike adapter.py:50), any leading dims of x.
//
// Launch errors: libgemm.so links the CUDA runtime statically, so PyTorch's
// cudaGetLastError() does not see its launches; every operator asks the
// library instead (gemm_launch_error(), which never synchronizes and is safe
// inside CUDA graph capture).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cstdint>
#include <optional>

#include "gemm_b200.h"

namespace {

const gemm_half_t* in_ptr(const at::Tensor& t) {
  return reinterpret_cast<const gemm_half_t*>(t.const_data_ptr<at::Half>());
}

gemm_half_t* out_ptr(at::Tensor& t) {
  return reinterpret_cast<gemm_half_t*>(t.mutable_data_ptr<at::Half>());
}

void check_launch() {
  const int e = gemm_launch_error();
  TORCH_CHECK(e == 0, "gemm_b200 kernel launch failed (CUDA error ", e, ")");
}

cudaStream_t current_stream(const at::Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.get_device()).stream();
}

// --- trtllm_gemm_sample::gemm: the reference sample's operator ------------
at::Tensor sample_gemm(const at::Tensor& a, const at::Tensor& b) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && a.device() == b.device(), "CUDA device mismatch");
  TORCH_CHECK(a.scalar_type() == at::kHalf && b.scalar_type() == at::kHalf, "FP16 required");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(0), "Invalid GEMM dimensions");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous(), "Contiguous operands required");
  const auto m = a.size(0);
  const auto k = a.size(1);
  const auto n = b.size(1);
  TORCH_CHECK(m >= 1 && m <= 16 && n >= 512 && n % 64 == 0 && k >= 512 && k % 32 == 0,
              "Shape outside sample dispatch");
  TORCH_CHECK(((reinterpret_cast<std::uintptr_t>(a.data_ptr()) |
                reinterpret_cast<std::uintptr_t>(b.data_ptr())) &
               15U) == 0,
              "16-byte alignment required");
  const c10::cuda::CUDAGuard guard(a.device());
  auto output = at::empty({m, n}, a.options());
  const bool launched = launchGemmSample(in_ptr(a), in_ptr(b), out_ptr(output), static_cast<int>(m),
                                         static_cast<int>(n), static_cast<int>(k), current_stream(a));
  TORCH_CHECK(launched, "Supported dispatch did not launch");
  check_launch();
  return output;
}

at::Tensor sample_gemm_meta(const at::Tensor& a, const at::Tensor& b) {
  return at::empty({a.size(0), b.size(1)}, a.options());
}

// --- gemm_b200::gemm -------------------------------------------------------
void check_operand(const at::Tensor& t, const at::Tensor& ref, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.device() == ref.device(), name, " must be on ", ref.device());
  TORCH_CHECK(t.scalar_type() == at::kHalf, name, " must be float16");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous (row-major)");
}

at::Tensor gemm(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>& c,
                double alpha, double beta) {
  check_operand(a, a, "a");
  check_operand(b, a, "b");
  TORCH_CHECK(a.size(1) == b.size(0), "a is [M, K] and b [K, N]: inner sizes differ");
  const auto m = a.size(0), k = a.size(1), n = b.size(1);
  TORCH_CHECK(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX, "sizes must fit in int32");
  const c10::cuda::CUDAGuard guard(a.device());
  at::Tensor out;
  if (beta != 0.0) {
    TORCH_CHECK(c.has_value(), "beta != 0 needs c");
    check_operand(*c, a, "c");
    TORCH_CHECK(c->size(0) == m && c->size(1) == n, "c must be [M, N]");
    out = c->clone();
  } else {
    out = at::empty({m, n}, a.options());
  }
  const int rc = gemm_launcher_ex(in_ptr(a), in_ptr(b), out_ptr(out), static_cast<int>(m),
                                  static_cast<int>(n), static_cast<int>(k),
                                  static_cast<float>(alpha), static_cast<float>(beta),
                                  current_stream(a), /*path=*/0, /*tile_n=*/0);
  TORCH_CHECK(rc == 0, "gemm_b200 could not launch this shape");
  check_launch();
  return out;
}

at::Tensor gemm_meta(const at::Tensor& a, const at::Tensor& b, const std::optional<at::Tensor>&,
                     double, double) {
  return at::empty({a.size(0), b.size(1)}, a.options());
}

// --- gemm_b200::linear -------------------------------------------------------
at::Tensor linear(const at::Tensor& x, const at::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.device() == w.device(), "CUDA device mismatch");
  TORCH_CHECK(x.scalar_type() == at::kHalf && w.scalar_type() == at::kHalf, "FP16 required");
  TORCH_CHECK(x.dim() >= 1 && w.dim() == 2 && x.size(-1) == w.size(1),
              "x is [..., K] and w [N, K]: K differs");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous(), "Contiguous operands required");
  const auto k = w.size(1), n = w.size(0);
  const auto m = k > 0 ? x.numel() / k : 0;
  TORCH_CHECK(m <= INT32_MAX && n <= INT32_MAX && k <= INT32_MAX, "sizes must fit in int32");
  auto out_shape = x.sizes().vec();
  out_shape.back() = n;
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = at::empty(out_shape, x.options());
  if (m == 0 || n == 0) return out;
  if (k == 0) return out.zero_();
  const int rc = gemm_launcher_tn(in_ptr(x), in_ptr(w), out_ptr(out), static_cast<int>(m),
                                  static_cast<int>(n), static_cast<int>(k), 1.0f, 0.0f,
                                  current_stream(x), /*tile_n=*/0);
  TORCH_CHECK(rc == 0, "gemm_b200 could not launch this shape");
  check_launch();
  return out;
}

at::Tensor linear_meta(const at::Tensor& x, const at::Tensor& w) {
  auto out_shape = x.sizes().vec();
  out_shape.back() = w.size(0);
  return at::empty(out_shape, x.options());
}

}  // namespace

TORCH_LIBRARY(trtllm_gemm_sample, m) { m.def("gemm(Tensor a, Tensor b) -> Tensor"); }
TORCH_LIBRARY_IMPL(trtllm_gemm_sample, CUDA, m) { m.impl("gemm", &sample_gemm); }
TORCH_LIBRARY_IMPL(trtllm_gemm_sample, Meta, m) { m.impl("gemm", &sample_gemm_meta); }

TORCH_LIBRARY(gemm_b200, m) {
  m.def("gemm(Tensor a, Tensor b, Tensor? c=None, float alpha=1.0, float beta=0.0) -> Tensor");
  m.def("linear(Tensor x, Tensor w) -> Tensor");
}
TORCH_LIBRARY_IMPL(gemm_b200, CUDA, m) {
  m.impl("gemm", &gemm);
  m.impl("linear", &linear);
}
TORCH_LIBRARY_IMPL(gemm_b200, Meta, m) {
  m.impl("gemm", &gemm_meta);
  m.impl("linear", &linear_meta);
}
