// PyTorch binding of the sm_100a attention forward: the counterpart of the reference's
// src/mini_flash_attention/flash_attn.cpp (input validation with the same messages, output
// allocation, scale = 1/sqrt(D), device guard and current stream), calling the C ABI of
// include/mfa_b200.h instead of C++ launchers.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <cstdint>
#include <limits>
#include <stdexcept>

#include "mfa_b200.h"

namespace {

using LaunchFn = int (*)(const void*, const void*, const void*, void*, int64_t, int64_t, int32_t,
                         float, int32_t, void*);

// flash_attn.cpp:45-75. Differences: a 3-D [B*H, N, D] view is accepted next to [B, H, N, D]
// (same memory layout), and k / v must live on q's device.
void check_forward_inputs(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v) {
  TORCH_CHECK(q.is_cuda(), "q must be a CUDA tensor");
  TORCH_CHECK(k.is_cuda(), "k must be a CUDA tensor");
  TORCH_CHECK(v.is_cuda(), "v must be a CUDA tensor");

  TORCH_CHECK(q.scalar_type() == torch::kFloat16, "q must be float16");
  TORCH_CHECK(k.scalar_type() == torch::kFloat16, "k must be float16");
  TORCH_CHECK(v.scalar_type() == torch::kFloat16, "v must be float16");

  TORCH_CHECK(q.is_contiguous(), "q must be contiguous");
  TORCH_CHECK(k.is_contiguous(), "k must be contiguous");
  TORCH_CHECK(v.is_contiguous(), "v must be contiguous");

  TORCH_CHECK(q.dim() == 4 || q.dim() == 3, "q must have shape [B, H, N, D]");
  TORCH_CHECK(k.sizes() == q.sizes(), "k must have the same shape as q");
  TORCH_CHECK(v.sizes() == q.sizes(), "v must have the same shape as q");
  TORCH_CHECK(k.device() == q.device(), "k must be on the same device as q");
  TORCH_CHECK(v.device() == q.device(), "v must be on the same device as q");

  const int64_t BH = q.dim() == 4 ? q.size(0) * q.size(1) : q.size(0);
  const int64_t N = q.size(-2);
  const int64_t D = q.size(-1);
  TORCH_CHECK(D > 0, "D must be greater than 0");
  TORCH_CHECK(BH <= std::numeric_limits<int>::max(), "B * H is too large");
  TORCH_CHECK(N <= std::numeric_limits<int>::max(), "N is too large");
  TORCH_CHECK(D <= std::numeric_limits<int>::max(), "D is too large");
}

// flash_attn.cpp:77-109, with empty_like instead of zeros_like: the kernel writes every
// element of the output, so the extra memset pass of the reference is dropped.
torch::Tensor forward_impl(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                           bool causal, LaunchFn launch) {
  check_forward_inputs(q, k, v);
  const c10::cuda::CUDAGuard device_guard(q.device());
  auto out = torch::empty_like(q);

  const int64_t BH = q.dim() == 4 ? q.size(0) * q.size(1) : q.size(0);
  const int64_t N = q.size(-2);
  const int64_t D = q.size(-1);
  const float scale = 1.0f / std::sqrt(static_cast<float>(D));

  const int rc = launch(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), BH, N,
                        static_cast<int32_t>(D), scale, causal ? 1 : 0,
                        static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()));
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
  return out;
}

// Same as forward, writing into a caller-provided contiguous fp16 tensor of q's shape
// (used by the pipelined host-buffer path to fill slices of one device buffer).
void flash_attn_forward_into(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                             bool causal) {
  check_forward_inputs(q, k, v);
  TORCH_CHECK(out.is_cuda() && out.device() == q.device(), "out must be on q's device");
  TORCH_CHECK(out.scalar_type() == torch::kFloat16, "out must be float16");
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  TORCH_CHECK(out.sizes() == q.sizes(), "out must have the same shape as q");
  const c10::cuda::CUDAGuard device_guard(q.device());
  const int64_t BH = q.dim() == 4 ? q.size(0) * q.size(1) : q.size(0);
  const int64_t N = q.size(-2);
  const int64_t D = q.size(-1);
  const float scale = 1.0f / std::sqrt(static_cast<float>(D));
  const int rc = mfa_fwd_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), BH, N,
                             static_cast<int32_t>(D), scale, causal ? 1 : 0,
                             static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()));
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
}

torch::Tensor flash_attn_forward(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal) {
  return forward_impl(q, k, v, causal, &mfa_fwd_f16);
}

torch::Tensor flash_attn_forward_wmma(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                      bool causal) {
  return forward_impl(q, k, v, causal, &mfa_fwd_simple_f16);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &flash_attn_forward, "Mini Flash Attention forward (sm_100a tcgen05)");
  m.def("forward_wmma", &flash_attn_forward_wmma,
        "Mini Flash Attention forward, single-tile sm_100a kernel (replaces the WMMA path)");
  m.def("forward_into", &flash_attn_forward_into,
        "Mini Flash Attention forward into a preallocated output tensor");
  m.def("version", []() { return std::string(mfa_version()); });
}
