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
#include <string>
#include <vector>

#include "mfa_b200.h"

namespace {

enum class Layout { kBHND, kBNHD };

// flash_attn.cpp:45-75. Differences: a 3-D [B*H, N, D] view is accepted next to [B, H, N, D]
// (same memory layout); k / v must live on q's device; with `allow_bf16` the three tensors may
// all be bf16 instead of fp16; the [B, N, H, D] entry point checks its own shape.
void check_forward_inputs(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                          bool allow_bf16, Layout layout) {
  TORCH_CHECK(q.is_cuda(), "q must be a CUDA tensor");
  TORCH_CHECK(k.is_cuda(), "k must be a CUDA tensor");
  TORCH_CHECK(v.is_cuda(), "v must be a CUDA tensor");

  if (allow_bf16) {
    TORCH_CHECK(q.scalar_type() == torch::kFloat16 || q.scalar_type() == torch::kBFloat16,
                "q must be float16 or bfloat16");
    TORCH_CHECK(k.scalar_type() == q.scalar_type(), "k must have the same dtype as q");
    TORCH_CHECK(v.scalar_type() == q.scalar_type(), "v must have the same dtype as q");
  } else {
    TORCH_CHECK(q.scalar_type() == torch::kFloat16, "q must be float16");
    TORCH_CHECK(k.scalar_type() == torch::kFloat16, "k must be float16");
    TORCH_CHECK(v.scalar_type() == torch::kFloat16, "v must be float16");
  }

  TORCH_CHECK(q.is_contiguous(), "q must be contiguous");
  TORCH_CHECK(k.is_contiguous(), "k must be contiguous");
  TORCH_CHECK(v.is_contiguous(), "v must be contiguous");

  if (layout == Layout::kBNHD) {
    TORCH_CHECK(q.dim() == 4, "q must have shape [B, N, H, D]");
  } else {
    TORCH_CHECK(q.dim() == 4 || q.dim() == 3, "q must have shape [B, H, N, D]");
  }
  TORCH_CHECK(k.sizes() == q.sizes(), "k must have the same shape as q");
  TORCH_CHECK(v.sizes() == q.sizes(), "v must have the same shape as q");
  TORCH_CHECK(k.device() == q.device(), "k must be on the same device as q");
  TORCH_CHECK(v.device() == q.device(), "v must be on the same device as q");

  const int64_t BH = q.dim() == 4 ? q.size(0) * q.size(layout == Layout::kBNHD ? 2 : 1)
                                  : q.size(0);
  const int64_t N = q.size(layout == Layout::kBNHD ? 1 : -2);
  const int64_t D = q.size(-1);
  TORCH_CHECK(D > 0, "D must be greater than 0");
  TORCH_CHECK(BH <= std::numeric_limits<int>::max(), "B * H is too large");
  TORCH_CHECK(N <= std::numeric_limits<int>::max(), "N is too large");
  TORCH_CHECK(D <= std::numeric_limits<int>::max(), "D is too large");
}

// The (B, H, N) of q for `layout` (3-D [B*H, N, D] counts as B = 1, H = B*H).
struct Extents {
  int64_t batch, heads, n, d;
};
Extents extents_of(const torch::Tensor& q, Layout layout) {
  if (layout == Layout::kBNHD) return {q.size(0), q.size(2), q.size(1), q.size(3)};
  if (q.dim() == 3) return {1, q.size(0), q.size(1), q.size(2)};
  return {q.size(0), q.size(1), q.size(2), q.size(3)};
}

void launch_general(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v,
                    torch::Tensor& out, bool causal, Layout layout) {
  const Extents e = extents_of(q, layout);
  const float scale = 1.0f / std::sqrt(static_cast<float>(e.d));
  const int dtype = q.scalar_type() == torch::kBFloat16 ? MFA_DTYPE_BF16 : MFA_DTYPE_FP16;
  const int rc = mfa_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), e.batch,
                         e.heads, e.n, static_cast<int32_t>(e.d), scale, causal ? 1 : 0, dtype,
                         layout == Layout::kBNHD ? MFA_LAYOUT_BNHD : MFA_LAYOUT_BHND,
                         static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()));
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
}

// flash_attn.cpp:77-109, with empty_like instead of zeros_like: the kernel writes every
// element of the output, so the extra memset pass of the reference is dropped. fp16 or bf16.
torch::Tensor flash_attn_forward(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal) {
  check_forward_inputs(q, k, v, true, Layout::kBHND);
  const c10::cuda::CUDAGuard device_guard(q.device());
  auto out = torch::empty_like(q);
  launch_general(q, k, v, out, causal, Layout::kBHND);
  return out;
}

// Same computation on [B, N, H, D] tensors (the flash-attn layout), output in that layout.
torch::Tensor flash_attn_forward_bnhd(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                      bool causal) {
  check_forward_inputs(q, k, v, true, Layout::kBNHD);
  const c10::cuda::CUDAGuard device_guard(q.device());
  auto out = torch::empty_like(q);
  launch_general(q, k, v, out, causal, Layout::kBNHD);
  return out;
}

// The WMMA entry point keeps the reference's fp16-only contract and launcher messages.
torch::Tensor flash_attn_forward_wmma(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                      bool causal) {
  check_forward_inputs(q, k, v, false, Layout::kBHND);
  const c10::cuda::CUDAGuard device_guard(q.device());
  auto out = torch::empty_like(q);
  const int64_t BH = q.dim() == 4 ? q.size(0) * q.size(1) : q.size(0);
  const int64_t N = q.size(-2);
  const int64_t D = q.size(-1);
  const float scale = 1.0f / std::sqrt(static_cast<float>(D));
  const int rc = mfa_fwd_simple_f16(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), BH,
                                    N, static_cast<int32_t>(D), scale, causal ? 1 : 0,
                                    static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()));
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
  return out;
}

// forward plus the row log-sum-exp (fp32 [B*H, N] viewed as q's leading dims + N).
std::vector<torch::Tensor> flash_attn_forward_lse(torch::Tensor q, torch::Tensor k,
                                                  torch::Tensor v, bool causal) {
  check_forward_inputs(q, k, v, true, Layout::kBHND);
  const c10::cuda::CUDAGuard device_guard(q.device());
  auto out = torch::empty_like(q);
  auto lse_shape = q.sizes().vec();
  lse_shape.pop_back();
  auto lse = torch::empty(lse_shape, q.options().dtype(torch::kFloat32));
  const Extents e = extents_of(q, Layout::kBHND);
  const float scale = 1.0f / std::sqrt(static_cast<float>(e.d));
  const int dtype = q.scalar_type() == torch::kBFloat16 ? MFA_DTYPE_BF16 : MFA_DTYPE_FP16;
  const int rc = mfa_fwd_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                             lse.data_ptr<float>(), e.batch, e.heads, e.n,
                             static_cast<int32_t>(e.d), scale, causal ? 1 : 0, dtype,
                             MFA_LAYOUT_BHND,
                             static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()));
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
  return {out, lse};
}

// Backward of forward: dq, dk, dv from q, k, v, out, lse (of forward_lse) and dout.
std::vector<torch::Tensor> flash_attn_backward(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                               torch::Tensor out, torch::Tensor lse,
                                               torch::Tensor dout, bool causal) {
  check_forward_inputs(q, k, v, true, Layout::kBHND);
  TORCH_CHECK(out.is_cuda() && out.device() == q.device() && dout.is_cuda() &&
                  dout.device() == q.device() && lse.is_cuda() && lse.device() == q.device(),
              "out, lse and dout must be on q's device");
  TORCH_CHECK(out.sizes() == q.sizes() && dout.sizes() == q.sizes(),
              "out and dout must have the same shape as q");
  TORCH_CHECK(out.scalar_type() == q.scalar_type() && dout.scalar_type() == q.scalar_type(),
              "out and dout must have q's dtype");
  TORCH_CHECK(out.is_contiguous() && dout.is_contiguous() && lse.is_contiguous(),
              "out, lse and dout must be contiguous");
  TORCH_CHECK(lse.scalar_type() == torch::kFloat32, "lse must be float32");
  TORCH_CHECK(lse.numel() * q.size(-1) == q.numel(), "lse must have one value per query row");
  const c10::cuda::CUDAGuard device_guard(q.device());
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  const Extents e = extents_of(q, Layout::kBHND);
  const float scale = 1.0f / std::sqrt(static_cast<float>(e.d));
  const int dtype = q.scalar_type() == torch::kBFloat16 ? MFA_DTYPE_BF16 : MFA_DTYPE_FP16;
  const int rc = mfa_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                         dout.data_ptr(), lse.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(),
                         dv.data_ptr(), e.batch, e.heads, e.n, static_cast<int32_t>(e.d), scale,
                         causal ? 1 : 0, dtype, MFA_LAYOUT_BHND,
                         static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()));
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
  return {dq, dk, dv};
}

// Same as forward, writing into a caller-provided contiguous tensor of q's shape and dtype
// (used by the pipelined host-buffer path to fill slices of one device buffer).
void flash_attn_forward_into(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                             bool causal) {
  check_forward_inputs(q, k, v, true, Layout::kBHND);
  TORCH_CHECK(out.is_cuda() && out.device() == q.device(), "out must be on q's device");
  TORCH_CHECK(out.scalar_type() == q.scalar_type(), "out must have q's dtype");
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  TORCH_CHECK(out.sizes() == q.sizes(), "out must have the same shape as q");
  const c10::cuda::CUDAGuard device_guard(q.device());
  launch_general(q, k, v, out, causal, Layout::kBHND);
}

// Query rows [q_begin, q_end) of every head of out ([B, H, N, D] or [B*H, N, D], the shape of
// q), each against all N keys (causal: the keys up to the row); the other rows of out are left
// as they are. A causal range starts at a multiple of 256 rows.
void flash_attn_forward_rows(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                             int64_t q_begin, int64_t q_end, bool causal) {
  check_forward_inputs(q, k, v, true, Layout::kBHND);
  TORCH_CHECK(out.is_cuda() && out.device() == q.device(), "out must be on q's device");
  TORCH_CHECK(out.scalar_type() == q.scalar_type(), "out must have q's dtype");
  TORCH_CHECK(out.is_contiguous(), "out must be contiguous");
  TORCH_CHECK(out.sizes() == q.sizes(), "out must have the same shape as q");
  const c10::cuda::CUDAGuard device_guard(q.device());
  const Extents e = extents_of(q, Layout::kBHND);
  const float scale = 1.0f / std::sqrt(static_cast<float>(e.d));
  const int dtype = q.scalar_type() == torch::kBFloat16 ? MFA_DTYPE_BF16 : MFA_DTYPE_FP16;
  const int rc = mfa_fwd_rows(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), e.batch,
                              e.heads, e.n, q_begin, q_end, static_cast<int32_t>(e.d), scale,
                              causal ? 1 : 0, dtype, MFA_LAYOUT_BHND,
                              static_cast<void*>(at::cuda::getCurrentCUDAStream().stream()));
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
}

// CUDA events of the pipelined calls, kept per calling thread and device from one call to the
// next: creating them costs several microseconds each, on the path before the first copy.
// Every call drains its streams before it returns, so the next call on the same thread may
// record them again; other threads have their own.
struct PipelineEvents {
  std::vector<cudaEvent_t> ev;
  ~PipelineEvents() {
    for (auto e : ev)
      if (e) cudaEventDestroy(e);
  }
};

// At least `count` events of `device` (current) for this thread.
const std::vector<cudaEvent_t>& pipeline_events(int64_t device, size_t count) {
  thread_local std::vector<PipelineEvents> per_device;
  if (per_device.size() <= static_cast<size_t>(device)) per_device.resize(device + 1);
  auto& ev = per_device[device].ev;
  while (ev.size() < count) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
      throw std::runtime_error("cudaEventCreateWithFlags failed");
    ev.push_back(e);
  }
  return ev;
}

void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// The host-buffer pipeline behind mini_flash_attention.forward_pinned in one call: q, k, v and
// out are contiguous host tensors [rows, N, D] (pinned for overlap), `bounds` cuts the rows into
// pieces. Piece i is copied in on one stream, computed on a second once it has arrived and
// copied back on a third once it is computed, so the copies of neighbouring pieces overlap the
// kernels. Returns when `out` holds the result. One plain cudaMemcpyAsync per tensor and piece.
void flash_attn_forward_pinned(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                               torch::Tensor out, bool causal, std::vector<int64_t> bounds,
                               int64_t device) {
  for (const auto* x : {&q, &k, &v, &out}) {
    TORCH_CHECK(!x->is_cuda(), "forward_pinned expects host tensors");
    TORCH_CHECK(x->is_contiguous(), "host tensors must be contiguous");
    TORCH_CHECK(x->dim() == 3, "host tensors must be [rows, N, D] views");
    TORCH_CHECK(x->sizes() == q.sizes(), "k must have the same shape as q");
    TORCH_CHECK(x->scalar_type() == q.scalar_type(), "k must have the same dtype as q");
  }
  TORCH_CHECK(q.scalar_type() == torch::kFloat16 || q.scalar_type() == torch::kBFloat16,
              "q must be float16 or bfloat16");
  const int64_t rows = q.size(0), n = q.size(1), d = q.size(2);
  TORCH_CHECK(bounds.size() >= 2 && bounds.front() == 0 && bounds.back() == rows,
              "bounds must run from 0 to the number of rows");
  for (size_t i = 1; i < bounds.size(); ++i)
    TORCH_CHECK(bounds[i] > bounds[i - 1], "bounds must increase");
  if (rows == 0 || n == 0) return;
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  const auto opts = q.options().device(torch::kCUDA, static_cast<c10::DeviceIndex>(device));
  auto dq = torch::empty({rows, n, d}, opts), dk = torch::empty({rows, n, d}, opts);
  auto dv = torch::empty({rows, n, d}, opts), dout = torch::empty({rows, n, d}, opts);
  const size_t pieces = bounds.size() - 1;
  const cudaStream_t cur = at::cuda::getCurrentCUDAStream().stream();
  const cudaStream_t s_in = at::cuda::getStreamFromPool().stream();
  const cudaStream_t s_run = at::cuda::getStreamFromPool().stream();
  const cudaStream_t s_out = at::cuda::getStreamFromPool().stream();
  const std::vector<cudaEvent_t>& ev = pipeline_events(device, 2 * pieces + 1);
  // the device buffers come from the caching allocator on the current stream
  check_cuda(cudaEventRecord(ev[2 * pieces], cur), "cudaEventRecord");
  check_cuda(cudaStreamWaitEvent(s_in, ev[2 * pieces], 0), "cudaStreamWaitEvent");
  const size_t row_bytes = static_cast<size_t>(n) * d * q.element_size();
  const float scale = 1.0f / std::sqrt(static_cast<float>(d));
  const int dtype = q.scalar_type() == torch::kBFloat16 ? MFA_DTYPE_BF16 : MFA_DTYPE_FP16;
  auto at_row = [&](const torch::Tensor& x, int64_t r) {
    return static_cast<char*>(x.data_ptr()) + static_cast<size_t>(r) * row_bytes;
  };
  // The first error stops further issue; the streams are drained before it is reported, so
  // the device buffers never go back to the allocator while a copy or kernel still uses them.
  int rc = MFA_OK;
  cudaError_t err = cudaSuccess;
  const char* what = nullptr;
  auto ok = [&](cudaError_t e, const char* w) {
    if (err == cudaSuccess && e != cudaSuccess) {
      err = e;
      what = w;
    }
    return err == cudaSuccess;
  };
  // copies in (s_in) and forwards (s_run), piece by piece
  size_t issued = 0;
  for (size_t i = 0; i < pieces; ++i) {
    const int64_t a = bounds[i], b = bounds[i + 1];
    const size_t bytes = static_cast<size_t>(b - a) * row_bytes;
    if (!ok(cudaMemcpyAsync(at_row(dq, a), at_row(q, a), bytes, cudaMemcpyHostToDevice, s_in),
            "copy of q") ||
        !ok(cudaMemcpyAsync(at_row(dk, a), at_row(k, a), bytes, cudaMemcpyHostToDevice, s_in),
            "copy of k") ||
        !ok(cudaMemcpyAsync(at_row(dv, a), at_row(v, a), bytes, cudaMemcpyHostToDevice, s_in),
            "copy of v") ||
        !ok(cudaEventRecord(ev[2 * i], s_in), "cudaEventRecord") ||
        !ok(cudaStreamWaitEvent(s_run, ev[2 * i], 0), "cudaStreamWaitEvent"))
      break;
    rc = mfa_fwd(at_row(dq, a), at_row(dk, a), at_row(dv, a), at_row(dout, a), 1, b - a, n,
                 static_cast<int32_t>(d), scale, causal ? 1 : 0, dtype, MFA_LAYOUT_BHND,
                 static_cast<void*>(s_run));
    if (rc != MFA_OK || !ok(cudaEventRecord(ev[2 * i + 1], s_run), "cudaEventRecord"))
      break;
    issued = i + 1;
  }
  // copies out (s_out), each after its piece's forward. When a copy out overlaps copies in,
  // the copy out takes the larger share of PCIe (measured: ~40 of ~60 GB/s), so the
  // second-to-last piece's copy waits until the last piece is in: it then runs while the last
  // forward does, and the last piece reaches the GPU sooner.
  for (size_t i = 0; i < issued; ++i) {
    const int64_t a = bounds[i], b = bounds[i + 1];
    const size_t bytes = static_cast<size_t>(b - a) * row_bytes;
    if (!ok(cudaStreamWaitEvent(s_out, ev[2 * i + 1], 0), "cudaStreamWaitEvent") ||
        (i + 2 == pieces && issued == pieces &&
         !ok(cudaStreamWaitEvent(s_out, ev[2 * (pieces - 1)], 0), "cudaStreamWaitEvent")) ||
        !ok(cudaMemcpyAsync(at_row(out, a), at_row(dout, a), bytes, cudaMemcpyDeviceToHost, s_out),
            "copy of the output"))
      break;
  }
  // Every use of the device buffers is on these three streams: once they are drained the
  // buffers may return to the allocator's current stream. When every piece was issued, the
  // last copy out waits for the last forward, which waits for the last copies in, so draining
  // the copy-out stream drains all three.
  const bool complete = rc == MFA_OK && err == cudaSuccess && issued == pieces;
  const cudaError_t e_out = cudaStreamSynchronize(s_out);
  const cudaError_t e_in = complete ? cudaSuccess : cudaStreamSynchronize(s_in);
  const cudaError_t e_run = complete ? cudaSuccess : cudaStreamSynchronize(s_run);
  if (rc != MFA_OK) throw std::runtime_error(mfa_last_error_string());
  check_cuda(err, what ? what : "");
  check_cuda(e_in, "copies in");
  check_cuda(e_run, "forward");
  check_cuda(e_out, "copies out");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &flash_attn_forward, "Mini Flash Attention forward (sm_100a tcgen05)");
  m.def("forward_lse", &flash_attn_forward_lse,
        "Mini Flash Attention forward returning (out, lse), lse = row log-sum-exp (fp32)");
  m.def("backward", &flash_attn_backward,
        "Mini Flash Attention backward: (dq, dk, dv) from q, k, v, out, lse, dout (D = 64)");
  m.def("forward_bnhd", &flash_attn_forward_bnhd,
        "Mini Flash Attention forward on [B, N, H, D] tensors (fp16 or bf16)");
  m.def("forward_wmma", &flash_attn_forward_wmma,
        "Mini Flash Attention forward, single-tile sm_100a kernel (replaces the WMMA path)");
  m.def("forward_into", &flash_attn_forward_into,
        "Mini Flash Attention forward into a preallocated output tensor");
  m.def("forward_rows", &flash_attn_forward_rows,
        "Forward of the query rows [q_begin, q_end) of every head into out");
  m.def("forward_pinned", &flash_attn_forward_pinned,
        "Pipelined forward on host tensors [rows, N, D] cut into pieces at `bounds`");
  m.def("version", []() { return std::string(mfa_version()); });
}
