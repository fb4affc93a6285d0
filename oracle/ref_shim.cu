// C-ABI shim over the reference's own launchers, compiled together with the unmodified
// reference sources (src/mini_flash_attention/flash_attn_cuda.cu and
// flash_attn_wmma_cuda.cu) by oracle/build_ref.py into oracle/_ref/libmfa_ref.so.
// Test infrastructure only: the oracle checks the product, it is never part of it.
//
// The reference declares both launchers with C++ linkage and this signature
// (src/mini_flash_attention/flash_attn.cpp:9-31). The WMMA translation unit defines its
// launcher under the CuTe launcher's name (flash_attn_wmma_cuda.cu:253); the build renames it
// with -Dlaunch_flash_attn_forward=launch_flash_attn_forward_wmma so both can be linked.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <exception>
#include <string>

void launch_flash_attn_forward(const half* q, const half* k, const half* v, half* out, int BH,
                               int N, int D, float scale, bool causal, cudaStream_t stream);
void launch_flash_attn_forward_wmma(const half* q, const half* k, const half* v, half* out,
                                    int BH, int N, int D, float scale, bool causal,
                                    cudaStream_t stream);

namespace {
thread_local std::string g_error;

template <class Fn>
int guarded(Fn&& fn) {
  try {
    fn();
    return 0;
  } catch (const std::exception& e) {
    g_error = e.what();
    return 1;
  }
}
}  // namespace

extern "C" __attribute__((visibility("default"))) int ref_cute_fwd(
    const void* q, const void* k, const void* v, void* out, int bh, int n, int d, float scale,
    int causal, void* stream) {
  return guarded([&] {
    launch_flash_attn_forward(static_cast<const half*>(q), static_cast<const half*>(k),
                              static_cast<const half*>(v), static_cast<half*>(out), bh, n, d,
                              scale, causal != 0, static_cast<cudaStream_t>(stream));
  });
}

extern "C" __attribute__((visibility("default"))) int ref_wmma_fwd(
    const void* q, const void* k, const void* v, void* out, int bh, int n, int d, float scale,
    int causal, void* stream) {
  return guarded([&] {
    launch_flash_attn_forward_wmma(static_cast<const half*>(q), static_cast<const half*>(k),
                                   static_cast<const half*>(v), static_cast<half*>(out), bh, n,
                                   d, scale, causal != 0, static_cast<cudaStream_t>(stream));
  });
}

extern "C" __attribute__((visibility("default"))) const char* ref_last_error() {
  return g_error.c_str();
}
