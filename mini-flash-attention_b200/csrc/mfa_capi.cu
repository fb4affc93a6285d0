// C-ABI launchers of the sm_100a attention forward (declared in include/mfa_b200.h).
//
// Host-side duties of the reference launchers (src/mini_flash_attention/flash_attn_cuda.cu:
// 370-420 and flash_attn_wmma_cuda.cu:253-289): validate D / N / causal with the same
// messages, build the grid, launch on the caller's stream, report launch errors. On top of
// that this layer encodes the four TMA tensor maps and converts every failure into a status
// code plus a thread-local message instead of a C++ exception.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/mfa_b200.h"
#include "mfa_bwd_kernel.cuh"
#include "mfa_fwd_kernel.cuh"

namespace mfa {
namespace {

constexpr int kMaxDevices = 64;
constexpr const char* kVersion = "mini-flash-attention-b200 0.1.0 (sm_100a)";

thread_local std::string g_last_error;

// Device status word written by the watchdog of every forward kernel in this library.
__device__ int g_device_status = 0;

unsigned long long g_watchdog_ns = 2000000000ull;  // 2 s per wait

// Two 128-row query tiles per CTA and a 3-slot K/V ring, except for D = 128, whose O would
// not fit twice in TMEM next to S and P: one tile per CTA and a 2-slot ring (shared memory).
template <bool kCausal, bool kBF16, int D = 64, bool kLSE = false>
using Full = FwdConfig<D == 128 ? 1 : 2, D == 128 ? 2 : 3, kCausal, kBF16, D, kLSE>;
template <bool kCausal>
using Simple = FwdConfig<1, 2, kCausal, false, 64>;

template <class Cfg>
cudaError_t set_smem_attribute() {
  return cudaFuncSetAttribute(
      mfa_fwd_kernel<Cfg::NQ, Cfg::STAGES, Cfg::kCausal, Cfg::kBF16, Cfg::kHeadDim, Cfg::kLSE>,
      cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
}

template <bool kCausal, bool kBF16>
cudaError_t set_bwd_attribute() {
  cudaError_t e = cudaFuncSetAttribute(mfa_bwd_kernel<kCausal, kBF16>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       bwd_smem_bytes<kCausal, kBF16>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(mfa_bwd_mixed_kernel<kCausal, kBF16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             bwd_smem_bytes<kCausal, kBF16>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(mfa_bwd_pass_kernel<false, kCausal, kBF16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             BwdConfig<false, kCausal, kBF16>::kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(mfa_bwd_pass_kernel<true, kCausal, kBF16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             BwdConfig<true, kCausal, kBF16>::kSmemBytes);
  return e;
}

cudaError_t set_bwd_attributes() {
  cudaError_t e = set_bwd_attribute<false, false>();
  if (e == cudaSuccess) e = set_bwd_attribute<true, false>();
  if (e == cudaSuccess) e = set_bwd_attribute<false, true>();
  if (e == cudaSuccess) e = set_bwd_attribute<true, true>();
  return e;
}

template <int D, bool kLSE>
cudaError_t set_smem_attributes_dl() {
  cudaError_t e = set_smem_attribute<Full<false, false, D, kLSE>>();
  if (e == cudaSuccess) e = set_smem_attribute<Full<true, false, D, kLSE>>();
  if (e == cudaSuccess) e = set_smem_attribute<Full<false, true, D, kLSE>>();
  if (e == cudaSuccess) e = set_smem_attribute<Full<true, true, D, kLSE>>();
  return e;
}

template <int D>
cudaError_t set_smem_attributes_d() {
  cudaError_t e = set_smem_attributes_dl<D, false>();
  if (e == cudaSuccess) e = set_smem_attributes_dl<D, true>();
  return e;
}

struct DeviceState {
  std::once_flag once;
  int error = MFA_OK;
  std::string message;
  int* status_ptr = nullptr;
  int num_sms = 0;
  cudaMemPool_t pool = nullptr;  // split-mode scratch; keeps its memory between calls
};
DeviceState g_devices[kMaxDevices];

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int check_device_pointers(const void* q, const void* k, const void* v, const void* out, int dev);

int fail_cuda(cudaError_t e, const char* what) {
  return fail(MFA_ERR_CUDA, std::string("CUDA error: ") + cudaGetErrorString(e) + " (" + what + ")");
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder(std::string* why) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  static std::string err;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    cudaError_t e =
        cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || ptr == nullptr) {
      err = std::string("cannot resolve cuTensorMapEncodeTiled: ") + cudaGetErrorString(e);
      return;
    }
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (!fn && why) *why = err;
  return fn;
}

// Architecture check shared by the set-up of every entry point: device `dev` must be an
// sm_100 GPU. Returns MFA_OK with its SM count, MFA_ERR_DEVICE (a permanent condition) or
// MFA_ERR_CUDA, with the message in *msg.
int check_architecture(int dev, int* num_sms, std::string* msg) {
  int major = 0, minor = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (e == cudaSuccess && (major != 10 || minor != 0)) {
    *msg = "mini_flash_attention_b200 kernels are built for sm_100a only; device " +
           std::to_string(dev) + " is sm_" + std::to_string(major) + std::to_string(minor);
    return MFA_ERR_DEVICE;
  }
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(num_sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) {
    *msg = std::string("CUDA error: ") + cudaGetErrorString(e);
    return MFA_ERR_CUDA;
  }
  return MFA_OK;
}

// One-time per-device set-up: architecture check, kernel attributes, status word address.
int prepare_device(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return fail(MFA_ERR_DEVICE, "device index out of range");
  DeviceState& ds = g_devices[dev];
  std::call_once(ds.once, [&ds, dev] {
    ds.error = check_architecture(dev, &ds.num_sms, &ds.message);
    if (ds.error != MFA_OK) return;
    cudaError_t e = set_smem_attributes_d<32>();
    if (e == cudaSuccess) e = set_smem_attributes_d<64>();
    if (e == cudaSuccess) e = set_smem_attributes_d<128>();
    if (e == cudaSuccess) e = set_bwd_attributes();
    if (e == cudaSuccess) e = set_smem_attribute<Simple<false>>();
    if (e == cudaSuccess) e = set_smem_attribute<Simple<true>>();
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ds.status_ptr), g_device_status);
    if (e == cudaSuccess) {
      // A private stream-ordered pool for the split-mode partial results: the scratch is
      // allocated and freed on the caller's stream around each launch, and the pool keeps
      // the memory mapped so that later calls do not pay for mapping it again.
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      e = cudaMemPoolCreate(&ds.pool, &props);
      if (e == cudaSuccess) {
        uint64_t keep = UINT64_MAX;
        e = cudaMemPoolSetAttribute(ds.pool, cudaMemPoolAttrReleaseThreshold, &keep);
      }
    }
    if (e != cudaSuccess) {
      ds.error = MFA_ERR_CUDA;
      ds.message = std::string("CUDA error: ") + cudaGetErrorString(e) + " (device set-up)";
    }
  });
  if (ds.error != MFA_OK) return fail(ds.error, ds.message);
  return MFA_OK;
}

// Element strides (n, h, b) of a [B, H, N, D] (layout 0) or [B, N, H, D] (layout 1) tensor.
struct Strides {
  int64_t n, h, b;
};
Strides layout_strides(int layout, int64_t heads, int64_t n, int64_t d) {
  if (layout == MFA_LAYOUT_BNHD) return {heads * d, d, n * heads * d};
  return {d, n * d, heads * n * d};
}

// 4-D TMA view {D, N, H, B} of one tensor, box {min(D, 64), 128, 1, 1}: 128-byte swizzle for
// 64-column boxes, 64-byte swizzle for D = 32. The N extent keeps tiles inside their head:
// rows past N read as zero and are not stored.
// `rows` (default n) rows per head starting at `base`; the strides are those of an N = n tensor.
int encode_tensor(CUtensorMap* map, const void* base, int64_t batch, int64_t heads, int64_t n,
                  int64_t d, int layout, bool bf16, int64_t rows = -1) {
  std::string why;
  auto encode = tensor_map_encoder(&why);
  if (!encode) return fail(MFA_ERR_CUDA, why);
  const Strides st = layout_strides(layout, heads, n, d);
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(d),
                              static_cast<cuuint64_t>(rows < 0 ? n : rows),
                              static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(st.n) * 2,
                                 static_cast<cuuint64_t>(st.h) * 2,
                                 static_cast<cuuint64_t>(st.b) * 2};
  const cuuint32_t box_cols = d < 64 ? static_cast<cuuint32_t>(d) : 64;
  const cuuint32_t box[4] = {box_cols, 128, 1, 1};
  const cuuint32_t elem_strides[4] = {1, 1, 1, 1};
  CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      4, const_cast<void*>(base), dims, strides, box, elem_strides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                      box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MFA_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return MFA_OK;
}

// Launches the split-mode merge as a programmatic dependent of the forward kernel just
// queued on `stream` (it may start while the forward kernel drains; it reads the workspace
// only after griddepcontrol.wait).
template <class Cfg>
cudaError_t launch_merge(const MergeParams& mp, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(mp.ctas));
  cfg.blockDim = dim3(Cfg::kRowsPerUnit * kMergeThreadsPerRow);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg,
                            mfa_merge_kernel<Cfg::kRowsPerUnit, Cfg::kSlotFloats, Cfg::kCausal,
                                             Cfg::kBF16, Cfg::kHeadDim, Cfg::kLSE>,
                            mp);
}

// Launch plan, shared by every entry point. Persistent: one CTA per SM (or fewer for small
// problems). When whole query blocks divide badly over the SMs (more than 3% idle in the last
// wave), and always with causal masking (query blocks of unequal length), the global steps
// are split evenly over the CTAs and a merge kernel combines the pieces of the query blocks
// cut by a CTA boundary.
struct Plan {
  Schedule sc;
  int64_t ctas = 0;
  int split = 0;
  size_t workspace_bytes = 0;  // split mode: partial-result slots
};

// nq query rows and n keys per head (nq == n but for a row range; causal: qb0 query blocks of
// the head come before the range, and n is one past its last row).
template <class Cfg>
int plan_forward(int64_t bh, int64_t nq, int64_t n, int64_t sms, Plan& pl, int64_t qb0 = 0) {
  const int64_t q_blocks = (nq + Cfg::kRowsPerUnit - 1) / Cfg::kRowsPerUnit;
  const int64_t nkb = (n + Cfg::kKeys - 1) / Cfg::kKeys;
  const int64_t units = q_blocks * bh;
  if (static_cast<double>(units) * static_cast<double>(nkb) > static_cast<double>(int64_t(1) << 40) ||
      units > 0x7fffffffLL)
    return fail(MFA_ERR_INVALID_ARGUMENT, "B * H * N is too large");
  pl.sc = make_schedule(bh, nq, n, Cfg::kRowsPerUnit, Cfg::kKeys, Cfg::kCausal,
                        static_cast<int>(qb0));
  const int64_t total = pl.sc.total();
  pl.ctas = units < sms ? units : sms;
  pl.split = 0;
  if (Cfg::kCausal) {
    pl.split = 1;
  } else if (units % sms != 0 && units < 32 * sms) {
    // idle fraction of the last wave if only whole query blocks are handed out
    const double waves = static_cast<double>(units) / sms;
    const double busy = waves / static_cast<double>((units + sms - 1) / sms);
    if (busy < 0.97) pl.split = 1;
  }
  if (pl.split) pl.ctas = total < sms ? total : sms;
  set_ctas(pl.sc, static_cast<int>(pl.ctas));
  // every CTA's work must stay below 2^31 steps (32-bit step counters in the kernel)
  if ((pl.split ? total / pl.ctas + 1 : (units + pl.ctas - 1) / pl.ctas * nkb) >= 0x7fffffffLL)
    return fail(MFA_ERR_INVALID_ARGUMENT, "B * H * N is too large");
  pl.workspace_bytes =
      pl.split ? static_cast<size_t>(2 * pl.ctas) * Cfg::kSlotFloats * sizeof(float) : 0;
  return MFA_OK;
}

// Queues the forward kernel (and the merge kernel in split mode) of plan `pl` on `stream`;
// `workspace` holds pl.workspace_bytes.
// Query rows [q_begin, q_end) of every head (all of them by default) against all n keys.
template <class Cfg>
cudaError_t launch_planned(const void* q, const void* k, const void* v, void* out, int64_t batch,
                           int64_t heads, int64_t n, int layout, float scale, const Plan& pl,
                           float* workspace, int* status_ptr, cudaStream_t stream, int* rc,
                           float* lse = nullptr, int64_t q_begin = 0, int64_t q_end = -1) {
  FwdParams p;
  *rc = MFA_OK;
  const bool bf16 = Cfg::kBF16;
  const int64_t d = Cfg::kHeadDim;
  if (q_end < 0) q_end = n;
  const int64_t nq = q_end - q_begin;
  const Strides st = layout_strides(layout, heads, n, d);
  const size_t row_off = static_cast<size_t>(q_begin) * static_cast<size_t>(st.n) * 2;  // bytes
  const void* q_rows = static_cast<const char*>(q) + row_off;
  void* out_rows = static_cast<char*>(out) + row_off;
  if ((*rc = encode_tensor(&p.tm_q, q_rows, batch, heads, n, d, layout, bf16, nq)) != MFA_OK)
    return cudaSuccess;
  if ((*rc = encode_tensor(&p.tm_k, k, batch, heads, n, d, layout, bf16)) != MFA_OK)
    return cudaSuccess;
  if ((*rc = encode_tensor(&p.tm_v, v, batch, heads, n, d, layout, bf16)) != MFA_OK)
    return cudaSuccess;
  if ((*rc = encode_tensor(&p.tm_o, out_rows, batch, heads, n, d, layout, bf16, nq)) != MFA_OK)
    return cudaSuccess;
  // keys: all n, or with the mask the first q_end (later keys are masked for every row)
  p.n = static_cast<int>(Cfg::kCausal ? q_end : n);
  p.nq = static_cast<int>(nq);
  p.q0 = static_cast<int>(q_begin);
  p.heads = static_cast<int>(heads);
  p.sc = pl.sc;
  p.split = pl.split;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.timeout_ns = g_watchdog_ns;
  p.status = status_ptr;
  p.workspace = workspace;
  p.lse = lse;
  // a programmatic dependent of the stream's previous kernel: its set-up overlaps that
  // kernel's tail, its memory accesses wait for its completion (griddepcontrol.wait)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.ctas));
  cfg.blockDim = dim3(Cfg::kThreads);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(
      &cfg, mfa_fwd_kernel<Cfg::NQ, Cfg::STAGES, Cfg::kCausal, Cfg::kBF16, Cfg::kHeadDim, Cfg::kLSE>,
      p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e == cudaSuccess && pl.split) {
    MergeParams mp;
    mp.out = out_rows;
    mp.lse = lse;
    mp.workspace = workspace;
    mp.n = p.n;
    mp.nq = p.nq;
    mp.heads = p.heads;
    mp.stride_b = st.b;
    mp.stride_h = st.h;
    mp.stride_n = st.n;
    mp.sc = pl.sc;
    mp.ctas = static_cast<int>(pl.ctas);
    e = launch_merge<Cfg>(mp, stream);
  }
  return e;
}

// The split plan's partial results live in a stream-ordered scratch allocation from a private
// pool, freed on the same stream.
template <class Cfg>
int launch_forward(const void* q, const void* k, const void* v, void* out, int64_t batch,
                   int64_t heads, int64_t n, int layout, float scale, cudaStream_t stream,
                   float* lse = nullptr, int64_t q_begin = 0, int64_t q_end = -1) {
  const int64_t bh = batch * heads;
  if (q_end < 0) q_end = n;
  if (bh == 0 || n == 0 || q_end == q_begin) return MFA_OK;
  if (Cfg::kCausal && q_begin % Cfg::kRowsPerUnit != 0)
    return fail(MFA_ERR_INVALID_ARGUMENT,
                "a causal query row range must start at a multiple of 256 rows");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  int rc = prepare_device(dev);
  if (rc != MFA_OK) return rc;
  if ((rc = check_device_pointers(q, k, v, out, dev)) != MFA_OK) return rc;
  Plan pl;
  if ((rc = plan_forward<Cfg>(bh, q_end - q_begin, Cfg::kCausal ? q_end : n,
                              g_devices[dev].num_sms, pl, q_begin / Cfg::kRowsPerUnit)) != MFA_OK)
    return rc;
  float* workspace = nullptr;
  if (pl.split) {
    e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&workspace), pl.workspace_bytes,
                                g_devices[dev].pool, stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMallocFromPoolAsync (split workspace)");
  }
  e = launch_planned<Cfg>(q, k, v, out, batch, heads, n, layout, scale, pl, workspace,
                          g_devices[dev].status_ptr, stream, &rc, lse, q_begin, q_end);
  if (pl.split) {
    const cudaError_t ef = cudaFreeAsync(workspace, stream);
    if (e == cudaSuccess) e = ef;
  }
  if (rc != MFA_OK) return rc;
  if (e != cudaSuccess) return fail_cuda(e, "kernel launch");
  return MFA_OK;
}

int check_common(const void* q, const void* k, const void* v, void* out, int64_t bh, int64_t n,
                 int32_t d) {
  if (bh < 0 || n < 0 || d <= 0) return fail(MFA_ERR_INVALID_ARGUMENT, "negative extent");
  if (bh > 0x7fffffffLL) return fail(MFA_ERR_INVALID_ARGUMENT, "B * H is too large");
  if (n > 0x7fffffffLL) return fail(MFA_ERR_INVALID_ARGUMENT, "N is too large");
  if (bh == 0 || n == 0) return MFA_OK;
  if (!q || !k || !v || !out) return fail(MFA_ERR_INVALID_ARGUMENT, "null tensor pointer");
  const uintptr_t any = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                        reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(out);
  if (any & 15u)
    return fail(MFA_ERR_INVALID_ARGUMENT, "q, k, v and out must be 16-byte aligned");
  return MFA_OK;
}

// q, k, v and out must be memory that device `dev` addresses directly (its own device memory
// or managed memory). A host, foreign or dangling pointer is refused here, before anything is
// launched, instead of faulting the GPU inside the kernel.
int check_device_pointers(const void* q, const void* k, const void* v, const void* out, int dev) {
  const void* ptrs[4] = {q, k, v, out};
  const char* names[4] = {"q", "k", "v", "out"};
  for (int i = 0; i < 4; ++i) {
    cudaPointerAttributes a = {};
    const cudaError_t e = cudaPointerGetAttributes(&a, ptrs[i]);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return fail(MFA_ERR_INVALID_ARGUMENT, std::string(names[i]) + " is not a CUDA pointer");
    }
    const bool ok = (a.type == cudaMemoryTypeDevice && a.device == dev) ||
                    a.type == cudaMemoryTypeManaged;
    if (!ok)
      return fail(MFA_ERR_INVALID_ARGUMENT,
                  std::string(names[i]) + " must point to memory of the current device");
  }
  return MFA_OK;
}

}  // namespace
}  // namespace mfa

// ------------------------------------------------------------------ allocation-free entry
// Scratch of mfa_fwd_f16_noalloc, part of the library's device image: the split plan's partial
// results, two slots of 256 query rows x (64 + 2) floats (67,584 bytes each) per forward CTA,
// so 20 MiB covers up to 155 CTAs; a B200 launches at most 148. Shared by every call on a device.
static __device__ __align__(256) float g_noalloc_scratch[MFA_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace mfa {
namespace {

struct NoAllocState {
  std::mutex mu;                  // serialises the set-up
  std::atomic<bool> ready{false};  // set-up completed: the fields below are valid
  int error = MFA_OK;             // a permanent failure (wrong architecture), reported by every call
  std::string message;
  int* status_ptr = nullptr;
  float* scratch = nullptr;
  int num_sms = 0;
};
NoAllocState g_noalloc[kMaxDevices];

// Per-device set-up of the allocation-free entry point, run with `dev` current: the
// architecture check and kernel attributes of prepare_device, plus the device addresses of
// the status word and of the static scratch. It creates no memory pool and allocates nothing.
// Only a wrong architecture is remembered; after any other failure (a CUDA error, e.g. a first
// call made during stream capture) the set-up runs again on the next call.
int prepare_noalloc(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return fail(MFA_ERR_DEVICE, "device index out of range");
  NoAllocState& st = g_noalloc[dev];
  if (st.ready.load(std::memory_order_acquire)) return MFA_OK;
  std::lock_guard<std::mutex> lock(st.mu);
  if (st.ready.load(std::memory_order_relaxed)) return MFA_OK;
  if (st.error != MFA_OK) return fail(st.error, st.message);
  std::string msg;
  int num_sms = 0;
  const int rc = check_architecture(dev, &num_sms, &msg);
  if (rc == MFA_ERR_DEVICE) {
    st.error = rc;
    st.message = msg;
  }
  if (rc != MFA_OK) return fail(rc, msg);
  int* status_ptr = nullptr;
  float* scratch = nullptr;
  cudaError_t e = set_smem_attribute<Full<false, false>>();
  if (e == cudaSuccess) e = set_smem_attribute<Full<true, false>>();
  if (e == cudaSuccess)
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&status_ptr), g_device_status);
  if (e == cudaSuccess)
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&scratch), g_noalloc_scratch);
  if (e != cudaSuccess) return fail_cuda(e, "no-alloc set-up");
  st.num_sms = num_sms;
  st.status_ptr = status_ptr;
  st.scratch = scratch;
  st.ready.store(true, std::memory_order_release);
  return MFA_OK;
}

// launch_forward with the split workspace taken from the static scratch instead of a
// stream-ordered allocation.
template <class Cfg>
int launch_forward_noalloc(const void* q, const void* k, const void* v, void* out, int64_t bh,
                           int64_t n, float scale, cudaStream_t stream) {
  if (bh == 0 || n == 0) return MFA_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  int rc = prepare_noalloc(dev);
  if (rc != MFA_OK) return rc;
  if ((rc = check_device_pointers(q, k, v, out, dev)) != MFA_OK) return rc;
  const NoAllocState& st = g_noalloc[dev];
  Plan pl;
  if ((rc = plan_forward<Cfg>(bh, n, n, st.num_sms, pl)) != MFA_OK) return rc;
  // Every slot the merge kernel reads is written by the forward kernel of the same call, so
  // nothing in the scratch has to start at zero.
  if (pl.workspace_bytes > MFA_NOALLOC_SCRATCH_BYTES)
    return fail(MFA_ERR_INVALID_ARGUMENT,
                "mfa_fwd_f16_noalloc: this launch needs " + std::to_string(pl.workspace_bytes) +
                    " bytes of scratch, more than its static " +
                    std::to_string(MFA_NOALLOC_SCRATCH_BYTES) + "-byte array");
  e = launch_planned<Cfg>(q, k, v, out, 1, bh, n, MFA_LAYOUT_BHND, scale, pl,
                          pl.split ? st.scratch : nullptr, st.status_ptr, stream, &rc);
  if (rc != MFA_OK) return rc;
  if (e != cudaSuccess) return fail_cuda(e, "kernel launch");
  return MFA_OK;
}

// ------------------------------------------------------------------ watchdog self-test
__device__ int g_selftest_status = 0;

__global__ void __launch_bounds__(32, 1) watchdog_selftest_kernel(unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar_storage;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const uint32_t bar = smem_addr(&bar_storage);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(bar, 1);
    mbar_init_fence();
  }
  tmem_alloc(smem_addr(&tmem_slot), 32);
  tmem_relinquish();
  tc_fence_before();
  __syncwarp();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const Watchdog wd{&abort_flag, &g_selftest_status, timeout_ns};
  // Nothing ever arrives on `bar`: the wait must expire, trip the watchdog and return.
  const bool ok = wait_warp(bar, 0, wd, kSiteSoftSFull);
  (void)ok;
  tc_fence_before();
  __syncwarp();
  tmem_dealloc(tmem, 32);
}

}  // namespace
}  // namespace mfa

using namespace mfa;

extern "C" int mfa_fwd_f16(const void* q, const void* k, const void* v, void* out, int64_t bh,
                           int64_t n, int32_t d, float scale, int32_t causal, void* stream) {
  int rc = check_common(q, k, v, out, bh, n, d);
  if (rc != MFA_OK) return rc;
  // The D check and message of flash_attn_cuda.cu:399-401. Any N is supported (the reference
  // requires N % 128 == 0, flash_attn_cuda.cu:402-407: here the TMA maps zero-fill rows past N,
  // the last key block masks keys past N and the stores clip rows past N), and so is causal
  // masking (rejected by flash_attn_cuda.cu:408-410).
  if (d != 64) return fail(MFA_ERR_HEAD_DIM, "This kernel supports only D=64");
  if (!(scale > 0.0f) || !std::isfinite(scale))
    return fail(MFA_ERR_INVALID_ARGUMENT, "scale must be positive and finite");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return causal ? launch_forward<Full<true, false>>(q, k, v, out, 1, bh, n, MFA_LAYOUT_BHND, scale, s)
                : launch_forward<Full<false, false>>(q, k, v, out, 1, bh, n, MFA_LAYOUT_BHND, scale,
                                                     s);
}

extern "C" int mfa_fwd_simple_f16(const void* q, const void* k, const void* v, void* out,
                                  int64_t bh, int64_t n, int32_t d, float scale, int32_t causal,
                                  void* stream) {
  int rc = check_common(q, k, v, out, bh, n, d);
  if (rc != MFA_OK) return rc;
  // The D and N checks and messages of flash_attn_wmma_cuda.cu:269-274, in that order.
  // Causal masking (rejected by flash_attn_wmma_cuda.cu:275-277) is supported.
  if (d != 64) return fail(MFA_ERR_HEAD_DIM, "This WMMA prototype supports only D=64 yet");
  if (n % 64 != 0)
    return fail(MFA_ERR_SEQ_LEN, "Only N (seq len) divisible by 64 and 64 are supported yet");
  if (!(scale > 0.0f) || !std::isfinite(scale))
    return fail(MFA_ERR_INVALID_ARGUMENT, "scale must be positive and finite");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return causal ? launch_forward<Simple<true>>(q, k, v, out, 1, bh, n, MFA_LAYOUT_BHND, scale, s)
                : launch_forward<Simple<false>>(q, k, v, out, 1, bh, n, MFA_LAYOUT_BHND, scale, s);
}

namespace mfa {
namespace {
template <int D, bool kLSE>
int launch_general_l(const void* q, const void* k, const void* v, void* out, int64_t batch,
                     int64_t heads, int64_t n, float scale, int32_t causal, int32_t dtype,
                     int32_t layout, cudaStream_t s, float* lse, int64_t q_begin,
                     int64_t q_end) {
  if (dtype == MFA_DTYPE_BF16)
    return causal ? launch_forward<Full<true, true, D, kLSE>>(q, k, v, out, batch, heads, n,
                                                              layout, scale, s, lse, q_begin, q_end)
                  : launch_forward<Full<false, true, D, kLSE>>(q, k, v, out, batch, heads, n,
                                                               layout, scale, s, lse, q_begin, q_end);
  return causal ? launch_forward<Full<true, false, D, kLSE>>(q, k, v, out, batch, heads, n,
                                                             layout, scale, s, lse, q_begin, q_end)
                : launch_forward<Full<false, false, D, kLSE>>(q, k, v, out, batch, heads, n,
                                                              layout, scale, s, lse, q_begin, q_end);
}

// The row log-sum-exp is a compile-time option: the plain forward kernels carry none of it.
template <int D>
int launch_general(const void* q, const void* k, const void* v, void* out, int64_t batch,
                   int64_t heads, int64_t n, float scale, int32_t causal, int32_t dtype,
                   int32_t layout, cudaStream_t s, float* lse, int64_t q_begin = 0,
                   int64_t q_end = -1) {
  return lse ? launch_general_l<D, true>(q, k, v, out, batch, heads, n, scale, causal, dtype,
                                         layout, s, lse, q_begin, q_end)
             : launch_general_l<D, false>(q, k, v, out, batch, heads, n, scale, causal, dtype,
                                          layout, s, nullptr, q_begin, q_end);
}

int fwd_general(const void* q, const void* k, const void* v, void* out, float* lse,
                int64_t batch, int64_t heads, int64_t n, int32_t d, float scale, int32_t causal,
                int32_t dtype, int32_t layout, void* stream, int64_t q_begin = 0,
                int64_t q_end = -1) {
  if (batch < 0 || heads < 0) return fail(MFA_ERR_INVALID_ARGUMENT, "negative extent");
  if (heads > 0 && batch > 0x7fffffffLL / heads)
    return fail(MFA_ERR_INVALID_ARGUMENT, "B * H is too large");
  int rc = check_common(q, k, v, out, batch * heads, n, d);
  if (rc != MFA_OK) return rc;
  if (d != 32 && d != 64 && d != 128)
    return fail(MFA_ERR_HEAD_DIM, "This kernel supports only D=32, D=64 and D=128");
  if (dtype != MFA_DTYPE_FP16 && dtype != MFA_DTYPE_BF16)
    return fail(MFA_ERR_INVALID_ARGUMENT, "dtype must be MFA_DTYPE_FP16 or MFA_DTYPE_BF16");
  if (layout != MFA_LAYOUT_BHND && layout != MFA_LAYOUT_BNHD)
    return fail(MFA_ERR_INVALID_ARGUMENT, "layout must be MFA_LAYOUT_BHND or MFA_LAYOUT_BNHD");
  if (!(scale > 0.0f) || !std::isfinite(scale))
    return fail(MFA_ERR_INVALID_ARGUMENT, "scale must be positive and finite");
  if (batch * heads > 0 && n > 0 && lse != nullptr) {
    if (reinterpret_cast<uintptr_t>(lse) & 3u)
      return fail(MFA_ERR_INVALID_ARGUMENT, "lse must be 4-byte aligned");
  }
  if (q_end < 0) q_end = n;
  if (q_begin < 0 || q_begin > q_end || q_end > n)
    return fail(MFA_ERR_INVALID_ARGUMENT, "query rows must satisfy 0 <= q_begin <= q_end <= N");
  if (lse != nullptr && (q_begin != 0 || q_end != n))
    return fail(MFA_ERR_INVALID_ARGUMENT, "a query row range writes no log-sum-exp");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d == 32)
    return launch_general<32>(q, k, v, out, batch, heads, n, scale, causal, dtype, layout, s, lse,
                              q_begin, q_end);
  if (d == 128)
    return launch_general<128>(q, k, v, out, batch, heads, n, scale, causal, dtype, layout, s,
                               lse, q_begin, q_end);
  return launch_general<64>(q, k, v, out, batch, heads, n, scale, causal, dtype, layout, s, lse,
                            q_begin, q_end);
}

// ---------------------------------------------------------------- backward
// Tensor maps of one pass: x, y resident, s0, s1 streamed, o0 (and o1) written.
template <bool kBF16>
int encode_bwd_pass(BwdParams& bp, const void* x, const void* y, const void* s0, const void* s1,
                    void* o0, void* o1, int64_t batch, int64_t heads, int64_t n, int layout) {
  int rc = MFA_OK;
  if ((rc = encode_tensor(&bp.tm_x, x, batch, heads, n, 64, layout, kBF16)) != MFA_OK ||
      (rc = encode_tensor(&bp.tm_y, y, batch, heads, n, 64, layout, kBF16)) != MFA_OK ||
      (rc = encode_tensor(&bp.tm_s0, s0, batch, heads, n, 64, layout, kBF16)) != MFA_OK ||
      (rc = encode_tensor(&bp.tm_s1, s1, batch, heads, n, 64, layout, kBF16)) != MFA_OK ||
      (rc = encode_tensor(&bp.tm_o0, o0, batch, heads, n, 64, layout, kBF16)) != MFA_OK ||
      (rc = encode_tensor(&bp.tm_o1, o1 ? o1 : o0, batch, heads, n, 64, layout, kBF16)) != MFA_OK)
    return rc;
  return MFA_OK;
}

// How the backward's two passes use the SMs (see launch_backward).
struct BwdPlan {
  enum Mode { kPasses, kSplit, kMixed } mode;
  int64_t cq, ckv;  // CTAs of the dQ pass and the dK/dV pass (kMixed: the same CTAs)
};

BwdPlan plan_backward(int64_t units, int64_t sms, bool causal) {
  constexpr double kKvCost = 1.05;    // a dK/dV step in dQ steps
  constexpr double kRestart = 0.05;   // mixed: pipeline restart between passes, in units
  const double waves = static_cast<double>(units) / static_cast<double>(sms);
  if (sms < 2 || std::ceil(waves) / waves <= 1.05)
    return {BwdPlan::kPasses, sms < units ? sms : units, sms < units ? sms : units};
  double best = 1e300;
  int64_t cq = sms;
  const double ideal = static_cast<double>(sms) / (1.0 + kKvCost);
  for (int64_t c = 1; c < sms; ++c) {
    const int64_t ck = sms - c;
    const double tq = causal ? static_cast<double>(units) / c
                             : static_cast<double>((units + c - 1) / c);
    const double tk = kKvCost * (causal ? static_cast<double>(units) / ck
                                        : static_cast<double>((units + ck - 1) / ck));
    const double cost = tq > tk ? tq : tk;
    const bool nearer = std::fabs(c - ideal) < std::fabs(cq - ideal);
    if (cost < best * (1.0 - 1e-9) || (cost <= best * (1.0 + 1e-9) && nearer)) {
      best = cost;
      cq = c;
    }
  }
  const int64_t ckv = sms - cq;
  // Mixed: CTA c takes units c, c + C, ... of the dK/dV pass and C - 1 - c, 2C - 1 - c, ...
  // of the dQ pass, so the rem CTAs with an extra dK/dV unit get an extra dQ unit only when
  // rem > C / 2. With at least one unit per SM it measured 2.6-4% faster than the split at
  // every shape tried (256 and 512 units per pass, fp16, with and without the mask; the
  // model's masked estimates of the two are within 0.1% of each other), so it is taken there
  // outright; below that (each CTA then runs two units where a split CTA runs one) by the model.
  const int64_t ctas = sms < units ? sms : units;
  const int64_t base = units / ctas, rem = units % ctas;
  double mixed;
  if (causal)
    mixed = static_cast<double>(units) * (1.0 + kKvCost) / static_cast<double>(ctas);
  else if (rem == 0)
    mixed = base * (1.0 + kKvCost);
  else if (2 * rem <= ctas)
    mixed = (base + 1) * kKvCost + base;
  else
    mixed = (base + 1) * (1.0 + kKvCost);
  mixed += kRestart;
  if (units >= sms || mixed < best) return {BwdPlan::kMixed, ctas, ctas};
  return {BwdPlan::kSplit, cq < units ? cq : units, ckv < units ? ckv : units};
}

template <bool kCausal, bool kBF16>
int launch_backward(const void* q, const void* k, const void* v, const void* out,
                    const void* dout, const float* lse, void* dq, void* dk, void* dv,
                    int64_t batch, int64_t heads, int64_t n, int layout, float scale,
                    cudaStream_t stream) {
  const int64_t bh = batch * heads;
  if (bh == 0 || n == 0) return MFA_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  int rc = prepare_device(dev);
  if (rc != MFA_OK) return rc;
  if ((rc = check_device_pointers(q, k, v, out, dev)) != MFA_OK) return rc;
  if ((rc = check_device_pointers(dout, dq, dk, dv, dev)) != MFA_OK) return rc;
  if ((rc = check_device_pointers(lse, lse, lse, lse, dev)) != MFA_OK) return rc;
  const int64_t blocks = (n + 127) / 128;
  const int64_t units = bh * blocks;
  if (units > 0x7fff0000LL) return fail(MFA_ERR_INVALID_ARGUMENT, "B * H * N is too large");
  const int64_t sms = g_devices[dev].num_sms;
  // L2 and D per row, padded to whole 128-row blocks per head
  const size_t rows = static_cast<size_t>(units) * 128;
  float* ws = nullptr;
  e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&ws), 2 * rows * sizeof(float),
                              g_devices[dev].pool, stream);
  if (e != cudaSuccess) return fail_cuda(e, "cudaMallocFromPoolAsync (backward workspace)");
  float* lse2 = ws;
  float* di = ws + rows;
  const Strides st = layout_strides(layout, heads, n, 64);
  const int64_t prep_blocks_needed = (static_cast<int64_t>(rows) / 4 + 7) / 8;
  const unsigned prep_grid =
      static_cast<unsigned>(prep_blocks_needed < sms * 16 ? prep_blocks_needed : sms * 16);
  mfa_bwd_prep_kernel<kBF16><<<prep_grid, 256, 0, stream>>>(
      out, dout, lse, lse2, di, static_cast<int>(bh), static_cast<int>(n),
      static_cast<int>(heads), st.b, st.h, st.n, static_cast<int>(blocks));
  e = cudaGetLastError();
  BwdParams bp;
  bp.n = static_cast<int>(n);
  bp.heads = static_cast<int>(heads);
  bp.bh = static_cast<int>(bh);
  bp.blocks = static_cast<int>(blocks);
  bp.scale = scale;
  bp.scale_log2 = scale * 1.4426950408889634f;
  bp.lse2 = lse2;
  bp.di = di;
  bp.timeout_ns = g_watchdog_ns;
  bp.status = g_devices[dev].status_ptr;
  // A dK/dV step (two accumulators, two operand tiles) costs about kKvCost dQ steps.
  // Many units per SM: one pass per launch, each over all SMs, units strided. Few (the last
  // wave of a pass would leave >= 5% of the SMs idle): both passes in one launch, either on
  // separate SMs (split to minimise the slower pass: equal units take ceil(units / CTAs) x
  // cost, masked ones dealt out by length about units / CTAs) or mixed, every CTA taking
  // dK/dV units and then dQ units dealt from the other end of the grid, whichever the cost
  // model finishes first (mixed pays a pipeline restart between its passes).
  const BwdPlan plan = plan_backward(units, sms, kCausal);
  BwdParams pq = bp, pkv = bp;
  pq.by_length = pkv.by_length = plan.mode != BwdPlan::kPasses && kCausal ? 1 : 0;
  pq.reverse = plan.mode == BwdPlan::kMixed ? 1 : 0;
  pkv.reverse = 0;
  const int64_t cq = plan.cq, ckv = plan.ckv;
  // dQ: q, dO resident; k, v streamed. dK, dV: k, v resident; q, dO streamed.
  rc = encode_bwd_pass<kBF16>(pq, q, dout, k, v, dq, nullptr, batch, heads, n, layout);
  if (rc == MFA_OK)
    rc = encode_bwd_pass<kBF16>(pkv, k, v, q, dout, dk, dv, batch, heads, n, layout);
  constexpr int kThreads = BwdConfig<true, kCausal, kBF16>::kThreads;
  constexpr int kSmem = bwd_smem_bytes<kCausal, kBF16>();
  if (e == cudaSuccess && rc == MFA_OK) {
    if (plan.mode == BwdPlan::kSplit) {
      pq.cta0 = 0;
      pq.ctas = static_cast<int>(cq);
      pkv.cta0 = static_cast<int>(cq);
      pkv.ctas = static_cast<int>(ckv);
      mfa_bwd_kernel<kCausal, kBF16>
          <<<static_cast<unsigned>(cq + ckv), kThreads, kSmem, stream>>>(pq, pkv);
    } else if (plan.mode == BwdPlan::kMixed) {
      pq.cta0 = pkv.cta0 = 0;
      pq.ctas = pkv.ctas = static_cast<int>(cq);
      mfa_bwd_mixed_kernel<kCausal, kBF16>
          <<<static_cast<unsigned>(cq), kThreads, kSmem, stream>>>(pq, pkv);
    } else {
      pq.cta0 = pkv.cta0 = 0;
      pq.ctas = static_cast<int>(cq);
      pkv.ctas = static_cast<int>(ckv);
      mfa_bwd_pass_kernel<false, kCausal, kBF16>
          <<<static_cast<unsigned>(cq), kThreads, BwdConfig<false, kCausal, kBF16>::kSmemBytes,
             stream>>>(pq);
      e = cudaGetLastError();
      if (e == cudaSuccess)
        mfa_bwd_pass_kernel<true, kCausal, kBF16>
            <<<static_cast<unsigned>(ckv), kThreads, BwdConfig<true, kCausal, kBF16>::kSmemBytes,
               stream>>>(pkv);
    }
    e = cudaGetLastError();
  }
  const cudaError_t ef = cudaFreeAsync(ws, stream);
  if (rc != MFA_OK) return rc;
  if (e == cudaSuccess) e = ef;
  if (e != cudaSuccess) return fail_cuda(e, "backward launch");
  return MFA_OK;
}

}  // namespace
}  // namespace mfa

extern "C" int mfa_fwd(const void* q, const void* k, const void* v, void* out, int64_t batch,
                       int64_t heads, int64_t n, int32_t d, float scale, int32_t causal,
                       int32_t dtype, int32_t layout, void* stream) {
  return fwd_general(q, k, v, out, nullptr, batch, heads, n, d, scale, causal, dtype, layout,
                     stream);
}

extern "C" int mfa_fwd_rows(const void* q, const void* k, const void* v, void* out,
                            int64_t batch, int64_t heads, int64_t n, int64_t q_begin,
                            int64_t q_end, int32_t d, float scale, int32_t causal, int32_t dtype,
                            int32_t layout, void* stream) {
  return fwd_general(q, k, v, out, nullptr, batch, heads, n, d, scale, causal, dtype, layout,
                     stream, q_begin, q_end);
}

extern "C" int mfa_fwd_lse(const void* q, const void* k, const void* v, void* out, float* lse,
                           int64_t batch, int64_t heads, int64_t n, int32_t d, float scale,
                           int32_t causal, int32_t dtype, int32_t layout, void* stream) {
  if (!lse && batch * heads > 0 && n > 0)
    return fail(MFA_ERR_INVALID_ARGUMENT, "null lse pointer");
  return fwd_general(q, k, v, out, lse, batch, heads, n, d, scale, causal, dtype, layout,
                     stream);
}

extern "C" int mfa_bwd(const void* q, const void* k, const void* v, const void* out,
                       const void* dout, const float* lse, void* dq, void* dk, void* dv,
                       int64_t batch, int64_t heads, int64_t n, int32_t d, float scale,
                       int32_t causal, int32_t dtype, int32_t layout, void* stream) {
  if (batch < 0 || heads < 0) return fail(MFA_ERR_INVALID_ARGUMENT, "negative extent");
  if (heads > 0 && batch > 0x7fffffffLL / heads)
    return fail(MFA_ERR_INVALID_ARGUMENT, "B * H is too large");
  int rc = check_common(q, k, v, const_cast<void*>(out), batch * heads, n, d);
  if (rc != MFA_OK) return rc;
  if (batch * heads > 0 && n > 0) {
    if ((rc = check_common(dout, dq, dk, dv, batch * heads, n, d)) != MFA_OK) return rc;
    if (!lse) return fail(MFA_ERR_INVALID_ARGUMENT, "null lse pointer");
    if (reinterpret_cast<uintptr_t>(lse) & 3u)
      return fail(MFA_ERR_INVALID_ARGUMENT, "lse must be 4-byte aligned");
  }
  if (d != 64) return fail(MFA_ERR_HEAD_DIM, "The backward pass supports only D=64");
  if (dtype != MFA_DTYPE_FP16 && dtype != MFA_DTYPE_BF16)
    return fail(MFA_ERR_INVALID_ARGUMENT, "dtype must be MFA_DTYPE_FP16 or MFA_DTYPE_BF16");
  if (layout != MFA_LAYOUT_BHND && layout != MFA_LAYOUT_BNHD)
    return fail(MFA_ERR_INVALID_ARGUMENT, "layout must be MFA_LAYOUT_BHND or MFA_LAYOUT_BNHD");
  if (!(scale > 0.0f) || !std::isfinite(scale))
    return fail(MFA_ERR_INVALID_ARGUMENT, "scale must be positive and finite");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == MFA_DTYPE_BF16)
    return causal ? launch_backward<true, true>(q, k, v, out, dout, lse, dq, dk, dv, batch,
                                                heads, n, layout, scale, s)
                  : launch_backward<false, true>(q, k, v, out, dout, lse, dq, dk, dv, batch,
                                                 heads, n, layout, scale, s);
  return causal ? launch_backward<true, false>(q, k, v, out, dout, lse, dq, dk, dv, batch, heads,
                                               n, layout, scale, s)
                : launch_backward<false, false>(q, k, v, out, dout, lse, dq, dk, dv, batch,
                                                heads, n, layout, scale, s);
}

extern "C" int mfa_fwd_f16_noalloc(const void* q, const void* k, const void* v, void* out,
                                   int64_t bh, int64_t n, int32_t d, float scale, int32_t causal,
                                   void* stream) {
  int rc = check_common(q, k, v, out, bh, n, d);
  if (rc != MFA_OK) return rc;
  if (d != 64) return fail(MFA_ERR_HEAD_DIM, "This kernel supports only D=64");
  if (!(scale > 0.0f) || !std::isfinite(scale))
    return fail(MFA_ERR_INVALID_ARGUMENT, "scale must be positive and finite");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return causal ? launch_forward_noalloc<Full<true, false>>(q, k, v, out, bh, n, scale, s)
                : launch_forward_noalloc<Full<false, false>>(q, k, v, out, bh, n, scale, s);
}

namespace mfa {
namespace {
template <class Cfg>
int workspace_of(int64_t bh, int64_t n, int64_t sms, uint64_t* bytes) {
  Plan pl;
  const int rc = plan_forward<Cfg>(bh, n, n, sms, pl);
  if (rc == MFA_OK) *bytes = pl.workspace_bytes;
  return rc;
}
}  // namespace
}  // namespace mfa

// The plan only: nothing is launched or allocated, and the answer is the size that
// launch_forward takes from its pool (or, for D = 64 fp16, mfa_fwd_f16_noalloc from its array).
extern "C" int mfa_fwd_workspace_bytes(int64_t batch, int64_t heads, int64_t n, int32_t d,
                                       int32_t causal, uint64_t* bytes) {
  if (!bytes) return fail(MFA_ERR_INVALID_ARGUMENT, "bytes must not be null");
  *bytes = 0;
  if (batch < 0 || heads < 0 || n < 0) return fail(MFA_ERR_INVALID_ARGUMENT, "negative extent");
  if (heads > 0 && batch > 0x7fffffffLL / heads)
    return fail(MFA_ERR_INVALID_ARGUMENT, "B * H is too large");
  if (n > 0x7fffffffLL) return fail(MFA_ERR_INVALID_ARGUMENT, "N is too large");
  if (d != 32 && d != 64 && d != 128)
    return fail(MFA_ERR_HEAD_DIM, "This kernel supports only D=32, D=64 and D=128");
  const int64_t bh = batch * heads;
  if (bh == 0 || n == 0) return MFA_OK;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaDeviceGetAttribute (multiprocessor count)");
  // dtype, layout and the log-sum-exp option do not change the plan
  if (d == 32)
    return causal ? workspace_of<Full<true, false, 32>>(bh, n, sms, bytes)
                  : workspace_of<Full<false, false, 32>>(bh, n, sms, bytes);
  if (d == 128)
    return causal ? workspace_of<Full<true, false, 128>>(bh, n, sms, bytes)
                  : workspace_of<Full<false, false, 128>>(bh, n, sms, bytes);
  return causal ? workspace_of<Full<true, false>>(bh, n, sms, bytes)
                : workspace_of<Full<false, false>>(bh, n, sms, bytes);
}

extern "C" const char* mfa_last_error_string(void) { return g_last_error.c_str(); }

extern "C" int mfa_device_status(int device, int* status, int reset) {
  if (!status) return fail(MFA_ERR_INVALID_ARGUMENT, "status must not be null");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if ((e = cudaSetDevice(device)) != cudaSuccess) return fail_cuda(e, "cudaSetDevice");
  int rc = prepare_device(device);
  if (rc == MFA_OK) {
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(status, g_device_status, sizeof(int));
    if (e == cudaSuccess && reset) {
      const int zero = 0;
      e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    }
    if (e != cudaSuccess) rc = fail_cuda(e, "reading the device status word");
  }
  cudaSetDevice(prev);
  return rc;
}

extern "C" int mfa_set_watchdog_ns(uint64_t ns) {
  if (ns < 1000000ull) return fail(MFA_ERR_INVALID_ARGUMENT, "watchdog limit must be >= 1 ms");
  g_watchdog_ns = ns;
  return MFA_OK;
}

extern "C" int mfa_watchdog_selftest(void* stream, uint64_t timeout_ns, int* status_out) {
  if (!status_out) return fail(MFA_ERR_INVALID_ARGUMENT, "status_out must not be null");
  if (timeout_ns < 1000000ull || timeout_ns > 10000000000ull)
    return fail(MFA_ERR_INVALID_ARGUMENT, "self-test limit must be within [1 ms, 10 s]");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  int rc = prepare_device(dev);
  if (rc != MFA_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int zero = 0;
  e = cudaMemcpyToSymbolAsync(g_selftest_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return fail_cuda(e, "clearing the self-test status");
  watchdog_selftest_kernel<<<1, 32, 0, s>>>(timeout_ns);
  if ((e = cudaGetLastError()) != cudaSuccess) return fail_cuda(e, "self-test launch");
  e = cudaMemcpyFromSymbolAsync(status_out, g_selftest_status, sizeof(int), 0,
                                cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail_cuda(e, "self-test");
  return MFA_OK;
}

extern "C" const char* mfa_version(void) { return kVersion; }
