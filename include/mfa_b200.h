/*
 * mini-flash-attention for B200 (sm_100a) -- C ABI of the attention forward.
 *
 * Plain pointers and sizes only; no torch or C++ types cross this boundary, and no call
 * throws. Every entry point returns MFA_OK (0) or an MFA_ERR_* code; the message of the last
 * failure on the calling thread is available from mfa_last_error_string().
 *
 * Tensor contract (identical to the reference binding, src/mini_flash_attention/flash_attn.cpp:
 * 45-109): q, k, v and out are device pointers to contiguous fp16 arrays laid out [BH, N, D]
 * (BH = batch * heads), D = 64, out is written completely by the kernel. Launches are
 * asynchronous on `stream` (a cudaStream_t; NULL = legacy default stream) and on the device
 * that is current for the calling thread, exactly like the reference launchers.
 */
#ifndef MFA_B200_H
#define MFA_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define MFA_API __attribute__((visibility("default")))
#else
#define MFA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum mfa_status_code {
  MFA_OK = 0,
  MFA_ERR_INVALID_ARGUMENT = 1, /* null / misaligned pointer, negative or oversized extent */
  MFA_ERR_HEAD_DIM = 2,         /* unsupported D (64 only, or 32 / 64 / 128 for mfa_fwd) */
  MFA_ERR_SEQ_LEN = 3,          /* N not a multiple of 64 (mfa_fwd_simple_f16 only) */
  MFA_ERR_CAUSAL = 4,           /* reserved: causal masking is supported by every entry point */
  MFA_ERR_CUDA = 5,             /* CUDA runtime or driver error; message has the details */
  MFA_ERR_DEVICE = 6            /* current device is not an sm_100 (B200-class) GPU */
};

/*
 * Attention forward, tcgen05 kernel with two query tiles (256 rows) per CTA.
 * Replaces the reference launcher launch_flash_attn_forward
 * (src/mini_flash_attention/flash_attn_cuda.cu:370-420): same arguments, the same D == 64 check
 * and message; any N >= 1 (the reference requires N % 128 == 0, flash_attn_cuda.cu:402-407).
 * `scale` multiplies q.k before the softmax (the reference binding passes 1/sqrt(D),
 * flash_attn.cpp:94); it must be positive and finite (MFA_ERR_INVALID_ARGUMENT otherwise).
 * q, k, v and out must be memory of the current device (checked: other pointers return
 * MFA_ERR_INVALID_ARGUMENT before any launch). causal != 0 masks
 * key index > query index (the reference launcher rejects causal, flash_attn_cuda.cu:408-410;
 * the mask is the one its test and benchmark build, tests/test_forward.py:30-32).
 * bh == 0 or n == 0 is a no-op that returns MFA_OK.
 */
MFA_API int mfa_fwd_f16(const void* q, const void* k, const void* v, void* out, int64_t bh, int64_t n,
                int32_t d, float scale, int32_t causal, void* stream);

/*
 * Attention forward, single-query-tile tcgen05 kernel (128 rows per CTA, 2-stage K/V ring).
 * Replaces the reference's WMMA launcher, declared as launch_flash_attn_forward_wmma
 * (src/mini_flash_attention/flash_attn.cpp:21-31) and implemented at
 * src/mini_flash_attention/flash_attn_wmma_cuda.cu:253-289: checks D == 64 and N % 64 == 0
 * with that launcher's messages; causal != 0 masks key index > query index (that launcher
 * rejects causal, flash_attn_wmma_cuda.cu:275-277).
 */
MFA_API int mfa_fwd_simple_f16(const void* q, const void* k, const void* v, void* out, int64_t bh,
                       int64_t n, int32_t d, float scale, int32_t causal, void* stream);

/* Element type and memory layout of mfa_fwd's q, k, v and out. */
enum mfa_dtype { MFA_DTYPE_FP16 = 0, MFA_DTYPE_BF16 = 1 };
enum mfa_layout {
  MFA_LAYOUT_BHND = 0, /* [B, H, N, D] contiguous: the reference's layout */
  MFA_LAYOUT_BNHD = 1  /* [B, N, H, D] contiguous: the flash-attn style layout */
};

/*
 * General forward: `dtype` (fp16 or bf16; out has the same type), `layout` (above), B = batch
 * and H = heads given separately, head dim d = 32, 64 or 128 (others: MFA_ERR_HEAD_DIM, "This
 * kernel supports only D=32, D=64 and D=128"), any N, same causal semantics as mfa_fwd_f16; bf16 rounds P to bf16 for the P.V product, as fp16
 * inputs round it to fp16. No counterpart in the reference launchers, which take fp16
 * [B*H, N, D] only; its benchmark exposes bf16 and converts to [B, N, H, D] for flash-attn
 * (benchs/benchmark_forward.py:162-167, 188, 210-215). mfa_fwd_f16(q, k, v, out, bh, ...)
 * equals mfa_fwd(q, k, v, out, 1, bh, ..., MFA_DTYPE_FP16, MFA_LAYOUT_BHND, stream).
 */
MFA_API int mfa_fwd(const void* q, const void* k, const void* v, void* out, int64_t batch,
                    int64_t heads, int64_t n, int32_t d, float scale, int32_t causal,
                    int32_t dtype, int32_t layout, void* stream);

/*
 * mfa_fwd restricted to the query rows [q_begin, q_end) of every head: q, k, v and out are the
 * whole tensors (as for mfa_fwd), every query row in the range attends to all N keys, and only
 * those rows of out are written. For multi-GPU sharding when B*H is smaller than the number of
 * GPUs: each GPU holds the whole k and v and takes a range of query rows. causal != 0 masks
 * key index > query index as in mfa_fwd (absolute indices); a causal range must start at a
 * multiple of 256 rows (MFA_ERR_INVALID_ARGUMENT otherwise). 0 <= q_begin <= q_end <= N.
 * No counterpart in the reference, which has no multi-GPU mode.
 */
MFA_API int mfa_fwd_rows(const void* q, const void* k, const void* v, void* out, int64_t batch,
                         int64_t heads, int64_t n, int64_t q_begin, int64_t q_end, int32_t d,
                         float scale, int32_t causal, int32_t dtype, int32_t layout,
                         void* stream);

/*
 * mfa_fwd that also writes the row log-sum-exp of the scaled scores,
 * lse[bh * N + row] = ln(sum over keys of exp(scale * q.k)), fp32 [B*H, N] whatever the
 * layout: the state the backward pass needs. No counterpart in the reference (no backward).
 */
MFA_API int mfa_fwd_lse(const void* q, const void* k, const void* v, void* out, float* lse,
                        int64_t batch, int64_t heads, int64_t n, int32_t d, float scale,
                        int32_t causal, int32_t dtype, int32_t layout, void* stream);

/*
 * Backward pass (D = 64, fp16 or bf16, either layout, any N, optional causal mask): from q,
 * k, v, the forward output `out`, its gradient `dout` and `lse` of mfa_fwd_lse (same scale and
 * causal), writes dq, dk, dv (type and layout of q). dV = P^T dout, dS = P * (dout v^T - D)
 * with D = rowsum(dout * out), dq = scale * dS k, dk = scale * dS^T q. Two tcgen05 passes
 * (dq; dk and dv) and a small row pass; a stream-ordered scratch of 8 bytes per row from the
 * library's pool. Other D: MFA_ERR_HEAD_DIM "The backward pass supports only D=64". No
 * counterpart in the reference: its README lists the backward pass as future work
 * (README.md:125).
 */
MFA_API int mfa_bwd(const void* q, const void* k, const void* v, const void* out,
                    const void* dout, const float* lse, void* dq, void* dk, void* dv,
                    int64_t batch, int64_t heads, int64_t n, int32_t d, float scale,
                    int32_t causal, int32_t dtype, int32_t layout, void* stream);

/*
 * Device scratch, in bytes, that one call of mfa_fwd (or mfa_fwd_f16 / mfa_fwd_lse, and with d
 * = 64 and fp16 mfa_fwd_f16_noalloc) takes on the current device for these extents: 0 when
 * whole query blocks fill the SMs evenly, else the split plan's partial-result slots (2 x
 * (256 rows x (D + 2) floats) per CTA, one CTA per SM). dtype and layout do not change it.
 * Nothing is launched or allocated. The allocating entry points take it from a stream-ordered
 * pool of the library (outside any framework allocator) and return it on the same stream;
 * the output tensor is the caller's. No counterpart in the reference, whose launchers need
 * no scratch (its benchmark reports the allocator's peak over the calls,
 * benchs/benchmark_forward.py:266-289).
 */
MFA_API int mfa_fwd_workspace_bytes(int64_t batch, int64_t heads, int64_t n, int32_t d,
                                    int32_t causal, uint64_t* bytes);

/* Size of the static device scratch array used by mfa_fwd_f16_noalloc (20 MiB). */
#define MFA_NOALLOC_SCRATCH_BYTES 20971520u

/*
 * Allocation-free variant of mfa_fwd_f16: same kernels, arguments, checks, messages and
 * results, but it calls no cudaMalloc / cudaFree / stream-ordered or library allocator.
 * No counterpart in the reference (whose launchers need no scratch at all).
 *
 * For callers that cannot allocate device memory on this path: an engine or framework that
 * reserves the device's memory for its own allocator at start-up (a further allocation may
 * fail or fragment its pool), and code that must not enter the CUDA allocator in the middle
 * of a step (an allocation there can block or fail at a point the caller cannot recover from).
 *
 * When B*H*(N/256) does not fill the GPU evenly, the key dimension is split and partial
 * results are merged; mfa_fwd_f16 takes that scratch from a stream-ordered pool, this entry
 * point from one file-scope device array of MFA_NOALLOC_SCRATCH_BYTES in the library's device
 * image (2 x 67,584 bytes per CTA: enough for up to 155 SMs; a B200 has 148). A launch that
 * would need more returns MFA_ERR_INVALID_ARGUMENT with the required size in the message.
 *   - Nothing in the scratch has to start at zero: every part a call reads, it first writes.
 *   - The array is shared by every call on a device: calls that overlap on the GPU (issued
 *     on different streams without ordering between them) race on it and may return wrong
 *     results. Serialise them, e.g. by issuing them on one stream.
 *   - The first call on each device runs its one-time set-up (device checks, kernel
 *     attributes, cudaGetSymbolAddress of the scratch); make that first call before any
 *     stream capture. If the set-up fails with a CUDA error, the call returns MFA_ERR_CUDA
 *     and the next call tries the set-up again; only a device of the wrong architecture
 *     fails every call.
 *   - Memory cost to every user of the library: the array belongs to the library's device
 *     image, so each device on which any kernel of this library is loaded holds
 *     MFA_NOALLOC_SCRATCH_BYTES for it until the process exits, whether or not this entry
 *     point is ever called.
 */
MFA_API int mfa_fwd_f16_noalloc(const void* q, const void* k, const void* v, void* out, int64_t bh,
                        int64_t n, int32_t d, float scale, int32_t causal, void* stream);

/* Message of the last failing call made by this thread ("" if none). Replaces the
 * std::runtime_error text of the reference launchers and check_cuda
 * (src/mini_flash_attention/utils.cuh:15-21). */
MFA_API const char* mfa_last_error_string(void);

/*
 * Reads the device-side status word of `device` (synchronises that device first).
 * 0 = every kernel finished normally; 0x100 + site = a bounded mbarrier wait in some CTA
 * expired and that CTA unwound without writing its output tile. If `reset` is non-zero the
 * word is cleared afterwards. No reference counterpart: the reference kernels have no
 * bounded waits.
 */
MFA_API int mfa_device_status(int device, int* status, int reset);

/* Per-wait watchdog limit in nanoseconds used by later launches (default 2 s, min 1 ms).
 * No reference counterpart. */
MFA_API int mfa_set_watchdog_ns(uint64_t ns);

/*
 * Self-test of the watchdog path: launches a one-CTA kernel on `stream` that allocates TMEM,
 * waits on an mbarrier that nothing arrives at with the given limit, records the expiry in
 * its own status word, frees TMEM and returns. *status_out receives that word (0x100 + site
 * when the wait expired as designed). Synchronises `stream`. No reference counterpart.
 */
MFA_API int mfa_watchdog_selftest(void* stream, uint64_t timeout_ns, int* status_out);

/* Library version string. */
MFA_API const char* mfa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MFA_B200_H */
