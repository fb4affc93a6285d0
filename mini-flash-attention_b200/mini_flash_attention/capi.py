"""ctypes view of the C ABI in include/mfa_b200.h (libmfa_b200.so).

This is the boundary a non-Python host binds; the tests use it to call the kernels exactly
as such a host would: raw device pointers, sizes and a stream handle.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmfa_b200.so"

# Every symbol declared in include/mfa_b200.h.
EXPORTED_SYMBOLS = (
    "mfa_fwd_f16",
    "mfa_fwd_simple_f16",
    "mfa_fwd_f16_noalloc",
    "mfa_fwd",
    "mfa_fwd_rows",
    "mfa_fwd_lse",
    "mfa_bwd",
    "mfa_fwd_workspace_bytes",
    "mfa_last_error_string",
    "mfa_device_status",
    "mfa_set_watchdog_ns",
    "mfa_watchdog_selftest",
    "mfa_version",
)

MFA_OK = 0
MFA_ERR_INVALID_ARGUMENT = 1
MFA_ERR_HEAD_DIM = 2
MFA_ERR_SEQ_LEN = 3
MFA_ERR_CAUSAL = 4
MFA_ERR_CUDA = 5
MFA_ERR_DEVICE = 6
STATUS_TIMEOUT_BASE = 0x100
NOALLOC_SCRATCH_BYTES = 20971520  # MFA_NOALLOC_SCRATCH_BYTES
DTYPE_FP16, DTYPE_BF16 = 0, 1
LAYOUT_BHND, LAYOUT_BNHD = 0, 1

_LIB: ctypes.CDLL | None = None


class MfaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def load(path: str | Path | None = None) -> ctypes.CDLL:
    """Load libmfa_b200.so (once) and declare the C signatures."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    lib = ctypes.CDLL(str(path or LIB_PATH), mode=ctypes.RTLD_GLOBAL)
    fwd_args = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                ctypes.c_int64, ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_int32,
                ctypes.c_void_p]
    for name in ("mfa_fwd_f16", "mfa_fwd_simple_f16", "mfa_fwd_f16_noalloc"):
        fn = getattr(lib, name)
        fn.argtypes = fwd_args
        fn.restype = ctypes.c_int
    lib.mfa_fwd.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                    ctypes.c_int32, ctypes.c_float, ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_int32,
                                                    ctypes.c_void_p]
    lib.mfa_fwd.restype = ctypes.c_int
    lib.mfa_fwd_rows.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 5 + [
        ctypes.c_int32, ctypes.c_float, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
        ctypes.c_void_p]
    lib.mfa_fwd_rows.restype = ctypes.c_int
    lib.mfa_fwd_lse.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64, ctypes.c_int64,
                                                        ctypes.c_int64, ctypes.c_int32,
                                                        ctypes.c_float, ctypes.c_int32,
                                                        ctypes.c_int32, ctypes.c_int32,
                                                        ctypes.c_void_p]
    lib.mfa_fwd_lse.restype = ctypes.c_int
    lib.mfa_bwd.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int64, ctypes.c_int64,
                                                    ctypes.c_int64, ctypes.c_int32, ctypes.c_float,
                                                    ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                    ctypes.c_void_p]
    lib.mfa_bwd.restype = ctypes.c_int
    lib.mfa_last_error_string.argtypes = []
    lib.mfa_last_error_string.restype = ctypes.c_char_p
    lib.mfa_device_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.c_int]
    lib.mfa_device_status.restype = ctypes.c_int
    lib.mfa_set_watchdog_ns.argtypes = [ctypes.c_uint64]
    lib.mfa_set_watchdog_ns.restype = ctypes.c_int
    lib.mfa_watchdog_selftest.argtypes = [ctypes.c_void_p, ctypes.c_uint64,
                                          ctypes.POINTER(ctypes.c_int)]
    lib.mfa_watchdog_selftest.restype = ctypes.c_int
    lib.mfa_version.argtypes = []
    lib.mfa_version.restype = ctypes.c_char_p
    lib.mfa_fwd_workspace_bytes.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int32, ctypes.c_int32,
                                            ctypes.POINTER(ctypes.c_uint64)]
    lib.mfa_fwd_workspace_bytes.restype = ctypes.c_int
    if path is None:
        _LIB = lib
    return lib


def last_error() -> str:
    return load().mfa_last_error_string().decode()


def _check(rc: int) -> None:
    if rc != MFA_OK:
        raise MfaError(rc, last_error())


def fwd(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, bh: int, n: int, d: int,
        scale: float, causal: bool = False, stream: int = 0, simple: bool = False) -> None:
    """Launch mfa_fwd_f16 (or mfa_fwd_simple_f16) on raw device pointers; raises MfaError."""
    lib = load()
    fn = lib.mfa_fwd_simple_f16 if simple else lib.mfa_fwd_f16
    _check(fn(q_ptr, k_ptr, v_ptr, out_ptr, bh, n, d, scale, int(causal), stream))


def fwd_noalloc(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, bh: int, n: int, d: int,
                scale: float, causal: bool = False, stream: int = 0) -> None:
    """Launch mfa_fwd_f16_noalloc (no device allocation; static scratch shared by all calls
    on a device, so calls must not overlap on the GPU); raises MfaError."""
    _check(load().mfa_fwd_f16_noalloc(q_ptr, k_ptr, v_ptr, out_ptr, bh, n, d, scale,
                                       int(causal), stream))


def fwd_general(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, batch: int, heads: int,
                n: int, d: int, scale: float, causal: bool = False, dtype: int = DTYPE_FP16,
                layout: int = LAYOUT_BHND, stream: int = 0) -> None:
    """Launch mfa_fwd (dtype and layout selectable); raises MfaError."""
    _check(load().mfa_fwd(q_ptr, k_ptr, v_ptr, out_ptr, batch, heads, n, d, scale, int(causal),
                          dtype, layout, stream))


def fwd_rows(q_ptr: int, k_ptr: int, v_ptr: int, out_ptr: int, batch: int, heads: int,
             n: int, q_begin: int, q_end: int, d: int, scale: float, causal: bool = False,
             dtype: int = DTYPE_FP16, layout: int = LAYOUT_BHND, stream: int = 0) -> None:
    """Launch mfa_fwd_rows (query rows [q_begin, q_end) of every head); raises MfaError."""
    _check(load().mfa_fwd_rows(q_ptr, k_ptr, v_ptr, out_ptr, batch, heads, n, q_begin, q_end, d,
                               scale, int(causal), dtype, layout, stream))


def bwd(q_ptr: int, k_ptr: int, v_ptr: int, o_ptr: int, do_ptr: int, lse_ptr: int, dq_ptr: int,
        dk_ptr: int, dv_ptr: int, batch: int, heads: int, n: int, d: int, scale: float,
        causal: bool = False, dtype: int = DTYPE_FP16, layout: int = LAYOUT_BHND,
        stream: int = 0) -> None:
    """Launch mfa_bwd; raises MfaError."""
    _check(load().mfa_bwd(q_ptr, k_ptr, v_ptr, o_ptr, do_ptr, lse_ptr, dq_ptr, dk_ptr, dv_ptr,
                          batch, heads, n, d, scale, int(causal), dtype, layout, stream))


def fwd_workspace_bytes(batch: int, heads: int, n: int, d: int = 64,
                        causal: bool = False) -> int:
    """Device scratch bytes one forward call takes on the current device (0 unless the
    key dimension is split); nothing is launched or allocated. Raises MfaError."""
    out = ctypes.c_uint64(0)
    _check(load().mfa_fwd_workspace_bytes(batch, heads, n, d, int(causal), ctypes.byref(out)))
    return out.value


def device_status(device: int = 0, reset: bool = True) -> int:
    st = ctypes.c_int(0)
    _check(load().mfa_device_status(device, ctypes.byref(st), int(reset)))
    return st.value


def set_watchdog_ns(ns: int) -> None:
    _check(load().mfa_set_watchdog_ns(ns))


def watchdog_selftest(timeout_ns: int, stream: int = 0) -> int:
    st = ctypes.c_int(-1)
    _check(load().mfa_watchdog_selftest(stream, timeout_ns, ctypes.byref(st)))
    return st.value


def version() -> str:
    return load().mfa_version().decode()
