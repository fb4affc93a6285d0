"""ctypes loader for oracle/_ref/libmfa_ref.so, the reference's own CuTe and WMMA kernels
compiled from its sources by oracle/build_ref.py (test infrastructure only; GPU only).

ref_cute_fwd / ref_wmma_fwd wrap launch_flash_attn_forward
(src/mini_flash_attention/flash_attn_cuda.cu:370-420) and the WMMA launcher
(src/mini_flash_attention/flash_attn_wmma_cuda.cu:253-289); exceptions become return code 1
with the message in ref_last_error().
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libmfa_ref.so"
_LIB = None


def available() -> bool:
    return LIB_PATH.exists()


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        lib = ctypes.CDLL(str(LIB_PATH))
        args = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
        for name in ("ref_cute_fwd", "ref_wmma_fwd"):
            getattr(lib, name).argtypes = args
            getattr(lib, name).restype = ctypes.c_int
        lib.ref_last_error.restype = ctypes.c_char_p
        _LIB = lib
    return _LIB


def reference_forward(q, k, v, kernel: str = "cute", causal: bool = False):
    """Run the reference kernel on CUDA fp16 tensors [..., N, D]; returns a new tensor.

    The output starts as zeros, as the reference binding allocates it (flash_attn.cpp:86).
    """
    import torch

    lib = load()
    fn = lib.ref_cute_fwd if kernel == "cute" else lib.ref_wmma_fwd
    out = torch.zeros_like(q)
    n, d = q.shape[-2], q.shape[-1]
    bh = q.numel() // (n * d)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bh, n, d,
            1.0 / (d ** 0.5), int(causal), stream)
    if rc != 0:
        raise RuntimeError(lib.ref_last_error().decode())
    return out
