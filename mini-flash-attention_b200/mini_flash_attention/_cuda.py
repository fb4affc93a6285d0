"""Extension loader and Python entry points.

Mirrors src/mini_flash_attention/_cuda.py:8-45 of the reference: a module-level cache of the
compiled extension and two thin wrappers that forward ``causal`` to it. Unlike the reference,
nothing is JIT-compiled at call time: the sm_100a library and its binding are built ahead of
time (``python -m mini_flash_attention._build``) into this package directory, and a missing
build is an error, never a fallback.
"""
import ctypes
from pathlib import Path

import torch

_EXTENSION = None
_PKG_DIR = Path(__file__).resolve().parent


def _load_extension():
    global _EXTENSION

    if _EXTENSION is not None:
        return _EXTENSION
    try:
        # The binding links libmfa_b200.so by soname; load that first from this directory.
        ctypes.CDLL(str(_PKG_DIR / "libmfa_b200.so"), mode=ctypes.RTLD_GLOBAL)
        from . import mfa_b200_C as ext  # noqa: PLC0415  (built in-tree)
    except (ImportError, OSError) as exc:
        raise RuntimeError(
            "mini_flash_attention: the sm_100a extension is not built in "
            f"{_PKG_DIR} ({exc}); run `python -m mini_flash_attention._build`"
        ) from exc
    _EXTENSION = ext
    return _EXTENSION


def forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    return _load_extension().forward(q, k, v, causal)


def forward_wmma(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    return _load_extension().forward_wmma(q, k, v, causal)
