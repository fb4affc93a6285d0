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
    """softmax(q k^T / sqrt(D)) v on [B, H, N, D] (or [B*H, N, D]) tensors: fp16 or bf16,
    D = 32, 64 or 128, any N; causal=True masks key index > query index."""
    return _load_extension().forward(q, k, v, causal)


def forward_lse(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                causal: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """forward plus the row log-sum-exp ln(sum_k exp(q.k / sqrt(D))) as fp32 of shape q.shape[:-1]."""
    out, lse = _load_extension().forward_lse(q, k, v, causal)
    return out, lse


def backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor,
             lse: torch.Tensor, dout: torch.Tensor,
             causal: bool = False) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients (dq, dk, dv) of forward(q, k, v, causal) for the output gradient dout, given
    the forward's out and lse (forward_lse). D = 64, fp16 or bf16."""
    dq, dk, dv = _load_extension().backward(q, k, v, out, lse, dout.contiguous(), causal)
    return dq, dk, dv


class _Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal):
        out, lse = forward_lse(q, k, v, causal)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal = causal
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = backward(q, k, v, out, lse, dout, ctx.causal)
        return dq, dk, dv, None


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
              causal: bool = False) -> torch.Tensor:
    """Differentiable forward: the tcgen05 forward kernel, with the tcgen05 backward kernels as
    its autograd backward (D = 64 for gradients)."""
    return _Attention.apply(q, k, v, causal)


def forward_rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_begin: int, q_end: int,
                 out: torch.Tensor | None = None, causal: bool = False) -> torch.Tensor:
    """Forward of the query rows [q_begin, q_end) of every head, each against all N keys (with
    ``causal``, the keys up to its own index; the range must then start at a multiple of 256
    rows), written into ``out`` (same shape as q; a new tensor if None) and nowhere else: the
    per-GPU call of the query-row sharding used when B*H is smaller than the number of GPUs
    (every GPU holds the whole k and v)."""
    if out is None:
        out = torch.empty_like(q)
    _load_extension().forward_rows(q, k, v, out, int(q_begin), int(q_end), bool(causal))
    return out


def forward_bnhd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 causal: bool = False) -> torch.Tensor:
    """forward on [B, N, H, D] tensors (the flash-attn layout); the output has that layout."""
    return _load_extension().forward_bnhd(q, k, v, causal)


def forward_wmma(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    return _load_extension().forward_wmma(q, k, v, causal)


def pinned_chunk_bounds(rows: int, chunks: int) -> list[int]:
    """Row bounds of the pieces of ``forward_pinned``: ``chunks`` pieces of decreasing size
    (weights 2^(c-2), ..., 2, 1, 1), every piece at least one row. The copy-in of all pieces
    bounds the pipeline; small last pieces keep short the compute and copy-out that follow
    it."""
    chunks = max(1, min(chunks, rows))
    weights = [2 ** (chunks - 2 - i) for i in range(chunks - 1)] + [1] if chunks > 1 else [1]
    total = sum(weights)
    bounds, acc = [0], 0
    for i, w in enumerate(weights):
        acc += w
        b = rows * acc // total
        b = max(b, bounds[-1] + 1)               # at least one row per piece
        b = min(b, rows - (chunks - 1 - i))      # leave a row for every later piece
        bounds.append(b)
    bounds[-1] = rows
    return bounds


def forward_pinned(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                   out: torch.Tensor | None = None, chunks: int = 4,
                   device: torch.device | int | None = None) -> torch.Tensor:
    """Attention forward on host tensors: fp16 / bf16 q, k, v in (preferably pinned) CPU
    memory, result written to a host tensor (``out`` or a new pinned one).

    The batch*head rows are cut into ``chunks`` pieces of decreasing size
    (``pinned_chunk_bounds``) that move through three CUDA streams: piece i+1 is copied in
    while piece i is computed and piece i-1 is copied back, so the host<->device transfers
    overlap the kernels. The pipeline runs in the C++ extension (one call, no per-piece Python
    work). Synchronous: returns when the result is in ``out``. Same shape / dtype / error
    contract as ``forward``.
    """
    if q.is_cuda or k.is_cuda or v.is_cuda:
        raise RuntimeError("forward_pinned expects host tensors; use forward for CUDA tensors")
    if not (q.shape == k.shape == v.shape):
        raise RuntimeError("k must have the same shape as q")
    if q.dim() not in (3, 4):
        raise RuntimeError("q must have shape [B, H, N, D]")
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    n, d = q.shape[-2], q.shape[-1]
    bh = q.numel() // (n * d) if n * d else 0
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
    if bh == 0 or n == 0:
        return out
    if not out.is_contiguous():
        raise RuntimeError("out must be contiguous")
    q3, k3, v3 = (x.contiguous().reshape(bh, n, d) for x in (q, k, v))
    o3 = out.reshape(bh, n, d)
    _load_extension().forward_pinned(q3, k3, v3, o3, causal, pinned_chunk_bounds(bh, chunks),
                                     dev.index)
    return out
