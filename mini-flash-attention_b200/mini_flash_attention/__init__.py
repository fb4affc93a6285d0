"""mini-flash-attention for B200 (sm_100a).

Drop-in for the reference package's public API (src/mini_flash_attention/__init__.py:1-3):
``forward`` and ``forward_wmma`` take q, k, v of shape [B, H, N, D] (or [B*H, N, D]) and return
softmax(q k^T / sqrt(D)) v, computed by hand-written tcgen05 kernels; ``causal=True`` masks key
index > query index. ``forward`` takes fp16 or bf16, D = 32, 64 or 128 and any N;
``forward_wmma`` keeps the reference's contract (fp16, D = 64, N % 64 == 0). There is no CPU or Triton fallback: without the built sm_100a extension
the calls raise.
``forward_bnhd`` is ``forward`` on [B, N, H, D] tensors (the flash-attn layout).
``forward_lse`` also returns the row log-sum-exp; ``backward`` computes (dq, dk, dv) from it
(D = 64); ``attention`` is the differentiable forward built from the two.
``forward_pinned`` runs the same forward on host tensors, overlapping the host<->device
copies of batch*head slices with the kernels. ``forward_rows`` computes a range of query rows
of every head (the per-GPU call when fewer batch*head rows than GPUs are sharded by query rows).
"""
from ._cuda import (attention, backward, forward, forward_bnhd, forward_lse, forward_pinned,
                    forward_rows, forward_wmma)

__all__ = ["forward", "forward_wmma", "forward_bnhd", "forward_pinned", "forward_rows",
           "forward_lse", "backward", "attention"]
