"""mini-flash-attention for B200 (sm_100a).

Drop-in for the reference package's public API (src/mini_flash_attention/__init__.py:1-3):
``forward`` and ``forward_wmma`` take fp16 q, k, v of shape [B, H, N, D] (or [B*H, N, D]),
D = 64, and return softmax(q k^T / sqrt(D)) v as fp16, computed by hand-written tcgen05
kernels. There is no CPU or Triton fallback: without the built sm_100a extension the calls
raise.
``forward_pinned`` runs the same forward on host tensors, overlapping the host<->device
copies of batch*head slices with the kernels.
"""
from ._cuda import forward, forward_pinned, forward_wmma

__all__ = ["forward", "forward_wmma", "forward_pinned"]
