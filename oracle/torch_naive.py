"""The reference benchmark's naive torch attention, for host CPU cores (oracle; test/bench
infrastructure only).

Restates benchs/benchmark_forward.py:98-115 (TorchBackend.run): upcast to fp32,
scores = q k^T * D^-0.5, optional causal mask, softmax, probs @ v, cast back to q's dtype.
This is the reference's own CPU-runnable path for the hot op; bench.py times it as the CPU
baseline and as the reference arm.
"""
from __future__ import annotations

import torch


def torch_naive_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          causal: bool = False) -> torch.Tensor:
    scale = q.shape[-1] ** -0.5
    scores = q.float() @ k.float().transpose(-2, -1) * scale
    if causal:
        seq_len = q.shape[-2]
        mask = torch.ones((seq_len, seq_len), dtype=torch.bool, device=q.device).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return (probs @ v.float()).to(q.dtype)
