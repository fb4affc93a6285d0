"""GPU tests of sequence lengths that are not multiples of 128 in `forward` (the reference
launcher rejects them, flash_attn_cuda.cu:402-407; the survey's third "next" row). The TMA
maps zero-fill rows past N, the last key block masks keys past N and the stores clip rows past
N; the oracle is the reference test's fp32 naive attention with its mask."""
from __future__ import annotations

import pytest
import torch

import mini_flash_attention as mfa

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-3


def naive_fp32(q, k, v, causal=False):
    d = q.shape[-1]
    scores = q.float() @ k.float().transpose(-2, -1) * d ** -0.5
    if causal:
        n = q.shape[-2]
        mask = torch.ones((n, n), dtype=torch.bool, device=q.device).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.softmax(scores, dim=-1) @ v.float()


def randn(shape, seed, dtype=torch.float16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, device="cuda", generator=g, dtype=torch.float32).to(dtype)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("bh,n", [(3, 1), (2, 17), (4, 100), (2, 130), (5, 200), (3, 300),
                                  (2, 1000), (1, 4095), (8, 8191), (64, 333)])
def test_ragged_n_matches_naive(bh, n, causal):
    q, k, v = (randn((bh, n, 64), 110 + i) for i in range(3))
    out = mfa.forward(q, k, v, causal=causal)
    assert out.shape == q.shape
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v, causal), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_ragged_bf16_bnhd(causal):
    B, N, H = 2, 777, 4
    q, k, v = (randn((B, N, H, 64), 120 + i, torch.bfloat16) for i in range(3))
    out = mfa.forward_bnhd(q, k, v, causal=causal)
    t = [x.transpose(1, 2) for x in (q, k, v)]
    torch.testing.assert_close(out.transpose(1, 2).float(), naive_fp32(*t, causal),
                               rtol=1e-2, atol=1e-2)


def test_rows_past_n_untouched_by_neighbouring_heads():
    # a head's last tile reads zeros past its own N, never the next head's rows
    bh, n = 6, 136
    q, k, v = (randn((bh, n, 64), 130 + i) for i in range(3))
    out = mfa.forward(q, k, v)
    for h in range(bh):
        one = mfa.forward(q[h:h + 1].contiguous(), k[h:h + 1].contiguous(),
                          v[h:h + 1].contiguous())
        torch.testing.assert_close(out[h:h + 1].float(), one.float(), rtol=RTOL, atol=ATOL)
