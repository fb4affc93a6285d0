"""GPU tests of the bf16 inputs and the [B, N, H, D] layout (the reference benchmark offers
--dtype bf16 and converts inputs to [B, N, H, D] for flash-attn,
benchs/benchmark_forward.py:162-167, 188, 210-215).

bf16 is checked against the fp32 naive oracle with the reference test's tolerance
(rtol = atol = 1e-2, tests/test_forward.py:38) and a mean-error bound; the layout is checked
bit for bit: forward_bnhd on [B, N, H, D] must equal forward on the same data transposed to
[B, H, N, D] (the same arithmetic on the same values, only the addresses differ).
"""
from __future__ import annotations

import math

import pytest
import torch

import mini_flash_attention as mfa
from mini_flash_attention import capi

pytestmark = pytest.mark.gpu


def naive_fp32(q, k, v, causal=False):
    d = q.shape[-1]
    scores = q.float() @ k.float().transpose(-2, -1) * d ** -0.5
    if causal:
        n = q.shape[-2]
        mask = torch.ones((n, n), dtype=torch.bool, device=q.device).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.softmax(scores, dim=-1) @ v.float()


def randn(shape, seed, dtype, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g, dtype=torch.float32) * scale).to(dtype)


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("B,H,N", [(1, 2, 128), (2, 1, 256), (1, 2, 2048), (1, 8, 4096),
                                   (4, 16, 512)])
def test_bf16_matches_naive(B, H, N, causal):
    q, k, v = (randn((B, H, N, 64), 70 + i, torch.bfloat16) for i in range(3))
    out = mfa.forward(q, k, v, causal=causal)
    assert out.dtype == torch.bfloat16 and out.shape == q.shape
    expected = naive_fp32(q, k, v, causal)
    torch.testing.assert_close(out.float(), expected, rtol=1e-2, atol=1e-2)
    # bf16 keeps 8 mantissa bits: output rounding alone is ~2^-9 relative
    assert (out.float() - expected).abs().mean().item() < 2e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("B,N,H", [(1, 8192, 8), (2, 1024, 3), (16, 256, 16), (1, 384, 5)])
def test_bnhd_equals_bhnd_bitwise(B, N, H, causal, dtype):
    q, k, v = (randn((B, N, H, 64), 80 + i, dtype) for i in range(3))
    out = mfa.forward_bnhd(q, k, v, causal=causal)
    assert out.shape == q.shape and out.dtype == dtype
    t = [x.transpose(1, 2).contiguous() for x in (q, k, v)]
    ref = mfa.forward(*t, causal=causal).transpose(1, 2)
    assert torch.equal(out, ref)


def test_bnhd_rejects_3d():
    q = torch.zeros(4, 128, 64, device="cuda", dtype=torch.float16)
    with pytest.raises(RuntimeError, match=r"q must have shape \[B, N, H, D\]"):
        mfa.forward_bnhd(q, q, q)


def test_bf16_fp16_agree():
    # the same values in both types: the results differ only by bf16's coarser P and output
    qh, kh, vh = (randn((2, 4, 1024, 64), 90 + i, torch.bfloat16) for i in range(3))
    a = mfa.forward(qh, kh, vh).float()
    b = mfa.forward(qh.half(), kh.half(), vh.half()).float()
    torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("layout", [capi.LAYOUT_BHND, capi.LAYOUT_BNHD], ids=["bhnd", "bnhd"])
def test_capi_general_entry(layout):
    B, H, N = 2, 3, 1024
    shape = (B, H, N, 64) if layout == capi.LAYOUT_BHND else (B, N, H, 64)
    q, k, v = (randn(shape, 100 + i, torch.bfloat16) for i in range(3))
    out = torch.full_like(q, float("nan"))
    capi.fwd_general(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, N, 64,
                     1 / math.sqrt(64), causal=True, dtype=capi.DTYPE_BF16, layout=layout,
                     stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    expect = mfa.forward_bnhd(q, k, v, causal=True) if layout == capi.LAYOUT_BNHD else \
        mfa.forward(q, k, v, causal=True)
    assert torch.equal(out, expect)
    assert capi.device_status(torch.cuda.current_device()) == 0
