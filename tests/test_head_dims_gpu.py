"""GPU tests of head dims 32 and 128 in `forward` / `forward_bnhd` / `mfa_fwd` (the reference
kernels take D = 64 only, flash_attn_cuda.cu:399-401; its test lists D = 32 and D = 128 cases
commented out, tests/test_forward.py:12,15, which are run here). D = 32 uses 64-byte-swizzled
tiles and two 128-row tiles per CTA; D = 128 uses two 64-column TMA boxes per tile and one
128-row tile per CTA. Oracle: the reference test's fp32 naive attention, scale D^-0.5."""
from __future__ import annotations

import math

import pytest
import torch

import mini_flash_attention as mfa
from mini_flash_attention import capi

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


@pytest.mark.parametrize("D", [32, 128])
@pytest.mark.parametrize(("B", "H", "N"), [(1, 1, 128), (2, 3, 128), (1, 2, 2048)])
def test_reference_commented_out_shapes(B, H, N, D):
    # tests/test_forward.py:12,15 list (1, 1, 128, 32) and (2, 3, 128, 128)
    torch.manual_seed(0)
    q = torch.randn((B, H, N, D), device="cuda", dtype=torch.float16).contiguous()
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    out = mfa.forward(q, k, v)
    assert out.shape == q.shape and out.dtype == q.dtype
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("D", [32, 128])
@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("bh,n", [(8, 8192), (3, 1000), (16, 512), (1, 4096), (64, 256),
                                  (2, 77)])
def test_head_dim_shapes(D, causal, bh, n):
    q, k, v = (randn((bh, n, D), 200 + i) for i in range(3))
    out = mfa.forward(q, k, v, causal=causal)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v, causal), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("D", [32, 128])
def test_head_dim_bf16_bnhd(D):
    B, N, H = 2, 1024, 3
    q, k, v = (randn((B, N, H, D), 210 + i, torch.bfloat16) for i in range(3))
    out = mfa.forward_bnhd(q, k, v, causal=True)
    t = [x.transpose(1, 2).contiguous() for x in (q, k, v)]
    ref = mfa.forward(*t, causal=True).transpose(1, 2)
    assert torch.equal(out, ref)
    torch.testing.assert_close(out.transpose(1, 2).float(), naive_fp32(*t, True), rtol=1e-2,
                               atol=1e-2)


@pytest.mark.parametrize("D", [32, 128])
def test_v_scaling_exact(D):
    q, k, v = (randn((4, 1024, D), 220 + i) for i in range(3))
    a = mfa.forward(q, k, v)
    b = mfa.forward(q, k, v * 2)
    normal = a.abs() >= 2.0 ** -14
    assert torch.equal((a.float() * 2)[normal], b.float()[normal])


def test_capi_head_dim_128():
    B, H, N, D = 1, 4, 768, 128
    q, k, v = (randn((B, H, N, D), 230 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    capi.fwd_general(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, N, D,
                     1 / math.sqrt(D), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v), rtol=RTOL, atol=ATOL)
    assert capi.device_status(torch.cuda.current_device()) == 0
