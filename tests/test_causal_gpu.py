"""GPU parity tests of causal masking (key index > query index masked).

The reference kernels reject causal=True (flash_attn_cuda.cu:408-410,
flash_attn_wmma_cuda.cu:275-277); its test builds the mask for the naive oracle as
ones(N, N).triu(1) (tests/test_forward.py:30-32), and that oracle is the parity target here,
with the same tolerances as the non-causal tests. The shapes exercise the causal schedule:
query blocks of unequal length split evenly over the SMs, pieces that hold only masked keys
for some rows, a last query block of a single 128-row tile (N % 256 == 128), and the 64-key
tail of the single-tile entry point.
"""
from __future__ import annotations

import math

import pytest
import torch

import mini_flash_attention as mfa
from mini_flash_attention import capi

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 1e-3


def naive_fp32(q, k, v, causal=True):
    d = q.shape[-1]
    scores = q.float() @ k.float().transpose(-2, -1) * d ** -0.5
    if causal:
        n = q.shape[-2]
        mask = torch.ones((n, n), dtype=torch.bool, device=q.device).triu(1)
        scores = scores.masked_fill(mask, float("-inf"))
    return torch.softmax(scores, dim=-1) @ v.float()


def causal_rows_fp64(q, k, v, rows):
    """Exact causal attention for some query rows of every head."""
    d = q.shape[-1]
    q3 = q.reshape(-1, q.shape[-2], d).double()
    k3 = k.reshape(-1, k.shape[-2], d).double()
    v3 = v.reshape(-1, v.shape[-2], d).double()
    out = torch.empty(q3.shape[0], len(rows), d, dtype=torch.float64, device=q.device)
    for i, r in enumerate(rows):
        s = torch.einsum("hd,hkd->hk", q3[:, r], k3[:, : r + 1]) * d ** -0.5
        out[:, i] = torch.einsum("hk,hkd->hd", torch.softmax(s, dim=-1), v3[:, : r + 1])
    return out


def randn(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g, dtype=torch.float32) * scale).half()


@pytest.mark.parametrize("fn", [mfa.forward, mfa.forward_wmma], ids=["forward", "forward_wmma"])
@pytest.mark.parametrize(("B", "H", "N", "D"), [(1, 2, 128, 64), (2, 1, 256, 64),
                                                (1, 2, 2048, 64)])
def test_reference_shapes_causal(fn, B, H, N, D):
    torch.manual_seed(0)
    q = torch.randn((B, H, N, D), device="cuda", dtype=torch.float16).contiguous()
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    expected = naive_fp32(q, k, v, causal=True)
    actual = fn(q, k, v, causal=True)
    torch.testing.assert_close(actual.float(), expected, rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(actual, expected.half(), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize(("fn", "bh", "n"), [
    (mfa.forward, 1, 4096),     # 272 steps over 148 CTAs: many one- and two-block pieces
    (mfa.forward, 3, 384),      # last query block is a single 128-row tile
    (mfa.forward, 2, 1152),
    (mfa.forward, 16, 1024),
    (mfa.forward, 64, 512),
    (mfa.forward_wmma, 3, 192),  # 64-key tail
    (mfa.forward_wmma, 2, 640),
    (mfa.forward_wmma, 1, 4096),
], ids=["b1n4096", "b3n384", "b2n1152", "b16n1024", "b64n512", "wmma-b3n192", "wmma-b2n640",
        "wmma-b1n4096"])
def test_schedule_shapes_causal(fn, bh, n):
    q, k, v = (randn((bh, n, 64), 10 + i) for i in range(3))
    expected = naive_fp32(q, k, v)
    actual = fn(q, k, v, causal=True)
    assert torch.isfinite(actual).all()
    torch.testing.assert_close(actual.float(), expected, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("bh,n,qk_scale", [(8, 8192, 1.0), (4, 16384, 3.0)])
def test_full_size_causal_sampled_rows(bh, n, qk_scale):
    q, k = randn((bh, n, 64), 1, qk_scale), randn((bh, n, 64), 2, qk_scale)
    v = randn((bh, n, 64), 3)
    out = mfa.forward(q, k, v, causal=True)
    assert torch.isfinite(out).all()
    rows = sorted({0, 1, 127, 128, 255, 256, 1000, n // 2 - 1, n // 2, n - 129, n - 2, n - 1})
    exact = causal_rows_fp64(q, k, v, rows)
    got = out[:, rows].double()
    torch.testing.assert_close(got, exact, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("fn", [mfa.forward, mfa.forward_wmma], ids=["forward", "forward_wmma"])
def test_first_row_is_v0_exactly(fn):
    q, k, v = (randn((5, 1024, 64), 20 + i) for i in range(3))
    out = fn(q, k, v, causal=True)
    assert torch.equal(out[:, 0], v[:, 0])


def test_future_keys_do_not_matter():
    n = 2048
    q, k, v = (randn((4, n, 64), 30 + i) for i in range(3))
    full = mfa.forward(q, k, v, causal=True)
    # change the second half of K and V: the first half of the output must not move
    k2, v2 = k.clone(), v.clone()
    k2[:, n // 2:] = randn((4, n // 2, 64), 40)
    v2[:, n // 2:] = randn((4, n // 2, 64), 41)
    other = mfa.forward(q, k2, v2, causal=True)
    assert torch.equal(full[:, : n // 2], other[:, : n // 2])
    # and a shorter sequence gives the same first rows (different schedule: within tolerance)
    short = mfa.forward(q[:, : n // 2].contiguous(), k[:, : n // 2].contiguous(),
                        v[:, : n // 2].contiguous(), causal=True)
    torch.testing.assert_close(short.float(), full[:, : n // 2].float(), rtol=RTOL, atol=ATOL)


def test_last_row_matches_non_causal():
    q, k, v = (randn((6, 1024, 64), 50 + i) for i in range(3))
    c = mfa.forward(q, k, v, causal=True)
    f = mfa.forward(q, k, v, causal=False)
    torch.testing.assert_close(c[:, -1].float(), f[:, -1].float(), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("noalloc", [False, True], ids=["mfa_fwd_f16", "mfa_fwd_f16_noalloc"])
def test_capi_causal(noalloc):
    bh, n = 3, 1536
    q, k, v = (randn((bh, n, 64), 60 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    call = capi.fwd_noalloc if noalloc else capi.fwd
    call(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bh, n, 64, 1 / math.sqrt(64),
         causal=True, stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v), rtol=RTOL, atol=ATOL)
    assert capi.device_status(torch.cuda.current_device()) == 0
