"""mfa_fwd_f16_noalloc, the allocation-free entry point, called through the C ABI the way a
host that cannot allocate device memory would call it, checked against mfa_fwd_f16.

Both shapes take the split plan on a B200 (too few 256-row query blocks to fill 148 SMs), so
the partial results go through the static scratch array; the two no-alloc calls run back to
back on one stream and reuse that array."""
from __future__ import annotations

import math

import pytest
import torch

from mini_flash_attention import capi

pytestmark = pytest.mark.gpu

SHAPES = [(3, 2048), (5, 1024)]  # (B*H, N): 24 and 20 query blocks -> key dimension split
D = 64
TOL = dict(atol=1e-3, rtol=1e-3)


def _inputs(bh: int, n: int, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(bh, n, D, device="cuda", dtype=torch.float16, generator=g)
            for _ in range(3)]


def test_noalloc_matches_forward_on_two_calls_in_a_row():
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream().cuda_stream
    cases = []
    for i, (bh, n) in enumerate(SHAPES):
        q, k, v = _inputs(bh, n, 1234 + i)
        ref = torch.empty_like(q)
        capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), bh, n, D, scale,
                 stream=stream)
        out = torch.full_like(q, float("nan"))
        cases.append((bh, n, q, k, v, ref, out))
    torch.cuda.synchronize()
    # two no-alloc calls in a row, no synchronisation between them
    for bh, n, q, k, v, _, out in cases:
        capi.fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bh, n, D,
                         scale, stream=stream)
    torch.cuda.synchronize()
    for _, _, _, _, _, ref, out in cases:
        assert torch.isfinite(out).all()
        torch.testing.assert_close(out, ref, **TOL)
    assert capi.device_status(torch.cuda.current_device()) == 0


def test_noalloc_rejects_bad_arguments_like_forward():
    # fails argument validation before any device work (the pointers are never used)
    with pytest.raises(capi.MfaError) as e:
        capi.fwd_noalloc(0x10000, 0x10000, 0x10000, 0x10000, 2, 256, 32, 0.125)
    assert e.value.code == capi.MFA_ERR_HEAD_DIM
    assert str(e.value) == "This kernel supports only D=64"
