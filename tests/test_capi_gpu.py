"""GPU tests through the C ABI (include/mfa_b200.h via ctypes), as a non-Python host calls it:
raw device pointers, sizes, a stream handle; plus the device-side watchdog and status word."""
from __future__ import annotations

import pytest
import torch

from mini_flash_attention import capi

pytestmark = pytest.mark.gpu


def naive_fp32(q, k, v):
    d = q.shape[-1]
    return torch.softmax(q.float() @ k.float().transpose(-2, -1) * d ** -0.5, dim=-1) @ v.float()


@pytest.mark.parametrize("simple", [False, True], ids=["mfa_fwd_f16", "mfa_fwd_simple_f16"])
@pytest.mark.parametrize(("bh", "n"), [(1, 128), (3, 256), (4, 1024)])
def test_c_abi_forward(simple, bh, n):
    g = torch.Generator(device="cuda")
    g.manual_seed(bh * 1000 + n)
    q, k, v = (torch.randn((bh, n, 64), device="cuda", generator=g).half() for _ in range(3))
    out = torch.full_like(q, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bh, n, 64, 0.125,
             stream=stream, simple=simple)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all(), "kernel left output elements unwritten"
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v), atol=1e-3, rtol=1e-3)
    assert capi.device_status(torch.cuda.current_device()) == 0


def test_c_abi_scale_argument_is_used():
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    q, k, v = (torch.randn((2, 256, 64), device="cuda", generator=g).half() for _ in range(3))
    out = torch.empty_like(q)
    capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 2, 256, 64, 0.05,
             stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = torch.softmax(q.float() @ k.float().transpose(-2, -1) * 0.05, dim=-1) @ v.float()
    torch.testing.assert_close(out.float(), want, atol=1e-3, rtol=1e-3)


def test_watchdog_expires_and_context_survives():
    """A wait on a barrier that nothing signals must give up after its limit, report it in
    the status word, release TMEM and leave the context usable."""
    status = capi.watchdog_selftest(20_000_000)  # 20 ms
    assert status == capi.STATUS_TIMEOUT_BASE + 8
    # the context is still healthy: a real forward runs and is correct afterwards
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    q, k, v = (torch.randn((2, 512, 64), device="cuda", generator=g).half() for _ in range(3))
    out = torch.empty_like(q)
    capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 2, 512, 64, 0.125,
             stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v), atol=1e-3, rtol=1e-3)
    assert capi.device_status(torch.cuda.current_device()) == 0


def test_device_status_clean_after_many_launches():
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    q, k, v = (torch.randn((16, 2048, 64), device="cuda", generator=g).half() for _ in range(3))
    out = torch.empty_like(q)
    s = torch.cuda.current_stream().cuda_stream
    for _ in range(20):
        capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 16, 2048, 64, 0.125,
                 stream=s)
    assert capi.device_status(torch.cuda.current_device()) == 0
