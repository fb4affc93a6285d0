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


def test_workspace_query_matches_the_plan():
    """mfa_fwd_workspace_bytes: zero when whole 256-row query blocks fill the SMs evenly, else
    two partial-result slots of 256 rows x (D + 2) floats per SM."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    slot = lambda d: 256 * (d + 2) * 4  # noqa: E731
    # 256 query blocks on 148 SMs: split
    assert capi.fwd_workspace_bytes(1, 8, 8192) == 2 * sms * slot(64)
    assert capi.fwd_workspace_bytes(1, 8, 8192, d=32) == 2 * sms * slot(32)
    # 4096 query blocks (27.7 waves): whole blocks
    assert capi.fwd_workspace_bytes(16, 16, 4096) == 0
    # causal masking always splits; fewer steps than SMs use fewer CTAs
    assert capi.fwd_workspace_bytes(16, 16, 4096, causal=True) == 2 * sms * slot(64)
    assert 0 < capi.fwd_workspace_bytes(1, 1, 256, causal=True) < 2 * sms * slot(64)
    # the no-alloc entry point's array covers every D = 64 plan on this device
    assert capi.fwd_workspace_bytes(1, 8, 8192) <= capi.NOALLOC_SCRATCH_BYTES
