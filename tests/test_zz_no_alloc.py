"""mfa_fwd_f16_noalloc, the allocation-free entry point, called through the C ABI the way a
host that cannot allocate device memory would call it (an engine that has reserved the GPU's
memory for its own allocator, or a step that must not enter the CUDA allocator).

Both shapes take the split plan on a B200 (too few 256-row query blocks to fill 148 SMs), so
the partial results go through the static scratch array; the no-alloc calls run back to back
on one stream and reuse that array. Checked against mfa_fwd_f16 and against fp32 attention;
and, in a fresh process, that the calls leave the device's free memory unchanged while the
allocating entry point's first split call visibly takes its pool allocation."""
from __future__ import annotations

import math
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from mini_flash_attention import capi

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
SHAPES = [(3, 2048), (5, 1024)]  # (B*H, N): 24 and 20 query blocks -> key dimension split
D = 64
SCALE = 1.0 / math.sqrt(D)
TOL = dict(atol=1e-3, rtol=1e-3)  # as the other parity tests against fp32 attention


def _inputs(bh: int, n: int, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return [torch.randn(bh, n, D, device="cuda", dtype=torch.float16, generator=g)
            for _ in range(3)]


def _naive_fp32(q, k, v, causal=False):
    s = q.float() @ k.float().transpose(-2, -1) * SCALE
    if causal:
        n = q.shape[-2]
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=q.device).triu(1),
                          float("-inf"))
    return torch.softmax(s, dim=-1) @ v.float()


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_noalloc_matches_forward_on_two_calls_in_a_row(causal):
    stream = torch.cuda.current_stream().cuda_stream
    cases = []
    for i, (bh, n) in enumerate(SHAPES):
        q, k, v = _inputs(bh, n, 1234 + i)
        ref = torch.empty_like(q)
        capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), bh, n, D, SCALE,
                 causal=causal, stream=stream)
        out = torch.full_like(q, float("nan"))
        cases.append((bh, n, q, k, v, ref, out))
    torch.cuda.synchronize()
    # two no-alloc calls in a row, no synchronisation between them
    for bh, n, q, k, v, _, out in cases:
        capi.fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), bh, n, D,
                         SCALE, causal=causal, stream=stream)
    torch.cuda.synchronize()
    for _, _, q, k, v, ref, out in cases:
        assert torch.isfinite(out).all()
        torch.testing.assert_close(out, ref, **TOL)
        torch.testing.assert_close(out.float(), _naive_fp32(q, k, v, causal), **TOL)
    assert capi.device_status(torch.cuda.current_device()) == 0


def test_noalloc_rejects_bad_arguments_like_forward():
    # real device tensors of head dim 32: both entry points fail the D check before any launch
    q, k, v = (x[..., :32].contiguous() for x in _inputs(2, 256, 99))
    out = torch.full_like(q, 7.0)
    for call in (capi.fwd, capi.fwd_noalloc):
        with pytest.raises(capi.MfaError) as e:
            call(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 2, 256, 32, SCALE)
        assert e.value.code == capi.MFA_ERR_HEAD_DIM
        assert str(e.value) == "This kernel supports only D=64"
    q, k, v = _inputs(2, 256, 98)
    out = torch.full_like(q, 7.0)
    with pytest.raises(capi.MfaError) as e:
        capi.fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 2, 256, D,
                         0.0)
    assert e.value.code == capi.MFA_ERR_INVALID_ARGUMENT
    torch.cuda.synchronize()
    assert (out == 7.0).all()  # nothing was launched


# Runs in a fresh process so that no earlier test has mapped the allocating entry point's pool.
# The library's module is loaded and every forward kernel's attributes are set first
# (mfa_device_status runs the set-up of the allocating entry points, which allocates nothing),
# so that later differences in free device memory can only come from allocations.
_FREE_MEMORY_PROBE = r"""
import math, sys
import torch
from mini_flash_attention import capi
torch.cuda.init()
D, scale = 64, 1.0 / math.sqrt(64)
bufs = []
for bh, n in ((3, 2048), (5, 1024)):
    g = torch.Generator(device="cuda").manual_seed(bh)
    q, k, v = (torch.randn(bh, n, D, device="cuda", dtype=torch.float16, generator=g)
               for _ in range(3))
    bufs.append((bh, n, q, k, v, torch.empty_like(q)))
capi.device_status(0, reset=False)
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for _ in range(2):
    for bh, n, q, k, v, o in bufs:
        capi.fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), bh, n, D, scale)
torch.cuda.synchronize()
free1 = torch.cuda.mem_get_info()[0]
bh, n, q, k, v, o = bufs[0]
capi.fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), bh, n, D, scale)
torch.cuda.synchronize()
free2 = torch.cuda.mem_get_info()[0]
print(free0, free1, free2)
"""


def test_noalloc_takes_no_device_memory():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join(
        [str(ROOT / "mini-flash-attention_b200"), str(ROOT), env.get("PYTHONPATH", "")])
    res = subprocess.run([sys.executable, "-c", _FREE_MEMORY_PROBE], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-2000:]
    free0, free1, free2 = (int(x) for x in res.stdout.split()[-3:])
    mib = 1 << 20
    # Four no-alloc split calls: at most the lazily loaded code of the merge kernel (well
    # below 4 MiB); a 20 MB workspace allocation would show.
    assert free0 - free1 < 4 * mib, (free0, free1)
    # Contrast: the allocating entry point maps its ~20 MB split workspace from its pool on the
    # same shape, so the measurement above can see an allocation of that size.
    assert free1 - free2 >= 16 * mib, (free1, free2)
