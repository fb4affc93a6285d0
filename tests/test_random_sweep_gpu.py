"""Seeded random sweep over the forward's and backward's whole input space on a B200: batch,
heads, any N from 1 to 8192 (log-uniform, so short and ragged lengths are common), D = 32 /
64 / 128, fp16 / bf16, causal or not, [B, H, N, D] or [B, N, H, D]. Each case is checked
against fp32 attention (the reference test's naive oracle, tests/test_forward.py:28-34 of the
reference, with the causal mask and the log-sum-exp added), so that no combination of the
plan's modes (whole / split key ranges, merge, tails, masks) escapes the fixed-shape tests.
Each forward case also runs a random query row range through forward_rows and, where its
contract allows (fp16, D = 64, N % 64 == 0), the single-tile kernel behind forward_wmma."""
from __future__ import annotations

import math
import random

import pytest
import torch

import mini_flash_attention as mfa

pytestmark = pytest.mark.gpu

FWD_CASES = 48
BWD_CASES = 16


def naive_fp32(q, k, v, causal):
    """softmax(q k^T / sqrt(D)) v and the natural-log row log-sum-exp, in fp32."""
    d = q.shape[-1]
    s = q.float() @ k.float().transpose(-2, -1) * d ** -0.5
    if causal:
        n = q.shape[-2]
        s = s.masked_fill(torch.ones((n, n), dtype=torch.bool, device=q.device).triu(1),
                          float("-inf"))
    return torch.softmax(s, dim=-1) @ v.float(), torch.logsumexp(s, dim=-1)


def randn(shape, seed, dtype):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, device="cuda", generator=g, dtype=torch.float32).to(dtype)


def fwd_case(i):
    r = random.Random(1000 + i)
    c = dict(i=i, B=r.randint(1, 3), H=r.randint(1, 5),
             N=int(math.exp(r.uniform(0, math.log(8192)))), D=r.choice([32, 64, 128]),
             dtype=r.choice([torch.float16, torch.bfloat16]), causal=r.random() < 0.5,
             bnhd=r.random() < 0.3, seed=7000 + 10 * i)
    # a query row range of every head for forward_rows (whole 256-row units with the mask)
    n = c["N"]
    if c["causal"]:
        a = 256 * r.randint(0, (n - 1) // 256)
    else:
        a = r.randint(0, n - 1)
    c["rows"] = (a, r.randint(a + 1, n))
    return c


def case_id(c):
    return (f"{c['i']}-B{c['B']}H{c['H']}N{c['N']}D{c['D']}-"
            f"{'fp16' if c['dtype'] == torch.float16 else 'bf16'}"
            f"{'-causal' if c['causal'] else ''}{'-bnhd' if c.get('bnhd') else ''}")


FWD = [fwd_case(i) for i in range(FWD_CASES)]


@pytest.mark.parametrize("c", FWD, ids=[case_id(c) for c in FWD])
def test_forward_random(c):
    B, H, N, D, dtype, causal = c["B"], c["H"], c["N"], c["D"], c["dtype"], c["causal"]
    tol = 2e-3 if dtype == torch.float16 else 1.5e-2
    q, k, v = (randn((B, H, N, D), c["seed"] + j, dtype) for j in range(3))
    ref, ref_lse = naive_fp32(q, k, v, causal)
    if c["bnhd"]:
        out = mfa.forward_bnhd(*(x.transpose(1, 2).contiguous() for x in (q, k, v)),
                               causal=causal).transpose(1, 2)
        lse = None
    else:
        out, lse = mfa.forward_lse(q, k, v, causal=causal)
        plain = mfa.forward(q, k, v, causal=causal)
        # the log-sum-exp variant computes the same output
        torch.testing.assert_close(plain, out, rtol=0, atol=0)
    assert out.shape == q.shape and out.dtype == dtype
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.float(), ref, rtol=tol, atol=tol)
    if lse is not None:
        torch.testing.assert_close(lse, ref_lse, rtol=1e-4, atol=1e-4)
    if not c["bnhd"]:
        # the row range alone: its rows as in the whole forward, nothing else written
        a, b = c["rows"]
        ro = torch.full_like(q, 3.0)
        mfa.forward_rows(q, k, v, a, b, out=ro, causal=causal)
        torch.testing.assert_close(ro[:, :, a:b].float(), ref[:, :, a:b], rtol=tol, atol=tol)
        assert (ro[:, :, :a] == 3.0).all() and (ro[:, :, b:] == 3.0).all()
    if D == 64 and dtype == torch.float16 and N % 64 == 0:
        # the single-tile kernel behind forward_wmma (the reference's N % 64 contract)
        torch.testing.assert_close(mfa.forward_wmma(q, k, v, causal=causal).float(), ref,
                                   rtol=tol, atol=tol)


def bwd_case(i):
    r = random.Random(5000 + i)
    return dict(i=i, B=r.randint(1, 2), H=r.randint(1, 4),
                N=int(math.exp(r.uniform(0, math.log(4096)))), D=64,
                dtype=r.choice([torch.float16, torch.bfloat16]), causal=r.random() < 0.5)


BWD = [bwd_case(i) for i in range(BWD_CASES)]


@pytest.mark.parametrize("c", BWD, ids=[case_id(c) for c in BWD])
def test_backward_random(c):
    B, H, N, dtype, causal = c["B"], c["H"], c["N"], c["dtype"], c["causal"]
    q, k, v, dout = (randn((B, H, N, 64), 9000 + 7 * c["N"] + j, dtype) for j in range(4))
    out, lse = mfa.forward_lse(q, k, v, causal=causal)
    dq, dk, dv = mfa.backward(q, k, v, out, lse, dout, causal=causal)
    qf, kf, vf = (x.float().requires_grad_() for x in (q, k, v))
    ref, _ = naive_fp32(qf, kf, vf, causal)
    ref.backward(dout.float())
    for ours, want, name in ((dq, qf.grad, "dq"), (dk, kf.grad, "dk"), (dv, vf.grad, "dv")):
        assert ours.shape == want.shape and ours.dtype == dtype
        assert torch.isfinite(ours).all(), name
        # floor: at N = 1 the exact dq and dk are 0 (softmax of one key is constant)
        scale = max(want.abs().max().item(), 1e-2)
        err = (ours.float() - want).abs()
        rel = 2e-2 if dtype == torch.float16 else 3e-2
        assert err.max().item() <= rel * scale, f"{name}: max err {err.max().item()} vs {scale}"
        assert err.mean().item() <= 2e-3 * scale, f"{name}: mean err {err.mean().item()}"
