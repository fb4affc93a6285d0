"""GPU tests of the backward pass (the reference's README lists it as future work,
README.md:125): forward_lse's log-sum-exp and backward's dq, dk, dv against torch autograd
through the fp32 naive attention of the reference test (tests/test_forward.py:28-34), and the
autograd wrapper `attention` end to end.

Tolerances: gradients are compared relative to the largest reference gradient entry
(max |ours - ref| <= 2e-2 * max |ref|, mean |ours - ref| <= 2e-3 * max |ref|); P and dS are
rounded to fp16 / bf16 for the tensor-core products, as in every FlashAttention backward.
"""
from __future__ import annotations

import math

import pytest
import torch

import mini_flash_attention as mfa
from mini_flash_attention import capi

pytestmark = pytest.mark.gpu


def naive(q, k, v, causal):
    d = q.shape[-1]
    s = q @ k.transpose(-2, -1) * d ** -0.5
    if causal:
        n = q.shape[-2]
        mask = torch.ones((n, n), dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    return torch.softmax(s, dim=-1) @ v, torch.logsumexp(s, dim=-1)


def randn(shape, seed, dtype=torch.float16, scale=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return (torch.randn(shape, device="cuda", generator=g, dtype=torch.float32) * scale).to(dtype)


def reference_grads(q, k, v, dout, causal):
    qf, kf, vf = (x.float().requires_grad_() for x in (q, k, v))
    out, lse = naive(qf, kf, vf, causal)
    out.backward(dout.float())
    return out.detach(), lse.detach(), qf.grad, kf.grad, vf.grad


def check_grad(ours, ref, name):
    scale = ref.abs().max().item()
    err = (ours.float() - ref).abs()
    assert err.max().item() <= 2e-2 * scale, f"{name}: max err {err.max().item()} vs {scale}"
    assert err.mean().item() <= 2e-3 * scale, f"{name}: mean err {err.mean().item()} vs {scale}"


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("B,H,N", [(1, 2, 128), (2, 1, 256), (1, 2, 2048), (2, 4, 1000),
                                   (1, 8, 4096), (3, 3, 77), (1, 3, 8000)])
def test_backward_matches_autograd(B, H, N, dtype, causal):
    q, k, v, dout = (randn((B, H, N, 64), 300 + i, dtype) for i in range(4))
    out, lse = mfa.forward_lse(q, k, v, causal)
    ref_out, ref_lse, dq_ref, dk_ref, dv_ref = reference_grads(q, k, v, dout, causal)
    assert lse.shape == (B, H, N) and lse.dtype == torch.float32
    torch.testing.assert_close(lse, ref_lse, rtol=1e-4, atol=1e-4)
    dq, dk, dv = mfa.backward(q, k, v, out, lse, dout, causal)
    assert dq.dtype == dtype and dq.shape == q.shape
    for ours, ref, name in ((dq, dq_ref, "dq"), (dk, dk_ref, "dk"), (dv, dv_ref, "dv")):
        assert torch.isfinite(ours).all(), name
        check_grad(ours, ref, name)


def test_lse_from_split_and_whole_plans():
    # B1 H8 N8192 takes the split plan (merge kernel writes the LSE); B16 H16 N512 whole blocks
    for shape in ((1, 8, 8192), (16, 16, 512)):
        q, k, v = (randn((*shape, 64), 320 + i) for i in range(3))
        out, lse = mfa.forward_lse(q, k, v)
        s = q.float() @ k.float().transpose(-2, -1) / 8.0
        torch.testing.assert_close(lse, torch.logsumexp(s, dim=-1), rtol=1e-4, atol=1e-4)
        assert torch.equal(out, mfa.forward(q, k, v))


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
def test_attention_autograd(causal):
    q, k, v = (randn((2, 4, 1024, 64), 330 + i).requires_grad_() for i in range(3))
    w = randn((2, 4, 1024, 64), 334)
    (mfa.attention(q, k, v, causal) * w).sum().backward()
    _, _, dq_ref, dk_ref, dv_ref = reference_grads(q.detach(), k.detach(), v.detach(), w, causal)
    check_grad(q.grad, dq_ref, "dq")
    check_grad(k.grad, dk_ref, "dk")
    check_grad(v.grad, dv_ref, "dv")


def test_capi_backward_bnhd():
    B, N, H = 2, 640, 3
    q, k, v, dout = (randn((B, N, H, 64), 340 + i) for i in range(4))
    out = torch.empty_like(q)
    lse = torch.empty((B, H, N), device="cuda", dtype=torch.float32)
    s = torch.cuda.current_stream().cuda_stream
    lib = capi.load()
    rc = lib.mfa_fwd_lse(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), lse.data_ptr(),
                         B, H, N, 64, 0.125, 1, capi.DTYPE_FP16, capi.LAYOUT_BNHD, s)
    assert rc == 0, capi.last_error()
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    capi.bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(),
             lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, H, N, 64, 0.125,
             causal=True, layout=capi.LAYOUT_BNHD, stream=s)
    torch.cuda.synchronize()
    t = [x.transpose(1, 2).contiguous() for x in (q, k, v, dout)]
    _, _, dq_ref, dk_ref, dv_ref = reference_grads(*t, True)
    check_grad(dq.transpose(1, 2), dq_ref, "dq")
    check_grad(dk.transpose(1, 2), dk_ref, "dk")
    check_grad(dv.transpose(1, 2), dv_ref, "dv")
    assert capi.device_status(torch.cuda.current_device()) == 0


def test_backward_rejects_other_head_dims():
    q = randn((1, 1, 128, 32), 350)
    out, lse = mfa.forward_lse(q, q, q)
    with pytest.raises(RuntimeError, match="The backward pass supports only D=64"):
        mfa.backward(q, q, q, out, lse, q)
