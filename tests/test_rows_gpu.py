"""GPU tests of the query-row range forward (`forward_rows`, C ABI `mfa_fwd_rows`): the per-GPU
call of the multi-GPU sharding used when B*H is smaller than the number of GPUs (every GPU holds
the whole k and v and computes a range of query rows). Rows in the range match the whole
forward and fp32 attention, with and without the causal mask; rows outside it are not touched;
the ranges of `q_shard` reassemble the whole output."""
from __future__ import annotations

import pytest
import torch

import mini_flash_attention as mfa
from mini_flash_attention import capi
from mini_flash_attention.sharding import q_shard

pytestmark = pytest.mark.gpu


def randn(shape, seed, dtype=torch.float16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(shape, device="cuda", generator=g, dtype=torch.float32).to(dtype)


def naive_fp32(q, k, v, causal=False):
    s = q.float() @ k.float().transpose(-2, -1) * q.shape[-1] ** -0.5
    if causal:
        n = q.shape[-2]
        s = s.masked_fill(torch.ones((n, n), dtype=torch.bool, device=q.device).triu(1),
                          float("-inf"))
    return torch.softmax(s, dim=-1) @ v.float()


@pytest.mark.parametrize("shape,begin,end", [
    ((2, 3, 1024, 64), 0, 1024), ((2, 3, 1024, 64), 256, 768), ((1, 2, 1000, 64), 100, 999),
    ((1, 1, 4096, 64), 4000, 4096), ((3, 777, 64), 1, 2), ((1, 1, 8192, 64), 512, 8192),
    ((2, 2, 640, 32), 128, 640), ((2, 2, 640, 128), 0, 300)])
def test_rows_match_forward_and_leave_the_rest(shape, begin, end):
    q, k, v = (randn(shape, 40 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    mfa.forward_rows(q, k, v, begin, end, out=out)
    got = out[..., begin:end, :]
    assert torch.isfinite(got).all()
    assert torch.isnan(out[..., :begin, :]).all() and torch.isnan(out[..., end:, :]).all()
    ref = naive_fp32(q, k, v)[..., begin:end, :]
    torch.testing.assert_close(got.float(), ref, rtol=2e-3, atol=2e-3)
    whole = mfa.forward(q, k, v)[..., begin:end, :]
    torch.testing.assert_close(got, whole, rtol=0, atol=2e-3)


def test_empty_range_writes_nothing():
    q, k, v = (randn((1, 2, 512, 64), 50 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    mfa.forward_rows(q, k, v, 300, 300, out=out)
    assert torch.isnan(out).all()


@pytest.mark.parametrize("world", [2, 3, 8])
def test_query_shards_reassemble_the_output(world):
    n = 5000
    q, k, v = (randn((1, 1, n, 64), 60 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    for r in range(world):
        s = q_shard(n, r, world)
        mfa.forward_rows(q, k, v, s.begin, s.end, out=out)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v), rtol=2e-3, atol=2e-3)


def test_bf16_rows():
    q, k, v = (randn((1, 2, 2048, 64), 70 + i, torch.bfloat16) for i in range(3))
    out = mfa.forward_rows(q, k, v, 1024, 2048)
    torch.testing.assert_close(out[..., 1024:, :].float(), naive_fp32(q, k, v)[..., 1024:, :],
                               rtol=1.5e-2, atol=1.5e-2)


def test_capi_rows_bnhd():
    B, N, H, D = 2, 1500, 3, 64
    q, k, v = (randn((B, N, H, D), 80 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    capi.fwd_rows(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, N, 256, 1300,
                  D, D ** -0.5, layout=capi.LAYOUT_BNHD,
                  stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = naive_fp32(*(x.transpose(1, 2) for x in (q, k, v))).transpose(1, 2)
    torch.testing.assert_close(out[:, 256:1300].float(), ref[:, 256:1300], rtol=2e-3, atol=2e-3)
    assert torch.isnan(out[:, :256]).all() and torch.isnan(out[:, 1300:]).all()


@pytest.mark.parametrize("begin,end", [(0, 600), (-1, 10), (20, 10), (0, 513)])
def test_bad_ranges_raise(begin, end):
    q, k, v = (randn((1, 1, 512, 64), 90 + i) for i in range(3))
    out = torch.empty_like(q)
    with pytest.raises(RuntimeError, match="q_begin"):
        mfa.forward_rows(q, k, v, begin, end, out=out)


def test_causal_range_off_a_unit_boundary_rejected():
    q, k, v = (randn((1, 1, 512, 64), 95 + i) for i in range(3))
    out = torch.empty_like(q)
    with pytest.raises(capi.MfaError, match="multiple of 256"):
        capi.fwd_rows(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), 1, 1, 512, 100,
                      512, 64, 0.125, causal=True)


@pytest.mark.parametrize("shape,begin,end", [
    ((1, 2, 8192, 64), 0, 4096), ((1, 2, 8192, 64), 4096, 8192), ((2, 1, 1000, 64), 256, 1000),
    ((1, 3, 640, 64), 512, 640), ((2, 2, 3000, 64), 768, 1792), ((1, 2, 640, 128), 128, 640),
    ((1, 2, 640, 32), 256, 600), ((3, 2048, 64), 1024, 2048)])
def test_causal_rows_match_forward(shape, begin, end):
    q, k, v = (randn(shape, 100 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    mfa.forward_rows(q, k, v, begin, end, out=out, causal=True)
    got = out[..., begin:end, :]
    assert torch.isfinite(got).all()
    assert torch.isnan(out[..., :begin, :]).all() and torch.isnan(out[..., end:, :]).all()
    ref = naive_fp32(q, k, v, causal=True)[..., begin:end, :]
    torch.testing.assert_close(got.float(), ref, rtol=2e-3, atol=2e-3)
    whole = mfa.forward(q, k, v, causal=True)[..., begin:end, :]
    torch.testing.assert_close(got, whole, rtol=0, atol=2e-3)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_causal_query_shards_reassemble_the_output(world):
    n = 5000
    q, k, v = (randn((1, 2, n, 64), 110 + i) for i in range(3))
    out = torch.full_like(q, float("nan"))
    for r in range(world):
        s = q_shard(n, r, world, causal=True)
        mfa.forward_rows(q, k, v, s.begin, s.end, out=out, causal=True)
    assert torch.isfinite(out).all()
    torch.testing.assert_close(out.float(), naive_fp32(q, k, v, causal=True), rtol=2e-3,
                               atol=2e-3)
