"""CPU tests of the PyTorch binding (the flash_attn.cpp counterpart): it imports without a
GPU and validates its inputs with the reference's messages (flash_attn.cpp:50-52)."""
from __future__ import annotations

import pytest
import torch

import mini_flash_attention as mfa


@pytest.mark.parametrize("fn", [mfa.forward, mfa.forward_wmma, mfa.forward_bnhd])
def test_cpu_tensors_rejected(fn):
    q = torch.randn(1, 2, 128, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="q must be a CUDA tensor"):
        fn(q, q, q)


def test_public_signature_matches_reference():
    import inspect

    for fn in (mfa.forward, mfa.forward_wmma, mfa.forward_bnhd):
        params = inspect.signature(fn).parameters
        assert list(params) == ["q", "k", "v", "causal"]
        assert params["causal"].default is False


def test_extension_is_the_in_tree_build():
    ext = mfa._cuda._load_extension()
    assert "sm_100a" in ext.version()
    assert "mini-flash-attention_b200" in ext.__file__
