"""CPU tests of the C ABI: libmfa_b200.so loads, exports every symbol include/mfa_b200.h
declares, and rejects bad arguments with the reference launchers' messages before touching
the GPU (flash_attn_cuda.cu:399-410, flash_attn_wmma_cuda.cu:269-277)."""
from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest
import torch

from mini_flash_attention import capi

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "mfa_b200.h"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"MFA_API\s+[\w\s\*]+?\b(mfa_\w+)\s*\(", text)


def test_header_and_python_view_agree():
    assert sorted(declared_symbols()) == sorted(capi.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for sym in declared_symbols():
        assert sym in exported, sym
    lib = capi.load()
    for sym in declared_symbols():
        assert hasattr(lib, sym)


def test_build_targets_only_sm100a():
    from mini_flash_attention import _build

    assert _build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version():
    assert "sm_100a" in capi.version()


FAKE = 0x10000  # never dereferenced: every case below fails before a launch

# The cases that pass argument validation are only run without a GPU, where the call stops at
# the device. (With a GPU the launcher would refuse FAKE as a non-device pointer; they are
# skipped there all the same, so that no test of this file can ever reach a launch.)
needs_no_gpu = pytest.mark.skipif(torch.cuda.is_available(),
                                  reason="valid-argument calls on fake pointers: CPU only")


@pytest.mark.parametrize("simple", [False, True])
def test_head_dim_rejected(simple):
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, 2, 128, 32, 0.17, simple=simple)
    assert e.value.code == capi.MFA_ERR_HEAD_DIM
    want = ("This WMMA prototype supports only D=64 yet" if simple
            else "This kernel supports only D=64")
    assert str(e.value) == want


@needs_no_gpu
def test_any_seq_len_passes_validation_full_kernel():
    # The reference requires N % 128 == 0 (flash_attn_cuda.cu:402-407); this kernel takes any
    # N: the call gets past every argument check and, with no GPU here, fails at the device.
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, 2, 192, 64, 0.125)
    assert e.value.code in (capi.MFA_ERR_CUDA, capi.MFA_ERR_DEVICE)


def test_seq_len_rejected_simple_kernel():
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, 2, 96, 64, 0.125, simple=True)
    assert e.value.code == capi.MFA_ERR_SEQ_LEN
    assert str(e.value) == "Only N (seq len) divisible by 64 and 64 are supported yet"


@needs_no_gpu
@pytest.mark.parametrize("simple", [False, True])
def test_causal_passes_validation(simple):
    # Causal masking is supported (the reference launchers reject it, flash_attn_cuda.cu:
    # 408-410): the call gets past every argument check and, with no GPU here, fails only when
    # it reaches the device.
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, 2, 128, 64, 0.125, causal=True, simple=simple)
    assert e.value.code in (capi.MFA_ERR_CUDA, capi.MFA_ERR_DEVICE)


def test_check_order_matches_reference():
    # D is checked before N (flash_attn_cuda.cu:399-407; the WMMA launcher keeps its N check)
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, 1, 100, 32, 0.1, causal=True, simple=True)
    assert e.value.code == capi.MFA_ERR_HEAD_DIM
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, 1, 100, 64, 0.1, causal=True, simple=True)
    assert e.value.code == capi.MFA_ERR_SEQ_LEN
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, 1, 100, 32, 0.1, causal=True)
    assert e.value.code == capi.MFA_ERR_HEAD_DIM


def test_null_and_misaligned_pointers_rejected():
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(0, FAKE, FAKE, FAKE, 1, 128, 64, 0.125)
    assert e.value.code == capi.MFA_ERR_INVALID_ARGUMENT
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE + 2, FAKE, FAKE, FAKE, 1, 128, 64, 0.125)
    assert e.value.code == capi.MFA_ERR_INVALID_ARGUMENT


def test_negative_extent_rejected():
    with pytest.raises(capi.MfaError) as e:
        capi.fwd(FAKE, FAKE, FAKE, FAKE, -1, 128, 64, 0.125)
    assert e.value.code == capi.MFA_ERR_INVALID_ARGUMENT


def test_empty_problem_is_a_noop():
    capi.fwd(0, 0, 0, 0, 0, 128, 64, 0.125)
    capi.fwd(0, 0, 0, 0, 4, 0, 64, 0.125, simple=True)


@pytest.mark.parametrize("scale", [0.0, -0.125, float("nan"), float("inf")])
def test_scale_must_be_positive_and_finite(scale):
    # the kernels' row-max logic relies on scale > 0; rejected before any device access
    for call in (lambda: capi.fwd(FAKE, FAKE, FAKE, FAKE, 2, 256, 64, scale),
                 lambda: capi.fwd_general(FAKE, FAKE, FAKE, FAKE, 1, 2, 256, 64, scale)):
        with pytest.raises(capi.MfaError) as e:
            call()
        assert e.value.code == capi.MFA_ERR_INVALID_ARGUMENT
        assert str(e.value) == "scale must be positive and finite"


def test_watchdog_limit_validated():
    with pytest.raises(capi.MfaError) as e:
        capi.set_watchdog_ns(10)
    assert e.value.code == capi.MFA_ERR_INVALID_ARGUMENT
    capi.set_watchdog_ns(2_000_000_000)


@needs_no_gpu
def test_general_entry_validates_dtype_layout_and_shape():
    def call(**kw):
        args = dict(batch=2, heads=3, n=256, d=64, scale=0.125, dtype=capi.DTYPE_BF16,
                    layout=capi.LAYOUT_BNHD)
        args.update(kw)
        with pytest.raises(capi.MfaError) as e:
            capi.fwd_general(FAKE, FAKE, FAKE, FAKE, **args)
        return e.value
    assert call(dtype=7).code == capi.MFA_ERR_INVALID_ARGUMENT
    assert call(layout=5).code == capi.MFA_ERR_INVALID_ARGUMENT
    e = call(d=96)
    assert (e.code, str(e)) == (capi.MFA_ERR_HEAD_DIM,
                                "This kernel supports only D=32, D=64 and D=128")
    assert call(n=200).code in (capi.MFA_ERR_CUDA, capi.MFA_ERR_DEVICE)
    assert call(batch=-1).code == capi.MFA_ERR_INVALID_ARGUMENT
    # valid arguments reach the device (no GPU here)
    assert call().code in (capi.MFA_ERR_CUDA, capi.MFA_ERR_DEVICE)
    # empty problems are no-ops
    capi.fwd_general(FAKE, FAKE, FAKE, FAKE, 0, 3, 256, 64, 0.125)


def test_workspace_query_rejects_bad_arguments():
    with pytest.raises(capi.MfaError) as e:
        capi.fwd_workspace_bytes(1, 8, 1024, d=48)
    assert e.value.code == capi.MFA_ERR_HEAD_DIM
    with pytest.raises(capi.MfaError) as e:
        capi.fwd_workspace_bytes(-1, 8, 1024)
    assert e.value.code == capi.MFA_ERR_INVALID_ARGUMENT
    assert capi.fwd_workspace_bytes(0, 8, 1024) == 0  # empty: no device needed
