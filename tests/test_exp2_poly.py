"""CPU check of the FMA-pipe exp2 used by the softmax warps: the coefficients compiled into
csrc/mfa_exp2.cuh are the ones the Remez derivation (csrc/gen_exp2_poly.py) produces, and a
float32 emulation of the device sequence (range reduction + Horner + exponent add) stays
within 1e-4 relative error of 2^x over the range the kernel feeds it."""
from __future__ import annotations

import importlib.util
import re
from pathlib import Path

import numpy as np

CSRC = Path(__file__).resolve().parents[1] / "mini-flash-attention_b200" / "csrc"


def _gen():
    spec = importlib.util.spec_from_file_location("gen_exp2_poly", CSRC / "gen_exp2_poly.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _header_coeffs() -> np.ndarray:
    text = (CSRC / "mfa_exp2.cuh").read_text()
    vals = [float(re.search(rf"kC{i} = ([-0-9.e]+)f", text).group(1)) for i in range(4)]
    return np.array(vals, dtype=np.float32)


def test_header_coefficients_match_derivation():
    np.testing.assert_array_equal(_header_coeffs(), _gen().float32_coeffs())


def test_polynomial_error_bound():
    assert _gen().max_rel_error(_header_coeffs()) < 1e-4


def emulate_device_exp2(x: np.ndarray) -> np.ndarray:
    """float32 restatement of exp2_poly_pair (fma rounding emulated in float64 then rounded)."""
    c = _header_coeffs().astype(np.float64)
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    j = (t - np.float32(12582912.0)).astype(np.float32)
    f = (x.astype(np.float64) - j).astype(np.float32).astype(np.float64)
    p = np.float32(c[3] * f + c[2]).astype(np.float64)
    p = np.float32(p * f + c[1]).astype(np.float64)
    p = np.float32(p * f + c[0])
    bits = p.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def test_emulated_device_sequence():
    x = np.concatenate([np.linspace(-120, 8, 200001, dtype=np.float32),
                        np.array([0.0, -0.5, 0.5, 7.99, -1e-7], dtype=np.float32)])
    got = emulate_device_exp2(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got / want - 1.0)) < 1e-4
    # clamped tail: tiny and non-negative, never garbage
    tail = emulate_device_exp2(np.array([-126.0, -300.0, -np.inf], dtype=np.float32))
    assert np.all(tail >= 0) and np.all(tail < 1e-37)
