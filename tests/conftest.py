"""Shared test set-up: import paths, the `gpu` marker, seeded input helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "mini-flash-attention_b200", ROOT / "tests" / "golden"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and the built extension")


def pytest_sessionstart(session):
    # A broken pipeline must fail fast in tests: bound every in-kernel wait at 500 ms.
    try:
        import torch

        if torch.cuda.is_available():
            from mini_flash_attention import capi

            capi.set_watchdog_ns(500_000_000)
    except Exception:  # noqa: BLE001
        pass


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
