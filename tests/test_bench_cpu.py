"""CPU tests of bench.py, the measurement the round-end runs depend on: the reference arm's JSON
line (the reference's naive torch attention, benchs/benchmark_forward.py:98-115, timed on the
host cores), the flop and byte counts behind every TFLOPS and GB/s figure, the DRAM traffic read
from the committed ncu summaries, and the strong-scaling legs."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_reference_arm_prints_one_contract_line():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3",
                          "--warmup", "3"], cwd=ROOT, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["metric"] == bench.METRIC and line["unit"] == "TFLOPS"
    assert line["impl"] == "reference" and line["higher_is_better"] is True
    assert line["steps"] == 3 and line["warmup"] == 3
    assert line["config"]["workload"] == "b1h8n8192"
    assert line["value"] > 0 and line["ms_per_step"] > 0
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    assert cpu["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_warmup_below_three_is_refused():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "2"], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert res.returncode != 0 and "--warmup must be >= 3" in res.stderr


def test_flop_and_byte_counts():
    # 4 * BH * N^2 * D: 137.4 GFLOP at B1 H8 N8192, the reference's formula
    assert bench.attention_flops(8, 8192) == 4.0 * 8 * 8192 ** 2 * 64
    assert bench.attention_flops(8, 8192) == pytest.approx(137.44e9, rel=1e-4)
    # causal: the N(N+1)/2 attended pairs
    assert bench.attention_flops(1, 4, causal=True) == 4.0 * 10 * 64
    assert bench.attention_flops(2, 128, d=128) == 4.0 * 2 * 128 ** 2 * 128
    # q, k, v read once and out written once, fp16: 536.9 MB for B128 H16 N512
    assert bench.attention_bytes(2048, 512) == 4 * 2048 * 512 * 64 * 2
    assert bench.attention_bytes(2048, 512) == pytest.approx(536.9e6, rel=1e-3)


@pytest.mark.parametrize(("workload", "bytes_"), [("b1h8n8192", 25445120),
                                                  ("b16h16n4096", 518028032),
                                                  ("b128h16n512", 515125504)])
def test_traffic_comes_from_the_committed_profiles(workload, bytes_):
    assert bench.load_traffic("mfa_fwd", workload) == bytes_
    # a few percent below the algorithmic bytes: nothing is re-read from HBM
    wl = bench.WORKLOADS[workload]
    assert bytes_ <= bench.attention_bytes(wl["B"] * wl["H"], wl["N"])


def test_traffic_is_none_without_a_profile():
    assert bench.load_traffic("mfa_fwd", "b1h1n65536") is None


def test_strong_legs_cover_the_north_star_splits():
    names = [name for name, _, _ in bench.STRONG]
    assert sorted(names) == ["b128h16n512", "b16h16n4096", "b1h32n32768"]
    for name, warmup, steps in bench.STRONG:
        assert name in bench.WORKLOADS and bench.WORKLOADS[name]["scaling"] == "strong"
        assert warmup >= 3 and steps >= 1
