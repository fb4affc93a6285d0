"""CPU check of the backward kernel's unit assignment and launch plan, restated from
csrc/mfa_bwd_kernel.cuh (BwdCursor::unit_at, bounds) and csrc/mfa_capi.cu (plan_backward):
every unit of both passes runs exactly once, on one CTA, the dealing by length evens out the
CTAs' step counts with the causal mask, and the mixed plan (every CTA on both passes, the dQ
units dealt from the other end of the grid) gives no CTA an extra unit of both passes while
fewer than half of the CTAs get an extra one."""
from __future__ import annotations

import math

import pytest

KV_COST = 1.05
RESTART = 0.05
PASSES, SPLIT, MIXED = "passes", "split", "mixed"


def unit_at(k, c, ctas, bh, blocks, dkv, causal, by_length, reverse=False):
    units = bh * blocks
    if reverse:
        c = ctas - 1 - c
    if not causal or not by_length:
        u = k * ctas + c
        return u if u < units else -1
    i = k * ctas + (ctas - 1 - c if k & 1 else c)
    if i >= units:
        return -1
    wave, head = divmod(i, bh)
    blk = wave if dkv else blocks - 1 - wave
    return head * blocks + blk


def steps(u, blocks, dkv, causal):
    blk = u % blocks
    if dkv:
        return blocks - blk if causal else blocks
    return blk + 1 if causal else blocks


def plan(units, sms, causal):
    """(mode, CTAs of the dQ pass, CTAs of the dK/dV pass) as plan_backward chooses them."""
    waves = units / sms
    if sms < 2 or math.ceil(waves) / waves <= 1.05:
        return PASSES, min(sms, units), min(sms, units)
    best, ideal, cq = 1e300, sms / (1 + KV_COST), sms
    for c in range(1, sms):
        ck = sms - c
        tq = units / c if causal else -(-units // c)
        tk = KV_COST * (units / ck if causal else -(-units // ck))
        cost = max(tq, tk)
        nearer = abs(c - ideal) < abs(cq - ideal)
        if cost < best * (1 - 1e-9) or (cost <= best * (1 + 1e-9) and nearer):
            best, cq = cost, c
    ckv = sms - cq
    ctas = min(sms, units)
    base, rem = divmod(units, ctas)
    if causal:
        mixed = units * (1 + KV_COST) / ctas
    elif rem == 0:
        mixed = base * (1 + KV_COST)
    elif 2 * rem <= ctas:
        mixed = (base + 1) * KV_COST + base
    else:
        mixed = (base + 1) * (1 + KV_COST)
    mixed += RESTART
    if units >= sms or mixed < best:
        return MIXED, ctas, ctas
    return SPLIT, min(cq, units), min(ckv, units)


def walk(bh, blocks, ctas, dkv, causal, by_length, reverse=False):
    """Units of every CTA of one pass, in the cursor's order."""
    out = []
    for c in range(ctas):
        mine, k = [], 0
        while (u := unit_at(k, c, ctas, bh, blocks, dkv, causal, by_length, reverse)) >= 0:
            mine.append(u)
            k += 1
        out.append(mine)
    return out


def passes_of(bh, blocks, sms, causal):
    """[(dkv, ctas, by_length, reverse)] of both passes under the chosen plan."""
    mode, cq, ckv = plan(bh * blocks, sms, causal)
    by_length = mode != PASSES and causal
    return mode, [(False, cq, by_length, mode == MIXED), (True, ckv, by_length, False)]


CASES = [(8, 64, 148), (256, 32, 148), (2048, 4, 148), (32, 128, 148), (1, 1, 148), (3, 7, 13),
         (5, 9, 148), (1, 64, 148), (16, 3, 37), (4, 64, 148), (64, 8, 148), (2, 128, 148),
         (3, 50, 148)]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("bh,blocks,sms", CASES)
def test_every_unit_once_per_pass(bh, blocks, sms, causal):
    mode, passes = passes_of(bh, blocks, sms, causal)
    ctas = {c for _, c, _, _ in passes}
    assert min(ctas) >= 1
    if mode == SPLIT:
        assert sum(c for _, c, _, _ in passes) <= sms
    else:
        assert max(ctas) <= sms
    for dkv, c, by_length, reverse in passes:
        got = sorted(u for mine in walk(bh, blocks, c, dkv, causal, by_length, reverse)
                     for u in mine)
        assert got == list(range(bh * blocks))


def test_headline_shapes_take_the_expected_mode():
    # B1 H8 N8192: 512 units per pass on 148 SMs (3.46 waves) -> both passes on every CTA
    assert plan(8 * 64, 148, False) == (MIXED, 148, 148)
    assert plan(8 * 64, 148, True) == (MIXED, 148, 148)
    # B16 H16 N4096: 8192 units (55.4 waves) -> one pass per launch over all SMs
    assert plan(256 * 32, 148, False) == (PASSES, 148, 148)
    # B1 H1 N8192: 64 units, fewer than the SMs -> each pass on SMs of its own
    assert plan(64, 148, False)[0] == SPLIT


def test_mixed_plan_spreads_the_extra_units():
    # 512 units on 148 CTAs: 68 CTAs take a fourth dK/dV unit, 68 others a fourth dQ unit
    bh, blocks, sms = 8, 64, 148
    dq = walk(bh, blocks, sms, False, False, False, reverse=True)
    dkv = walk(bh, blocks, sms, True, False, False)
    counts = [(len(a), len(b)) for a, b in zip(dkv, dq)]
    assert max(k for k, _ in counts) == 4 and max(q for _, q in counts) == 4
    assert all(k + q <= 7 for k, q in counts)
    cost = max(KV_COST * k + q for k, q in counts)
    assert cost == pytest.approx(4 * KV_COST + 3)
    assert cost < 7 * KV_COST  # the split plan's slowest CTA: 7 dK/dV units


def test_dealing_by_length_balances_causal_steps():
    bh, blocks, sms = 8, 64, 148
    mode, passes = passes_of(bh, blocks, sms, True)
    assert mode == MIXED
    loads = [0] * sms
    for dkv, ctas, by_length, reverse in passes:
        assert by_length
        per = [sum(steps(u, blocks, dkv, True) for u in mine)
               for mine in walk(bh, blocks, ctas, dkv, True, True, reverse)]
        strided = [sum(steps(u, blocks, dkv, True) for u in mine)
                   for mine in walk(bh, blocks, ctas, dkv, True, False, reverse)]
        mean = sum(per) / len(per)
        assert max(per) <= 1.1 * mean
        assert max(per) < max(strided)
        for c, x in enumerate(per):
            loads[c] += x
    assert max(loads) <= 1.1 * sum(loads) / len(loads)
