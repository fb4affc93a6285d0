"""CPU check of the backward kernel's unit assignment and launch split, restated from
csrc/mfa_bwd_kernel.cuh (BwdCursor::unit_at, bounds) and csrc/mfa_capi.cu (launch_backward):
every unit of both passes runs exactly once, on one CTA of its own pass, and the dealing by
length evens out the CTAs' step counts with the causal mask."""
from __future__ import annotations

import math

import pytest

KV_COST = 1.05


def unit_at(k, c, ctas, bh, blocks, dkv, causal, by_length):
    units = bh * blocks
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


def plan(bh, blocks, sms, causal):
    """(together, cq, ckv, by_length) as launch_backward chooses them."""
    units = bh * blocks
    waves = units / sms
    together = sms >= 2 and math.ceil(waves) / waves > 1.05
    cq = ckv = sms
    if together:
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
    return together, min(cq, units), min(ckv, units), together and causal


def walk(bh, blocks, ctas, dkv, causal, by_length):
    """Units of every CTA of one pass, in the cursor's order."""
    out = []
    for c in range(ctas):
        mine, k = [], 0
        while (u := unit_at(k, c, ctas, bh, blocks, dkv, causal, by_length)) >= 0:
            mine.append(u)
            k += 1
        out.append(mine)
    return out


CASES = [(8, 64, 148), (256, 32, 148), (2048, 4, 148), (32, 128, 148), (1, 1, 148), (3, 7, 13),
         (5, 9, 148), (1, 64, 148), (16, 3, 37)]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("bh,blocks,sms", CASES)
def test_every_unit_once_per_pass(bh, blocks, sms, causal):
    together, cq, ckv, by_length = plan(bh, blocks, sms, causal)
    assert cq >= 1 and ckv >= 1
    if together:
        assert cq + ckv <= sms
    for dkv, ctas in ((False, cq), (True, ckv)):
        got = sorted(u for mine in walk(bh, blocks, ctas, dkv, causal, by_length) for u in mine)
        assert got == list(range(bh * blocks))


def test_headline_shapes_take_the_expected_mode():
    # B1 H8 N8192: 512 units per pass on 148 SMs (3.46 waves) -> both passes in one launch
    assert plan(8, 64, 148, False)[:3] == (True, 74, 74)
    # B16 H16 N4096: 8192 units (55.4 waves) -> one pass per launch over all SMs
    assert plan(256, 32, 148, False)[:3] == (False, 148, 148)


def test_dealing_by_length_balances_causal_steps():
    bh, blocks, sms = 8, 64, 148
    together, cq, ckv, by_length = plan(bh, blocks, sms, True)
    assert together and by_length
    for dkv, ctas in ((False, cq), (True, ckv)):
        loads = [sum(steps(u, blocks, dkv, True) for u in mine)
                 for mine in walk(bh, blocks, ctas, dkv, True, True)]
        strided = [sum(steps(u, blocks, dkv, True) for u in mine)
                   for mine in walk(bh, blocks, ctas, dkv, True, False)]
        mean = sum(loads) / len(loads)
        assert max(loads) <= 1.1 * mean
        assert max(loads) < max(strided)
