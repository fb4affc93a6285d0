"""CPU check of the persistent work schedule of mfa_fwd_kernel (restated here from
csrc/mfa_fwd_kernel.cuh: cta_range, StepCursor, mfa_merge_kernel's owner / piece rules, and
the launcher's split decision in csrc/mfa_capi.cu): every (query block, key block) unit is
processed exactly once, every partial piece lands in its own workspace slot, and every query
block cut into pieces is merged exactly once from exactly its pieces."""
from __future__ import annotations

import pytest


def cta_range(units, nkb, split, cta, ctas):
    if split:
        total = units * nkb
        return total * cta // ctas, total * (cta + 1) // ctas
    return units * cta // ctas * nkb, units * (cta + 1) // ctas * nkb


def segments(units, nkb, split, cta, ctas):
    if not split:  # whole query blocks, strided over the CTAs
        for i, u in enumerate(range(cta, units, ctas)):
            yield u, 0, nkb, i == 0
        return
    pos, end = cta_range(units, nkb, split, cta, ctas)
    first = True
    while pos < end:
        u = pos // nkb
        j0 = pos - u * nkb
        j1 = min(nkb, j0 + (end - pos))
        yield u, j0, j1, first
        first = False
        pos += j1 - j0


def cursor_segments(units, nkb, split, cta, ctas):
    """The kernel's StepCursor formulation (six 32-bit words) of the same walk."""
    if not split:
        if cta >= units:
            return
        u, rem, seg_idx = cta, (units - 1 - cta) // ctas, 0
        while True:
            yield u, 0, nkb, seg_idx == 0
            if rem <= 0:
                return
            u, rem, seg_idx = u + ctas, rem - 1, seg_idx + 1
    b, e = cta_range(units, nkb, split, cta, ctas)
    if b >= e:
        return
    u, j0 = divmod(b, nkb)
    j1 = min(nkb, j0 + (e - b))
    rem = (e - b) - (j1 - j0)
    seg_idx = 0
    while True:
        yield u, j0, j1, seg_idx == 0
        if rem <= 0:
            return
        u, j0, j1 = u + 1, 0, min(nkb, rem)
        rem -= j1
        seg_idx += 1


def merge_plan(units, nkb, c, ctas):
    """(u, [(cta, slot), ...]) for the query block merged by merge CTA c, or None."""
    b0, b1 = cta_range(units, nkb, 1, c, ctas)
    if b1 <= b0:
        return None
    u = (b1 - 1) // nkb
    if (u + 1) * nkb <= b1 or u * nkb < b0:
        return None
    pieces = []
    cc = c
    while cc < ctas and cta_range(units, nkb, 1, cc, ctas)[0] < (u + 1) * nkb:
        slot = (0 if b0 == u * nkb else 1) if cc == c else 0
        pieces.append((cc, slot))
        cc += 1
    return u, pieces


def launch_plan(bh, n, rows_per_unit, sms):
    q_blocks = -(-n // rows_per_unit)
    nkb = -(-n // 128)
    units = q_blocks * bh
    ctas, split = min(units, sms), 0
    if units % sms and units < 32 * sms:
        waves = units / sms
        if waves / (-(-units // sms)) < 0.97:
            split = 1
            ctas = min(units * nkb, sms)
    return units, nkb, ctas, split


CASES = [(8, 8192, 256, 148), (1, 128, 256, 148), (2, 2048, 256, 148), (256, 4096, 256, 148),
         (32, 32768, 256, 148), (2048, 512, 256, 148), (3, 192, 128, 148), (6, 256, 256, 148),
         (7, 1024, 256, 13), (5, 640, 128, 148)]


@pytest.mark.parametrize("bh,n,rows,sms", CASES)
def test_every_unit_once_and_pieces_merged_once(bh, n, rows, sms):
    units, nkb, ctas, split = launch_plan(bh, n, rows, sms)
    seen = {}
    written_slots = {}
    partial = {}
    for c in range(ctas):
        assert list(segments(units, nkb, split, c, ctas)) == list(
            cursor_segments(units, nkb, split, c, ctas))
        for u, j0, j1, first in segments(units, nkb, split, c, ctas):
            for j in range(j0, j1):
                assert (u, j) not in seen
                seen[(u, j)] = c
            if not (j0 == 0 and j1 == nkb):
                assert split, "whole-block mode produced a partial segment"
                slot = (c, 0 if first else 1)
                assert slot not in written_slots
                written_slots[slot] = u
                partial.setdefault(u, set()).add(slot)
    assert len(seen) == units * nkb
    merged = {}
    if split:
        for c in range(ctas):
            plan = merge_plan(units, nkb, c, ctas)
            if plan is None:
                continue
            u, pieces = plan
            assert u not in merged
            merged[u] = set(pieces)
    assert set(merged) == set(partial)
    for u, pieces in merged.items():
        assert pieces == partial[u]


def test_headline_shape_uses_split_and_all_sms():
    units, nkb, ctas, split = launch_plan(8, 8192, 256, 148)
    assert (units, nkb, ctas, split) == (256, 64, 148, 1)
    work = [sum(j1 - j0 for _, j0, j1, _ in segments(units, nkb, 1, c, ctas)) for c in range(ctas)]
    assert max(work) - min(work) <= 1


def test_large_grid_keeps_whole_blocks():
    assert launch_plan(256, 4096, 256, 148)[3] == 0
