"""CPU check of the persistent work schedule of mfa_fwd_kernel, restated here from
csrc/mfa_schedule.cuh (Schedule: steps_of, first_of, locate; split_range), csrc/mfa_fwd_kernel.cuh
(StepCursor; mfa_merge_kernel's owner / piece rules) and the launcher's plan (plan_forward in
csrc/mfa_capi.cu). Checked, with and without causal masking: every (query block, key block)
step that the mask needs is processed exactly once, every partial piece lands in its own
workspace slot, and every query block cut into pieces is merged exactly once from exactly its
pieces."""
from __future__ import annotations

import math

import pytest


class Schedule:
    def __init__(self, bh, n, rows_per_unit, causal, keys=128):
        self.bh = bh
        self.q_blocks = -(-n // rows_per_unit)
        self.nkb = -(-n // keys)
        self.group = rows_per_unit // keys
        self.causal = causal
        self.head_steps = self.first_of(self.q_blocks - 1) + self.steps_of(self.q_blocks - 1)

    def steps_of(self, qb):
        return min(self.nkb, (qb + 1) * self.group) if self.causal else self.nkb

    def first_of(self, qb):
        return self.group * qb * (qb + 1) // 2 if self.causal else qb * self.nkb

    def total(self):
        return self.head_steps * self.bh

    def unit_first(self, u):
        return u // self.q_blocks * self.head_steps + self.first_of(u % self.q_blocks)

    def locate(self, s):
        head, r = divmod(s, self.head_steps)
        if not self.causal:
            qb = r // self.nkb
        else:
            qb = int((math.sqrt(8.0 * r / self.group + 1.0) - 1.0) * 0.5)
            qb = max(0, min(qb, self.q_blocks - 1))
            while qb + 1 < self.q_blocks and self.first_of(qb + 1) <= r:
                qb += 1
            while qb > 0 and self.first_of(qb) > r:
                qb -= 1
        return head * self.q_blocks + qb, r - self.first_of(qb)


def split_range(total, cta, ctas):
    return total * cta // ctas, total * (cta + 1) // ctas


def plan(bh, n, rows_per_unit, sms, causal):
    sc = Schedule(bh, n, rows_per_unit, causal)
    units = sc.q_blocks * bh
    ctas, split = min(units, sms), 0
    if causal:
        split = 1
    elif units % sms and units < 32 * sms:
        if (units / sms) / (-(-units // sms)) < 0.97:
            split = 1
    if split:
        ctas = min(sc.total(), sms)
    return sc, ctas, split


def segments(sc, split, cta, ctas):
    """Brute force: (u, j0, j1, first_of_range) segments of CTA `cta`."""
    units = sc.bh * sc.q_blocks
    if not split:
        for i, u in enumerate(range(cta, units, ctas)):
            yield u, 0, sc.nkb, i == 0
        return
    b, e = split_range(sc.total(), cta, ctas)
    steps = []
    for u in range(units):
        for j in range(sc.steps_of(u % sc.q_blocks)):
            steps.append((u, j))
    mine = steps[b:e]
    first = True
    i = 0
    while i < len(mine):
        u, j0 = mine[i]
        k = i
        while k < len(mine) and mine[k][0] == u:
            k += 1
        yield u, j0, mine[k - 1][1] + 1, first
        first = False
        i = k


def cursor_segments(sc, split, cta, ctas):
    """The kernel's StepCursor formulation (six 32-bit words) of the same walk."""
    units = sc.bh * sc.q_blocks
    if not split:
        if cta >= units:
            return
        u, rem, seg = cta, (units - 1 - cta) // ctas, 0
        while True:
            yield u, 0, sc.nkb, seg == 0
            if rem <= 0:
                return
            u, rem, seg = u + ctas, rem - 1, seg + 1
    b, e = split_range(sc.total(), cta, ctas)
    if b >= e:
        return
    u, j0 = sc.locate(b)
    length = e - b
    avail = sc.steps_of(u % sc.q_blocks) - j0
    j1 = j0 + min(length, avail)
    rem = length - (j1 - j0)
    seg = 0
    while True:
        yield u, j0, j1, seg == 0
        if rem <= 0:
            return
        u += 1
        j0, j1 = 0, min(rem, sc.steps_of(u % sc.q_blocks))
        rem -= j1
        seg += 1


def merge_plan(sc, c, ctas):
    """(u, [(cta, slot), ...]) merged by merge CTA c, or None (mfa_merge_kernel)."""
    total = sc.total()
    b0, b1 = split_range(total, c, ctas)
    if b1 <= b0:
        return None
    u, _ = sc.locate(b1 - 1)
    u0 = sc.unit_first(u)
    u1 = u0 + sc.steps_of(u % sc.q_blocks)
    if not (u1 > b1 and u0 >= b0):
        return None
    pieces = []
    cc = c
    while cc < ctas and split_range(total, cc, ctas)[0] < u1:
        pieces.append((cc, (0 if b0 == u0 else 1) if cc == c else 0))
        cc += 1
    return u, pieces


CASES = [(8, 8192, 256, 148), (1, 128, 256, 148), (2, 2048, 256, 148), (256, 4096, 256, 148),
         (2048, 512, 256, 148), (3, 192, 128, 148), (6, 256, 256, 148),
         (7, 1024, 256, 13), (5, 640, 128, 148), (1, 4096, 256, 148), (3, 384, 256, 148),
         (2, 1152, 256, 148), (4, 2304, 128, 37), (3, 300, 256, 148), (1, 1, 256, 148),
         (5, 1000, 256, 148), (2, 4095, 256, 148), (7, 77, 256, 13)]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("bh,n,rows,sms", CASES)
def test_every_step_once_and_pieces_merged_once(bh, n, rows, sms, causal):
    sc, ctas, split = plan(bh, n, rows, sms, causal)
    seen = set()
    partial = {}
    written = set()
    for c in range(ctas):
        segs = list(segments(sc, split, c, ctas))
        assert segs == list(cursor_segments(sc, split, c, ctas))
        for u, j0, j1, first in segs:
            for j in range(j0, j1):
                assert (u, j) not in seen
                seen.add((u, j))
            if not (j0 == 0 and j1 == sc.steps_of(u % sc.q_blocks)):
                assert split
                slot = (c, 0 if first else 1)
                assert slot not in written
                written.add(slot)
                partial.setdefault(u, set()).add(slot)
    units = bh * sc.q_blocks
    need = {(u, j) for u in range(units) for j in range(sc.steps_of(u % sc.q_blocks))}
    assert seen == need
    if causal:
        # the mask needs exactly the key blocks that start at or before a block's last row
        for u in range(units):
            qb = u % sc.q_blocks
            last_row = min(n, (qb + 1) * rows) - 1
            assert sc.steps_of(qb) == last_row // 128 + 1
    merged = {}
    if split:
        for c in range(ctas):
            mp = merge_plan(sc, c, ctas)
            if mp is None:
                continue
            u, pieces = mp
            assert u not in merged
            merged[u] = set(pieces)
    assert set(merged) == set(partial)
    for u, pieces in merged.items():
        assert pieces == partial[u]


@pytest.mark.parametrize("bh,n,rows", [(1, 4096, 256), (3, 384, 256), (2, 1 << 20, 256),
                                       (1, 640, 128), (5, 32768, 256)])
def test_locate_inverts_the_triangle(bh, n, rows):
    sc = Schedule(bh, n, rows, causal=True)
    step = max(1, sc.total() // 5000)
    for s in list(range(0, sc.total(), step)) + [sc.total() - 1]:
        u, j = sc.locate(s)
        assert 0 <= j < sc.steps_of(u % sc.q_blocks)
        assert sc.unit_first(u) + j == s


def test_headline_shape_uses_split_and_all_sms():
    sc, ctas, split = plan(8, 8192, 256, 148, False)
    assert (sc.bh * sc.q_blocks, sc.nkb, ctas, split) == (256, 64, 148, 1)
    work = [sum(j1 - j0 for _, j0, j1, _ in cursor_segments(sc, 1, c, ctas)) for c in range(ctas)]
    assert max(work) - min(work) <= 1


def test_large_grid_keeps_whole_blocks():
    assert plan(256, 4096, 256, 148, False)[2] == 0


def test_causal_halves_the_work():
    sc = Schedule(1, 8192, 256, causal=True)
    full = Schedule(1, 8192, 256, causal=False)
    # 32 query blocks: 2 + 4 + ... + 64 key blocks
    assert sc.total() == 2 * 32 * 33 // 2
    assert abs(sc.total() / full.total() - 0.5) < 0.02
