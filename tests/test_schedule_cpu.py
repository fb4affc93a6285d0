"""CPU check of the persistent work schedule of mfa_fwd_kernel, restated here from
csrc/mfa_schedule.cuh (Schedule: steps_of, first_of, locate; split_range), csrc/mfa_fwd_kernel.cuh
(StepCursor; mfa_merge_kernel's owner / piece rules) and the launcher's plan (plan_forward in
csrc/mfa_capi.cu). Checked, with and without causal masking: every (query block, key block)
step that the mask needs is processed exactly once, every partial piece lands in its own
workspace slot, and every query block cut into pieces is merged exactly once from exactly its
pieces. With causal masking the query blocks of a head run in the order 0, Q-1, 1, Q-2, ...
(pairs of short and long blocks), which spreads unit epilogues and diagonal blocks evenly over
the CTAs; the brute force below walks the steps in that order and is checked against the
O(1) locate of the kernels."""
from __future__ import annotations


import pytest


class Schedule:
    """Query rows [q_begin, q_end) of every head (all n by default); with the mask the range
    starts on a unit boundary, its blocks are numbered from qb0 = q_begin / rows_per_unit and
    the keys end at q_end (make_schedule's nq, nk, qb0)."""

    def __init__(self, bh, n, rows_per_unit, causal, keys=128, q_begin=0, q_end=None):
        q_end = n if q_end is None else q_end
        self.bh = bh
        self.q_blocks = -(-(q_end - q_begin) // rows_per_unit)
        self.nkb = -(-(q_end if causal else n) // keys)
        self.group = rows_per_unit // keys
        self.causal = causal
        self.qb0 = q_begin // rows_per_unit if causal else 0
        self.head_steps = sum(self.steps_of(qb) for qb in range(self.q_blocks))

    def steps_of(self, qb):
        if not self.causal:
            return self.nkb
        return self.nkb if qb == self.q_blocks - 1 else (qb + 1 + self.qb0) * self.group

    # causal processing order within a head: position k holds query block qb_at(k)
    def qb_at(self, k):
        return self.q_blocks - 1 - k // 2 if k % 2 else k // 2

    def pos_of(self, qb):
        return 2 * qb if 2 * qb < self.q_blocks else 2 * (self.q_blocks - 1 - qb) + 1

    def order(self):
        """Query blocks of a head in processing order (brute force)."""
        return [self.qb_at(k) for k in range(self.q_blocks)] if self.causal \
            else list(range(self.q_blocks))

    def pair0(self):
        return self.group * (1 + self.qb0) + self.nkb

    def pair(self):
        return self.group * (self.q_blocks + 1 + 2 * self.qb0)

    def pos_first(self, k):
        pair0, pair = self.pair0(), self.pair()
        m = k // 2
        f = 0 if m == 0 else pair0 + (m - 1) * pair
        return f + (self.steps_of(m) if k % 2 else 0)

    def first_of(self, qb):
        return self.pos_first(self.pos_of(qb)) if self.causal else qb * self.nkb

    def total(self):
        return self.head_steps * self.bh

    def unit_first(self, u):
        return u // self.q_blocks * self.head_steps + self.first_of(u % self.q_blocks)

    def next_unit(self, u):
        if not self.causal:
            return u + 1
        head, qb = divmod(u, self.q_blocks)
        k = self.pos_of(qb) + 1
        return head * self.q_blocks + self.qb_at(k) if k < self.q_blocks \
            else (head + 1) * self.q_blocks

    def locate(self, s):
        head, r = divmod(s, self.head_steps)
        if not self.causal:
            return head * self.q_blocks + r // self.nkb, r % self.nkb
        pairs = self.q_blocks // 2
        pair0, pair = self.pair0(), self.pair()
        if pairs > 0 and r < pair0:
            k, rem = 0, r
        elif pairs > 1 and r < pair0 + (pairs - 1) * pair:
            m = 1 + (r - pair0) // pair
            k, rem = 2 * m, r - pair0 - (m - 1) * pair
        else:
            k = self.q_blocks - 1
            rem = r - self.pos_first(k)
        if k % 2 == 0 and k + 1 < self.q_blocks and rem >= self.steps_of(k // 2):
            rem -= self.steps_of(k // 2)
            k += 1
        return head * self.q_blocks + self.qb_at(k), rem


def split_range(total, cta, ctas):
    return total * cta // ctas, total * (cta + 1) // ctas


def plan(bh, n, rows_per_unit, sms, causal, q_begin=0, q_end=None):
    sc = Schedule(bh, n, rows_per_unit, causal, q_begin=q_begin, q_end=q_end)
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
    for head in range(sc.bh):
        for qb in sc.order():
            u = head * sc.q_blocks + qb
            for j in range(sc.steps_of(qb)):
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
        u = sc.next_unit(u)
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
                                       (1, 640, 128), (5, 32768, 256), (2, 256, 256),
                                       (2, 257, 256), (3, 640, 256), (1, 129, 128)])
def test_locate_inverts_the_causal_order(bh, n, rows):
    sc = Schedule(bh, n, rows, causal=True)
    assert sorted(sc.order()) == list(range(sc.q_blocks))
    assert all(sc.pos_of(sc.qb_at(k)) == k for k in range(sc.q_blocks))
    step = max(1, sc.total() // 5000)
    for s in list(range(0, sc.total(), step)) + [sc.total() - 1]:
        u, j = sc.locate(s)
        assert 0 <= j < sc.steps_of(u % sc.q_blocks)
        assert sc.unit_first(u) + j == s
    # the order walks every unit of every head once
    u, seen = 0, []
    while u < sc.bh * sc.q_blocks:
        seen.append(u)
        u = sc.next_unit(u)
    assert sorted(seen) == list(range(sc.bh * sc.q_blocks))


def test_causal_order_balances_unit_counts():
    # B1 H8 N8192 causal: every CTA gets one to three query blocks (ascending order: 1 to 8)
    sc, ctas, split = plan(8, 8192, 256, 148, True)
    units = [len(list(cursor_segments(sc, split, c, ctas))) for c in range(ctas)]
    assert split and max(units) <= 3


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


def magic(d):
    """Multiplier and shift of Schedule::head_of (make_schedule in csrc/mfa_schedule.cuh)."""
    lg = 0
    while (1 << lg) < d:
        lg += 1
    shift = 31 + lg
    return -(-(1 << shift) // d), shift


@pytest.mark.parametrize("d", [1, 2, 3, 5, 7, 31, 32, 33, 64, 100, 127, 129, 4095, 65537,
                               (1 << 20) + 1, (1 << 30) + 3, (1 << 31) - 1])
def test_magic_division_by_query_blocks(d):
    import random
    mul, shift = magic(d)
    assert mul < 1 << 32
    rng = random.Random(d)
    us = [0, 1, d - 1, d, d + 1, (1 << 31) - 1, (1 << 31) - 2] + \
        [rng.randrange(1 << 31) for _ in range(2000)] + [d * k - 1 for k in range(1, 50)]
    for u in us:
        if 0 <= u < 1 << 31:
            assert (u * mul) >> shift == u // d, (u, d)


# query row ranges (mfa_fwd_rows): the ranges of sharding.q_shard and a few others
RANGES = [(1, 8192, 256, 148, 0, 4096), (1, 8192, 256, 148, 4096, 8192),
          (2, 5000, 256, 37, 2048, 5000), (3, 3000, 256, 148, 768, 1792),
          (1, 65536, 256, 148, 57344, 65536), (2, 1000, 128, 13, 512, 1000),
          (1, 640, 256, 148, 512, 640)]


@pytest.mark.parametrize("causal", [False, True], ids=["full", "causal"])
@pytest.mark.parametrize("bh,n,rows,sms,q0,q1", RANGES)
def test_row_range_steps_once_and_locate(bh, n, rows, sms, q0, q1, causal):
    sc, ctas, split = plan(bh, n, rows, sms, causal, q0, q1)
    seen = set()
    for c in range(ctas):
        segs = list(segments(sc, split, c, ctas))
        assert segs == list(cursor_segments(sc, split, c, ctas))
        for u, j0, j1, _ in segs:
            for j in range(j0, j1):
                assert (u, j) not in seen
                seen.add((u, j))
    units = bh * sc.q_blocks
    assert seen == {(u, j) for u in range(units) for j in range(sc.steps_of(u % sc.q_blocks))}
    for u in range(units):
        qb = u % sc.q_blocks
        last_row = min(q1, q0 + (qb + 1) * rows) - 1  # absolute row of the block's last query
        want = last_row // 128 + 1 if causal else -(-n // 128)
        assert sc.steps_of(qb) == want
    if causal:
        step = max(1, sc.total() // 3000)
        for s_ in list(range(0, sc.total(), step)) + [sc.total() - 1]:
            u, j = sc.locate(s_)
            assert sc.unit_first(u) + j == s_
