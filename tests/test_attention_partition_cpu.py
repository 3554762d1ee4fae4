"""The paged decode attention's work partition, restated on the host: the flattened
page list cut into equal ranges of a virtual space where each row is preceded by
kRowWeight units (csrc/attention.cu: range_bound, the first-row search, find_piece,
and the merge kernel's cta_of of a row's first and last page).  For every weight and
many ragged batches: each page is processed exactly once, pieces stay inside their
row, a row split over several CTAs is exactly the CTAs [c_lo, c_hi] the merge reads,
and segment ids c + b are distinct and below ctas + rows (the work capacity).  With
no more pages than ranges the weight is 0 and every range is one page, so a row's split
does not depend on the other rows (the batch-invariance the GPU tests rely on)."""

from __future__ import annotations

import random

import pytest


def range_bound(c, total, ctas):
    return (total * c) // ctas


def cta_of(pos, total, ctas):
    c = (pos * ctas) // total
    while c + 1 < ctas and range_bound(c + 1, total, ctas) <= pos:
        c += 1
    while c > 0 and range_bound(c, total, ctas) > pos:
        c -= 1
    return c


def row_weight(total, grid_ctas, weight):
    """w = the row weight once the batch has more pages than ranges, else 0."""
    return weight if total > grid_ctas else 0


def pieces_of(c, pptr, rows, ctas, w):
    total = pptr[rows]
    tv = total + rows * w
    a0, a1 = range_bound(c, tv, ctas), range_bound(c + 1, tv, ctas)
    lo, hi = 0, rows - 1
    while lo < hi:
        mid = (lo + hi) >> 1
        if pptr[mid + 1] + (mid + 1) * w > a0:
            hi = mid
        else:
            lo = mid + 1
    out = []
    b = lo
    while b < rows and pptr[b] + (b + 1) * w < a1:
        off = (b + 1) * w
        r0, r1 = max(a0 - off, pptr[b]), min(a1 - off, pptr[b + 1])
        if r0 < r1:
            out.append((b, r0, r1))
        b += 1
    return out


@pytest.mark.parametrize("w", [0, 1, 2, 4, 8])
@pytest.mark.parametrize("seed", range(25))
def test_partition_covers_every_page_once(w, seed):
    rng = random.Random(seed * 31 + w)
    rows = rng.choice([1, 2, 7, 64, 200, 513])
    npages = [rng.choice([0, 1, 1, 2, 3, 5, 20, 60, 400]) if rng.random() < 0.9 else rng.randint(1, 600)
              for _ in range(rows)]
    if sum(npages) == 0:
        npages[0] = 1
    pptr = [0]
    for n in npages:
        pptr.append(pptr[-1] + n)
    total = pptr[-1]
    grid = rng.choice([1, 3, 74, 148, 296])
    ctas = min(grid, total)
    w = row_weight(total, grid, w)
    seen = [0] * total
    by_row: dict[int, list] = {}
    segs = set()
    for c in range(ctas):
        for b, r0, r1 in pieces_of(c, pptr, rows, ctas, w):
            assert pptr[b] <= r0 < r1 <= pptr[b + 1]
            for q in range(r0, r1):
                seen[q] += 1
            by_row.setdefault(b, []).append((c, r0, r1))
            seg = c + b
            assert seg not in segs and seg < ctas + rows - 1 + 1
            segs.add(seg)
    assert all(v == 1 for v in seen)
    tv = total + rows * w
    for b in range(rows):
        rp0, rp1 = pptr[b], pptr[b + 1]
        if rp0 == rp1:
            assert b not in by_row
            continue
        off = (b + 1) * w
        c_lo, c_hi = cta_of(rp0 + off, tv, ctas), cta_of(rp1 - 1 + off, tv, ctas)
        got = by_row[b]
        assert [c for c, _, _ in got] == list(range(c_lo, c_hi + 1))
        whole = [(r0 == rp0 and r1 == rp1) for _, r0, r1 in got]
        assert whole == ([True] if c_lo == c_hi else [False] * len(got))


def test_small_batches_split_by_page_whatever_the_other_rows():
    """With no more pages than ranges, a row's pieces are its single pages, whichever
    rows surround it."""
    grid = 148
    for extra in ([], [3], [1, 7, 20], [50, 2]):
        npages = [2, 1, 3] + extra
        pptr = [0]
        for n in npages:
            pptr.append(pptr[-1] + n)
        total = pptr[-1]
        w = row_weight(total, grid, 4)
        assert w == 0
        ctas = min(grid, total)
        split = [(r1 - r0) for c in range(ctas) for b, r0, r1 in pieces_of(c, pptr, len(npages), ctas, w) if b < 3]
        assert split == [1] * 6
