"""The stream-K work split of both GEMMs (b2_device.cuh: sk_begin / sk_owner / sk_slot), checked
on the CPU: every unit has exactly one owner, the owner formula agrees with the ranges, a CTA's
shared tiles map to distinct slots, and the reduction order of a tile is fixed."""

from __future__ import annotations

import itertools

import pytest


def sk_begin(total, ctas, i):
    return total * i // ctas


def sk_owner(total, ctas, u):
    return ((u + 1) * ctas - 1) // total


def sk_slot(total, ctas, upt, cta, tile):
    return 0 if sk_begin(total, ctas, cta) // upt == tile else 1


CASES = list(itertools.product([1, 2, 3, 7, 32, 40, 1187], [1, 2, 17, 40, 80], [1, 5, 148, 296, 444]))


@pytest.mark.parametrize("tiles,upt,ctas", CASES)
def test_split(tiles, upt, ctas):
    total = tiles * upt
    ctas = min(ctas, total)  # the host never launches more CTAs than units
    owners = []
    for i in range(ctas):
        lo, hi = sk_begin(total, ctas, i), sk_begin(total, ctas, i + 1)
        assert hi > lo, "every CTA owns at least one unit"
        owners += [i] * (hi - lo)
    assert len(owners) == total
    if total > 20000:
        us = range(0, total, max(1, total // 5000))
    else:
        us = range(total)
    for u in us:
        assert sk_owner(total, ctas, u) == owners[u]
    used = {}
    for t in range(tiles):
        first, last = sk_owner(total, ctas, t * upt), sk_owner(total, ctas, t * upt + upt - 1)
        contributors = sorted({owners[u] for u in range(t * upt, t * upt + upt)})
        assert contributors == list(range(first, last + 1))
        if first == last:
            continue
        first_starts_inside = sk_begin(total, ctas, first) >= t * upt
        for c in contributors:
            # division-free rule of the kernels: only `first` can start before the tile
            fast = 0 if (c != first or first_starts_inside) else 1
            assert fast == sk_slot(total, ctas, upt, c, t)
            key = (c, sk_slot(total, ctas, upt, c, t))
            assert key not in used, f"slot {key} used by tiles {used[key]} and {t}"
            used[key] = t


def test_largest_split_fits_workspace():
    # b2_internal.h: kWsMaxCtas = 1024 CTAs x 2 slots; kWsMaxTiles = 65536
    total = 1187 * 80
    ctas = min(148 * 8, 1024)
    assert sk_owner(total, ctas, total - 1) == ctas - 1
