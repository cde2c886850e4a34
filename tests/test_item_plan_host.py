"""The march kernel's work plan (bst_march_item_plan), on the host.

The persistent march kernel takes work items (a tile column x a chunk of output planes)
round-robin: CTA b runs items b, b + S, b + 2S, ... on S resident CTAs.  The plan is one band
of equal chunks, or two bands whose second, one chunk finer, fills the last wave.  These tests
check that every plan covers every plane of every tile column exactly once with chunks of whole
RB groups, and that the chosen plan is never worse than the uniform one under the launch model
the library uses (an item costs its planes plus a fixed ramp), restated here.
"""
import ctypes

import pytest


def _plan(tiles, planes, rb, overhead, resident):
    from basalto import _abi
    out = (ctypes.c_int64 * 5)()
    _abi.check(_abi.lib().bst_march_item_plan(tiles, planes, rb, overhead, resident, out))
    return tuple(out)


def _items(tiles, planes, plan):
    tiles1, chunk1, n1, chunk2, n2 = plan
    items = []
    for ci in range(n1):
        items += [min(chunk1, planes - ci * chunk1)] * tiles1
    for ci in range(n2):
        items += [min(chunk2, planes - ci * chunk2)] * (tiles - tiles1)
    return items


def _cost(items, overhead, resident):
    loads = [0] * resident
    for i, size in enumerate(items):
        loads[i % resident] += size + overhead
    return max(loads)


def _uniform_cost(tiles, planes, rb, overhead, resident):
    best = None
    for nc in range(1, min(planes // rb + 1, 4096) + 1):
        ch = -(-planes // nc)
        ch = -(-ch // rb) * rb
        real = -(-planes // ch)
        t = -(-(tiles * real) // resident) * (ch + overhead)
        if best is None or t < best[0] * 0.999:
            best = (t, ch, real)
    return _cost(_items(tiles, planes, (tiles, best[1], best[2], best[1], best[2])), overhead, resident)


CASES = [(1024, 1024, 2, 20, 296), (1024, 504, 2, 20, 296), (1024, 248, 2, 20, 296), (1024, 120, 2, 20, 296),
         (1024, 4, 2, 20, 296), (288, 768, 2, 16, 296), (64, 512, 1, 12, 296), (4096, 512, 1, 12, 592),
         (1, 77, 2, 20, 296), (37, 9, 4, 10, 148), (1024, 1, 2, 20, 296)]


@pytest.mark.parametrize("tiles,planes,rb,overhead,resident", CASES)
def test_plan_covers_every_plane_once(tiles, planes, rb, overhead, resident):
    tiles1, chunk1, n1, chunk2, n2 = plan = _plan(tiles, planes, rb, overhead, resident)
    assert 1 <= tiles1 <= tiles
    for ch, n in ((chunk1, n1), (chunk2, n2)):
        assert ch % rb == 0 or ch >= planes  # whole RB groups
        assert (n - 1) * ch < planes <= n * ch  # the chunks of a column tile [0, planes)
    if tiles1 < tiles:
        assert n2 > n1  # the second band is the finer one
    assert sum(_items(tiles, planes, plan)) == tiles * planes


@pytest.mark.parametrize("tiles,planes,rb,overhead,resident", CASES)
def test_plan_no_worse_than_uniform(tiles, planes, rb, overhead, resident):
    plan = _plan(tiles, planes, rb, overhead, resident)
    assert _cost(_items(tiles, planes, plan), overhead, resident) <= _uniform_cost(tiles, planes, rb, overhead,
                                                                                   resident)


def test_two_bands_fill_the_last_wave_at_1024_cubed():
    """1024 tile columns of 1024 planes on 296 CTAs: 864 whole columns, then 160 halved ones
    (1184 items = four full waves) instead of 2048 half columns in seven waves."""
    assert _plan(1024, 1024, 2, 20, 296) == (864, 1024, 1, 512, 2)


def test_plan_rejects_bad_arguments():
    from basalto import _abi
    out = (ctypes.c_int64 * 5)()
    assert _abi.lib().bst_march_item_plan(0, 10, 2, 20, 296, out) != 0
    assert _abi.lib().bst_march_item_plan(10, 10, 2, 20, 0, out) != 0
