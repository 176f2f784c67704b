"""Host checks of the persistent tile schedule (b200gemm_schedule_host, the
same function the device builder runs).  Reference: include/hilbert.hpp."""
import numpy as np
import pytest

from b200_gemm_b200 import schedule


def _d2xy_py(side, d):
    """Independent restatement of the published Hilbert index -> cell walk."""
    x = y = 0
    s = 1
    while s < side:
        rx = 1 & (d // 2)
        ry = 1 & (d ^ rx)
        if ry == 0:
            if rx == 1:
                x, y = s - 1 - x, s - 1 - y
            x, y = y, x
        x += s * rx
        y += s * ry
        d //= 4
        s *= 2
    return x, y


@pytest.mark.parametrize("tm,tn", [(1, 1), (1, 32), (2, 2), (3, 1), (32, 32), (64, 56), (7, 13), (5, 300)])
def test_schedule_is_curve_order_permutation(tm, tn):
    order = schedule(tm, tn)
    assert len(order) == tm * tn
    assert len(set(order)) == tm * tn
    assert all(0 <= m < tm and 0 <= n < tn for m, n in order)
    side = 1
    while side < max(tm, tn):
        side *= 2
    expect = [c for c in (_d2xy_py(side, d) for d in range(side * side)) if c[0] < tm and c[1] < tn]
    assert order == expect


def test_square_power_of_two_grid_steps_to_neighbours():
    order = schedule(32, 32)
    steps = [abs(a[0] - b[0]) + abs(a[1] - b[1]) for a, b in zip(order, order[1:])]
    assert max(steps) == 1


def _operand_panels_per_wave(order, wave):
    """Distinct A row-panels + B column-panels touched by each window of
    `wave` consecutive tiles (the tiles that run concurrently)."""
    out = []
    for i in range(0, len(order) - wave + 1, wave):
        w = order[i:i + wave]
        out.append(len({m for m, _ in w}) + len({n for _, n in w}))
    return np.mean(out)


@pytest.mark.parametrize("tm,tn", [(32, 32), (64, 64), (64, 56)])
def test_curve_order_reuses_operands_better_than_raster(tm, tn):
    wave = 74  # co-resident 2-CTA clusters on a 148-SM B200
    hil = _operand_panels_per_wave(schedule(tm, tn), wave)
    raster = _operand_panels_per_wave([(m, n) for m in range(tm) for n in range(tn)], wave)
    assert hil < 0.6 * raster, (hil, raster)


def test_round_robin_assignment_is_balanced():
    tiles = 32 * 32
    for clusters in (74, 72, 64):
        per = np.bincount(np.arange(tiles) % clusters, minlength=clusters)
        assert per.max() - per.min() <= 1
