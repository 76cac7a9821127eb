"""Synthetic input generator: shapes, determinism and DREAMPlace's stretch rule."""
import math

import numpy as np

from dreamplacett_framework_b200 import synth


def test_layout_and_determinism():
    a = synth.make_placement("c3", scale=0.01)
    b = synth.make_placement("c3", scale=0.01)
    np.testing.assert_array_equal(a.x, b.x)
    assert a.num_nodes == a.num_movable + a.num_terminals + a.num_filler
    (b0, e0), (b1, e1) = a.ranges
    assert (b0, e0) == (0, a.num_movable) and e1 == a.num_nodes and e1 - b1 == a.num_filler
    # cells lie inside the die
    assert (a.x >= 0).all() and (a.x + a.size_x <= a.xh + 1e-3).all()
    assert (a.y >= 0).all() and (a.y + a.size_y <= a.yh + 1e-3).all()
    # movable: height 12, width in [2, 80]; fillers 8 x 12
    mv = slice(0, a.num_movable)
    assert (a.size_y[mv] == 12).all() and a.size_x[mv].min() >= 2 and a.size_x[mv].max() <= 80
    assert (a.size_x[b1:] == 8).all() and (a.size_y[b1:] == 12).all()


def test_stretch_rule():
    p = synth.make_placement("c1", scale=0.01)
    bs = p.bin_size_x
    assert bs == 10000.0 / 512
    lim = np.float32(bs * math.sqrt(2))
    assert (p.size_x_clamped >= lim).all()
    np.testing.assert_allclose(p.offset_x, (p.size_x - p.size_x_clamped) * 0.5, rtol=0, atol=1e-6)
    np.testing.assert_allclose(p.ratio, p.size_x * p.size_y / (p.size_x_clamped * p.size_y_clamped), rtol=1e-6)
    # stretched cells keep their original area as density mass
    area = p.size_x_clamped * p.size_y_clamped * p.ratio
    np.testing.assert_allclose(area, p.size_x * p.size_y, rtol=1e-5)


def test_macros_do_not_overlap_and_rasterise_exactly():
    p = synth.make_placement("c3", scale=0.02)
    t = slice(p.num_movable, p.num_movable + p.num_terminals)
    x, y, w, h = p.x[t], p.y[t], p.size_x[t], p.size_y[t]
    assert p.num_terminals == 20
    for i in range(len(x)):
        ov = (x[i] < x + w) & (x < x[i] + w[i]) & (y[i] < y + h) & (y < y[i] + h[i])
        assert ov.sum() == 1
    total = float(np.sum(w.astype(np.float64) * h))
    assert abs(p.initial_density_map.sum() / total - 1.0) < 1e-5
