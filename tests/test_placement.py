"""Placement-loop pieces: the device overflow metric (epb_overflow), the
normalised descent step (epb_descent_step) and the benchmark's C5 loop
(dreamplacett_framework_b200.placement) against the CPU restatement.

CPU: known answers of the restated overflow and step, and the committed C5
trajectory fixture re-derived for its first steps.  GPU: overflow and step
against the restatement on the same inputs, and the full 200-step C5 loop
against the fixture."""
import os

import numpy as np
import pytest
import torch

from dreamplacett_framework_b200 import synth

from gpu_util import engine_for, geometry_for, np_, placement_cells, to_device, to_oracle

HERE = os.path.dirname(os.path.abspath(__file__))
C5_GOLDEN = os.path.join(HERE, "golden", "c5_trajectory.npz")


# ---------------------------------------------------------------- CPU ----

def test_overflow_known_answer(oracle):
    """One 2-bin-area cell inside bin (3, 5) of a 16 x 16 grid of unit bins:
    rho = 2 there, so overflow = (2 - 1) * bin_area = 1 and max density 2."""
    g = oracle.Geometry(16, 16, 0.0, 0.0, 16.0, 16.0)
    S = g.default_fixed_bits()
    cells = oracle.Cells(np.array([3.0], np.float32), np.array([5.0], np.float32), np.array([1.0], np.float32),
                         np.array([1.0], np.float32), ratio=np.array([2.0], np.float32))
    area, mx = oracle.overflow(cells, g, S, target=1.0)
    assert area == 1.0 and mx == 2.0
    init = np.zeros((16, 16), np.float32)
    init[0, 0] = 1.5
    area, mx = oracle.overflow(cells, g, S, init_norm=init, target=1.0)
    assert area == 1.5 and mx == 2.0
    assert oracle.overflow(cells, g, S, target=3.0) == (0.0, 2.0)


def test_descent_step_known_answers(oracle):
    g = oracle.Geometry(16, 16, 0.0, 0.0, 160.0, 160.0)  # bins of 10
    x = np.array([50.0, 0.5, 150.0, 70.0], np.float32)
    y = np.array([50.0, 50.0, 50.0, 70.0], np.float32)
    w = np.full(4, 8.0, np.float32)
    h = np.full(4, 12.0, np.float32)
    gx = np.array([2.0, 4.0, -4.0, np.nan], np.float32)
    gy = np.array([-1.0, 0.0, 0.0, 1.0], np.float32)
    nodes = np.arange(4)
    linf = oracle.descent_step(x, y, gx, gy, w, h, nodes, g, step_bins=0.5)
    assert linf == np.float32(4.0)                # the NaN node is skipped
    # node 0: x - (5 / 4) * 2 = 47.5, y + 1.25
    assert x[0] == np.float32(47.5) and y[0] == np.float32(51.25)
    assert x[1] == np.float32(0.0)                 # clamped at xl
    assert x[2] == np.float32(152.0)               # clamped at xh - w
    assert x[3] == np.float32(70.0) and y[3] == np.float32(70.0)  # non-finite gradient: stays
    x0 = x.copy()
    assert oracle.descent_step(x, y, np.zeros(4, np.float32), np.zeros(4, np.float32), w, h, nodes, g) == 0
    np.testing.assert_array_equal(x, x0)


def test_c5_golden_first_steps(oracle):
    """The committed C5 trajectory is the restatement's: its first steps re-run here."""
    gold = np.load(C5_GOLDEN)
    assert int(gold["steps"]) == 200 and gold["overflow"].shape == (201,)
    p = synth.make_placement("c5")
    g = geometry_for(oracle, p)
    threads = os.cpu_count() or 1
    r = oracle.descent_trajectory(p.x, p.y, p.size_x, p.size_y, p.size_x_clamped, p.size_y_clamped, p.offset_x,
                                  p.offset_y, p.ratio, p.ranges, (0, p.num_movable), g, g.default_fixed_bits(),
                                  p.initial_density_norm(), steps=2, nthreads=threads, workers=threads)
    np.testing.assert_allclose(r["overflow"], gold["overflow"][:3], rtol=1e-12)
    np.testing.assert_allclose(r["energy"], gold["energy"][:2], rtol=1e-9)
    np.testing.assert_array_equal(r["linf"], gold["linf"][:2])
    # the loop spreads the cells: the maximum density falls
    assert gold["max_density"][-1] < 0.25 * gold["max_density"][0]
    assert gold["overflow"][-1] < gold["overflow"][0]


# ---------------------------------------------------------------- GPU ----

@pytest.mark.gpu
@pytest.mark.parametrize("config,scale", [("c5", 1.0), ("c3", 0.25), ("c1", 1.0)])
def test_overflow_matches_oracle(oracle, cuda_device, config, scale):
    p = synth.make_placement(config, scale=scale)
    arrs, _ = placement_cells(p)
    mov = ((0, p.num_movable), (0, 0))
    g = geometry_for(oracle, p)
    init = p.initial_density_norm()
    ref_area, ref_max = oracle.overflow(to_oracle(oracle, arrs, mov), g, g.default_fixed_bits(), init)
    with engine_for(p, cuda_device) as eng:
        eng.set_initial_density(torch.from_numpy(init).to(cuda_device))
        cells = to_device(arrs, mov, cuda_device)
        for _ in range(2):  # the grid must be left zeroed for the next call
            out = np_(eng.overflow(cells, 1.0))
            assert out[0] == pytest.approx(ref_area, rel=1e-12, abs=1e-9)
            assert out[1] == ref_max
        assert eng.error_flags() == 0
        # the forward after an overflow call still sees a zeroed grid
        dens = eng.forward(to_device(arrs, p.ranges, cuda_device))["density"]
    grid, _ = oracle.density_fixed(to_oracle(oracle, arrs, p.ranges), g, g.default_fixed_bits())
    rho, _ = oracle.fixed_to_density(grid, g, g.default_fixed_bits(), init)
    np.testing.assert_array_equal(np_(dens), rho)


@pytest.mark.gpu
def test_descent_step_bit_exact(oracle, cuda_device):
    p = synth.make_placement("c3", scale=0.1, grid=512)
    arrs, ranges = placement_cells(p)
    with engine_for(p, cuda_device) as eng:
        cells = to_device(arrs, ranges, cuda_device)
        eng.forward(cells)
        gx, gy = eng.backward(cells)
        gx_h, gy_h = np_(gx), np_(gy)
        gx_h[5] = np.nan  # a non-finite gradient stays put on both sides
        gx.copy_(torch.from_numpy(gx_h))
        w = torch.from_numpy(p.size_x).to(cuda_device)
        h = torch.from_numpy(p.size_y).to(cuda_device)
        linf = eng.descent_step(cells, gx, gy, w, h, 0.5)
        x_ref, y_ref = p.x.copy(), p.y.copy()
        ref_linf = oracle.descent_step(x_ref, y_ref, gx_h, gy_h, p.size_x, p.size_y,
                                       to_oracle(oracle, arrs, ranges).nodes(), geometry_for(oracle, p), 0.5)
        assert float(linf.item()) == float(ref_linf)
        np.testing.assert_array_equal(np_(cells.x), x_ref)
        np.testing.assert_array_equal(np_(cells.y), y_ref)
        assert eng.error_flags() & 0x1  # the NaN was reported


@pytest.mark.gpu
def test_descent_step_rejects_bad_arguments(cuda_device):
    from dreamplacett_framework_b200 import _lib
    p = synth.make_placement("c1", scale=0.01)
    arrs, ranges = placement_cells(p)
    with engine_for(p, cuda_device) as eng:
        cells = to_device(arrs, ranges, cuda_device)
        z = torch.zeros(p.num_nodes, device=cuda_device)
        with pytest.raises(_lib.EpbError):
            eng.descent_step(cells, z, z, z, z, float("nan"))
        st = eng.lib.epb_descent_step(eng.handle, eng._cells(cells), None, None, None, None, None, None,
                                      0.5, None, None)
        assert st == _lib.EPB_EINVAL


@pytest.mark.gpu
def test_c5_loop_matches_golden_trajectory(cuda_device):
    """200 steps of the C5 loop on the GPU against the restatement's fp64
    trajectory.  fp32 fields move the trajectory by about 1e-7 relative (an
    fp32 DCT in the restatement itself moves it by 2e-7), so the bound is
    1e-5 of each series' largest value."""
    from dreamplacett_framework_b200.placement import DensityDescent
    gold = np.load(C5_GOLDEN)
    p = synth.make_placement("c5")
    with DensityDescent(p, device=cuda_device) as loop:
        r = loop.run(200, graph=True)
        assert r["flags"] == 0
        x_sum = float(loop.x.double().sum())
        y_sum = float(loop.y.double().sum())
    for k in ("overflow", "max_density", "energy", "linf"):
        a, b = np.asarray(r[k], np.float64), np.asarray(gold[k], np.float64)
        assert a.shape == b.shape, k
        assert np.max(np.abs(a - b)) / np.max(np.abs(b)) < 1e-5, k
    assert x_sum == pytest.approx(float(gold["x_sum"]), rel=1e-6)
    assert y_sum == pytest.approx(float(gold["y_sum"]), rel=1e-6)


@pytest.mark.gpu
def test_c5_loop_graph_equals_eager(cuda_device):
    """The captured step is the eager step: identical trajectories."""
    from dreamplacett_framework_b200.placement import DensityDescent
    p = synth.make_placement("c5", scale=0.1, grid=256)
    runs = []
    for graph in (False, True):
        with DensityDescent(p, device=cuda_device) as loop:
            runs.append((loop.run(20, graph=graph), np_(loop.x), np_(loop.y)))
    (a, ax, ay), (b, bx, by) = runs
    for k in ("overflow", "max_density", "energy", "linf"):
        np.testing.assert_array_equal(a[k], b[k])
    np.testing.assert_array_equal(ax, bx)
    np.testing.assert_array_equal(ay, by)


@pytest.mark.gpu
@pytest.mark.parametrize("config,scale,grid", [("c5", 1.0, None), ("c3", 0.25, None), ("c1", 0.05, 64)])
def test_forward_overflow_equals_separate_calls(cuda_device, config, scale, grid):
    """epb_forward_overflow: the movable range's overflow exactly as epb_overflow
    reports it, and the forward of both ranges exactly as epb_forward (twice in
    a row, so both grids are left zeroed)."""
    p = synth.make_placement(config, scale=scale, grid=grid)
    arrs, ranges = placement_cells(p)
    with engine_for(p, cuda_device) as eng:
        eng.set_initial_density(torch.from_numpy(p.initial_density_norm()).to(cuda_device))
        cells = to_device(arrs, ranges, cuda_device)
        movable = to_device(arrs, (ranges[0], (0, 0)), cuda_device)
        ref_ovf = eng.overflow(movable, 1.0).clone()
        ref = {k: v.clone() for k, v in eng.forward(cells).items()}
        for _ in range(2):
            out, ovf = eng.forward_overflow(cells, 1.0)
            assert torch.equal(ovf, ref_ovf)
            for k in ("density", "potential", "field_x", "field_y", "energy"):
                assert torch.equal(out[k], ref[k]), k
        rgx, rgy = eng.backward(cells)
        assert eng.error_flags() == 0
