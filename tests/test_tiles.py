"""The cell-tile path (EPB_CONFIG_TILES) against the cell-order path (the
default) and the CPU oracle.

Both paths sum the same integer contributions, so the density is compared bit
for bit, and their gathers do the same fp32 arithmetic per cell, so the
gradients are compared bit for bit too.  The cases exercise what only the tile
path has: hot tiles split over several work items, cells that take the escape
path (non-finite, empty, off the die, wider than the tile lists allow), cells
moved between forward and backward, a backward on other cells than the
forward's, and host buffers.
"""
import numpy as np
import pytest
import torch

from dreamplacett_framework_b200 import synth
from dreamplacett_framework_b200.engine import CellTensors, ElectricPotentialEngine

from gpu_util import geometry_for, np_, placement_cells, to_device, to_oracle

pytestmark = pytest.mark.gpu


def _engines(p, dev):
    mk = lambda path: ElectricPotentialEngine(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh, device=dev,
                                              path=path)
    return mk("tiles"), mk("cell_order")


def _step(eng, cells, init=None):
    if init is not None:
        eng.set_initial_density(init)
    out = {k: v.clone() for k, v in eng.forward(cells).items()}
    gx, gy = eng.backward(cells)
    return out, gx.clone(), gy.clone()


def _same(a, b):
    (oa, gxa, gya), (ob, gxb, gyb) = a, b
    for k in ("density", "potential", "field_x", "field_y", "energy"):
        assert torch.equal(oa[k], ob[k]), k
    assert torch.equal(gxa, gxb) and torch.equal(gya, gyb)


@pytest.mark.parametrize("config,scale,grid", [("c1", 1.0, None), ("c2", 1.0, None), ("c3", 0.3, 1024),
                                               ("c3", 1.0, None)])
def test_tiles_match_cell_order(cuda_device, config, scale, grid):
    p = synth.make_placement(config, scale=scale, grid=grid)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    init = torch.from_numpy(p.initial_density_norm()).to(cuda_device)
    et, ec = _engines(p, cuda_device)
    with et, ec:
        a = _step(et, cells, init)
        b = _step(ec, cells, init)
        _same(a, b)
        # a second call on the same engine: nothing of the first is left over
        _same(_step(et, cells), a)
        assert et.error_flags() == 0 and ec.error_flags() == 0


def _hot_and_escape_cells(dev, M=256, die=2560.0, seed=5):
    """Cells piled on a few bins (tiles far above one work item), plus cells
    that take the escape path: non-finite, zero-sized, off the die and wider
    than four tiles."""
    rng = np.random.default_rng(seed)
    n = 60000
    x = rng.uniform(0, die - 40, n).astype(np.float32)
    y = rng.uniform(0, die - 40, n).astype(np.float32)
    hot = rng.random(n) < 0.5
    x[hot] = rng.normal(700.0, 6.0, hot.sum()).astype(np.float32)   # one 32x32 tile holds ~30k cells
    y[hot] = rng.normal(1300.0, 6.0, hot.sum()).astype(np.float32)
    sx = rng.uniform(3, 30, n).astype(np.float32)
    sy = rng.uniform(3, 30, n).astype(np.float32)
    ratio = rng.uniform(0.2, 1.0, n).astype(np.float32)
    sx[:40] = rng.uniform(400, 1200, 40)     # wider than 32 bins of 10: more than four tiles
    sy[:40] = rng.uniform(400, 1200, 40)
    x[40] = np.nan                            # non-finite
    sy[41] = 0.0                              # empty
    x[42] = die + 100.0                       # off the die
    y[43] = -500.0                            # partly off the die
    arrs = dict(x=x, y=y, size_x=sx, size_y=sy, offset_x=None, offset_y=None, ratio=ratio)
    ranges = ((0, 30000), (30500, n))
    return arrs, ranges, M, die


def test_hot_tiles_and_escape_cells(cuda_device, oracle):
    arrs, ranges, M, die = _hot_and_escape_cells(cuda_device)
    cells = to_device(arrs, ranges, cuda_device)
    mk = lambda path: ElectricPotentialEngine(M, M, 0.0, 0.0, die, die, device=cuda_device, path=path)
    with mk("tiles") as et, mk("cell_order") as ec:
        a, b = _step(et, cells), _step(ec, cells)
        _same(a, b)
        assert et.error_flags() == 1 and ec.error_flags() == 1   # the NaN cell, reported by both
        # twice in a row: the escape grid is left zeroed
        _same(_step(et, cells), a)
        et.error_flags()
        g = oracle.Geometry(M, M, 0.0, 0.0, die, die)
        ref, bad = oracle.density_fixed(to_oracle(oracle, arrs, ranges), g, et.fixed_point_bits)
        rho, _ = oracle.fixed_to_density(ref, g, et.fixed_point_bits)
        np.testing.assert_array_equal(np_(a[0]["density"]), rho)


def test_backward_uses_the_forward_positions(cuda_device):
    """The backward computes the gradient at the positions of the last forward
    on the same cell arrays (as DREAMPlace's backward uses the positions its
    forward saved): moving the cells in place in between changes nothing."""
    p = synth.make_placement("c1", scale=0.5)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    with _engines(p, cuda_device)[0] as et:
        et.forward(cells)
        gx0, gy0 = (t.clone() for t in et.backward(cells))
        cells.x.add_(7.0)
        gx1, gy1 = et.backward(cells)
        assert torch.equal(gx0, gx1) and torch.equal(gy0, gy1)


@pytest.mark.parametrize("max_move_bins", [1.5, 6.0])
def test_moving_cells_validate_escape_and_rebuild(cuda_device, max_move_bins):
    """Cells moved between forwards: within the listing margin (2 bins) the
    lists stay valid; further moves take the escape path in that call and the
    next forward rebuilds the lists.  Every step equals the cell-order path."""
    p = synth.make_placement("c1", scale=0.5)
    arrs, ranges = placement_cells(p)
    ct = to_device(arrs, ranges, cuda_device)
    cc = to_device(arrs, ranges, cuda_device)
    et, ec = _engines(p, cuda_device)
    g = torch.Generator(device="cpu").manual_seed(11)
    with et, ec:
        for step in range(4):
            _same(_step(et, ct), _step(ec, cc))
            dx = ((torch.rand(ct.x.shape, generator=g) * 2 - 1) * max_move_bins * p.bin_size_x).to(cuda_device)
            dy = ((torch.rand(ct.y.shape, generator=g) * 2 - 1) * max_move_bins * p.bin_size_y).to(cuda_device)
            for c in (ct, cc):
                c.x.add_(dx)
                c.y.add_(dy)
        assert et.error_flags() == 0 and ec.error_flags() == 0


def test_backward_on_other_cells(cuda_device):
    """A backward on other cell arrays than the forward's bins them first."""
    p = synth.make_placement("c1", scale=0.3)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    movable = CellTensors(cells.x, cells.y, cells.size_x, cells.size_y, cells.offset_x, cells.offset_y,
                          cells.ratio, ranges=((0, p.num_movable), (0, 0)))
    et, ec = _engines(p, cuda_device)
    with et, ec:
        et.forward(cells)
        ec.forward(cells)
        gxa, gya = et.backward(movable)
        gxb, gyb = ec.backward(movable)
        assert torch.equal(gxa, gxb) and torch.equal(gya, gyb)


def test_host_buffers_match(cuda_device):
    p = synth.make_placement("c1", scale=0.5)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    n = p.num_nodes
    hx = torch.from_numpy(np.ascontiguousarray(p.x, np.float32)).pin_memory()
    hy = torch.from_numpy(np.ascontiguousarray(p.y, np.float32)).pin_memory()
    et, ec = _engines(p, cuda_device)
    with et, ec:
        res = []
        for eng in (et, ec):
            cells.x.zero_()
            cells.y.zero_()
            out = {k: v.clone() for k, v in eng.forward_host(cells, hx, hy).items()}
            hgx = torch.zeros(n).pin_memory()
            hgy = torch.zeros(n).pin_memory()
            gx = torch.zeros(n, device=cuda_device)
            gy = torch.zeros(n, device=cuda_device)
            eng.backward_host(cells, hgx, hgy, grad_x=gx, grad_y=gy)
            torch.cuda.synchronize(cuda_device)
            for a, b in ranges:
                assert torch.equal(cells.x[a:b].cpu(), hx[a:b]) and torch.equal(cells.y[a:b].cpu(), hy[a:b])
            res.append((out, hgx.clone(), hgy.clone()))
        (oa, ax, ay), (ob, bx, by) = res
        for k in ("density", "potential", "field_x", "field_y", "energy"):
            assert torch.equal(oa[k], ob[k]), k
        assert torch.equal(ax, bx) and torch.equal(ay, by)


def test_profile_reports_bin_stage(cuda_device):
    p = synth.make_placement("c1", scale=0.2)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    with _engines(p, cuda_device)[0] as eng:
        eng.profile_start(4)
        for _ in range(2):
            eng.forward(cells)
            eng.backward(cells)
        st = eng.profile_stop()
    assert st["bin"][1] == 2 and st["scatter"][1] == 2 and st["gather"][1] == 2
    assert all(st[k][0] > 0 for k in ("bin", "scatter", "row_fwd", "column", "row_inv", "gather"))
