"""The Nesterov global placer (dreamplacett_framework_b200.nesterov) and the
multi-stage driver (global_place), against the CPU restatement in
oracle/nesterov.py.

CPU tests pin the restatement itself: the schedules' closed forms, the
accelerated iteration on a quadratic, and a placement run that lowers the
overflow while keeping the wirelength in check.  GPU tests run the device
placer and compare its per-iteration trajectory with the restatement's on the
same seeded design; the multi-stage driver is checked stage by stage (density
bit-exact on each stage's grid at the positions it hands on).
"""
import json
import math
import os

import numpy as np
import pytest

import nesterov as onest
from dreamplacett_framework_b200 import synth
from dreamplacett_framework_b200.wirelength import synthetic_netlist


# C5-size trajectory bars (relative), about twice the measured differences: the first
# C5_TIGHT iterations per quantity, then the whole 200 for hpwl and overflow
C5_TIGHT = 20
C5_TOL_TIGHT = {"hpwl": 5e-3, "overflow": 5e-3, "step": 5e-3, "density_weight": 2e-2, "wirelength": 1e-2}
C5_TOL_ALL = {"hpwl": 6e-2, "overflow": 1e-2}


def _design(scale=0.02, grid=128, seed=4, spread=0.01):
    """A small C1-like design started clustered at the die centre."""
    p = synth.center_init(synth.make_placement("c1", scale=scale, grid=grid, seed=seed), seed=seed, spread=spread)
    nl = synthetic_netlist(p.size_x, p.size_y, np.arange(p.num_movable), p.num_nodes, seed=1)
    return p, nl


def test_schedules_closed_forms():
    P = dict(onest.PARAMS)
    # gamma: gamma0 * bin * 10^((20/9) tau - 11/9): 10 bins x gamma0 at tau = 1, 0.1 at tau = 0.1
    assert math.isclose(onest.gamma_of(P, 1.0, 10.0, 10.0), 4.0 * 10.0 * 10.0)
    assert math.isclose(onest.gamma_of(P, 0.1, 10.0, 10.0), 4.0 * 10.0 * 0.1)
    # mu: mu0 at no change, clamped at both ends
    assert math.isclose(onest.mu_of(P, 0.0), 1.1)
    assert onest.mu_of(P, 1e9) == 0.75 and onest.mu_of(P, -1e9) == 1.1
    # HPWL changes far beyond the reference (a large design's first iterations) saturate, not overflow
    assert onest.mu_of(P, 1e13) == 0.75 and onest.mu_of(P, -1e13) == 1.1
    from dreamplacett_framework_b200 import nesterov as dn
    dp = dn.NesterovParams()
    for tau in (0.0, 0.07, 0.5, 1.0):
        assert math.isclose(dn.gamma_of(dp, tau, 9.0, 11.0), onest.gamma_of(P, tau, 9.0, 11.0))
    for d in (-1e13, -1e6, 0.0, 3e5, 1e7, 1e13):
        assert math.isclose(dn.mu_of(dp, d), onest.mu_of(P, d))


def test_accelerated_iteration_on_a_quadratic():
    """The update (u, v, a) with the Lipschitz step of a quadratic reaches its
    minimum far faster than plain gradient descent with the same step."""
    rng = np.random.default_rng(0)
    d = np.linspace(1.0, 100.0, 50)
    x0 = rng.standard_normal(50)
    grad = lambda z: d * z
    u = v = x0.copy()
    a = 1.0
    alpha = 1.0 / d.max()
    for _ in range(60):
        u_new = v - alpha * grad(v)
        a_new = 0.5 * (1 + math.sqrt(4 * a * a + 1))
        v = u_new + (a - 1) / a_new * (u_new - u)
        u, a = u_new, a_new
    z = x0.copy()
    for _ in range(60):
        z = z - alpha * grad(z)
    f = lambda z: 0.5 * float(np.sum(d * z * z))
    assert f(u) < 0.05 * f(z)


def test_restated_placer_spreads_cells(oracle):
    p, nl = _design()
    pl = onest.Placer(p, nl, dict(iterations=300), nthreads=2, workers=2)
    h = pl.run()
    # from the centre cluster (overflow 0.75) to the stop overflow 0.07
    assert h["overflow"][0] > 0.5 and h["overflow"][-1] < 0.07 and 20 < len(h["hpwl"]) < 300
    assert np.all(np.isfinite(h["hpwl"])) and np.all(h["step"] > 0)
    # the density weight follows the schedule: each ratio is mu of the hpwl change
    lam, hp = h["density_weight"], h["hpwl"]
    for k in range(2, len(lam)):
        assert math.isclose(lam[k] / lam[k - 1], onest.mu_of(pl.P, hp[k - 1] - hp[k - 2]), rel_tol=1e-12)


@pytest.mark.gpu
def test_device_placer_follows_the_restatement(cuda_device, oracle):
    """Per-iteration hpwl, overflow, step length and density weight of the
    device placer against the CPU restatement on the same design, run to the
    stop overflow: fp32 device arithmetic against float64, so the first 20
    iterations agree to 1e-3 relative and the whole runs end alike (the
    iteration count within 10%, the final hpwl within 5%)."""
    import torch
    from dreamplacett_framework_b200.nesterov import NesterovParams, NesterovPlacer
    p, nl = _design()
    ref = onest.Placer(p, nl, dict(iterations=300), nthreads=4, workers=4).run()
    x = torch.from_numpy(p.x.copy()).to(cuda_device)
    y = torch.from_numpy(p.y.copy()).to(cuda_device)
    with NesterovPlacer(p, nl, x, y, NesterovParams(iterations=300)) as pl:
        got = pl.run().as_arrays()
    n = 20
    assert np.array_equal(got["backtracks"][:n], ref["backtracks"][:n])
    # the WA wirelength f - h cancels at the early, large smoothing (gamma of
    # thousands of units): its fp32 value carries a few 1e-3 relative error
    for k, tol in (("hpwl", 1e-3), ("overflow", 1e-3), ("step", 1e-3), ("density_weight", 1e-3),
                   ("wirelength", 5e-3)):
        rel = np.max(np.abs(got[k][:n] - ref[k][:n]) / np.maximum(np.abs(ref[k][:n]), 1e-12))
        assert rel < tol, (k, rel)
    assert got["overflow"][-1] < 0.07 and ref["overflow"][-1] < 0.07
    assert abs(len(got["hpwl"]) - len(ref["hpwl"])) <= 0.1 * len(ref["hpwl"])
    assert abs(got["hpwl"][-1] / ref["hpwl"][-1] - 1) < 0.05


@pytest.mark.gpu
def test_c5_nesterov_follows_the_restatement(cuda_device):
    """C5 size: 1.1M movable cells + 300k fillers on 1024² bins, the seeded
    synthetic netlist (1.1M nets, 4.0M pins), 200 iterations from the C5
    positions with the stop overflow at 0.  The device placer against the CPU
    restatement's trajectory (tests/golden/c5_nesterov.npz, made by
    tests/golden/make_c5_nesterov.py): fp32 device sums against float64.  The
    first 20 iterations agree within 0.1-0.5% (the density weight within 1%:
    its update exponent divides HPWL changes of a 2.9e10 HPWL) with equal
    backtracks, and the whole runs within 3% (hpwl) and 0.2% (overflow).
    On this random-netlist design the wirelength term dominates both runs:
    the cells gather (overflow 0.064 -> 0.954) as the HPWL falls 160x."""
    import torch
    from dreamplacett_framework_b200.nesterov import NesterovParams, NesterovPlacer
    ref = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "c5_nesterov.npz"))
    p = synth.make_placement("c5")
    nl = synthetic_netlist(p.size_x, p.size_y, np.arange(p.num_movable), p.num_nodes, seed=0)
    x = torch.from_numpy(p.x.copy()).to(cuda_device)
    y = torch.from_numpy(p.y.copy()).to(cuda_device)
    with NesterovPlacer(p, nl, x, y, NesterovParams(iterations=200, stop_overflow=0.0)) as pl:
        got = pl.run().as_arrays()
    K = len(ref["hpwl"])
    assert len(got["hpwl"]) == K
    n = C5_TIGHT
    assert np.array_equal(got["backtracks"][:n], ref["backtracks"][:n])
    for k, tol in C5_TOL_TIGHT.items():
        rel = np.max(np.abs(got[k][:n] - ref[k][:n]) / np.maximum(np.abs(ref[k][:n]), 1e-12))
        assert rel < tol, (k, rel)
    for k, tol in C5_TOL_ALL.items():
        rel = np.max(np.abs(got[k] - ref[k]) / np.maximum(np.abs(ref[k]), 1e-12))
        assert rel < tol, (k, rel)


@pytest.mark.gpu
def test_multistage_density_bit_exact_per_stage(cuda_device, oracle, tmp_path):
    """Two stages (128^2, then 256^2) with positions carried on the device:
    after each stage the engine's density at the positions it hands on equals
    the oracle's on that stage's grid, bit for bit."""
    import torch
    from dreamplacett_framework_b200 import global_place
    from dreamplacett_framework_b200.engine import CellTensors, ElectricPotentialEngine
    p, nl = _design(grid=128)
    cfg = dict(target_density=1.0, density_weight=8e-5, gamma=4.0, stop_overflow=0.0, ignore_net_degree=100,
               stages=[dict(num_bins_x=128, num_bins_y=128, iteration=8, learning_rate=0.01),
                       dict(num_bins_x=256, num_bins_y=256, iteration=8, learning_rate=0.01)])
    x = torch.from_numpy(p.x.copy()).to(cuda_device)
    y = torch.from_numpy(p.y.copy()).to(cuda_device)
    x_ptr = x.data_ptr()
    checks = []
    for k, st in enumerate(cfg["stages"]):
        one = dict(cfg, stages=[st])
        res = global_place.place(p, nl, one, device=cuda_device, x=x, y=y)
        assert res["x"].data_ptr() == x_ptr   # the same device tensors all along
        ps = p.regrid(st["num_bins_x"], st["num_bins_y"])
        f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda_device)
        cells = CellTensors(x, y, f(ps.size_x_clamped), f(ps.size_y_clamped), f(ps.offset_x), f(ps.offset_y),
                            f(ps.ratio), ranges=ps.ranges)
        with ElectricPotentialEngine(ps.num_bins_x, ps.num_bins_y, ps.xl, ps.yl, ps.xh, ps.yh,
                                     device=cuda_device) as eng:
            eng.set_initial_density(f(ps.initial_density_norm()))
            dens = eng.forward(cells)["density"].cpu().numpy()
            S = eng.fixed_point_bits
        g = oracle.Geometry(ps.num_bins_x, ps.num_bins_y, ps.xl, ps.yl, ps.xh, ps.yh)
        xc, yc = x.cpu().numpy(), y.cpu().numpy()
        oc = oracle.Cells(xc, yc, ps.size_x_clamped, ps.size_y_clamped, ps.offset_x, ps.offset_y, ps.ratio,
                          ranges=ps.ranges)
        grid, _ = oracle.density_fixed(oc, g, S, nthreads=4)
        rho, _ = oracle.fixed_to_density(grid, g, S, ps.initial_density_norm())
        np.testing.assert_array_equal(dens, rho)
        checks.append(float(np.abs(xc - p.x).max()))
    assert checks[0] > 0 and checks[1] > checks[0] * 0   # cells moved in the first stage


@pytest.mark.gpu
def test_command_line_writes_reference_outputs(cuda_device, tmp_path):
    from dreamplacett_framework_b200 import global_place
    cfg = dict(aux_input="", gpu=0, num_bins_x=128, num_bins_y=128, target_density=1.0, density_weight=8e-5,
               gamma=4.0, stop_overflow=0.0, ignore_net_degree=100,
               global_place_stages=[dict(num_bins_x=128, num_bins_y=128, iteration=5, learning_rate=0.01,
                                         wirelength="weighted_average", optimizer="nesterov")])
    path = tmp_path / "cfg.json"
    path.write_text(json.dumps(cfg))
    out = tmp_path / "res"
    global_place.main(["--benchmark", str(path), "--synthetic", "c1", "--scale", "0.02", "--results-dir", str(out)])
    m = json.loads((out / "synthetic_c1_b200_metrics.json").read_text())
    assert m["n_ep_calls"] == 5 and m["hpwl"] > 0 and m["ep_median_ms"] > 0
    lines = (out / "synthetic_c1_b200_iters.csv").read_text().splitlines()
    assert lines[0].split(",")[:4] == ["stage", "iteration", "num_bins_x", "num_bins_y"] and len(lines) == 6
