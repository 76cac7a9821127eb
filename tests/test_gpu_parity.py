"""Parity of the CUDA engine (through the C ABI) with the CPU oracle.

Bars (the north star's):
* fixed-point density grid: bit-exact (integer equality);
* normalised density map: bit-exact (same IEEE operations on both sides);
* potential, fields, energy: 1e-5 relative L-infinity against the float64 oracle;
* per-cell gradients: 1e-5 relative L-infinity against the float64-accumulating
  oracle gather on the same field maps, and end to end.
"""
import numpy as np
import pytest
import torch

from dreamplacett_framework_b200 import synth
from dreamplacett_framework_b200.engine import CellTensors, ElectricPotentialEngine
from dreamplacett_framework_b200 import _lib

from gpu_util import engine_for, geometry_for, np_, placement_cells, to_device, to_oracle

pytestmark = pytest.mark.gpu

TOL_FP = 1e-5  # relative L-inf for potential / fields / energy / gradients


# ---------------------------------------------------------------- density

def test_golden_cases_scatter_bit_exact(cuda_device, oracle, golden_density):
    d = golden_density
    for i in range(int(d["num_density_cases"])):
        M, N = int(d[f"case{i}_M"]), int(d[f"case{i}_N"])
        g = oracle.Geometry(M, N, 0.0, 0.0, float(d[f"case{i}_xh"]), float(d[f"case{i}_yh"]))
        arrs = dict(x=d[f"case{i}_px"], y=d[f"case{i}_py"], size_x=d[f"case{i}_sx"], size_y=d[f"case{i}_sy"])
        n = len(arrs["x"])
        cells = to_device(arrs, ((0, n), (0, 0)), cuda_device)
        with ElectricPotentialEngine(M, N, 0.0, 0.0, g.xh, g.yh, device=cuda_device) as eng:
            grid = np_(eng.scatter_fixed(cells))
            ref, _ = oracle.density_fixed(to_oracle(oracle, arrs, ((0, n), (0, 0))), g, eng.fixed_point_bits)
            np.testing.assert_array_equal(grid, ref)
            out = eng.forward(cells)
            rho_ref, _ = oracle.fixed_to_density(ref, g, eng.fixed_point_bits)
            np.testing.assert_array_equal(np_(out["density"]), rho_ref)
            # and against the reference's own fp32 density oracle (client:55-93)
            assert oracle.rel_linf(np_(out["density"]), d[f"case{i}_client_fp32"]) < 2e-6


@pytest.mark.parametrize("config", ["c1", "c2", "c3"])
def test_full_config_scatter_bit_exact(cuda_device, oracle, config):
    p = synth.make_placement(config)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    g = geometry_for(oracle, p)
    with engine_for(p, cuda_device) as eng:
        grid = np_(eng.scatter_fixed(cells))
        ref, bad = oracle.density_fixed(to_oracle(oracle, arrs, ranges), g, eng.fixed_point_bits, nthreads=4)
        assert bad == 0
        np.testing.assert_array_equal(grid, ref)
        init = p.initial_density_norm()
        eng.set_initial_density(torch.from_numpy(init).to(cuda_device))
        out = eng.forward(cells)
        rho_ref, sat = oracle.fixed_to_density(ref, g, eng.fixed_point_bits, init)
        assert sat == 0
        np.testing.assert_array_equal(np_(out["density"]), rho_ref)
        assert eng.error_flags() == 0


def test_scatter_deterministic_run_to_run(cuda_device):
    p = synth.make_placement("c2", scale=0.5)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    with engine_for(p, cuda_device) as eng:
        outs = [eng.forward(cells) for _ in range(3)]
        for o in outs[1:]:
            for k in ("density", "potential", "field_x", "field_y", "energy"):
                assert torch.equal(o[k], outs[0][k]), k


def test_atomic_probe_leaves_the_grid_zeroed(cuda_device):
    """The bench's atomic-rate probe writes the engine's own grid: a forward
    after it gives the same bits as one before it, and bad sizes are refused."""
    p = synth.make_placement("c1", scale=0.2)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    with engine_for(p, cuda_device) as eng:
        before = eng.forward(cells)
        ms = eng.atomic_probe(200000, 2, 3)
        assert ms > 0.0
        after = eng.forward(cells)
        for k in ("density", "potential", "field_x", "field_y", "energy"):
            assert torch.equal(after[k], before[k]), k
        for args in ((-1, 2, 2), (10, 0, 2), (10, 2, 9)):
            with pytest.raises(_lib.EpbError):
                eng.atomic_probe(*args)


# ---------------------------------------------------------------- DCT solve

@pytest.mark.parametrize("M,N", [(16, 16), (32, 64), (64, 16), (128, 128), (256, 512), (512, 512),
                                 (1024, 256), (1024, 1024), (2048, 2048), (4096, 4096), (16, 4096)])
def test_dct_solve_matches_oracle(cuda_device, oracle, M, N):
    rng = np.random.default_rng(M * 7 + N)
    # a density-like map: positive, with structure at all scales
    rho = (rng.random((M, N)) * 0.5 + 0.75).astype(np.float32)
    rho[M // 4:M // 2, N // 3:N // 2] += 2.0
    bsx, bsy = 10.0, 10.0 * (N / M) ** 0  # square bins
    with ElectricPotentialEngine(M, N, 0.0, 0.0, bsx * M, bsy * N, device=cuda_device) as eng:
        res = eng.dct_solve(torch.from_numpy(rho).to(cuda_device))
        ref = oracle.solve_fft(rho, eng.bin_size_x, eng.bin_size_y, workers=4)
    for k in ("potential", "field_x", "field_y"):
        err = oracle.rel_linf(np_(res[k]), ref[k])
        assert err < TOL_FP, (k, err)
    assert abs(float(res["energy"].item()) / ref["energy"] - 1.0) < TOL_FP


def test_dct_solve_anisotropic_bins(cuda_device, oracle):
    M, N = 256, 128
    rho = np.random.default_rng(9).random((M, N)).astype(np.float32)
    with ElectricPotentialEngine(M, N, 0.0, 0.0, 2560.0, 640.0, device=cuda_device) as eng:
        assert eng.bin_size_x != eng.bin_size_y
        res = eng.dct_solve(torch.from_numpy(rho).to(cuda_device))
        ref = oracle.solve_fft(rho, eng.bin_size_x, eng.bin_size_y)
    for k in ("potential", "field_x", "field_y"):
        assert oracle.rel_linf(np_(res[k]), ref[k]) < TOL_FP, k


def test_dct_golden_reference_chain(cuda_device, oracle, golden_dct):
    t = golden_dct
    for j in range(int(t["num_dct_cases"])):
        M, N = (int(v) for v in t[f"s{j}_shape"])
        bsx, bsy = (float(v) for v in t[f"s{j}_bins"])
        if M < 16 or N < 16:
            continue  # the engine's smallest transform is 16
        with ElectricPotentialEngine(M, N, 0.0, 0.0, bsx * M, bsy * N, device=cuda_device) as eng:
            res = eng.dct_solve(torch.from_numpy(t[f"s{j}_rho"]).to(cuda_device))
        # the golden chain used the reference's fp32 matrices: 1e-6 of their own rounding
        assert oracle.rel_linf(np_(res["field_x"]), t[f"s{j}_field_x"]) < TOL_FP + 1e-6
        assert oracle.rel_linf(np_(res["field_y"]), t[f"s{j}_field_y"]) < TOL_FP + 1e-6


# ---------------------------------------------------------------- gather

def test_gather_matches_oracle(cuda_device, oracle):
    p = synth.make_placement("c3", scale=0.2)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    g = geometry_for(oracle, p)
    rng = np.random.default_rng(1)
    fx = rng.standard_normal((p.num_bins_x, p.num_bins_y)).astype(np.float32)
    fy = rng.standard_normal((p.num_bins_x, p.num_bins_y)).astype(np.float32)
    gout = torch.tensor([0.75], device=cuda_device)
    with engine_for(p, cuda_device) as eng:
        gx, gy = eng.gather(cells, torch.from_numpy(fx).to(cuda_device), torch.from_numpy(fy).to(cuda_device),
                            grad_out=gout)
    rx, ry = oracle.gather(to_oracle(oracle, arrs, ranges), g, fx, fy, grad_out=0.75, nthreads=4)
    assert oracle.rel_linf(np_(gx), rx) < TOL_FP
    assert oracle.rel_linf(np_(gy), ry) < TOL_FP
    # terminals (outside both ranges) are untouched (zeros from allocation)
    t0, t1 = p.num_movable, p.num_movable + p.num_terminals
    assert torch.count_nonzero(gx[t0:t1]) == 0


# ---------------------------------------------------------------- end to end

@pytest.mark.parametrize("config,scale", [("c1", 1.0), ("c2", 1.0), ("c3", 1.0), ("c4", 1.0)])
def test_forward_backward_end_to_end(cuda_device, oracle, config, scale):
    """Every BASELINE config at full size: C1 (512^2), C2 (2048^2, clustered),
    C3 (2048^2, 1.4M cells) and C4 (4096^2, 2.5M cells, 2000 macros)."""
    p = synth.make_placement(config, scale=scale)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    g = geometry_for(oracle, p)
    init = p.initial_density_norm()
    with engine_for(p, cuda_device) as eng:
        eng.set_initial_density(torch.from_numpy(init).to(cuda_device))
        out = eng.forward(cells)
        gx, gy = eng.backward(cells)
        S = eng.fixed_point_bits
    oc = to_oracle(oracle, arrs, ranges)
    grid, _ = oracle.density_fixed(oc, g, S, nthreads=4)
    rho, _ = oracle.fixed_to_density(grid, g, S, init)
    np.testing.assert_array_equal(np_(out["density"]), rho)
    ref = oracle.solve_fft(rho, g.bsx, g.bsy, workers=4)
    for k in ("potential", "field_x", "field_y"):
        err = oracle.rel_linf(np_(out[k]), ref[k])
        assert err < TOL_FP, (k, err)
    assert abs(float(out["energy"].item()) / ref["energy"] - 1.0) < TOL_FP
    # gradients: against the oracle gather of the float64 fields
    rx, ry = oracle.gather(oc, g, ref["field_x"].astype(np.float32), ref["field_y"].astype(np.float32), nthreads=4)
    assert oracle.rel_linf(np_(gx), rx) < TOL_FP
    assert oracle.rel_linf(np_(gy), ry) < TOL_FP


# ---------------------------------------------------------------- edge cases

def _small_engine(dev, M=64, N=64, die=640.0):
    return ElectricPotentialEngine(M, N, 0.0, 0.0, die, die, device=dev)


def test_empty_cells_give_initial_density_only(cuda_device):
    z = torch.empty(0, device=cuda_device)
    cells = CellTensors(z, z, z, z)
    init = torch.rand(64, 64, device=cuda_device)
    with _small_engine(cuda_device) as eng:
        eng.set_initial_density(init)
        out = eng.forward(cells)
        assert torch.equal(out["density"], init)
        gx, gy = eng.backward(cells)
        assert gx.numel() == 0


def test_nonfinite_cells_are_flagged_and_skipped(cuda_device, oracle):
    x = torch.tensor([10.0, float("nan"), 100.0, 200.0], device=cuda_device)
    y = torch.tensor([10.0, 50.0, float("inf"), 300.0], device=cuda_device)
    s = torch.full((4,), 12.0, device=cuda_device)
    with _small_engine(cuda_device) as eng:
        out = eng.forward(CellTensors(x, y, s, s))
        flags = eng.error_flags()
        assert flags & _lib.EPB_FLAG_NONFINITE_CELL
        assert eng.error_flags() == 0  # cleared
        ok = CellTensors(x[[0, 3]].contiguous(), y[[0, 3]].contiguous(), s[:2].contiguous(), s[:2].contiguous())
        ref = eng.forward(ok)
        assert torch.equal(out["density"], ref["density"])


def test_zero_size_and_offdie_cells_contribute_nothing(cuda_device):
    x = torch.tensor([10.0, 20.0, 1000.0, -100.0], device=cuda_device)
    y = torch.tensor([10.0, 20.0, 10.0, 10.0], device=cuda_device)
    sx = torch.tensor([0.0, 5.0, 5.0, 5.0], device=cuda_device)
    sy = torch.tensor([5.0, -1.0, 5.0, 5.0], device=cuda_device)
    with _small_engine(cuda_device) as eng:
        grid = eng.scatter_fixed(CellTensors(x, y, sx, sy))
        assert torch.count_nonzero(grid) == 0
        assert eng.error_flags() == 0


def test_saturation_is_reported(cuda_device):
    x = torch.tensor([10.0], device=cuda_device)
    s = torch.tensor([20.0], device=cuda_device)
    r = torch.tensor([1e30], device=cuda_device)
    with _small_engine(cuda_device) as eng:
        eng.forward(CellTensors(x, x, s, s, ratio=r))
        with pytest.raises(_lib.EpbError) as e:
            eng.error_flags()
        assert e.value.status == _lib.EPB_EOVERFLOW
        assert eng.error_flags() == 0


def test_backward_before_forward_and_bad_args(cuda_device):
    x = torch.zeros(3, device=cuda_device)
    with _small_engine(cuda_device) as eng:
        with pytest.raises(_lib.EpbError) as e:
            eng.backward(CellTensors(x, x, x, x))
        assert e.value.status == _lib.EPB_ENOSTATE
        with pytest.raises(ValueError):
            eng.forward(CellTensors(x, x, x, x, ranges=((0, 5), (0, 0))))
        with pytest.raises(ValueError):
            eng.forward(CellTensors(x.double(), x, x, x))


def test_grad_out_scaling_and_ranges(cuda_device):
    p = synth.make_placement("c3", scale=0.05)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    with engine_for(p, cuda_device) as eng:
        eng.forward(cells)
        g1x, g1y = eng.backward(cells)
        g2x, g2y = eng.backward(cells, grad_out=torch.tensor([2.0], device=cuda_device))
        torch.testing.assert_close(g2x, 2 * g1x, rtol=0, atol=0)
        sentinel = torch.full((p.num_nodes,), 7.0, device=cuda_device)
        gx, _ = eng.backward(cells, grad_x=sentinel.clone(), grad_y=sentinel.clone())
        t0, t1 = p.num_movable, p.num_movable + p.num_terminals
        assert torch.all(gx[t0:t1] == 7.0)


def test_multiple_engines_and_streams(cuda_device):
    p = synth.make_placement("c1", scale=0.2)
    arrs, ranges = placement_cells(p)
    cells = to_device(arrs, ranges, cuda_device)
    s = torch.cuda.Stream(cuda_device)
    with engine_for(p, cuda_device) as a, engine_for(p, cuda_device) as b:
        ra = a.forward(cells)
        s.wait_stream(torch.cuda.current_stream(cuda_device))
        with torch.cuda.stream(s):
            rb = b.forward(cells, stream=s)
        s.synchronize()
        assert torch.equal(ra["density"], rb["density"])
        assert torch.equal(ra["field_x"], rb["field_x"])


@pytest.mark.gpu
def test_host_buffer_entry_points(cuda_device):
    """epb_forward_host / epb_backward_host: positions read from pinned host
    memory by the scatter, gradients stored to it by the gather, results
    identical to the device entry points."""
    p = synth.make_placement("c3", scale=0.1, grid=512)
    arrs, ranges = placement_cells(p)
    with engine_for(p, cuda_device) as eng:
        eng.set_initial_density(torch.from_numpy(p.initial_density_norm()).to(cuda_device))
        cells = to_device(arrs, ranges, cuda_device)
        ref = {k: v.clone() for k, v in eng.forward(cells).items()}
        rgx, rgy = (t.clone() for t in eng.backward(cells))
        hx = torch.from_numpy(p.x.copy()).pin_memory()
        hy = torch.from_numpy(p.y.copy()).pin_memory()
        cells.x.zero_()
        cells.y.zero_()
        out = eng.forward_host(cells, hx, hy)
        hgx = torch.zeros(p.num_nodes).pin_memory()
        hgy = torch.zeros(p.num_nodes).pin_memory()
        gx, gy = eng.backward_host(cells, hgx, hgy)
        torch.cuda.synchronize(cuda_device)
        # the positions of the scattered nodes (not the terminals) are kept on the device
        (b0, e0), (b1, e1) = ranges
        for a, b in ((b0, e0), (b1, e1)):
            assert torch.equal(cells.x[a:b].cpu(), hx[a:b]) and torch.equal(cells.y[a:b].cpu(), hy[a:b])
        for k in ("density", "potential", "field_x", "field_y", "energy"):
            assert torch.equal(out[k], ref[k]), k
        assert torch.equal(gx, rgx) and torch.equal(gy, rgy)
        assert torch.equal(hgx, rgx.cpu()) and torch.equal(hgy, rgy.cpu())
        with pytest.raises(ValueError):
            eng.forward_host(cells, torch.zeros(p.num_nodes), hy)  # not pinned
