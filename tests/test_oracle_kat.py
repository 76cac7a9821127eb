"""Known-answer and property tests of the CPU oracle (no GPU)."""
import math

import numpy as np
import pytest


def _geom(o, M=16, N=16, die=160.0):
    return o.Geometry(M, N, 0.0, 0.0, die, die)


def _density(o, g, x, y, sx, sy, ratio=None, init=None):
    c = o.Cells(np.array(x, np.float32), np.array(y, np.float32), np.array(sx, np.float32),
                np.array(sy, np.float32), ratio=None if ratio is None else np.array(ratio, np.float32))
    S = g.default_fixed_bits()
    grid, bad = o.density_fixed(c, g, S)
    rho, sat = o.fixed_to_density(grid, g, S, init)
    return rho, grid, bad


def test_cell_inside_one_bin(oracle):
    g = _geom(oracle)
    rho, _, _ = _density(oracle, g, [12.0], [33.0], [5.0], [4.0])
    nz = np.argwhere(rho != 0)
    assert nz.tolist() == [[1, 3]]
    assert rho[1, 3] == np.float32(20.0 / 100.0)


def test_cell_straddles_four_bins(oracle):
    g = _geom(oracle)
    rho, _, _ = _density(oracle, g, [15.0], [25.0], [10.0], [10.0])
    assert np.argwhere(rho != 0).tolist() == [[1, 2], [1, 3], [2, 2], [2, 3]]
    np.testing.assert_array_equal(rho[1:3, 2:4], np.full((2, 2), 0.25, np.float32))


def test_exact_edges(oracle):
    # [10, 20) covers bin 1 exactly; bin 2 starts at the cell's right edge
    assert oracle.bin_range(10.0, 10.0, 0.0, 10.0, 16) == (1, 2)
    g = _geom(oracle)
    rho, _, _ = _density(oracle, g, [10.0], [20.0], [10.0], [10.0])
    assert np.argwhere(rho != 0).tolist() == [[1, 2]]
    assert rho[1, 2] == 1.0


def test_die_boundary_clamp(oracle):
    g = _geom(oracle)
    # partly left of the die, partly above the top, and entirely outside
    rho, _, bad = _density(oracle, g, [-5.0, 155.0, 200.0], [0.0, 157.0, 10.0], [10.0, 10.0, 5.0], [10.0, 10.0, 5.0])
    assert bad == 0
    assert rho[0, 0] == np.float32(0.5)                 # 5 x 10 inside bin (0, 0)
    assert rho[15, 15] == np.float32(5.0 * 3.0 / 100)   # 5 x 3 inside the die
    assert np.count_nonzero(rho) == 2


def test_mass_is_area_times_ratio(oracle):
    rng = np.random.default_rng(3)
    g = oracle.Geometry(64, 32, 0.0, 0.0, 640.0, 640.0)
    n = 2000
    sx = rng.uniform(1, 40, n).astype(np.float32)
    sy = rng.uniform(1, 40, n).astype(np.float32)
    x = rng.uniform(0, 640 - sx).astype(np.float32)
    y = rng.uniform(0, 640 - sy).astype(np.float32)
    r = rng.uniform(0.1, 1.0, n).astype(np.float32)
    rho, _, _ = _density(oracle, g, x, y, sx, sy, ratio=r)
    mass = float(rho.astype(np.float64).sum()) * g.bin_area
    expect = float(np.sum(sx.astype(np.float64) * sy * r))
    assert abs(mass / expect - 1.0) < 1e-5


def test_nonfinite_and_empty_cells(oracle):
    g = _geom(oracle)
    rho, _, bad = _density(oracle, g, [np.nan, 10.0, 20.0, 30.0], [0.0, np.inf, 20.0, 30.0],
                           [5.0, 5.0, 0.0, 5.0], [5.0, 5.0, 5.0, -1.0])
    assert bad == 2
    assert np.count_nonzero(rho) == 0
    rho, _, bad = _density(oracle, g, [], [], [], [])
    assert bad == 0 and np.count_nonzero(rho) == 0


def test_initial_density_fold(oracle):
    g = _geom(oracle)
    init = np.random.default_rng(0).random((16, 16)).astype(np.float32)
    rho, _, _ = _density(oracle, g, [12.0], [33.0], [5.0], [4.0], init=init)
    expect = init.copy()
    expect[1, 3] = np.float32(0.2) + init[1, 3]
    np.testing.assert_array_equal(rho, expect)


def test_fixed_point_independent_of_threads(oracle):
    rng = np.random.default_rng(5)
    g = oracle.Geometry(128, 128, 0.0, 0.0, 1000.0, 1000.0)
    n = 20000
    c = oracle.Cells(rng.uniform(0, 990, n), rng.uniform(0, 990, n), rng.uniform(1, 30, n), rng.uniform(1, 30, n),
                     ratio=rng.uniform(0.2, 1, n))
    S = g.default_fixed_bits()
    a, _ = oracle.density_fixed(c, g, S, nthreads=1)
    b, _ = oracle.density_fixed(c, g, S, nthreads=4)
    np.testing.assert_array_equal(a, b)


def test_node_ranges_skip_terminals(oracle):
    g = _geom(oracle)
    x = np.array([12.0, 50.0, 90.0], np.float32)
    c_all = oracle.Cells(x, x, np.full(3, 5.0), np.full(3, 5.0))
    c_rng = oracle.Cells(x, x, np.full(3, 5.0), np.full(3, 5.0), ranges=((0, 1), (2, 3)))
    S = g.default_fixed_bits()
    ga, _ = oracle.density_fixed(c_all, g, S)
    gr, _ = oracle.density_fixed(c_rng, g, S)
    assert ga[5, 5] > 0 and gr[5, 5] == 0
    assert gr[1, 1] == ga[1, 1] and gr[9, 9] == ga[9, 9]


def test_dct_single_cosine_mode(oracle):
    M, N, u0, v0 = 32, 16, 5, 3
    k = np.arange(M)[:, None] + 0.5
    l = np.arange(N)[None, :] + 0.5
    rho = np.cos(math.pi * u0 * k / M) * np.cos(math.pi * v0 * l / N)
    sol = oracle.solve_fft(rho, 1.0, 1.0)
    auv = sol["auv"]
    assert abs(auv[u0, v0] - 1.0) < 1e-12
    auv[u0, v0] = 0.0
    assert np.max(np.abs(auv)) < 1e-12
    # potential of a single mode is rho scaled by 4/(wu^2 + wv^2) (IDCT of DCT2 doubles per axis)
    wu = 2 * math.pi * u0 / M
    wv = 2 * math.pi * v0 / N
    np.testing.assert_allclose(sol["potential"], rho * 4.0 / (wu * wu + wv * wv), rtol=1e-10, atol=1e-12)


def test_field_is_minus_gradient_of_potential(oracle):
    M, N = 16, 32
    rho = np.random.default_rng(1).random((M, N))
    sol = oracle.solve_matrix(rho, 1.0, 1.0)
    c = np.where(np.arange(M) == 0, 1.0, 2.0)
    k = np.arange(M)[:, None] + 0.5
    u = np.arange(M)[None, :]
    d_idct = -(np.pi * u / M) * np.sin(np.pi * u * k / M) * c[None, :]
    _, _, inv = oracle.weights(M, N, 1.0, 1.0)
    dphi = d_idct @ (sol["auv"] * inv) @ oracle.build_idct(N).T
    assert oracle.rel_linf(sol["field_x"], -dphi) < 1e-12


def test_spectral_energy_identity(oracle):
    M, N = 32, 64
    rho = np.random.default_rng(2).random((M, N))
    sol = oracle.solve_fft(rho, 1.0, 2.0)
    _, _, inv = oracle.weights(M, N, 1.0, 2.0)
    cu = np.where(np.arange(M) == 0, 1.0, 2.0)[:, None]
    cv = np.where(np.arange(N) == 0, 1.0, 2.0)[None, :]
    e = M * N / 4.0 * np.sum(cu * cv * inv * sol["auv"] ** 2)
    assert abs(e / sol["energy"] - 1.0) < 1e-12


def test_mirror_symmetry(oracle):
    M, N = 32, 32
    rho = np.random.default_rng(4).random((M, N))
    a = oracle.solve_fft(rho, 1.0, 1.0)
    b = oracle.solve_fft(rho[::-1, :], 1.0, 1.0)
    np.testing.assert_allclose(b["field_x"], -a["field_x"][::-1, :], atol=1e-12)
    np.testing.assert_allclose(b["field_y"], a["field_y"][::-1, :], atol=1e-12)
    np.testing.assert_allclose(b["potential"], a["potential"][::-1, :], atol=1e-12)


def test_gather_matches_python_loop(oracle):
    rng = np.random.default_rng(6)
    g = oracle.Geometry(16, 16, 0.0, 0.0, 160.0, 160.0)
    n = 50
    x = rng.uniform(0, 140, n).astype(np.float32)
    y = rng.uniform(0, 140, n).astype(np.float32)
    sx = rng.uniform(1, 20, n).astype(np.float32)
    sy = rng.uniform(1, 20, n).astype(np.float32)
    r = rng.uniform(0.2, 1, n).astype(np.float32)
    fx = rng.standard_normal((16, 16)).astype(np.float32)
    fy = rng.standard_normal((16, 16)).astype(np.float32)
    gx, gy = oracle.gather(oracle.Cells(x, y, sx, sy, ratio=r), g, fx, fy, grad_out=2.0)
    for i in range(n):
        ax = ay = 0.0
        for kx in range(16):
            ox = max(0.0, min(x[i] + sx[i], (kx + 1) * 10.0) - max(x[i], kx * 10.0))
            for ky in range(16):
                oy = max(0.0, min(y[i] + sy[i], (ky + 1) * 10.0) - max(y[i], ky * 10.0))
                ax += ox * oy * fx[kx, ky]
                ay += ox * oy * fy[kx, ky]
        assert gx[i] == pytest.approx(-2.0 * r[i] * ax, rel=1e-5, abs=1e-4)
        assert gy[i] == pytest.approx(-2.0 * r[i] * ay, rel=1e-5, abs=1e-4)
