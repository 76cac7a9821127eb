"""CPU oracle for the electric-potential step.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by __graft_entry__.smoke() and
by bench.py's cpu_baseline / --impl reference legs, as the checker and as the
timed CPU baseline.  The product package never imports it.

Density and gather come from the C restatement in oracle/epb_oracle.c (loaded
with ctypes).  The DCT Poisson chain is restated here in float64 numpy, two
ways that must agree:

* ``solve_matrix``: the reference's dense matrix chain,
  host/density_scatter_ttnn_server_host.cpp:124-181 (matrix builders),
  :252-263 (wu/wv eigenvalue weights) and :281-295 (the six matmuls):
      auv = DCT_M rho DCT_N^T
      fx  = (2 IDXST_M) (auv * wu) IDCT_N^T
      fy  = (2 IDCT_M)  (auv * wv) IDXST_N^T
  built in float64 instead of the reference's float32 copies.
* ``solve_fft``: the same chain through scipy.fft (pocketfft) DCT-II/DCT-III/
  DST-III with the scale factors that reproduce the matrices above.

The potential and energy are not computed by the reference's TT path
(integration/scatter_ttnn_client.py:860 returns 0).  They follow DREAMPlace's
form (argument names inv_wu2_plus_wv2 / idct2 at
integration/scatter_ttnn_client.py:569-572):
      phi = IDCT_M (auv * inv_wu2_plus_wv2) IDCT_N^T,   energy = sum(rho * phi)
with the IDCT matrices of the field chain, so that -d(phi)/d(bin) equals the
field chain's fx and fy.
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libepb_oracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)


def lib():
    """Load liboracle (built by oracle/build_oracle.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            raise RuntimeError(f"oracle library missing: {_LIB_PATH}; run oracle/build_oracle.py")
        L = ctypes.CDLL(_LIB_PATH)
        cell_args = [_f32p] * 7 + [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int] + [ctypes.c_float] * 4
        L.ora_density_fixed.argtypes = cell_args + [ctypes.c_int, _i64p, ctypes.c_int, _i64p]
        L.ora_density_fixed.restype = ctypes.c_int64
        L.ora_density_f64.argtypes = cell_args + [_f64p]
        L.ora_density_f64.restype = ctypes.c_int64
        L.ora_fixed_to_density.argtypes = [_i64p, _f32p, ctypes.c_int64, ctypes.c_double, _f32p]
        L.ora_fixed_to_density.restype = ctypes.c_int64
        L.ora_gather.argtypes = cell_args + [_f32p, _f32p, ctypes.c_double, _f32p, _f32p, ctypes.c_int]
        L.ora_gather.restype = ctypes.c_int64
        L.ora_bin_range.argtypes = [ctypes.c_float] * 4 + [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
        L.ora_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


class Geometry:
    """Die and bin geometry.  bin sizes are fp32 as the reference server
    computes them: (xh - xl) / M (host/density_scatter_ttnn_server_host.cpp:411)."""

    def __init__(self, M, N, xl, yl, xh, yh):
        self.M, self.N = int(M), int(N)
        self.xl, self.yl, self.xh, self.yh = float(xl), float(yl), float(xh), float(yh)
        self.bsx = float(np.float32(np.float32(xh) - np.float32(xl)) / np.float32(M))
        self.bsy = float(np.float32(np.float32(yh) - np.float32(yl)) / np.float32(N))
        self.bsx = float(np.float32(self.bsx))
        self.bsy = float(np.float32(self.bsy))

    @property
    def bin_area(self):
        return float(self.bsx) * float(self.bsy)

    def default_fixed_bits(self):
        """Fraction bits S: keep enough integer bits for twice the die area in
        one bin, at least 32; the rest of a signed 63-bit word is fraction."""
        area = (self.xh - self.xl) * (self.yh - self.yl)
        ibits = max(int(math.ceil(math.log2(max(area, 1.0)))) + 1, 32)
        return 63 - ibits

    def density_scale(self, S):
        return math.ldexp(1.0, -S) / self.bin_area


class Cells:
    """Scattered cells in DREAMPlace's node layout: node arrays plus up to two
    node ranges (movable, fillers).  offset/ratio may be None."""

    def __init__(self, x, y, size_x, size_y, offset_x=None, offset_y=None, ratio=None,
                 ranges=None):
        f = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
        self.x, self.y, self.size_x, self.size_y = f(x), f(y), f(size_x), f(size_y)
        self.offset_x, self.offset_y, self.ratio = f(offset_x), f(offset_y), f(ratio)
        n = len(self.x)
        if ranges is None:
            ranges = ((0, n), (0, 0))
        (self.b0, self.e0), (self.b1, self.e1) = ranges

    @property
    def count(self):
        return (self.e0 - self.b0) + (self.e1 - self.b1)

    def nodes(self):
        return np.concatenate([np.arange(self.b0, self.e0), np.arange(self.b1, self.e1)]).astype(np.int64)

    def _args(self, g: Geometry):
        return ([_fp(self.x), _fp(self.y), _fp(self.size_x), _fp(self.size_y),
                 _fp(self.offset_x), _fp(self.offset_y), _fp(self.ratio),
                 self.b0, self.e0, self.b1, self.e1, g.M, g.N,
                 g.xl, g.yl, g.bsx, g.bsy])


def density_fixed(cells: Cells, g: Geometry, S: int, nthreads: int = 1, ws=None):
    """int64 fixed-point density grid [M, N] and the count of skipped cells."""
    grid = np.empty((g.M, g.N), dtype=np.int64)
    nthreads = max(1, int(nthreads))
    if nthreads > 1 and ws is None:
        ws = np.empty((nthreads - 1) * g.M * g.N, dtype=np.int64)
    wsp = ws.ctypes.data_as(_i64p) if (ws is not None and nthreads > 1) else None
    bad = lib().ora_density_fixed(*cells._args(g), int(S), grid.ctypes.data_as(_i64p), nthreads, wsp)
    return grid, int(bad)


def density_f64(cells: Cells, g: Geometry):
    grid = np.empty((g.M, g.N), dtype=np.float64)
    lib().ora_density_f64(*cells._args(g), grid.ctypes.data_as(_f64p))
    return grid


def fixed_to_density(grid, g: Geometry, S: int, init_norm=None):
    """Normalised fp32 density rho = fp32(q * 2^-S / bin_area) + init_norm."""
    rho = np.empty((g.M, g.N), dtype=np.float32)
    init = None if init_norm is None else np.ascontiguousarray(init_norm, dtype=np.float32)
    sat = lib().ora_fixed_to_density(np.ascontiguousarray(grid).ctypes.data_as(_i64p), _fp(init),
                                     g.M * g.N, g.density_scale(S), _fp(rho))
    return rho, int(sat)


def gather(cells: Cells, g: Geometry, field_x, field_y, grad_out=1.0, nthreads=1,
           grad_x=None, grad_y=None):
    """Per-node gradient -grad_out*ratio*sum(area*field) (fp64 accumulation)."""
    nn = len(cells.x)
    gx = np.zeros(nn, np.float32) if grad_x is None else grad_x
    gy = np.zeros(nn, np.float32) if grad_y is None else grad_y
    fx = np.ascontiguousarray(field_x, dtype=np.float32)
    fy = np.ascontiguousarray(field_y, dtype=np.float32)
    lib().ora_gather(*cells._args(g), _fp(fx), _fp(fy), float(grad_out), _fp(gx), _fp(gy), int(nthreads))
    return gx, gy


def bin_range(v, s, origin, bs, nb):
    lo, hi = ctypes.c_int(), ctypes.c_int()
    lib().ora_bin_range(v, s, origin, bs, nb, ctypes.byref(lo), ctypes.byref(hi))
    return lo.value, hi.value


# --------------------------------------------------------------------------
# DCT chain (float64)
# --------------------------------------------------------------------------

def build_dct2(N):
    """host/density_scatter_ttnn_server_host.cpp:124-131: (2/N) cos(pi k (n+1/2) / N)."""
    k = np.arange(N, dtype=np.float64)[:, None]
    n = np.arange(N, dtype=np.float64)[None, :]
    return (2.0 / N) * np.cos(np.pi * k * (n + 0.5) / N)


def build_idct(N):
    """host/density_scatter_ttnn_server_host.cpp:143-152: m[k,0]=1, m[k,n]=2cos(pi n (k+1/2)/N)."""
    k = np.arange(N, dtype=np.float64)[:, None]
    n = np.arange(N, dtype=np.float64)[None, :]
    m = 2.0 * np.cos(np.pi * n * (k + 0.5) / N)
    m[:, 0] = 1.0
    return m


def build_idxst(N):
    """host/density_scatter_ttnn_server_host.cpp:164-171: sin(pi n (k+1/2) / N)."""
    k = np.arange(N, dtype=np.float64)[:, None]
    n = np.arange(N, dtype=np.float64)[None, :]
    return np.sin(np.pi * n * (k + 0.5) / N)


def weights(M, N, bsx, bsy):
    """Eigenvalue weights, host/density_scatter_ttnn_server_host.cpp:252-263
    (wu/wv: w/(wu^2+wv^2)/2, zero at (0,0)) plus DREAMPlace's
    inv_wu2_plus_wv2 (1/(wu^2+wv^2), zero at (0,0))."""
    ratio = float(np.float32(np.float32(bsx) / np.float32(bsy)))
    wu = (2.0 * np.pi * np.arange(M, dtype=np.float64) / M)[:, None]
    wv = (2.0 * np.pi * np.arange(N, dtype=np.float64) / N * ratio)[None, :]
    d = wu * wu + wv * wv
    d[0, 0] = 1.0
    inv = 1.0 / d
    inv[0, 0] = 0.0
    wu_half = wu * inv * 0.5
    wv_half = wv * inv * 0.5
    return wu_half, wv_half, inv


def solve_matrix(rho, bsx, bsy):
    """Dense float64 matrix chain (reference TTNNDCTSolver::solve)."""
    rho = np.asarray(rho, dtype=np.float64)
    M, N = rho.shape
    wu, wv, inv = weights(M, N, bsx, bsy)
    auv = build_dct2(M) @ rho @ build_dct2(N).T
    fx = (2.0 * build_idxst(M)) @ (auv * wu) @ build_idct(N).T
    fy = (2.0 * build_idct(M)) @ (auv * wv) @ build_idxst(N).T
    phi = build_idct(M) @ (auv * inv) @ build_idct(N).T
    energy = float(np.sum(rho * phi))
    return dict(auv=auv, field_x=fx, field_y=fy, potential=phi, energy=energy)


def _dct2(a, axis, workers):
    import scipy.fft as sf
    return sf.dct(a, type=2, axis=axis, workers=workers) / a.shape[axis]


def _idct(a, axis, workers):
    import scipy.fft as sf
    return sf.dct(a, type=3, axis=axis, workers=workers)


def _idxst(a, axis, workers):
    import scipy.fft as sf
    a = np.moveaxis(a, axis, -1)
    b = np.zeros_like(a)
    b[..., :-1] = a[..., 1:]
    y = 0.5 * sf.dst(b, type=3, axis=-1, workers=workers)
    return np.moveaxis(y, -1, axis)


def solve_fft(rho, bsx, bsy, workers=1, dtype=np.float64):
    """Same chain via scipy.fft; dtype float64 for the oracle, float32 is
    allowed for the timed CPU baseline."""
    rho = np.asarray(rho, dtype=dtype)
    M, N = rho.shape
    wu, wv, inv = (w.astype(dtype) for w in weights(M, N, bsx, bsy))
    auv = _dct2(_dct2(rho, 0, workers), 1, workers)
    fx = 2.0 * _idxst(_idct(auv * wu, 1, workers), 0, workers)
    fy = 2.0 * _idct(_idxst(auv * wv, 1, workers), 0, workers)
    phi = _idct(_idct(auv * inv, 1, workers), 0, workers)
    energy = float(np.sum(rho.astype(np.float64) * phi.astype(np.float64)))
    return dict(auv=auv, field_x=fx, field_y=fy, potential=phi, energy=energy)


def rel_linf(a, b):
    """max|a-b| / max|b| (the north star's relative L-infinity)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = float(np.max(np.abs(b))) if b.size else 0.0
    num = float(np.max(np.abs(a - b))) if b.size else 0.0
    return num / den if den > 0 else num


def electric_potential(cells: Cells, g: Geometry, S: int, init_norm=None, nthreads=1,
                       workers=1, method="fft"):
    """Whole oracle step: fixed density -> rho -> DCT chain -> gradients."""
    grid, bad = density_fixed(cells, g, S, nthreads=nthreads)
    rho, sat = fixed_to_density(grid, g, S, init_norm)
    if method == "fft":
        sol = solve_fft(rho, g.bsx, g.bsy, workers)
    else:
        sol = solve_matrix(rho, g.bsx, g.bsy)
    fx32 = sol["field_x"].astype(np.float32)
    fy32 = sol["field_y"].astype(np.float32)
    gx, gy = gather(cells, g, fx32, fy32, 1.0, nthreads=nthreads)
    sol.update(grid=grid, density=rho, grad_x=gx, grad_y=gy, bad=bad, saturated=sat)
    return sol


# --------------------------------------------------------------------------
# Global-placement loop pieces (the operator's callers)
# --------------------------------------------------------------------------

def overflow(cells: Cells, g: Geometry, S: int, init_norm=None, target=1.0, nthreads=1):
    """(bin_area * sum_b max(rho_b - target, 0), max_b rho_b) of the cells'
    fixed-point density map plus the initial density, in float64.

    DREAMPlace's ElectricOverflow (not in the reference tree; the reference
    reads its result per iteration in integration/run_dreamplace.py:333-370)
    sums relu(density_map - target * bin_area) over bins; in normalised units
    that is bin_area * sum relu(rho - target)."""
    grid, _ = density_fixed(cells, g, S, nthreads=nthreads)
    rho, _ = fixed_to_density(grid, g, S, init_norm)
    ex = rho.astype(np.float64) - float(np.float32(target))
    return float(np.sum(np.maximum(ex, 0.0))) * g.bin_area, float(rho.max())


def descent_step(x, y, grad_x, grad_y, width, height, nodes, g: Geometry, step_bins=0.5):
    """One normalised density-descent step in place (fp32, one rounding per
    operation, as epb_descent_step):
        linf = max over nodes of max(|gx|, |gy|) (finite gradients only)
        x <- max(min(x - (step_bins*bsx / linf) * gx, xh - w), xl), same for y.
    Returns linf (float32)."""
    f32 = np.float32
    gx, gy = grad_x[nodes], grad_y[nodes]
    ok = np.isfinite(gx) & np.isfinite(gy)
    linf = f32(0.0)
    if ok.any():
        linf = f32(max(np.max(np.abs(gx[ok])), np.max(np.abs(gy[ok]))))
    if not linf > 0:
        return linf
    sx = f32(f32(step_bins) * f32(g.bsx)) / linf
    sy = f32(f32(step_bins) * f32(g.bsy)) / linf
    n = nodes[ok]
    nx = x[n] - sx * grad_x[n]
    ny = y[n] - sy * grad_y[n]
    nx = np.maximum(np.minimum(nx, f32(g.xh) - width[n]), f32(g.xl))
    ny = np.maximum(np.minimum(ny, f32(g.yh) - height[n]), f32(g.yl))
    x[n] = nx.astype(np.float32)
    y[n] = ny.astype(np.float32)
    return linf


def descent_trajectory(x, y, size_x, size_y, size_x_clamped, size_y_clamped, offset_x, offset_y, ratio,
                       ranges, movable_range, g: Geometry, S: int, init_norm=None, steps=200, step_bins=0.5,
                       target=1.0, lam0=8e-5, lam_every=50, nthreads=1, workers=1, solve_dtype=np.float64):
    """The benchmark's density-only placement loop (config C5) on the CPU.

    Per step t: electric-potential forward + backward of every scattered cell,
    the overflow of the movable cells, then one normalised descent step of all
    scattered cells; lambda_t = lam0 * 2^(t // lam_every) scales the reported
    objective lambda_t * energy (it cancels in the normalised step).  Returns
    per-step arrays (overflow ratio, max density, energy, objective, linf) and
    the final positions; overflow has steps + 1 entries (the last one after
    the final step)."""
    x = np.array(x, dtype=np.float32, copy=True)
    y = np.array(y, dtype=np.float32, copy=True)
    (m0, m1) = movable_range
    mov_area = float(np.sum(size_x[m0:m1].astype(np.float64) * size_y[m0:m1].astype(np.float64)))
    ovf = np.zeros(steps + 1)
    maxd = np.zeros(steps + 1)
    energy = np.zeros(steps)
    objective = np.zeros(steps)
    linf = np.zeros(steps, dtype=np.float32)
    for t in range(steps + 1):
        mov = Cells(x, y, size_x_clamped, size_y_clamped, offset_x, offset_y, ratio, ranges=((m0, m1), (0, 0)))
        a, mx = overflow(mov, g, S, init_norm, target, nthreads)
        ovf[t], maxd[t] = a / mov_area, mx
        if t == steps:
            break
        cells = Cells(x, y, size_x_clamped, size_y_clamped, offset_x, offset_y, ratio, ranges=ranges)
        grid, _ = density_fixed(cells, g, S, nthreads=nthreads)
        rho, _ = fixed_to_density(grid, g, S, init_norm)
        sol = solve_fft(rho, g.bsx, g.bsy, workers, dtype=solve_dtype)
        gx, gy = gather(cells, g, sol["field_x"].astype(np.float32), sol["field_y"].astype(np.float32), 1.0,
                        nthreads=nthreads)
        energy[t] = sol["energy"]
        objective[t] = lam0 * 2.0 ** (t // lam_every) * sol["energy"]
        linf[t] = descent_step(x, y, gx, gy, size_x, size_y, cells.nodes(), g, step_bins)
    return dict(overflow=ovf, max_density=maxd, energy=energy, objective=objective, linf=linf, x=x, y=y)
