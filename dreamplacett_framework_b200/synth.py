"""Seeded synthetic placement inputs standing in for the ISPD-2005 designs.

The reference measures on ISPD-2005 bookshelf benchmarks through DREAMPlace
(benchmarks/configs/*.json); neither the design files nor DREAMPlace are
available, so these generators reproduce the BASELINE configurations' shapes,
sizes and distributions:

* movable standard cells: height 12, width clip(lognormal(ln 8, 0.5), 2, 80);
* fillers: 8 x 12;
* fixed macros: sides U[100, 800], non-overlapping by rejection sampling,
  rasterised once into the initial (fixed-cell) density map;
* positions: lower-left corners, uniform and/or Gaussian hotspots, clamped so
  every cell lies inside the die.

Nodes are laid out as DREAMPlace orders them, [movable | terminals | fillers],
and the electric-potential inputs follow DREAMPlace's ElectricPotential set-up
(tools/v13_offset_ratio_stats.py:54-67 of the reference restates it):
  size_clamped = max(size, sqrt(2) * bin_size)
  offset       = (size - size_clamped) / 2
  ratio        = size_x * size_y / (size_x_clamped * size_y_clamped)
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional

import numpy as np

CONFIGS: Dict[str, dict] = {
    # BASELINE.json configs[0..4]
    "c1": dict(die=10000.0, grid=512, movable=210_000, fillers=60_000, macros=0,
               hotspots=0, hot_frac=0.0, sigma=0.0, seed=0),
    "c2": dict(die=10000.0, grid=2048, movable=210_000, fillers=60_000, macros=0,
               hotspots=8, hot_frac=0.7, sigma=400.0, seed=1),
    "c3": dict(die=20000.0, grid=2048, movable=1_100_000, fillers=300_000, macros=1000,
               hotspots=16, hot_frac=0.5, sigma=800.0, seed=2),
    "c4": dict(die=40000.0, grid=4096, movable=2_000_000, fillers=500_000, macros=2000,
               hotspots=16, hot_frac=0.5, sigma=800.0, seed=3),
    "c5": dict(die=20000.0, grid=1024, movable=1_100_000, fillers=300_000, macros=0,
               hotspots=16, hot_frac=0.5, sigma=800.0, seed=4),
}


@dataclass
class Placement:
    """A synthetic design in DREAMPlace's node layout (all float32 numpy)."""
    name: str
    xl: float
    yl: float
    xh: float
    yh: float
    num_bins_x: int
    num_bins_y: int
    num_movable: int
    num_terminals: int
    num_filler: int
    x: np.ndarray            # lower-left x per node
    y: np.ndarray
    size_x: np.ndarray       # original sizes
    size_y: np.ndarray
    size_x_clamped: np.ndarray = field(default=None)
    size_y_clamped: np.ndarray = field(default=None)
    offset_x: np.ndarray = field(default=None)
    offset_y: np.ndarray = field(default=None)
    ratio: np.ndarray = field(default=None)
    initial_density_map: Optional[np.ndarray] = None   # fixed-cell overlap area per bin (area units)

    @property
    def num_nodes(self):
        return len(self.x)

    @property
    def bin_size_x(self):
        return float(np.float32(np.float32(self.xh) - np.float32(self.xl)) / np.float32(self.num_bins_x))

    @property
    def bin_size_y(self):
        return float(np.float32(np.float32(self.yh) - np.float32(self.yl)) / np.float32(self.num_bins_y))

    @property
    def ranges(self):
        """(movable, fillers) node ranges: terminals are skipped."""
        n = self.num_nodes
        return (0, self.num_movable), (n - self.num_filler, n)

    @property
    def num_cells(self):
        return self.num_movable + self.num_filler

    def initial_density_norm(self) -> np.ndarray:
        """initial_density_map / bin_area in fp32, as the reference client
        uploads it (integration/scatter_ttnn_client.py:792-794)."""
        ba = np.float32(self.bin_size_x * self.bin_size_y)
        if self.initial_density_map is None:
            return np.zeros((self.num_bins_x, self.num_bins_y), np.float32)
        return (self.initial_density_map.astype(np.float32) / ba).astype(np.float32)


    def regrid(self, num_bins_x: int, num_bins_y: int) -> "Placement":
        """The same design on another grid (a stage of multi-stage placement):
        stretched sizes, offsets, ratio and the fixed-cell density for those
        bins; the node arrays are shared."""
        import dataclasses
        q = dataclasses.replace(self, num_bins_x=int(num_bins_x), num_bins_y=int(num_bins_y))
        bsx, bsy = q.bin_size_x, q.bin_size_y
        q.size_x_clamped, q.size_y_clamped, q.offset_x, q.offset_y, q.ratio = stretch(q.size_x, q.size_y, bsx, bsy)
        t = slice(q.num_movable, q.num_movable + q.num_terminals)
        if q.num_terminals:
            q.initial_density_map = rasterise(q.x[t].astype(np.float64), q.y[t].astype(np.float64),
                                              q.size_x[t].astype(np.float64), q.size_y[t].astype(np.float64),
                                              q.xl, q.yl, bsx, bsy, q.num_bins_x, q.num_bins_y)
        else:
            q.initial_density_map = np.zeros((q.num_bins_x, q.num_bins_y), np.float64)
        return q


def center_init(p: "Placement", seed: int = 1000, spread: float = 0.001) -> "Placement":
    """Movable cells and fillers at the die centre with Gaussian noise of
    spread * die size (DREAMPlace's random_center_init_flag, the reference
    configs' default), clamped to the die; terminals stay.  In place."""
    rng = np.random.default_rng(seed)
    n = p.num_nodes
    mov = np.r_[0:p.num_movable, n - p.num_filler:n]
    cx, cy = 0.5 * (p.xl + p.xh), 0.5 * (p.yl + p.yh)
    w, h = p.size_x[mov], p.size_y[mov]
    x = cx - 0.5 * w + spread * (p.xh - p.xl) * rng.standard_normal(len(mov))
    y = cy - 0.5 * h + spread * (p.yh - p.yl) * rng.standard_normal(len(mov))
    p.x[mov] = np.clip(x, p.xl, p.xh - w).astype(np.float32)
    p.y[mov] = np.clip(y, p.yl, p.yh - h).astype(np.float32)
    return p


def stretch(size_x, size_y, bin_size_x, bin_size_y):
    """DREAMPlace's clamp to sqrt(2) bins with area ratio (fp32)."""
    sx = np.asarray(size_x, np.float32)
    sy = np.asarray(size_y, np.float32)
    cx = np.maximum(sx, np.float32(bin_size_x * math.sqrt(2.0)))
    cy = np.maximum(sy, np.float32(bin_size_y * math.sqrt(2.0)))
    ox = ((sx - cx) * np.float32(0.5)).astype(np.float32)
    oy = ((sy - cy) * np.float32(0.5)).astype(np.float32)
    ratio = ((sx * sy) / (cx * cy)).astype(np.float32)
    return cx.astype(np.float32), cy.astype(np.float32), ox, oy, ratio


def _place_macros(rng, n, die, max_tries=4000):
    """Non-overlapping macros, largest first, rejection sampled."""
    w = rng.uniform(100.0, 800.0, n)
    h = rng.uniform(100.0, 800.0, n)
    order = np.argsort(-(w * h))
    px = np.empty(0); py = np.empty(0); pw = np.empty(0); ph = np.empty(0)
    for i in order:
        for _ in range(max_tries // 64):
            cx = rng.uniform(0.0, die - w[i], 64)
            cy = rng.uniform(0.0, die - h[i], 64)
            if len(px):
                ov = ((cx[:, None] < px[None, :] + pw[None, :]) & (px[None, :] < cx[:, None] + w[i]) &
                      (cy[:, None] < py[None, :] + ph[None, :]) & (py[None, :] < cy[:, None] + h[i]))
                ok = np.flatnonzero(~ov.any(axis=1))
            else:
                ok = np.array([0])
            if len(ok):
                j = ok[0]
                px = np.append(px, cx[j]); py = np.append(py, cy[j])
                pw = np.append(pw, w[i]); ph = np.append(ph, h[i])
                break
    return px, py, pw, ph


def rasterise(px, py, pw, ph, xl, yl, bsx, bsy, M, N):
    """Exact overlap area of axis-aligned rectangles with each bin (float64)."""
    out = np.zeros((M, N), np.float64)
    for x, y, w, h in zip(px, py, pw, ph):
        kx0 = max(int((x - xl) // bsx), 0); kx1 = min(int((x + w - xl) // bsx), M - 1)
        ky0 = max(int((y - yl) // bsy), 0); ky1 = min(int((y + h - yl) // bsy), N - 1)
        ex = xl + np.arange(kx0, kx1 + 2) * bsx
        ey = yl + np.arange(ky0, ky1 + 2) * bsy
        ox = np.clip(np.minimum(x + w, ex[1:]) - np.maximum(x, ex[:-1]), 0.0, None)
        oy = np.clip(np.minimum(y + h, ey[1:]) - np.maximum(y, ey[:-1]), 0.0, None)
        out[kx0:kx1 + 1, ky0:ky1 + 1] += ox[:, None] * oy[None, :]
    return out


def _positions(rng, w, h, die, hotspots, hot_frac, sigma):
    n = len(w)
    cx = rng.uniform(0.0, die, n)
    cy = rng.uniform(0.0, die, n)
    if hotspots > 0 and hot_frac > 0:
        centres = rng.uniform(0.0, die, (hotspots, 2))
        hot = rng.random(n) < hot_frac
        k = rng.integers(0, hotspots, n)
        cx = np.where(hot, centres[k, 0] + sigma * rng.standard_normal(n), cx)
        cy = np.where(hot, centres[k, 1] + sigma * rng.standard_normal(n), cy)
    x = np.clip(cx - 0.5 * w, 0.0, die - w)
    y = np.clip(cy - 0.5 * h, 0.0, die - h)
    return x, y


def make_placement(config: str = "c1", scale: float = 1.0, grid: Optional[int] = None,
                   seed: Optional[int] = None) -> Placement:
    """Build a BASELINE configuration.  scale < 1 shrinks the cell and macro
    counts (die, grid and distributions unchanged) for quick tests."""
    c = dict(CONFIGS[config])
    if grid is not None:
        c["grid"] = grid
    if seed is not None:
        c["seed"] = seed
    rng = np.random.default_rng(c["seed"])
    die = c["die"]
    n_mov = max(1, int(round(c["movable"] * scale)))
    n_fil = int(round(c["fillers"] * scale))
    n_mac = int(round(c["macros"] * scale))
    # movable standard cells
    w_m = np.clip(rng.lognormal(math.log(8.0), 0.5, n_mov), 2.0, 80.0)
    h_m = np.full(n_mov, 12.0)
    x_m, y_m = _positions(rng, w_m, h_m, die, c["hotspots"], c["hot_frac"], c["sigma"])
    # fillers
    w_f = np.full(n_fil, 8.0)
    h_f = np.full(n_fil, 12.0)
    x_f, y_f = _positions(rng, w_f, h_f, die, c["hotspots"], c["hot_frac"], c["sigma"])
    # macros (fixed terminals)
    mx, my, mw, mh = _place_macros(rng, n_mac, die) if n_mac else (np.empty(0),) * 4
    M = N = c["grid"]
    f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    p = Placement(
        name=config, xl=0.0, yl=0.0, xh=die, yh=die, num_bins_x=M, num_bins_y=N,
        num_movable=n_mov, num_terminals=len(mx), num_filler=n_fil,
        x=f32(np.concatenate([x_m, mx, x_f])), y=f32(np.concatenate([y_m, my, y_f])),
        size_x=f32(np.concatenate([w_m, mw, w_f])), size_y=f32(np.concatenate([h_m, mh, h_f])))
    bsx, bsy = p.bin_size_x, p.bin_size_y
    p.size_x_clamped, p.size_y_clamped, p.offset_x, p.offset_y, p.ratio = stretch(p.size_x, p.size_y, bsx, bsy)
    if len(mx):
        # from the fp32 node arrays the engine is given, so every consumer sees one geometry
        t = slice(n_mov, n_mov + len(mx))
        p.initial_density_map = rasterise(p.x[t].astype(np.float64), p.y[t].astype(np.float64),
                                          p.size_x[t].astype(np.float64), p.size_y[t].astype(np.float64),
                                          p.xl, p.yl, bsx, bsy, M, N)
    else:
        p.initial_density_map = np.zeros((M, N), np.float64)
    return p
