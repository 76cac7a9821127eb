"""CPU restatement of the Nesterov global placer (TEST INFRASTRUCTURE ONLY).

Imported by tests/ as the checker of dreamplacett_framework_b200.nesterov; the
product package never imports it.

The method is restated from its publications (DREAMPlace, the optimiser the
reference's driver runs through NonLinearPlace, integration/run_dreamplace.py:315-370,
is absent from the reference tree):
* ePlace (Lu et al., ACM TODAES 2015), Algorithm 2 and section 5: Nesterov's
  method with the Lipschitz-predicted step length and its backtracking, the
  preconditioner max(1, pins + lambda * area), the density-weight update
  mu0^(1 - dHPWL / dHPWL_ref) within [mu_min, mu_max], and the WA smoothing
  gamma0 * bin * 10^((20/9) overflow - 11/9);
* DREAMPlace (Lin et al., DAC 2019): the initial density weight
  density_weight * |grad W|_1 / |grad E|_1 and the probe step that predicts
  the first step length.

Everything is float64 except what the device keeps in fp32 by design: the
positions (rounded to fp32 after every update), the fp32 density map and the
fields handed to the gather.  The electric potential is the oracle chain
(fixed-point density, float64 DCT solve, gather) and the wirelength is
oracle/wirelength.py.
"""
from __future__ import annotations

import math

import numpy as np

import oracle as o
import wirelength as owl


def gamma_of(p, overflow, bin_w, bin_h):
    return p["gamma"] * 0.5 * (bin_w + bin_h) * 10.0 ** ((20.0 / 9.0) * overflow - 11.0 / 9.0)


def mu_of(p, d_hpwl):
    # the exponent bounded first: a change far beyond the reference saturates at the clamp
    e = min(max(1.0 - d_hpwl / p["hpwl_ref_delta"], -1000.0), 1000.0)
    return min(max(p["mu0"] ** e, p["mu_min"]), p["mu_max"])


PARAMS = dict(iterations=100, target_density=1.0, density_weight=8e-5, gamma=4.0, learning_rate=0.01,
              stop_overflow=0.07, ignore_net_degree=100, mu0=1.1, mu_min=0.75, mu_max=1.1, hpwl_ref_delta=3.5e5,
              backtrack_ratio=0.95, backtrack_limit=10)


class Placer:
    """The restated placer on one grid: placement p (synth.Placement layout) on
    its own bins, netlist arrays (net_start, net_pins, pin_node, pin offsets)."""

    def __init__(self, p, netlist, params=None, nthreads=4, workers=4):
        self.p = p
        self.nl = netlist
        self.P = dict(PARAMS, **(params or {}))
        self.nthreads, self.workers = nthreads, workers
        self.g = o.Geometry(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh)
        self.S = self.g.default_fixed_bits()
        self.init = p.initial_density_norm()
        n = p.num_nodes
        self.n, self.m, self.f = n, p.num_movable, p.num_filler
        self.x = p.x.astype(np.float32).copy()
        self.y = p.y.astype(np.float32).copy()
        deg = np.bincount(netlist.pin_node, minlength=n).astype(np.float32)
        area = (p.size_x.astype(np.float64) * p.size_y.astype(np.float64)).astype(np.float32)
        self.deg = self._moving(deg).astype(np.float64)
        self.area = self._moving(area).astype(np.float64)
        self.movable_area = float(np.sum(area[:self.m].astype(np.float64)))
        k = self.m + self.f
        self.lo = np.concatenate([np.full(k, p.xl), np.full(k, p.yl)])
        w32 = np.float32
        self.hi = np.concatenate([(w32(p.xh) - self._moving(p.size_x)).astype(np.float32),
                                  (w32(p.yh) - self._moving(p.size_y)).astype(np.float32)]).astype(np.float64)
        self.bin_w, self.bin_h = p.bin_size_x, p.bin_size_y

    def _moving(self, a):
        return np.concatenate([a[:self.m], a[self.n - self.f:]])

    def _get(self):
        return np.concatenate([self._moving(self.x), self._moving(self.y)]).astype(np.float64)

    def _set(self, z):
        k = self.m + self.f
        zx = z[:k].astype(np.float32)
        zy = z[k:].astype(np.float32)
        self.x[:self.m] = zx[:self.m]
        self.x[self.n - self.f:] = zx[self.m:]
        self.y[:self.m] = zy[:self.m]
        self.y[self.n - self.f:] = zy[self.m:]

    def _clamp(self, z):
        # positions live in fp32 on the device: round after every update
        return np.minimum(np.maximum(z, self.lo), self.hi).astype(np.float32).astype(np.float64)

    def evaluate(self, z, lam, gamma):
        p = self.p
        self._set(z)
        cells = o.Cells(self.x, self.y, p.size_x_clamped, p.size_y_clamped, p.offset_x, p.offset_y, p.ratio,
                        ranges=((0, self.m), (self.n - self.f, self.n)))
        mov = o.Cells(self.x, self.y, p.size_x_clamped, p.size_y_clamped, p.offset_x, p.offset_y, p.ratio,
                      ranges=((0, self.m), (0, 0)))
        ovf_area, _ = o.overflow(mov, self.g, self.S, self.init, self.P["target_density"], self.nthreads)
        sol = o.electric_potential(cells, self.g, self.S, self.init, self.nthreads, self.workers)
        nl = self.nl
        wl, hp, wgx, wgy = owl.wirelength(self.x, self.y, nl.net_start, nl.net_pins, nl.pin_node, nl.pin_offset_x,
                                          nl.pin_offset_y, gamma, self.n, nl.net_weight, self.P["ignore_net_degree"])
        gw = np.concatenate([self._moving(wgx), self._moving(wgy)])
        ge = np.concatenate([self._moving(sol["grad_x"]), self._moving(sol["grad_y"])]).astype(np.float64)
        return self.combine(gw, ge, lam), wl, hp, float(sol["energy"]), ovf_area / self.movable_area, gw, ge

    def combine(self, gw, ge, lam):
        """Preconditioned gradient of W + lam * E from its two parts."""
        pre = np.maximum(self.deg + lam * self.area, 1.0)
        pre = np.concatenate([pre, pre])
        return (gw + lam * ge) / pre

    def run(self, iterations=None):
        P = self.P
        K = P["iterations"] if iterations is None else iterations
        hist = {k: [] for k in ("hpwl", "overflow", "wirelength", "energy", "density_weight", "gamma", "step",
                                "backtracks")}
        u = self._clamp(self._get())
        v = u.copy()
        # the smoothing of the start's overflow, then the initial density weight
        ovf = self.evaluate(v, 0.0, gamma_of(P, 1.0, self.bin_w, self.bin_h))[4]
        gamma = gamma_of(P, ovf, self.bin_w, self.bin_h)
        _, wl, hp, en, ovf, gw, ge = self.evaluate(v, 0.0, gamma)
        lam = P["density_weight"] * float(np.abs(gw).sum()) / max(float(np.abs(ge).sum()), 1e-30)
        g = self.combine(gw, ge, lam)
        step0 = P["learning_rate"] * 0.5 * (self.bin_w + self.bin_h) / max(float(np.abs(g).max()), 1e-30)
        v_prev = self._clamp(v - step0 * g)
        g_prev = self.evaluate(v_prev, lam, gamma)[0]
        a = 1.0
        hp_prev = hp
        for _ in range(K):
            dv = float(np.linalg.norm(v - v_prev))
            dg = float(np.linalg.norm(g - g_prev))
            alpha = dv / dg if dg > 0 else step0
            bt = 0
            while True:
                u_new = self._clamp(v - alpha * g)
                a_new = 0.5 * (1.0 + math.sqrt(4.0 * a * a + 1.0))
                v_new = self._clamp(u_new + ((a - 1.0) / a_new) * (u_new - u))
                g_new, wl, hp, en, ovf, gw, ge = self.evaluate(v_new, lam, gamma)
                dv = float(np.linalg.norm(v_new - v))
                dg = float(np.linalg.norm(g_new - g))
                alpha_hat = dv / dg if dg > 0 else alpha
                if alpha_hat >= P["backtrack_ratio"] * alpha or bt >= P["backtrack_limit"] or alpha_hat == 0.0:
                    break
                alpha = alpha_hat
                bt += 1
            v_prev, g_prev = v, g
            u, v, a, g = u_new, v_new, a_new, g_new
            for k, val in (("hpwl", hp), ("overflow", ovf), ("wirelength", wl), ("energy", en),
                           ("density_weight", lam), ("gamma", gamma), ("step", alpha), ("backtracks", bt)):
                hist[k].append(val)
            lam *= mu_of(P, hp - hp_prev)
            hp_prev = hp
            gamma = gamma_of(P, ovf, self.bin_w, self.bin_h)
            g = self.combine(gw, ge, lam)   # the gradient at v under the new density weight
            if ovf < P["stop_overflow"]:
                break
        self._set(u)
        return {k: np.asarray(v) for k, v in hist.items()}
