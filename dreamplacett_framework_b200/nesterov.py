"""Global placement on the device: the objective W_gamma(x, y) + lambda * E(x, y)
minimised with Nesterov's accelerated gradient and a Lipschitz-predicted step
length, the optimiser of DREAMPlace's global placement.

The reference's driver runs DREAMPlace's NonLinearPlace, whose optimiser is
Nesterov's method (benchmarks/configs/*.json: "optimizer": "nesterov",
"learning_rate", "density_weight", "gamma", "stop_overflow"), and reads the
hpwl and overflow of every iteration (integration/run_dreamplace.py:315-370).
DREAMPlace is absent from the reference tree, so the method is restated here
from its publications:

* ePlace (Lu et al., "ePlace: Electrostatics-Based Placement Using Fast
  Fourier Transform and Nesterov's Method", ACM TODAES 2015), Algorithm 2 and
  section 5: the major / reference solutions u, v and the parameter a,
      u_{k+1} = v_k - alpha_k g(v_k),
      a_{k+1} = (1 + sqrt(4 a_k^2 + 1)) / 2,
      v_{k+1} = u_{k+1} + (a_k - 1) (u_{k+1} - u_k) / a_{k+1},
  the step length alpha_k = ||v_k - v_{k-1}|| / ||g(v_k) - g(v_{k-1})|| (the
  inverse of a local Lipschitz estimate) with backtracking while the estimate
  at the new point falls below 0.95 alpha_k; the preconditioner
  H_ii = max(1, |E_i| + lambda q_i) (pins of node i, its area); the density
  weight update lambda_{k+1} = mu_k lambda_k with
  mu_k = mu0^(1 - dHPWL_k / dHPWL_ref) clamped to [mu_min, mu_max]; the WA
  smoothing gamma = gamma0 * bin * 10^((20/9) tau - 11/9) for overflow tau.
* DREAMPlace (Lin et al., "DREAMPlace: Deep Learning Toolkit-Enabled GPU
  Acceleration for Modern VLSI Placement", DAC 2019): the same objective with
  the WA wirelength, fillers, the initial density weight
  lambda_0 = density_weight * ||grad W||_1 / ||grad E||_1, and a first step
  length predicted from a probe step of size learning_rate.

The operator calls are this package's CUDA kernels (forward_overflow, backward,
the WA wirelength); the vector arithmetic of the method is torch on the same
device.  Each iteration reads back a few scalars to take the backtracking
decision and to log hpwl / overflow, as the reference's driver does.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from .engine import CellTensors, ElectricPotentialEngine
from .wirelength import Netlist, NetlistArrays, WirelengthOp


@dataclass
class NesterovParams:
    iterations: int = 100
    target_density: float = 1.0
    density_weight: float = 8e-5     # multiplier of the initial density weight
    gamma: float = 4.0               # WA smoothing base, in bins
    learning_rate: float = 0.01      # probe step of the first step-length prediction, in bins
    stop_overflow: float = 0.07
    ignore_net_degree: int = 100
    mu0: float = 1.1
    mu_min: float = 0.75
    mu_max: float = 1.1
    hpwl_ref_delta: float = 3.5e5    # dHPWL_ref of the density weight update
    backtrack_ratio: float = 0.95
    backtrack_limit: int = 10


def gamma_of(params: NesterovParams, overflow: float, bin_w: float, bin_h: float) -> float:
    """WA smoothing for the current overflow (ePlace's exponent form)."""
    return params.gamma * 0.5 * (bin_w + bin_h) * 10.0 ** ((20.0 / 9.0) * overflow - 11.0 / 9.0)


def mu_of(params: NesterovParams, d_hpwl: float) -> float:
    """mu0^(1 - dHPWL / dHPWL_ref) clamped to [mu_min, mu_max].  The exponent
    is bounded to +-1000 first, so an HPWL change far beyond dHPWL_ref
    saturates at the clamp instead of overflowing the power."""
    e = min(max(1.0 - d_hpwl / params.hpwl_ref_delta, -1000.0), 1000.0)
    return min(max(params.mu0 ** e, params.mu_min), params.mu_max)


@dataclass
class History:
    hpwl: List[float] = field(default_factory=list)
    overflow: List[float] = field(default_factory=list)
    wirelength: List[float] = field(default_factory=list)
    energy: List[float] = field(default_factory=list)
    density_weight: List[float] = field(default_factory=list)
    gamma: List[float] = field(default_factory=list)
    step: List[float] = field(default_factory=list)
    backtracks: List[int] = field(default_factory=list)
    ep_ms: List[float] = field(default_factory=list)   # device time of the operator (forward + backward)

    def as_arrays(self) -> Dict[str, np.ndarray]:
        return {k: np.asarray(v) for k, v in self.__dict__.items()}


class NesterovPlacer:
    """One global-placement stage on one grid.

    `x`, `y` are device tensors of all node positions (DREAMPlace's pos halves,
    nodes ordered [movable | terminals | fillers]) and are updated in place;
    the movable and filler nodes move, terminals stay.  `size_x`, `size_y` are
    the nodes' sizes; `netlist` the pins (fillers have none)."""

    def __init__(self, placement, netlist: NetlistArrays, x: torch.Tensor, y: torch.Tensor,
                 params: NesterovParams):
        p = placement
        self.p = p
        self.params = params
        self.device = x.device
        dev = self.device
        self.x, self.y = x, y
        n = p.num_nodes
        self.n = n
        self.m, self.f = p.num_movable, p.num_filler
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
        self.w, self.h = f32(p.size_x), f32(p.size_y)
        # the stage's grid: stretched sizes, offsets, ratio and fixed-cell density of its bins
        self.M, self.N = p.num_bins_x, p.num_bins_y
        self.bin_w, self.bin_h = p.bin_size_x, p.bin_size_y
        self.cells = CellTensors(x, y, f32(p.size_x_clamped), f32(p.size_y_clamped), f32(p.offset_x),
                                 f32(p.offset_y), f32(p.ratio), ranges=((0, self.m), (n - self.f, n)))
        self.engine = ElectricPotentialEngine(self.M, self.N, p.xl, p.yl, p.xh, p.yh, device=dev)
        self.engine.set_initial_density(f32(p.initial_density_norm()))
        self.wl = WirelengthOp(Netlist(netlist, dev, ignore_net_degree=params.ignore_net_degree))
        # preconditioner pieces: pins per node and node areas (moving nodes)
        deg = np.bincount(netlist.pin_node, minlength=n).astype(np.float32)
        area = (p.size_x.astype(np.float64) * p.size_y.astype(np.float64)).astype(np.float32)
        self.deg = self._moving(f32(deg))
        self.area = self._moving(f32(area))
        self.movable_area = float(np.sum(area[:self.m].astype(np.float64)))
        # clamp bounds of the moving coordinates
        self.lo = torch.cat([torch.full((self.m + self.f,), p.xl, device=dev),
                             torch.full((self.m + self.f,), p.yl, device=dev)])
        self.hi = torch.cat([p.xh - self._moving(self.w), p.yh - self._moving(self.h)])
        self._ovf = torch.zeros(2, dtype=torch.float64, device=dev)
        self._gx = torch.zeros(n, dtype=torch.float32, device=dev)
        self._gy = torch.zeros(n, dtype=torch.float32, device=dev)
        self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
        self.last_ep_ms = 0.0

    def close(self):
        self.engine.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- moving coordinates z = [x_movable | x_fillers | y_movable | y_fillers]
    def _moving(self, t: torch.Tensor) -> torch.Tensor:
        return torch.cat([t[:self.m], t[self.n - self.f:]])

    def _get(self) -> torch.Tensor:
        return torch.cat([self._moving(self.x), self._moving(self.y)])

    def _set(self, z: torch.Tensor):
        k = self.m + self.f
        zx, zy = z[:k], z[k:]
        self.x[:self.m] = zx[:self.m]
        self.x[self.n - self.f:] = zx[self.m:]
        self.y[:self.m] = zy[:self.m]
        self.y[self.n - self.f:] = zy[self.m:]

    def _clamp(self, z: torch.Tensor) -> torch.Tensor:
        return torch.minimum(torch.maximum(z, self.lo), self.hi)

    def evaluate(self, z: torch.Tensor, lam: float, gamma: float):
        """Preconditioned gradient of W + lam * E at z, with the terms:
        (g, wirelength, hpwl, energy, overflow) -- the scalars as floats."""
        self._set(z)
        st = torch.cuda.current_stream(self.device)
        self._ev[0].record(st)
        out, _ = self.engine.forward_overflow(self.cells, self.params.target_density, overflow=self._ovf,
                                              want_density=False, want_potential=False, want_fields=False,
                                              want_energy=True)
        ge_x, ge_y = self.engine.backward(self.cells, grad_x=self._gx, grad_y=self._gy)
        self._ev[1].record(st)
        r = self.wl(self.x, self.y, gamma)
        gw = torch.cat([self._moving(r["grad_x"]), self._moving(r["grad_y"])])
        ge = torch.cat([self._moving(ge_x), self._moving(ge_y)])
        g = self.combine(gw, ge, lam)
        vals = torch.stack([r["wirelength"].double(), r["hpwl"].double(), out["energy"].double().reshape(()),
                            self._ovf[0]]).cpu().numpy()
        self.last_ep_ms = self._ev[0].elapsed_time(self._ev[1])
        return g, float(vals[0]), float(vals[1]), float(vals[2]), float(vals[3]) / self.movable_area, gw, ge

    @staticmethod
    def _norms(a: torch.Tensor, b: torch.Tensor):
        """(||a||, ||b||) as floats with one device-to-host read."""
        n = torch.stack([torch.linalg.vector_norm(a), torch.linalg.vector_norm(b)]).tolist()
        return float(n[0]), float(n[1])

    def combine(self, gw: torch.Tensor, ge: torch.Tensor, lam: float) -> torch.Tensor:
        """Preconditioned gradient of W + lam * E from its two parts."""
        pre = torch.clamp(self.deg + lam * self.area, min=1.0)
        return (gw + lam * ge) / torch.cat([pre, pre])

    def run(self, lam: Optional[float] = None, iterations: Optional[int] = None) -> History:
        """Iterate from the current positions; returns the per-iteration history
        (hpwl, overflow, ... of the reference point v_k).  Positions are left at
        the last major solution u."""
        P = self.params
        K = P.iterations if iterations is None else iterations
        hist = History()
        u = self._clamp(self._get())
        v = u.clone()
        # the smoothing of the start's overflow, then the initial density weight
        ovf = self.evaluate(v, 0.0, gamma_of(P, 1.0, self.bin_w, self.bin_h))[4]
        gamma = gamma_of(P, ovf, self.bin_w, self.bin_h)
        _, wl, hp, en, ovf, gw, ge = self.evaluate(v, 0.0, gamma)
        if lam is None:
            lam = P.density_weight * float(gw.abs().sum()) / max(float(ge.abs().sum()), 1e-30)
        g = self.combine(gw, ge, lam)
        # first step length: from a probe step of learning_rate bins along -g
        step0 = P.learning_rate * 0.5 * (self.bin_w + self.bin_h) / max(float(g.abs().max()), 1e-30)
        v_prev = self._clamp(v - step0 * g)
        g_prev = self.evaluate(v_prev, lam, gamma)[0]
        a = 1.0
        hp_prev = hp
        for it in range(K):
            dv, dg = self._norms(v - v_prev, g - g_prev)
            alpha = dv / dg if dg > 0 else step0
            bt = 0
            while True:
                u_new = self._clamp(v - alpha * g)
                a_new = 0.5 * (1.0 + math.sqrt(4.0 * a * a + 1.0))
                v_new = self._clamp(u_new + ((a - 1.0) / a_new) * (u_new - u))
                g_new, wl, hp, en, ovf, gw, ge = self.evaluate(v_new, lam, gamma)
                dv, dg = self._norms(v_new - v, g_new - g)
                alpha_hat = dv / dg if dg > 0 else alpha
                if alpha_hat >= P.backtrack_ratio * alpha or bt >= P.backtrack_limit or alpha_hat == 0.0:
                    break
                alpha = alpha_hat
                bt += 1
            v_prev, g_prev = v, g
            u, v, a, g = u_new, v_new, a_new, g_new
            hist.hpwl.append(hp)
            hist.overflow.append(ovf)
            hist.wirelength.append(wl)
            hist.energy.append(en)
            hist.density_weight.append(lam)
            hist.gamma.append(gamma)
            hist.step.append(alpha)
            hist.backtracks.append(bt)
            hist.ep_ms.append(self.last_ep_ms)
            # schedules for the next iteration
            lam *= mu_of(P, hp - hp_prev)
            hp_prev = hp
            gamma = gamma_of(P, ovf, self.bin_w, self.bin_h)
            g = self.combine(gw, ge, lam)   # the gradient at v under the new density weight
            if ovf < P.stop_overflow:
                break
        self._set(u)
        self.lam = lam
        return hist
