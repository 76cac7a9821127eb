"""Density-driven global-placement loop on the GPU (the operator's callers).

The reference hands each iteration's positions to its electric-potential
server from DREAMPlace's Python placer (integration/run_dreamplace.py:315-331)
and reads the per-iteration overflow back through EvalMetrics on the host
(run_dreamplace.py:333-370).  Here the whole iteration stays on the device:

    per step t (lambda_t = lam0 * 2^(t // lam_every)):
      overflow_t, energy_t = epb_forward_overflow(movable | filler cells)
                             (overflow of the movable cells / total movable area;
                              forward of both ranges, fields kept inside)
      grad        = epb_backward(movable + filler cells)
      objective_t = lambda_t * energy_t
      epb_descent_step: x <- clamp(x - step_bins * bin_w * grad / max|grad|)

which is the benchmark's C5 loop: a density-only descent whose normalised
step makes lambda cancel (it is reported in the objective).  Nothing is read
back to the host inside the loop; the per-step values land in device arrays.
With `graph=True` one step is captured as a CUDA graph (the step index lives
on the device) and replayed.

    python -m dreamplacett_framework_b200.placement [--config c5] [--steps 200]
    python -m dreamplacett_framework_b200.placement --design benchmarks/configs/adaptec1_2048.json

(--design takes a reference-style benchmark config naming a bookshelf design.)
"""
from __future__ import annotations

import argparse
import json
import time
from typing import Optional

import numpy as np
import torch

from .engine import CellTensors, ElectricPotentialEngine


class DensityDescent:
    """The C5 loop over one synthetic (or caller-supplied) placement."""

    def __init__(self, placement, device=None, step_bins: float = 0.5, target_density: float = 1.0,
                 lam0: float = 8e-5, lam_every: int = 50):
        if not torch.cuda.is_available():
            raise RuntimeError("DensityDescent needs a CUDA device (no CPU path)")
        p = placement
        self.p = p
        idx = None if device is None else torch.device(device).index
        self.device = torch.device("cuda", torch.cuda.current_device() if idx is None else idx)
        to = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(self.device)
        self.x, self.y = to(p.x), to(p.y)
        self.width, self.height = to(p.size_x), to(p.size_y)
        sx, sy, ox, oy, ratio = (to(a) for a in (p.size_x_clamped, p.size_y_clamped, p.offset_x, p.offset_y,
                                                 p.ratio))
        self.cells = CellTensors(self.x, self.y, sx, sy, ox, oy, ratio, ranges=p.ranges)
        self.movable = CellTensors(self.x, self.y, sx, sy, ox, oy, ratio, ranges=((0, p.num_movable), (0, 0)))
        self.engine = ElectricPotentialEngine(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh,
                                              device=self.device)
        self.engine.set_initial_density(to(p.initial_density_norm()))
        self.step_bins, self.target = float(step_bins), float(target_density)
        self.lam0, self.lam_every = float(lam0), int(lam_every)
        m = p.num_movable
        self.movable_area = float(np.sum(p.size_x[:m].astype(np.float64) * p.size_y[:m].astype(np.float64)))
        n = p.num_nodes
        self.gx = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.gy = torch.zeros(n, dtype=torch.float32, device=self.device)
        # per-step scratch the engine writes; copied into the trajectories at the device-side index
        self._ovf = torch.zeros(2, dtype=torch.float64, device=self.device)
        self._energy = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._linf = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._t = torch.zeros(1, dtype=torch.int64, device=self.device)
        self._graph: Optional[torch.cuda.CUDAGraph] = None

    def close(self):
        self._graph = None
        self.engine.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _step(self, traj_ovf, traj_energy, traj_linf):
        eng = self.engine
        # one scatter: movable cells (first range) give the overflow, fillers join for the forward
        eng.forward_overflow(self.cells, self.target, overflow=self._ovf, want_density=False,
                             want_potential=False, want_fields=False, want_energy=True,
                             out={"energy": self._energy})
        eng.backward(self.cells, grad_x=self.gx, grad_y=self.gy)
        eng.descent_step(self.cells, self.gx, self.gy, self.width, self.height, self.step_bins,
                         grad_linf=self._linf)
        traj_ovf.index_copy_(0, self._t, self._ovf.view(1, 2))
        traj_energy.index_copy_(0, self._t, self._energy)
        traj_linf.index_copy_(0, self._t, self._linf)
        self._t.add_(1)

    def run(self, steps: int = 200, graph: bool = True, sync: bool = True):
        """Run `steps` steps from the current positions (updated in place).
        Returns numpy trajectories like the CPU restatement's: overflow and
        max_density with steps + 1 entries, energy, objective and linf with
        `steps`, plus `ms` (device time of the loop, CUDA events)."""
        dev = self.device
        traj_ovf = torch.zeros((steps + 1, 2), dtype=torch.float64, device=dev)
        traj_energy = torch.zeros(steps, dtype=torch.float32, device=dev)
        traj_linf = torch.zeros(steps, dtype=torch.float32, device=dev)
        self._t.zero_()
        stream = torch.cuda.current_stream(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if graph and steps > 0:
            # one eager step on a scratch trajectory, then capture one step
            scratch = (torch.zeros((1, 2), dtype=torch.float64, device=dev),
                       torch.zeros(1, dtype=torch.float32, device=dev), torch.zeros(1, dtype=torch.float32, device=dev))
            x0, y0 = self.x.clone(), self.y.clone()
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(stream)
            with torch.cuda.stream(cap):
                self._t.zero_()
                self._step(*scratch)
                self._t.zero_()
            stream.wait_stream(cap)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                self._step(traj_ovf, traj_energy, traj_linf)
            # the warm-up and capture moved nothing that counts: restore the start
            self.x.copy_(x0)
            self.y.copy_(y0)
            self._t.zero_()
            torch.cuda.synchronize(dev)
            t0.record(stream)
            for _ in range(steps):
                g.replay()
            t1.record(stream)
            self._graph = g
        else:
            t0.record(stream)
            for _ in range(steps):
                self._step(traj_ovf, traj_energy, traj_linf)
            t1.record(stream)
        # the overflow after the last step
        self.engine.overflow(self.movable, self.target, out=self._ovf)
        traj_ovf[steps].copy_(self._ovf)
        if not sync:
            return None
        torch.cuda.synchronize(dev)
        flags = self.engine.error_flags()
        ovf = traj_ovf.cpu().numpy()
        energy = traj_energy.cpu().numpy().astype(np.float64)
        lam = self.lam0 * 2.0 ** (np.arange(steps) // self.lam_every)
        return dict(overflow=ovf[:, 0] / self.movable_area, max_density=ovf[:, 1], energy=energy,
                    objective=lam * energy, linf=traj_linf.cpu().numpy(), ms=t0.elapsed_time(t1) if steps else 0.0,
                    flags=flags)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--config", default="c5")
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--scale", type=float, default=1.0)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--design", help="reference-style JSON config with aux_input (bookshelf files)")
    args = ap.parse_args()
    if args.design:
        from . import bookshelf
        p = bookshelf.placement_from_config(args.design)
        args.config = p.name
    else:
        from . import synth
        p = synth.make_placement(args.config, scale=args.scale)
    with DensityDescent(p) as loop:
        r = loop.run(args.steps, graph=not args.no_graph)
    every = max(1, args.steps // 10)
    out = {
        "config": args.config, "cells": p.num_cells, "grid": [p.num_bins_x, p.num_bins_y], "steps": args.steps,
        "ms_per_step": r["ms"] / max(1, args.steps), "steps_per_s": 1000.0 * args.steps / r["ms"] if r["ms"] else None,
        "overflow": {str(k): float(r["overflow"][k]) for k in range(0, args.steps + 1, every)},
        "max_density_final": float(r["max_density"][-1]), "energy_final": float(r["energy"][-1]),
        "error_flags": r["flags"],
    }
    print(json.dumps(out))


if __name__ == "__main__":
    main()
