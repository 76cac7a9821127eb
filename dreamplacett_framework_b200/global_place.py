"""Multi-stage global placement and the reference driver's command line.

A reference benchmark config (benchmarks/configs/*.json) lists
`global_place_stages`, each with its own grid (num_bins_x / num_bins_y), an
iteration budget and a learning rate, plus the design-wide target_density,
density_weight, gamma, stop_overflow and ignore_net_degree.  `place` runs the
stages in order with the Nesterov placer of `nesterov.py`: every stage gets an
engine on its own grid (the stretched sizes and the fixed-cell density are
re-derived for its bins), and the positions pass from one stage to the next
as the same device tensors (no host round trip inside or between stages).

    python -m dreamplacett_framework_b200.global_place --benchmark CONFIG.json
        [--synthetic c1 --scale 0.1] [--results-dir DIR]

mirrors integration/run_dreamplace.py (its --benchmark / --results-dir and
outputs, :63-90 and :564-596): `<name>_b200_iters.csv` with one row per
electric-potential call (stage, iteration, hpwl, overflow, the objective's
terms and the operator's device time) and `<name>_b200_metrics.json` (wall
time, call count, mean / median operator time, final hpwl and overflow).
With --synthetic, or when the config's aux_input is not on disk, a seeded
synthetic stand-in of the given BASELINE configuration is placed with a
synthetic netlist (no ISPD-2005 design is available here).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import time
from typing import Dict, List

import numpy as np
import torch

from .nesterov import NesterovParams, NesterovPlacer
from .wirelength import NetlistArrays


def stage_params(cfg: dict, stage: dict) -> NesterovParams:
    return NesterovParams(iterations=int(stage.get("iteration", 1000)),
                          learning_rate=float(stage.get("learning_rate", 0.01)),
                          target_density=float(cfg.get("target_density", 1.0)),
                          density_weight=float(cfg.get("density_weight", 8e-5)),
                          gamma=float(cfg.get("gamma", 4.0)),
                          stop_overflow=float(cfg.get("stop_overflow", 0.07)),
                          ignore_net_degree=int(cfg.get("ignore_net_degree", 100)))


def place(placement, netlist: NetlistArrays, cfg: dict, device=None, x=None, y=None) -> dict:
    """Run cfg's global-placement stages from the placement's positions (or
    the device tensors x, y, updated in place).  Returns per-stage histories
    and the positions (device tensors)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if x is None:
        x = torch.from_numpy(np.ascontiguousarray(placement.x, np.float32)).to(dev)
        y = torch.from_numpy(np.ascontiguousarray(placement.y, np.float32)).to(dev)
    stages = cfg.get("stages") or cfg.get("global_place_stages") or [{}]
    out: List[dict] = []
    for k, st in enumerate(stages):
        M = int(st.get("num_bins_x", cfg.get("num_bins_x", placement.num_bins_x)))
        N = int(st.get("num_bins_y", cfg.get("num_bins_y", placement.num_bins_y)))
        ps = placement.regrid(M, N)
        params = stage_params(cfg, st)
        with NesterovPlacer(ps, netlist, x, y, params) as pl:
            hist = pl.run()
        out.append(dict(stage=k, num_bins=[M, N], history=hist.as_arrays()))
    return dict(stages=out, x=x, y=y)


def _design(args, cfg):
    from . import bookshelf, synth
    from .wirelength import synthetic_netlist
    aux = cfg.get("aux_input", "")
    if not args.synthetic and aux and os.path.exists(aux):
        p = bookshelf.placement_from_config(args.benchmark)
        nl = bookshelf.netlist_for_placement(aux, p)
        return p, nl, os.path.splitext(os.path.basename(aux))[0]
    name = args.synthetic or "c1"
    p = synth.make_placement(name, scale=args.scale)
    nl = synthetic_netlist(p.size_x, p.size_y, np.arange(p.num_movable), p.num_nodes, seed=args.seed)
    return p, nl, f"synthetic_{name}"


def main(argv=None):
    ap = argparse.ArgumentParser(description="Global placement with the B200 electric-potential engine.")
    ap.add_argument("--benchmark", required=True, help="reference-style JSON config (global_place_stages, ...)")
    ap.add_argument("--device", default="b200", choices=["b200"], help="the engine (CUDA, sm_100a)")
    ap.add_argument("--results-dir", default="results")
    ap.add_argument("--synthetic", default=None, help="place a synthetic BASELINE configuration (c1..c5) instead")
    ap.add_argument("--scale", type=float, default=0.1, help="cell-count scale of the synthetic design")
    ap.add_argument("--seed", type=int, default=0, help="seed of the synthetic netlist")
    args = ap.parse_args(argv)
    from . import bookshelf
    cfg = bookshelf.load_config(args.benchmark)
    p, nl, name = _design(args, cfg)
    os.makedirs(args.results_dir, exist_ok=True)
    t0 = time.perf_counter()
    res = place(p, nl, cfg)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    rows: List[Dict] = []
    for s in res["stages"]:
        h = s["history"]
        for i in range(len(h["hpwl"])):
            rows.append(dict(stage=s["stage"], iteration=i, num_bins_x=s["num_bins"][0], num_bins_y=s["num_bins"][1],
                             **{k: float(h[k][i]) for k in ("hpwl", "overflow", "wirelength", "energy",
                                                            "density_weight", "gamma", "step", "ep_ms")},
                             backtracks=int(h["backtracks"][i])))
    csv_path = os.path.join(args.results_dir, f"{name}_{args.device}_iters.csv")
    keys = list(rows[0]) if rows else []
    with open(csv_path, "w") as f:
        f.write(",".join(keys) + "\n")
        for r in rows:
            f.write(",".join(str(r[k]) for k in keys) + "\n")
    ep = [r["ep_ms"] for r in rows]
    metrics = dict(wall_time_s=wall, device=args.device, benchmark=name, n_ep_calls=len(rows),
                   ep_mean_ms=float(np.mean(ep)) if ep else None,
                   ep_median_ms=float(statistics.median(ep)) if ep else None,
                   ep_total_ms=float(np.sum(ep)) if ep else None,
                   hpwl=rows[-1]["hpwl"] if rows else None, overflow=rows[-1]["overflow"] if rows else None,
                   n_evalmetrics=len(rows), cells=int(p.num_cells), nets=int(nl.num_nets),
                   stages=[dict(stage=s["stage"], num_bins=s["num_bins"], iterations=len(s["history"]["hpwl"]))
                           for s in res["stages"]])
    with open(os.path.join(args.results_dir, f"{name}_{args.device}_metrics.json"), "w") as f:
        json.dump(metrics, f, indent=2)
    print(json.dumps(metrics))


if __name__ == "__main__":
    main()
