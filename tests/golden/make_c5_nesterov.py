"""Generate tests/golden/c5_nesterov.npz: the CPU restatement's trajectory of
the Nesterov global placer (oracle/nesterov.py) at C5 size: 1.1M movable
cells + 300k fillers on a 1024 x 1024 grid, the seeded synthetic netlist (one
net per movable cell, seed 0), started from the C5 positions, 200 iterations
with the stop overflow at 0.

    python tests/golden/make_c5_nesterov.py [--iterations 200] [--threads N]

The restatement is float64 apart from the positions, which it keeps in fp32
as the device does.  The fixture holds the per-iteration hpwl, overflow,
wirelength, energy, density weight, gamma, step length and backtrack count;
tests/test_nesterov.py runs the device placer on the same design and compares.
About 6 s per evaluation on 8 host threads (some 20 minutes in all).
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iterations", type=int, default=200)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    import build_oracle
    build_oracle.build_oracle()
    import nesterov as onest
    from dreamplacett_framework_b200 import synth
    from dreamplacett_framework_b200.wirelength import synthetic_netlist
    p = synth.make_placement("c5")
    nl = synthetic_netlist(p.size_x, p.size_y, np.arange(p.num_movable), p.num_nodes, seed=0)
    t0 = time.time()
    pl = onest.Placer(p, nl, dict(iterations=args.iterations, stop_overflow=0.0), nthreads=args.threads,
                      workers=args.threads)
    h = pl.run()
    print(f"{len(h['hpwl'])} iterations in {time.time() - t0:.0f} s; hpwl {h['hpwl'][0]:.6g} -> {h['hpwl'][-1]:.6g}, "
          f"overflow {h['overflow'][0]:.4f} -> {h['overflow'][-1]:.4f}", flush=True)
    np.savez_compressed(os.path.join(HERE, "c5_nesterov.npz"), **h)


if __name__ == "__main__":
    main()
