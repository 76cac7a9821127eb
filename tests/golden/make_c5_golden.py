"""Generate tests/golden/c5_trajectory.npz: the CPU restatement's trajectory
of the benchmark's C5 placement loop (1.1M movable cells + 300k fillers on a
1024 x 1024 grid, 200 normalised density-descent steps of 0.5 bin).

    python tests/golden/make_c5_golden.py [--steps 200] [--threads N]

The oracle (oracle/oracle.py: descent_trajectory, float64 DCT chain) runs on
the seeded synthetic C5 placement (dreamplacett_framework_b200/synth.py);
the fixture keeps the per-step overflow ratio, maximum density, energy,
objective and gradient norm plus fp64 sums of the final positions.  The GPU
test replays the same loop through the engine and compares.
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
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    args = ap.parse_args()
    import build_oracle
    build_oracle.build_oracle()
    import oracle as o
    from dreamplacett_framework_b200 import synth
    p = synth.make_placement("c5")
    g = o.Geometry(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh)
    S = g.default_fixed_bits()
    t0 = time.time()
    r = o.descent_trajectory(p.x, p.y, p.size_x, p.size_y, p.size_x_clamped, p.size_y_clamped, p.offset_x,
                             p.offset_y, p.ratio, p.ranges, (0, p.num_movable), g, S, p.initial_density_norm(),
                             steps=args.steps, nthreads=args.threads, workers=args.threads)
    out = os.path.join(HERE, "c5_trajectory.npz")
    np.savez(out, overflow=r["overflow"], max_density=r["max_density"], energy=r["energy"],
             objective=r["objective"], linf=r["linf"], steps=np.int64(args.steps),
             x_sum=np.float64(r["x"].astype(np.float64).sum()), y_sum=np.float64(r["y"].astype(np.float64).sum()))
    print(f"wrote {out} ({time.time() - t0:.1f} s): overflow {r['overflow'][0]:.6f} -> {r['overflow'][-1]:.6f}")


if __name__ == "__main__":
    main()
