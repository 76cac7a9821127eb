"""Build the CPU oracle (TEST INFRASTRUCTURE ONLY).

* oracle/libepb_oracle.so from oracle/epb_oracle.c (gcc, OpenMP,
  -ffp-contract=off so fp32 contributions are not fused into FMAs);
* oracle/_ref/ref_dct from the reference's own DCT builders, when the
  reference tree is present (oracle/build_ref.sh).
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def build_oracle(verbose=False):
    src = os.path.join(HERE, "epb_oracle.c")
    out = os.path.join(HERE, "libepb_oracle.so")
    if os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
        return out
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
           "-fPIC", "-shared", "-std=c11", src, "-o", out, "-lm"]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    return out


def reference_root(ref_root=None):
    """Where the reference tree is: the argument, else the REF_ROOT environment
    variable, else BASELINE.json's `reference_path`; None when none is set."""
    if ref_root:
        return ref_root
    if os.environ.get("REF_ROOT"):
        return os.environ["REF_ROOT"]
    cfg = os.path.join(os.path.dirname(HERE), "BASELINE.json")
    if os.path.exists(cfg):
        import json
        with open(cfg) as f:
            return json.load(f).get("reference_path") or None
    return None


def build_ref(ref_root=None, verbose=False):
    """Returns the ref_dct path, or None when the reference tree is absent."""
    ref_root = reference_root(ref_root)
    exe = os.path.join(HERE, "_ref", "ref_dct")
    if not ref_root or not os.path.isdir(ref_root):
        return exe if os.path.exists(exe) else None
    r = subprocess.run(["bash", os.path.join(HERE, "build_ref.sh"), ref_root],
                       capture_output=not verbose, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build_ref.sh failed: {r.stderr}")
    return exe


if __name__ == "__main__":
    print(build_oracle(verbose=True))
    print(build_ref(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True))
