"""Generate the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference tree (read-only) mounted:

    python tests/golden/make_golden.py [REF_ROOT]

Sources (paths relative to the reference project):
* integration/scatter_ttnn_client.py:55-93   _cpu_density_fp32 (fp32 overlaps, 8x8 footprint)
* tools/v11_phase2_smoke.py:21-94              cpu_triangle_density (fp32 floor + exact-edge
                                               correction, fp64 overlaps)
* tools/cpu_vs_tt_density.py:45-76             cpu_density (scalar fp64)
* host/density_scatter_ttnn_server_host.cpp:124-181, 252-263
                                               DCT matrix builders and wu/wv weights,
                                               compiled by oracle/build_ref.sh
The reference modules are imported from the reference tree at generation
time only; the fixtures (inputs and outputs) are what the tests read.
"""
from __future__ import annotations

import importlib.util
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _import(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def density_cases(rng):
    """Small seeded cases in the reference smoke test's style
    (tools/v11_phase2_smoke.py:112-117: sizes U[0.5, 2] x 1.5 bins)."""
    cases = []
    for (M, N, nc, die, seed) in [(32, 32, 400, 1000.0, 11), (64, 32, 1500, 2000.0, 12), (64, 64, 3000, 640.0, 13)]:
        r = np.random.default_rng(seed)
        avg = die / M * 1.5
        px = r.uniform(0.0, die - avg, nc).astype(np.float32)
        py = r.uniform(0.0, die - avg, nc).astype(np.float32)
        sx = r.uniform(avg * 0.5, avg * 2.0, nc).astype(np.float32)
        sy = r.uniform(avg * 0.5, avg * 2.0, nc).astype(np.float32)
        cases.append(dict(M=M, N=N, xl=0.0, yl=0.0, xh=die, yh=die, px=px, py=py, sx=sx, sy=sy))
    # exact-edge and die-boundary case: positions on bin edges, cells ending on edges,
    # cells touching the die's right/top boundary
    M = N = 16
    die = 160.0  # bin 10.0, exactly representable
    e = np.arange(0.0, 150.0, 10.0, dtype=np.float32)
    px = np.concatenate([e, e + 0.5, e[:8] + 9.999999, np.array([150.0, 155.0, 0.0], np.float32)])
    py = np.concatenate([e[::-1], e + 2.5, e[:8], np.array([150.0, 0.0, 155.0], np.float32)])
    n = len(px)
    sx = np.concatenate([np.full(15, 10.0), np.full(15, 9.0), np.full(8, 20.0), np.array([10.0, 5.0, 3.0])]).astype(np.float32)
    sy = np.concatenate([np.full(15, 20.0), np.full(15, 7.5), np.full(8, 10.0), np.array([10.0, 3.0, 5.0])]).astype(np.float32)
    assert len(sx) == n and len(sy) == n
    cases.append(dict(M=M, N=N, xl=0.0, yl=0.0, xh=die, yh=die, px=px.astype(np.float32),
                      py=py.astype(np.float32), sx=sx, sy=sy))
    return cases


def main(ref_root):
    client = _import(os.path.join(ref_root, "integration", "scatter_ttnn_client.py"), "ref_client")
    smoke = _import(os.path.join(ref_root, "tools", "v11_phase2_smoke.py"), "ref_smoke")
    cvt = _import(os.path.join(ref_root, "tools", "cpu_vs_tt_density.py"), "ref_cvt")
    rng = np.random.default_rng(2024)
    out = {}
    for i, c in enumerate(density_cases(rng)):
        M, N = c["M"], c["N"]
        bsx = (c["xh"] - c["xl"]) / M
        bsy = (c["yh"] - c["yl"]) / N
        d_fp32 = client._cpu_density_fp32(c["px"], c["py"], c["sx"], c["sy"], M, N,
                                          np.float32(c["xl"]), np.float32(c["yl"]), bsx, bsy)
        d_fp32 = d_fp32 * np.float32(1.0 / (bsx * bsy))  # client:123-124 normalisation
        d_tri = smoke.cpu_triangle_density(c["px"], c["py"], c["sx"], c["sy"], c["xl"], c["yl"],
                                           c["xh"], c["yh"], M, N)
        d_scalar = cvt.cpu_density(M, N, c["xl"], c["yl"], c["xh"], c["yh"], c["px"], c["py"], c["sx"], c["sy"])
        for k, v in c.items():
            out[f"case{i}_{k}"] = np.asarray(v)
        out[f"case{i}_client_fp32"] = d_fp32.astype(np.float32)
        out[f"case{i}_smoke_triangle"] = d_tri.astype(np.float32)
        out[f"case{i}_scalar_fp64"] = d_scalar.astype(np.float64)
    out["num_density_cases"] = np.array(len(density_cases(rng)))
    np.savez_compressed(os.path.join(HERE, "density_ref.npz"), **out)

    # DCT matrices and weights from the compiled reference builders
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import build_oracle as obuild  # noqa: E402
    exe = obuild.build_ref(ref_root)
    dct = {}
    for j, (M, N, bsx, bsy) in enumerate([(8, 8, 1.0, 1.0), (16, 32, 9.765625, 9.765625), (32, 16, 2.0, 1.0)]):
        tmp = os.path.join(HERE, f"_tmp_{j}.bin")
        subprocess.check_call([exe, str(M), str(N), repr(bsx), repr(bsy), tmp])
        a = np.fromfile(tmp, dtype=np.float32)
        os.remove(tmp)
        sizes = [M * M] * 3 + [N * N] * 3 + [M * N] * 2
        parts = np.split(a, np.cumsum(sizes)[:-1])
        names = ["dct2_M", "idct_M", "idxst_M", "dct2_N", "idct_N", "idxst_N", "wu", "wv"]
        dct[f"s{j}_shape"] = np.array([M, N])
        dct[f"s{j}_bins"] = np.array([bsx, bsy])
        for nm, p in zip(names, parts):
            shp = (M, M) if nm.endswith("_M") else (N, N) if nm.endswith("_N") else (M, N)
            dct[f"s{j}_{nm}"] = p.reshape(shp)
        # the reference chain (host:281-295) evaluated with the reference's fp32 matrices
        rho = np.random.default_rng(100 + j).random((M, N)).astype(np.float32)
        D = {nm: dct[f"s{j}_{nm}"].astype(np.float64) for nm in names}
        auv = D["dct2_M"] @ rho.astype(np.float64) @ D["dct2_N"].T
        fx = (2.0 * D["idxst_M"]) @ (auv * D["wu"]) @ D["idct_N"].T
        fy = (2.0 * D["idct_M"]) @ (auv * D["wv"]) @ D["idxst_N"].T
        dct[f"s{j}_rho"] = rho
        dct[f"s{j}_field_x"] = fx
        dct[f"s{j}_field_y"] = fy
    dct["num_dct_cases"] = np.array(3)
    np.savez_compressed(os.path.join(HERE, "dct_ref.npz"), **dct)
    print("wrote", os.path.join(HERE, "density_ref.npz"), os.path.join(HERE, "dct_ref.npz"))


if __name__ == "__main__":
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
    import build_oracle
    root = build_oracle.reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if not root:
        raise SystemExit("make_golden: give the reference tree as an argument or in REF_ROOT")
    main(root)
