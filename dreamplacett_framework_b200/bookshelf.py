"""Bookshelf (ISPD-2005) placement reader and writer.

The reference's benchmark configs name a bookshelf design through
`aux_input` (benchmarks/configs/adaptec1_2048.json: "aux_input",
"num_bins_x/y", "target_density", "enable_fillers", "density_weight") and let
DREAMPlace's parser load it; DREAMPlace is not part of the reference tree and
the ISPD-2005 files are not shipped with it.  This module reads the same
files into the `synth.Placement` structure the engine, the placement loop and
the benchmark take, so a real design replaces the synthetic stand-in when the
files are available:

* `.aux`   "RowBasedPlacement : a.nodes a.nets a.wts a.pl a.scl"
* `.nodes` "name width height [terminal | terminal_NI]"
* `.pl`    "name x y : orient [/FIXED | /FIXED_NI]"   (lower-left corners)
* `.scl`   CoreRow blocks (Coordinate, Height, Sitewidth, Sitespacing,
           SubrowOrigin, NumSites)
* `.nets`  NetDegree blocks: "NetDegree : k [name]", then k lines
           "node I|O|B [: dx dy]" with the pin offset from the node's centre.
           `read_aux` keeps the counts; `netlist_for_placement` reads the pins
           into the wirelength op's input (offsets from the lower-left corner,
           w/2 + dx and h/2 + dy, as DREAMPlace stores them).

Layout follows DREAMPlace's node order [movable | terminals | terminal_NI |
fillers]: `num_terminals` covers both fixed kinds, and only `terminal` nodes
(not the non-image `terminal_NI` pins) enter the fixed-cell density.  The die
is the bounding box of the placement rows.  Fillers follow DREAMPlace's
published rule when `enable_fillers` is set: width = mean movable width over
the 5%..95% range of widths, height = row height, count = round(max(0,
target_density * (die area - fixed area inside the die) - movable area) /
filler area), placed uniformly at random inside the die.
"""
from __future__ import annotations

import json
import math
import os
import re
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from .synth import Placement, rasterise, stretch


@dataclass
class Row:
    y: float
    height: float
    site_width: float
    site_spacing: float
    x: float
    num_sites: int

    @property
    def xh(self) -> float:
        return self.x + self.num_sites * self.site_spacing


@dataclass
class Design:
    """The raw contents of a bookshelf design (node order as in the .nodes file)."""
    name: str
    names: List[str]
    width: np.ndarray          # float64
    height: np.ndarray
    kind: np.ndarray           # 0 movable, 1 terminal, 2 terminal_NI
    x: np.ndarray              # lower-left, float64 (0 when absent from .pl)
    y: np.ndarray
    rows: List[Row]
    num_nets: int = 0
    num_pins: int = 0

    @property
    def die(self) -> Tuple[float, float, float, float]:
        xl = min(r.x for r in self.rows)
        yl = min(r.y for r in self.rows)
        xh = max(r.xh for r in self.rows)
        yh = max(r.y + r.height for r in self.rows)
        return xl, yl, xh, yh

    @property
    def row_height(self) -> float:
        return self.rows[0].height


def _lines(path):
    with open(path) as f:
        for raw in f:
            line = raw.split("#", 1)[0].strip()
            if line and not line.startswith("UCLA"):
                yield line


def _aux_files(aux_path) -> Dict[str, str]:
    base = os.path.dirname(os.path.abspath(aux_path))
    files = []
    for line in _lines(aux_path):
        if ":" in line:
            files += line.split(":", 1)[1].split()
    out = {}
    for fn in files:
        ext = os.path.splitext(fn)[1].lstrip(".").lower()
        out[ext] = os.path.join(base, fn)
    for need in ("nodes", "pl", "scl"):
        if need not in out:
            raise ValueError(f"{aux_path}: no .{need} file listed")
    return out


def _read_nodes(path):
    names, w, h, kind = [], [], [], []
    for line in _lines(path):
        if line.startswith("NumNodes") or line.startswith("NumTerminals"):
            continue
        tok = line.split()
        if len(tok) < 3:
            raise ValueError(f"{path}: bad node line {line!r}")
        names.append(tok[0])
        w.append(float(tok[1]))
        h.append(float(tok[2]))
        k = 0
        if len(tok) > 3:
            t = tok[3].lower()
            k = 2 if t == "terminal_ni" else (1 if t == "terminal" else 0)
        kind.append(k)
    return names, np.array(w), np.array(h), np.array(kind, np.int8)


def _read_pl(path, index):
    x = np.zeros(len(index))
    y = np.zeros(len(index))
    for line in _lines(path):
        tok = line.split()
        if len(tok) < 3 or tok[0] not in index:
            continue
        i = index[tok[0]]
        x[i], y[i] = float(tok[1]), float(tok[2])
    return x, y


def _read_scl(path):
    rows, cur = [], None
    kv = re.compile(r"(\w+)\s*:\s*(\S+)")
    for line in _lines(path):
        low = line.lower()
        if low.startswith("corerow"):
            cur = {}
            continue
        if low.startswith("end"):
            if cur is not None:
                rows.append(Row(y=float(cur["coordinate"]), height=float(cur["height"]),
                                site_width=float(cur.get("sitewidth", 1)),
                                site_spacing=float(cur.get("sitespacing", cur.get("sitewidth", 1))),
                                x=float(cur["subroworigin"]), num_sites=int(float(cur["numsites"]))))
            cur = None
            continue
        if cur is not None:
            for k, v in kv.findall(line):
                cur[k.lower()] = v
    if not rows:
        raise ValueError(f"{path}: no CoreRow blocks")
    return rows


def _read_nets(path):
    nets = pins = 0
    for line in _lines(path):
        if line.startswith("NetDegree"):
            nets += 1
            pins += int(line.split(":", 1)[1].split()[0])
    return nets, pins


def _read_net_pins(path, index):
    """(net_start, pin_node in file order, dx, dy from the node centre)."""
    starts = [0]
    nodes: List[int] = []
    dxs: List[float] = []
    dys: List[float] = []
    expect = 0
    for line in _lines(path):
        if line.startswith("NetDegree"):
            if expect:
                raise ValueError(f"{path}: a net ended {expect} pins early")
            expect = int(line.split(":", 1)[1].split()[0])
            starts.append(starts[-1] + expect)
            continue
        if line.startswith("Num"):
            continue
        if expect <= 0:
            raise ValueError(f"{path}: pin line outside a net: {line!r}")
        head, _, off = line.partition(":")
        name = head.split()[0]
        if name not in index:
            raise ValueError(f"{path}: unknown node {name!r}")
        nodes.append(index[name])
        o = off.split()
        dxs.append(float(o[0]) if len(o) > 0 else 0.0)
        dys.append(float(o[1]) if len(o) > 1 else 0.0)
        expect -= 1
    if expect:
        raise ValueError(f"{path}: the last net ended {expect} pins early")
    return (np.asarray(starts, np.int64), np.asarray(nodes, np.int64), np.asarray(dxs, np.float64),
            np.asarray(dys, np.float64))


def read_aux(aux_path: str) -> Design:
    files = _aux_files(aux_path)
    names, w, h, kind = _read_nodes(files["nodes"])
    index = {n: i for i, n in enumerate(names)}
    x, y = _read_pl(files["pl"], index)
    rows = _read_scl(files["scl"])
    nets = pins = 0
    if "nets" in files and os.path.exists(files["nets"]):
        nets, pins = _read_nets(files["nets"])
    name = os.path.splitext(os.path.basename(aux_path))[0]
    return Design(name, names, w, h, kind, x, y, rows, nets, pins)


def placement_order(d: Design) -> np.ndarray:
    """File index of each node in DREAMPlace's order [movable | terminals | terminal_NI]."""
    return np.concatenate([np.flatnonzero(d.kind == 0), np.flatnonzero(d.kind == 1), np.flatnonzero(d.kind == 2)])


def netlist_for_placement(aux_path: str, p: Placement):
    """The design's nets as a wirelength.NetlistArrays over the nodes of
    `p = to_placement(read_aux(aux_path), ...)`: pins in file order, pin_node in
    the placement's node order, offsets from the node's lower-left corner."""
    from .wirelength import NetlistArrays
    files = _aux_files(aux_path)
    names, w, h, kind = _read_nodes(files["nodes"])
    d = Design(os.path.splitext(os.path.basename(aux_path))[0], names, w, h, kind, np.zeros(len(names)),
               np.zeros(len(names)), [], 0, 0)
    order = placement_order(d)
    to_place = np.empty(len(order), np.int64)
    to_place[order] = np.arange(len(order))
    starts, nodes, dx, dy = _read_net_pins(files["nets"], {n: i for i, n in enumerate(names)})
    pin_node = to_place[nodes]
    ox = (np.float32(0.5) * p.size_x[pin_node] + dx.astype(np.float32)).astype(np.float32)
    oy = (np.float32(0.5) * p.size_y[pin_node] + dy.astype(np.float32)).astype(np.float32)
    P = len(pin_node)
    return NetlistArrays(starts.astype(np.int32), np.arange(P, dtype=np.int32), pin_node.astype(np.int32), ox, oy,
                         p.num_nodes)


def filler_plan(d: Design, target_density: float) -> Tuple[int, float, float]:
    """(count, width, height) of DREAMPlace-style fillers for the design."""
    mov = d.kind == 0
    wm = np.sort(d.width[mov])
    n = len(wm)
    if n == 0:
        return 0, 0.0, 0.0
    lo, hi = int(n * 0.05), int(n * 0.95)
    fw = float(np.mean(wm[lo:hi])) if hi > lo else float(np.mean(wm))
    fh = d.row_height
    xl, yl, xh, yh = d.die
    fixed = d.kind == 1
    ox = np.clip(np.minimum(d.x[fixed] + d.width[fixed], xh) - np.maximum(d.x[fixed], xl), 0, None)
    oy = np.clip(np.minimum(d.y[fixed] + d.height[fixed], yh) - np.maximum(d.y[fixed], yl), 0, None)
    fixed_area = float(np.sum(ox * oy))
    movable_area = float(np.sum(d.width[mov] * d.height[mov]))
    free = target_density * ((xh - xl) * (yh - yl) - fixed_area) - movable_area
    count = int(round(max(0.0, free) / (fw * fh))) if fw > 0 and fh > 0 else 0
    return count, fw, fh


def to_placement(d: Design, num_bins_x: int, num_bins_y: int, target_density: float = 1.0,
                 enable_fillers: bool = True, seed: int = 1000, init: str = "pl") -> Placement:
    """Order the design as DREAMPlace does and build the engine's inputs.

    init = "pl" keeps the .pl positions of movable cells; "center" places them
    at the die centre plus N(0, 0.001 * die size) noise (DREAMPlace's
    random_center_init_flag)."""
    rng = np.random.default_rng(seed)
    order = placement_order(d)
    w, h, x, y = (a[order].astype(np.float64) for a in (d.width, d.height, d.x, d.y))
    n_mov = int(np.sum(d.kind == 0))
    n_term = int(np.sum(d.kind == 1))
    n_ni = int(np.sum(d.kind == 2))
    xl, yl, xh, yh = d.die
    if init == "center":
        cx, cy = 0.5 * (xl + xh), 0.5 * (yl + yh)
        x[:n_mov] = rng.normal(cx, 0.001 * (xh - xl), n_mov) - 0.5 * w[:n_mov]
        y[:n_mov] = rng.normal(cy, 0.001 * (yh - yl), n_mov) - 0.5 * h[:n_mov]
    elif init != "pl":
        raise ValueError("init must be 'pl' or 'center'")
    nf, fw, fh = filler_plan(d, target_density) if enable_fillers else (0, 0.0, 0.0)
    if nf:
        fx = rng.uniform(xl, max(xl, xh - fw), nf)
        fy = rng.uniform(yl, max(yl, yh - fh), nf)
        x = np.concatenate([x, fx])
        y = np.concatenate([y, fy])
        w = np.concatenate([w, np.full(nf, fw)])
        h = np.concatenate([h, np.full(nf, fh)])
    f32 = lambda a: np.ascontiguousarray(a, dtype=np.float32)
    p = Placement(name=d.name, xl=xl, yl=yl, xh=xh, yh=yh, num_bins_x=int(num_bins_x), num_bins_y=int(num_bins_y),
                  num_movable=n_mov, num_terminals=n_term + n_ni, num_filler=nf,
                  x=f32(x), y=f32(y), size_x=f32(w), size_y=f32(h))
    bsx, bsy = p.bin_size_x, p.bin_size_y
    p.size_x_clamped, p.size_y_clamped, p.offset_x, p.offset_y, p.ratio = stretch(p.size_x, p.size_y, bsx, bsy)
    t = slice(n_mov, n_mov + n_term)  # terminal_NI pins carry no density
    if n_term:
        p.initial_density_map = rasterise(x[t], y[t], w[t], h[t], xl, yl, bsx, bsy, p.num_bins_x, p.num_bins_y)
    else:
        p.initial_density_map = np.zeros((p.num_bins_x, p.num_bins_y), np.float64)
    return p


def load_config(path: str) -> dict:
    """A reference benchmark config (benchmarks/configs/*.json) with the fields
    the electric-potential path uses; aux_input is resolved relative to the
    config's directory unless absolute or found relative to the working
    directory."""
    with open(path) as f:
        cfg = json.load(f)
    aux = cfg.get("aux_input", "")
    if aux and not os.path.isabs(aux) and not os.path.exists(aux):
        cand = os.path.join(os.path.dirname(os.path.abspath(path)), aux)
        if os.path.exists(cand):
            aux = cand
    stages = cfg.get("global_place_stages") or [{}]
    return dict(aux_input=aux,
                num_bins_x=int(stages[0].get("num_bins_x", cfg.get("num_bins_x", 512))),
                num_bins_y=int(stages[0].get("num_bins_y", cfg.get("num_bins_y", 512))),
                iterations=int(stages[0].get("iteration", 1000)),
                target_density=float(cfg.get("target_density", 1.0)),
                density_weight=float(cfg.get("density_weight", 8e-5)),
                enable_fillers=bool(cfg.get("enable_fillers", 1)),
                random_seed=int(cfg.get("random_seed", 1000)),
                random_center_init=bool(cfg.get("random_center_init_flag", 0)),
                gamma=float(cfg.get("gamma", 4.0)),
                stop_overflow=float(cfg.get("stop_overflow", 0.07)),
                ignore_net_degree=int(cfg.get("ignore_net_degree", 100)),
                stages=stages)


def placement_from_config(path: str) -> Placement:
    c = load_config(path)
    d = read_aux(c["aux_input"])
    return to_placement(d, c["num_bins_x"], c["num_bins_y"], c["target_density"], c["enable_fillers"],
                        c["random_seed"], "center" if c["random_center_init"] else "pl")


def write_bookshelf(p: Placement, directory: str, name: Optional[str] = None, netlist=None) -> str:
    """Write a Placement's movable cells and terminals as a bookshelf design
    (fillers are not written: a reader re-creates them); rows of height
    `row_height` = the most common movable height cover the die.  `netlist`
    (a wirelength.NetlistArrays over p's nodes, optional) is written to the
    .nets file with offsets from the node centres.  Returns the .aux path."""
    name = name or p.name
    os.makedirs(directory, exist_ok=True)
    n_real = p.num_movable + p.num_terminals
    names = [f"o{i}" for i in range(n_real)]
    mov_h = p.size_y[:p.num_movable]
    row_h = float(np.bincount(np.round(mov_h).astype(np.int64)).argmax()) if len(mov_h) else 12.0
    with open(os.path.join(directory, name + ".nodes"), "w") as f:
        f.write("UCLA nodes 1.0\n\n")
        f.write(f"NumNodes : {n_real}\nNumTerminals : {p.num_terminals}\n")
        for i in range(n_real):
            term = "\tterminal" if i >= p.num_movable else ""
            f.write(f"\t{names[i]}\t{float(p.size_x[i])!r}\t{float(p.size_y[i])!r}{term}\n")
    with open(os.path.join(directory, name + ".pl"), "w") as f:
        f.write("UCLA pl 1.0\n\n")
        for i in range(n_real):
            fixed = " /FIXED" if i >= p.num_movable else ""
            f.write(f"{names[i]}\t{float(p.x[i])!r}\t{float(p.y[i])!r}\t: N{fixed}\n")
    nrows = max(1, int(math.floor((p.yh - p.yl) / row_h)))
    with open(os.path.join(directory, name + ".scl"), "w") as f:
        f.write("UCLA scl 1.0\n\n")
        f.write(f"NumRows : {nrows}\n\n")
        for r in range(nrows):
            y0 = p.yl + r * row_h
            h = row_h if r < nrows - 1 else (p.yh - y0)
            f.write("CoreRow Horizontal\n")
            f.write(f"  Coordinate    :   {y0!r}\n  Height        :   {h!r}\n")
            f.write("  Sitewidth     :    1\n  Sitespacing   :    1\n  Siteorient    :    1\n  Sitesymmetry  :    1\n")
            f.write(f"  SubrowOrigin  :    {p.xl!r}\tNumSites  :  {int(round(p.xh - p.xl))}\n")
            f.write("End\n")
    with open(os.path.join(directory, name + ".nets"), "w") as f:
        if netlist is None:
            f.write("UCLA nets 1.0\n\nNumNets : 0\nNumPins : 0\n")
        else:
            if np.any(netlist.pin_node >= n_real):
                raise ValueError("a pin on a filler cannot be written")
            f.write(f"UCLA nets 1.0\n\nNumNets : {netlist.num_nets}\nNumPins : {netlist.num_pins}\n\n")
            for e in range(netlist.num_nets):
                pins = netlist.net_pins[netlist.net_start[e]:netlist.net_start[e + 1]]
                f.write(f"NetDegree : {len(pins)}   n{e}\n")
                for q in pins:
                    v = int(netlist.pin_node[q])
                    dx = float(netlist.pin_offset_x[q]) - 0.5 * float(p.size_x[v])
                    dy = float(netlist.pin_offset_y[q]) - 0.5 * float(p.size_y[v])
                    f.write(f"\t{names[v]}  B : {dx!r} {dy!r}\n")
    aux = os.path.join(directory, name + ".aux")
    with open(aux, "w") as f:
        f.write(f"RowBasedPlacement : {name}.nodes {name}.nets {name}.wts {name}.pl {name}.scl\n")
    return aux


def main():
    import argparse
    ap = argparse.ArgumentParser(description="Summarise a bookshelf design as the engine sees it")
    ap.add_argument("aux")
    ap.add_argument("--bins", type=int, default=512)
    args = ap.parse_args()
    d = read_aux(args.aux)
    p = to_placement(d, args.bins, args.bins)
    print(json.dumps({"design": d.name, "die": d.die, "rows": len(d.rows), "movable": p.num_movable,
                      "terminals": p.num_terminals, "fillers": p.num_filler, "nets": d.num_nets,
                      "pins": d.num_pins, "bins": [p.num_bins_x, p.num_bins_y]}))


if __name__ == "__main__":
    main()
