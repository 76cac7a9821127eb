"""Bookshelf (ISPD-2005) reader: a hand-written design with known answers, a
write -> read round trip of a synthetic design, the reference-style JSON
config, and (GPU) the engine on a design loaded from files."""
import json
import os

import numpy as np
import pytest

from dreamplacett_framework_b200 import bookshelf, synth

TINY = {
    "t.aux": "RowBasedPlacement : t.nodes t.nets t.wts t.pl t.scl\n",
    "t.nodes": """UCLA nodes 1.0
# comment line
NumNodes : 5
NumTerminals : 2
   a   4   10
   b   6   10
   m   20  20  terminal
   p   1   1   terminal_NI
   c   8   10
""",
    "t.pl": """UCLA pl 1.0
a 1 2 : N
b 3.5 4 : N
m 30 0 : N /FIXED
p 0 0 : N /FIXED_NI
c 10 10 : N
""",
    "t.scl": """UCLA scl 1.0
NumRows : 2
CoreRow Horizontal
  Coordinate    :   0
  Height        :   10
  Sitewidth     :    1
  Sitespacing   :    1
  Siteorient    :    1
  Sitesymmetry  :    1
  SubrowOrigin  :    0	NumSites  :  40
End
CoreRow Horizontal
  Coordinate    :   10
  Height        :   10
  Sitewidth     :    1
  Sitespacing   :    1
  Siteorient    :    1
  Sitesymmetry  :    1
  SubrowOrigin  :    0	NumSites  :  40
End
""",
    "t.nets": """UCLA nets 1.0
NumNets : 2
NumPins : 5
NetDegree : 3 n0
  a I : 0 0
  b O : 0 0
  c I : 0 0
NetDegree : 2 n1
  a I : 0 0
  m O : 0 0
""",
}


def _write_tiny(d):
    for name, text in TINY.items():
        (d / name).write_text(text)
    return str(d / "t.aux")


def test_tiny_design_known_answers(tmp_path):
    d = bookshelf.read_aux(_write_tiny(tmp_path))
    assert d.names == ["a", "b", "m", "p", "c"]
    assert list(d.kind) == [0, 0, 1, 2, 0]
    assert d.die == (0.0, 0.0, 40.0, 20.0)
    assert (d.num_nets, d.num_pins) == (2, 5)
    assert d.x[1] == 3.5 and d.y[1] == 4.0
    # fillers: widths 4, 6, 8 -> 5%..95% slice [0:2] of the sorted widths = mean(4, 6) = 5;
    # fixed area inside the die = 10 x 20 (the macro at x = 30 reaches 50 > 40);
    # free = 1.0 * (800 - 200) - (40 + 60 + 80) = 420 -> round(420 / (5 * 10)) = 8
    assert bookshelf.filler_plan(d, 1.0) == (8, 5.0, 10.0)
    p = bookshelf.to_placement(d, 16, 16, seed=3)
    # DREAMPlace's order: [movable | terminal | terminal_NI | fillers]
    assert (p.num_movable, p.num_terminals, p.num_filler) == (3, 2, 8)
    np.testing.assert_array_equal(p.size_x[:5], np.array([4, 6, 8, 20, 1], np.float32))
    assert p.ranges == ((0, 3), (5, 13))
    # only the terminal (not the terminal_NI pin) is in the fixed-cell density
    assert p.initial_density_map.sum() == pytest.approx(200.0)
    assert np.all(p.x[5:] >= 0) and np.all(p.x[5:] + 5.0 <= 40.0 + 1e-9)


def test_tiny_netlist_offsets(tmp_path):
    """Pins in file order, nodes in DREAMPlace's order, offsets from the lower-left
    corner (w/2 + dx, h/2 + dy)."""
    aux = _write_tiny(tmp_path)
    (tmp_path / "t.nets").write_text(TINY["t.nets"].replace("  c I : 0 0", "  c I : 1.5 -2")
                                     .replace("  m O : 0 0", "  m O"))
    p = bookshelf.to_placement(bookshelf.read_aux(aux), 16, 16, enable_fillers=False)
    nl = bookshelf.netlist_for_placement(aux, p)
    nl.validate()
    np.testing.assert_array_equal(nl.net_start, [0, 3, 5])
    # order [a, b, c | m | p] -> a=0, b=1, c=2, m=3
    np.testing.assert_array_equal(nl.pin_node, [0, 1, 2, 0, 3])
    np.testing.assert_array_equal(nl.pin_offset_x, np.array([2, 3, 4 + 1.5, 2, 10], np.float32))
    np.testing.assert_array_equal(nl.pin_offset_y, np.array([5, 5, 5 - 2, 5, 10], np.float32))
    assert nl.num_nodes == p.num_nodes


@pytest.mark.parametrize("nets,msg", [
    ("NetDegree : 2 n0\n  a I : 0 0\n  zz O : 0 0\n", "unknown node"),
    ("  a I : 0 0\nNetDegree : 1 n0\n  b I\n", "outside a net"),
    ("NetDegree : 3 n0\n  a I\n  b I\nNetDegree : 1 n1\n  c I\n", "early"),
    ("NetDegree : 2 n0\n  a I\n", "early"),
])
def test_malformed_netlists_are_reported(tmp_path, nets, msg):
    aux = _write_tiny(tmp_path)
    (tmp_path / "t.nets").write_text("UCLA nets 1.0\n" + nets)
    p = bookshelf.to_placement(bookshelf.read_aux(aux), 16, 16, enable_fillers=False)
    with pytest.raises(ValueError, match=msg):
        bookshelf.netlist_for_placement(aux, p)


def test_netlist_round_trip(tmp_path):
    import sys
    from dreamplacett_framework_b200.wirelength import synthetic_netlist
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import wirelength as wlo
    p = synth.make_placement("c1", scale=0.01)
    n_real = p.num_movable + p.num_terminals
    arr = synthetic_netlist(p.size_x, p.size_y, np.arange(n_real), p.num_nodes, seed=5)
    aux = bookshelf.write_bookshelf(p, str(tmp_path), "nl", netlist=arr)
    d = bookshelf.read_aux(aux)
    assert (d.num_nets, d.num_pins) == (arr.num_nets, arr.num_pins)
    q = bookshelf.to_placement(d, p.num_bins_x, p.num_bins_y, enable_fillers=False)
    got = bookshelf.netlist_for_placement(aux, q)
    got.validate()
    np.testing.assert_array_equal(got.net_start, arr.net_start)
    np.testing.assert_array_equal(got.pin_node, arr.pin_node[arr.net_pins])
    np.testing.assert_allclose(got.pin_offset_x, arr.pin_offset_x[arr.net_pins], rtol=0, atol=1e-4)
    np.testing.assert_allclose(got.pin_offset_y, arr.pin_offset_y[arr.net_pins], rtol=0, atol=1e-4)
    # the same design: the same HPWL (unit weights on both sides)
    a = wlo.wirelength(p.x, p.y, arr.net_start, arr.net_pins, arr.pin_node, arr.pin_offset_x, arr.pin_offset_y,
                       4.0, p.num_nodes)
    b = wlo.wirelength(q.x, q.y, got.net_start, got.net_pins, got.pin_node, got.pin_offset_x, got.pin_offset_y,
                       4.0, q.num_nodes)
    assert b[1] == pytest.approx(a[1], rel=1e-6) and b[0] == pytest.approx(a[0], rel=1e-6)


def test_round_trip_of_synthetic_design(tmp_path):
    p = synth.make_placement("c3", scale=0.01)
    aux = bookshelf.write_bookshelf(p, str(tmp_path), "c3s")
    q = bookshelf.to_placement(bookshelf.read_aux(aux), p.num_bins_x, p.num_bins_y, enable_fillers=False)
    n = p.num_movable + p.num_terminals
    assert (q.num_movable, q.num_terminals, q.num_filler) == (p.num_movable, p.num_terminals, 0)
    assert (q.xl, q.yl, q.xh, q.yh) == (p.xl, p.yl, p.xh, p.yh)
    for k in ("x", "y", "size_x", "size_y", "size_x_clamped", "size_y_clamped", "offset_x", "offset_y", "ratio"):
        np.testing.assert_array_equal(getattr(q, k), getattr(p, k)[:n], err_msg=k)
    np.testing.assert_array_equal(q.initial_density_map, p.initial_density_map)


def test_reference_style_config(tmp_path):
    aux = _write_tiny(tmp_path)
    cfg = {"aux_input": os.path.basename(aux), "num_bins_x": 64, "num_bins_y": 64,
           "global_place_stages": [{"num_bins_x": 32, "num_bins_y": 16, "iteration": 100}],
           "target_density": 0.9, "density_weight": 8e-05, "enable_fillers": 1, "random_seed": 7,
           "random_center_init_flag": 1}
    path = tmp_path / "design.json"
    path.write_text(json.dumps(cfg))
    c = bookshelf.load_config(str(path))
    assert (c["num_bins_x"], c["num_bins_y"], c["iterations"]) == (32, 16, 100)
    assert c["target_density"] == 0.9 and c["density_weight"] == 8e-05
    p = bookshelf.placement_from_config(str(path))
    assert (p.num_bins_x, p.num_bins_y) == (32, 16)
    # random centre init: movable cells start near the die centre
    cx = p.x[:3] + 0.5 * p.size_x[:3]
    assert np.all(np.abs(cx - 20.0) < 1.0)


def test_missing_files_are_reported(tmp_path):
    (tmp_path / "x.aux").write_text("RowBasedPlacement : x.nodes x.nets\n")
    with pytest.raises(ValueError):
        bookshelf.read_aux(str(tmp_path / "x.aux"))


@pytest.mark.gpu
def test_engine_on_bookshelf_design(oracle, cuda_device, tmp_path):
    """Density of a design loaded from bookshelf files: bit-exact against the oracle."""
    import torch
    from gpu_util import engine_for, geometry_for, np_, placement_cells, to_device, to_oracle
    src = synth.make_placement("c3", scale=0.05, grid=512)
    aux = bookshelf.write_bookshelf(src, str(tmp_path), "d")
    p = bookshelf.to_placement(bookshelf.read_aux(aux), 512, 512, seed=5)
    arrs, ranges = placement_cells(p)
    g = geometry_for(oracle, p)
    grid, _ = oracle.density_fixed(to_oracle(oracle, arrs, ranges), g, g.default_fixed_bits())
    rho, _ = oracle.fixed_to_density(grid, g, g.default_fixed_bits(), p.initial_density_norm())
    with engine_for(p, cuda_device) as eng:
        eng.set_initial_density(torch.from_numpy(p.initial_density_norm()).to(cuda_device))
        out = eng.forward(to_device(arrs, ranges, cuda_device))
        np.testing.assert_array_equal(np_(out["density"]), rho)
        assert eng.error_flags() == 0
