"""CPU oracle for the placement loop's wirelength terms.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, as the checker.  The product
package never imports it.

The reference hands these terms to DREAMPlace, which is absent from the
reference tree (an un-vendored submodule, README.md:54-59).  What the
reference shows is the call surface around them:
* integration/run_dreamplace.py:315-331 wraps NonLinearPlace.__call__ and reads
  the last iteration's hpwl and overflow;
* integration/run_dreamplace.py:333-370 wraps EvalMetrics.evaluate to log the
  hpwl and overflow of every iteration;
* benchmarks/configs/adaptec1_2048.json selects "wirelength":
  "weighted_average" with gamma 4.0 and ignore_net_degree 100.

The weighted-average (WA) wirelength restated here is the published form
(Hsu, Chang and Balabanov, DAC 2011; used by DREAMPlace).  For a net e and one
axis, with pin coordinates x_i:
    WA_e = sum_i x_i exp(x_i/g) / sum_i exp(x_i/g) - sum_i x_i exp(-x_i/g) / sum_i exp(-x_i/g)
    dWA_e/dx_i = (a_i/b)(1 + (x_i - f)/g) - (a'_i/b')(1 - (x_i - f')/g)
where a_i = exp((x_i - max x)/g), b = sum a_i, f = sum x_i a_i / b, and
a'_i = exp((min x - x_i)/g), b' = sum a'_i, f' = sum x_i a'_i / b' (the shifts
cancel in every ratio).  A pin sits at its node's lower-left corner plus the
pin offset, added in fp32 as the device does.  Nets with fewer than 2 pins
contribute nothing; nets with more than ignore_net_degree pins are left out
of the WA objective (DREAMPlace's ignore_net_degree) but kept in the HPWL.
HPWL_e = (max x - min x) + (max y - min y).  Both are weighted by the net
weight.  Node gradients sum the gradients of the node's pins.

Everything after the pin positions is float64.

Parity unpinned against DREAMPlace: its wirelength op is absent here, and the
reference holds no golden values for it.  The restatement is pinned to
mathematics instead: the closed form of a two-pin net (L tanh(L / 2g)),
central finite differences of the gradient, and the degree cap and weights
(tests/test_wirelength.py).
"""
from __future__ import annotations

import numpy as np


def pin_positions(x, y, pin_node, pin_ox, pin_oy):
    """fp32 pin coordinates: node corner + pin offset, one fp32 addition each."""
    px = (np.asarray(x, np.float32)[pin_node] + np.asarray(pin_ox, np.float32)).astype(np.float32)
    py = (np.asarray(y, np.float32)[pin_node] + np.asarray(pin_oy, np.float32)).astype(np.float32)
    return px, py


def _axis(v, net_of, starts, g):
    """WA value per net and WA gradient per (net-ordered) pin along one axis."""
    vmax = np.maximum.reduceat(v, starts)
    vmin = np.minimum.reduceat(v, starts)
    a = np.exp((v - vmax[net_of]) / g)
    an = np.exp((vmin[net_of] - v) / g)
    b = np.add.reduceat(a, starts)
    bn = np.add.reduceat(an, starts)
    f = np.add.reduceat(v * a, starts) / b
    fn = np.add.reduceat(v * an, starts) / bn
    wa = f - fn
    grad = (a / b[net_of]) * (1.0 + (v - f[net_of]) / g) - (an / bn[net_of]) * (1.0 - (v - fn[net_of]) / g)
    return wa, grad, vmax - vmin


def wirelength(x, y, net_start, net_pins, pin_node, pin_ox, pin_oy, gamma, num_nodes,
               net_weight=None, ignore_net_degree=100):
    """(WA wirelength, HPWL, grad_x[num_nodes], grad_y[num_nodes]) in float64.

    net_start [E+1] / net_pins [P]: the pins of net e are net_pins[net_start[e]:net_start[e+1]]
    (DREAMPlace's netpin_start / flat_netpin); pin_node [P] maps a pin to its node."""
    net_start = np.asarray(net_start, np.int64)
    net_pins = np.asarray(net_pins, np.int64)
    pin_node = np.asarray(pin_node, np.int64)
    E = len(net_start) - 1
    deg = np.diff(net_start)
    w = np.ones(E) if net_weight is None else np.asarray(net_weight, np.float64)
    px32, py32 = pin_positions(x, y, pin_node, pin_ox, pin_oy)
    gx = np.zeros(num_nodes)
    gy = np.zeros(num_nodes)
    wl = hp = 0.0
    used = deg >= 2
    if not used.any():
        return 0.0, 0.0, gx, gy
    idx = np.nonzero(used)[0]
    # the pin slots of the used nets, net by net: net_start[e] + j for j < deg[e]
    d = deg[idx]
    starts = (np.cumsum(d) - d).astype(np.int64)          # where each used net begins
    seg = np.repeat(net_start[idx], d) + (np.arange(d.sum()) - np.repeat(starts, d))
    pins = net_pins[seg]
    net_of = np.repeat(np.arange(len(idx)), deg[idx])
    g = float(gamma)
    vx = px32[pins].astype(np.float64)
    vy = py32[pins].astype(np.float64)
    wax, gax, hx = _axis(vx, net_of, starts, g)
    way, gay, hy = _axis(vy, net_of, starts, g)
    we = w[idx]
    hp = float(np.sum(we * (hx + hy)))
    in_wa = deg[idx] <= ignore_net_degree
    wl = float(np.sum((we * (wax + way))[in_wa]))
    pw = (we * in_wa)[net_of]
    np.add.at(gx, pin_node[pins], pw * gax)
    np.add.at(gy, pin_node[pins], pw * gay)
    return wl, hp, gx, gy


def node_pin_csr(pin_node, num_nodes):
    """DREAMPlace's flat_node2pin_start_map / flat_node2pin_map: the pins of each
    node in increasing pin order."""
    pin_node = np.asarray(pin_node, np.int64)
    order = np.argsort(pin_node, kind="stable").astype(np.int32)
    counts = np.bincount(pin_node, minlength=num_nodes)
    start = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return start, order
