"""Wirelength half of the placement objective on the device: the weighted-average
(WA) wirelength, its gradient and the HPWL (epb_wirelength in include/epb.h).

In the reference these come from DREAMPlace, which is absent from the
reference tree: benchmarks/configs/adaptec1_2048.json selects the
"weighted_average" wirelength with gamma 4.0 and ignore_net_degree 100, and
integration/run_dreamplace.py:315-370 reads the hpwl of every iteration from
EvalMetrics.  The netlist uses DREAMPlace's flat maps (netpin_start /
flat_netpin, pin2node_map, pin offsets from the node's lower-left corner,
flat_node2pin_start_map / flat_node2pin_map).

There is no CPU path: the op runs the CUDA kernels or raises.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib


@dataclass
class NetlistArrays:
    """A netlist on the host.  The pins of net e are
    net_pins[net_start[e]:net_start[e+1]]; every pin is listed once."""
    net_start: np.ndarray           # int32 [E + 1]
    net_pins: np.ndarray            # int32 [P]
    pin_node: np.ndarray            # int32 [P]
    pin_offset_x: np.ndarray        # float32 [P], from the node's lower-left corner
    pin_offset_y: np.ndarray
    num_nodes: int
    net_weight: Optional[np.ndarray] = None   # float32 [E]

    @property
    def num_nets(self) -> int:
        return len(self.net_start) - 1

    @property
    def num_pins(self) -> int:
        return len(self.net_pins)

    def node_pin_csr(self):
        """(node_pin_start [V + 1], node_pins [P]): the pins of each node in
        increasing pin order (DREAMPlace's flat_node2pin_start_map / _map)."""
        order = np.argsort(self.pin_node, kind="stable").astype(np.int32)
        counts = np.bincount(self.pin_node, minlength=self.num_nodes)
        start = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        return start, order

    def validate(self):
        E, P = self.num_nets, self.num_pins
        if self.net_start[0] != 0 or self.net_start[-1] != P or np.any(np.diff(self.net_start) < 0):
            raise ValueError("net_start must rise from 0 to num_pins")
        if not np.array_equal(np.sort(self.net_pins), np.arange(P)):
            raise ValueError("net_pins must list every pin exactly once")
        if P and (self.pin_node.min() < 0 or self.pin_node.max() >= self.num_nodes):
            raise ValueError("pin_node out of range")
        if self.net_weight is not None and len(self.net_weight) != E:
            raise ValueError("net_weight must have num_nets entries")


def synthetic_netlist(size_x, size_y, nodes, num_nodes, seed=0, nets_per_node=1.0, max_degree=400,
                      shuffle_pins=False):
    """Seeded nets over the given nodes, with degrees shaped like the ISPD-2005
    designs (mostly 2 and 3 pins, a tail past 100) and pin offsets inside each
    node's original outline.  A stand-in for the benchmark netlists, which are
    not available here.  Pins are numbered net by net, as a bookshelf reader
    numbers them while it reads the .nets file (net_pins is then 0..P-1);
    shuffle_pins numbers them in a random order instead."""
    rng = np.random.default_rng(seed)
    nodes = np.asarray(nodes, np.int64)
    E = max(1, int(round(len(nodes) * nets_per_node)))
    deg = 2 + np.floor(rng.exponential(1.6, E)).astype(np.int64)
    big = rng.random(E) < 0.002                      # a few nets beyond ignore_net_degree
    deg[big] = rng.integers(101, max_degree + 1, int(big.sum()))
    deg = np.minimum(deg, max_degree)
    P = int(deg.sum())
    net_start = np.concatenate([[0], np.cumsum(deg)]).astype(np.int32)
    pin_node = nodes[rng.integers(0, len(nodes), P)].astype(np.int32)
    sx = np.asarray(size_x, np.float32)[pin_node]
    sy = np.asarray(size_y, np.float32)[pin_node]
    ox = (rng.random(P, dtype=np.float32) * sx).astype(np.float32)
    oy = (rng.random(P, dtype=np.float32) * sy).astype(np.float32)
    net_pins = (rng.permutation(P) if shuffle_pins else np.arange(P)).astype(np.int32)
    # pin_node / offsets are indexed by pin id
    pn = np.empty(P, np.int32)
    pn[net_pins] = pin_node
    px = np.empty(P, np.float32)
    py = np.empty(P, np.float32)
    px[net_pins] = ox
    py[net_pins] = oy
    w = (1.0 + rng.random(E, dtype=np.float32)).astype(np.float32)
    return NetlistArrays(net_start, net_pins, pn, px, py, int(num_nodes), w)


class Netlist:
    """A netlist in device memory, ready for WirelengthOp."""

    def __init__(self, arrays: NetlistArrays, device, ignore_net_degree: int = 100, validate: bool = True):
        if validate:
            arrays.validate()
        d = torch.device(device)
        self.device = torch.device("cuda", torch.cuda.current_device() if d.index is None else d.index)
        self.arrays = arrays
        i32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(self.device)
        f32 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(self.device)
        nps, npn = arrays.node_pin_csr()
        self.net_start, self.net_pins, self.pin_node = i32(arrays.net_start), i32(arrays.net_pins), i32(arrays.pin_node)
        self.pin_offset_x, self.pin_offset_y = f32(arrays.pin_offset_x), f32(arrays.pin_offset_y)
        self.net_weight = None if arrays.net_weight is None else f32(arrays.net_weight)
        self.node_pin_start, self.node_pins = i32(nps), i32(npn)
        p = lambda t: None if t is None else t.data_ptr()
        self.c = _lib.EpbNetlist(p(self.net_start), p(self.net_pins), p(self.pin_node), p(self.pin_offset_x),
                                 p(self.pin_offset_y), p(self.net_weight), p(self.node_pin_start), p(self.node_pins),
                                 arrays.num_nets, arrays.num_pins, arrays.num_nodes, int(ignore_net_degree),
                                 self.device.index)


class WirelengthOp:
    """WA wirelength, HPWL and the WA gradient of every node, on the device.
    Allocation-free per call: the scratch is made once here."""

    def __init__(self, netlist: Netlist):
        if netlist.device.type != "cuda":
            raise ValueError("WirelengthOp needs a CUDA device")
        self.lib = _lib.load()
        self.nl = netlist
        nbytes = int(self.lib.epb_wirelength_scratch_bytes(netlist.arrays.num_pins))
        self.scratch = torch.empty(nbytes, dtype=torch.uint8, device=netlist.device)
        self.out = torch.zeros(2, dtype=torch.float64, device=netlist.device)
        self.flags = torch.zeros(1, dtype=torch.int32, device=netlist.device)
        self._err = ctypes.create_string_buffer(256)

    def __call__(self, x: torch.Tensor, y: torch.Tensor, gamma: float, grad_x: Optional[torch.Tensor] = None,
                 grad_y: Optional[torch.Tensor] = None, want_grad: bool = True, stream=None):
        """{"wirelength": WA, "hpwl": HPWL} as device fp64 scalars, and the WA
        gradient of every node in grad_x / grad_y (allocated when not given)."""
        V = self.nl.arrays.num_nodes
        for name, t in (("x", x), ("y", y)):
            if t.dtype != torch.float32 or t.device != self.nl.device or t.numel() < V or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous float32 tensor of {V} nodes on {self.nl.device}")
        if want_grad:
            if grad_x is None:
                grad_x = torch.empty(V, dtype=torch.float32, device=self.nl.device)
            if grad_y is None:
                grad_y = torch.empty(V, dtype=torch.float32, device=self.nl.device)
        else:
            grad_x = grad_y = None
        st = torch.cuda.current_stream(self.nl.device) if stream is None else stream
        p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())
        rc = self.lib.epb_wirelength(ctypes.byref(self.nl.c), p(x), p(y), float(gamma), ctypes.c_void_p(st.cuda_stream),
                                     p(self.scratch), self.scratch.numel(), p(self.out), p(grad_x), p(grad_y),
                                     p(self.flags), self._err, len(self._err))
        if rc != _lib.EPB_OK:
            raise _lib.EpbError(rc, self._err.value.decode() or _lib.load().epb_status_string(rc).decode())
        return {"wirelength": self.out[0], "hpwl": self.out[1], "grad_x": grad_x, "grad_y": grad_y}

    def error_flags(self) -> int:
        """Flags OR-ed in by every call since the last clear_flags (synchronises):
        EPB_FLAG_BAD_INDEX (0x10), EPB_FLAG_NONFINITE_CELL (0x1)."""
        return int(self.flags.item())

    def clear_flags(self):
        self.flags.zero_()
