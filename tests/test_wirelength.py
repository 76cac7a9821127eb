"""Wirelength half of the placement objective: the WA wirelength, its gradient
and the HPWL (epb_wirelength) against the CPU restatement in
oracle/wirelength.py.

CPU: the restatement's closed form for a two-pin net, its gradient against
finite differences, the degree cap and the net weights; the synthetic
netlists; the C ABI's argument checks.  GPU: the device result against the
restatement, run-to-run determinism and out-of-range indices."""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch

from dreamplacett_framework_b200 import synth
from dreamplacett_framework_b200.wirelength import NetlistArrays, synthetic_netlist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
import wirelength as wlo  # noqa: E402  (the CPU restatement)


def _two_pin(x0, x1, w=None):
    arr = NetlistArrays(np.array([0, 2], np.int32), np.array([0, 1], np.int32), np.array([0, 1], np.int32),
                        np.zeros(2, np.float32), np.zeros(2, np.float32), 2, w)
    x = np.array([x0, x1], np.float32)
    return arr, x, np.array([5.0, 5.0], np.float32)


def _oracle(arr, x, y, gamma, ignore=100):
    return wlo.wirelength(x, y, arr.net_start, arr.net_pins, arr.pin_node, arr.pin_offset_x, arr.pin_offset_y,
                          gamma, arr.num_nodes, arr.net_weight, ignore)


def _small_random(seed=0, n=60, E=40, max_deg=7):
    rng = np.random.default_rng(seed)
    deg = rng.integers(1, max_deg, E)
    ns = np.concatenate([[0], np.cumsum(deg)]).astype(np.int32)
    P = int(ns[-1])
    arr = NetlistArrays(ns, rng.permutation(P).astype(np.int32), rng.integers(0, n, P).astype(np.int32),
                        rng.integers(0, 4, P).astype(np.float32), rng.integers(0, 4, P).astype(np.float32), n,
                        (1 + rng.random(E)).astype(np.float32))
    x = rng.integers(0, 200, n).astype(np.float32)
    y = rng.integers(0, 200, n).astype(np.float32)
    return arr, x, y


# ---------------------------------------------------------------- CPU ----

@pytest.mark.parametrize("gamma", [0.5, 1.0, 4.0, 16.0])
def test_two_pin_net_closed_form(gamma):
    """Two pins L apart: WA = L tanh(L / 2g), HPWL = L, gradients -+ dWA/dL."""
    arr, x, y = _two_pin(3.0, 13.0)
    wl, hp, gx, gy = _oracle(arr, x, y, gamma)
    L = 10.0
    assert wl == pytest.approx(L * np.tanh(L / (2 * gamma)), rel=1e-12)
    assert hp == L
    d = np.tanh(L / (2 * gamma)) + L / (2 * gamma) / np.cosh(L / (2 * gamma)) ** 2
    np.testing.assert_allclose(gx, [-d, d], rtol=1e-12)
    np.testing.assert_array_equal(gy, [0.0, 0.0])


def test_gradient_matches_finite_differences():
    arr, x, y = _small_random()
    gamma = 6.0
    _, _, gx, gy = _oracle(arr, x, y, gamma)
    h = 0.25   # exact in fp32 at these coordinates
    for i in range(0, arr.num_nodes, 7):
        for v, g in ((x, gx), (y, gy)):
            vp, vm = v.copy(), v.copy()
            vp[i] += h
            vm[i] -= h
            args = (vp, y) if v is x else (x, vp)
            argm = (vm, y) if v is x else (x, vm)
            num = (_oracle(arr, *args, gamma)[0] - _oracle(arr, *argm, gamma)[0]) / (2 * h)
            assert num == pytest.approx(g[i], rel=2e-3, abs=2e-3)


def test_degree_cap_and_weights():
    arr, x, y = _small_random(seed=1, max_deg=9)
    full = _oracle(arr, x, y, 3.0, ignore=100)
    capped = _oracle(arr, x, y, 3.0, ignore=4)
    assert capped[1] == full[1]                    # HPWL keeps every net
    assert capped[0] < full[0]                     # the WA leaves the big nets out
    deg = np.diff(arr.net_start)
    keep = np.nonzero((deg >= 2) & (deg <= 4))[0]
    # the capped WA is the WA of the kept nets alone
    sub_ns = np.concatenate([[0], np.cumsum(deg[keep])]).astype(np.int32)
    sub_pins = np.concatenate([arr.net_pins[arr.net_start[e]:arr.net_start[e + 1]] for e in keep])
    sub = NetlistArrays(sub_ns, sub_pins, arr.pin_node, arr.pin_offset_x, arr.pin_offset_y, arr.num_nodes,
                        arr.net_weight[keep])
    assert _oracle(sub, x, y, 3.0)[0] == pytest.approx(capped[0], rel=1e-12)
    twice = NetlistArrays(arr.net_start, arr.net_pins, arr.pin_node, arr.pin_offset_x, arr.pin_offset_y,
                          arr.num_nodes, 2 * arr.net_weight)
    t = _oracle(twice, x, y, 3.0)
    assert t[0] == pytest.approx(2 * full[0], rel=1e-12) and t[1] == pytest.approx(2 * full[1], rel=1e-12)
    np.testing.assert_allclose(t[2], 2 * full[2], rtol=1e-12, atol=1e-15)


@pytest.mark.parametrize("shuffle", [False, True])
def test_synthetic_netlist_shape(shuffle):
    p = synth.make_placement("c1", scale=0.05)
    arr = synthetic_netlist(p.size_x, p.size_y, np.arange(p.num_movable), p.num_nodes, seed=3, shuffle_pins=shuffle)
    arr.validate()
    assert np.array_equal(arr.net_pins, np.arange(arr.num_pins)) != shuffle
    deg = np.diff(arr.net_start)
    assert deg.min() >= 2 and (deg > 100).any() and np.mean(deg) < 6
    # offsets inside the pin's node
    assert np.all(arr.pin_offset_x < p.size_x[arr.pin_node]) and np.all(arr.pin_offset_x >= 0)
    start, order = arr.node_pin_csr()
    s2, o2 = wlo.node_pin_csr(arr.pin_node, arr.num_nodes)
    np.testing.assert_array_equal(start, s2)
    np.testing.assert_array_equal(order, o2)
    assert np.all(np.diff(arr.pin_node[order]) >= 0)


def test_abi_rejects_bad_arguments_without_cuda():
    from dreamplacett_framework_b200 import _lib, build
    build.build()
    L = _lib.load()
    # the block counter, 1184 block partials (WA, HPWL), then pin gradients and pin positions
    assert L.epb_wirelength_scratch_bytes(1000) == 16 + 16 * 1184 + 16 * 1000
    fake = ctypes.c_void_p(1 << 20)   # never dereferenced: every case fails its host check first
    nl = _lib.EpbNetlist(fake, fake, fake, fake, fake, None, fake, fake, 10, 20, 5, 100, 0)
    err = ctypes.create_string_buffer(128)
    big = L.epb_wirelength_scratch_bytes(20)
    cases = [
        (None, 1.0, big, fake),                                  # no netlist
        (ctypes.byref(nl), 0.0, big, fake),                      # gamma <= 0
        (ctypes.byref(nl), float("nan"), big, fake),
        (ctypes.byref(nl), 1.0, big - 1, fake),                  # scratch too small
        (ctypes.byref(nl), 1.0, big, ctypes.c_void_p((1 << 20) + 8)),   # scratch misaligned
    ]
    for nlp, gamma, nbytes, scratch in cases:
        rc = L.epb_wirelength(nlp, fake, fake, gamma, None, scratch, nbytes, fake, fake, fake, None, err, 128)
        assert rc == _lib.EPB_EINVAL and err.value
    bad = _lib.EpbNetlist(fake, fake, fake, fake, fake, None, fake, fake, -1, 20, 5, 100, 0)
    assert L.epb_wirelength(ctypes.byref(bad), fake, fake, 1.0, None, fake, big, fake, None, None, None, err,
                            128) == _lib.EPB_EINVAL


# ---------------------------------------------------------------- GPU ----

def _device_op(arr, device, ignore=100):
    from dreamplacett_framework_b200.wirelength import Netlist, WirelengthOp
    return WirelengthOp(Netlist(arr, device, ignore_net_degree=ignore, validate=False))


@pytest.mark.gpu
@pytest.mark.parametrize("config,scale,ignore,shuffle", [("c1", 0.2, 100, False), ("c3", 0.05, 100, True),
                                                         ("c1", 0.05, 4, True)])
def test_wirelength_matches_oracle(cuda_device, config, scale, ignore, shuffle):
    p = synth.make_placement(config, scale=scale)
    arr = synthetic_netlist(p.size_x, p.size_y, np.arange(p.num_movable), p.num_nodes, seed=7, shuffle_pins=shuffle)
    gamma = 4.0 * p.bin_size_x
    wl, hp, gx, gy = _oracle(arr, p.x, p.y, gamma, ignore)
    op = _device_op(arr, cuda_device, ignore)
    x = torch.from_numpy(p.x).to(cuda_device)
    y = torch.from_numpy(p.y).to(cuda_device)
    r = op(x, y, gamma)
    assert float(r["wirelength"].item()) == pytest.approx(wl, rel=1e-5)
    assert float(r["hpwl"].item()) == pytest.approx(hp, rel=1e-6)
    for a, b in ((r["grad_x"], gx), (r["grad_y"], gy)):
        a = a.cpu().numpy().astype(np.float64)
        assert np.max(np.abs(a - b)) / np.max(np.abs(b)) < 1e-5
    assert op.error_flags() == 0


@pytest.mark.gpu
def test_wirelength_is_deterministic(cuda_device):
    p = synth.make_placement("c3", scale=0.05)
    arr = synthetic_netlist(p.size_x, p.size_y, np.arange(p.num_movable), p.num_nodes, seed=8)
    op = _device_op(arr, cuda_device)
    x = torch.from_numpy(p.x).to(cuda_device)
    y = torch.from_numpy(p.y).to(cuda_device)
    a = {k: v.clone() for k, v in op(x, y, 40.0).items()}
    b = op(x, y, 40.0)
    for k in a:
        assert torch.equal(a[k], b[k]), k


@pytest.mark.gpu
def test_wirelength_skips_out_of_range_entries(cuda_device):
    """A pin whose node index is out of range is reported and its net skipped;
    every other net is computed as usual."""
    arr, x, y = _small_random(seed=2)
    good = _oracle(arr, x, y, 5.0)
    deg = np.diff(arr.net_start)
    e = int(np.nonzero(deg >= 2)[0][0])
    victim = arr.net_pins[arr.net_start[e]]
    bad_node = arr.pin_node.copy()
    bad_node[victim] = arr.num_nodes + 5
    bad = NetlistArrays(arr.net_start, arr.net_pins, bad_node, arr.pin_offset_x, arr.pin_offset_y, arr.num_nodes,
                        arr.net_weight)
    op = _device_op(bad, cuda_device)
    r = op(torch.from_numpy(x).to(cuda_device), torch.from_numpy(y).to(cuda_device), 5.0, want_grad=False)
    assert op.error_flags() & 0x10
    # the result is the netlist without net e
    keep = [k for k in range(arr.num_nets) if k != e]
    sub_ns = np.concatenate([[0], np.cumsum(deg[keep])]).astype(np.int32)
    sub_pins = np.concatenate([arr.net_pins[arr.net_start[k]:arr.net_start[k + 1]] for k in keep])
    sub = NetlistArrays(sub_ns, sub_pins, arr.pin_node, arr.pin_offset_x, arr.pin_offset_y, arr.num_nodes,
                        arr.net_weight[keep])
    ref = _oracle(sub, x, y, 5.0)
    assert float(r["wirelength"].item()) == pytest.approx(ref[0], rel=1e-5)
    assert float(r["hpwl"].item()) == pytest.approx(ref[1], rel=1e-6)
    assert ref[1] < good[1]
