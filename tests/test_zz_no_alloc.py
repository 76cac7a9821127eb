"""The allocation-free density entry point, epb_density_noalloc.

Some callers cannot allocate device memory: their memory belongs to another
allocator (a framework's caching allocator or a fixed pool that accounts for
every byte), or they run on a path where cudaMalloc/cudaFree, which can
synchronise the whole device, are not acceptable.  For them the library keeps
the density accumulation grid in a fixed device array of its own
(EPB_NOALLOC_MAX_BINS bins) and needs no handle.

This file checks, through the C ABI, that two calls in a row give exactly the
density map of the regular entry point (epb_forward), including a second call
on a smaller grid that would show any leftovers of the first, and that a grid
beyond the limit is refused with a message.  It is named so pytest collects
it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from dreamplacett_framework_b200 import _lib, synth
from dreamplacett_framework_b200.engine import CellTensors, ElectricPotentialEngine

pytestmark = pytest.mark.gpu


def _device_cells(p, dev):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
    return CellTensors(t(p.x), t(p.y), t(p.size_x_clamped), t(p.size_y_clamped), t(p.offset_x), t(p.offset_y),
                       t(p.ratio), ranges=p.ranges)


def _cells_struct(c):
    (b0, e0), (b1, e1) = c.resolved_ranges()
    ptr = lambda t: None if t is None else t.data_ptr()
    return _lib.EpbCells(ptr(c.x), ptr(c.y), ptr(c.size_x), ptr(c.size_y), ptr(c.offset_x), ptr(c.offset_y),
                         ptr(c.ratio), b0, e0, b1, e1)


def _noalloc_density(lib, p, cells, init, dev):
    cfg = _lib.EpbConfig(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh, 0, dev.index, 0, 0)
    out = torch.full((p.num_bins_x, p.num_bins_y), float("nan"), dtype=torch.float32, device=dev)
    err = ctypes.create_string_buffer(256)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    st = lib.epb_density_noalloc(ctypes.byref(cfg), ctypes.byref(_cells_struct(cells)),
                                 None if init is None else init.data_ptr(), stream, out.data_ptr(), err, len(err))
    assert st == _lib.EPB_OK, err.value.decode()
    return out


def _regular_density(p, cells, init, dev):
    with ElectricPotentialEngine(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh, device=dev) as eng:
        if init is not None:
            eng.set_initial_density(init)
        out = eng.forward(cells, want_potential=False, want_fields=False, want_energy=False)
        return out["density"].clone()


def test_noalloc_matches_regular_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but CUDA is not available")
    dev = torch.device("cuda", 0)
    lib = _lib.load()
    # first call: 1024 x 1024 bins (the largest accepted), many cells and fixed macros
    p1 = synth.make_placement("c3", scale=0.25, grid=1024)
    c1 = _device_cells(p1, dev)
    init1 = torch.from_numpy(p1.initial_density_norm()).to(dev)
    got1 = _noalloc_density(lib, p1, c1, init1, dev)
    # second call right after: a smaller grid and other cells; leftovers of the
    # first call in the shared array would show up here
    p2 = synth.make_placement("c1", scale=0.5)
    c2 = _device_cells(p2, dev)
    got2 = _noalloc_density(lib, p2, c2, None, dev)
    torch.cuda.synchronize(dev)
    ref1 = _regular_density(p1, c1, init1, dev)
    ref2 = _regular_density(p2, c2, None, dev)
    # the density map is bit-exact between entry points (same integer sums, same conversion)
    assert torch.equal(got1, ref1)
    assert torch.equal(got2, ref2)
    assert float(got2.sum()) > 0


def test_noalloc_refuses_grids_beyond_its_limit():
    lib = _lib.load()
    cfg = _lib.EpbConfig(2048, 1024, 0.0, 0.0, 1.0, 1.0, 0, 0, 0, 0)
    z = _lib.EpbCells(None, None, None, None, None, None, None, 0, 0, 0, 0)
    err = ctypes.create_string_buffer(256)
    st = lib.epb_density_noalloc(ctypes.byref(cfg), ctypes.byref(z), None, None, ctypes.c_void_p(1), err, len(err))
    assert st == _lib.EPB_EINVAL
    assert b"exceeds the allocation-free limit" in err.value
    assert 2048 * 1024 > _lib.NOALLOC_MAX_BINS


@pytest.mark.parametrize("box", [(0.0, 0.0, float("inf"), 1.0), (0.0, float("nan"), 1.0, 1.0),
                                 (float("-inf"), 0.0, 1.0, 1.0), (1.0, 0.0, 1.0, 1.0)])
def test_noalloc_refuses_bad_die_box(box):
    """Non-finite or empty die bounds are refused before any device work, as
    epb_create refuses them."""
    lib = _lib.load()
    cfg = _lib.EpbConfig(64, 64, *box, 0, 0, 0, 0)
    z = _lib.EpbCells(None, None, None, None, None, None, None, 0, 0, 0, 0)
    err = ctypes.create_string_buffer(256)
    st = lib.epb_density_noalloc(ctypes.byref(cfg), ctypes.byref(z), None, None, ctypes.c_void_p(1), err, len(err))
    assert st == _lib.EPB_EINVAL
    assert b"invalid die box" in err.value
