"""Torch-facing wrapper of the C-ABI engine (libepb200.so).

PyTorch provides device memory and streams; every computation is a call into
the CUDA engine.  There is no CPU path: constructing an engine without CUDA or
without the built library raises.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch

from . import _lib


@dataclass
class CellTensors:
    """Cells in DREAMPlace's node layout (see epb_cells in include/epb.h).

    x, y, size_x, size_y (and optional offset_x, offset_y, ratio) are fp32
    CUDA tensors indexed by node.  ranges = ((begin0, end0), (begin1, end1))
    selects the scattered nodes, by default all of them."""
    x: torch.Tensor
    y: torch.Tensor
    size_x: torch.Tensor
    size_y: torch.Tensor
    offset_x: Optional[torch.Tensor] = None
    offset_y: Optional[torch.Tensor] = None
    ratio: Optional[torch.Tensor] = None
    ranges: Optional[Tuple[Tuple[int, int], Tuple[int, int]]] = None

    @property
    def num_nodes(self) -> int:
        return int(self.x.numel())

    def resolved_ranges(self):
        if self.ranges is None:
            return (0, self.num_nodes), (0, 0)
        return self.ranges

    @property
    def count(self) -> int:
        (b0, e0), (b1, e1) = self.resolved_ranges()
        return (e0 - b0) + (e1 - b1)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _check_f32(name, t, device, n=None):
    if t is None:
        return
    if not t.is_cuda or t.device != device:
        raise ValueError(f"{name} must be a CUDA tensor on {device}")
    if t.dtype != torch.float32:
        raise ValueError(f"{name} must be float32 (got {t.dtype})")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if n is not None and t.numel() < n:
        raise ValueError(f"{name} has {t.numel()} elements, need {n}")


def _stream_ptr(stream: Optional[torch.cuda.Stream], device):
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return ctypes.c_void_p(s.cuda_stream)


class ElectricPotentialEngine:
    """One placement grid on one GPU.

    Mirrors the reference server's lifetime (start -> call* -> stop,
    integration/scatter_ttnn_client.py:293-407) as create -> forward/backward*
    -> close, in process, on device tensors."""

    def __init__(self, num_bins_x: int, num_bins_y: int, xl: float, yl: float, xh: float, yh: float,
                 fixed_point_bits: int = 0, device=None, path: Optional[str] = None):
        if not torch.cuda.is_available():
            raise RuntimeError("ElectricPotentialEngine needs a CUDA device (no CPU path)")
        self.lib = _lib.load()
        idx = None if device is None else torch.device(device).index
        self.device = torch.device("cuda", torch.cuda.current_device() if idx is None else idx)
        self.M, self.N = int(num_bins_x), int(num_bins_y)
        self.xl, self.yl, self.xh, self.yh = float(xl), float(yl), float(xh), float(yh)
        cfg = _lib.EpbConfig(self.M, self.N, self.xl, self.yl, self.xh, self.yh,
                             int(fixed_point_bits), self.device.index,
                             {None: 0, "cell_order": _lib.CONFIG_CELL_ORDER, "tiles": _lib.CONFIG_TILES}[path], 0)
        h = ctypes.c_void_p()
        st = self.lib.epb_create(ctypes.byref(cfg), ctypes.byref(h))
        if st != _lib.EPB_OK:
            raise _lib.EpbError(st, f"epb_create({self.M}x{self.N}) failed: "
                                f"{self.lib.epb_status_string(st).decode()}")
        self._h = h
        bx, by, bits = ctypes.c_float(), ctypes.c_float(), ctypes.c_int32()
        _lib.check(h, self.lib.epb_geometry(h, ctypes.byref(bx), ctypes.byref(by), ctypes.byref(bits)))
        self.bin_size_x, self.bin_size_y, self.fixed_point_bits = bx.value, by.value, bits.value
        self._cells_struct = _lib.EpbCells()

    # -- lifetime ---------------------------------------------------------
    def close(self):
        if getattr(self, "_h", None):
            self.lib.epb_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def bin_area(self) -> float:
        return float(self.bin_size_x) * float(self.bin_size_y)

    @property
    def handle(self):
        return self._h

    # -- helpers ----------------------------------------------------------
    def _cells(self, c: CellTensors) -> ctypes.POINTER(_lib.EpbCells):
        n = c.num_nodes
        for name in ("x", "y", "size_x", "size_y", "offset_x", "offset_y", "ratio"):
            _check_f32(name, getattr(c, name), self.device, n)
        (b0, e0), (b1, e1) = c.resolved_ranges()
        if not (0 <= b0 <= e0 <= n and 0 <= b1 <= e1 <= n):
            raise ValueError(f"cell ranges {c.resolved_ranges()} out of [0, {n}]")
        s = self._cells_struct
        s.x, s.y, s.size_x, s.size_y = _ptr(c.x), _ptr(c.y), _ptr(c.size_x), _ptr(c.size_y)
        s.offset_x, s.offset_y, s.ratio = _ptr(c.offset_x), _ptr(c.offset_y), _ptr(c.ratio)
        s.begin0, s.end0, s.begin1, s.end1 = b0, e0, b1, e1
        return ctypes.byref(s)

    def _grid(self, dtype=torch.float32):
        return torch.empty((self.M, self.N), dtype=dtype, device=self.device)

    def _outputs(self, want_density, want_potential, want_fields, want_energy, out):
        out = dict(out or {})
        res = {}
        for key, want, shape in (("density", want_density, (self.M, self.N)),
                                 ("potential", want_potential, (self.M, self.N)),
                                 ("field_x", want_fields, (self.M, self.N)),
                                 ("field_y", want_fields, (self.M, self.N)),
                                 ("energy", want_energy, (1,))):
            if not want:
                res[key] = None
                continue
            t = out.get(key)
            if t is None:
                t = torch.empty(shape, dtype=torch.float32, device=self.device)
            else:
                _check_f32(key, t, self.device, math.prod(shape))
            res[key] = t
        return res

    # -- API --------------------------------------------------------------
    def set_initial_density(self, init_norm: Optional[torch.Tensor], stream=None):
        """Normalised fixed-cell density (initial_density_map / bin_area)."""
        if init_norm is not None:
            _check_f32("init_norm", init_norm, self.device, self.M * self.N)
        _lib.check(self._h, self.lib.epb_set_initial_density(
            self._h, _ptr(init_norm), _stream_ptr(stream, self.device)))

    def forward(self, cells: CellTensors, want_density=True, want_potential=True, want_fields=True,
                want_energy=True, out=None, stream=None):
        """Returns dict with density, potential, field_x, field_y (M x N fp32)
        and energy (1-element fp32 tensor); entries are None when not wanted.
        `out` may supply preallocated tensors under the same keys."""
        res = self._outputs(want_density, want_potential, want_fields, want_energy, out)
        st = self.lib.epb_forward(self._h, self._cells(cells), _stream_ptr(stream, self.device),
                                  _ptr(res["density"]), _ptr(res["potential"]), _ptr(res["field_x"]),
                                  _ptr(res["field_y"]), _ptr(res["energy"]))
        _lib.check(self._h, st)
        return res

    def backward(self, cells: CellTensors, grad_out: Optional[torch.Tensor] = None,
                 grad_x: Optional[torch.Tensor] = None, grad_y: Optional[torch.Tensor] = None, stream=None):
        """Per-node gradient from the last forward's fields.  Nodes outside the
        cell ranges keep the values they have in grad_x/grad_y (zeros when the
        tensors are allocated here)."""
        n = cells.num_nodes
        if grad_x is None:
            grad_x = torch.zeros(n, dtype=torch.float32, device=self.device)
        if grad_y is None:
            grad_y = torch.zeros(n, dtype=torch.float32, device=self.device)
        _check_f32("grad_x", grad_x, self.device, n)
        _check_f32("grad_y", grad_y, self.device, n)
        _check_f32("grad_out", grad_out, self.device, 1)
        st = self.lib.epb_backward(self._h, self._cells(cells), _ptr(grad_out), _stream_ptr(stream, self.device),
                                   _ptr(grad_x), _ptr(grad_y))
        _lib.check(self._h, st)
        return grad_x, grad_y

    def scatter_fixed(self, cells: CellTensors, grid: Optional[torch.Tensor] = None, stream=None):
        if grid is None:
            grid = self._grid(torch.int64)
        st = self.lib.epb_scatter_fixed(self._h, self._cells(cells), _stream_ptr(stream, self.device), _ptr(grid))
        _lib.check(self._h, st)
        return grid

    def dct_solve(self, density: torch.Tensor, want_potential=True, stream=None):
        _check_f32("density", density, self.device, self.M * self.N)
        res = {"potential": self._grid() if want_potential else None,
               "field_x": self._grid(), "field_y": self._grid(),
               "energy": torch.empty(1, dtype=torch.float32, device=self.device)}
        st = self.lib.epb_dct_solve(self._h, _ptr(density), _stream_ptr(stream, self.device),
                                    _ptr(res["potential"]), _ptr(res["field_x"]), _ptr(res["field_y"]),
                                    _ptr(res["energy"]))
        _lib.check(self._h, st)
        return res

    def gather(self, cells: CellTensors, field_x: torch.Tensor, field_y: torch.Tensor,
               grad_out: Optional[torch.Tensor] = None, grad_x=None, grad_y=None, stream=None):
        _check_f32("field_x", field_x, self.device, self.M * self.N)
        _check_f32("field_y", field_y, self.device, self.M * self.N)
        n = cells.num_nodes
        if grad_x is None:
            grad_x = torch.zeros(n, dtype=torch.float32, device=self.device)
        if grad_y is None:
            grad_y = torch.zeros(n, dtype=torch.float32, device=self.device)
        st = self.lib.epb_gather(self._h, self._cells(cells), _ptr(field_x), _ptr(field_y), _ptr(grad_out),
                                 _stream_ptr(stream, self.device), _ptr(grad_x), _ptr(grad_y))
        _lib.check(self._h, st)
        return grad_x, grad_y

    def overflow(self, cells: CellTensors, target_density: float = 1.0, out: Optional[torch.Tensor] = None,
                 stream=None) -> torch.Tensor:
        """Device float64[2]: bin_area * sum_b max(rho_b - target, 0) and max_b rho_b
        of the cells' density map plus the initial density (epb_overflow)."""
        if out is None:
            out = torch.empty(2, dtype=torch.float64, device=self.device)
        if out.dtype != torch.float64 or out.device != self.device or out.numel() < 2 or not out.is_contiguous():
            raise ValueError("out must be a contiguous float64 tensor of 2 elements on the engine's device")
        st = self.lib.epb_overflow(self._h, self._cells(cells), float(target_density),
                                   _stream_ptr(stream, self.device), _ptr(out))
        _lib.check(self._h, st)
        return out

    # -- host buffers -------------------------------------------------------
    @staticmethod
    def _check_host(name, t, n):
        if t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous() or t.numel() < n:
            raise ValueError(f"{name} must be a contiguous float32 host tensor of at least {n} elements")
        if not t.is_pinned():
            raise ValueError(f"{name} must be in pinned memory (tensor.pin_memory())")

    def forward_host(self, cells: CellTensors, host_x: torch.Tensor, host_y: torch.Tensor,
                     want_density=True, want_potential=True, want_fields=True, want_energy=True, out=None,
                     stream=None):
        """forward() with the positions read from pinned host tensors by the
        scatter itself (over PCIe); the positions of the nodes in the cell
        ranges are kept in cells.x / cells.y (epb_forward_host)."""
        n = cells.num_nodes
        self._check_host("host_x", host_x, n)
        self._check_host("host_y", host_y, n)
        res = self._outputs(want_density, want_potential, want_fields, want_energy, out)
        st = self.lib.epb_forward_host(self._h, self._cells(cells), _ptr(host_x), _ptr(host_y),
                                       _stream_ptr(stream, self.device), _ptr(res["density"]),
                                       _ptr(res["potential"]), _ptr(res["field_x"]), _ptr(res["field_y"]),
                                       _ptr(res["energy"]))
        _lib.check(self._h, st)
        return res

    def backward_host(self, cells: CellTensors, host_grad_x: torch.Tensor, host_grad_y: torch.Tensor,
                      grad_out: Optional[torch.Tensor] = None, grad_x: Optional[torch.Tensor] = None,
                      grad_y: Optional[torch.Tensor] = None, stream=None):
        """backward() whose gradients the gather also stores to pinned host
        tensors over PCIe (epb_backward_host).  The host tensors are complete
        once `stream` has been synchronised."""
        n = cells.num_nodes
        self._check_host("host_grad_x", host_grad_x, n)
        self._check_host("host_grad_y", host_grad_y, n)
        if grad_x is None:
            grad_x = torch.zeros(n, dtype=torch.float32, device=self.device)
        if grad_y is None:
            grad_y = torch.zeros(n, dtype=torch.float32, device=self.device)
        _check_f32("grad_x", grad_x, self.device, n)
        _check_f32("grad_y", grad_y, self.device, n)
        _check_f32("grad_out", grad_out, self.device, 1)
        st = self.lib.epb_backward_host(self._h, self._cells(cells), _ptr(grad_out),
                                        _stream_ptr(stream, self.device), _ptr(grad_x), _ptr(grad_y),
                                        _ptr(host_grad_x), _ptr(host_grad_y))
        _lib.check(self._h, st)
        return grad_x, grad_y

    def forward_overflow(self, cells: CellTensors, target_density: float = 1.0,
                         overflow: Optional[torch.Tensor] = None, want_density=True, want_potential=True,
                         want_fields=True, want_energy=True, out=None, stream=None):
        """forward() of both cell ranges plus the first range's overflow (as
        overflow() of that range alone) with one scatter (epb_forward_overflow).
        Returns (forward outputs, device float64[2] overflow)."""
        if overflow is None:
            overflow = torch.empty(2, dtype=torch.float64, device=self.device)
        if (overflow.dtype != torch.float64 or overflow.device != self.device or overflow.numel() < 2
                or not overflow.is_contiguous()):
            raise ValueError("overflow must be a contiguous float64 tensor of 2 elements on the engine's device")
        res = self._outputs(want_density, want_potential, want_fields, want_energy, out)
        st = self.lib.epb_forward_overflow(self._h, self._cells(cells), float(target_density),
                                           _stream_ptr(stream, self.device), _ptr(overflow), _ptr(res["density"]),
                                           _ptr(res["potential"]), _ptr(res["field_x"]), _ptr(res["field_y"]),
                                           _ptr(res["energy"]))
        _lib.check(self._h, st)
        return res, overflow

    def descent_step(self, cells: CellTensors, grad_x: torch.Tensor, grad_y: torch.Tensor, width: torch.Tensor,
                     height: torch.Tensor, step_bins: float = 0.5, x: Optional[torch.Tensor] = None,
                     y: Optional[torch.Tensor] = None, grad_linf: Optional[torch.Tensor] = None, stream=None):
        """Normalised descent step in place on x, y (default: cells.x, cells.y)
        for the nodes of the cells' ranges (epb_descent_step).  Returns the
        device scalar max(|grad|) used to normalise."""
        x = cells.x if x is None else x
        y = cells.y if y is None else y
        n = cells.num_nodes
        for name, t in (("x", x), ("y", y), ("grad_x", grad_x), ("grad_y", grad_y), ("width", width),
                        ("height", height)):
            _check_f32(name, t, self.device, n)
        if grad_linf is None:
            grad_linf = torch.empty(1, dtype=torch.float32, device=self.device)
        _check_f32("grad_linf", grad_linf, self.device, 1)
        st = self.lib.epb_descent_step(self._h, self._cells(cells), _ptr(x), _ptr(y), _ptr(grad_x), _ptr(grad_y),
                                       _ptr(width), _ptr(height), float(step_bins),
                                       _stream_ptr(stream, self.device), _ptr(grad_linf))
        _lib.check(self._h, st)
        return grad_linf

    def profile_start(self, max_calls: int):
        """Record CUDA events between this engine's kernels for the next
        max_calls forward/backward calls (no host synchronisation)."""
        _lib.check(self._h, self.lib.epb_profile_start(self._h, int(max_calls)))

    def profile_stop(self) -> dict:
        """{stage: (total_ms, launches)} for the calls timed since profile_start."""
        ms = (ctypes.c_double * len(_lib.STAGES))()
        cnt = (ctypes.c_int32 * len(_lib.STAGES))()
        _lib.check(self._h, self.lib.epb_profile_stop(self._h, ms, cnt))
        return {name: (float(ms[i]), int(cnt[i])) for i, name in enumerate(_lib.STAGES)}

    def atomic_probe(self, n_cells, fw=2, fh=3, stream=None) -> float:
        """Milliseconds of n_cells * fw * fh 64-bit atomic adds into this
        engine's grid (the scatter's atomic at hashed footprints); the grid is
        zeroed again afterwards.  Synchronises."""
        ms = ctypes.c_double()
        _lib.check(self._h, self.lib.epb_atomic_probe(self._h, int(n_cells), int(fw), int(fh),
                                                      _stream_ptr(stream, self.device), ctypes.byref(ms)))
        return ms.value

    def error_flags(self, stream=None) -> int:
        """Synchronises; returns and clears EPB_FLAG_* bits.  Raises EpbError
        with EPB_EOVERFLOW when the fixed-point grid saturated."""
        f = ctypes.c_uint32()
        st = self.lib.epb_error_flags(self._h, _stream_ptr(stream, self.device), ctypes.byref(f))
        if st not in (_lib.EPB_OK, _lib.EPB_EOVERFLOW):
            _lib.check(self._h, st)
        if st == _lib.EPB_EOVERFLOW:
            raise _lib.EpbError(st, f"fixed-point density saturated (flags={f.value:#x})")
        return int(f.value)
