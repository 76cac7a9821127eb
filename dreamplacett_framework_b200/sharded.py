"""One placement grid over P GPUs: row-band shards and torch.distributed exchanges.

Each GPU (one process per GPU) owns a row band of the bin grid.  One forward
and backward run these steps:

  1. scatter every cell overlapping the band (clipped to it) and take the row
     DCT-II of the band's rows                  -> t1_send            [kernels]
  2. all-to-all: row bands -> column strips      t1_send -> t1_recv  [NCCL]
  3. column DCT-II, weights, column inverses of the strip; strip energy
                                                -> g_send, energy     [kernels]
  4. all-reduce of the energy (fp64); all-to-all: column strips -> row bands
                                                 g_send -> g_recv     [NCCL]
  5. row inverses of the band: potential, field_x, field_y, interleaved fields
                                                                      [kernels]
  6. halo: the first H field rows go to the previous band (point-to-point)
                                                                      [NCCL]
  7. backward: gradient of the cells whose first bin row is in the band
                                                                      [kernels]

The exchange is split from the arithmetic by a small backend interface so the
same orchestration runs on the CUDA engine (`EngineShard`, NCCL) and, in the
CPU tests, on a restatement with gloo.

transport="peer" fuses steps 2, 4 and 6 into the kernels instead: they store
their blocks straight into the other GPUs' buffers over NVLink (CUDA IPC
mappings), and bounded one-thread waits on epoch signals order the stages
(epb_shard_forward_peer in include/epb.h).

Integer density sums make the density map identical to the one-GPU result for
any P.  The fields and the energy differ from it only by fp32 rounding.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from .engine import CellTensors, _check_f32, _ptr, _stream_ptr


class EngineShard:
    """Backend: the CUDA engine's epb_shard_* stages (one shard handle)."""

    def __init__(self, num_bins_x, num_bins_y, xl, yl, xh, yh, num_shards, shard, device,
                 fixed_point_bits=0, path=None):
        self.lib = _lib.load()
        self.device = device
        flags = {None: 0, "cell_order": _lib.CONFIG_CELL_ORDER, "tiles": _lib.CONFIG_TILES}[path]
        cfg = _lib.EpbConfig(int(num_bins_x), int(num_bins_y), float(xl), float(yl), float(xh), float(yh),
                             int(fixed_point_bits), device.index, flags, 0)
        h = ctypes.c_void_p()
        st = self.lib.epb_create_shard(ctypes.byref(cfg), int(num_shards), int(shard), ctypes.byref(h))
        if st != _lib.EPB_OK:
            raise _lib.EpbError(st, f"epb_create_shard({num_bins_x}x{num_bins_y}, P={num_shards}, p={shard})")
        self._h = h
        vals = [ctypes.c_int32() for _ in range(4)]
        _lib.check(h, self.lib.epb_shard_geometry(h, *[ctypes.byref(v) for v in vals]))
        self.P, self.p, self.RB, self.NB = (v.value for v in vals)
        bx, by, bits = ctypes.c_float(), ctypes.c_float(), ctypes.c_int32()
        _lib.check(h, self.lib.epb_geometry(h, ctypes.byref(bx), ctypes.byref(by), ctypes.byref(bits)))
        self.bin_size_x, self.bin_size_y, self.fixed_point_bits = bx.value, by.value, bits.value
        self._cs = _lib.EpbCells()

    def close(self):
        if getattr(self, "_h", None):
            self.lib.epb_destroy(self._h)
            self._h = None

    def _cells(self, c: CellTensors):
        n = c.num_nodes
        for name in ("x", "y", "size_x", "size_y", "offset_x", "offset_y", "ratio"):
            _check_f32(name, getattr(c, name), self.device, n)
        (b0, e0), (b1, e1) = c.resolved_ranges()
        s = self._cs
        s.x, s.y, s.size_x, s.size_y = _ptr(c.x), _ptr(c.y), _ptr(c.size_x), _ptr(c.size_y)
        s.offset_x, s.offset_y, s.ratio = _ptr(c.offset_x), _ptr(c.offset_y), _ptr(c.ratio)
        s.begin0, s.end0, s.begin1, s.end1 = b0, e0, b1, e1
        return ctypes.byref(s)

    def set_initial_density(self, init_norm_full):
        _lib.check(self._h, self.lib.epb_set_initial_density(self._h, _ptr(init_norm_full),
                                                             _stream_ptr(None, self.device)))

    def rows_forward(self, cells, density_band, t1_send):
        _lib.check(self._h, self.lib.epb_shard_rows_forward(self._h, self._cells(cells), _stream_ptr(None, self.device),
                                                            _ptr(density_band), _ptr(t1_send)))

    def columns(self, t1_recv, g_send, want_potential, energy_partial):
        _lib.check(self._h, self.lib.epb_shard_columns(self._h, _ptr(t1_recv), _stream_ptr(None, self.device),
                                                       _ptr(g_send), int(bool(want_potential)), _ptr(energy_partial)))

    def rows_inverse(self, g_recv, potential_band, fx_band, fy_band, fxy_ext):
        _lib.check(self._h, self.lib.epb_shard_rows_inverse(self._h, _ptr(g_recv), _stream_ptr(None, self.device),
                                                            _ptr(potential_band), _ptr(fx_band), _ptr(fy_band),
                                                            _ptr(fxy_ext)))

    def gather(self, cells, fxy_ext, halo_rows, grad_out, grad_x, grad_y):
        _lib.check(self._h, self.lib.epb_shard_gather(self._h, self._cells(cells), _ptr(fxy_ext), int(halo_rows),
                                                      _ptr(grad_out), _stream_ptr(None, self.device),
                                                      _ptr(grad_x), _ptr(grad_y)))

    # ---- peer transport (exchanges fused into the kernels) ----
    def setup_peer(self, halo_rows, group=None):
        """Create the IPC-shared receive buffers and map every shard's (collective)."""
        buf = ctypes.create_string_buffer(4 * _lib.IPC_HANDLE_BYTES)
        _lib.check(self._h, self.lib.epb_shard_peer_buffers(self._h, int(halo_rows), buf))
        mine = torch.frombuffer(bytearray(buf.raw), dtype=torch.uint8).to(self.device)
        allh = [torch.empty_like(mine) for _ in range(self.P)]
        dist.all_gather(allh, mine, group=group)
        blob = torch.cat(allh).cpu().numpy().tobytes()
        _lib.check(self._h, self.lib.epb_shard_connect(self._h, blob))

    def set_timeout(self, max_polls):
        _lib.check(self._h, self.lib.epb_shard_set_timeout(self._h, int(max_polls)))

    def forward_peer(self, cells, density_band, potential_band, fx_band, fy_band, energy):
        _lib.check(self._h, self.lib.epb_shard_forward_peer(
            self._h, self._cells(cells), _stream_ptr(None, self.device), _ptr(density_band), _ptr(potential_band),
            _ptr(fx_band), _ptr(fy_band), _ptr(energy)))

    def backward_peer(self, cells, grad_out, grad_x, grad_y):
        _lib.check(self._h, self.lib.epb_shard_backward_peer(self._h, self._cells(cells), _ptr(grad_out),
                                                             _stream_ptr(None, self.device), _ptr(grad_x),
                                                             _ptr(grad_y)))

    def wait_test(self, max_polls):
        _lib.check(self._h, self.lib.epb_shard_wait_test(self._h, _stream_ptr(None, self.device), int(max_polls)))

    def profile_start(self, max_calls):
        _lib.check(self._h, self.lib.epb_profile_start(self._h, int(max_calls)))

    def profile_stop(self):
        ms = (ctypes.c_double * len(_lib.STAGES))()
        cnt = (ctypes.c_int32 * len(_lib.STAGES))()
        _lib.check(self._h, self.lib.epb_profile_stop(self._h, ms, cnt))
        return {name: (float(ms[i]), int(cnt[i])) for i, name in enumerate(_lib.STAGES)}

    def error_flags(self):
        f = ctypes.c_uint32()
        st = self.lib.epb_error_flags(self._h, _stream_ptr(None, self.device), ctypes.byref(f))
        if st not in (_lib.EPB_OK, _lib.EPB_EOVERFLOW, _lib.EPB_ETIMEOUT):
            _lib.check(self._h, st)
        return int(f.value)


def halo_rows_for(max_cell_size_x: float, bin_size_x: float) -> int:
    """Rows a footprint can reach below its first row: a cell of width w spans
    at most floor(w / bin) + 1 bins after its first one."""
    return int(math.floor(float(max_cell_size_x) / float(bin_size_x))) + 2


class ShardedElectricPotential:
    """Forward/backward of one grid over the ranks of a process group."""

    def __init__(self, num_bins_x, num_bins_y, xl, yl, xh, yh, max_cell_size_x, group=None, device=None,
                 backend=None, fixed_point_bits=0, transport="nccl", path=None):
        self.group = group
        self.P = dist.get_world_size(group)
        self.p = dist.get_rank(group)
        self.M, self.N = int(num_bins_x), int(num_bins_y)
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        self.be = backend if backend is not None else EngineShard(
            num_bins_x, num_bins_y, xl, yl, xh, yh, self.P, self.p, self.device, fixed_point_bits, path)
        RB, NB, M, N = self.M // self.P, self.N // self.P, self.M, self.N
        self.RB, self.NB = RB, NB
        H = halo_rows_for(max_cell_size_x, self.be.bin_size_x)
        if H > RB and self.P > 1:
            raise ValueError(f"cell footprints span {H} rows but a band has only {RB}: use fewer shards")
        # the last band has nothing below it
        self.H = 0 if self.p == self.P - 1 else min(H, M - (self.p + 1) * RB)
        f32 = dict(dtype=torch.float32, device=self.device)
        self.t1_send = torch.empty(RB * N, **f32)
        self.t1_recv = torch.empty(M * NB, **f32)
        self.g_send = torch.empty(_lib.COL_OUTPUTS * M * NB, **f32)
        self.g_recv = torch.empty(_lib.COL_OUTPUTS * M * NB, **f32)
        self.fxy_ext = torch.zeros((RB + H) * N * 2, **f32)  # room for the largest halo of any rank
        self.energy = torch.zeros(1, dtype=torch.float64, device=self.device)
        self._Hsend = min(H, RB) if self.p > 0 else 0  # rows the previous band needs from us
        if transport not in ("nccl", "peer"):
            raise ValueError(f"transport must be 'nccl' or 'peer', not {transport!r}")
        self.transport = transport
        if transport == "peer":
            # exchanges fused into the kernels: stores into the peers' buffers over NVLink
            self.be.setup_peer(H if self.P > 1 else 0, group)
            self.energy = torch.zeros(1, dtype=torch.float32, device=self.device)

    @property
    def row_range(self):
        return self.p * self.RB, (self.p + 1) * self.RB

    def set_initial_density(self, init_norm_full: torch.Tensor):
        self.be.set_initial_density(init_norm_full.reshape(-1))

    def _halo_exchange(self):
        N = self.N
        ops = []
        if self._Hsend > 0:
            ops.append(dist.P2POp(dist.isend, self.fxy_ext[: self._Hsend * N * 2], self.p - 1, self.group))
        if self.H > 0:
            lo = self.RB * N * 2
            ops.append(dist.P2POp(dist.irecv, self.fxy_ext[lo: lo + self.H * N * 2], self.p + 1, self.group))
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()

    def forward(self, cells: CellTensors, want_density=True, want_potential=True, want_fields=True, out=None):
        """Band outputs ([RB][N] tensors) and the total energy (fp64 tensor)."""
        out = dict(out or {})
        band = lambda k, want: (out.get(k) if out.get(k) is not None else
                                torch.empty(self.RB, self.N, dtype=torch.float32, device=self.device)) if want else None
        dens = band("density", want_density)
        phi = band("potential", want_potential)
        fx = band("field_x", want_fields)
        fy = band("field_y", want_fields)
        if self.transport == "peer":
            self.be.forward_peer(cells, dens, phi, fx, fy, self.energy)
            return {"density": dens, "potential": phi, "field_x": fx, "field_y": fy, "energy": self.energy}
        self.be.rows_forward(cells, dens, self.t1_send)
        dist.all_to_all_single(self.t1_recv, self.t1_send, group=self.group)
        self.be.columns(self.t1_recv, self.g_send, want_potential, self.energy)
        work = dist.all_reduce(self.energy, group=self.group, async_op=True)
        dist.all_to_all_single(self.g_recv, self.g_send, group=self.group)
        self.be.rows_inverse(self.g_recv, phi, fx, fy, self.fxy_ext)
        self._halo_exchange()
        work.wait()
        return {"density": dens, "potential": phi, "field_x": fx, "field_y": fy, "energy": self.energy}

    def backward(self, cells: CellTensors, grad_out: Optional[torch.Tensor] = None, grad_x=None, grad_y=None):
        """Gradient of the cells owned by this band (first bin row in the band);
        other entries of grad_x / grad_y keep their values (zeros when allocated here)."""
        n = cells.num_nodes
        if grad_x is None:
            grad_x = torch.zeros(n, dtype=torch.float32, device=self.device)
        if grad_y is None:
            grad_y = torch.zeros(n, dtype=torch.float32, device=self.device)
        if self.transport == "peer":
            self.be.backward_peer(cells, grad_out, grad_x, grad_y)
        else:
            self.be.gather(cells, self.fxy_ext, self.H, grad_out, grad_x, grad_y)
        return grad_x, grad_y

    # ---- positions in and gradients out through host memory, split over the ranks ----
    def node_slice(self, n):
        """This rank's node slice [lo, hi) of n nodes (contiguous, 1/P each) and
        the padded slice length."""
        chunk = (int(n) + self.P - 1) // self.P
        lo = min(self.p * chunk, int(n))
        return lo, min(lo + chunk, int(n)), chunk

    def _host_buffers(self, n):
        lo, hi, chunk = self.node_slice(n)
        if getattr(self, "_hb_n", None) != n:
            f32 = dict(dtype=torch.float32, device=self.device)
            self._stage = torch.zeros(2, chunk, **f32)            # this rank's slice of x and y
            self._gathered = torch.zeros(2, self.P * chunk, **f32)
            self._gpad = torch.zeros(2, self.P * chunk, **f32)    # this rank's gradients, padded
            self._gslice = torch.zeros(2, chunk, **f32)           # slice r of the summed gradient
            self._hb_n = n
        return lo, hi, chunk

    def forward_host(self, cells: CellTensors, host_pos: torch.Tensor, **kw):
        """The forward with DREAMPlace's positions [x | y] (2n floats) in host
        memory (pinned for an asynchronous copy).  Rank r copies only node
        slice r of x and y (1/P of them) to its GPU, and an all-gather over
        NVLink fills cells.x and cells.y on every rank: each GPU moves 1/P of
        the positions over PCIe instead of all of them."""
        n = cells.num_nodes
        lo, hi, chunk = self._host_buffers(n)
        self._stage[0, : hi - lo].copy_(host_pos[lo:hi], non_blocking=True)
        self._stage[1, : hi - lo].copy_(host_pos[n + lo:n + hi], non_blocking=True)
        for k, dst in ((0, cells.x), (1, cells.y)):
            dist.all_gather_into_tensor(self._gathered[k], self._stage[k], group=self.group)
            dst.copy_(self._gathered[k, :n])
        return self.forward(cells, **kw)

    def backward_host(self, cells: CellTensors, host_grad: torch.Tensor, grad_out: Optional[torch.Tensor] = None):
        """The backward with the gradient [gx | gy] (2n floats) going to host
        memory, split over the ranks: the per-rank gradients (each cell's from
        the band that owns it, zeros elsewhere) are summed by a reduce-scatter
        over NVLink, and rank r stores node slice r of the sum to host_grad
        (other entries untouched).  The store is asynchronous on the current
        stream when host_grad is pinned: synchronise before reading it.
        Returns this rank's slice on the device."""
        n = cells.num_nodes
        lo, hi, chunk = self._host_buffers(n)
        self._gpad.zero_()
        self.backward(cells, grad_out, self._gpad[0, :n], self._gpad[1, :n])
        for k in (0, 1):
            dist.reduce_scatter_tensor(self._gslice[k], self._gpad[k], group=self.group)
        host_grad[lo:hi].copy_(self._gslice[0, : hi - lo], non_blocking=True)
        host_grad[n + lo:n + hi].copy_(self._gslice[1, : hi - lo], non_blocking=True)
        return self._gslice[0, : hi - lo], self._gslice[1, : hi - lo]

    def close(self):
        if hasattr(self.be, "close"):
            self.be.close()
