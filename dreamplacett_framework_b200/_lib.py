"""ctypes binding of libepb200.so (include/epb.h).

The library is the product's compute path; there is no fallback.  Loading
fails with an exception when the shared object is missing.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libepb200.so")

EPB_OK = 0
EPB_EINVAL = 1
EPB_ECUDA = 2
EPB_ENCCL = 3
EPB_ETIMEOUT = 4
EPB_EOVERFLOW = 5
EPB_ENOSTATE = 6
EPB_FLAG_NONFINITE_CELL = 0x1
EPB_FLAG_SATURATED = 0x2
EPB_FLAG_HALO = 0x4
EPB_FLAG_TIMEOUT = 0x8
IPC_HANDLE_BYTES = 64
# Column-pass outputs per bin in the exchanged layout (field_x form, potential form).
COL_OUTPUTS = 2

# Every symbol include/epb.h declares (the CPU tests check the exports).
EXPORTS = (
    "epb_version", "epb_status_string", "epb_create", "epb_destroy", "epb_last_error",
    "epb_geometry", "epb_set_initial_density", "epb_forward", "epb_backward",
    "epb_scatter_fixed", "epb_dct_solve", "epb_gather", "epb_error_flags",
    "epb_profile_start", "epb_profile_stop", "epb_density_noalloc",
    "epb_create_shard", "epb_shard_geometry", "epb_shard_rows_forward", "epb_shard_columns",
    "epb_shard_rows_inverse", "epb_shard_gather",
    "epb_shard_peer_buffers", "epb_shard_connect", "epb_shard_set_timeout", "epb_shard_forward_peer",
    "epb_shard_backward_peer", "epb_shard_wait_test",
    "epb_overflow", "epb_descent_step", "epb_forward_overflow",
    "epb_forward_host", "epb_backward_host",
    "epb_wirelength_scratch_bytes", "epb_wirelength", "epb_atomic_probe",
)

# Largest grid (M*N bins) epb_density_noalloc accepts (EPB_NOALLOC_MAX_BINS).
NOALLOC_MAX_BINS = 1024 * 1024

# Stage indices of epb_profile_stop (EPB_STAGE_* in include/epb.h).
STAGES = ("scatter", "row_fwd", "column", "row_inv", "gather", "bin")
# epb_config.flags: the cell-order scatter / gather, or the cell tiles.
CONFIG_CELL_ORDER = 0x1
CONFIG_TILES = 0x2


class EpbConfig(ctypes.Structure):
    _fields_ = [
        ("num_bins_x", ctypes.c_int32), ("num_bins_y", ctypes.c_int32),
        ("xl", ctypes.c_double), ("yl", ctypes.c_double),
        ("xh", ctypes.c_double), ("yh", ctypes.c_double),
        ("fixed_point_bits", ctypes.c_int32), ("device", ctypes.c_int32),
        ("flags", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class EpbCells(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("y", ctypes.c_void_p),
        ("size_x", ctypes.c_void_p), ("size_y", ctypes.c_void_p),
        ("offset_x", ctypes.c_void_p), ("offset_y", ctypes.c_void_p),
        ("ratio", ctypes.c_void_p),
        ("begin0", ctypes.c_int64), ("end0", ctypes.c_int64),
        ("begin1", ctypes.c_int64), ("end1", ctypes.c_int64),
    ]


class EpbNetlist(ctypes.Structure):
    _fields_ = [
        ("net_start", ctypes.c_void_p), ("net_pins", ctypes.c_void_p), ("pin_node", ctypes.c_void_p),
        ("pin_offset_x", ctypes.c_void_p), ("pin_offset_y", ctypes.c_void_p), ("net_weight", ctypes.c_void_p),
        ("node_pin_start", ctypes.c_void_p), ("node_pins", ctypes.c_void_p),
        ("num_nets", ctypes.c_int32), ("num_pins", ctypes.c_int32), ("num_nodes", ctypes.c_int32),
        ("ignore_net_degree", ctypes.c_int32), ("device", ctypes.c_int32),
    ]


class EpbError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"epb status {status}: {message}")
        self.status = status


_lib = None


def load():
    """Load and prototype libepb200.so; raises when it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"libepb200.so not found at {LIB_PATH}: build it with "
            "`python -m dreamplacett_framework_b200.build` (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    cp = ctypes.POINTER(EpbCells)
    L.epb_version.restype = ctypes.c_char_p
    L.epb_status_string.argtypes = [ctypes.c_int]
    L.epb_status_string.restype = ctypes.c_char_p
    L.epb_create.argtypes = [ctypes.POINTER(EpbConfig), ctypes.POINTER(vp)]
    L.epb_destroy.argtypes = [vp]
    L.epb_last_error.argtypes = [vp]
    L.epb_last_error.restype = ctypes.c_char_p
    L.epb_geometry.argtypes = [vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float),
                               ctypes.POINTER(i32)]
    L.epb_set_initial_density.argtypes = [vp, vp, vp]
    L.epb_forward.argtypes = [vp, cp, vp, vp, vp, vp, vp, vp]
    L.epb_backward.argtypes = [vp, cp, vp, vp, vp, vp]
    L.epb_scatter_fixed.argtypes = [vp, cp, vp, vp]
    L.epb_dct_solve.argtypes = [vp, vp, vp, vp, vp, vp, vp]
    L.epb_gather.argtypes = [vp, cp, vp, vp, vp, vp, vp, vp]
    L.epb_error_flags.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint32)]
    L.epb_profile_start.argtypes = [vp, i32]
    L.epb_profile_stop.argtypes = [vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(i32)]
    L.epb_density_noalloc.argtypes = [ctypes.POINTER(EpbConfig), cp, vp, vp, vp, ctypes.c_char_p, i32]
    L.epb_create_shard.argtypes = [ctypes.POINTER(EpbConfig), i32, i32, ctypes.POINTER(vp)]
    L.epb_shard_geometry.argtypes = [vp] + [ctypes.POINTER(i32)] * 4
    L.epb_shard_rows_forward.argtypes = [vp, cp, vp, vp, vp]
    L.epb_shard_columns.argtypes = [vp, vp, vp, vp, i32, vp]
    L.epb_shard_rows_inverse.argtypes = [vp, vp, vp, vp, vp, vp, vp]
    L.epb_shard_gather.argtypes = [vp, cp, vp, i32, vp, vp, vp, vp]
    L.epb_shard_peer_buffers.argtypes = [vp, i32, ctypes.c_char_p]
    L.epb_shard_connect.argtypes = [vp, ctypes.c_char_p]
    L.epb_shard_set_timeout.argtypes = [vp, i64]
    L.epb_shard_forward_peer.argtypes = [vp, cp, vp, vp, vp, vp, vp, vp]
    L.epb_shard_backward_peer.argtypes = [vp, cp, vp, vp, vp, vp]
    L.epb_shard_wait_test.argtypes = [vp, vp, i64]
    L.epb_overflow.argtypes = [vp, cp, ctypes.c_float, vp, vp]
    L.epb_descent_step.argtypes = [vp, cp, vp, vp, vp, vp, vp, vp, ctypes.c_float, vp, vp]
    L.epb_forward_overflow.argtypes = [vp, cp, ctypes.c_float, vp, vp, vp, vp, vp, vp, vp]
    L.epb_forward_host.argtypes = [vp, cp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.epb_backward_host.argtypes = [vp, cp, vp, vp, vp, vp, vp, vp]
    L.epb_atomic_probe.argtypes = [vp, i64, i32, i32, vp, ctypes.POINTER(ctypes.c_double)]
    L.epb_wirelength_scratch_bytes.argtypes = [i32]
    L.epb_wirelength_scratch_bytes.restype = ctypes.c_size_t
    L.epb_wirelength.argtypes = [ctypes.POINTER(EpbNetlist), vp, vp, ctypes.c_float, vp, vp, ctypes.c_size_t, vp,
                                 vp, vp, vp, ctypes.c_char_p, i32]
    for name in EXPORTS:
        if name not in ("epb_version", "epb_status_string", "epb_last_error"):
            getattr(L, name).restype = ctypes.c_int
    _lib = L
    return L


def check(handle, status):
    if status != EPB_OK:
        L = load()
        msg = L.epb_last_error(handle) if handle else None
        msg = msg.decode() if msg else L.epb_status_string(status).decode()
        raise EpbError(status, msg or L.epb_status_string(status).decode())
