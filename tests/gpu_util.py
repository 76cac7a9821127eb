"""Helpers shared by the GPU parity tests: the same seeded arrays are handed
to the CUDA engine (as torch tensors) and to the CPU oracle (as numpy)."""
import numpy as np
import torch

from dreamplacett_framework_b200.engine import CellTensors, ElectricPotentialEngine


def placement_cells(p, stretched=True):
    """(numpy dict, ranges) of a synth.Placement in DREAMPlace's layout."""
    if stretched:
        arrs = dict(x=p.x, y=p.y, size_x=p.size_x_clamped, size_y=p.size_y_clamped,
                    offset_x=p.offset_x, offset_y=p.offset_y, ratio=p.ratio)
    else:
        arrs = dict(x=p.x, y=p.y, size_x=p.size_x, size_y=p.size_y, offset_x=None, offset_y=None, ratio=None)
    return arrs, p.ranges


def to_device(arrs, ranges, device):
    t = {k: (None if v is None else torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(device))
         for k, v in arrs.items()}
    return CellTensors(ranges=ranges, **t)


def to_oracle(o, arrs, ranges):
    return o.Cells(arrs["x"], arrs["y"], arrs["size_x"], arrs["size_y"], arrs.get("offset_x"),
                   arrs.get("offset_y"), arrs.get("ratio"), ranges=ranges)


def engine_for(p, device, bits=0):
    return ElectricPotentialEngine(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh,
                                   fixed_point_bits=bits, device=device)


def geometry_for(o, p):
    return o.Geometry(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh)


def np_(t):
    return t.detach().cpu().numpy()
