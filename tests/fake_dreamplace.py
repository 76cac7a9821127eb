"""A stand-in for the DREAMPlace modules the reference's shim patches.

DREAMPlace is not installed; patch_dreamplace() only needs the module path
dreamplace.ops.electric_potential.electric_potential with an
ElectricPotentialFunction class whose forward/backward it replaces.  The
stand-in's own methods record that they were called, so a test can tell the
original from the patched path."""
import sys
import types

import torch


def install():
    calls = {"orig_forward": 0, "orig_backward": 0}

    class ElectricPotentialFunction(torch.autograd.Function):
        @staticmethod
        def forward(ctx, pos, *args):
            calls["orig_forward"] += 1
            ctx.n = pos.numel()
            return torch.zeros(1, dtype=pos.dtype, device=pos.device)

        @staticmethod
        def backward(ctx, grad):
            calls["orig_backward"] += 1
            return (torch.zeros(ctx.n, dtype=grad.dtype, device=grad.device),) + (None,) * 37

    names = ["dreamplace", "dreamplace.ops", "dreamplace.ops.electric_potential",
             "dreamplace.ops.electric_potential.electric_potential"]
    mods = {}
    for n in names:
        mods[n] = types.ModuleType(n)
        sys.modules[n] = mods[n]
    mods["dreamplace"].ops = mods["dreamplace.ops"]
    mods["dreamplace.ops"].electric_potential = mods["dreamplace.ops.electric_potential"]
    mods["dreamplace.ops.electric_potential"].electric_potential = mods[names[-1]]
    mods[names[-1]].ElectricPotentialFunction = ElectricPotentialFunction
    return ElectricPotentialFunction, calls


def uninstall():
    for n in list(sys.modules):
        if n == "dreamplace" or n.startswith("dreamplace."):
            del sys.modules[n]


def ep_args(p, tensors, fast_mode=False):
    """The 37 arguments after pos, in DREAMPlace's order
    (integration/scatter_ttnn_client.py:554-574), for a synth.Placement."""
    t = tensors
    return (t["size_x_clamped"], t["size_y_clamped"], t["offset_x"], t["offset_y"], t["ratio"],
            None, None, t["initial_density_map"], 1.0,
            p.xl, p.yl, p.xh, p.yh, p.bin_size_x, p.bin_size_y,
            p.num_movable, p.num_filler, 0, None, p.num_bins_x, p.num_bins_y,
            0, 0, 0, 0, True, None,
            None, None, None, None, None, None, None, None, None, fast_mode)
