"""CPU restatement of the four shard stages (epb_shard_* in include/epb.h),
used to test the multi-rank orchestration in dreamplacett_framework_b200.sharded
with gloo ranks on the CPU.  TEST CODE: built on the oracle; it writes the
same exchanged layouts as the CUDA kernels (see the layout note in
dreamplacett_framework_b200/csrc/epb_kernels.cuh)."""
import numpy as np
import scipy.fft as sf
import torch


def _dct2(a, axis):
    return sf.dct(a, type=2, axis=axis) / a.shape[axis]


def _idct(a, axis):
    return sf.dct(a, type=3, axis=axis)


def _idxst(a, axis):
    a = np.moveaxis(a, axis, -1)
    b = np.zeros_like(a)
    b[..., :-1] = a[..., 1:]
    return np.moveaxis(0.5 * sf.dst(b, type=3, axis=-1), -1, axis)


def strip_width(M, NB):
    """Strip width SW of the exchanged column-pass layout: the column kernel's
    columns per CTA (ColCfg<M>::W = 2 * max(2, 4096 / M)) or 32 (kStripWidth),
    whichever is larger, at most NB."""
    return min(max(2 * max(2, 4096 // M), 32), NB)


def to_strips(a, SW):
    """[RB][NB] -> strip-major [NB/SW][RB][SW], flattened."""
    RB, NB = a.shape
    return a.reshape(RB, NB // SW, SW).transpose(1, 0, 2).ravel()


def from_strips(v, RB, NB, SW):
    return v.reshape(NB // SW, RB, SW).transpose(1, 0, 2).reshape(RB, NB)


class CpuShard:
    def __init__(self, oracle, M, N, xl, yl, xh, yh, P, p):
        self.o = oracle
        self.g = oracle.Geometry(M, N, xl, yl, xh, yh)
        self.M, self.N, self.P, self.p = M, N, P, p
        self.RB, self.NB = M // P, N // P
        self.row0, self.col0 = p * self.RB, p * self.NB
        self.bin_size_x, self.bin_size_y = self.g.bsx, self.g.bsy
        self.S = self.g.default_fixed_bits()
        self.init = None

    def _ocells(self, c):
        n = lambda t: None if t is None else t.numpy()
        return self.o.Cells(n(c.x), n(c.y), n(c.size_x), n(c.size_y), n(c.offset_x), n(c.offset_y), n(c.ratio),
                            ranges=c.resolved_ranges())

    def set_initial_density(self, init_full):
        self.init = init_full.numpy().reshape(self.M, self.N)[self.row0:self.row0 + self.RB].copy()

    def rows_forward(self, cells, density_band, t1_send):
        grid, _ = self.o.density_fixed(self._ocells(cells), self.g, self.S)
        band = np.ascontiguousarray(grid[self.row0:self.row0 + self.RB])
        rho = np.empty((self.RB, self.N), np.float32)
        self.o.lib().ora_fixed_to_density(band.ctypes.data_as(self.o._i64p),
                                          None if self.init is None else self.o._fp(self.init),
                                          self.RB * self.N, self.g.density_scale(self.S), self.o._fp(rho))
        if density_band is not None:
            density_band.copy_(torch.from_numpy(rho))
        t1 = _dct2(rho.astype(np.float64), 1)
        blocks = [t1[:, q * self.NB:(q + 1) * self.NB].ravel() for q in range(self.P)]
        t1_send.copy_(torch.from_numpy(np.concatenate(blocks).astype(np.float32)))

    def columns(self, t1_recv, g_send, want_potential, energy):
        strip = t1_recv.numpy().reshape(self.M, self.NB).astype(np.float64)
        auv = _dct2(strip, 0)
        u = np.arange(self.M)[:, None]
        v = (self.col0 + np.arange(self.NB))[None, :]
        wu = 2 * np.pi * u / self.M
        wv = 2 * np.pi * v / self.N * (self.g.bsx / self.g.bsy)
        d = wu * wu + wv * wv
        inv = np.where(d == 0, 0.0, 1.0 / np.where(d == 0, 1.0, d))
        gx = 2.0 * _idxst(auv * wu * inv * 0.5, 0)
        gp = _idct(auv * inv, 0)  # the field_y form is wv * gp, applied in the row pass
        cu = np.where(u == 0, 1.0, 2.0)
        cv = np.where(v == 0, 1.0, 2.0)
        energy.copy_(torch.tensor([self.M * self.N / 4.0 * float(np.sum(cu * cv * inv * auv * auv))],
                                  dtype=torch.float64))
        out = []
        SW = strip_width(self.M, self.NB)
        for dd in range(self.P):
            rows = slice(dd * self.RB, (dd + 1) * self.RB)
            out += [to_strips(gx[rows], SW), to_strips(gp[rows], SW)]
        g_send.copy_(torch.from_numpy(np.concatenate(out).astype(np.float32)))

    def rows_inverse(self, g_recv, potential_band, fx_band, fy_band, fxy_ext):
        SW = strip_width(self.M, self.NB)
        g = g_recv.numpy().reshape(self.P, 2, self.RB * self.NB)
        band = [np.concatenate([from_strips(g[q, o], self.RB, self.NB, SW) for q in range(self.P)],
                               axis=1).astype(np.float64) for o in range(2)]
        v = np.arange(self.N)[None, :]
        wv = 2 * np.pi * v / self.N * (self.g.bsx / self.g.bsy)
        fx = _idct(band[0], 1).astype(np.float32)
        fy = _idxst(wv * band[1], 1).astype(np.float32)
        phi = _idct(band[1], 1).astype(np.float32)
        if fx_band is not None:
            fx_band.copy_(torch.from_numpy(fx))
            fy_band.copy_(torch.from_numpy(fy))
        if potential_band is not None:
            potential_band.copy_(torch.from_numpy(phi))
        inter = np.stack([fx, fy], axis=-1).ravel()
        fxy_ext[: inter.size].copy_(torch.from_numpy(inter))

    def gather(self, cells, fxy_ext, halo_rows, grad_out, grad_x, grad_y):
        oc = self._ocells(cells)
        ext = fxy_ext.numpy().reshape(-1, self.N, 2)[: self.RB + halo_rows]
        fx = np.zeros((self.M, self.N), np.float32)
        fy = np.zeros((self.M, self.N), np.float32)
        fx[self.row0:self.row0 + self.RB + halo_rows] = ext[..., 0]
        fy[self.row0:self.row0 + self.RB + halo_rows] = ext[..., 1]
        g = 1.0 if grad_out is None else float(grad_out.item())
        gx, gy = self.o.gather(oc, self.g, fx, fy, grad_out=g)
        for node in oc.nodes():
            x = float(oc.x[node]) + (0.0 if oc.offset_x is None else float(oc.offset_x[node]))
            s = float(oc.size_x[node])
            lo, _ = self.o.bin_range(np.float32(x), np.float32(s), self.g.xl, self.g.bsx, self.M)
            if self.row0 <= lo < self.row0 + self.RB and s > 0:
                grad_x[node] = float(gx[node])
                grad_y[node] = float(gy[node])
