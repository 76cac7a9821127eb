"""Multi-rank path (dreamplacett_framework_b200.sharded).

CPU: two gloo ranks run the real orchestration (all-to-all transposes, fp64
energy all-reduce, halo point-to-point) over a CPU restatement of the stage
kernels, and the assembled result must equal the one-process oracle.
GPU: the CUDA stages on one GPU with P = 1 reproduce epb_forward/backward
bit for bit; with 2+ GPUs the NCCL pipeline reproduces the one-GPU engine.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dreamplacett_framework_b200 import synth
from dreamplacett_framework_b200.engine import CellTensors

from gpu_util import np_

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _small_placement():
    p = synth.make_placement("c3", scale=0.0004, grid=64, seed=7)
    return p


def _cells_cpu(p):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32))
    return CellTensors(t(p.x), t(p.y), t(p.size_x_clamped), t(p.size_y_clamped), t(p.offset_x), t(p.offset_y),
                       t(p.ratio), ranges=p.ranges)


def _gloo_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    import build_oracle
    build_oracle.build_oracle()
    import oracle as o
    from shard_cpu_backend import CpuShard
    from dreamplacett_framework_b200.sharded import ShardedElectricPotential
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        p = _small_placement()
        be = CpuShard(o, p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh, world, rank)
        sh = ShardedElectricPotential(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh,
                                      float(p.size_x_clamped.max()), device=torch.device("cpu"), backend=be)
        sh.set_initial_density(torch.from_numpy(p.initial_density_norm()))
        cells = _cells_cpu(p)
        out = {k: v.clone() for k, v in sh.forward(cells).items()}
        gx, gy = sh.backward(cells)
        # the host-buffer path: positions in from [x | y], each rank copying its node slice and an
        # all-gather completing them; the summed gradient out, each rank storing its slice
        n = p.num_nodes
        host_pos = torch.cat([cells.x, cells.y])
        cells2 = CellTensors(torch.zeros(n), torch.zeros(n), cells.size_x, cells.size_y, cells.offset_x,
                             cells.offset_y, cells.ratio, ranges=p.ranges)
        out2 = sh.forward_host(cells2, host_pos)
        host_grad = torch.full((2 * n,), float("nan"))
        sh.backward_host(cells2, host_grad)
        lo, hi, _ = sh.node_slice(n)
        assert torch.equal(cells2.x, cells.x) and torch.equal(cells2.y, cells.y)
        for k in ("density", "potential", "field_x", "field_y", "energy"):
            assert torch.equal(out2[k], out[k]), k
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), density=out["density"].numpy(),
                 potential=out["potential"].numpy(), field_x=out["field_x"].numpy(),
                 field_y=out["field_y"].numpy(), energy=out["energy"].numpy(), gx=gx.numpy(), gy=gy.numpy(),
                 host_gx=host_grad[lo:hi].numpy(), host_gy=host_grad[n + lo:n + hi].numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_ranks_match_oracle(oracle, tmp_path, world):
    port = _free_port()
    mp.start_processes(_gloo_worker, args=(world, port, str(tmp_path)), nprocs=world, start_method="spawn")
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    p = _small_placement()
    g = oracle.Geometry(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh)
    S = g.default_fixed_bits()
    oc = oracle.Cells(p.x, p.y, p.size_x_clamped, p.size_y_clamped, p.offset_x, p.offset_y, p.ratio,
                      ranges=p.ranges)
    grid, _ = oracle.density_fixed(oc, g, S)
    rho, _ = oracle.fixed_to_density(grid, g, S, p.initial_density_norm())
    ref = oracle.solve_fft(rho, g.bsx, g.bsy)
    # density: bit-exact, band by band
    np.testing.assert_array_equal(np.concatenate([q["density"] for q in parts]), rho)
    for k in ("potential", "field_x", "field_y"):
        assert oracle.rel_linf(np.concatenate([q[k] for q in parts]), ref[k]) < 1e-5, k
    for q in parts:
        assert abs(float(q["energy"][0]) / ref["energy"] - 1) < 1e-6
    rx, ry = oracle.gather(oc, g, ref["field_x"].astype(np.float32), ref["field_y"].astype(np.float32))
    # every scattered cell is owned by exactly one rank: the per-rank gradients add up
    gx = sum(q["gx"] for q in parts)
    gy = sum(q["gy"] for q in parts)
    assert oracle.rel_linf(gx, rx) < 1e-5 and oracle.rel_linf(gy, ry) < 1e-5
    # the host-buffer path's slices, in rank order, are the summed gradient
    np.testing.assert_array_equal(np.concatenate([q["host_gx"] for q in parts]), gx)
    np.testing.assert_array_equal(np.concatenate([q["host_gy"] for q in parts]), gy)


@pytest.mark.gpu
def test_single_shard_stages_match_forward(cuda_device):
    """P = 1: the shard stages run the same kernels as epb_forward/epb_backward."""
    from dreamplacett_framework_b200 import _lib
    from dreamplacett_framework_b200.engine import ElectricPotentialEngine
    from dreamplacett_framework_b200.sharded import EngineShard
    p = synth.make_placement("c3", scale=0.1, grid=1024)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda_device)
    cells = CellTensors(t(p.x), t(p.y), t(p.size_x_clamped), t(p.size_y_clamped), t(p.offset_x), t(p.offset_y),
                        t(p.ratio), ranges=p.ranges)
    init = t(p.initial_density_norm())
    M, N = p.num_bins_x, p.num_bins_y
    with ElectricPotentialEngine(M, N, p.xl, p.yl, p.xh, p.yh, device=cuda_device) as eng:
        eng.set_initial_density(init)
        ref = eng.forward(cells)
        rgx, rgy = eng.backward(cells)
    be = EngineShard(M, N, p.xl, p.yl, p.xh, p.yh, 1, 0, cuda_device)
    try:
        be.set_initial_density(init.reshape(-1))
        f = lambda *s: torch.empty(*s, dtype=torch.float32, device=cuda_device)
        dens, phi, fx, fy = f(M, N), f(M, N), f(M, N), f(M, N)
        t1 = f(M * N)
        g = f(_lib.COL_OUTPUTS * M * N)
        fxy = f(M * N * 2)
        e = torch.zeros(1, dtype=torch.float64, device=cuda_device)
        be.rows_forward(cells, dens, t1)
        be.columns(t1, g, True, e)
        be.rows_inverse(g, phi, fx, fy, fxy)
        gx = torch.zeros(p.num_nodes, device=cuda_device)
        gy = torch.zeros(p.num_nodes, device=cuda_device)
        be.gather(cells, fxy, 0, None, gx, gy)
        torch.cuda.synchronize()
        for a, b in ((dens, ref["density"]), (phi, ref["potential"]), (fx, ref["field_x"]), (fy, ref["field_y"]),
                     (gx, rgx), (gy, rgy)):
            assert torch.equal(a, b)
        assert float(e.item()) == pytest.approx(float(ref["energy"].item()), rel=1e-7)
    finally:
        be.close()


@pytest.mark.gpu
def test_bounded_wait_times_out_without_hanging(cuda_device):
    """A wait for a signal nobody publishes runs out of polls, sets the timeout
    flag and returns; the context stays usable."""
    from dreamplacett_framework_b200 import _lib
    from dreamplacett_framework_b200.sharded import EngineShard
    be = EngineShard(64, 64, 0.0, 0.0, 640.0, 640.0, 1, 0, cuda_device)
    try:
        buf = __import__("ctypes").create_string_buffer(4 * _lib.IPC_HANDLE_BYTES)
        _lib.check(be._h, be.lib.epb_shard_peer_buffers(be._h, 0, buf))
        be.wait_test(2000)
        assert be.error_flags() & _lib.EPB_FLAG_TIMEOUT
        assert be.error_flags() == 0  # cleared; the GPU keeps working
        x = torch.ones(10, device=cuda_device)
        assert float(x.sum()) == 10.0
    finally:
        be.close()


def _failing_worker(rank, world, port, out_dir):
    """Rank 1 leaves before the first exchange; rank 0 must get an error from
    its next collective (process-group timeout), not hang."""
    import datetime
    import sys
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "oracle"))
    import build_oracle
    build_oracle.build_oracle()
    import oracle as o
    from shard_cpu_backend import CpuShard
    from dreamplacett_framework_b200.sharded import ShardedElectricPotential
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    p = _small_placement()
    be = CpuShard(o, p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh, world, rank)
    sh = ShardedElectricPotential(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh,
                                  float(p.size_x_clamped.max()), device=torch.device("cpu"), backend=be)
    if rank == 1:
        os._exit(0)  # the rank disappears between steps, with nothing in flight
    try:
        sh.forward(_cells_cpu(p))
        result = "no error"
    except Exception as e:  # noqa: BLE001 - any collective error is the expected outcome
        result = f"error: {type(e).__name__}"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(result)
    os._exit(0)


def test_lost_rank_gives_error_not_hang(tmp_path):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=120)
    alive = [pr for pr in procs if pr.is_alive()]
    for pr in alive:
        pr.kill()
    assert not alive, "a rank hung"
    assert (tmp_path / "rank0.txt").read_text().startswith("error")


def _shard_inputs(p, device):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)
    return CellTensors(t(p.x), t(p.y), t(p.size_x_clamped), t(p.size_y_clamped), t(p.offset_x), t(p.offset_y),
                       t(p.ratio), ranges=p.ranges)


def _cloned(c):
    return CellTensors(c.x.clone(), c.y.clone(), c.size_x.clone(), c.size_y.clone(), c.offset_x.clone(),
                       c.offset_y.clone(), c.ratio.clone(), ranges=c.ranges)


@pytest.mark.gpu
def test_shard_gather_reuses_forward_band_list(cuda_device):
    """A shard's gather uses the band list its forward kept when it gets the
    same cell arrays, lists again for other arrays, and checks the list again
    once epb_descent_step has moved the cells: every way gives the gradient of
    a fresh listing."""
    import ctypes
    from dreamplacett_framework_b200 import _lib
    from dreamplacett_framework_b200.sharded import EngineShard, halo_rows_for
    p = synth.make_placement("c3", scale=0.1, grid=512)
    M, N, P = p.num_bins_x, p.num_bins_y, 2
    cells = _shard_inputs(p, cuda_device)
    be = EngineShard(M, N, p.xl, p.yl, p.xh, p.yh, P, 0, cuda_device)
    try:
        RB = be.RB
        halo = halo_rows_for(float(np.max(p.size_x_clamped)), be.bin_size_x)
        gen = torch.Generator(device=cuda_device).manual_seed(5)
        fxy = torch.randn((RB + halo) * N * 2, generator=gen, device=cuda_device)
        dens = torch.empty(RB * N, device=cuda_device)
        t1 = torch.empty(RB * N, device=cuda_device)
        n = p.num_nodes

        def gather(c):
            gx = torch.zeros(n, device=cuda_device)
            gy = torch.zeros(n, device=cuda_device)
            be.gather(c, fxy, halo, None, gx, gy)
            return gx, gy

        be.rows_forward(cells, dens, t1)
        reused = gather(cells)
        fresh = gather(_cloned(cells))       # other pointers: a selection of its own
        again = gather(cells)
        for a, b, c in zip(reused, fresh, again):
            assert torch.equal(a, b) and torch.equal(a, c)
        # move the cells by up to 40 bins: some change band; the gather must see it
        gx, gy = reused
        first_row = lambda: np.floor((np_(cells.x) + np_(cells.offset_x) - p.xl) / be.bin_size_x)
        row_before = first_row()
        w, h = cells.size_x, cells.size_y
        linf = torch.zeros(1, device=cuda_device)
        st = be.lib.epb_descent_step(be._h, be._cells(cells), ctypes.c_void_p(cells.x.data_ptr()),
                                     ctypes.c_void_p(cells.y.data_ptr()), ctypes.c_void_p(gx.data_ptr()),
                                     ctypes.c_void_p(gy.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                     ctypes.c_void_p(h.data_ptr()), 40.0, None,
                                     ctypes.c_void_p(linf.data_ptr()))
        assert st == _lib.EPB_OK
        row_after = first_row()
        assert np.count_nonzero((row_before < RB) & (row_after >= RB)) > 0  # cells left band 0
        moved = gather(cells)
        ref = gather(_cloned(cells))
        for a, b in zip(moved, ref):
            assert torch.equal(a, b)
        assert not torch.equal(moved[0], reused[0])
        assert be.error_flags() & ~0x4 == 0
    finally:
        be.close()


@pytest.mark.gpu
def test_shard_stages_reject_misaligned_buffers(cuda_device):
    """The exchanged blocks move as float4 (the field map as float2): a
    misaligned caller buffer is an EPB_EINVAL, before any kernel runs."""
    from dreamplacett_framework_b200 import _lib
    from dreamplacett_framework_b200.sharded import EngineShard
    M = N = 64
    be = EngineShard(M, N, 0.0, 0.0, 640.0, 640.0, 2, 0, cuda_device)
    try:
        f = lambda k: torch.zeros(k + 4, dtype=torch.float32, device=cuda_device)
        t1, g, fxy = f(M * N // 2), f(_lib.COL_OUTPUTS * M * N // 2), f(M * N)
        e = torch.zeros(1, dtype=torch.float64, device=cuda_device)
        with pytest.raises(_lib.EpbError) as ex:
            be.columns(t1[1:], g, True, e)
        assert ex.value.status == _lib.EPB_EINVAL
        with pytest.raises(_lib.EpbError) as ex:
            be.columns(t1, g[2:], True, e)
        assert ex.value.status == _lib.EPB_EINVAL
        with pytest.raises(_lib.EpbError) as ex:
            be.rows_inverse(g[1:], None, None, None, fxy)
        assert ex.value.status == _lib.EPB_EINVAL
        with pytest.raises(_lib.EpbError) as ex:
            be.rows_inverse(g, None, None, None, fxy[1:])
        assert ex.value.status == _lib.EPB_EINVAL
        # aligned buffers pass the checks
        be.columns(t1, g, True, e)
        be.rows_inverse(g, None, None, None, fxy)
        torch.cuda.synchronize()
    finally:
        be.close()


def _shards_vs_one_gpu(p, cells, P, dev):
    """Every band's density and its gather over the one-GPU field maps, against
    the one-GPU engine on the same cells: (band densities, summed gradients,
    one-GPU outputs, one-GPU gradients, the shards' flags, the engine's flags)."""
    from dreamplacett_framework_b200.engine import ElectricPotentialEngine
    from dreamplacett_framework_b200.sharded import EngineShard, halo_rows_for
    M, N, n = p.num_bins_x, p.num_bins_y, p.num_nodes
    with ElectricPotentialEngine(M, N, p.xl, p.yl, p.xh, p.yh, device=dev) as eng:
        ref = {k: v.clone() for k, v in eng.forward(cells).items()}
        rgx, rgy = (g.clone() for g in eng.backward(cells))
        eflags = eng.error_flags()
    shards = [EngineShard(M, N, p.xl, p.yl, p.xh, p.yh, P, q, dev) for q in range(P)]
    try:
        RB = shards[0].RB
        H = halo_rows_for(float(np.nanmax(np.asarray(p.size_x_clamped))), shards[0].bin_size_x)
        dens = torch.zeros(P, RB * N, device=dev)
        t1 = torch.zeros(P, RB * N, device=dev)
        gx = torch.zeros(n, device=dev)
        gy = torch.zeros(n, device=dev)
        for q, be in enumerate(shards):
            be.rows_forward(cells, dens[q], t1[q])
            r0, h = q * RB, (0 if q == P - 1 else H)
            fxy = torch.stack([ref["field_x"][r0:r0 + RB + h], ref["field_y"][r0:r0 + RB + h]], dim=-1)
            be.gather(cells, fxy.reshape(-1).contiguous(), h, None, gx, gy)
        torch.cuda.synchronize()
        flags = [be.error_flags() for be in shards]
    finally:
        for be in shards:
            be.close()
    return dens.reshape(M, N), gx, gy, ref, rgx, rgy, flags, eflags


@pytest.mark.gpu
def test_band_lists_edge_cells(cuda_device):
    """Cells on and across the band edges, beyond the die on every side,
    non-finite and zero-size, then a larger cell set on the same shards' grid
    (the band lists grow): every band's density is the one-GPU density bit for
    bit, the gradients are the one-GPU gradients bit for bit, and the
    non-finite cells are flagged by the shards as by the one GPU."""
    P = 2
    p = synth.make_placement("c1", scale=0.05, grid=256, seed=3)
    n = p.num_nodes
    bsx = (p.xh - p.xl) / p.num_bins_x
    RB = p.num_bins_x // P
    x = p.x.copy()
    sx = np.asarray(p.size_x_clamped, np.float32).copy()
    mov = np.arange(p.num_movable)
    edge = np.float32(p.xl + RB * bsx)
    x[mov[0:50]] = edge                          # starting exactly on the band edge
    x[mov[50:100]] = edge - sx[mov[50:100]]      # ending exactly on it
    x[mov[100:150]] = edge - 0.5 * sx[mov[100:150]]   # straddling it
    x[mov[150:160]] = p.xh + 100.0               # beyond the die, both sides
    x[mov[160:170]] = p.xl - 500.0
    x[mov[170:175]] = np.nan                     # non-finite
    x[mov[175:180]] = np.inf
    sx[mov[180:190]] = 0.0                       # zero width
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda_device)
    cells = CellTensors(t(x), t(p.y), t(sx), t(p.size_y_clamped), t(p.offset_x), t(p.offset_y), t(p.ratio),
                        ranges=p.ranges)
    pe = synth.make_placement("c1", scale=0.05, grid=256, seed=3)
    pe.size_x_clamped = sx
    dens, gx, gy, ref, rgx, rgy, flags, eflags = _shards_vs_one_gpu(pe, cells, P, cuda_device)
    assert torch.equal(dens, ref["density"])
    assert torch.equal(gx, rgx) and torch.equal(gy, rgy)
    assert eflags & 0x1 and any(f & 0x1 for f in flags)
    assert all((f & ~0x1) == 0 for f in flags)
    # a larger cell set: the lists grow and are made again
    p2 = synth.make_placement("c1", scale=0.2, grid=256, seed=5)
    cells2 = CellTensors(t(p2.x), t(p2.y), t(p2.size_x_clamped), t(p2.size_y_clamped), t(p2.offset_x),
                         t(p2.offset_y), t(p2.ratio), ranges=p2.ranges)
    dens, gx, gy, ref, rgx, rgy, flags, eflags = _shards_vs_one_gpu(p2, cells2, P, cuda_device)
    assert torch.equal(dens, ref["density"])
    assert torch.equal(gx, rgx) and torch.equal(gy, rgy)
    assert eflags == 0 and all(f == 0 for f in flags)


@pytest.mark.gpu
@pytest.mark.parametrize("P", [2, 4])
def test_band_lists_follow_moving_cells(cuda_device, P):
    """The band lists are kept across forwards and checked against the
    positions every time.  Cells moved in place by less than the list margin
    (nothing to list again), then by tens of bins (cells enter other bands and
    are listed), then a little again: each time every band's density is the
    one-GPU density bit for bit, and the bands' gathers over the one-GPU field
    maps give the one-GPU gradients bit for bit (each cell by its owner band)."""
    from dreamplacett_framework_b200.engine import ElectricPotentialEngine
    from dreamplacett_framework_b200.sharded import EngineShard, halo_rows_for
    p = synth.make_placement("c3", scale=0.1, grid=512)
    M, N = p.num_bins_x, p.num_bins_y
    cells = _shard_inputs(p, cuda_device)
    n = p.num_nodes
    shards = [EngineShard(M, N, p.xl, p.yl, p.xh, p.yh, P, q, cuda_device) for q in range(P)]
    gen = torch.Generator(device=cuda_device).manual_seed(3)
    try:
        RB = shards[0].RB
        H = halo_rows_for(float(np.max(p.size_x_clamped)), shards[0].bin_size_x)
        dens = torch.zeros(P, RB * N, device=cuda_device)
        t1 = torch.zeros(P, RB * N, device=cuda_device)
        with ElectricPotentialEngine(M, N, p.xl, p.yl, p.xh, p.yh, device=cuda_device) as eng:
            for bins in (0.0, 3.0, 30.0, 2.0):
                if bins:
                    for a, lo, hi, bs in ((cells.x, p.xl, p.xh, shards[0].bin_size_x),
                                          (cells.y, p.yl, p.yh, shards[0].bin_size_y)):
                        step = (torch.rand(n, generator=gen, device=cuda_device) * 2 - 1) * bins * bs
                        a.add_(step).clamp_(lo, hi - 1.0)
                ref = {k: v.clone() for k, v in eng.forward(cells).items()}
                rgx, rgy = (g.clone() for g in eng.backward(cells))
                gx = torch.zeros(n, device=cuda_device)
                gy = torch.zeros(n, device=cuda_device)
                for q, be in enumerate(shards):
                    be.rows_forward(cells, dens[q], t1[q])
                    r0, h = q * RB, (0 if q == P - 1 else H)
                    fxy = torch.stack([ref["field_x"][r0:r0 + RB + h], ref["field_y"][r0:r0 + RB + h]], dim=-1)
                    be.gather(cells, fxy.reshape(-1).contiguous(), h, None, gx, gy)
                torch.cuda.synchronize()
                assert torch.equal(dens.reshape(M, N), ref["density"]), bins
                assert torch.equal(gx, rgx) and torch.equal(gy, rgy), bins
                for be in shards:
                    assert be.error_flags() == 0
    finally:
        for be in shards:
            be.close()


@pytest.mark.gpu
@pytest.mark.parametrize("path", ["cell_order", "tiles"])
@pytest.mark.parametrize("P", [2, 4, 8])
def test_shards_on_one_gpu_match_single_gpu(cuda_device, P, path):
    """Every shard of a P-way split run in turn on one GPU, the all-to-alls, the
    energy sum and the field halo done by tensor copies in the layouts the NCCL
    transport moves: the density is the one-GPU density bit for bit, the fields,
    energy and summed gradients agree within 1e-5.  At 2048² and P >= 4 a band's
    row pass and a strip's column pass launch fewer CTAs than the GPU has SMs, so
    this covers their half-size CTAs.  Both shard paths: the band lists in cell
    order (the default), or each band's tile lists."""
    from dreamplacett_framework_b200 import _lib
    from dreamplacett_framework_b200.engine import ElectricPotentialEngine
    from dreamplacett_framework_b200.sharded import EngineShard, halo_rows_for
    p = synth.make_placement("c3", scale=0.25)
    M, N = p.num_bins_x, p.num_bins_y
    cells = _shard_inputs(p, cuda_device)
    init = torch.from_numpy(p.initial_density_norm()).to(cuda_device)
    with ElectricPotentialEngine(M, N, p.xl, p.yl, p.xh, p.yh, device=cuda_device) as eng:
        eng.set_initial_density(init)
        ref = {k: v.clone() for k, v in eng.forward(cells).items()}
        rgx, rgy = (g.clone() for g in eng.backward(cells))
    RB, NB, K = M // P, N // P, _lib.COL_OUTPUTS
    f = lambda *s, dt=torch.float32: torch.zeros(*s, dtype=dt, device=cuda_device)
    shards = [EngineShard(M, N, p.xl, p.yl, p.xh, p.yh, P, q, cuda_device, path=path) for q in range(P)]
    try:
        H = halo_rows_for(float(np.max(p.size_x_clamped)), shards[0].bin_size_x)
        assert H <= RB
        dens, phi, fx, fy = f(P, RB, N), f(P, RB, N), f(P, RB, N), f(P, RB, N)
        t1_send, t1_recv = f(P, RB * N), f(P, M * NB)
        g_send, g_recv = f(P, K * M * NB), f(P, K * M * NB)
        fxy = f(P, (RB + H) * N * 2)
        energy = f(P, 1, dt=torch.float64)
        for q, be in enumerate(shards):
            be.set_initial_density(init.reshape(-1))
            be.rows_forward(cells, dens[q], t1_send[q])
        # all-to-all: block d of every source goes to rank d, in source order
        for d in range(P):
            for s in range(P):
                t1_recv[d, s * RB * NB:(s + 1) * RB * NB] = t1_send[s, d * RB * NB:(d + 1) * RB * NB]
        for q, be in enumerate(shards):
            be.columns(t1_recv[q], g_send[q], True, energy[q])
        blk = K * RB * NB
        for d in range(P):
            for s in range(P):
                g_recv[d, s * blk:(s + 1) * blk] = g_send[s, d * blk:(d + 1) * blk]
        for q, be in enumerate(shards):
            be.rows_inverse(g_recv[q], phi[q], fx[q], fy[q], fxy[q])
        for q in range(P - 1):  # the first H rows of band q + 1 extend band q
            fxy[q, RB * N * 2:(RB + H) * N * 2] = fxy[q + 1, :H * N * 2]
        gx, gy = f(p.num_nodes), f(p.num_nodes)
        for q, be in enumerate(shards):
            be.gather(cells, fxy[q], 0 if q == P - 1 else H, None, gx, gy)
        torch.cuda.synchronize()
        for be in shards:
            assert be.error_flags() == 0
        assert torch.equal(dens.reshape(M, N), ref["density"])
        rel = lambda a, b: float((a - b).abs().max() / b.abs().max())
        for a, k in ((phi, "potential"), (fx, "field_x"), (fy, "field_y")):
            assert rel(a.reshape(M, N), ref[k]) < 1e-5, k
        assert float(energy.sum().item()) == pytest.approx(float(ref["energy"].item()), rel=1e-5)
        assert rel(gx, rgx) < 1e-5 and rel(gy, rgy) < 1e-5
    finally:
        for be in shards:
            be.close()
