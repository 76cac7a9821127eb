"""NCCL multi-GPU parity: the sharded pipeline over 2..4 GPUs against the
one-GPU engine on the same cells.  Needs two or more GPUs (skipped otherwise);
every rank runs on its own GPU.  NVLS is disabled (NCCL_NVLS_ENABLE=0)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir, config, grid, scale, transport):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from dreamplacett_framework_b200 import synth
    from dreamplacett_framework_b200.engine import CellTensors
    from dreamplacett_framework_b200.sharded import ShardedElectricPotential
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    sh = None
    try:
        p = synth.make_placement(config, scale=scale, grid=grid)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
        cells = CellTensors(t(p.x), t(p.y), t(p.size_x_clamped), t(p.size_y_clamped), t(p.offset_x),
                            t(p.offset_y), t(p.ratio), ranges=p.ranges)
        sh = ShardedElectricPotential(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh,
                                      float(p.size_x_clamped.max()), device=dev, transport=transport)
        sh.set_initial_density(t(p.initial_density_norm()))
        for _ in range(2):  # the second call checks the band grid was left zeroed
            out = sh.forward(cells)
            gx, gy = sh.backward(cells)
        if transport == "peer":
            # a captured step (the signal epoch lives on the device) replays to the eager results
            ref = {k: out[k].clone() for k in ("density", "potential", "field_x", "field_y", "energy")}
            rgx, rgy = gx.clone(), gy.clone()
            o2 = {k: torch.empty_like(out[k]) for k in ("density", "potential", "field_x", "field_y")}
            g2x, g2y = torch.zeros_like(gx), torch.zeros_like(gy)
            cur = torch.cuda.current_stream(dev)
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(cur)
            graph = torch.cuda.CUDAGraph()
            dist.barrier()
            with torch.cuda.graph(graph, stream=cap):
                o2c = sh.forward(cells, out=o2)
                sh.backward(cells, grad_x=g2x, grad_y=g2y)
            dist.barrier()
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize(dev)
            for k in ("density", "potential", "field_x", "field_y", "energy"):
                assert torch.equal(o2c[k], ref[k]), k
            assert torch.equal(g2x, rgx) and torch.equal(g2y, rgy)
            graph = None
        # the host-buffer calls: positions from pinned [x | y], each rank copying its node slice and an
        # all-gather completing them; the summed gradient back, each rank storing its slice
        n = p.num_nodes
        keep = {k: out[k].clone() for k in ("density", "potential", "field_x", "field_y", "energy")}
        host_pos = torch.cat([cells.x, cells.y]).cpu().pin_memory()
        cells2 = CellTensors(torch.zeros_like(cells.x), torch.zeros_like(cells.y), cells.size_x, cells.size_y,
                             cells.offset_x, cells.offset_y, cells.ratio, ranges=p.ranges)
        out2 = sh.forward_host(cells2, host_pos)
        host_grad = torch.full((2 * n,), float("nan")).pin_memory()
        sh.backward_host(cells2, host_grad)
        torch.cuda.synchronize(dev)
        for k in keep:
            assert torch.equal(out2[k], keep[k]), k
        lo, hi, _ = sh.node_slice(n)
        flags = sh.be.error_flags()
        torch.cuda.synchronize(dev)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"),
                 **{k: keep[k].cpu().numpy() for k in keep},
                 gx=gx.cpu().numpy(), gy=gy.cpu().numpy(), flags=np.array(flags),
                 host_gx=host_grad[lo:hi].numpy(), host_gy=host_grad[n + lo:n + hi].numpy())
        dist.barrier()
        torch.cuda.synchronize(dev)
    finally:
        if sh is not None:
            sh.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "peer"])
@pytest.mark.parametrize("config,grid,scale", [("c3", 1024, 0.2), ("c3", 2048, 1.0), ("c4", None, 1.0)])
def test_nccl_shards_match_single_gpu(cuda_device, tmp_path, config, grid, scale, transport):
    """The full C3 (2048²) and C4 (4096², 2.5M cells) steps, and a small C3-like
    case, on 2 (or 4) GPUs against the one-GPU engine."""
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs 2+ GPUs")
    world = 4 if ngpu >= 4 else 2
    from dreamplacett_framework_b200 import synth
    from dreamplacett_framework_b200.engine import CellTensors, ElectricPotentialEngine
    p = synth.make_placement(config, scale=scale, grid=grid)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda_device)
    cells = CellTensors(t(p.x), t(p.y), t(p.size_x_clamped), t(p.size_y_clamped), t(p.offset_x), t(p.offset_y),
                        t(p.ratio), ranges=p.ranges)
    with ElectricPotentialEngine(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh, device=cuda_device) as eng:
        eng.set_initial_density(t(p.initial_density_norm()))
        ref = {k: v.cpu().numpy() for k, v in eng.forward(cells).items()}
        rgx, rgy = (a.cpu().numpy() for a in eng.backward(cells))
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path), config, grid, scale, transport), nprocs=world,
                       start_method="spawn")
    parts = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    np.testing.assert_array_equal(np.concatenate([q["density"] for q in parts]), ref["density"])
    rel = lambda a, b: float(np.max(np.abs(a - b)) / np.max(np.abs(b)))
    for k in ("potential", "field_x", "field_y"):
        assert rel(np.concatenate([q[k] for q in parts]), ref[k]) < 1e-5, k
    for q in parts:
        assert abs(float(q["energy"][0]) / float(ref["energy"][0]) - 1) < 1e-5
        assert int(q["flags"]) == 0
    assert rel(sum(q["gx"] for q in parts), rgx) < 1e-5
    assert rel(sum(q["gy"] for q in parts), rgy) < 1e-5
    # the host-buffer path: the ranks' slices, in rank order, are the summed gradient
    np.testing.assert_array_equal(np.concatenate([q["host_gx"] for q in parts]), sum(q["gx"] for q in parts))
    np.testing.assert_array_equal(np.concatenate([q["host_gy"] for q in parts]), sum(q["gy"] for q in parts))
