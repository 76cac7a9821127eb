"""The reference's client surface (scatter_ttnn_client / DREAMPlace operator)
on the B200 engine.  CPU tests check the patching and argument handling;
GPU tests check the numbers against the oracle."""
import numpy as np
import pytest
import torch

import fake_dreamplace
from dreamplacett_framework_b200 import scatter_ttnn_client as stc
from dreamplacett_framework_b200 import synth

REF_TIMING_KEYS = {"pos_write_ms", "kernel_wait_ms", "field_read_ms", "h2d_ms", "scatter_ms", "gather_ms",
                   "d2h_density_ms", "ttnn_upload_ms", "ttnn_compute_ms", "ttnn_download_ms", "fw_ms",
                   "total_server_ms", "total_client_ms", "gather_mode"}


@pytest.fixture
def fake_dp():
    cls, calls = fake_dreamplace.install()
    yield cls, calls
    fake_dreamplace.uninstall()


def test_patch_replaces_forward_and_backward(fake_dp):
    cls, _ = fake_dp
    f0, b0 = cls.forward, cls.backward
    stc.patch_dreamplace(container="", ipc_dir="/tmp/unused", num_cells=0, direct=True)
    assert cls.forward is not f0 and cls.backward is not b0
    assert stc.get_timing_summary() == {}


def test_start_argument_rules():
    c = stc.ScatterTTNNClient("", "", num_bins_x=64, num_bins_y=64, nc_max=0)
    with pytest.raises(ValueError, match="nc_max=0"):
        c.start()
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="CUDA"):
            c.start(nc_actual=10)


@pytest.mark.gpu
def test_cpu_cutover_switch_not_honoured(cuda_device, fake_dp, monkeypatch):
    """The reference's V13_USE_CPU_AFTER_ITER hands later calls back to
    DREAMPlace's own forward; the B200 operator has no CPU path, so every call
    stays on the engine whatever the variable says."""
    cls, calls = fake_dp
    stc.patch_dreamplace()
    monkeypatch.setenv("V13_USE_CPU_AFTER_ITER", "1")
    p = synth.make_placement("c1", scale=0.01)
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda_device)
    t = {k: f(getattr(p, k)) for k in ("size_x_clamped", "size_y_clamped", "offset_x", "offset_y", "ratio")}
    t["initial_density_map"] = f(p.initial_density_map)
    for i in range(3):
        pos = torch.cat([f(p.x), f(p.y)]).requires_grad_(True)
        e = cls.apply(pos, *fake_dreamplace.ep_args(p, t))
        e.backward()
    assert calls["orig_forward"] == 0 and calls["orig_backward"] == 0
    assert stc.get_timing_summary()["n_iters"] == 3
    stc.teardown()


def test_timing_summary_key_contract():
    """timing_summary follows the reference's keys (client:511-531): K_mean and
    K_median for numeric keys, the most frequent value for the others, n_iters
    and n_timed; warm-up calls are dropped only when more calls were made."""
    c = stc.ScatterTTNNClient("", "", num_bins_x=64, num_bins_y=64, nc_max=10)
    assert c.timing_summary() == {}
    for i in range(6):
        c._timings.append({"scatter_ms": float(i), "h2d_ms": 2 * i, "gather_mode": "a" if i != 5 else "b"})
    s = c.timing_summary(n_warmup=2)
    assert set(s) == {"scatter_ms_mean", "scatter_ms_median", "h2d_ms_mean", "h2d_ms_median", "gather_mode",
                      "n_iters", "n_timed"}
    assert s["n_iters"] == 6 and s["n_timed"] == 4
    assert s["scatter_ms_mean"] == pytest.approx(3.5) and s["scatter_ms_median"] == pytest.approx(3.5)
    assert s["h2d_ms_mean"] == pytest.approx(7.0) and s["gather_mode"] == "a"
    s_all = c.timing_summary(n_warmup=10)
    assert s_all["n_timed"] == 6 and s_all["scatter_ms_mean"] == pytest.approx(2.5)
    # a full per-call record gives the reference's summary keys
    c2 = stc.ScatterTTNNClient("", "", num_bins_x=64, num_bins_y=64, nc_max=10)
    rec = {k: 1.0 for k in REF_TIMING_KEYS if k != "gather_mode"}
    rec["gather_mode"] = "epb200"
    c2._timings.append(rec)
    want = {k + sfx for k in REF_TIMING_KEYS if k != "gather_mode" for sfx in ("_mean", "_median")}
    assert set(c2.timing_summary()) == want | {"gather_mode", "n_iters", "n_timed"}


@pytest.mark.gpu
def test_client_call_matches_oracle(cuda_device, oracle):
    p = synth.make_placement("c1", scale=0.3)
    nm = slice(0, p.num_movable)
    px, py, sx, sy = p.x[nm], p.y[nm], p.size_x[nm], p.size_y[nm]
    init = np.random.default_rng(0).random((p.num_bins_x, p.num_bins_y)).astype(np.float32) * 0.1
    c = stc.ScatterTTNNClient("", "", p.num_bins_x, p.num_bins_y, 0, p.xl, p.yl, p.xh, p.yh, direct=True,
                              device=cuda_device)
    c.start(nc_actual=len(px))
    c.set_initial_density(init)
    fx, fy, timing = c.call(px, py, sx, sy)
    assert set(timing) == REF_TIMING_KEYS
    assert fx.device.type == "cpu" and fx.shape == (p.num_bins_x, p.num_bins_y)
    g = oracle.Geometry(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh)
    S = g.default_fixed_bits()
    grid, _ = oracle.density_fixed(oracle.Cells(px, py, sx, sy), g, S)
    rho, _ = oracle.fixed_to_density(grid, g, S, init)
    ref = oracle.solve_fft(rho, g.bsx, g.bsy)
    assert oracle.rel_linf(fx.numpy(), ref["field_x"]) < 1e-5
    assert oracle.rel_linf(fy.numpy(), ref["field_y"]) < 1e-5
    # device inputs give device outputs
    fxd, _, _ = c.call(*(torch.from_numpy(a).to(cuda_device) for a in (px, py, sx, sy)))
    assert fxd.is_cuda and torch.equal(fxd.cpu(), fx)
    for _ in range(5):
        c.call(px, py, sx, sy)
    s = c.timing_summary()
    assert s["n_iters"] == 7 and s["n_timed"] == 3 and s["gather_mode"] == "epb200"
    c.stop()


@pytest.mark.gpu
@pytest.mark.parametrize("on_gpu", [True, False])
def test_patched_operator_forward_backward(cuda_device, oracle, fake_dp, on_gpu):
    cls, calls = fake_dp
    stc.patch_dreamplace(num_cells=0, direct=True)
    p = synth.make_placement("c3", scale=0.05, grid=512)
    dev = cuda_device if on_gpu else torch.device("cpu")
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
    pos = torch.cat([f(p.x), f(p.y)]).requires_grad_(True)
    t = {k: f(getattr(p, k)) for k in ("size_x_clamped", "size_y_clamped", "offset_x", "offset_y", "ratio")}
    t["initial_density_map"] = f(p.initial_density_map)
    energy = cls.apply(pos, *fake_dreamplace.ep_args(p, t))
    energy.backward()
    assert calls["orig_forward"] == 0 and calls["orig_backward"] == 0
    assert energy.device == pos.device and pos.grad.device == pos.device
    # oracle: same stretched cells, initial density normalised in fp32 as the shim does
    g = oracle.Geometry(p.num_bins_x, p.num_bins_y, p.xl, p.yl, p.xh, p.yh)
    init = (t["initial_density_map"] / (p.bin_size_x * p.bin_size_y)).cpu().numpy().astype(np.float32)
    oc = oracle.Cells(p.x, p.y, p.size_x_clamped, p.size_y_clamped, p.offset_x, p.offset_y, p.ratio,
                      ranges=p.ranges)
    S = g.default_fixed_bits()
    grid, _ = oracle.density_fixed(oc, g, S)
    rho, _ = oracle.fixed_to_density(grid, g, S, init)
    ref = oracle.solve_fft(rho, g.bsx, g.bsy)
    assert abs(energy.item() / ref["energy"] - 1) < 1e-5
    gx, gy = oracle.gather(oc, g, ref["field_x"].astype(np.float32), ref["field_y"].astype(np.float32))
    n = p.num_nodes
    got = pos.grad.detach().cpu().numpy()
    assert oracle.rel_linf(got[:n], gx) < 1e-5
    assert oracle.rel_linf(got[n:], gy) < 1e-5
    stc.teardown()


@pytest.mark.gpu
def test_electric_potential_module(cuda_device, oracle):
    from dreamplacett_framework_b200.electric_potential import ElectricPotential
    p = synth.make_placement("c3", scale=0.05, grid=512)
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda_device)
    op = ElectricPotential(f(p.size_x), f(p.size_y), None, None, 1.0, p.xl, p.yl, p.xh, p.yh,
                           p.bin_size_x, p.bin_size_y, p.num_movable, p.num_terminals, p.num_filler)
    pos = torch.cat([f(p.x), f(p.y)]).requires_grad_(True)
    e = op(pos)
    e.backward()
    # the module's stretch equals the generator's and its terminal rasterisation the exact one
    np.testing.assert_allclose(op.ratio.cpu().numpy(), p.ratio, rtol=1e-6)
    idm = op.initial_density_map.cpu().numpy()
    assert np.max(np.abs(idm - p.initial_density_map)) <= 1e-4 * max(1.0, p.initial_density_map.max())
    assert torch.isfinite(pos.grad).all() and float(pos.grad.abs().sum()) > 0
    n = p.num_nodes
    t0, t1 = p.num_movable, p.num_movable + p.num_terminals
    assert torch.count_nonzero(pos.grad[t0:t1]) == 0 and torch.count_nonzero(pos.grad[n + t0:n + t1]) == 0
