"""GPU parity tests: the CUDA path (through the C ABI) against the float64 oracle.

Tolerance (north_star): relative L2 <= 1e-5 for outputs, loss and both parameter
gradients; discrete ste_ternary states must match exactly.
"""
import os

import numpy as np
import pytest
import torch

import neurocell_b200 as nc
from oracle import vnn_oracle as O

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(autouse=True)
def _check_wait_status():
    """Every library call of these tests reads its workspace's status word afterwards and
    fails if a kernel's bounded wait for its own bulk copies gave up."""
    nc.ops.CHECK_WAIT_STATUS = True
    yield
    nc.ops.CHECK_WAIT_STATUS = False
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ACT = {None: None, "tanh": torch.tanh, "sigmoid": torch.sigmoid, "relu": torch.relu,
       "leaky_relu": "leaky_relu", "gelu": "gelu", "identity": "identity"}


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _to_nc_port(p):
    if isinstance(p, O.CoordPort):
        return nc.CoordinatePortSpec(p.coords, p.name)
    return nc.PortSpec(p.offset, p.size, p.name)


def _nc_topo(g: O.Geometry):
    return nc.ChipTopology2D.create(g.grid_shape, g.kernel_size, g.directions, g.depth,
                                    tuple(_to_nc_port(p) for p in g.in_ports),
                                    _to_nc_port(g.out_port), padding_mode=g.padding_mode,
                                    allow_border_output=not g.out_in_roi)


def run_gpu(geom, cfg, cell, filt, inputs, targets, loss="mse", train=True, backend="b200"):
    topo = _nc_topo(geom)
    dev = torch.device("cuda:0")
    cp = torch.tensor(cell, dtype=torch.float32, device=dev, requires_grad=train)
    fl = torch.tensor(filt, dtype=torch.float32, device=dev, requires_grad=train)
    if isinstance(inputs, (list, tuple)):
        xin = [torch.tensor(np.asarray(a), dtype=torch.float32, device=dev) for a in inputs]
    else:
        xin = torch.tensor(inputs, dtype=torch.float32, device=dev)
    out = nc.propagate_vnn_2d(
        nc.VNNParams(cp, fl), xin, topo, activate=ACT[cfg.activate],
        final_activate=ACT[cfg.final_activate], norm=cfg.norm, gated_filters=cfg.gated_filters,
        hard_pin_io=cfg.hard_pin_io, codd_mode=cfg.codd_mode,
        state_temperature=cfg.state_temperature, active_threshold=cfg.active_threshold,
        sharpen_filter=nc.filters.sharpen(norm=True) if cfg.sharpen else None, backend=backend)
    if not train:
        return out.detach().cpu().numpy(), None, None, None
    y = torch.tensor(np.asarray(targets), device=dev)
    L = nc.ops.mse_loss(out, y.float()) if loss == "mse" else nc.ops.softmax_ce_loss(out, y)
    L.backward()
    torch.cuda.synchronize()
    return (out.detach().cpu().numpy(), float(L.detach()), cp.grad.cpu().numpy(),
            fl.grad.cpu().numpy())


def run_oracle(geom, cfg, cell, filt, inputs, targets, loss="mse"):
    out, tape = O.forward(cell, filt, inputs, geom, cfg)
    lval, gout = O.mse_loss(out, targets) if loss == "mse" else O.softmax_ce_loss(out, targets)
    gc, gf = O.backward(gout, tape, geom, cfg)
    return out, lval, gc, gf


def check_case(geom, cfg, cell, filt, inputs, targets, loss="mse", tol=TOL, backend="b200"):
    o_g, l_g, gc_g, gf_g = run_gpu(geom, cfg, cell, filt, inputs, targets, loss, backend=backend)
    o_r, l_r, gc_r, gf_r = run_oracle(geom, cfg, cell, filt, inputs, targets, loss)
    errs = dict(out=_rel(o_g, o_r), loss=abs(l_g - l_r) / max(abs(l_r), 1e-30),
                g_cell=_rel(gc_g, gc_r), g_filters=_rel(gf_g, gf_r))
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"parity failure {bad} (all: {errs})"
    return errs


def alu_problem(B, seed, codd="continuous", tau=1.0, s_uniform=False):
    """Config-0 synthetic distribution: W,B,S ~ N(0,0.1); filters ~ N(0, 1/sqrt(299))."""
    rng = np.random.default_rng(seed)
    geom = O.alu_geometry()
    cell = rng.normal(0, 0.1, (3, 62, 62)).astype(np.float32)
    if s_uniform:
        u = rng.uniform(1e-6, 1 - 1e-6, (62, 62))
        cell[2] = np.log(u / (1 - u)).astype(np.float32)
    filt = (rng.normal(0, 1, (16, 1, 23, 13)) / np.sqrt(299)).astype(np.float32)
    x, y, _ = O.alu_batch(rng, B, noise=0.0)
    return geom, O.Config(codd_mode=codd, state_temperature=tau), cell, filt, x, y


def random_problem(geom, B, seed, pscale=0.3, fscale=None, loss="mse"):
    rng = np.random.default_rng(seed)
    H, W = geom.grid_shape
    kh, kw = geom.kernel_size
    cell = rng.normal(0, pscale, (3, H, W)).astype(np.float32)
    fscale = fscale if fscale is not None else 1.0 / np.sqrt(kh * kw)
    filt = rng.normal(0, fscale, (geom.directions, 1, kh, kw)).astype(np.float32)
    ins = [rng.normal(size=(B,) + tuple(p.size)).astype(np.float32) for p in geom.in_ports]
    n_out = int(np.prod(geom.out_port.size))
    y = (rng.normal(size=(B, n_out)).astype(np.float32) if loss == "mse"
         else rng.integers(0, n_out, size=B).astype(np.int32))
    return cell, filt, ins, y


# ---- BASELINE config 0 shape: ALU train step ------------------------------------------
# "b200" (auto) runs the fused FFT kernels on the ALU chip; "nchw_direct" the specialised
# direct kernels.
ALU_BACKENDS = ("b200", "nchw_direct")


@pytest.mark.parametrize("backend", ALU_BACKENDS)
@pytest.mark.parametrize("codd,tau", [("continuous", 1.0), ("annealed", 0.4),
                                      ("ste_binary", 0.3), ("ste_ternary", 0.3)])
def test_alu_train_step_parity(codd, tau, backend):
    geom, cfg, cell, filt, x, y = alu_problem(16, 100, codd, tau)
    check_case(geom, cfg, cell, filt, x, y, backend=backend)


@pytest.mark.parametrize("backend", ALU_BACKENDS)
def test_alu_train_step_parity_full_batch(backend):
    geom, cfg, cell, filt, x, y = alu_problem(128, 7)
    check_case(geom, cfg, cell, filt, x, y, backend=backend)


# ---- BASELINE config 1 shape: ALU inference, ste_ternary, sigma(S) uniform --------------
@pytest.mark.parametrize("backend", ALU_BACKENDS)
def test_alu_inference_ste_ternary_and_exact_roles(backend):
    geom, cfg, cell, filt, x, y = alu_problem(256, 11, "ste_ternary", 1.0, s_uniform=True)
    o_g, *_ = run_gpu(geom, cfg, cell, filt, x, y, train=False, backend=backend)
    o_r, _ = O.forward(cell, filt, x, geom, cfg)
    assert _rel(o_g, o_r) <= TOL
    topo = _nc_topo(geom)
    s_gpu = nc.compute_codd_state_probs(torch.tensor(cell[2], device="cuda"), topo.io_state_mask,
                                        codd_mode="ste_ternary", state_temperature=1.0,
                                        active_threshold=0.6).cpu().numpy()
    s_ref, _ = O.codd_state_probs(cell[2], geom.io_state_mask, codd_mode="ste_ternary")
    assert np.array_equal(s_gpu, s_ref.astype(np.float32))      # exact discrete roles
    assert set(np.unique(s_gpu)).issubset({0.0, 0.5, 1.0})


def test_ste_ternary_zero_threshold_gap():
    """Outputs with raw states equal outputs with their thresholded roles, bit for bit
    (tests/unit_milestone8_pallas_and_codd.py:235-252)."""
    geom, cfg, cell, filt, x, y = alu_problem(32, 12, "ste_ternary", 0.25, s_uniform=True)
    o1, *_ = run_gpu(geom, cfg, cell, filt, x, y, train=False)
    roles = O.threshold_states(cell[2], 0.6)
    cell2 = cell.copy()
    cell2[2] = np.where(roles >= 2.0, 1.0, np.where(roles > 0.0, 0.3, -1.0))
    o2, *_ = run_gpu(geom, cfg, cell2, filt, x, y, train=False)
    assert np.array_equal(o1, o2)


# ---- BASELINE config 2 shape (SAME, K=31^2, M=16), reduced grid -------------------------
def test_same_mode_large_kernel_parity():
    geom = O.make_geometry(48, (31, 31), 16, 3, (O.CoordPort(tuple((r, 12) for r in range(16, 32))),),
                           O.CoordPort(tuple((r, 36) for r in range(20, 28))), padding_mode="SAME")
    cell, filt, ins, y = random_problem(geom, 2, 21)
    check_case(geom, O.Config(), cell, filt, ins, y)


# ---- BASELINE config 3 shape (96^2, K=15^2, border inputs, CE); planes exceed smem -----
def test_image_classifier_shape_parity():
    ports = (O.RectPort((0, 32), (32, 32)), O.RectPort((32, 32), (32, 32)), O.RectPort((64, 32), (32, 32)))
    out = O.CoordPort(tuple((r, 80) for r in range(43, 53)))
    geom = O.make_geometry(96, (15, 15), 16, 3, ports, out)
    assert not geom.in_in_roi
    cell, filt, ins, y = random_problem(geom, 3, 31, loss="ce")
    check_case(geom, O.Config(), cell, filt, ins, y, loss="ce")


# ---- BASELINE config 4 shape (VALID, K=63^2, M=32, annealed), reduced grid --------------
def test_large_kernel_many_directions_parity():
    geom = O.make_geometry(96, (63, 63), 32, 2, (O.CoordPort(tuple((r, 40) for r in range(40, 56))),),
                           O.CoordPort(tuple((r, 56) for r in range(40, 56))))
    cell, filt, ins, y = random_problem(geom, 2, 41)
    check_case(geom, O.Config(codd_mode="annealed", state_temperature=0.5), cell, filt, ins, y)


# ---- modes and options ------------------------------------------------------------------
@pytest.mark.parametrize("mode", ["VALID", "SAME", "CIRCULAR"])
@pytest.mark.parametrize("cfg", [
    O.Config(),
    O.Config(activate="gelu", final_activate="tanh"),
    O.Config(activate="leaky_relu", final_activate="sigmoid", gated_filters=True),
    O.Config(activate="relu", norm=False, hard_pin_io=True),
    O.Config(activate=None, codd_mode="ste_binary", state_temperature=0.5),
])
def test_modes_and_options_parity(mode, cfg):
    geom = O.make_geometry((20, 22), (5, 3), 4, 3, (O.RectPort((6, 5), (4, 1)),),
                           O.RectPort((6, 14), (4, 1)), padding_mode=mode)
    cell, filt, ins, y = random_problem(geom, 5, 51)
    check_case(geom, cfg, cell, filt, ins, y)


@pytest.mark.parametrize("depth", [1, 2, 5])
def test_depth_and_border_inputs_parity(depth):
    geom = O.make_geometry((24, 24), (7, 5), 6, depth,
                           (O.RectPort((0, 4), (6, 6)), O.CoordPort(((12, 12), (13, 9)))),
                           O.CoordPort(((10, 18), (11, 18), (14, 6))))
    cell, filt, ins, y = random_problem(geom, 4, 61 + depth)
    check_case(geom, O.Config(), cell, filt, ins, y)


@pytest.mark.parametrize("backend", ALU_BACKENDS)
def test_backward_is_deterministic(backend):
    geom, cfg, cell, filt, x, y = alu_problem(32, 5)
    a = run_gpu(geom, cfg, cell, filt, x, y, backend=backend)
    b = run_gpu(geom, cfg, cell, filt, x, y, backend=backend)
    for u, v in zip(a, b):
        assert np.array_equal(np.asarray(u), np.asarray(v))


# ---- functional known answer: the reference's trained checkpoint ------------------------
def test_trained_checkpoint_accuracy_on_gpu():
    params = nc.VonNeumannNetwork.load_checkpoint(os.path.join(GOLDEN, "alu_trained_cells.npz"))
    with np.load(os.path.join(GOLDEN, "alu_trained_eval.npz")) as d:
        x, packed, out_ref = d["inputs"], d["packed"], d["out_f64"]
    model = nc.VonNeumannNetwork(nc.ChipTopology2D.alu_chip(), codd_mode="ste_ternary",
                                 state_temperature=0.2)
    with torch.no_grad():
        out = model.apply(params, torch.tensor(x, device="cuda")).cpu().numpy()
    assert _rel(out, out_ref) <= TOL
    pred = np.packbits(np.clip(np.round(out[:, :, 0]), 0, 255).astype(np.uint8), axis=1)[:, 0]
    assert float((pred == packed).mean()) >= 0.97


def test_sgd_step_matches_oracle():
    geom, cfg, cell, filt, x, y = alu_problem(16, 9)
    topo = _nc_topo(geom)
    p = nc.VNNParams(torch.tensor(cell, device="cuda"), torch.tensor(filt, device="cuda"))
    tr = nc.VNNTrainer(lambda prm, bx: nc.propagate_vnn_2d(prm, bx, topo), lr=1e-2)
    _, loss = tr.train_step(p, torch.tensor(x, device="cuda"), torch.tensor(y, device="cuda"))
    lval, new_cell, new_filt, _, _ = O.train_step(cell, filt, x, y, geom, O.Config(), lr=1e-2)
    assert abs(float(loss) - lval) / lval <= TOL
    # the updated parameters themselves (their fp32 deltas cannot be recovered exactly)
    assert _rel(p.cell_params.cpu().numpy(), new_cell) <= 1e-6
    assert _rel(p.greens_filters.cpu().numpy(), new_filt) <= 1e-6
    assert not np.array_equal(p.cell_params.cpu().numpy(), cell)


# ---- FFT convolution regime ("pallas_sram" backend) -------------------------------------
@pytest.mark.parametrize("mode", ["VALID", "SAME", "CIRCULAR"])
@pytest.mark.parametrize("cfg", [
    O.Config(),
    O.Config(activate="gelu", final_activate="tanh"),
    O.Config(activate="leaky_relu", final_activate="sigmoid", gated_filters=True),
    O.Config(activate="relu", norm=False, hard_pin_io=True),
    O.Config(activate=None, codd_mode="ste_binary", state_temperature=0.5),
])
def test_fft_modes_and_options_parity(mode, cfg):
    geom = O.make_geometry((20, 22), (5, 3), 4, 3, (O.RectPort((6, 5), (4, 1)),),
                           O.RectPort((6, 14), (4, 1)), padding_mode=mode)
    cell, filt, ins, y = random_problem(geom, 5, 51)
    check_case(geom, cfg, cell, filt, ins, y, backend="pallas_sram")


@pytest.mark.parametrize("depth", [1, 2, 5])
def test_fft_depth_and_border_inputs_parity(depth):
    geom = O.make_geometry((24, 24), (7, 5), 6, depth,
                           (O.RectPort((0, 4), (6, 6)), O.CoordPort(((12, 12), (13, 9)))),
                           O.CoordPort(((10, 18), (11, 18), (14, 6))))
    cell, filt, ins, y = random_problem(geom, 4, 61 + depth)
    check_case(geom, O.Config(), cell, filt, ins, y, backend="pallas_sram")


@pytest.mark.parametrize("B", [1, 6])
def test_fft_alu_train_step_parity(B):
    geom, cfg, cell, filt, x, y = alu_problem(B, 71)
    check_case(geom, cfg, cell, filt, x, y, backend="pallas_sram")


def test_fft_and_direct_agree_on_image_classifier_shape():
    ports = (O.RectPort((0, 32), (32, 32)), O.RectPort((32, 32), (32, 32)), O.RectPort((64, 32), (32, 32)))
    out = O.CoordPort(tuple((r, 80) for r in range(43, 53)))
    geom = O.make_geometry(96, (15, 15), 16, 3, ports, out)
    cell, filt, ins, y = random_problem(geom, 3, 31, loss="ce")
    check_case(geom, O.Config(), cell, filt, ins, y, loss="ce", backend="pallas_sram")


def test_fft_backward_is_deterministic():
    geom = O.make_geometry(48, (31, 31), 16, 3, (O.CoordPort(tuple((r, 12) for r in range(16, 32))),),
                           O.CoordPort(tuple((r, 36) for r in range(20, 28))), padding_mode="SAME")
    cell, filt, ins, y = random_problem(geom, 4, 23)
    a = run_gpu(geom, O.Config(), cell, filt, ins, y)
    b = run_gpu(geom, O.Config(), cell, filt, ins, y)
    assert np.array_equal(a[2], b[2]) and np.array_equal(a[3], b[3])


def test_fft_backend_runs_the_fft_kernels():
    """The FFT backend launches the transform kernels (more launches than the two of the
    direct forward) and matches the direct backend on the same inputs."""
    geom = O.make_geometry((20, 22), (5, 3), 4, 3, (O.RectPort((6, 5), (4, 1)),),
                           O.RectPort((6, 14), (4, 1)))
    cell, filt, ins, y = random_problem(geom, 4, 81)
    lib = nc._lib.load()
    n0 = lib.nc_launch_count()
    o_d, *_ = run_gpu(geom, O.Config(), cell, filt, ins, y, train=False, backend="nchw_direct")
    n1 = lib.nc_launch_count()
    o_f, *_ = run_gpu(geom, O.Config(), cell, filt, ins, y, train=False, backend="pallas_sram")
    n2 = lib.nc_launch_count()
    assert n1 - n0 == 2 and n2 - n1 > 10
    assert _rel(o_f, o_d) <= TOL


# ---- fused small-grid FFT kernels (FFT side 64, even M) ---------------------------------
@pytest.mark.parametrize("mode", ["VALID", "SAME", "CIRCULAR"])
@pytest.mark.parametrize("cfg", [
    O.Config(),
    O.Config(activate="gelu", final_activate="tanh"),
    O.Config(activate="leaky_relu", final_activate="sigmoid", gated_filters=True),
    O.Config(activate="relu", norm=False, hard_pin_io=True),
    O.Config(activate=None, codd_mode="ste_binary", state_temperature=0.5),
])
def test_fft_fused_small_grid_parity(mode, cfg):
    geom = O.make_geometry((40, 44), (9, 7), 6, 3, (O.RectPort((10, 8), (4, 1)),),
                           O.RectPort((12, 30), (4, 1)), padding_mode=mode)
    cell, filt, ins, y = random_problem(geom, 3, 91)
    check_case(geom, cfg, cell, filt, ins, y, backend="pallas_sram")


@pytest.mark.parametrize("depth", [1, 2, 5])
def test_fft_fused_depth_and_border_inputs_parity(depth):
    geom = O.make_geometry((48, 50), (9, 7), 4, depth,
                           (O.RectPort((0, 4), (6, 6)), O.CoordPort(((20, 20), (21, 17)))),
                           O.CoordPort(((18, 30), (19, 30), (24, 12))))
    cell, filt, ins, y = random_problem(geom, 4, 95 + depth)
    check_case(geom, O.Config(), cell, filt, ins, y, backend="pallas_sram")


def test_fft_fused_kernel_is_used_for_the_alu_grid():
    """FFT side 64 with even M runs the fused per-sample kernel: one launch for the pre-step
    and the direction-pair filter spectra, one propagation kernel; odd M falls back to the
    per-step kernels and still matches."""
    geom, cfg, cell, filt, x, y = alu_problem(4, 97)
    lib = nc._lib.load()
    n0 = lib.nc_launch_count()
    o_f, *_ = run_gpu(geom, cfg, cell, filt, x, y, train=False, backend="pallas_sram")
    n1 = lib.nc_launch_count()
    o_d, *_ = run_gpu(geom, cfg, cell, filt, x, y, train=False, backend="nchw_direct")
    assert n1 - n0 == 2
    assert _rel(o_f, o_d) <= TOL
    geom5 = O.make_geometry((40, 44), (9, 7), 5, 3, (O.RectPort((10, 8), (4, 1)),),
                            O.RectPort((12, 30), (4, 1)))
    cell, filt, ins, y = random_problem(geom5, 3, 98)
    check_case(geom5, O.Config(), cell, filt, ins, y, backend="pallas_sram")


# ---- return_universe=True (propagator.py:657-734) ----------------------------------------
def _universe_case(geom, cfg, backend, seed):
    cell, filt, ins, _ = random_problem(geom, 3, seed)
    rng = np.random.default_rng(seed + 1)
    H, W = geom.grid_shape
    oh, ow = geom.out_port.size
    wo = rng.normal(size=(3, oh, ow))
    wu = rng.normal(size=(3, H, W))
    topo = _nc_topo(geom)
    dev = torch.device("cuda:0")
    cp = torch.tensor(cell, device=dev, requires_grad=True)
    fl = torch.tensor(filt, device=dev, requires_grad=True)
    xin = [torch.tensor(np.asarray(a), dtype=torch.float32, device=dev) for a in ins]
    out, uni = nc.propagate_vnn_2d(
        nc.VNNParams(cp, fl), xin, topo, activate=ACT[cfg.activate],
        final_activate=ACT[cfg.final_activate], norm=cfg.norm, return_universe=True, backend=backend)
    L = (out * torch.tensor(wo, device=dev, dtype=torch.float32)).sum() + \
        (uni * torch.tensor(wu, device=dev, dtype=torch.float32)).sum()
    L.backward()
    o_r, u_r, tape = O.forward_universe(cell, filt, ins, geom, cfg)
    gu = wu.copy()
    rr, cc = O._out_grid_index(geom)
    gu[:, rr, cc] += wo.reshape(3, -1)
    gc_r, gf_r = O.backward_universe(gu, tape, geom, cfg)
    errs = dict(out=_rel(out.detach().cpu().numpy(), o_r), uni=_rel(uni.detach().cpu().numpy(), u_r),
                g_cell=_rel(cp.grad.cpu().numpy(), gc_r), g_filters=_rel(fl.grad.cpu().numpy(), gf_r))
    bad = {k: v for k, v in errs.items() if not v <= TOL}
    assert not bad, f"universe parity failure {bad} (all: {errs})"


@pytest.mark.parametrize("backend", ["nchw_direct", "pallas_sram"])
@pytest.mark.parametrize("mode", ["VALID", "SAME", "CIRCULAR"])
@pytest.mark.parametrize("final", [None, "tanh"])
def test_return_universe_parity(backend, mode, final):
    geom = O.make_geometry((20, 22), (5, 3), 4, 3, (O.RectPort((6, 5), (4, 1)),),
                           O.RectPort((6, 14), (4, 1)), padding_mode=mode)
    _universe_case(geom, O.Config(final_activate=final), backend, 111)


@pytest.mark.parametrize("mode", ["VALID", "SAME"])
@pytest.mark.parametrize("final", [None, "sigmoid"])
def test_return_universe_fused_fft_parity(mode, final):
    geom = O.make_geometry((40, 44), (9, 7), 6, 3, (O.RectPort((10, 8), (4, 1)),),
                           O.RectPort((12, 30), (4, 1)), padding_mode=mode)
    _universe_case(geom, O.Config(final_activate=final), "pallas_sram", 121)


@pytest.mark.parametrize("backend", ["nchw_direct", "pallas_sram"])
def test_full_grid_outputs_parity(backend):
    """Output port covering the whole grid, ring cells included (the reference's full-grid
    output path, propagator.py:684-734; Game-of-Life style chips)."""
    geom = O.make_geometry((16, 16), (3, 3), 2, 2, (O.RectPort((0, 0), (16, 16)),),
                           O.RectPort((0, 0), (16, 16)))
    assert not geom.out_in_roi
    cell, filt, ins, _ = random_problem(geom, 3, 131)
    rng = np.random.default_rng(132)
    wo = rng.normal(size=(3, 16, 16))
    topo = _nc_topo(geom)
    dev = torch.device("cuda:0")
    cp = torch.tensor(cell, device=dev, requires_grad=True)
    fl = torch.tensor(filt, device=dev, requires_grad=True)
    xin = [torch.tensor(np.asarray(a), dtype=torch.float32, device=dev) for a in ins]
    for final in (None, "sigmoid"):
        cp.grad = None
        fl.grad = None
        cfg = O.Config(final_activate=final)
        out = nc.propagate_vnn_2d(nc.VNNParams(cp, fl), xin, topo, final_activate=ACT[final],
                                  backend=backend)
        (out * torch.tensor(wo, device=dev, dtype=torch.float32)).sum().backward()
        o_r, u_r, tape = O.forward_universe(cell, filt, ins, geom, cfg)
        gu = np.zeros_like(u_r)
        rr, cc = O._out_grid_index(geom)
        gu[:, rr, cc] += wo.reshape(3, -1)
        gc_r, gf_r = O.backward_universe(gu, tape, geom, cfg)
        assert _rel(out.detach().cpu().numpy(), o_r) <= TOL
        assert _rel(cp.grad.cpu().numpy(), gc_r) <= TOL
        assert _rel(fl.grad.cpu().numpy(), gf_r) <= TOL


# ---- adaptive sub-ROI masks (adaptive_mask.py; propagator.py:228-241, 343-371) ----------
def _mask(geom, bbox):
    from neurocell_b200.adaptive_mask import AdaptiveMaskSpec
    r0, r1, c0, c1 = bbox
    return AdaptiveMaskSpec(bbox, (r0 + geom.pad_h, r1 + geom.pad_h, c0 + geom.pad_w, c1 + geom.pad_w),
                            (r1 - r0, c1 - c0), None, None, None, (1, 1), 0.5, 0, False, None, (0, 0))


def _sub_roi_case(geom, cfg, cell, filt, inputs, targets, bbox, backend):
    from oracle import torch_port as T
    topo = _nc_topo(geom)
    dev = torch.device("cuda:0")
    cp = torch.tensor(cell, dtype=torch.float32, device=dev, requires_grad=True)
    fl = torch.tensor(filt, dtype=torch.float32, device=dev, requires_grad=True)
    if isinstance(inputs, (list, tuple)):
        xin = [torch.tensor(np.asarray(a), dtype=torch.float32, device=dev) for a in inputs]
    else:
        xin = torch.tensor(inputs, dtype=torch.float32, device=dev)
    out = nc.propagate_vnn_2d(nc.VNNParams(cp, fl), xin, topo, activate=ACT[cfg.activate],
                              final_activate=ACT[cfg.final_activate], codd_mode=cfg.codd_mode,
                              state_temperature=cfg.state_temperature,
                              active_threshold=cfg.active_threshold,
                              spatial_mask=_mask(geom, bbox), backend=backend)
    L = nc.ops.mse_loss(out, torch.tensor(np.asarray(targets), device=dev).float())
    L.backward()
    l_r, o_r, gc_r, gf_r = T.value_and_grad(geom, cfg, cell, filt, inputs, targets, roi_bbox=bbox)
    errs = dict(out=_rel(out.detach().cpu().numpy(), o_r), loss=abs(float(L.detach()) - l_r) / l_r,
                g_cell=_rel(cp.grad.cpu().numpy(), gc_r), g_filters=_rel(fl.grad.cpu().numpy(), gf_r))
    bad = {k: v for k, v in errs.items() if not v <= TOL}
    assert not bad, f"sub-ROI parity failure {bad} (all: {errs})"


@pytest.mark.parametrize("backend", ALU_BACKENDS)
def test_adaptive_sub_roi_trained_alu_parity(backend):
    params = nc.VonNeumannNetwork.load_checkpoint(os.path.join(GOLDEN, "alu_trained_cells.npz"))
    topo = nc.ChipTopology2D.alu_chip()
    spec = nc.compute_adaptive_spatial_mask(params, topo)
    assert not spec.is_full_roi and spec.active_shape[1] < 50
    geom = O.alu_geometry()
    rng = np.random.default_rng(141)
    x, y, _ = O.alu_batch(rng, 8, noise=0.0)
    _sub_roi_case(geom, O.Config(codd_mode="ste_ternary", state_temperature=0.2),
                  params.cell_params.cpu().numpy(), params.greens_filters.cpu().numpy(), x, y,
                  spec.roi_bbox, backend)


@pytest.mark.parametrize("backend", ["nchw_direct", "pallas_sram"])
@pytest.mark.parametrize("mode", ["VALID", "SAME"])
def test_adaptive_sub_roi_border_inputs_parity(backend, mode):
    """Inputs on the dead ring (VALID) take the full-grid t=0 convolution cropped to the
    sub-ROI; SAME crops the grid itself."""
    ports = ((O.RectPort((0, 4), (6, 6)), O.CoordPort(((12, 12), (13, 9)))) if mode == "VALID"
             else (O.CoordPort(((12, 12), (13, 9), (16, 14))),))
    geom = O.make_geometry((28, 30), (7, 5), 4, 3, ports, O.CoordPort(((14, 16), (15, 16), (18, 12))),
                           padding_mode=mode)
    cell, filt, ins, y = random_problem(geom, 3, 151)
    _sub_roi_case(geom, O.Config(), cell, filt, ins, y, (6, 20, 6, 22), backend)


def _sub_roi_universe_case(geom, cfg, cell, filt, inputs, bbox, backend, seed):
    """return_universe=True with an adaptive sub-ROI (propagator.py:700-718, 726-733)."""
    from oracle import torch_port as T
    rng = np.random.default_rng(seed)
    B = (inputs[0] if isinstance(inputs, (list, tuple)) else inputs).shape[0]
    H, W = geom.grid_shape
    wo = rng.normal(size=(B,) + tuple(geom.out_port.size))
    wu = rng.normal(size=(B, H, W))
    topo = _nc_topo(geom)
    dev = torch.device("cuda:0")
    cp = torch.tensor(cell, dtype=torch.float32, device=dev, requires_grad=True)
    fl = torch.tensor(filt, dtype=torch.float32, device=dev, requires_grad=True)
    if isinstance(inputs, (list, tuple)):
        xin = [torch.tensor(np.asarray(a), dtype=torch.float32, device=dev) for a in inputs]
    else:
        xin = torch.tensor(inputs, dtype=torch.float32, device=dev)
    out, uni = nc.propagate_vnn_2d(nc.VNNParams(cp, fl), xin, topo, activate=ACT[cfg.activate],
                                   final_activate=ACT[cfg.final_activate], codd_mode=cfg.codd_mode,
                                   state_temperature=cfg.state_temperature,
                                   active_threshold=cfg.active_threshold, return_universe=True,
                                   spatial_mask=_mask(geom, bbox), backend=backend)
    assert uni.shape == (B, H, W)
    L = (out * torch.tensor(wo, device=dev, dtype=torch.float32)).sum() + \
        (uni * torch.tensor(wu, device=dev, dtype=torch.float32)).sum()
    L.backward()
    o_r, u_r, gc_r, gf_r = T.universe_value_and_grad(geom, cfg, cell, filt, inputs, wo, wu, roi_bbox=bbox)
    errs = dict(out=_rel(out.detach().cpu().numpy(), o_r), uni=_rel(uni.detach().cpu().numpy(), u_r),
                g_cell=_rel(cp.grad.cpu().numpy(), gc_r), g_filters=_rel(fl.grad.cpu().numpy(), gf_r))
    bad = {k: v for k, v in errs.items() if not v <= TOL}
    assert not bad, f"sub-ROI universe parity failure {bad} (all: {errs})"


@pytest.mark.parametrize("backend", ALU_BACKENDS)
def test_adaptive_sub_roi_universe_trained_alu_parity(backend):
    params = nc.VonNeumannNetwork.load_checkpoint(os.path.join(GOLDEN, "alu_trained_cells.npz"))
    spec = nc.compute_adaptive_spatial_mask(params, nc.ChipTopology2D.alu_chip())
    geom = O.alu_geometry()
    x, _, _ = O.alu_batch(np.random.default_rng(161), 6, noise=0.0)
    _sub_roi_universe_case(geom, O.Config(codd_mode="ste_ternary", state_temperature=0.2),
                           params.cell_params.cpu().numpy(), params.greens_filters.cpu().numpy(), x,
                           spec.roi_bbox, backend, 162)


@pytest.mark.parametrize("backend", ["nchw_direct", "pallas_sram"])
@pytest.mark.parametrize("mode", ["VALID", "SAME"])
@pytest.mark.parametrize("final", [None, "sigmoid"])
def test_adaptive_sub_roi_universe_outputs_outside_window(backend, mode, final):
    """Output cells inside the sub-ROI, in the ROI outside the window and on the VALID ring:
    the outputs are read from the assembled full grid."""
    ports = ((O.RectPort((0, 4), (6, 6)), O.CoordPort(((12, 12), (13, 9)))) if mode == "VALID"
             else (O.CoordPort(((12, 12), (13, 9), (16, 14))),))
    outs = ((14, 16), (4, 10), (2, 3), (27, 28)) if mode == "VALID" else ((14, 16), (4, 10), (1, 1))
    geom = O.make_geometry((28, 30), (7, 5), 4, 3, ports, O.CoordPort(outs), padding_mode=mode,
                           allow_border_output=True)
    cell, filt, ins, _ = random_problem(geom, 3, 171)
    _sub_roi_universe_case(geom, O.Config(final_activate=final), cell, filt, ins, (6, 20, 6, 22),
                           backend, 172)


def test_zz_workspace_status_was_read():
    """Runs after the parity tests of this module.  Their library calls had their workspace
    status words read (a bounded wait that gave up would have failed them), and a forward
    clears a status word that holds a stale value when it starts (nc_workspace_status)."""
    import ctypes
    from neurocell_b200 import _lib
    assert nc.ops.STATUS_CHECKS > 0
    lib = _lib.load()
    dev = torch.device("cuda:0")
    geom, cfg, cell, filt, x, y = alu_problem(4, 5)
    plan = nc.ops.get_plan(_nc_topo(geom), ((8, 1),) * 3, dev, "tanh", 0.0, "identity", 1.0,
                           True, False, False)
    B = 4
    ws_bytes = lib.nc_workspace_bytes(ctypes.byref(plan.topo), B, 0)
    ws = torch.full((ws_bytes,), 0xFF, dtype=torch.uint8, device=dev)   # stale word: -1
    assert nc.ops.workspace_status(ws) == -1
    out = torch.empty((B, plan.n_out), device=dev)
    xs = torch.tensor(x.reshape(B, -1), device=dev)
    c = torch.tensor(cell, device=dev)
    f = torch.tensor(filt, device=dev)
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(lib.nc_vnn_forward(ctypes.byref(plan.topo), ctypes.c_void_p(plan.buf.data_ptr()),
                                  ctypes.c_void_p(c.data_ptr()), ctypes.c_void_p(f.data_ptr()),
                                  ctypes.c_void_p(xs.data_ptr()), B, ctypes.byref(nc.ops._codd("continuous", 1.0, 0.6)),
                                  0, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(ws.data_ptr()),
                                  ws_bytes, st), "nc_vnn_forward")
    assert nc.ops.workspace_status(ws) == 0


# ---- two-stage line transforms of the FFT regime (N = 64 R: 128 .. 1024) ----------------
# The planner takes the smallest N = 64 R >= the field side with R in {2, 3, 4, 5, 6, 8, 16}
# (a power of two up to 64).  FFT grid (rows x columns of the transform) noted per case.
@pytest.mark.parametrize("grid,kernel,mode", [
    ((160, 160), (31, 31), "VALID"),     # 192 x 192 (R = 3, 3)
    ((220, 140), (9, 9), "VALID"),       # 256 x 192 (R = 4 columns, R = 3 rows)
    ((300, 100), (9, 9), "VALID"),       # 320 x 128 (R = 5, R = 2)
    ((280, 20), (17, 5), "SAME"),        # 320 x 32: two-stage columns, radix-4 rows
    ((350, 70), (7, 7), "VALID"),        # 384 x 128 (R = 6, R = 2)
    ((100, 350), (5, 9), "SAME"),        # 128 x 384 (R = 2, R = 6)
    ((260, 40), (7, 7), "CIRCULAR"),     # 320 x 64 (R = 5, R = 1), wrapped halo
    ((450, 64), (9, 9), "VALID"),        # 512 x 64 (R = 8, R = 1)
    ((600, 60), (25, 5), "VALID"),       # 1024 x 64 (R = 16, R = 1)
])
def test_fft_two_stage_line_transforms_parity(grid, kernel, mode):
    H, W = grid
    r0 = H // 2 - 2
    geom = O.make_geometry(grid, kernel, 4, 2, (O.CoordPort(tuple((r, W // 3) for r in range(r0, r0 + 4))),),
                           O.CoordPort(tuple((r, 2 * W // 3) for r in range(r0, r0 + 3))), padding_mode=mode)
    cell, filt, ins, y = random_problem(geom, 2, 181)
    check_case(geom, O.Config(codd_mode="ste_ternary", state_temperature=0.5), cell, filt, ins, y,
               backend="pallas_sram")


# ---- direction blocks of the filter-gradient accumulation, odd direction counts ---------
@pytest.mark.parametrize("grid,kernel,M", [
    ((300, 150), (9, 9), 16),    # FFT 320 x 192: the accumulation holds 8 directions per thread
    ((160, 160), (31, 31), 5),   # FFT 192 x 192, M odd: blocks of 2 with a partial last block,
                                 # and the paired-direction reductions end on a single direction
])
def test_fft_direction_blocks_parity(grid, kernel, M):
    H, W = grid
    r0 = H // 2 - 2
    geom = O.make_geometry(grid, kernel, M, 2, (O.CoordPort(tuple((r, W // 3) for r in range(r0, r0 + 4))),),
                           O.CoordPort(tuple((r, 2 * W // 3) for r in range(r0, r0 + 3))))
    cell, filt, ins, y = random_problem(geom, 3, 191 + M)
    check_case(geom, O.Config(), cell, filt, ins, y, backend="pallas_sram")


# ---- the sharpen weight filter (model.py:65-66, params.py:246-247) ----------------------
@pytest.mark.parametrize("backend", ["b200", "nchw_direct", "pallas_sram"])
def test_sharpen_filter_parity(backend):
    """W sharpened by the normalised 3x3 stencil before the pin, on every kernel family
    (the ALU chip: fused 64x64 FFT kernels for "b200", direct kernels, per-step FFT kernels)."""
    geom, cfg, cell, filt, x, y = alu_problem(4, 211)
    check_case(geom, O.Config(sharpen=True), cell, filt, x, y, backend=backend)


def test_sharpen_option_of_the_model_facade():
    geom, cfg, cell, filt, x, y = alu_problem(2, 212)
    topo = _nc_topo(geom)
    dev = torch.device("cuda:0")
    p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
    xin = torch.tensor(x, dtype=torch.float32, device=dev)
    out = nc.VonNeumannNetwork(topo, sharpen=True).apply(p, xin)
    ref, _ = O.forward(cell, filt, x, geom, O.Config(sharpen=True))
    assert _rel(out.cpu().numpy(), ref) <= TOL


# ---- an output cell listed twice ----------------------------------------------------------
# Legal in the reference (CoordinatePortSpec does not require distinct coordinates,
# topology.py:38-56; its gather gives such a cell the sum of its ports' gradients).  The
# library's port kernels assume one port per cell, so the plan refuses the port list with
# NC_ERR_UNSUPPORTED on every path instead of computing a wrong gradient.
@pytest.mark.parametrize("backend,grid,ks", [
    ("b200", 62, (23, 13)),          # fused per-sample FFT kernels (64 x 64 grid)
    ("nchw_direct", 62, (23, 13)),   # direct kernels
    ("pallas_sram", 96, (23, 23)),   # FFT regime (128-point lines)
])
def test_duplicate_output_cell_is_refused(backend, grid, ks):
    c = grid // 2
    inp = O.CoordPort(((c - 5, 12), (c, 12), (c + 5, 12)))
    out = O.CoordPort(((c, grid - 14), (c + 3, grid - 14), (c, grid - 14), (c - 2, grid - 14)))
    geom = O.make_geometry(grid, ks, 4, 3, (inp,), out)
    cell, filt, ins, y = random_problem(geom, 6, 61)
    with pytest.raises(NotImplementedError, match="duplicate output cell"):
        run_gpu(geom, O.Config(), cell, filt, ins, y, backend=backend)
