"""GPU parity at the full shapes of BASELINE configs 2, 3 and 4 (depth 8 included), and the
full-ROI gradients of the reference's trained ALU checkpoint, against the float64 oracle.

The reduced-grid cases in test_gpu_parity.py exercise each kernel family; these run the
configurations the scaling target names at their own size, so the run-time radix line
transforms of a 1024 x 1024 FFT grid, the 512 x 512 SAME grid of config 2, depth 8 and the
tiled plane statistics of 65,536- and 925,444-pixel planes are all checked (the reference
runs its tiled epilogue at real plane sizes too: tests/unit_milestone6_general_vnn.py:56-112,
dispatch neurocell/kernels_pallas.py:740-837).  The batch is reduced (2-4 samples) so the
oracle finishes in about a minute at config 4; every other dimension is the config's own.

Tolerance (north_star): relative L2 <= 1e-5 for outputs, loss and both parameter gradients.
"""
import os

import numpy as np
import pytest

from oracle import vnn_oracle as O
from test_gpu_parity import GOLDEN, _rel, check_case, run_gpu, run_oracle

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _config_params(rng_p, rng_f, H, M, kh):
    """Config 0's initialisation at another size: W, B, S ~ N(0, 0.1); filters N(0, 1/kh)."""
    cell = rng_p.normal(0, 0.1, (3, H, H)).astype(np.float32)
    filt = (rng_f.normal(0, 1, (M, 1, kh, kh)) / kh).astype(np.float32)
    return cell, filt


def test_config2_full_shape_parity():
    """256 x 256 SAME grid (65,536-pixel ROI, tiled statistics), K = 31 x 31 (FFT grid
    512 x 512), M = 16, d = 8, 64 coordinate inputs ~ N(0, 1) at column 64, 32 coordinate
    outputs at column 192 with {0, 1} targets, MSE."""
    inp = O.CoordPort(tuple((r, 64) for r in range(96, 160)))
    out = O.CoordPort(tuple((r, 192) for r in range(112, 144)))
    geom = O.make_geometry((256, 256), (31, 31), 16, 8, (inp,), out, padding_mode="SAME")
    assert geom.roi_shape == (256, 256) and geom.fft_shape == (512, 512)
    rng = [np.random.default_rng(2000 + k) for k in range(4)]
    cell, filt = _config_params(rng[0], rng[1], 256, 16, 31)
    B = 2
    x = [rng[2].normal(size=(B, 64)).astype(np.float32)]
    y = rng[3].integers(0, 2, size=(B, 32)).astype(np.float32)
    check_case(geom, O.Config(), cell, filt, x, y)


def test_config3_full_shape_parity():
    """96 x 96 VALID grid, three 32 x 32 image planes on border-touching ports (t = 0 runs
    the full-grid convolution), K = 15 x 15, M = 16, d = 6, ten output cells, softmax CE."""
    ports = (O.RectPort((0, 32), (32, 32)), O.RectPort((32, 32), (32, 32)), O.RectPort((64, 32), (32, 32)))
    out = O.CoordPort(tuple((r, 80) for r in range(43, 53)))
    geom = O.make_geometry(96, (15, 15), 16, 6, ports, out)
    assert not geom.in_in_roi and geom.roi_shape == (82, 82)
    rng = [np.random.default_rng(3000 + k) for k in range(4)]
    cell, filt = _config_params(rng[0], rng[1], 96, 16, 15)
    B = 4
    x = [rng[2].normal(size=(B, 32, 32)).astype(np.float32) for _ in range(3)]
    y = rng[3].integers(0, 10, size=B).astype(np.int32)
    for backend in ("b200", "nchw_direct"):     # FFT regime (auto) and the direct kernels
        check_case(geom, O.Config(), cell, filt, x, y, loss="ce", backend=backend)


def test_config4_full_shape_parity():
    """1024 x 1024 VALID grid (ROI 962 x 962 = 925,444 pixels, FFT grid 1024 x 1024), M = 32,
    K = 63 x 63, d = 8, annealed Codd mode, 128 coordinate inputs and outputs, MSE."""
    inp = O.CoordPort(tuple((r, 128) for r in range(448, 576)))
    out = O.CoordPort(tuple((r, 896) for r in range(448, 576)))
    geom = O.make_geometry((1024, 1024), (63, 63), 32, 8, (inp,), out)
    assert geom.roi_shape == (962, 962) and geom.fft_shape == (1024, 1024)
    rng = [np.random.default_rng(4000 + k) for k in range(4)]
    cell, filt = _config_params(rng[0], rng[1], 1024, 32, 63)
    B = 2
    x = [rng[2].normal(size=(B, 128)).astype(np.float32)]
    y = rng[3].normal(size=(B, 128)).astype(np.float32)
    check_case(geom, O.Config(codd_mode="annealed", state_temperature=0.25), cell, filt, x, y)


@pytest.mark.parametrize("backend", ["b200", "nchw_direct"])
def test_alu_depth8_parity(backend):
    """The ALU chip at depth 8 on the fused per-sample FFT kernels and the direct kernels."""
    geom = O.alu_geometry(depth=8)
    rng = np.random.default_rng(808)
    cell = rng.normal(0, 0.1, (3, 62, 62)).astype(np.float32)
    filt = (rng.normal(0, 1, (16, 1, 23, 13)) / np.sqrt(299)).astype(np.float32)
    x, y, _ = O.alu_batch(rng, 16, noise=0.0)
    check_case(geom, O.Config(), cell, filt, x, y, backend=backend)


@pytest.mark.parametrize("backend", ["b200", "nchw_direct"])
def test_trained_checkpoint_full_roi_gradient_parity(backend):
    """The reference's trained ALU checkpoint (states in [-9.7, 10.2], filters in [-41, 42]:
    the ill-conditioned case for FFT round-off) on the full ROI under ste_ternary: outputs,
    loss and both gradients through the fused FFT kernels (``b200`` on the ALU chip) and the
    direct kernels."""
    import neurocell_b200 as nc
    params = nc.VonNeumannNetwork.load_checkpoint(os.path.join(GOLDEN, "alu_trained_cells.npz"))
    cell = params.cell_params.cpu().numpy()
    filt = params.greens_filters.cpu().numpy()
    assert np.abs(filt).max() > 30.0
    geom = O.alu_geometry()
    rng = np.random.default_rng(909)
    x, y, _ = O.alu_batch(rng, 32, noise=0.0)
    check_case(geom, O.Config(codd_mode="ste_ternary", state_temperature=0.2), cell, filt, x, y,
               backend=backend)
