"""CPU tests of the host side: the C-ABI library loads and exports every declared symbol,
host-only entry points validate geometry, and the Python mirror of the reference API
(topology, port flattening, errors) matches the oracle's restatement."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

import neurocell_b200 as nc
from neurocell_b200 import _lib, ops
from neurocell_b200.propagator import flatten_inputs
from oracle import vnn_oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "neurocell_b200.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(nc_[a-z0-9_]+)\s*\(", src)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert sorted(_lib.EXPORTED) == declared
    assert lib.nc_abi_version() == _lib.ABI_VERSION


def _alu_topo():
    t = _lib.NcTopo()
    t.H, t.W, t.kh, t.kw, t.M, t.depth = 62, 62, 23, 13, 16, 4
    t.padding, t.n_in, t.n_out, t.act, t.final_act, t.norm = 0, 24, 8, 1, 0, 1
    return t


def test_host_only_entry_points_validate_geometry():
    lib = _lib.load()
    t = _alu_topo()
    assert lib.nc_plan_bytes(ctypes.byref(t)) > 0
    ws_train = lib.nc_workspace_bytes(ctypes.byref(t), 128, _lib.NC_FLAG_TRAIN)
    ws_inf = lib.nc_workspace_bytes(ctypes.byref(t), 128, 0)
    # train keeps (d, M, P) standardised planes per sample: 4*16*2000 floats
    assert ws_train > 128 * 4 * 16 * 2000 * 4 > ws_inf > 0
    t.kh = 22   # even kernel -> invalid
    assert lib.nc_plan_bytes(ctypes.byref(t)) == 0
    assert lib.nc_workspace_bytes(ctypes.byref(t), 128, 0) == 0
    t.kh = 23
    assert lib.nc_workspace_bytes(ctypes.byref(t), 0, 0) == 0


def _ws(t, algo, B=8):
    t.conv_algo = algo
    return _lib.load().nc_workspace_bytes(ctypes.byref(t), B, _lib.NC_FLAG_TRAIN)


def test_conv_algorithm_selection():
    """AUTO picks the FFT regime for large kernels (the reference's kh*kw > 512 rule), for
    mid-size kernels whose planes do not fit on chip and for 64 x 64 FFT grids with at least
    11 x 11 taps (the fused kernels); small kernels stay direct; FFT grids above 1024 per
    side are refused."""
    lib = _lib.load()
    t = _alu_topo()
    assert _ws(t, 0) == _ws(t, 2) != _ws(t, 1)    # ALU chip: fused 64 x 64 FFT kernels
    t.kh, t.kw = 5, 3
    assert _ws(t, 0) == _ws(t, 1) != _ws(t, 2)    # small kernels: direct
    t.kh, t.kw = 23, 13
    t.H = t.W = 256
    t.kh = t.kw = 31
    t.padding = 1                     # BASELINE config 2 shape
    assert _ws(t, 0) == _ws(t, 2) != _ws(t, 1)
    t.H = t.W = 96
    t.kh = t.kw = 15
    t.padding = 0                     # BASELINE config 3 shape: planes off chip
    assert _ws(t, 0) == _ws(t, 2) != _ws(t, 1)
    t.H = t.W = 24
    t.kh = t.kw = 9                   # small planes stay on chip
    assert _ws(t, 0) == _ws(t, 1) != _ws(t, 2)
    t.H = t.W = 1500
    t.kh = t.kw = 63                  # FFT side 2048
    t.conv_algo = 2
    assert lib.nc_plan_bytes(ctypes.byref(t)) == 0
    assert b"exceeds" in lib.nc_last_error()
    t.conv_algo = 0                   # AUTO falls back to the direct path
    assert lib.nc_plan_bytes(ctypes.byref(t)) > 0
    t.conv_algo = 7
    assert lib.nc_plan_bytes(ctypes.byref(t)) == 0


def test_backend_names_select_the_convolution():
    from neurocell_b200.propagator import CONV_OF_BACKEND, SUPPORTED_BACKENDS
    assert set(CONV_OF_BACKEND) == set(SUPPORTED_BACKENDS)
    assert CONV_OF_BACKEND["pallas_sram"] == "fft" and CONV_OF_BACKEND["nchw_direct"] == "direct"


def test_null_and_invalid_arguments_fail_without_touching_the_gpu():
    lib = _lib.load()
    t = _alu_topo()
    c = _lib.NcCodd(0, 1.0, 0.6)
    st = lib.nc_vnn_forward(ctypes.byref(t), None, None, None, None, 8, ctypes.byref(c), 0, None,
                            None, 0, None)
    assert st == _lib.NC_ERR_INVALID
    assert b"null" in lib.nc_last_error()
    c.mode = 9
    assert lib.nc_codd_states(ctypes.byref(t), ctypes.c_void_p(256), ctypes.c_void_p(256),
                              ctypes.byref(c), ctypes.c_void_p(256), None) == _lib.NC_ERR_INVALID
    assert b"codd_mode" in lib.nc_last_error()
    assert lib.nc_sgd_update(None, None, 0, 0.1, None) == _lib.NC_ERR_INVALID


@pytest.mark.parametrize("make", [
    lambda: (nc.ChipTopology2D.alu_chip(), O.alu_geometry()),
    lambda: (nc.ChipTopology2D.create((24, 24), (7, 5), 4, 3, (nc.PortSpec((0, 4), (6, 6)),),
                                      nc.CoordinatePortSpec([(10, 18), (11, 18)]), padding_mode="VALID"),
             O.make_geometry((24, 24), (7, 5), 4, 3, (O.RectPort((0, 4), (6, 6)),),
                             O.CoordPort(((10, 18), (11, 18))))),
    lambda: (nc.ChipTopology2D.create(32, (31, 31), 16, 8, (nc.CoordinatePortSpec([(r, 8) for r in range(4, 20)]),),
                                      nc.CoordinatePortSpec([(r, 24) for r in range(8, 16)]), padding_mode="SAME"),
             O.make_geometry(32, (31, 31), 16, 8, (O.CoordPort(tuple((r, 8) for r in range(4, 20))),),
                             O.CoordPort(tuple((r, 24) for r in range(8, 16))), padding_mode="SAME")),
])
def test_topology_mirror_matches_oracle(make):
    t, g = make()
    assert t.grid_shape == g.grid_shape and t.roi_shape == g.roi_shape
    assert (t.pad_h, t.pad_w) == (g.pad_h, g.pad_w) and t.fft_shape == g.fft_shape
    assert t.roi_out_offset == g.roi_out_offset
    assert (t.in_in_roi, t.out_in_roi) == (g.in_in_roi, g.out_in_roi)
    assert np.array_equal(t.io_state_mask, g.io_state_mask)
    assert np.array_equal(t.out_weight_mask, g.out_weight_mask)


def test_topology_errors_mirror_reference_messages():
    with pytest.raises(ValueError, match="must be odd"):
        nc.ChipTopology2D.create((62, 62), (22, 13), 16, 4, (nc.PortSpec((23, 23), (8, 1)),),
                                 nc.PortSpec((27, 41), (8, 1)))
    with pytest.raises(ValueError, match="outside the active VALID"):
        nc.ChipTopology2D.create((62, 62), (23, 13), 16, 4, (nc.PortSpec((23, 23), (8, 1)),),
                                 nc.PortSpec((2, 41), (8, 1)))
    with pytest.raises(ValueError, match="padding_mode"):
        nc.ChipTopology2D.create((62, 62), (23, 13), 16, 4, (nc.PortSpec((23, 23), (8, 1)),),
                                 nc.PortSpec((27, 41), (8, 1)), padding_mode="REFLECT")


def test_input_flattening_reproduces_ctrl_column_quirk():
    """(B,3,8,1) ALU inputs: ctrl's (8,1) array lands as a column at (18,28) (propagator.py:183-185)."""
    topo = nc.ChipTopology2D.alu_chip()
    g = O.alu_geometry()
    rng = np.random.default_rng(0)
    x = rng.normal(size=(4, 3, 8, 1)).astype(np.float32)
    flat, shapes = flatten_inputs(torch.from_numpy(x), topo)
    assert shapes == ((8, 1), (8, 1), (8, 1)) and flat.shape == (4, 24)
    idx = ops._input_index(topo, shapes)
    field = np.zeros((4, 62 * 62), np.float32)
    field[:, idx] = flat.numpy()
    ref = O.inject_full(x, g, np.float32).reshape(4, -1)
    assert np.array_equal(field, ref)
    ctrl_cells = idx[16:]
    assert list(ctrl_cells // 62) == list(range(18, 26)) and set(ctrl_cells % 62) == {28}


def test_duplicate_input_cells_keep_the_last_write():
    topo = nc.ChipTopology2D.create((16, 16), (3, 3), 2, 2,
                                    (nc.PortSpec((4, 4), (2, 2)), nc.PortSpec((5, 5), (2, 2))),
                                    nc.PortSpec((8, 8), (1, 1)))
    idx = ops._input_index(topo, ((2, 2), (2, 2)))
    assert idx[3] == -1 and idx[4] == 5 * 16 + 5


def test_api_errors_mirror_reference():
    topo = nc.ChipTopology2D.alu_chip()
    p = nc.VNNParams(torch.zeros(3, 62, 62), torch.zeros(16, 1, 23, 13))
    x = torch.zeros(2, 3, 8, 1)
    with pytest.raises(ValueError, match="Unsupported backend"):
        nc.propagate_vnn_2d(p, x, topo, backend="tpu")
    with pytest.raises(ValueError, match="Unsupported codd_mode"):
        nc.propagate_vnn_2d(p, x, topo, codd_mode="soft")
    with pytest.raises(ValueError, match="Unsupported activation"):
        nc.propagate_vnn_2d(p, x, topo, activate=torch.exp)
    with pytest.raises(ValueError, match="CUDA tensor"):   # no CPU path
        nc.propagate_vnn_2d(p, x, topo)
    assert set(nc.SUPPORTED_CODD_MODES) == {"continuous", "annealed", "ste_binary", "ste_ternary"}


def test_annealed_temperature_schedule():
    assert nc.compute_annealed_temperature(0, 10, 1.0, 0.1) == pytest.approx(1.0)
    assert nc.compute_annealed_temperature(9, 10, 1.0, 0.1) == pytest.approx(0.1)
    assert nc.compute_annealed_temperature(5, 11, 1.0, 0.1, "linear") == pytest.approx(0.55)
    with pytest.raises(ValueError):
        nc.compute_annealed_temperature(1, 3, schedule="step")


def test_filter_stencils_and_spatial_filter():
    """The reference's stencils (filters.py:12-83) and apply_spatial_filter_2d
    (kernels_greens.py:220-237) on CPU tensors, against the oracle's SAME correlation."""
    f = nc.filters
    assert f.sharpen(norm=False).tolist() == [[0, -1, 0], [-1, 5, -1], [0, -1, 0]]
    assert torch.allclose(f.sharpen(), f.sharpen(norm=False) / 5)
    assert f.smooth(norm=True).tolist() == [[1, 1, 1], [1, 8, 1], [1, 1, 1]]
    assert f.backward(norm=True).tolist() == [[1, 0, 0], [1, 3, 0], [1, 0, 0]]
    assert f.forward().tolist() == [[0, 0, 1], [0, 0, 1], [0, 0, 1]]
    assert f.von_neumann().tolist() == [[1, 0, 1], [1, 1, 1], [1, 0, 1]]
    k3 = f.sharpen_3d(norm=False)
    assert k3.shape == (3, 3, 3) and float(k3.sum()) == -1.0 and float(k3[1, 1, 1]) == 5.0
    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.normal(size=(10, 8)))
    k = torch.from_numpy(rng.normal(size=(3, 3)))
    same = nc.apply_spatial_filter_2d(x, k)
    assert same.shape == (10, 8)
    assert np.allclose(same.numpy(), O.spatial_filter_same(x.numpy(), k.numpy()), atol=1e-13)
    assert nc.apply_spatial_filter_2d(x, k, padding="VALID").shape == (8, 6)
    with pytest.raises(ValueError):
        nc.apply_spatial_filter_2d(x, torch.ones(2, 2))
    with pytest.raises(ValueError):
        nc.apply_spatial_filter_2d(x, k, padding="FULL")


def test_product_path_refuses_cpu_tensors():
    """No CPU fallback: the public entry points refuse host tensors instead of computing."""
    topo = nc.ChipTopology2D.alu_chip()
    cell = torch.zeros(3, 62, 62)
    filt = torch.zeros(16, 1, 23, 13)
    p = nc.VNNParams(cell, filt)
    x = torch.zeros(2, 3, 8, 1)
    with pytest.raises(ValueError, match="no CPU path"):
        nc.propagate_vnn_2d(p, x, topo)
    with pytest.raises(ValueError, match="no CPU path"):
        nc.VonNeumannNetwork(topo).apply(p, x)
    with pytest.raises(ValueError, match="no CPU path"):
        nc.VNNTrainStep(topo, p, 2)
