"""Host-side pieces of the path (CPU): the chip presets' geometry, checkpoint and legacy
parameter round trips, and the packed 8-bit prediction formula.

Expected geometry values are worked out by hand from the reference's presets
(neurocell/topology.py:323-458) and its geometry rules (topology.py:152-284): VALID pads are
(k - 1) / 2 per side, the ROI is the grid minus the pads, fft_shape is the next power of two
of ROI + k - 1 per axis, and the I/O state mask covers every input and output cell.
"""
import os

import numpy as np
import pytest
import torch

import neurocell_b200 as nc
from oracle import vnn_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _rect(port):
    return tuple(port.offset), tuple(port.size)


def test_mlp_chip_geometry():
    # padding 2*17 = 34, N = 16 + 34 = 50, centre 25, gap 2*5+1 = 11;
    # input (25 - 25//2, 25 - 11//2) = (13, 20), size (3*8+1, 1); output (25 - 4, 20 + 11);
    # depth = output_left - input_left = 11
    t = nc.ChipTopology2D.mlp_chip()
    assert t.grid_shape == (50, 50) and t.kernel_size == (17, 3) and t.directions == 8
    assert t.depth == 11
    assert [_rect(p) for p in t.in_ports] == [((13, 20), (25, 1))]
    assert _rect(t.out_port) == ((21, 31), (8, 1))
    assert (t.pad_h, t.pad_w) == (8, 1) and t.roi_shape == (34, 48)
    assert t.fft_shape == (64, 64) and t.roi_out_offset == (13, 30)
    assert int(t.io_state_mask.sum()) == 33 and int(t.out_weight_mask.sum()) == 8
    assert t.in_in_roi and t.out_in_roi


def test_tm_chip_geometry():
    # length 16, padding 2*13 = 26, N = 16 + 52 = 68, centre 34; input (34, 26) size (1, 16);
    # output (34, 26 + 16 + 1) size (1, 8); depth = 43 - 26 = 17
    t = nc.ChipTopology2D.tm_chip()
    assert t.grid_shape == (68, 68) and t.kernel_size == (13, 13) and t.directions == 16
    assert t.depth == 17
    assert [_rect(p) for p in t.in_ports] == [((34, 26), (1, 16))]
    assert _rect(t.out_port) == ((34, 43), (1, 8))
    assert (t.pad_h, t.pad_w) == (6, 6) and t.roi_shape == (56, 56)
    assert t.fft_shape == (128, 128) and t.roi_out_offset == (28, 37)
    assert int(t.io_state_mask.sum()) == 24 and int(t.out_weight_mask.sum()) == 8


def test_clp_chip_geometry():
    # 8 x 8 VALID, K = 3 x 3: radius 1; inputs (2, 2), (5, 2); outputs (2, 5), (5, 5)
    t = nc.ChipTopology2D.clp_chip()
    assert t.grid_shape == (8, 8) and t.kernel_size == (3, 3) and t.directions == 1 and t.depth == 4
    assert tuple(map(tuple, t.in_ports[0].coords)) == ((2, 2), (5, 2))
    assert tuple(map(tuple, t.out_port.coords)) == ((2, 5), (5, 5))
    assert (t.pad_h, t.pad_w) == (1, 1) and t.roi_shape == (6, 6) and t.fft_shape == (8, 8)
    assert t.roi_out_offset == ((1, 4), (4, 4))
    assert int(t.io_state_mask.sum()) == 4 and int(t.out_weight_mask.sum()) == 2
    # SAME: radius 0, the default coordinates move to the grid's second row / column
    s = nc.ChipTopology2D.clp_chip(grid_shape=10, padding_mode="SAME")
    assert tuple(map(tuple, s.in_ports[0].coords)) == ((1, 1), (8, 1))
    assert tuple(map(tuple, s.out_port.coords)) == ((1, 8), (8, 8))
    assert s.roi_shape == (10, 10) and s.fft_shape == (16, 16)


def test_gol_chip_geometry():
    t = nc.ChipTopology2D.gol_chip()
    assert t.grid_shape == (64, 64) and t.directions == 64 and t.depth == 2
    assert _rect(t.out_port) == ((0, 0), (64, 64)) and not t.out_in_roi
    assert t.roi_shape == (62, 62) and t.fft_shape == (64, 64)


def test_checkpoint_save_load_round_trip(tmp_path):
    """save_checkpoint -> load_checkpoint gives back the same packed parameters, in the
    reference's npz layout (weights/biases/states (H, W), filters IHWO; model.py:197-227)."""
    topo = nc.ChipTopology2D.alu_chip()
    p = nc.init_vnn_params(3, topo, device="cpu")
    model = nc.VonNeumannNetwork(topo)
    f = str(tmp_path / "ckpt.npz")
    model.save_checkpoint(f, p)
    with np.load(f) as d:
        assert d["weights"].shape == (62, 62) and d["filters"].shape == (1, 23, 13, 16)
        assert np.array_equal(d["filters"], p.greens_filters.numpy().transpose(1, 2, 3, 0))
        assert int(d["N"]) == 62 and int(d["depth"]) == 4 and int(d["directions"]) == 16
    q = nc.VonNeumannNetwork.load_checkpoint(f, device="cpu")
    assert torch.equal(q.cell_params, p.cell_params)
    assert torch.equal(q.greens_filters, p.greens_filters)


def test_trained_checkpoint_reload_round_trip(tmp_path):
    p = nc.VonNeumannNetwork.load_checkpoint(os.path.join(GOLDEN, "alu_trained_cells.npz"), device="cpu")
    f = str(tmp_path / "again.npz")
    nc.VonNeumannNetwork(nc.ChipTopology2D.alu_chip()).save_checkpoint(f, p)
    q = nc.VonNeumannNetwork.load_checkpoint(f, device="cpu")
    assert torch.equal(q.cell_params, p.cell_params) and torch.equal(q.greens_filters, p.greens_filters)


def test_legacy_haiku_export_import_round_trip():
    """export_legacy_haiku_params -> import_legacy_haiku_params (params.py:325-346): the
    legacy leaves hold W, B, S as (H, W) planes and the filters as IHWO."""
    topo = nc.ChipTopology2D.alu_chip()
    p = nc.init_vnn_params(11, topo, device="cpu")
    hk = nc.params.export_legacy_haiku_params(p)
    sub = hk["universe_lp"]
    assert set(sub) == {"w", "b", "s", "f"} and tuple(sub["f"].shape) == (1, 23, 13, 16)
    assert torch.equal(sub["w"], p.cell_params[0]) and torch.equal(sub["s"], p.cell_params[2])
    q = nc.params.import_legacy_haiku_params(hk)
    assert torch.equal(q.cell_params, p.cell_params) and torch.equal(q.greens_filters, p.greens_filters)
    q2 = nc.params.import_legacy_haiku_params({"m": {k: v.numpy() for k, v in sub.items()}}, "m")
    assert torch.equal(q2.cell_params, p.cell_params)


# ---- packed 8-bit predictions (trainer.py:49-54, 122-138) --------------------------------
CRAFTED = np.array([
    [1.0, 0.0, 1.0, 0.0, 1.0, 0.0, 1.0, 0.0],      # 0b10101010 = 170
    [2.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 1.0],      # 2 * 128 wraps to 0, + 1 -> 1
    [-1.0, 1.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],     # -1 saturates to 0 -> 64
    [0.49, 0.51, 1.5, 2.5, 0.0, 0.0, 0.0, 0.0],    # half to even: 0, 1, 2, 2 -> 64 + 64 + 32
    [300.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 3.0],    # 255 * 128 = 32640 = 128 (mod 256); + 3
    [1.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0, 1.0],      # 255
], dtype=np.float32)
CRAFTED_BYTES = [170, 1, 64, 160, 131, 255]


def test_oracle_packed_predictions_follow_the_bit_weight_formula():
    got = O.packed_predictions(CRAFTED)[:, 0]
    assert got.tolist() == CRAFTED_BYTES
    assert O.packed_predictions(CRAFTED[:, :, None]).shape == (6, 1)
    assert O.packed_accuracy(CRAFTED, np.array(CRAFTED_BYTES, np.uint8)) == 1.0


def test_package_packing_matches_the_oracle_formula():
    """The package's packing of rounded logits (VNNTrainer.evaluate_packed) equals the
    oracle's restatement byte for byte, including values that are not bits."""
    t = torch.tensor(CRAFTED)
    u8 = torch.round(t).clamp(0, 255).to(torch.uint8)
    got = nc.packbits_u8_on_device(u8)[:, 0].tolist()
    assert got == CRAFTED_BYTES
    rng = np.random.default_rng(5)
    r = rng.uniform(-2, 4, (500, 8)).astype(np.float32)
    mine = nc.packbits_u8_on_device(torch.round(torch.tensor(r)).clamp(0, 255).to(torch.uint8))
    assert np.array_equal(mine.numpy(), O.packed_predictions(r))
