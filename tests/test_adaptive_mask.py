"""Adaptive sub-ROI mask heuristics on the host (neurocell/adaptive_mask.py), checked
against the geometric claims of the reference's tests/unit_milestone7_adaptive_mask.py.
The reference seeds its parameters with jax.random, which is not available here, so the
parameters come from this package's seeded init_vnn_params; every claim below depends on
the I/O anchors and on cells set explicitly, not on the random draw."""
import numpy as np
import pytest
import torch

import neurocell_b200 as nc


def _alu():
    return nc.ChipTopology2D.alu_chip(n=8, kernel_size=(23, 13), directions=16, depth=4, gap=5,
                                      ctrl_gap=5)


def test_alu_mask_geometry_and_frontier_growth():
    """unit_milestone7_adaptive_mask.py:52-90: a (32, 32) box of the 40x50 ROI at init, and
    the box grows to cover a cell that becomes salient beyond the margin."""
    topo = _alu()
    p0 = nc.init_vnn_params(701, topo, legacy_compat=True, device="cpu")
    m0 = nc.compute_adaptive_spatial_mask(p0, topo, margin=4, bucket_multiple=8)
    assert isinstance(m0, nc.AdaptiveMaskSpec)
    assert not m0.is_full_roi
    assert m0.active_shape == (32, 32)
    assert abs(m0.active_fraction - 1024.0 / 2000.0) < 1e-6
    r0, r1, c0, c1 = m0.roi_bbox
    assert (r1 - r0, c1 - c0) == (32, 32)
    assert m0.grid_bbox == (r0 + topo.pad_h, r1 + topo.pad_h, c0 + topo.pad_w, c1 + topo.pad_w)
    # the I/O anchors lie inside the box
    for port in tuple(topo.in_ports) + (topo.out_port,):
        pr, pc = port.offset
        assert r0 <= pr - topo.pad_h < r1 and c0 <= pc - topo.pad_w < c1

    rh, rw = topo.pad_h, topo.pad_w
    cp = p0.cell_params.clone()
    cp[1, rh + 35, rw + 44] = 0.8
    cp[2, rh + 35, rw + 44] = 2.0
    m1 = nc.compute_adaptive_spatial_mask(nc.VNNParams(cp, p0.greens_filters), topo, margin=4,
                                          bucket_multiple=8)
    assert m1.roi_bbox[1] >= 39 and m1.roi_bbox[3] >= 48
    assert m1.active_shape[0] > m0.active_shape[0] and m1.active_shape[1] > m0.active_shape[1]


def test_alu_mask_ignores_biases_below_threshold():
    """unit_milestone7_adaptive_mask.py:98-109: N(0, 0.02) biases stay below bias_threshold."""
    topo = _alu()
    p0 = nc.init_vnn_params(702, topo, legacy_compat=True, device="cpu")
    cp = p0.cell_params.clone()
    cp[1] = torch.from_numpy(np.random.default_rng(703).normal(size=topo.grid_shape) * 0.02).float()
    m = nc.compute_adaptive_spatial_mask(nc.VNNParams(cp, p0.greens_filters), topo, margin=4,
                                         bucket_multiple=8, bias_threshold=0.5)
    assert m.active_shape == (32, 32)


def test_full_grid_gol_and_large_grid_masks():
    """unit_milestone7_adaptive_mask.py:152-184: a full-grid Game of Life keeps its whole
    ROI; an 82x82 chip with local ports crops to at most 32x32 (< 20 % of the ROI); K=3
    filters have radius (1, 1)."""
    tg = nc.ChipTopology2D.gol_chip(n=64, kernel_size=(3, 3), directions=16, depth=4)
    mg = nc.compute_adaptive_spatial_mask(nc.init_vnn_params(705, tg, device="cpu"), tg, margin=4)
    assert mg.is_full_roi and mg.active_shape == tg.roi_shape

    tl = nc.ChipTopology2D.create(grid_shape=(82, 82), kernel_size=(3, 3), directions=16, depth=6,
                                  in_ports=(nc.PortSpec(offset=(20, 20), size=(8, 1), name="in"),),
                                  out_port=nc.PortSpec(offset=(24, 32), size=(8, 1), name="out"))
    pl = nc.init_vnn_params(706, tl, device="cpu")
    ml = nc.compute_adaptive_spatial_mask(pl, tl, margin=4, bucket_multiple=8)
    assert not ml.is_full_roi
    assert ml.active_shape[0] <= 32 and ml.active_shape[1] <= 32
    assert ml.active_fraction < 0.20
    assert nc.estimate_effective_filter_radii(pl.greens_filters) == (1, 1)


def test_mask_buckets_are_multiples_of_bucket_multiple():
    topo = _alu()
    p0 = nc.init_vnn_params(707, topo, legacy_compat=True, device="cpu")
    for margin in (0, 2, 4, 6):
        m = nc.compute_adaptive_spatial_mask(p0, topo, margin=margin, bucket_multiple=8)
        h, w = m.active_shape
        assert m.is_full_roi or (h % 8 == 0 or h == topo.roi_shape[0]) and (w % 8 == 0 or w == topo.roi_shape[1])
        r0, r1, c0, c1 = m.roi_bbox
        assert 0 <= r0 < r1 <= topo.roi_shape[0] and 0 <= c0 < c1 <= topo.roi_shape[1]


def test_exact_match_metric_and_packbits():
    logits = torch.tensor([[[0.2], [0.9], [1.4]], [[-0.3], [0.51], [0.49]]])
    targets = torch.tensor([[0.0, 1.0, 1.0], [0.0, 1.0, 1.0]])
    assert abs(float(nc.default_exact_match_metric(logits, targets)) - 5.0 / 6.0) < 1e-7
    bits = torch.tensor([[1, 0, 1, 1, 0, 0, 0, 1]], dtype=torch.uint8)
    assert int(nc.packbits_u8_on_device(bits)[0, 0]) == int(np.packbits(bits.numpy(), axis=1)[0, 0])
