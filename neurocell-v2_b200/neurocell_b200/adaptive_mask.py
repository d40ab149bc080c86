"""Epoch-adaptive spatial extent masks (mirror of ``neurocell/adaptive_mask.py``).

``compute_adaptive_spatial_mask`` estimates, once per epoch and on the host, the active
sub-ROI of a chip from its learned parameters, its I/O anchors and an optional activity
map, dilates it by a safety margin and quantises it to bucket multiples
(adaptive_mask.py:318-481).  ``propagate_vnn_2d(..., spatial_mask=spec)`` then runs the
B200 kernels on the sub-ROI only, with the reference's semantics (propagator.py:228-241,
343-371): cells of the full ROI outside the sub-ROI are dead (zero), the VALID border
template still feeds the sub-ROI where its window reaches the grid's dead ring.

The heuristics are host bookkeeping (a few hundred thousand float32 operations per epoch),
restated with numpy; the propagation itself runs in ``libneurocell_b200.so``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .topology import ChipTopology2D, CoordinatePortSpec, PortSpec

TILED_BLOCK_N = 1024      # tile size of the reference's tiled epilogue (kernels_pallas.py:58)


@dataclass(frozen=True)
class AdaptiveMaskSpec:
    """Active sub-ROI bounding box and masks for one epoch (adaptive_mask.py:38-58).

    ``roi_bbox`` = (r0, r1, c0, c1) in ROI coordinates; ``grid_bbox`` the same box in grid
    coordinates.  ``cropped_topology`` is the full topology (the B200 path runs the crop
    from ``roi_bbox``), ``fft_shape`` the reference's FFT size for the sub-ROI."""
    roi_bbox: tuple
    grid_bbox: tuple
    active_shape: tuple
    active_mask_roi: np.ndarray
    cropped_mask_roi: np.ndarray
    tile_mask: np.ndarray
    eff_kernel_radii: tuple
    active_fraction: float
    salient_cell_count: int
    is_full_roi: bool
    cropped_topology: ChipTopology2D
    fft_shape: tuple
    raw_roi_bbox: tuple | None = None


def _np(x) -> np.ndarray:
    if hasattr(x, "detach"):
        x = x.detach().cpu().numpy()
    return np.asarray(x)


def _next_pow2(n: int) -> int:
    p = 1
    while p < n:
        p <<= 1
    return p


def _select_tile_block_n(n_pix: int, max_block_n: int = TILED_BLOCK_N) -> int:
    """kernels_pallas.py:65-73."""
    for cand in (1024, 512, 256, 128):
        if cand <= max_block_n and n_pix % cand == 0:
            return cand
    return max_block_n


def estimate_effective_filter_radii(greens_filters, threshold: float = 0.05) -> tuple:
    """Half-radii of the taps with max_m |G| >= threshold * max |G| (adaptive_mask.py:61-85)."""
    G = _np(greens_filters).astype(np.float32)
    kh, kw = G.shape[-2], G.shape[-1]
    ch, cw = (kh - 1) // 2, (kw - 1) // 2
    per_tap = np.abs(G[:, 0]).max(axis=0)
    active = per_tap >= (np.float32(threshold) * per_tap.max() + np.float32(1e-12))
    rows = np.arange(kh)[:, None]
    cols = np.arange(kw)[None, :]
    r_h = max(1, int(np.where(active, np.abs(rows - ch), 0).max()))
    r_w = max(1, int(np.where(active, np.abs(cols - cw), 0).max()))
    return r_h, r_w


def _dilate_mask_2d(mask: np.ndarray, margin_h: int, margin_w: int) -> np.ndarray:
    """Rectangular dilation by half-radii (margin_h, margin_w) (adaptive_mask.py:88-106)."""
    if margin_h <= 0 and margin_w <= 0:
        return mask.copy()
    mh, mw = max(0, int(margin_h)), max(0, int(margin_w))
    m = mask.astype(bool)
    out = np.zeros_like(m)
    H, W = m.shape
    rows = np.zeros_like(m)
    for d in range(-mh, mh + 1):               # separable max: rows, then columns
        lo, hi = max(0, d), min(H, H + d)
        rows[lo - d:hi - d] |= m[lo:hi]
    for d in range(-mw, mw + 1):
        lo, hi = max(0, d), min(W, W + d)
        out[:, lo - d:hi - d] |= rows[:, lo:hi]
    return out


def _quantize_interval(lo: int, hi: int, max_len: int, bucket_multiple: int) -> tuple:
    """Grows [lo, hi) to a bucket-multiple length on a snapped start (adaptive_mask.py:109-161)."""
    lo = max(0, min(lo, max_len - 1))
    hi = max(lo + 1, min(hi, max_len))
    raw = hi - lo
    if bucket_multiple <= 1 or raw >= max_len:
        return 0, max_len
    q_len = min(max_len, ((raw + bucket_multiple - 1) // bucket_multiple) * bucket_multiple)
    if q_len >= max_len or (max_len - q_len) < bucket_multiple:
        return 0, max_len
    ideal = lo - 0.5 * (q_len - raw)
    lo_min = max(0, hi - q_len)
    lo_max = min(lo, max_len - q_len)

    def nearest(step):
        first = ((lo_min + step - 1) // step) * step
        if first > lo_max:
            return None
        cands = range(first, lo_max + 1, step)
        return min(cands, key=lambda v: (abs(v - ideal), v))

    best = nearest(max(1, bucket_multiple // 2))
    if best is None:
        best = nearest(max(1, bucket_multiple // 4))
    if best is None:
        best = max(lo_min, min(int(round(ideal)), lo_max))
    return int(best), int(best + q_len)


def _mask_tensors(cell, filters, io_roi, act_roi, r_h, r_w, roi_h, roi_w, margin_h, margin_w,
                  block_n, num_tiles, salience_threshold, bias_threshold, filter_threshold,
                  activity_threshold, has_activity):
    """Salience, dilation, bounding box and tile mask (adaptive_mask.py:200-315), float32."""
    f32 = np.float32
    r_eff = estimate_effective_filter_radii(filters, filter_threshold)
    w = cell[0, r_h:r_h + roi_h, r_w:r_w + roi_w]
    b = cell[1, r_h:r_h + roi_h, r_w:r_w + roi_w]
    s_raw = cell[2, r_h:r_h + roi_h, r_w:r_w + roi_w]
    s = (f32(1) / (f32(1) + np.exp(-s_raw))).astype(f32)
    non_io = ~io_roi
    non_io_n = max(f32(1), f32(non_io.sum()))
    # 1. bias-driven salience above the background drift floor
    drive = np.abs(b) * s
    upd = non_io & (np.abs(b) > f32(1e-5))
    upd_n = max(f32(1), f32(upd.sum()))
    mean = np.where(upd, drive, f32(0)).sum(dtype=f32) / upd_n
    std = np.sqrt(np.where(upd, (drive - mean) ** 2, f32(0)).sum(dtype=f32) / upd_n)
    z = (drive - mean) / (std + f32(1e-6))
    sal_bias = non_io & (s > 0.5) & (drive > bias_threshold) & ((z > salience_threshold) |
                                                                (drive > 4.0 * bias_threshold))
    # 2. differentiated high-gain relays
    wmag = np.abs(w) * s
    wmean = np.where(non_io, wmag, f32(0)).sum(dtype=f32) / non_io_n
    wstd = np.sqrt(np.where(non_io, (wmag - wmean) ** 2, f32(0)).sum(dtype=f32) / non_io_n)
    zw = (wmag - wmean) / (wstd + f32(1e-6))
    sal_relay = non_io & (np.abs(b) > 0.5 * bias_threshold) & (zw > salience_threshold) & (s > 0.85)
    seed = io_roi | sal_bias | sal_relay
    if has_activity:
        seed = seed | (act_roi > activity_threshold)
    dil = _dilate_mask_2d(seed, margin_h, margin_w)
    rows_on, cols_on = dil.any(axis=1), dil.any(axis=0)
    any_on = bool(rows_on.any())
    r0 = int(np.where(rows_on, np.arange(roi_h), roi_h).min())
    r1 = int(np.where(rows_on, np.arange(roi_h), -1).max()) + 1
    c0 = int(np.where(cols_on, np.arange(roi_w), roi_w).min())
    c1 = int(np.where(cols_on, np.arange(roi_w), -1).max()) + 1
    flat = dil.reshape(-1)
    if num_tiles * block_n > flat.size:
        flat = np.pad(flat, (0, num_tiles * block_n - flat.size))
    tiles = flat.reshape(num_tiles, block_n).any(axis=1)
    return r_eff, int(seed.sum()), any_on, (r0, r1, c0, c1), dil, tiles


def compute_adaptive_spatial_mask(params, topology: ChipTopology2D, margin=4, bucket_multiple: int = 8,
                                  salience_threshold: float = 2.5, bias_threshold: float = 0.05,
                                  filter_threshold: float = 0.05, activity_map=None,
                                  activity_threshold: float = 1e-3,
                                  prev_mask: AdaptiveMaskSpec | None = None) -> AdaptiveMaskSpec:
    """The pre-epoch active sub-ROI estimate (adaptive_mask.py:318-481)."""
    mh, mw = (int(margin), int(margin)) if isinstance(margin, int) else (int(margin[0]), int(margin[1]))
    H, W = topology.grid_shape
    r_h, r_w = topology.pad_h, topology.pad_w
    roi_h, roi_w = topology.roi_shape
    io_roi = np.asarray(topology.io_state_mask, bool)[r_h:H - r_h, r_w:W - r_w]
    n_pix = roi_h * roi_w
    block_n = _select_tile_block_n(n_pix, TILED_BLOCK_N)
    num_tiles = (n_pix + block_n - 1) // block_n
    cell = _np(params.cell_params).astype(np.float32)
    filt = _np(params.greens_filters).astype(np.float32)
    kh, kw = topology.kernel_size

    full_out = isinstance(topology.out_port, PortSpec) and tuple(topology.out_port.size) == (H, W)
    if full_out and activity_map is None:
        full = np.ones((roi_h, roi_w), bool)
        return AdaptiveMaskSpec((0, roi_h, 0, roi_w), (r_h, H - r_h, r_w, W - r_w), (roi_h, roi_w),
                                full, full, np.ones(num_tiles, bool),
                                estimate_effective_filter_radii(filt, filter_threshold), 1.0,
                                int(roi_h * roi_w), True, topology,
                                (_next_pow2(roi_h + kh - 1), _next_pow2(roi_w + kw - 1)))
    if activity_map is not None:
        act = _np(activity_map).astype(np.float32)
        act_roi = act[r_h:H - r_h, r_w:W - r_w] if act.shape == (H, W) else act
        has_act = True
    else:
        act_roi, has_act = io_roi.astype(np.float32), False
    r_eff, salient, any_on, raw, dil, tiles = _mask_tensors(
        cell, filt, io_roi, act_roi, r_h, r_w, roi_h, roi_w, mh, mw, block_n, num_tiles,
        salience_threshold, bias_threshold, filter_threshold, activity_threshold, has_act)
    r0, r1, c0, c1 = raw if any_on else (0, roi_h, 0, roi_w)
    if prev_mask is not None:
        pr = prev_mask.raw_roi_bbox if prev_mask.raw_roi_bbox is not None else prev_mask.roi_bbox
        r0, r1, c0, c1 = min(r0, pr[0]), max(r1, pr[1]), min(c0, pr[2]), max(c1, pr[3])
    raw_bbox = (r0, r1, c0, c1)
    # hysteresis: keep the previous quantised box when it still contains the raw box
    if prev_mask is not None and prev_mask.roi_bbox[0] <= r0 and r1 <= prev_mask.roi_bbox[1]:
        qr0, qr1 = prev_mask.roi_bbox[0], prev_mask.roi_bbox[1]
    else:
        qr0, qr1 = _quantize_interval(r0, r1, roi_h, bucket_multiple)
    if prev_mask is not None and prev_mask.roi_bbox[2] <= c0 and c1 <= prev_mask.roi_bbox[3]:
        qc0, qc1 = prev_mask.roi_bbox[2], prev_mask.roi_bbox[3]
    else:
        qc0, qc1 = _quantize_interval(c0, c1, roi_w, bucket_multiple)
    h_act, w_act = qr1 - qr0, qc1 - qc0
    return AdaptiveMaskSpec(
        roi_bbox=(qr0, qr1, qc0, qc1), grid_bbox=(r_h + qr0, r_h + qr1, r_w + qc0, r_w + qc1),
        active_shape=(h_act, w_act), active_mask_roi=dil, cropped_mask_roi=dil[qr0:qr1, qc0:qc1],
        tile_mask=tiles, eff_kernel_radii=r_eff,
        active_fraction=float(h_act * w_act) / float(roi_h * roi_w), salient_cell_count=salient,
        is_full_roi=(h_act == roi_h and w_act == roi_w), cropped_topology=topology,
        fft_shape=(_next_pow2(h_act + kh - 1), _next_pow2(w_act + kw - 1)), raw_roi_bbox=raw_bbox)
