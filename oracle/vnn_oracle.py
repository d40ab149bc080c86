"""CPU oracle for the Neurocell v2 VNN propagation hot path -- TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.  The
product path (``neurocell_b200``) never imports it and fails loudly when its CUDA library
is missing.

What it restates (paths are relative to the shakes76/neurocell-v2 project root):

* geometry       -- ``neurocell/topology.py:152-284`` (``ChipTopology2D.create``),
                    ``:286-321`` (``alu_chip``), ``:19-83`` (port specs)
* Codd gating    -- ``neurocell/params.py:31-80`` (``compute_codd_state_probs``)
* pre-step fusion-- ``neurocell/params.py:220-322`` (``precompute_step_params``)
* injection      -- ``neurocell/propagator.py:88-191`` (incl. the 3-D input-shape quirk)
* d-step loop    -- ``neurocell/propagator.py:343-432`` (``backend="nchw_direct"``, the
                    semantic backend the reference's own parity tests compare against),
                    ``:657-682`` (output-port fast path), ``:284-341`` (CIRCULAR)
* convolution    -- ``neurocell/kernels_greens.py:177-217`` (cross-correlation, OIHW)
* epilogues      -- ``neurocell/epilogue.py:20-128``; centred variance with eps=1e-5 as in
                    ``neurocell/kernels_pallas.py:202-205``
* activations    -- ``neurocell/kernels_pallas.py:111-156``
* losses         -- ``neurocell/trainer.py:57-61`` (MSE); softmax cross-entropy with
                    integer labels as used by the reference's classification drivers
* ALU truth table-- ``neurocell/datasets.py:77-130``

The backward pass is written out by hand (reverse of the forward above); the tests check
it against central finite differences and against an independent torch float64 autograd
restatement.  Everything is numpy; the default dtype is float64.

Parity pinning: the reference (JAX/Pallas) cannot be imported or run in this environment
(no jax/jaxlib wheel, no network).  This oracle is pinned by (1) the exact geometry
constants of the reference's ``tests/unit_topology.py:29-81``, (2) the Codd-mode KATs of
``tests/unit_milestone8_pallas_and_codd.py:227-252``, and (3) a functional known-answer
test: the reference's trained ALU checkpoint (``alu_arithmetic_cells.npz``, exported to
``tests/golden/``) must reach the >= 98 % packed accuracy the reference reports for it when
run through this forward pass.  Numerical outputs are otherwise pinned only relatively.
"""
from __future__ import annotations

from dataclasses import dataclass, field
import math
from typing import Sequence

import numpy as np

STATE_ACTIVE_VALUE = 1.0
NORM_EPS = 1e-5
CODD_MODES = ("continuous", "annealed", "ste_binary", "ste_ternary")
ACTIVATIONS = ("identity", "tanh", "sigmoid", "relu", "leaky_relu", "gelu")


# ----------------------------------------------------------------------------------------
# Geometry (topology.py:19-321)
# ----------------------------------------------------------------------------------------
@dataclass(frozen=True)
class RectPort:
    """Rectangular port: ``PortSpec`` (topology.py:19-34)."""
    offset: tuple
    size: tuple
    name: str = ""


@dataclass(frozen=True)
class CoordPort:
    """Scattered port: ``CoordinatePortSpec`` (topology.py:37-83)."""
    coords: tuple
    name: str = ""

    @property
    def size(self):
        return (len(self.coords), 1)

    @property
    def offset(self):
        return (min(r for r, _ in self.coords), min(c for _, c in self.coords))


def _within(port, r0, r1, c0, c1) -> bool:
    """topology.py:95-106."""
    if isinstance(port, CoordPort):
        return all(r0 <= r < r1 and c0 <= c < c1 for r, c in port.coords)
    (pr, pc), (ph, pw) = port.offset, port.size
    return pr >= r0 and pc >= c0 and pr + ph <= r1 and pc + pw <= c1


def _next_pow2(x: int) -> int:
    return 1 << (x - 1).bit_length()


@dataclass
class Geometry:
    grid_shape: tuple
    kernel_size: tuple
    directions: int
    depth: int
    in_ports: tuple
    out_port: object
    padding_mode: str
    pad_h: int
    pad_w: int
    roi_shape: tuple
    roi_out_offset: tuple
    io_state_mask: np.ndarray
    out_weight_mask: np.ndarray
    fft_shape: tuple
    in_in_roi: bool
    out_in_roi: bool
    extra: dict = field(default_factory=dict)


def make_geometry(grid_shape, kernel_size, directions, depth, in_ports, out_port,
                  padding_mode="VALID", allow_border_output=False) -> Geometry:
    """Restates ``ChipTopology2D.create`` (topology.py:152-284)."""
    if isinstance(grid_shape, int):
        grid_shape = (grid_shape, grid_shape)
    H, W = int(grid_shape[0]), int(grid_shape[1])
    kh, kw = int(kernel_size[0]), int(kernel_size[1])
    if kh % 2 == 0 or kw % 2 == 0:
        raise ValueError("kernel_size must be odd")
    mode = padding_mode.upper()
    if mode not in ("VALID", "SAME", "CIRCULAR"):
        raise ValueError(mode)
    pad_h, pad_w = ((kh - 1) // 2, (kw - 1) // 2) if mode == "VALID" else (0, 0)
    roi_h, roi_w = H - 2 * pad_h, W - 2 * pad_w
    if roi_h <= 0 or roi_w <= 0:
        raise ValueError("grid too small for kernel")
    in_ports = tuple(in_ports)
    for p in in_ports + (out_port,):
        if not _within(p, 0, H, 0, W):
            raise ValueError("port exceeds grid")
    in_in_roi = all(_within(p, pad_h, H - pad_h, pad_w, W - pad_w) for p in in_ports)
    out_in_roi = _within(out_port, pad_h, H - pad_h, pad_w, W - pad_w)
    full_out = isinstance(out_port, RectPort) and tuple(out_port.offset) == (0, 0) \
        and tuple(out_port.size) == (H, W)
    if mode == "VALID" and not out_in_roi and not allow_border_output and not full_out:
        raise ValueError("output port outside VALID ROI")
    if isinstance(out_port, CoordPort):
        roi_out_offset = (tuple(r - pad_h for r, _ in out_port.coords),
                          tuple(c - pad_w for _, c in out_port.coords))
    else:
        roi_out_offset = (max(0, out_port.offset[0] - pad_h), max(0, out_port.offset[1] - pad_w))
    io = np.zeros((H, W), dtype=bool)
    for p in in_ports:
        if isinstance(p, CoordPort):
            for r, c in p.coords:
                io[r, c] = True
        else:
            io[p.offset[0]:p.offset[0] + p.size[0], p.offset[1]:p.offset[1] + p.size[1]] = True
    ow = np.zeros((H, W), dtype=bool)
    if isinstance(out_port, CoordPort):
        for r, c in out_port.coords:
            io[r, c] = True
            ow[r, c] = True
    else:
        sl = (slice(out_port.offset[0], out_port.offset[0] + out_port.size[0]),
              slice(out_port.offset[1], out_port.offset[1] + out_port.size[1]))
        io[sl] = True
        ow[sl] = True
    fft = (H, W) if mode == "CIRCULAR" else (_next_pow2(roi_h + kh - 1), _next_pow2(roi_w + kw - 1))
    return Geometry((H, W), (kh, kw), int(directions), int(depth), in_ports, out_port, mode,
                    pad_h, pad_w, (roi_h, roi_w), roi_out_offset, io, ow, fft, in_in_roi, out_in_roi)


def alu_geometry(n=8, kernel_size=(23, 13), directions=16, depth=4, gap=5, ctrl_gap=5) -> Geometry:
    """Restates ``ChipTopology2D.alu_chip`` (topology.py:286-321)."""
    padding = 2 * max(kernel_size)
    N = 2 * n + padding
    center = N // 2
    top = center - (2 * n) // 2
    left = center - n
    out_mid = center - n // 2
    out_left = left + n + 2 * gap
    ins = (RectPort((top, left), (n, 1), "x1"),
           RectPort((top + n + 1, left), (n, 1), "x2"),
           RectPort((top - ctrl_gap, left + gap), (1, n), "ctrl"))
    return make_geometry((N, N), kernel_size, directions, depth, ins,
                         RectPort((out_mid, out_left), (n, 1), "out"))


# ----------------------------------------------------------------------------------------
# Activations (kernels_pallas.py:111-156)
# ----------------------------------------------------------------------------------------
_GELU_C = math.sqrt(2.0 / math.pi)


_PAR_MIN = 1 << 22          # elementwise work above this size is split over threads


def _chunked(fn, x):
    """fn applied elementwise to ``x`` in chunks on a thread pool (numpy ufuncs release the
    GIL); the values are exactly fn(x)."""
    x = np.asarray(x)
    if x.size < _PAR_MIN:
        return fn(x)
    import concurrent.futures as cf
    import os
    flat = np.ascontiguousarray(x).reshape(-1)
    out = np.empty_like(flat)
    n = os.cpu_count() or 1
    step = -(-flat.size // (4 * n))

    def work(a):
        out[a:a + step] = fn(flat[a:a + step])

    with cf.ThreadPoolExecutor(max_workers=n) as ex:
        list(ex.map(work, range(0, flat.size, step)))
    return out.reshape(x.shape)


def act_fwd(x, name, slope=0.01):
    if name in (None, "identity"):
        return x
    if np.size(x) >= _PAR_MIN:
        return _chunked(lambda v: act_fwd(v, name, slope), x)
    if name == "tanh":
        return np.tanh(x)
    if name == "sigmoid":
        return 1.0 / (1.0 + np.exp(-x))
    if name == "relu":
        return np.maximum(x, 0.0)
    if name == "leaky_relu":
        return np.where(x >= 0.0, x, slope * x)
    if name == "gelu":
        return 0.5 * x * (1.0 + np.tanh(_GELU_C * (x + 0.044715 * x ** 3)))
    raise ValueError(name)


def act_deriv(x, name, slope=0.01):
    if name in (None, "identity"):
        return np.ones_like(x)
    if np.size(x) >= _PAR_MIN:
        return _chunked(lambda v: act_deriv(v, name, slope), x)
    if name == "tanh":
        y = np.tanh(x)
        return 1.0 - y * y
    if name == "sigmoid":
        y = 1.0 / (1.0 + np.exp(-x))
        return y * (1.0 - y)
    if name == "relu":
        return (x > 0.0).astype(x.dtype)
    if name == "leaky_relu":
        return np.where(x >= 0.0, 1.0, slope).astype(x.dtype)
    if name == "gelu":
        x2 = x * x
        th = np.tanh(_GELU_C * (x + 0.044715 * x2 * x))
        du = _GELU_C * (1.0 + 3.0 * 0.044715 * x2)
        return 0.5 * (1.0 + th) + 0.5 * x * (1.0 - th * th) * du
    raise ValueError(name)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


# ----------------------------------------------------------------------------------------
# Codd gating (params.py:31-80)
# ----------------------------------------------------------------------------------------
def codd_state_probs(s_raw, io_mask, hard_pin_io=False, codd_mode="continuous",
                     state_temperature=1.0, active_threshold=0.6):
    """Returns ``(s_prob, ds_prob/ds_raw)``; the derivative is the STE surrogate's."""
    if codd_mode not in CODD_MODES:
        raise ValueError(codd_mode)
    dt = s_raw.dtype
    s_base = s_raw if hard_pin_io else np.where(io_mask, STATE_ACTIVE_VALUE, s_raw).astype(dt)
    dbase = np.ones_like(s_raw) if hard_pin_io else (~io_mask).astype(dt)
    if codd_mode == "continuous":
        s = _sigmoid(s_base)
        ds = s * (1.0 - s) * dbase
    else:
        # the reference computes in float32: threshold and clamp are float32 constants
        tau = max(float(np.float32(state_temperature)), float(np.float32(1e-4)))
        inv_tau = 1.0 / tau
        soft = _sigmoid(s_base * inv_tau)
        ds = soft * (1.0 - soft) * inv_tau * dbase
        if codd_mode == "annealed":
            s = soft
        elif codd_mode == "ste_binary":
            hard = np.where(s_base >= 0.0, 1.0, 0.0).astype(dt)
            s = soft + (hard - soft)
        else:
            thr = float(np.float32(active_threshold))
            hard = np.where(s_base >= thr, 1.0, np.where(s_base > 0.0, 0.5, 0.0)).astype(dt)
            s = soft + (hard - soft)
    if hard_pin_io:
        s = np.where(io_mask, STATE_ACTIVE_VALUE, s).astype(dt)
        ds = np.where(io_mask, 0.0, ds).astype(dt)
    return s.astype(dt), ds.astype(dt)


def threshold_states(states_raw, active_threshold=0.6):
    """Discrete roles {0,1,2} (model.py:185-195)."""
    thr = np.float32(active_threshold)
    s = np.where(states_raw >= thr, 2.0, states_raw)
    return np.where((s > 0.0) & (s < thr), 1.0, s)


# ----------------------------------------------------------------------------------------
# Injection (propagator.py:88-191)
# ----------------------------------------------------------------------------------------
def normalize_port_inputs(inputs, geom: Geometry):
    """propagator.py:88-100."""
    if isinstance(inputs, (list, tuple)):
        return inputs[0].shape[0], list(inputs)
    B = inputs.shape[0]
    if len(geom.in_ports) == 1:
        p0 = geom.in_ports[0]
        if inputs.ndim == 2 or (inputs.ndim == 3 and tuple(inputs.shape[1:]) == tuple(p0.size)):
            return B, [inputs]
    return B, [inputs[:, i] for i in range(len(geom.in_ports))]


def inject_full(inputs, geom: Geometry, dtype=np.float64):
    """Full-grid injection (propagator.py:103-132)."""
    H, W = geom.grid_shape
    B, arrs = normalize_port_inputs(inputs, geom)
    cells = np.zeros((B, H, W), dtype=dtype)
    for inp, port in zip(arrs, geom.in_ports):
        inp = np.asarray(inp)
        if isinstance(port, CoordPort):
            flat = inp.reshape(B, len(port.coords)).astype(dtype)
            for j, (r, c) in enumerate(port.coords):
                cells[:, r, c] = flat[:, j]
        else:
            r0, c0 = port.offset
            if inp.ndim == 3:
                ih, iw = inp.shape[1], inp.shape[2]
                cells[:, r0:r0 + ih, c0:c0 + iw] = inp
            else:
                ph, pw = port.size
                cells[:, r0:r0 + ph, c0:c0 + pw] = inp.reshape(B, ph, pw)
    return cells


def inject_roi(inputs, geom: Geometry, dtype=np.float64):
    """ROI injection (propagator.py:135-191); returns ``(roi_cells, fits)``."""
    if not geom.in_in_roi:
        return None, False
    r_h, r_w = (geom.pad_h, geom.pad_w) if geom.padding_mode == "VALID" else (0, 0)
    roi_h, roi_w = geom.roi_shape
    B, arrs = normalize_port_inputs(inputs, geom)
    for inp, port in zip(arrs, geom.in_ports):
        if isinstance(port, CoordPort):
            continue  # coordinates already checked by in_in_roi
        r0, c0 = port.offset
        ih, iw = (inp.shape[1], inp.shape[2]) if np.ndim(inp) == 3 else port.size
        if r0 < r_h or c0 < r_w or r0 + ih > r_h + roi_h or c0 + iw > r_w + roi_w:
            return None, False
    full = inject_full(inputs, geom, dtype)
    H, W = geom.grid_shape
    return full[:, r_h:H - r_h, r_w:W - r_w].copy(), True


# ----------------------------------------------------------------------------------------
# Convolution (kernels_greens.py:177-217): cross-correlation, 1 in-channel -> M out
# ----------------------------------------------------------------------------------------
CONV_METHOD = "fft"   # "fft" (fast, float64-exact to ~1e-15) or "direct" (im2col)


def _fft_size(n):
    s = 8
    while s < n:
        s *= 2
    return s


try:                      # threaded transforms when scipy is present (same float64 results)
    import os as _os
    import scipy.fft as _sfft
    _WORKERS = _os.cpu_count() or 1

    def _rfft2(x, s):
        return _sfft.rfft2(x, s=s, workers=_WORKERS)

    def _irfft2(x, s):
        return _sfft.irfft2(x, s=s, workers=_WORKERS)
except ImportError:       # pragma: no cover
    def _rfft2(x, s):
        return np.fft.rfft2(x, s=s)

    def _irfft2(x, s):
        return np.fft.irfft2(x, s=s)


def conv_valid(x, G, chunk=16, method=None):
    """VALID cross-correlation: ``x`` (B, h+kh-1, w+kw-1), ``G`` (M, kh, kw) -> (B, M, h, w)."""
    if (method or CONV_METHOD) == "fft":
        return _conv_valid_fft(x, G)
    return _conv_valid_direct(x, G, chunk)


def conv_valid_bwd(x, G, gz, need_dx=True, chunk=16, method=None):
    """Adjoint of :func:`conv_valid`: returns ``(dx (B,Hp,Wp) or None, dG (M,kh,kw))``."""
    if (method or CONV_METHOD) == "fft":
        return _conv_valid_bwd_fft(x, G, gz, need_dx)
    return _conv_valid_bwd_direct(x, G, gz, need_dx, chunk)


def _conv_valid_fft(x, G):
    # correlation theorem: z[i] = sum_u G[u] x[i+u]  ->  Z = irfft(X * conj(Ghat))
    B, Hp, Wp = x.shape
    M, kh, kw = G.shape
    h, w = Hp - kh + 1, Wp - kw + 1
    N1, N2 = _fft_size(Hp), _fft_size(Wp)
    X = _rfft2(x, (N1, N2))
    Gh = np.conj(_rfft2(G, (N1, N2)))
    out = np.empty((B, M, h, w), dtype=np.result_type(x, G))
    for m in range(M):
        out[:, m] = _irfft2(X * Gh[m][None], (N1, N2))[:, :h, :w]
    return out


def _conv_valid_bwd_fft(x, G, gz, need_dx):
    B, Hp, Wp = x.shape
    M, kh, kw = G.shape
    N1, N2 = _fft_size(Hp), _fft_size(Wp)
    X = _rfft2(x, (N1, N2))
    GZ = _rfft2(gz, (N1, N2))                        # (B, M, N1, N2//2+1)
    # dG[u] = sum_i gz[i] x[i+u]  ->  irfft(sum_b X * conj(GZ))
    acc = np.einsum("bij,bmij->mij", X, np.conj(GZ))
    dG = _irfft2(acc, (N1, N2))[:, :kh, :kw].astype(np.result_type(x, G))
    dx = None
    if need_dx:
        # dx[j] = sum_u G[u] gz[j-u]  ->  irfft(sum_m GZ * Ghat)
        Gh = _rfft2(G, (N1, N2))
        dx = _irfft2(np.einsum("bmij,mij->bij", GZ, Gh), (N1, N2))[:, :Hp, :Wp]
        dx = dx.astype(x.dtype)
    return dx, dG


def _conv_valid_direct(x, G, chunk=16):
    B, Hp, Wp = x.shape
    M, kh, kw = G.shape
    h, w = Hp - kh + 1, Wp - kw + 1
    Gm = G.reshape(M, kh * kw).T
    out = np.empty((B, M, h, w), dtype=np.result_type(x, G))
    for b0 in range(0, B, chunk):
        xs = x[b0:b0 + chunk]
        cols = np.lib.stride_tricks.sliding_window_view(xs, (kh, kw), axis=(1, 2))
        cols = cols.reshape(xs.shape[0] * h * w, kh * kw)
        out[b0:b0 + chunk] = (cols @ Gm).reshape(xs.shape[0], h, w, M).transpose(0, 3, 1, 2)
    return out


def _conv_valid_bwd_direct(x, G, gz, need_dx=True, chunk=16):
    B, Hp, Wp = x.shape
    M, kh, kw = G.shape
    h, w = Hp - kh + 1, Wp - kw + 1
    dG = np.zeros((M, kh * kw), dtype=np.result_type(x, G))
    dx = np.zeros_like(x) if need_dx else None
    Gm = G.reshape(M, kh * kw)
    for b0 in range(0, B, chunk):
        xs = x[b0:b0 + chunk]
        nb = xs.shape[0]
        cols = np.lib.stride_tricks.sliding_window_view(xs, (kh, kw), axis=(1, 2))
        cols = cols.reshape(nb * h * w, kh * kw)
        g2 = gz[b0:b0 + chunk].transpose(0, 2, 3, 1).reshape(nb * h * w, M)
        dG += g2.T @ cols
        if need_dx:
            gcol = (g2 @ Gm).reshape(nb, h, w, kh, kw)
            for u in range(kh):
                for v in range(kw):
                    dx[b0:b0 + chunk, u:u + h, v:v + w] += gcol[:, :, :, u, v]
    return dx, dG.reshape(M, kh, kw)


def _pad_same(x, kh, kw):
    ph, pw = (kh - 1) // 2, (kw - 1) // 2
    return np.pad(x, ((0, 0), (ph, ph), (pw, pw)))


def _pad_wrap(x, kh, kw):
    ph, pw = (kh - 1) // 2, (kw - 1) // 2
    return np.pad(x, ((0, 0), (ph, ph), (pw, pw)), mode="wrap")


def _unpad_same(dx, kh, kw):
    ph, pw = (kh - 1) // 2, (kw - 1) // 2
    return dx[:, ph:dx.shape[1] - ph, pw:dx.shape[2] - pw]


def _unpad_wrap(dx, kh, kw, h, w):
    """Adjoint of ``np.pad(mode='wrap')``: fold the halo back onto the plane."""
    ph, pw = (kh - 1) // 2, (kw - 1) // 2
    out = np.zeros((dx.shape[0], h, w), dtype=dx.dtype)
    rows = (np.arange(h + 2 * ph) - ph) % h
    cols = (np.arange(w + 2 * pw) - pw) % w
    for i, r in enumerate(rows):
        for j, c in enumerate(cols):
            out[:, r, c] += dx[:, i, j]
    return out


# ----------------------------------------------------------------------------------------
# Pre-step fusion (params.py:220-322)
# ----------------------------------------------------------------------------------------
def _roi(geom):
    H, W = geom.grid_shape
    return (slice(geom.pad_h, H - geom.pad_h), slice(geom.pad_w, W - geom.pad_w))


def _out_index(geom):
    """Output-port pixel positions as (rows, cols) arrays in ROI coordinates."""
    op = geom.out_port
    if isinstance(op, CoordPort):
        return np.array(geom.roi_out_offset[0]), np.array(geom.roi_out_offset[1])
    ro_r, ro_c = geom.roi_out_offset
    oh, ow = op.size
    rr, cc = np.meshgrid(np.arange(ro_r, ro_r + oh), np.arange(ro_c, ro_c + ow), indexing="ij")
    return rr.ravel(), cc.ravel()


def _out_grid_index(geom):
    """Output-port cells as (rows, cols) arrays in grid coordinates (any position)."""
    op = geom.out_port
    if isinstance(op, CoordPort):
        return np.array([r for r, _ in op.coords]), np.array([c for _, c in op.coords])
    (r0, c0), (oh, ow) = op.offset, op.size
    rr, cc = np.meshgrid(np.arange(r0, r0 + oh), np.arange(c0, c0 + ow), indexing="ij")
    return rr.ravel(), cc.ravel()


def precompute(cell_params, geom, activate="tanh", act_slope=0.01, hard_pin_io=False,
               codd_mode="continuous", state_temperature=1.0, active_threshold=0.6):
    Wf, Bf, Sf = cell_params[0], cell_params[1], cell_params[2]
    M = geom.directions
    inv_M = 1.0 / float(M)
    w_pinned = np.where(geom.out_weight_mask, 1.0, Wf).astype(Wf.dtype)
    s_prob, ds = codd_state_probs(Sf, geom.io_state_mask, hard_pin_io, codd_mode,
                                  state_temperature, active_threshold)
    roi = _roi(geom)
    w_roi, b_roi, s_roi = w_pinned[roi], Bf[roi], s_prob[roi]
    sp = dict(
        w_pinned=w_pinned, s_prob=s_prob, ds_prob=ds,
        w_eff_roi=inv_M * w_roi * (1.0 - s_roi), s_eff_roi=inv_M * s_roi, b_roi=b_roi,
        border_2d=act_fwd(Bf, activate, act_slope) * s_prob,
    )
    if geom.out_in_roi:
        rr, cc = _out_index(geom)
        sp["w_eff_out"] = sp["w_eff_roi"][rr, cc]
        sp["s_eff_out"] = sp["s_eff_roi"][rr, cc]
        sp["b_out"] = b_roi[rr, cc]
    return sp


# ----------------------------------------------------------------------------------------
# Epilogues (epilogue.py:20-128)
# ----------------------------------------------------------------------------------------
def _by_planes(fn, *arrays):
    """fn over chunks of the (B, M) planes of same-shaped (B, M, h, w) arrays on a thread
    pool; returns the tuple of fn's outputs reassembled (each (B, M, ...))."""
    import concurrent.futures as cf
    import os
    B, M = arrays[0].shape[:2]
    flat = [np.ascontiguousarray(a).reshape((B * M,) + a.shape[2:]) for a in arrays]
    n = os.cpu_count() or 1
    step = max(1, -(-(B * M) // (2 * n)))
    parts = [None] * len(range(0, B * M, step))

    def work(i):
        a = i * step
        parts[i] = fn(*(f[a:a + step] for f in flat))

    with cf.ThreadPoolExecutor(max_workers=n) as ex:
        list(ex.map(work, range(len(parts))))
    return tuple(np.concatenate([p[k] for p in parts]).reshape((B, M) + parts[0][k].shape[1:])
                 for k in range(len(parts[0])))


def _standardize(z, norm=True):
    if not norm:
        return z, None
    if z.ndim == 4 and z.size >= _PAR_MIN:
        return _by_planes(lambda v: _standardize(v, True), z)
    mean = z.mean(axis=(-2, -1), keepdims=True)
    var = ((z - mean) ** 2).mean(axis=(-2, -1), keepdims=True)
    rstd = 1.0 / np.sqrt(var + NORM_EPS)
    return (z - mean) * rstd, rstd


def _standardize_bwd(gzh, zh, rstd, norm=True):
    if not norm:
        return gzh
    if zh.ndim == 4 and zh.size >= _PAR_MIN:
        g = np.broadcast_to(gzh, zh.shape)
        r = np.broadcast_to(rstd, zh.shape[:2] + (1, 1))
        return _by_planes(lambda a, b, c: (_standardize_bwd(a, b, c, True),), g, zh, r)[0]
    c1 = gzh.mean(axis=(-2, -1), keepdims=True)
    c2 = (gzh * zh).mean(axis=(-2, -1), keepdims=True)
    return rstd * (gzh - c1 - zh * c2)


def hidden_epilogue(z, sp, activate, act_slope, norm):
    """epilogue.py:28-56."""
    zh, rstd = _standardize(z, norm)
    M = z.shape[1]
    lin = zh.sum(axis=1)
    if activate in (None, "identity"):
        act = lin + float(M) * sp["b_roi"][None]
    else:
        act = act_fwd(zh + sp["b_roi"][None, None], activate, act_slope).sum(axis=1)
    out = sp["w_eff_roi"][None] * lin + sp["s_eff_roi"][None] * act
    return out, dict(zh=zh, rstd=rstd, lin=lin, act=act)


def hidden_epilogue_bwd(gy, tape, sp, activate, act_slope, norm, grads):
    zh = tape["zh"]
    M = zh.shape[1]
    grads["w_eff_roi"] += (gy * tape["lin"]).sum(axis=0)
    grads["s_eff_roi"] += (gy * tape["act"]).sum(axis=0)
    s_gy = sp["s_eff_roi"][None] * gy
    if activate in (None, "identity"):
        dact = np.broadcast_to(s_gy[:, None], zh.shape)
    else:
        dact = s_gy[:, None] * act_deriv(zh + sp["b_roi"][None, None], activate, act_slope)
    grads["b_roi"] += dact.sum(axis=(0, 1))
    gzh = (sp["w_eff_roi"][None] * gy)[:, None] + dact
    return _standardize_bwd(gzh, zh, tape["rstd"], norm)


def port_epilogue(z, sp, geom, final_activate, act_slope, norm):
    """epilogue.py:82-128."""
    zh, rstd = _standardize(z, norm)
    rr, cc = _out_index(geom)
    zo = zh[:, :, rr, cc]                       # (B, M, n_out)
    M = z.shape[1]
    lin = zo.sum(axis=1)
    if final_activate in (None,):
        out = (sp["w_eff_out"] + sp["s_eff_out"])[None] * lin + (float(M) * sp["s_eff_out"] * sp["b_out"])[None]
        tape = dict(zh=zh, rstd=rstd, zo=zo, lin=lin)
    else:
        act = act_fwd(zo + sp["b_out"][None, None], final_activate, act_slope).sum(axis=1)
        pre = sp["w_eff_out"][None] * lin + sp["s_eff_out"][None] * act
        out = act_fwd(pre, final_activate, act_slope)
        tape = dict(zh=zh, rstd=rstd, zo=zo, lin=lin, act=act, pre=pre)
    oh, ow = geom.out_port.size
    return out.reshape(z.shape[0], oh, ow), tape


def port_epilogue_bwd(gout, tape, sp, geom, final_activate, act_slope, norm, grads):
    zh, zo = tape["zh"], tape["zo"]
    B, M = zh.shape[:2]
    g = gout.reshape(B, -1)
    rr, cc = _out_index(geom)
    if final_activate is None:
        grads["w_eff_out"] += (g * tape["lin"]).sum(axis=0)
        grads["s_eff_out"] += (g * (tape["lin"] + float(M) * sp["b_out"][None])).sum(axis=0)
        grads["b_out"] += (g * float(M) * sp["s_eff_out"][None]).sum(axis=0)
        gzo = np.broadcast_to(((sp["w_eff_out"] + sp["s_eff_out"])[None] * g)[:, None], zo.shape)
    else:
        gp = g * act_deriv(tape["pre"], final_activate, act_slope)
        grads["w_eff_out"] += (gp * tape["lin"]).sum(axis=0)
        grads["s_eff_out"] += (gp * tape["act"]).sum(axis=0)
        d = act_deriv(zo + sp["b_out"][None, None], final_activate, act_slope)
        sgp = (sp["s_eff_out"][None] * gp)[:, None] * d
        grads["b_out"] += sgp.sum(axis=(0, 1))
        gzo = (sp["w_eff_out"][None] * gp)[:, None] + sgp
    gzh = np.zeros_like(zh)
    for j in range(len(rr)):
        gzh[:, :, rr[j], cc[j]] += gzo[:, :, j]
    return _standardize_bwd(gzh, zh, tape["rstd"], norm)


# ----------------------------------------------------------------------------------------
# Full forward / backward (propagator.py:209-682, backend="nchw_direct")
# ----------------------------------------------------------------------------------------
@dataclass
class Config:
    activate: str | None = "tanh"
    final_activate: str | None = None
    act_slope: float = 0.01
    final_act_slope: float = 0.01
    norm: bool = True
    hard_pin_io: bool = False
    gated_filters: bool = False
    codd_mode: str = "continuous"
    state_temperature: float = 1.0
    active_threshold: float = 0.6
    sharpen: bool = False          # model.py:65-66: the normalised 3x3 sharpen stencil on W


# ----------------------------------------------------------------------------------------
# Spatial stencils (filters.py:12-83) and their application to a weight plane
# (kernels_greens.py:220-237, applied to W before the output-port pin, params.py:246-249)
# ----------------------------------------------------------------------------------------
def sharpen_stencil(norm: bool = True, dtype=np.float64):
    """filters.py:56-68: [[0,-1,0],[-1,5,-1],[0,-1,0]], divided by 5 when ``norm``."""
    k = np.array([[0, -1, 0], [-1, 5, -1], [0, -1, 0]], dtype=dtype)
    return k / 5.0 if norm else k


def spatial_filter_same(x, k):
    """SAME cross-correlation of a 2-D plane with an odd stencil, zeros outside
    (``conv_general_dilated`` with padding "SAME", kernels_greens.py:220-237)."""
    kh, kw = k.shape
    ph, pw = kh // 2, kw // 2
    xp = np.pad(x, ((ph, ph), (pw, pw)))
    out = np.zeros_like(x)
    for a in range(kh):
        for b in range(kw):
            if k[a, b] != 0:
                out += k[a, b] * xp[a:a + x.shape[0], b:b + x.shape[1]]
    return out


def spatial_filter_same_adjoint(gy, k):
    """Adjoint of :func:`spatial_filter_same`: the SAME correlation with the flipped stencil."""
    return spatial_filter_same(gy, k[::-1, ::-1])


def forward(cell_params, filters, inputs, geom: Geometry, cfg: Config = Config(), dtype=np.float64,
            universe=False):
    """Returns ``(outputs (B, oh, ow), tape)``.  ``filters`` is OIHW (M, 1, kh, kw).
    ``universe=True`` stops before the output-port epilogue (``forward_universe``)."""
    if not geom.out_in_roi and not universe:
        raise NotImplementedError("output ports outside the ROI need forward_universe")
    cp = np.asarray(cell_params, dtype=dtype)
    G0 = np.asarray(filters, dtype=dtype)[:, 0]
    G = _sigmoid(G0) if cfg.gated_filters else G0
    kh, kw = geom.kernel_size
    H, W = geom.grid_shape
    cp_used = cp
    if cfg.sharpen:                     # params.py:246-247: W sharpened before the pin
        cp_used = cp.copy()
        cp_used[0] = spatial_filter_same(cp[0], sharpen_stencil(True, dtype))
    sp = precompute(cp_used, geom, cfg.activate, cfg.act_slope, cfg.hard_pin_io, cfg.codd_mode,
                    cfg.state_temperature, cfg.active_threshold)
    d = geom.depth
    tape = dict(sp=sp, G=G, G0=G0, convs=[], epis=[], cp=cp)
    circ = geom.padding_mode == "CIRCULAR"
    valid = geom.padding_mode == "VALID"
    if circ:
        cells = inject_full(inputs, geom, dtype)
        fits = True
    else:
        cells, fits = inject_roi(inputs, geom, dtype)
        if not fits:
            cells_t0 = inject_full(inputs, geom, dtype)
    if valid:
        border_only = sp["border_2d"].copy()
        border_only[_roi(geom)] = 0.0
        delta = conv_valid(border_only[None], G)
        tape["border_only"] = border_only
    else:
        delta = None

    def conv_step(t, x):
        if circ:
            xin = _pad_wrap(x, kh, kw)
            kind = "wrap"
        elif t == 0 and not fits:
            xin = cells_t0
            kind = "full"
        else:
            xin = _pad_same(x, kh, kw)
            kind = "same"
        z = conv_valid(xin, G)
        tape["convs"].append((kind, xin))
        if valid and t > 0:
            z = z + delta
        return z

    x = cells
    for t in range(d - 1):
        z = conv_step(t, x)
        x, et = hidden_epilogue(z, sp, cfg.activate, cfg.act_slope, cfg.norm)
        tape["epis"].append(et)
    z = conv_step(d - 1, x)
    tape["z_final"] = z
    if universe:
        return None, tape
    out, pt = port_epilogue(z, sp, geom, cfg.final_activate, cfg.final_act_slope, cfg.norm)
    tape["port"] = pt
    tape["B"] = out.shape[0]
    return out, tape


def forward_universe(cell_params, filters, inputs, geom: Geometry, cfg: Config = Config(),
                     dtype=np.float64):
    """``propagate_vnn_2d(..., return_universe=True)`` (propagator.py:657-734 and the
    CIRCULAR branch 330-341): the last step runs the ROI epilogue with ``final_activate``
    over the whole ROI; the universe is the (B, H, W) grid with the VALID ring
    ``f(B) * s_prob`` (``B * s_prob`` without a final activation) and ``f`` applied to every
    cell afterwards; the outputs are the port cells of the universe.  Returns
    ``(outputs (B, oh, ow), universe (B, H, W), tape)``."""
    _, tape = forward(cell_params, filters, inputs, geom, cfg, dtype, universe=True)
    sp = tape["sp"]
    fa, fs = cfg.final_activate, cfg.final_act_slope
    roi_final, et = hidden_epilogue(tape["z_final"], sp, fa, fs, cfg.norm)
    B = roi_final.shape[0]
    H, W = geom.grid_shape
    if geom.padding_mode == "VALID":
        Bf = tape["cp"][1]
        ring = (Bf if fa is None else act_fwd(Bf, fa, fs)) * sp["s_prob"]
        pre = np.broadcast_to(ring[None], (B, H, W)).copy()
        pre[(slice(None),) + _roi(geom)] = roi_final
    else:
        pre = roi_final
    uni = pre if fa is None else act_fwd(pre, fa, fs)
    rr, cc = _out_grid_index(geom)
    outputs = uni[:, rr, cc]
    oh, ow = geom.out_port.size
    tape["uni"] = dict(et=et, pre=pre)
    return outputs.reshape(B, oh, ow), uni, tape


def backward_universe(g_universe, tape, geom: Geometry, cfg: Config = Config()):
    """VJP of ``forward_universe`` from the gradient of the universe (add the outputs'
    gradient at the port cells first).  Returns ``(g_cell_params, g_filters)``."""
    g = np.asarray(g_universe, dtype=tape["G"].dtype)
    fa, fs = cfg.final_activate, cfg.final_act_slope
    pre = tape["uni"]["pre"]
    gpre = g if fa is None else g * act_deriv(pre, fa, fs)
    roi = _roi(geom)
    gy = gpre[(slice(None),) + roi]
    ring_g = None
    if geom.padding_mode == "VALID":
        ring_g = gpre.sum(axis=0)
        ring_g[roi] = 0.0
    return backward(None, tape, geom, cfg, final_gy=gy, ring_final_g=ring_g)


def backward(gout, tape, geom: Geometry, cfg: Config = Config(), final_gy=None, ring_final_g=None):
    """Returns ``(g_cell_params (3,H,W), g_filters (M,1,kh,kw))``.  ``final_gy`` (universe
    mode): gradient of the last step's ROI cells, which then run the ROI epilogue with the
    final activation; ``ring_final_g``: gradient of the VALID ring of the universe."""
    sp, G = tape["sp"], tape["G"]
    kh, kw = geom.kernel_size
    H, W = geom.grid_shape
    d = geom.depth
    valid = geom.padding_mode == "VALID"
    grads = {k: np.zeros_like(sp[k]) for k in ("w_eff_roi", "s_eff_roi", "b_roi")}
    if geom.out_in_roi:
        for k in ("w_eff_out", "s_eff_out", "b_out"):
            grads[k] = np.zeros_like(sp[k])
    dG = np.zeros_like(G)
    g_delta = None
    if final_gy is None:
        gz = port_epilogue_bwd(np.asarray(gout, dtype=G.dtype), tape["port"], sp, geom,
                               cfg.final_activate, cfg.final_act_slope, cfg.norm, grads)
    else:
        gz = hidden_epilogue_bwd(np.asarray(final_gy, dtype=G.dtype), tape["uni"]["et"], sp,
                                 cfg.final_activate, cfg.final_act_slope, cfg.norm, grads)
    for t in range(d - 1, -1, -1):
        kind, xin = tape["convs"][t]
        if valid and t > 0:
            s = gz.sum(axis=0, keepdims=True)
            g_delta = s if g_delta is None else g_delta + s
        need_dx = t > 0
        dxin, dGt = conv_valid_bwd(xin, G, gz, need_dx=need_dx)
        dG += dGt
        if not need_dx:
            break
        roi_h, roi_w = geom.roi_shape
        if kind == "wrap":
            gx = _unpad_wrap(dxin, kh, kw, roi_h, roi_w)
        else:
            gx = _unpad_same(dxin, kh, kw)
        gz = hidden_epilogue_bwd(gx, tape["epis"][t - 1], sp, cfg.activate, cfg.act_slope,
                                 cfg.norm, grads)
    # border hoist adjoint (propagator.py:354-371)
    g_border = np.zeros((H, W), dtype=G.dtype)
    if valid and g_delta is not None:
        db, dGb = conv_valid_bwd(tape["border_only"][None], G, g_delta, need_dx=True)
        dG += dGb
        g_border = db[0]
        g_border[_roi(geom)] = 0.0
    # pre-step adjoint (params.py:220-322)
    M = geom.directions
    inv_M = 1.0 / float(M)
    roi = _roi(geom)
    gwe, gse, gbr = grads["w_eff_roi"].copy(), grads["s_eff_roi"].copy(), grads["b_roi"].copy()
    if geom.out_in_roi:
        rr, cc = _out_index(geom)
        np.add.at(gwe, (rr, cc), grads["w_eff_out"])
        np.add.at(gse, (rr, cc), grads["s_eff_out"])
        np.add.at(gbr, (rr, cc), grads["b_out"])
    cp = tape["cp"]
    s_roi = sp["s_prob"][roi]
    w_roi = sp["w_pinned"][roi]
    g_wp = np.zeros((H, W), dtype=G.dtype)
    g_wp[roi] = gwe * inv_M * (1.0 - s_roi)
    g_s = np.zeros((H, W), dtype=G.dtype)
    g_s[roi] = -gwe * inv_M * w_roi + gse * inv_M
    g_B = np.zeros((H, W), dtype=G.dtype)
    g_B[roi] = gbr
    Bf = cp[1]
    g_B += g_border * act_deriv(Bf, cfg.activate, cfg.act_slope) * sp["s_prob"]
    g_s += g_border * act_fwd(Bf, cfg.activate, cfg.act_slope)
    if ring_final_g is not None:           # universe ring f(B) * s_prob (B * s_prob for None)
        fa, fs = cfg.final_activate, cfg.final_act_slope
        fb = Bf if fa is None else act_fwd(Bf, fa, fs)
        dfb = np.ones_like(Bf) if fa is None else act_deriv(Bf, fa, fs)
        g_B += ring_final_g * dfb * sp["s_prob"]
        g_s += ring_final_g * fb
    g_W = np.where(geom.out_weight_mask, 0.0, g_wp)
    if cfg.sharpen:
        g_W = spatial_filter_same_adjoint(g_W, sharpen_stencil(True, g_W.dtype))
    g_S = g_s * sp["ds_prob"]
    g_cell = np.stack([g_W, g_B, g_S]).astype(G.dtype)
    if cfg.gated_filters:
        sg = _sigmoid(tape["G0"])
        dG = dG * sg * (1.0 - sg)
    return g_cell, dG[:, None]


# ----------------------------------------------------------------------------------------
# Losses (trainer.py:57-61) and SGD
# ----------------------------------------------------------------------------------------
def mse_loss(out, targets):
    o = out.reshape(out.shape[0], -1)
    y = np.asarray(targets, dtype=o.dtype).reshape(o.shape)
    diff = o - y
    return float((diff * diff).mean()), (2.0 * diff / diff.size).reshape(out.shape)


def softmax_ce_loss(out, labels):
    """``optax.softmax_cross_entropy_with_integer_labels(...).mean()`` over outputs (B, n, 1)."""
    o = out.reshape(out.shape[0], -1)
    m = o.max(axis=1, keepdims=True)
    e = np.exp(o - m)
    ssum = e.sum(axis=1, keepdims=True)
    logp = o - m - np.log(ssum)
    lab = np.asarray(labels).astype(np.int64).reshape(-1)
    B = o.shape[0]
    loss = float(-logp[np.arange(B), lab].mean())
    p = e / ssum
    g = p.copy()
    g[np.arange(B), lab] -= 1.0
    return loss, (g / B).reshape(out.shape)


def train_step(cell_params, filters, inputs, targets, geom, cfg: Config = Config(), lr=1e-2,
               loss="mse", dtype=np.float64):
    """One value_and_grad + SGD step; returns ``(loss, new_cell, new_filters, g_cell, g_filt)``."""
    out, tape = forward(cell_params, filters, inputs, geom, cfg, dtype)
    if loss == "mse":
        lval, gout = mse_loss(out, targets)
    else:
        lval, gout = softmax_ce_loss(out, targets)
    g_cell, g_filt = backward(gout, tape, geom, cfg)
    cp = np.asarray(cell_params, dtype=dtype)
    fl = np.asarray(filters, dtype=dtype)
    return lval, cp - lr * g_cell, fl - lr * g_filt, g_cell, g_filt


# ----------------------------------------------------------------------------------------
# ALU data (datasets.py:77-130), seeded numpy stand-in
# ----------------------------------------------------------------------------------------
# ----------------------------------------------------------------------------------------
# Packed 8-bit evaluation (trainer.py:49-54, 122-138)
# ----------------------------------------------------------------------------------------
BIT_WEIGHTS_U8 = np.array([128, 64, 32, 16, 8, 4, 2, 1], dtype=np.uint8)


def packed_predictions(logits) -> np.ndarray:
    """``packbits_u8_on_device(jnp.round(logits).astype(jnp.uint8))`` of the reference: each
    rounded logit is cast to uint8 (XLA's float-to-integer conversion saturates: below 0
    gives 0, above 255 gives 255), multiplied by its bit weight and summed in uint8, which
    wraps modulo 256 -- so a rounded logit of 2 at bit weight 128 contributes 0, not a set
    bit.  ``logits`` (B, 8) or (B, 8, 1) -> (B, 1) uint8."""
    x = np.asarray(logits, dtype=np.float64)
    if x.ndim == 3 and x.shape[-1] == 1:
        x = x[..., 0]
    u8 = np.clip(np.round(x), 0, 255).astype(np.uint8)
    return ((u8.astype(np.int64) * BIT_WEIGHTS_U8.astype(np.int64)).sum(-1) % 256).astype(np.uint8)[:, None]


def packed_accuracy(logits, packed_targets) -> float:
    """Fraction of samples whose packed prediction equals the packed target byte."""
    p = packed_predictions(logits)[:, 0]
    return float((p == np.asarray(packed_targets).reshape(-1)).mean())


def alu_truth_table(numbers, operands, controls):
    """The vectorised uint8 ALU table of datasets.py:97-116."""
    one = np.uint8(1)
    conds = [(controls == 0) | (controls == 4), controls == 1, (controls == 2) | (controls == 8),
             controls == 3, controls == 5, controls == 6, controls == 7]
    choices = [numbers, (numbers + one).astype(np.uint8), (numbers + operands).astype(np.uint8),
               (numbers + operands + one).astype(np.uint8), (numbers - one).astype(np.uint8),
               (numbers - operands).astype(np.uint8), (numbers - operands - one).astype(np.uint8)]
    return np.select(conds, choices, default=numbers).astype(np.uint8)


def alu_batch(rng, B, n=8, ctrl_bits=4, noise=0.2, operand_range=(1, 128), ctrl_range=(1, 16)):
    """Returns ``(inputs (B,3,n,1) float32, targets (B,n) float32, packed (B,) uint8)``."""
    nums = rng.integers(operand_range[0], operand_range[1], size=(B, 1), dtype=np.uint8)
    ops = rng.integers(operand_range[0], operand_range[1], size=(B, 1), dtype=np.uint8)
    ctl = rng.integers(ctrl_range[0], ctrl_range[1], size=(B, 1), dtype=np.uint8)
    y = alu_truth_table(nums, ops, ctl)
    X1 = np.unpackbits(nums, axis=1, count=n).astype(np.float32)
    X2 = np.unpackbits(ops, axis=1, count=n).astype(np.float32)
    C = np.unpackbits(ctl, axis=1, count=n).astype(np.float32)
    if noise:
        X1 += rng.uniform(-noise, noise, X1.shape).astype(np.float32)
        X2 += rng.uniform(-noise, noise, X2.shape).astype(np.float32)
        C += rng.uniform(-noise, noise, C.shape).astype(np.float32)
    inputs = np.stack([X1, X2, C], axis=1)[..., None].astype(np.float32)
    targets = np.unpackbits(y, axis=1, count=n).astype(np.float32)
    return inputs, targets, y[:, 0]
