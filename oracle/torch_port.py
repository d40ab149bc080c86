"""Torch-CPU restatement of the VNN hot path -- TEST INFRASTRUCTURE / CPU BASELINE ONLY.

A second, independent restatement of ``neurocell/propagator.py:343-432`` (the reference's
``nchw_direct`` semantic backend) written with ``torch.nn.functional.conv2d`` and torch
autograd instead of hand-written adjoints.  It serves two purposes:

* in float64 it cross-checks the hand-written backward of :mod:`oracle.vnn_oracle`;
* in float32 with all host threads it is the timed CPU baseline of ``bench.py`` (the
  reference's own JAX CPU path cannot be installed in this environment), which is the
  same algorithm the reference's XLA CPU path runs: direct convolution, standardisation,
  factored Codd epilogue, output-port epilogue, loss, autograd, SGD.

It always runs on the CPU.  Only ``tests/`` and ``bench.py`` import it.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import vnn_oracle as O


def _act(x, name, slope):
    if name in (None, "identity"):
        return x
    if name == "tanh":
        return torch.tanh(x)
    if name == "sigmoid":
        return torch.sigmoid(x)
    if name == "relu":
        return torch.relu(x)
    if name == "leaky_relu":
        return torch.where(x >= 0, x, slope * x)
    if name == "gelu":
        c = float(np.sqrt(2.0 / np.pi))
        return 0.5 * x * (1.0 + torch.tanh(c * (x + 0.044715 * x ** 3)))
    raise ValueError(name)


class TorchVNN:
    """Precomputes static geometry tensors for one :class:`oracle.vnn_oracle.Geometry`."""

    def __init__(self, geom: O.Geometry, cfg: O.Config = O.Config(), dtype=torch.float64):
        self.g, self.cfg, self.dtype = geom, cfg, dtype
        self.io = torch.from_numpy(geom.io_state_mask)
        self.ow = torch.from_numpy(geom.out_weight_mask)
        rr, cc = O._out_index(geom)
        self.rr, self.cc = torch.from_numpy(np.asarray(rr)), torch.from_numpy(np.asarray(cc))

    def codd(self, s_raw):
        c, g = self.cfg, self.g
        s_base = s_raw if c.hard_pin_io else torch.where(self.io, torch.ones_like(s_raw), s_raw)
        if c.codd_mode == "continuous":
            s = torch.sigmoid(s_base)
        else:
            tau = max(float(np.float32(c.state_temperature)), float(np.float32(1e-4)))
            soft = torch.sigmoid(s_base / tau)
            if c.codd_mode == "annealed":
                s = soft
            elif c.codd_mode == "ste_binary":
                hard = (s_base >= 0).to(s_raw.dtype)
                s = soft + (hard - soft).detach()
            else:
                thr = float(np.float32(c.active_threshold))
                hard = torch.where(s_base >= thr, 1.0, torch.where(s_base > 0, 0.5, 0.0)).to(s_raw.dtype)
                s = soft + (hard - soft).detach()
        if c.hard_pin_io:
            s = torch.where(self.io, torch.ones_like(s), s)
        return s

    def _inputs_fit(self, lo_r, hi_r, lo_c, hi_c):
        for p in self.g.in_ports:
            cells = (p.coords if isinstance(p, O.CoordPort) else
                     [(p.offset[0] + i, p.offset[1] + j) for i in range(p.size[0]) for j in range(p.size[1])])
            if not all(lo_r <= r < hi_r and lo_c <= c < hi_c for r, c in cells):
                return False
        return True

    def forward(self, cell, filt, cells_t0_full, roi_bbox=None, universe=False):
        """``cells_t0_full``: (B, H, W) injected field (inputs already placed).
        ``roi_bbox``: adaptive sub-ROI (r0, r1, c0, c1) in ROI coordinates (propagator.py:
        228-241, 343-371, 394-397, 657-660): step parameters sliced to it, t=0 inputs injected
        into it when they fit (else the full-grid VALID conv cropped to it), SAME convolution
        of the sub-ROI cells, the border hoist over the window of the border template whose
        whole ROI is zeroed, the output port epilogue on the cropped planes.
        ``universe``: returns ``(outputs, (B, H, W) universe)`` by the full-grid path
        (propagator.py:684-733): the last step's ROI epilogue with the final activation, the
        cells outside the (sub-)ROI f(B) * s_prob (VALID) or 0 (SAME), f over the grid, the
        outputs read from it.  Not for CIRCULAR chips."""
        g, c = self.g, self.cfg
        H, W = g.grid_shape
        kh, kw = g.kernel_size
        M = g.directions
        ph, pw = g.pad_h, g.pad_w
        Wf, Bf, Sf = cell[0], cell[1], cell[2]
        if c.sharpen:                   # params.py:246-247 (kernels_greens.py:220-237)
            k = torch.from_numpy(O.sharpen_stencil(True)).to(Wf.dtype)
            Wf = torch.nn.functional.conv2d(Wf[None, None], k[None, None], padding=1)[0, 0]
        G = torch.sigmoid(filt) if c.gated_filters else filt
        w_pinned = torch.where(self.ow, torch.ones_like(Wf), Wf)
        s = self.codd(Sf)
        roi = (slice(ph, H - ph), slice(pw, W - pw))
        w_eff = w_pinned[roi] * (1.0 - s[roi]) / M
        s_eff = s[roi] / M
        b_roi = Bf[roi]
        roi_h, roi_w = g.roi_shape
        br0, br1, bc0, bc1 = roi_bbox if roi_bbox is not None else (0, roi_h, 0, roi_w)
        sub = (slice(br0, br1), slice(bc0, bc1))
        w_eff, s_eff, b_roi = w_eff[sub], s_eff[sub], b_roi[sub]
        circ = g.padding_mode == "CIRCULAR"
        valid = g.padding_mode == "VALID"
        if valid:
            border = _act(Bf, c.activate, c.act_slope) * s
            mask = torch.ones_like(border)
            mask[roi] = 0.0
            bo = (border * mask)[br0:br1 + kh - 1, bc0:bc1 + kw - 1]
            delta = F.conv2d(bo[None, None], G)
        fits = g.in_in_roi and not circ and self._inputs_fit(ph + br0, ph + br1, pw + bc0, pw + bc1)
        x = (cells_t0_full[:, ph + br0:ph + br1, pw + bc0:pw + bc1] if fits else cells_t0_full)
        cp = ((kh - 1) // 2, (kw - 1) // 2)

        def conv(t, x):
            if circ:
                xp = F.pad(x[:, None], (cp[1], cp[1], cp[0], cp[0]), mode="circular")
                return F.conv2d(xp, G)
            if t == 0 and not fits:
                z = F.conv2d(x[:, None], G)[:, :, br0:br1, bc0:bc1]
            else:
                z = F.conv2d(x[:, None], G, padding=cp)
            if valid and t > 0:
                z = z + delta
            return z

        def std(z):
            if not c.norm:
                return z
            mu = z.mean(dim=(-2, -1), keepdim=True)
            var = ((z - mu) ** 2).mean(dim=(-2, -1), keepdim=True)
            return (z - mu) / torch.sqrt(var + O.NORM_EPS)

        for t in range(g.depth - 1):
            zh = std(conv(t, x))
            lin = zh.sum(1)
            if c.activate in (None, "identity"):
                act = lin + M * b_roi
            else:
                act = _act(zh + b_roi, c.activate, c.act_slope).sum(1)
            x = w_eff * lin + s_eff * act
        zh = std(conv(g.depth - 1, x))
        if universe:
            if circ:
                raise NotImplementedError("the torch port's universe path is for VALID / SAME chips")
            fa, fsl = c.final_activate, c.final_act_slope
            lin = zh.sum(1)
            act = lin + M * b_roi if fa in (None, "identity") else _act(zh + b_roi, fa, fsl).sum(1)
            roi_final = w_eff * lin + s_eff * act
            fill = _act(Bf, fa, fsl) * s if valid else torch.zeros_like(Bf)
            final = fill[None].expand(zh.shape[0], H, W).clone()
            final[:, ph + br0:ph + br1, pw + bc0:pw + bc1] = roi_final
            final = _act(final, fa, fsl)
            gr, gc = O._out_grid_index(g)
            oh, ow = g.out_port.size
            return final[:, torch.as_tensor(gr), torch.as_tensor(gc)].reshape(-1, oh, ow), final
        rr, cc = self.rr - br0, self.cc - bc0
        zo = zh[:, :, rr, cc]
        lin = zo.sum(1)
        w_o, s_o, b_o = w_eff[rr, cc], s_eff[rr, cc], b_roi[rr, cc]
        if c.final_activate is None:
            out = (w_o + s_o) * lin + M * s_o * b_o
        else:
            act = _act(zo + b_o, c.final_activate, c.final_act_slope).sum(1)
            out = _act(w_o * lin + s_o * act, c.final_activate, c.final_act_slope)
        oh, ow = g.out_port.size
        return out.reshape(-1, oh, ow)


def value_and_grad(geom, cfg, cell_params, filters, inputs, targets, loss="mse", dtype=torch.float64,
                   roi_bbox=None):
    """Returns ``(loss, out, g_cell, g_filters)`` as numpy arrays (autograd)."""
    tv = TorchVNN(geom, cfg, dtype)
    cell = torch.tensor(np.asarray(cell_params), dtype=dtype, requires_grad=True)
    filt = torch.tensor(np.asarray(filters)[:, :1], dtype=dtype, requires_grad=True)
    x0 = torch.from_numpy(O.inject_full(inputs, geom, np.float64)).to(dtype)
    out = tv.forward(cell, filt, x0, roi_bbox)
    o = out.reshape(out.shape[0], -1)
    if loss == "mse":
        y = torch.as_tensor(np.asarray(targets), dtype=dtype).reshape(o.shape)
        L = ((o - y) ** 2).mean()
    else:
        lab = torch.as_tensor(np.asarray(targets)).long().reshape(-1)
        L = F.cross_entropy(o, lab)
    L.backward()
    return float(L.detach()), out.detach().numpy(), cell.grad.numpy(), filt.grad.numpy()


def universe_value_and_grad(geom, cfg, cell_params, filters, inputs, w_out, w_uni, roi_bbox=None,
                            dtype=torch.float64):
    """Full-grid path (``return_universe=True``) under the scalar loss
    sum(out * w_out) + sum(universe * w_uni); returns ``(out, universe, g_cell, g_filters)``."""
    tv = TorchVNN(geom, cfg, dtype)
    cell = torch.tensor(np.asarray(cell_params), dtype=dtype, requires_grad=True)
    filt = torch.tensor(np.asarray(filters)[:, :1], dtype=dtype, requires_grad=True)
    x0 = torch.from_numpy(O.inject_full(inputs, geom, np.float64)).to(dtype)
    out, uni = tv.forward(cell, filt, x0, roi_bbox, universe=True)
    L = (out * torch.as_tensor(np.asarray(w_out), dtype=dtype).reshape(out.shape)).sum() + \
        (uni * torch.as_tensor(np.asarray(w_uni), dtype=dtype)).sum()
    L.backward()
    return out.detach().numpy(), uni.detach().numpy(), cell.grad.numpy(), filt.grad.numpy()
