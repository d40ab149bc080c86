"""Stateless d-step VNN propagation on B200 (drop-in for ``propagate_vnn_2d``).

Mirrors ``neurocell/propagator.py:209-734`` of shakes76/neurocell-v2: same signature,
argument meaning and ValueError behaviour.  Every reference backend name is accepted and
runs the B200 path, whose numerics follow the reference's semantic backend
``nchw_direct`` (propagator.py:413-432).  The backend name picks the Green's convolution
algorithm the way the reference's backends do: the FFT backends ("pallas_sram",
"rfft_hoisted", "nchw_rfft_bwd") run the FFT convolution, "nchw_direct" and
"pallas_fused" the direct one, and "auto" / "b200" apply the reference's auto rule
(propagator.py:68-85: FFT for kh*kw > 512 outside CIRCULAR mode).
"""
from __future__ import annotations

from typing import Sequence

import torch

from . import ops
from .filters import apply_spatial_filter_2d
from .params import VNNParams, check_codd_mode
from .topology import ChipTopology2D, CoordinatePortSpec

SUPPORTED_BACKENDS = (
    "auto",
    "nchw_direct",
    "rfft_hoisted",
    "nchw_rfft_bwd",
    "pallas_fused",
    "pallas_sram",
    "b200",
)


CONV_OF_BACKEND = {
    "auto": "auto", "b200": "auto",
    "nchw_direct": "direct", "pallas_fused": "direct",
    "rfft_hoisted": "fft", "nchw_rfft_bwd": "fft", "pallas_sram": "fft",
}


def select_optimal_backend(topology: ChipTopology2D) -> str:
    """``backend="auto"`` (propagator.py:68-85): the B200 path serves every topology."""
    return "b200"


def _normalize_port_inputs(inputs, topology: ChipTopology2D):
    """Single-port or multi-port batched inputs -> list of per-port tensors (propagator.py:88-100)."""
    if isinstance(inputs, (list, tuple)):
        return inputs[0].shape[0], list(inputs)
    bsz = inputs.shape[0]
    if len(topology.in_ports) == 1:
        port0 = topology.in_ports[0]
        if inputs.ndim == 2 or (inputs.ndim == 3 and tuple(inputs.shape[1:]) == tuple(port0.size)):
            return bsz, [inputs]
    return bsz, [inputs[:, idx] for idx in range(len(topology.in_ports))]


def flatten_inputs(inputs, topology: ChipTopology2D):
    """Returns ``(flat (B, n_in) float32 CUDA tensor, per-port sample shapes)``."""
    B, arrs = _normalize_port_inputs(inputs, topology)
    shapes = []
    flats = []
    for a, port in zip(arrs, topology.in_ports):
        if not isinstance(a, torch.Tensor):
            a = torch.as_tensor(a)
        if isinstance(port, CoordinatePortSpec):
            shapes.append((port.num_points,))
        elif a.ndim == 3:
            shapes.append((int(a.shape[1]), int(a.shape[2])))
        else:
            shapes.append(tuple(int(s) for s in a.shape[1:]))
        flats.append(a.reshape(B, -1))
    if not flats:
        raise ValueError("topology has no input ports")
    if len(flats) == 1:
        flat = flats[0]
    elif isinstance(inputs, torch.Tensor) and inputs.is_contiguous() and \
            sum(f.shape[1] for f in flats) == inputs[0].numel():
        flat = inputs.reshape(B, -1)          # ports stacked along dim 1: already in order
    else:
        flat = torch.cat([f.to(flats[0].device) for f in flats], dim=1)
    return flat, tuple(shapes)


def propagate_vnn_2d(
    params: VNNParams,
    inputs,
    topology: ChipTopology2D,
    activate=torch.tanh,
    final_activate=None,
    norm: bool = True,
    sharpen_filter=None,
    gated_filters: bool = False,
    hard_pin_io: bool = False,
    backend: str = "b200",
    return_universe: bool = False,
    spatial_mask=None,
    codd_mode: str = "continuous",
    state_temperature: float = 1.0,
    active_threshold: float = 0.6,
) -> torch.Tensor:
    """Batched forward propagation over ``topology.depth`` steps -> (B, out_h, out_w).

    Differentiable with respect to ``params`` through the library's hand-written VJP.
    """
    if backend not in SUPPORTED_BACKENDS:
        raise ValueError(f"Unsupported backend '{backend}'; choose from {SUPPORTED_BACKENDS}.")
    check_codd_mode(codd_mode)
    act, slope = ops.resolve_activation(activate)
    fact, fslope = ops.resolve_activation(final_activate)
    if sharpen_filter is not None:
        # params.py:246-247: W is filtered (SAME, zeros outside) before the output-port pin,
        # on the full grid, ahead of any sub-ROI crop; autograd takes the gradient back to W
        cp = params.cell_params
        w_sharp = apply_spatial_filter_2d(cp[0], torch.as_tensor(sharpen_filter), padding="SAME")
        params = VNNParams(torch.cat([w_sharp[None], cp[1:]], dim=0), params.greens_filters)
    roi_bbox = None
    if (spatial_mask is not None and not spatial_mask.is_full_roi
            and topology.padding_mode != "CIRCULAR"):
        # adaptive sub-ROI (propagator.py:235-241): the kernels run on the sub-ROI's window
        roi_bbox = tuple(int(v) for v in spatial_mask.roi_bbox)
    full_grid = return_universe or not topology.out_in_roi
    ops._require_cuda(params.cell_params, "params.cell_params")
    ops._require_cuda(params.greens_filters, "params.greens_filters")
    flat, shapes = flatten_inputs(inputs, topology)
    device = params.cell_params.device
    if flat.device != device:
        flat = flat.to(device, non_blocking=True)
    plan = ops.get_plan(topology, shapes, device, act, slope, fact, fslope, norm, hard_pin_io,
                        gated_filters, CONV_OF_BACKEND[backend], roi_bbox, universe=full_grid)
    if plan.window is not None:
        r0, r1, c0, c1 = plan.window
        cell_w = params.cell_params[:, r0:r1, c0:c1]
        if full_grid:
            # the sub-ROI's window universe placed in the full grid, outputs read from it
            # (propagator.py:700-718, 726-733)
            _, uni_w = ops.propagate_universe(cell_w, params.greens_filters, flat, plan, codd_mode,
                                              state_temperature, active_threshold)
            full = ops.get_plan(topology, shapes, device, act, slope, fact, fslope, norm,
                                hard_pin_io, gated_filters, CONV_OF_BACKEND[backend])
            out, uni = ops.embed_universe(params.cell_params, uni_w, full, plan.window, codd_mode,
                                          state_temperature, active_threshold)
            out = out.reshape((out.shape[0],) + full.out_shape)
            return (out, uni) if return_universe else out
        out = ops.propagate(cell_w, params.greens_filters, flat, plan, codd_mode, state_temperature,
                            active_threshold)
        return out.reshape((out.shape[0],) + plan.out_shape)
    if full_grid:
        # (outputs, full-grid universe) as the reference returns them (propagator.py:730-733);
        # output ports outside the ROI always take this full-grid path (propagator.py:684)
        out, uni = ops.propagate_universe(params.cell_params, params.greens_filters, flat, plan,
                                          codd_mode, state_temperature, active_threshold)
        out = out.reshape((out.shape[0],) + plan.out_shape)
        return (out, uni) if return_universe else out
    out = ops.propagate(params.cell_params, params.greens_filters, flat, plan, codd_mode,
                        state_temperature, active_threshold)
    return out.reshape((out.shape[0],) + plan.out_shape)
