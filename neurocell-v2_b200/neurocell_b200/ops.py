"""Torch-facing operators over the C ABI (include/neurocell_b200.h).

PyTorch supplies device memory (caching allocator), the current CUDA stream and autograd;
every FLOP runs in ``libneurocell_b200.so``.  Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from .topology import ChipTopology2D, CoordinatePortSpec


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"neurocell_b200: `{name}` must be a CUDA tensor (there is no CPU path)")


def resolve_activation(activate) -> tuple[str, float]:
    """Maps a callable or name to ``(name, leaky_slope)`` (kernels_pallas.py:76-103)."""
    if activate is None or activate == "identity":
        return "identity", 1.0
    import functools
    import torch.nn.functional as F
    table = {
        torch.tanh: "tanh", F.tanh: "tanh", torch.sigmoid: "sigmoid", F.sigmoid: "sigmoid",
        torch.relu: "relu", F.relu: "relu", F.leaky_relu: "leaky_relu", F.gelu: "gelu",
    }
    if isinstance(activate, str):
        if activate in ("tanh", "sigmoid", "relu", "leaky_relu", "gelu"):
            return activate, (0.01 if activate == "leaky_relu" else 0.0)
    elif activate in table:
        name = table[activate]
        return name, (0.01 if name == "leaky_relu" else 0.0)
    elif isinstance(activate, functools.partial) and activate.func is F.leaky_relu:
        slope = activate.keywords.get("negative_slope", activate.args[0] if activate.args else 0.01)
        return "leaky_relu", float(slope)
    else:
        name = getattr(activate, "__name__", "")
        if name in ("tanh", "sigmoid", "relu", "leaky_relu", "gelu"):
            return name, (0.01 if name == "leaky_relu" else 0.0)
    raise ValueError(f"Unsupported activation function: {activate}")


# ---------------------------------------------------------------------------------------
# static plan (port tables and masks on the device)
# ---------------------------------------------------------------------------------------
@dataclass
class Plan:
    topology: ChipTopology2D
    topo: _lib.NcTopo
    buf: torch.Tensor              # device plan buffer
    n_in: int
    n_out: int
    out_shape: tuple
    window: tuple | None = None    # adaptive sub-ROI: grid slice (r0, r1, c0, c1) of the plan


_PLANS: dict = {}


def _input_index(topology: ChipTopology2D, shapes) -> np.ndarray:
    """Flat grid index of every input value, in injection order (propagator.py:103-132).

    ``shapes`` are the per-sample shapes of the port arrays.  A 3-D rectangular input is
    written with its own (ih, iw) shape, which reproduces the reference's quirk of placing
    the ALU's (8, 1) ``ctrl`` input as a column although its port is (1, 8).  Later writes
    to the same cell win, as in the reference's sequential ``.at[].set``.
    """
    H, W = topology.grid_shape
    idx = []
    for shp, port in zip(shapes, topology.in_ports):
        if isinstance(port, CoordinatePortSpec):
            if int(np.prod(shp)) != port.num_points:
                raise ValueError(f"input for port '{port.name}' has {int(np.prod(shp))} values, "
                                 f"expected {port.num_points}")
            idx.extend(int(r) * W + int(c) for r, c in port.coords)
        else:
            r0, c0 = port.offset
            if len(shp) == 2:
                ih, iw = shp
            else:
                ih, iw = port.size
                if int(np.prod(shp)) != ih * iw:
                    raise ValueError(f"input for port '{port.name}' has shape {shp}, "
                                     f"expected {port.size}")
            if r0 + ih > H or c0 + iw > W:
                raise ValueError(f"input of shape {(ih, iw)} at {port.offset} exceeds the grid")
            for r in range(r0, r0 + ih):
                for c in range(c0, c0 + iw):
                    idx.append(r * W + c)
    arr = np.asarray(idx, dtype=np.int32)
    seen = set()
    for j in range(len(arr) - 1, -1, -1):      # keep the last write to each cell
        if arr[j] in seen:
            arr[j] = -1
        else:
            seen.add(int(arr[j]))
    return arr


def _output_index(topology: ChipTopology2D) -> tuple[np.ndarray, tuple]:
    H, W = topology.grid_shape
    op = topology.out_port
    if isinstance(op, CoordinatePortSpec):
        return (op.rows.astype(np.int64) * W + op.cols).astype(np.int32), op.size
    r0, c0 = op.offset
    oh, ow = op.size
    rr, cc = np.meshgrid(np.arange(r0, r0 + oh), np.arange(c0, c0 + ow), indexing="ij")
    return (rr * W + cc).ravel().astype(np.int32), (oh, ow)


def _window_tables(topology: ChipTopology2D, roi_bbox, in_idx, out_idx, universe=False):
    """Adaptive sub-ROI (propagator.py:228-241, 343-371) as its own VALID / SAME problem: the
    grid window that holds the sub-ROI and its kernel halo.  Returns the window slice, its
    shape, the remapped port tables (inputs outside the window dropped), the cropped masks
    and the border mask (the full ROI is dead in the reference's border template).

    ``universe``: the window plan of the full-grid path, whose outputs are gathered from the
    assembled full grid (nc_universe_embed_forward); its own output table is one placeholder
    cell, the sub-ROI's first cell, so output ports may lie anywhere on the chip."""
    H, W = topology.grid_shape
    ph, pw = topology.pad_h, topology.pad_w
    r0, r1, c0, c1 = roi_bbox
    gr0, gr1, gc0, gc1 = r0, r1 + 2 * ph, c0, c1 + 2 * pw       # grid rows / cols of the window
    wh, ww = gr1 - gr0, gc1 - gc0

    def remap(idx, required):
        r, c = idx // W - gr0, idx % W - gc0
        inside = (idx >= 0) & (r >= 0) & (r < wh) & (c >= 0) & (c < ww)
        if required and not inside.all():
            raise NotImplementedError("output ports outside the adaptive sub-ROI")
        return np.where(inside, r * ww + c, -1).astype(np.int32)

    io = np.asarray(topology.io_state_mask, np.uint8)[gr0:gr1, gc0:gc1]
    ow = np.asarray(topology.out_weight_mask, np.uint8)[gr0:gr1, gc0:gc1]
    bmask = np.ones((H, W), np.uint8)
    if topology.padding_mode == "VALID":
        bmask[ph:H - ph, pw:W - pw] = 0
    if universe:
        out_w = np.array([ph * ww + pw], np.int32)
        return ((gr0, gr1, gc0, gc1), (wh, ww), remap(in_idx, False), out_w, np.ascontiguousarray(io),
                np.ascontiguousarray(ow), np.ascontiguousarray(bmask[gr0:gr1, gc0:gc1]))
    out_w = remap(out_idx, True)
    orr, occ = out_w // ww - ph, out_w % ww - pw
    if ((orr < 0) | (orr >= r1 - r0) | (occ < 0) | (occ >= c1 - c0)).any():
        raise NotImplementedError("output ports outside the adaptive sub-ROI")
    return ((gr0, gr1, gc0, gc1), (wh, ww), remap(in_idx, False), out_w, np.ascontiguousarray(io),
            np.ascontiguousarray(ow), np.ascontiguousarray(bmask[gr0:gr1, gc0:gc1]))


def get_plan(topology: ChipTopology2D, in_shapes: tuple, device: torch.device, act: str,
             act_slope: float, final_act: str, final_act_slope: float, norm: bool,
             hard_pin_io: bool, gated_filters: bool, conv: str = "auto", roi_bbox=None,
             universe: bool = False) -> Plan:
    """``conv``: Green's convolution algorithm, "auto" | "direct" | "fft" (nc_conv_algo).
    ``roi_bbox``: adaptive sub-ROI (r0, r1, c0, c1) in ROI coordinates, or None.
    ``universe``: with ``roi_bbox``, the window plan of the full-grid universe path."""
    if conv not in _lib.NC_CONV:
        raise ValueError(f"Unsupported conv algorithm '{conv}'; choose from {tuple(_lib.NC_CONV)}.")
    key = (topology.key(), in_shapes, str(device), act, act_slope, final_act, final_act_slope,
           bool(norm), bool(hard_pin_io), bool(gated_filters), conv,
           None if roi_bbox is None else tuple(int(v) for v in roi_bbox),
           bool(universe) and roi_bbox is not None)
    plan = _PLANS.get(key)
    if plan is not None:
        return plan
    lib = _lib.load()
    in_idx = _input_index(topology, in_shapes)
    out_idx, out_shape = _output_index(topology)
    io = np.ascontiguousarray(topology.io_state_mask, dtype=np.uint8)
    ow = np.ascontiguousarray(topology.out_weight_mask, dtype=np.uint8)
    bmask, window = None, None
    grid = topology.grid_shape
    if roi_bbox is not None:
        if topology.padding_mode == "CIRCULAR":
            raise NotImplementedError("adaptive sub-ROIs are not defined for CIRCULAR chips")
        window, grid, in_idx, out_idx, io, ow, bmask = _window_tables(topology, roi_bbox, in_idx,
                                                                      out_idx, universe)
    t = _lib.NcTopo()
    t.H, t.W = grid
    t.kh, t.kw = topology.kernel_size
    t.M, t.depth = topology.directions, topology.depth
    t.padding = _lib.NC_PAD[topology.padding_mode]
    t.n_in, t.n_out = int(in_idx.size), int(out_idx.size)
    t.act, t.final_act = _lib.NC_ACT[act], _lib.NC_ACT[final_act]
    t.act_slope, t.final_act_slope = float(act_slope), float(final_act_slope)
    t.norm, t.hard_pin_io, t.gated_filters = int(norm), int(hard_pin_io), int(gated_filters)
    t.conv_algo = _lib.NC_CONV[conv]
    nbytes = lib.nc_plan_bytes(ctypes.byref(t))
    if nbytes == 0:
        msg = lib.nc_last_error().decode(errors="replace")
        if "exceeds" in msg:
            raise NotImplementedError(f"neurocell_b200: {msg}")
        raise ValueError(f"neurocell_b200: invalid topology for the B200 path ({msg})")
    buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
    in_c = np.ascontiguousarray(in_idx) if in_idx.size else np.zeros(1, np.int32)
    with torch.cuda.device(device):
        _lib.check(lib.nc_plan_build(ctypes.byref(t), in_c.ctypes.data, out_idx.ctypes.data,
                                     io.ctypes.data, ow.ctypes.data,
                                     None if bmask is None else bmask.ctypes.data, _ptr(buf),
                                     nbytes, _stream(device)), "nc_plan_build")
    plan = Plan(topology, t, buf, int(in_idx.size), int(out_idx.size), tuple(out_shape), window)
    _PLANS[key] = plan
    return plan


def _codd(mode: str, tau, thr) -> _lib.NcCodd:
    c = _lib.NcCodd()
    c.mode = _lib.NC_CODD[mode]
    c.temperature = float(tau)
    c.active_threshold = float(thr)
    return c


# ---------------------------------------------------------------------------------------
# the propagation operator with a hand-written VJP
# ---------------------------------------------------------------------------------------
class _VNNPropagate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cell_params, filters, flat_inputs, plan: Plan, codd: _lib.NcCodd, train: bool):
        lib = _lib.load()
        dev = cell_params.device
        B = flat_inputs.shape[0]
        flags = _lib.NC_FLAG_TRAIN if train else 0
        ws_bytes = lib.nc_workspace_bytes(ctypes.byref(plan.topo), B, flags)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        out = torch.empty((B, plan.n_out), dtype=torch.float32, device=dev)
        _lib.check(lib.nc_vnn_forward(ctypes.byref(plan.topo), _ptr(plan.buf), _ptr(cell_params),
                                      _ptr(filters), _ptr(flat_inputs), B, ctypes.byref(codd),
                                      flags, _ptr(out), _ptr(ws), ws_bytes, _stream(dev)),
                   "nc_vnn_forward")
        _after_call(ws, "nc_vnn_forward")
        if train:
            ctx.save_for_backward(cell_params, filters, flat_inputs)
            ctx.ws, ctx.ws_bytes, ctx.plan, ctx.codd = ws, ws_bytes, plan, codd
        return out

    @staticmethod
    def backward(ctx, g_out):
        lib = _lib.load()
        cell_params, filters, flat_inputs = ctx.saved_tensors
        plan = ctx.plan
        dev = cell_params.device
        g_out = g_out.contiguous().float()
        g_cell = torch.empty_like(cell_params)
        g_filt = torch.empty_like(filters)
        _lib.check(lib.nc_vnn_backward(ctypes.byref(plan.topo), _ptr(plan.buf), _ptr(cell_params),
                                       _ptr(filters), _ptr(flat_inputs), flat_inputs.shape[0],
                                       ctypes.byref(ctx.codd), _ptr(g_out), _ptr(g_cell),
                                       _ptr(g_filt), _ptr(ctx.ws), ctx.ws_bytes, _stream(dev)),
                   "nc_vnn_backward")
        _after_call(ctx.ws, "nc_vnn_backward")
        ctx.ws = None
        return g_cell, g_filt, None, None, None, None


class _VNNPropagateUniverse(torch.autograd.Function):
    """``propagate_vnn_2d(..., return_universe=True)``: (outputs, universe) through
    nc_vnn_forward_universe / nc_vnn_backward_universe."""

    @staticmethod
    def forward(ctx, cell_params, filters, flat_inputs, plan: Plan, codd: _lib.NcCodd, train: bool):
        lib = _lib.load()
        dev = cell_params.device
        B = flat_inputs.shape[0]
        H, W = plan.topo.H, plan.topo.W          # a window plan's universe is its window
        flags = _lib.NC_FLAG_TRAIN if train else 0
        ws_bytes = lib.nc_workspace_bytes(ctypes.byref(plan.topo), B, flags)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        out = torch.empty((B, plan.n_out), dtype=torch.float32, device=dev)
        uni = torch.empty((B, H, W), dtype=torch.float32, device=dev)
        _lib.check(lib.nc_vnn_forward_universe(ctypes.byref(plan.topo), _ptr(plan.buf), _ptr(cell_params),
                                               _ptr(filters), _ptr(flat_inputs), B, ctypes.byref(codd),
                                               flags, _ptr(out), _ptr(uni), _ptr(ws), ws_bytes,
                                               _stream(dev)), "nc_vnn_forward_universe")
        _after_call(ws, "nc_vnn_forward_universe")
        if train:
            ctx.save_for_backward(cell_params, filters, flat_inputs)
            ctx.ws, ctx.ws_bytes, ctx.plan, ctx.codd = ws, ws_bytes, plan, codd
        return out, uni

    @staticmethod
    def backward(ctx, g_out, g_uni):
        lib = _lib.load()
        cell_params, filters, flat_inputs = ctx.saved_tensors
        plan = ctx.plan
        dev = cell_params.device
        B = flat_inputs.shape[0]
        H, W = plan.topo.H, plan.topo.W
        g_uni = (torch.zeros((B, H, W), dtype=torch.float32, device=dev) if g_uni is None
                 else g_uni.contiguous().float())
        g_out = None if g_out is None else g_out.contiguous().float()
        g_cell = torch.empty_like(cell_params)
        g_filt = torch.empty_like(filters)
        _lib.check(lib.nc_vnn_backward_universe(ctypes.byref(plan.topo), _ptr(plan.buf), _ptr(cell_params),
                                                _ptr(filters), _ptr(flat_inputs), B, ctypes.byref(ctx.codd),
                                                _ptr(g_out), _ptr(g_uni), _ptr(g_cell), _ptr(g_filt),
                                                _ptr(ctx.ws), ctx.ws_bytes, _stream(dev)),
                   "nc_vnn_backward_universe")
        _after_call(ctx.ws, "nc_vnn_backward_universe")
        ctx.ws = None
        return g_cell, g_filt, None, None, None, None


def propagate_universe(cell_params: torch.Tensor, filters: torch.Tensor, flat_inputs: torch.Tensor,
                       plan: Plan, codd_mode: str, tau, thr):
    """(B, n_in) -> ((B, n_out), (B, H, W)); differentiable in the parameters."""
    for t, n in ((cell_params, "cell_params"), (filters, "greens_filters"), (flat_inputs, "inputs")):
        _require_cuda(t, n)
    cp = cell_params.contiguous().float()
    fl = filters.contiguous().float()
    xi = flat_inputs.contiguous().float()
    train = torch.is_grad_enabled() and (cp.requires_grad or fl.requires_grad)
    return _VNNPropagateUniverse.apply(cp, fl, xi, plan, _codd(codd_mode, tau, thr), train)


class _UniverseEmbed(torch.autograd.Function):
    """Full-grid universe of an adaptive sub-ROI call (propagator.py:700-718, 726-733)
    through nc_universe_embed_forward / nc_universe_embed_backward."""

    @staticmethod
    def forward(ctx, cell_params, uni_window, full_plan: Plan, window, codd: _lib.NcCodd):
        lib = _lib.load()
        dev = cell_params.device
        B = uni_window.shape[0]
        H, W = full_plan.topology.grid_shape
        r0, r1, c0, c1 = window
        out = torch.empty((B, full_plan.n_out), dtype=torch.float32, device=dev)
        uni = torch.empty((B, H, W), dtype=torch.float32, device=dev)
        _lib.check(lib.nc_universe_embed_forward(ctypes.byref(full_plan.topo), _ptr(full_plan.buf),
                                                 _ptr(cell_params), ctypes.byref(codd), r0, c0,
                                                 r1 - r0, c1 - c0, _ptr(uni_window), B, _ptr(uni),
                                                 _ptr(out), _stream(dev)), "nc_universe_embed_forward")
        ctx.save_for_backward(cell_params)
        ctx.plan, ctx.window, ctx.codd, ctx.B = full_plan, window, codd, B
        return out, uni

    @staticmethod
    def backward(ctx, g_out, g_uni):
        lib = _lib.load()
        (cell_params,) = ctx.saved_tensors
        plan, (r0, r1, c0, c1), B = ctx.plan, ctx.window, ctx.B
        dev = cell_params.device
        g_out = None if g_out is None else g_out.contiguous().float()
        g_uni = None if g_uni is None else g_uni.contiguous().float()
        g_win = torch.empty((B, r1 - r0, c1 - c0), dtype=torch.float32, device=dev)
        g_cell = torch.empty_like(cell_params)
        _lib.check(lib.nc_universe_embed_backward(ctypes.byref(plan.topo), _ptr(plan.buf),
                                                  _ptr(cell_params), ctypes.byref(ctx.codd), r0, c0,
                                                  r1 - r0, c1 - c0, _ptr(g_out), _ptr(g_uni), B,
                                                  _ptr(g_win), _ptr(g_cell), _stream(dev)),
                   "nc_universe_embed_backward")
        return g_cell, g_win, None, None, None


def embed_universe(cell_params: torch.Tensor, uni_window: torch.Tensor, full_plan: Plan, window,
                   codd_mode: str, tau, thr):
    """(B, win_h, win_w) window universe -> ((B, n_out), (B, H, W)) on the full chip;
    differentiable in ``cell_params`` (cells outside the window) and ``uni_window``."""
    _require_cuda(cell_params, "cell_params")
    _require_cuda(uni_window, "uni_window")
    return _UniverseEmbed.apply(cell_params.contiguous().float(), uni_window.contiguous().float(),
                                full_plan, tuple(int(v) for v in window),
                                _codd(codd_mode, tau, thr))


def propagate(cell_params: torch.Tensor, filters: torch.Tensor, flat_inputs: torch.Tensor,
              plan: Plan, codd_mode: str, tau, thr) -> torch.Tensor:
    """(B, n_in) -> (B, n_out) through the CUDA library; differentiable in the parameters."""
    for t, n in ((cell_params, "cell_params"), (filters, "greens_filters"), (flat_inputs, "inputs")):
        _require_cuda(t, n)
    cp = cell_params.contiguous().float()
    fl = filters.contiguous().float()
    xi = flat_inputs.contiguous().float()
    train = torch.is_grad_enabled() and (cp.requires_grad or fl.requires_grad)
    return _VNNPropagate.apply(cp, fl, xi, plan, _codd(codd_mode, tau, thr), train)


def workspace_status(ws: torch.Tensor) -> int:
    """Status word of a workspace (nc_workspace_status): 0 ok, 1 when a kernel of the latest
    forward on ``ws`` (or a backward after it) gave up a bounded wait for its own
    asynchronous copies, so that call's results are invalid.  Synchronises the stream."""
    out = ctypes.c_int32(-1)
    _lib.check(_lib.load().nc_workspace_status(_ptr(ws), ctypes.byref(out), _stream(ws.device)),
               "nc_workspace_status")
    return int(out.value)


# When True, every forward and backward of the autograd operators reads its workspace's
# status word afterwards and raises if a bounded wait gave up (synchronises; for tests and
# health checks).  STATUS_CHECKS counts the reads.
CHECK_WAIT_STATUS = False
STATUS_CHECKS = 0


def _after_call(ws: torch.Tensor, what: str) -> None:
    global STATUS_CHECKS
    if not CHECK_WAIT_STATUS:
        return
    STATUS_CHECKS += 1
    if workspace_status(ws) != 0:
        raise RuntimeError(f"neurocell_b200: {what}: a kernel's bounded wait for its own copies "
                           "gave up; the results of this call are invalid")


def codd_states(s_raw: torch.Tensor, io_state_mask, hard_pin_io, codd_mode, tau, thr) -> torch.Tensor:
    """Codd gating of a raw state field through ``nc_codd_states``."""
    _require_cuda(s_raw, "s_raw")
    lib = _lib.load()
    H, W = s_raw.shape
    io = np.ascontiguousarray(np.asarray(io_state_mask, dtype=np.uint8))
    t = _lib.NcTopo()
    t.H, t.W, t.kh, t.kw, t.M, t.depth = H, W, 1, 1, 1, 1
    t.n_in, t.n_out, t.hard_pin_io = 0, 1, int(hard_pin_io)
    dev = s_raw.device
    nbytes = lib.nc_plan_bytes(ctypes.byref(t))
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    zero = np.zeros(1, dtype=np.int32)
    noio = np.zeros((H, W), dtype=np.uint8)
    _lib.check(lib.nc_plan_build(ctypes.byref(t), zero.ctypes.data, zero.ctypes.data, io.ctypes.data,
                                 noio.ctypes.data, None, _ptr(buf), nbytes, _stream(dev)),
               "nc_plan_build")
    out = torch.empty((H, W), dtype=torch.float32, device=dev)
    src = s_raw.contiguous().float()
    c = _codd(codd_mode, tau, thr)
    _lib.check(lib.nc_codd_states(ctypes.byref(t), _ptr(buf), _ptr(src), ctypes.byref(c), _ptr(out),
                                  _stream(dev)), "nc_codd_states")
    return out


# ---------------------------------------------------------------------------------------
# losses and the update
# ---------------------------------------------------------------------------------------
class _MSE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, out, targets):
        lib = _lib.load()
        o = out.contiguous().float()
        y = targets.contiguous().float()
        loss = torch.empty((), dtype=torch.float32, device=o.device)
        g = torch.empty_like(o)
        _lib.check(lib.nc_mse_loss(_ptr(o), _ptr(y), o.shape[0], o.numel() // o.shape[0], _ptr(loss),
                                   _ptr(g), _stream(o.device)), "nc_mse_loss")
        ctx.save_for_backward(g)
        return loss

    @staticmethod
    def backward(ctx, gl):
        (g,) = ctx.saved_tensors
        return g * gl, None


def mse_loss(out: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """``default_mse_loss`` (trainer.py:57-61): mean squared error over every element."""
    _require_cuda(out, "out")
    return _MSE.apply(out.reshape(out.shape[0], -1), targets.reshape(out.shape[0], -1))


class _CE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels):
        lib = _lib.load()
        x = logits.contiguous().float()
        lab = labels.to(torch.int32).contiguous()
        loss = torch.empty((), dtype=torch.float32, device=x.device)
        g = torch.empty_like(x)
        _lib.check(lib.nc_softmax_ce_loss(_ptr(x), _ptr(lab), x.shape[0], x.shape[1], _ptr(loss),
                                          _ptr(g), _stream(x.device)), "nc_softmax_ce_loss")
        ctx.save_for_backward(g)
        return loss

    @staticmethod
    def backward(ctx, gl):
        (g,) = ctx.saved_tensors
        return g * gl, None


def softmax_ce_loss(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    """Mean softmax cross-entropy with integer labels over logits (B, n[, 1])."""
    _require_cuda(logits, "logits")
    return _CE.apply(logits.reshape(logits.shape[0], -1), labels.reshape(-1))


def sgd_(params: torch.Tensor, grads: torch.Tensor, lr: float) -> None:
    """In-place ``params -= lr * grads`` on the current stream."""
    _require_cuda(params, "params")
    if not params.is_contiguous() or not grads.is_contiguous():
        raise ValueError("sgd_ needs contiguous tensors")
    lib = _lib.load()
    _lib.check(lib.nc_sgd_update(_ptr(params), _ptr(grads), params.numel(), float(lr),
                                 _stream(params.device)), "nc_sgd_update")
