"""Minimal training / evaluation engine around the B200 propagation path.

Mirrors the parts of ``neurocell/trainer.py`` that drive the hot path:
``compute_annealed_temperature`` (trainer.py:23-46), ``default_mse_loss`` (57-61),
``default_exact_match_metric`` (64-69), ``packbits_u8_on_device`` (49-54) and a
``VNNTrainer`` whose steps are value_and_grad + SGD (trainer.py:101-106 with optax.sgd),
with the reference's epoch, evaluation, adaptive sub-ROI, annealed-temperature and
multi-epoch entry points (trainer.py:108-156, 164-268, 270-356, 358-398).  The
``lax.scan`` programs become either an eager loop over the library's operators
(``VNNTrainer``) or one CUDA graph per step or per epoch (``VNNTrainStep``).  Optimizers
other than SGD are not part of the B200 hot path.
"""
from __future__ import annotations

import math

import torch

from . import ops
from .params import VNNParams


def compute_annealed_temperature(epoch: int, total_epochs: int, init_temp: float = 1.0,
                                 final_temp: float = 0.1, schedule: str = "exponential") -> float:
    if total_epochs <= 1:
        return float(final_temp)
    progress = min(1.0, max(0.0, float(epoch) / float(total_epochs - 1)))
    if schedule == "exponential":
        return float(init_temp * ((final_temp / init_temp) ** progress))
    if schedule == "cosine":
        return float(final_temp + (init_temp - final_temp) * 0.5 * (1.0 + math.cos(math.pi * progress)))
    if schedule == "linear":
        return float(init_temp + (final_temp - init_temp) * progress)
    raise ValueError(
        f"Unsupported temperature schedule '{schedule}'; choose from ('exponential', 'cosine', 'linear').")


def default_mse_loss(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean squared error (trainer.py:57-61), evaluated by the CUDA library."""
    return ops.mse_loss(logits, targets)


def default_exact_match_metric(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Rounded exact-match accuracy (trainer.py:64-69)."""
    if logits.ndim == 3 and logits.shape[-1] == 1 and targets.ndim == 2:
        logits = logits[..., 0]
    return (torch.round(logits) == torch.round(targets.to(logits.dtype))).float().mean()


def softmax_cross_entropy_loss(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return ops.softmax_ce_loss(logits, labels)


BIT_WEIGHTS_U8 = (128, 64, 32, 16, 8, 4, 2, 1)


def packbits_u8_on_device(bits: torch.Tensor) -> torch.Tensor:
    w = torch.tensor(BIT_WEIGHTS_U8, dtype=torch.int32, device=bits.device)
    return (bits.to(torch.int32) * w).sum(-1, keepdim=True).to(torch.uint8)


def allreduce_mean_(flat: torch.Tensor, process_group=None) -> int:
    """Data-parallel gradient exchange: sums ``flat`` over the ranks of ``process_group`` in
    place (one collective over the packed [g_cell | g_filters] buffer) and returns the world
    size, so the caller scales the update by 1/world.  Every rank computed the gradient of
    its own mean loss over an equal-sized shard, so (sum over ranks) / world is the gradient
    of the mean loss over the global batch.  No-op for a single process."""
    if process_group is None:
        return 1
    import torch.distributed as dist
    world = dist.get_world_size(process_group)
    if world > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=process_group)
    return world


class NVLinkExchange:
    """Gradient sum over the ranks of a process group fused with the SGD update, one kernel
    over NVLink peer memory (``nc_dp_allreduce_sgd``).

    Each rank allocates a double-buffered receive buffer (one slot per rank), the ranks swap
    CUDA IPC handles with one ``all_gather_object`` and map each other's buffers.  Every step
    each rank's kernel stores its gradient into every peer's buffer, each value in one 64-bit
    element together with the step number, waits (bounded by ``max_wait_iters`` polls of its
    own buffer) until the same slices of all peers carry this step's tag, sums them in rank
    order from local memory (bitwise the same on every rank) and applies
    ``params -= lr / world * sum``.  One process per GPU; ranks on one GPU are rejected,
    because kernels that wait on one another cannot share a device.  A timeout is terminal
    (``status()`` reads 1 and later exchanges do nothing) until every rank calls ``reset()``.
    ``close()`` unmaps and frees the buffers (collective: every rank calls it).
    """

    def __init__(self, n: int, process_group, device, max_wait_iters: int = 1 << 24):
        import ctypes
        import torch.distributed as dist
        from . import _lib
        self.lib = _lib.load()
        self._lib = _lib
        self.ctypes = ctypes
        self.pg = process_group
        self.n = int(n)
        self.world = dist.get_world_size(process_group)
        self.rank = dist.get_rank(process_group)
        self.max_wait = int(max_wait_iters)
        if not 1 <= self.world <= _lib.NC_DP_MAX_RANKS:
            raise ValueError(f"NVLink exchange supports 1..{_lib.NC_DP_MAX_RANKS} ranks, "
                             f"got {self.world}")
        dev = torch.device(device)
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        uuids = [None] * self.world
        dist.all_gather_object(uuids, uuid, group=process_group)
        if len(set(uuids)) != self.world:
            raise ValueError("NVLink exchange needs one GPU per rank (two ranks share a device)")
        self.shared = ctypes.c_void_p()
        self.state = ctypes.c_void_p()
        with torch.cuda.device(dev):
            _lib.check(self.lib.nc_dp_alloc(self.lib.nc_dp_shared_bytes(self.n, self.world),
                                            ctypes.byref(self.shared)), "nc_dp_alloc")
            _lib.check(self.lib.nc_dp_alloc(self.lib.nc_dp_state_bytes(), ctypes.byref(self.state)),
                       "nc_dp_alloc")
            handle = ctypes.create_string_buffer(_lib.NC_IPC_HANDLE_BYTES)
            _lib.check(self.lib.nc_ipc_get(self.shared, handle), "nc_ipc_get")
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=process_group)
            self.peers = (ctypes.c_void_p * self.world)()
            self._opened = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    self.peers[r] = self.shared.value
                    continue
                p = ctypes.c_void_p()
                _lib.check(self.lib.nc_ipc_open(ctypes.create_string_buffer(h, len(h)),
                                                ctypes.byref(p)), "nc_ipc_open")
                self.peers[r] = p.value
                self._opened.append(p)
        self.device = dev
        self.closed = False

    def allreduce_sgd(self, grads_ptr: int, params_ptr: int, lr: float, stream) -> None:
        """``stream``: a ``ctypes.c_void_p`` holding the cudaStream_t to launch on."""
        if self.closed:
            raise RuntimeError("NVLinkExchange is closed")
        c = self.ctypes
        self._lib.check(self.lib.nc_dp_allreduce_sgd(self.peers, self.world, self.rank, self.state,
                                                     c.c_void_p(grads_ptr), c.c_void_p(params_ptr),
                                                     self.n, float(lr), self.max_wait, stream),
                        "nc_dp_allreduce_sgd")

    def status(self) -> int:
        """0 = every exchange so far completed; 1 = a peer timed out.  Slices whose peers had
        arrived in that step were updated and the others were not, so the ranks' parameters
        no longer agree; later exchanges do nothing until ``reset()``.  Synchronises."""
        c = self.ctypes
        out = c.c_int32(-1)
        self._lib.check(self.lib.nc_dp_status(self.state, c.byref(out),
                                              c.c_void_p(torch.cuda.current_stream(self.device)
                                                         .cuda_stream)), "nc_dp_status")
        return int(out.value)

    def reset(self) -> None:
        """Clears the step counters, the status word and this rank's receive buffer, then
        passes a barrier of the process group (collective: every rank calls it, with no
        exchange in flight).  Restore consistent parameters before the next step."""
        if self.closed:
            raise RuntimeError("NVLinkExchange is closed")
        import torch.distributed as dist
        c = self.ctypes
        torch.cuda.synchronize(self.device)
        self._lib.check(self.lib.nc_dp_reset(self.state, self.shared,
                                             self.lib.nc_dp_shared_bytes(self.n, self.world),
                                             c.c_void_p(torch.cuda.current_stream(self.device)
                                                        .cuda_stream)), "nc_dp_reset")
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.pg)

    def close(self) -> None:
        if self.closed:
            return
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self._lib.check(self.lib.nc_ipc_close(p), "nc_ipc_close")
        self._opened = []
        dist.barrier(group=self.pg)       # no peer reads this rank's buffer any more
        self._lib.check(self.lib.nc_dp_free(self.shared), "nc_dp_free")
        self._lib.check(self.lib.nc_dp_free(self.state), "nc_dp_free")
        self.closed = True


class VNNTrainStep:
    """One fused training step over static device buffers: forward, loss, backward,
    optional data-parallel gradient exchange, SGD update.

    Parameters live in one packed device buffer ``[cell_params (3HW) | filters (MK)]`` and
    gradients in a second one, so the data-parallel exchange moves 3HW+MK floats (16,316
    for the ALU chip).  ``exchange`` picks how, when ``process_group`` spans several ranks:
    ``"nccl"`` all-reduces the packed gradient with the process group and then runs the SGD
    kernel; ``"nvlink"`` runs one kernel that sums the ranks' gradients over NVLink peer
    memory and applies SGD (:class:`NVLinkExchange`).  ``step(x, y)`` copies the batch into
    the static input buffers and returns the loss.  Page-locked host batches are read by one
    staging kernel (``nc_stage_from_host``) instead of two copy-engine transfers (each costs
    about 9 us on the GPU timeline at these sizes); other host tensors go through
    ``copy_``.  With ``host_loss=True`` the loss kernel writes the loss straight into a
    page-locked host scalar, returned by ``step()`` and valid once the stream has reached
    the end of the step (``torch.cuda.synchronize()`` or an event); otherwise ``step()``
    returns the device loss.  ``capture()`` records the launch sequence into a CUDA graph.
    Every kernel of the step except NCCL's comes from ``libneurocell_b200.so``.
    """

    def __init__(self, topology, params: VNNParams, batch_size: int, lr: float = 1e-2,
                 loss: str = "mse", activate=torch.tanh, final_activate=None, norm: bool = True,
                 hard_pin_io: bool = False, gated_filters: bool = False,
                 codd_mode: str = "continuous", state_temperature: float = 1.0,
                 active_threshold: float = 0.6, in_shapes=None, process_group=None,
                 exchange: str = "nccl", conv: str = "auto", spatial_mask=None,
                 host_loss: bool = False):
        import ctypes
        from . import _lib
        from .params import check_codd_mode
        check_codd_mode(codd_mode)
        if loss not in ("mse", "ce"):
            raise ValueError(f"Unsupported loss '{loss}'; choose from ('mse', 'ce').")
        if exchange not in ("nccl", "nvlink"):
            raise ValueError(f"Unsupported exchange '{exchange}'; choose from ('nccl', 'nvlink').")
        dev = params.cell_params.device
        ops._require_cuda(params.cell_params, "params.cell_params")
        if not topology.out_in_roi:
            raise NotImplementedError("VNNTrainStep needs output ports inside the ROI; use "
                                      "propagate_vnn_2d (full-grid path) with VNNTrainer")
        act, slope = ops.resolve_activation(activate)
        fact, fslope = ops.resolve_activation(final_activate)
        if in_shapes is None:
            in_shapes = tuple(tuple(p.size) if not hasattr(p, "num_points") else (p.num_points,)
                              for p in topology.in_ports)
        roi_bbox = None
        if (spatial_mask is not None and not spatial_mask.is_full_roi
                and topology.padding_mode != "CIRCULAR"):
            roi_bbox = tuple(int(v) for v in spatial_mask.roi_bbox)
        self.plan = ops.get_plan(topology, tuple(in_shapes), dev, act, slope, fact, fslope, norm,
                                 hard_pin_io, gated_filters, conv, roi_bbox)
        self.window = self.plan.window
        self.lib = _lib.load()
        self._lib = _lib
        self.ctypes = ctypes
        self.device = dev
        self.B = int(batch_size)
        self.lr = float(lr)
        self.loss_kind = loss
        self.pg = process_group
        self.world = 1
        if process_group is not None:
            import torch.distributed as dist
            self.world = dist.get_world_size(process_group)
        cell = params.cell_params.detach()
        self._full_cell = None
        if self.window is not None:
            # adaptive sub-ROI (trainer.py:164-268): the step trains the window's cells; the
            # cells outside it get no gradient and keep their values in the full copy
            r0, r1, c0, c1 = self.window
            self._full_cell = cell.to(torch.float32).clone()
            cell = self._full_cell[:, r0:r1, c0:c1]
        self.n_cell = int(cell.numel())
        self.n_filt = int(params.greens_filters.numel())
        self.flat = torch.empty(self.n_cell + self.n_filt, dtype=torch.float32, device=dev)
        self.flat[: self.n_cell].copy_(cell.reshape(-1))
        self.flat[self.n_cell:].copy_(params.greens_filters.reshape(-1))
        self.grads = torch.zeros_like(self.flat)
        self._cell_view = self.flat[: self.n_cell].view(tuple(cell.shape))
        self._filt_view = self.flat[self.n_cell:].view(params.greens_filters.shape)
        self.ws_bytes = self.lib.nc_workspace_bytes(ctypes.byref(self.plan.topo), self.B,
                                                    _lib.NC_FLAG_TRAIN)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.x = torch.zeros((self.B, self.plan.n_in), dtype=torch.float32, device=dev)
        if loss == "mse":
            self.y = torch.zeros((self.B, self.plan.n_out), dtype=torch.float32, device=dev)
        else:
            self.y = torch.zeros((self.B,), dtype=torch.int32, device=dev)
        self.out = torch.empty((self.B, self.plan.n_out), dtype=torch.float32, device=dev)
        self.g_out = torch.empty_like(self.out)
        self.loss = torch.zeros((), dtype=torch.float32, device=dev)
        # host_loss: the loss kernel stores into this page-locked scalar (device-mapped)
        self.loss_host = torch.zeros((), dtype=torch.float32).pin_memory() if host_loss else None
        self._stage = (_lib.NcStageSeg * 2)()
        self.codd = ops._codd(codd_mode, state_temperature, active_threshold)
        # tau lives on the device so captured graphs replay with the current temperature
        self.tau_dev = torch.full((1,), float(state_temperature), dtype=torch.float32, device=dev)
        self.codd.temperature_dev = self.tau_dev.data_ptr()
        self.graph = None
        self.epoch_graph = None
        # (start, stop) torch.cuda.Event pair recorded around the gradient exchange of eager
        # steps (timing only; a captured graph does not record them)
        self.exchange_events = None
        self.exchange = None
        if exchange == "nvlink" and self.world > 1:
            self.exchange = NVLinkExchange(self.n_cell + self.n_filt, process_group, dev)
        self._launches = None

    @property
    def params(self) -> VNNParams:
        """The trained parameters, full (3, H, W) cells and filters.  With a sub-ROI the
        window's cells are written into the full copy first (stream-ordered)."""
        if self.window is None:
            return VNNParams(self._cell_view, self._filt_view)
        r0, r1, c0, c1 = self.window
        self._full_cell[:, r0:r1, c0:c1].copy_(self._cell_view)
        return VNNParams(self._full_cell, self._filt_view)

    def launches_per_step(self) -> int:
        """Kernels ``libneurocell_b200.so`` launches per step, counted by the library while
        the step is captured (or, before ``capture()``, while one eager step runs)."""
        if self._launches is None:
            raise RuntimeError("run step() or capture() once before asking for the launch count")
        return self._launches

    def set_temperature(self, tau: float) -> None:
        """Codd temperature of the following steps (annealed and STE modes).  Stream-ordered
        device write, so it also reaches steps and epochs already captured as CUDA graphs."""
        self.codd.temperature = float(tau)
        self.tau_dev.fill_(float(tau))

    def _launch(self, loss_out: torch.Tensor | None = None) -> None:
        c, lib, P = self.ctypes, self.lib, ops._ptr
        loss_t = loss_out if loss_out is not None else (self.loss_host if self.loss_host is not None
                                                          else self.loss)
        st = ops._stream(self.device)
        n0 = lib.nc_launch_count()
        t = c.byref(self.plan.topo)
        cell = self.flat.data_ptr()
        filt = cell + 4 * self.n_cell
        gcell = self.grads.data_ptr()
        gfilt = gcell + 4 * self.n_cell
        self._lib.check(lib.nc_vnn_forward(t, P(self.plan.buf), c.c_void_p(cell), c.c_void_p(filt),
                                           P(self.x), self.B, c.byref(self.codd),
                                           self._lib.NC_FLAG_TRAIN, P(self.out), P(self.ws),
                                           self.ws_bytes, st), "nc_vnn_forward")
        if self.loss_kind == "mse":
            self._lib.check(lib.nc_mse_loss(P(self.out), P(self.y), self.B, self.plan.n_out,
                                            P(loss_t), P(self.g_out), st), "nc_mse_loss")
        else:
            self._lib.check(lib.nc_softmax_ce_loss(P(self.out), P(self.y), self.B, self.plan.n_out,
                                                   P(loss_t), P(self.g_out), st),
                            "nc_softmax_ce_loss")
        self._lib.check(lib.nc_vnn_backward(t, P(self.plan.buf), c.c_void_p(cell), c.c_void_p(filt),
                                            P(self.x), self.B, c.byref(self.codd), P(self.g_out),
                                            c.c_void_p(gcell), c.c_void_p(gfilt), P(self.ws),
                                            self.ws_bytes, st), "nc_vnn_backward")
        timed = self.exchange_events is not None and not torch.cuda.is_current_stream_capturing()
        if timed:
            self.exchange_events[0].record()
        if self.exchange is not None:
            # sum over ranks + params -= lr / world * sum, in one kernel over NVLink
            self.exchange.allreduce_sgd(gcell, cell, self.lr, st)
        else:
            world = allreduce_mean_(self.grads, self.pg)
            lr = self.lr / world            # mean of the per-rank mean-loss gradients
            self._lib.check(lib.nc_sgd_update(c.c_void_p(cell), c.c_void_p(gcell),
                                              self.n_cell + self.n_filt, lr, st), "nc_sgd_update")
        if timed:
            self.exchange_events[1].record()
        self._launches = int(lib.nc_launch_count() - n0)

    def load_batch(self, x: torch.Tensor, y: torch.Tensor) -> None:
        if (not x.is_cuda and not y.is_cuda and x.dtype == self.x.dtype and y.dtype == self.y.dtype
                and x.numel() == self.x.numel() and y.numel() == self.y.numel()
                and x.is_contiguous() and y.is_contiguous() and x.is_pinned() and y.is_pinned()):
            # page-locked host batch: one staging kernel reads both tensors
            sg = self._stage
            sg[0].dst, sg[0].src, sg[0].bytes = self.x.data_ptr(), x.data_ptr(), 4 * x.numel()
            sg[1].dst, sg[1].src, sg[1].bytes = self.y.data_ptr(), y.data_ptr(), 4 * y.numel()
            self._lib.check(self.lib.nc_stage_from_host(sg, 2, ops._stream(self.device)),
                            "nc_stage_from_host")
            return
        self.x.copy_(x.reshape(self.B, -1), non_blocking=True)
        self.y.copy_(y.reshape(self.y.shape), non_blocking=True)

    def step(self, x: torch.Tensor | None = None, y: torch.Tensor | None = None) -> torch.Tensor:
        if x is not None:
            self.load_batch(x, y)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._launch()
        return self.loss if self.loss_host is None else self.loss_host

    def capture(self) -> None:
        """Records one step into a CUDA graph (the gradient exchange included when data
        parallel; call ``release()`` before destroying the process group)."""
        if self.exchange is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.pg)      # ranks enter the first exchange together
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        saved = self.flat.clone()
        with torch.cuda.stream(s):
            for _ in range(2):
                self._launch()
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._launch()
        self.flat.copy_(saved)             # warm-up and capture must not move the parameters
        self.graph = g

    def exchange_status(self) -> int:
        """Status word of the NVLink exchange (0 ok, 1 a peer timed out); 0 without one."""
        return 0 if self.exchange is None else self.exchange.status()

    def capture_epoch(self, x_epoch: torch.Tensor, y_epoch: torch.Tensor) -> None:
        """Records a whole epoch as one CUDA graph (the reference's ``lax.scan`` epoch,
        trainer.py:108-119): for every batch i of the device-resident ``x_epoch``
        (n_batches, B, ...) / ``y_epoch`` the graph copies the batch into the step's static
        buffers, trains one step and writes that step's loss to ``epoch_losses[i]``.
        ``train_epoch()`` then replays the epoch with a single launch from the host."""
        if x_epoch.device != self.device or y_epoch.device != self.device:
            raise ValueError("capture_epoch needs device-resident batches")
        nb = int(x_epoch.shape[0])
        xs = x_epoch.reshape(nb, self.B, -1)
        ys = y_epoch.reshape((nb,) + tuple(self.y.shape))
        self.epoch_losses = torch.zeros(nb, dtype=torch.float32, device=self.device)
        if self.exchange is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.pg)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        saved = self.flat.clone()
        with torch.cuda.stream(s):
            for i in range(min(nb, 2)):      # warm-up (kernel attributes, lazy loading)
                self.x.copy_(xs[i])
                self.y.copy_(ys[i])
                self._launch(self.epoch_losses[i])
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(nb):
                self.x.copy_(xs[i])
                self.y.copy_(ys[i])
                self._launch(self.epoch_losses[i])
        self.flat.copy_(saved)
        self.epoch_graph = g
        self._epoch_src = (xs, ys)           # the graph reads these buffers

    def train_epoch(self) -> torch.Tensor:
        """Replays the captured epoch; returns the per-step losses (device tensor).  The
        reference's epoch loss is ``epoch_losses.sum() / batch_size``."""
        if getattr(self, "epoch_graph", None) is None:
            raise RuntimeError("call capture_epoch() first")
        self.epoch_graph.replay()
        return self.epoch_losses

    def release(self) -> None:
        """Drops the captured graph and unmaps the NVLink exchange buffers (collective when
        data parallel; required before destroy_process_group)."""
        self.graph = None
        self.epoch_graph = None
        if self.exchange is not None:
            self.exchange.close()


class VNNTrainer:
    """value_and_grad + SGD over ``apply_fn`` (trainer.py:71-106, optimizer = SGD(lr)).

    ``apply_fn(params, batch_x, **kw)`` is ``VonNeumannNetwork.apply`` or a closure over
    ``propagate_vnn_2d``; the adaptive and annealed entry points pass ``spatial_mask``,
    ``codd_mode`` and ``state_temperature`` through it as the reference does."""

    def __init__(self, apply_fn, lr: float = 1e-2, batch_size: int = 128, loss_fn=None,
                 eval_metric_fn=None):
        self.apply_fn = apply_fn
        self.lr = float(lr)
        self.batch_size = batch_size
        self.loss_fn = loss_fn or default_mse_loss
        self.eval_metric_fn = eval_metric_fn or default_exact_match_metric

    def value_and_grad(self, params: VNNParams, batch_x, batch_y, **apply_kw):
        cp = params.cell_params.detach().requires_grad_(True)
        fl = params.greens_filters.detach().requires_grad_(True)
        out = self.apply_fn(VNNParams(cp, fl), batch_x, **apply_kw)
        loss = self.loss_fn(out, batch_y)
        g_cp, g_fl = torch.autograd.grad(loss, (cp, fl))
        return loss.detach(), VNNParams(g_cp, g_fl)

    def train_step(self, params: VNNParams, batch_x, batch_y, **apply_kw):
        """Returns ``(new_params, loss)``; the update runs in place on ``params``' storage."""
        loss, grads = self.value_and_grad(params, batch_x, batch_y, **apply_kw)
        with torch.no_grad():
            ops.sgd_(params.cell_params, grads.cell_params, self.lr)
            ops.sgd_(params.greens_filters, grads.greens_filters, self.lr)
        return params, loss

    def train_epoch(self, params: VNNParams, x_epoch, y_epoch, **apply_kw):
        """Steps over the batches of ``x_epoch`` / ``y_epoch`` in order (trainer.py:108-119);
        returns ``(params, epoch_loss)`` with epoch_loss = sum of the batch losses /
        batch_size, as the reference reports it."""
        total = None
        for bx, by in zip(x_epoch, y_epoch):
            params, loss = self.train_step(params, bx, by, **apply_kw)
            total = loss if total is None else total + loss
        return params, total / float(self.batch_size)

    @torch.no_grad()
    def evaluate_packed(self, params: VNNParams, x_batches, y_packed_batches, **apply_kw):
        """Packed 8-bit exact-match accuracy (trainer.py:122-138)."""
        acc = 0.0
        preds = []
        for bx, by in zip(x_batches, y_packed_batches):
            logits = self.apply_fn(params, bx, **apply_kw)
            if logits.ndim == 3 and logits.shape[-1] == 1:
                logits = logits[..., 0]
            p = packbits_u8_on_device(torch.round(logits).clamp(0, 255).to(torch.uint8))
            acc += float((p.reshape(by.shape) == by).float().mean())
            preds.append(p)
        return acc / max(1, len(preds)), preds

    @torch.no_grad()
    def evaluate_metric(self, params: VNNParams, x_batches, y_batches, **apply_kw):
        """Mean of ``eval_metric_fn`` over the batches (trainer.py:140-153)."""
        total, n = 0.0, 0
        for bx, by in zip(x_batches, y_batches):
            total += float(self.eval_metric_fn(self.apply_fn(params, bx, **apply_kw), by))
            n += 1
        return total / max(1, n)

    # adaptive sub-ROI entry points (trainer.py:164-268); the library's plan cache keys the
    # sub-ROI windows by roi_bbox, as the reference caches one executable per bucket
    @staticmethod
    def _mask_kw(mask_spec) -> dict:
        return {} if mask_spec is None or mask_spec.is_full_roi else {"spatial_mask": mask_spec}

    def train_step_adaptive(self, params: VNNParams, batch_x, batch_y, mask_spec):
        return self.train_step(params, batch_x, batch_y, **self._mask_kw(mask_spec))

    def train_epoch_adaptive(self, params: VNNParams, x_epoch, y_epoch, mask_spec):
        return self.train_epoch(params, x_epoch, y_epoch, **self._mask_kw(mask_spec))

    def evaluate_packed_adaptive(self, params: VNNParams, x_batches, y_packed_batches, mask_spec):
        return self.evaluate_packed(params, x_batches, y_packed_batches, **self._mask_kw(mask_spec))

    def evaluate_metric_adaptive(self, params: VNNParams, x_batches, y_batches, mask_spec):
        return self.evaluate_metric(params, x_batches, y_batches, **self._mask_kw(mask_spec))

    # dynamic temperature and Codd mode (trainer.py:270-356): tau is a plain argument of
    # the library call, nothing is recompiled when it changes
    def train_step_annealed(self, params: VNNParams, batch_x, batch_y,
                            state_temperature: float = 1.0, codd_mode: str = "annealed",
                            mask_spec=None):
        return self.train_step(params, batch_x, batch_y, codd_mode=codd_mode,
                               state_temperature=float(state_temperature), **self._mask_kw(mask_spec))

    def train_epoch_annealed(self, params: VNNParams, x_epoch, y_epoch,
                             state_temperature: float = 1.0, codd_mode: str = "annealed",
                             mask_spec=None):
        return self.train_epoch(params, x_epoch, y_epoch, codd_mode=codd_mode,
                                state_temperature=float(state_temperature), **self._mask_kw(mask_spec))

    def train_epochs(self, params: VNNParams, x_train: torch.Tensor, y_train: torch.Tensor, rng,
                     num_epochs: int):
        """``num_epochs`` epochs with an on-device shuffle at every epoch boundary
        (trainer.py:358-398): a device permutation of the samples, truncated to whole
        batches.  ``rng``: int seed or ``torch.Generator`` on the data's device.  Returns
        ``(params, epoch_losses)`` with one device scalar per epoch."""
        dev = x_train.device
        gen = rng if isinstance(rng, torch.Generator) else torch.Generator(dev).manual_seed(int(rng))
        n = int(x_train.shape[0])
        steps = n // self.batch_size
        usable = steps * self.batch_size
        losses = []
        for _ in range(int(num_epochs)):
            perm = torch.randperm(n, generator=gen, device=dev)[:usable]
            xe = x_train[perm].reshape((steps, self.batch_size) + tuple(x_train.shape[1:]))
            ye = y_train[perm].reshape((steps, self.batch_size) + tuple(y_train.shape[1:]))
            params, ep = self.train_epoch(params, xe, ye)
            losses.append(ep)
        return params, torch.stack(losses) if losses else torch.zeros(0, device=dev)
