"""``VonNeumannNetwork`` facade (mirrors ``neurocell/model.py:29-227``).

Same constructor options, ``init`` / ``apply`` / ``effective_states`` /
``threshold_states`` / npz checkpoint API; ``apply`` runs the B200 propagation path.
"""
from __future__ import annotations

import numpy as np
import torch

from . import filters
from .params import VNNParams, compute_codd_state_probs, init_vnn_params
from .propagator import propagate_vnn_2d
from .topology import ChipTopology2D


class VonNeumannNetwork:
    def __init__(self, topology: ChipTopology2D, activate=torch.tanh, final_activate=None,
                 norm: bool = True, sharpen: bool = False, gated_filters: bool = False,
                 hard_pin_io: bool = False, backend: str = "b200", dtype=torch.float32,
                 codd_mode: str = "continuous", state_temperature: float = 1.0,
                 active_threshold: float = 0.6):
        self.topology = topology
        self.activate = activate
        self.final_activate = final_activate
        self.norm = norm
        self.sharpen = sharpen
        self.gated_filters = gated_filters
        self.hard_pin_io = hard_pin_io
        self.backend = backend
        self.dtype = dtype
        self.codd_mode = codd_mode
        self.state_temperature = state_temperature
        self.active_threshold = active_threshold
        # model.py:65-66: the normalised 3x3 sharpen stencil, applied to W in propagate_vnn_2d
        self.sharpen_filter = filters.sharpen(norm=True) if sharpen else None

    def init(self, rng, clear_outside_io: bool = False, legacy_compat: bool = True,
             device="cuda") -> VNNParams:
        return init_vnn_params(rng, self.topology, dtype=self.dtype,
                               clear_outside_io=clear_outside_io, legacy_compat=legacy_compat,
                               device=device)

    def compute_spatial_mask(self, params: VNNParams, margin=4, bucket_multiple: int = 8,
                             prev_mask=None, **kwargs):
        """The pre-epoch adaptive sub-ROI (model.py:84-103 -> adaptive_mask.py:318-481)."""
        from .adaptive_mask import compute_adaptive_spatial_mask
        return compute_adaptive_spatial_mask(params=params, topology=self.topology, margin=margin,
                                             bucket_multiple=bucket_multiple, prev_mask=prev_mask,
                                             **kwargs)

    def apply(self, params: VNNParams, inputs, return_universe: bool = False, spatial_mask=None,
              codd_mode: str | None = None, state_temperature=None, active_threshold=None):
        return propagate_vnn_2d(
            params=params, inputs=inputs, topology=self.topology, activate=self.activate,
            final_activate=self.final_activate, norm=self.norm, sharpen_filter=self.sharpen_filter,
            gated_filters=self.gated_filters, hard_pin_io=self.hard_pin_io, backend=self.backend,
            return_universe=return_universe, spatial_mask=spatial_mask,
            codd_mode=self.codd_mode if codd_mode is None else codd_mode,
            state_temperature=self.state_temperature if state_temperature is None else state_temperature,
            active_threshold=self.active_threshold if active_threshold is None else active_threshold)

    __call__ = apply

    def effective_states(self, params: VNNParams, codd_mode=None, state_temperature=None,
                         active_threshold=None) -> torch.Tensor:
        return compute_codd_state_probs(
            s_raw=params.states, io_state_mask=self.topology.io_state_mask,
            hard_pin_io=self.hard_pin_io,
            codd_mode=self.codd_mode if codd_mode is None else codd_mode,
            state_temperature=self.state_temperature if state_temperature is None else state_temperature,
            active_threshold=self.active_threshold if active_threshold is None else active_threshold)

    @staticmethod
    def threshold_states(states_raw: torch.Tensor, active_threshold: float = 0.6) -> torch.Tensor:
        """Discrete Codd roles {0, 1, 2} (model.py:185-195)."""
        s = torch.where(states_raw >= active_threshold, torch.full_like(states_raw, 2.0), states_raw)
        return torch.where((s > 0.0) & (s < active_threshold), torch.ones_like(s), s)

    def save_checkpoint(self, filename: str, params: VNNParams, **extra_metadata):
        """npz with the legacy keys weights/biases/states/filters(IHWO) (model.py:197-215)."""
        cpu = lambda t: t.detach().float().cpu().numpy()
        np.savez(filename, weights=cpu(params.weights), biases=cpu(params.biases),
                 states=cpu(params.states), filters=cpu(params.filters_ihwo),
                 N=self.topology.N, depth=self.topology.depth,
                 kernel_size=np.asarray(self.topology.kernel_size),
                 directions=self.topology.directions, allow_pickle=False, **extra_metadata)

    @staticmethod
    def load_checkpoint(filename: str, device="cuda") -> VNNParams:
        """Loads an npz checkpoint into packed ``VNNParams`` (model.py:217-227)."""
        with np.load(filename, allow_pickle=False) as d:
            cell = np.stack([d["weights"], d["biases"], d["states"]]).astype(np.float32)
            filt = np.ascontiguousarray(np.transpose(d["filters"], (3, 0, 1, 2))).astype(np.float32)
        return VNNParams(torch.tensor(cell, device=device), torch.tensor(filt, device=device))
