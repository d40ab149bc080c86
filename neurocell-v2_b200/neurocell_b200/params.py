"""VNN parameter PyTree, Codd modes and initialisers (torch tensors on the GPU).

Mirrors ``neurocell/params.py`` of shakes76/neurocell-v2:

* ``VNNParams``                 -- params.py:83-113 ((3,H,W) cell_params + OIHW filters)
* ``SUPPORTED_CODD_MODES``      -- params.py:23-28
* ``compute_codd_state_probs``  -- params.py:31-80 (evaluated by the CUDA library)
* ``init_vnn_params``           -- params.py:145-217 (same variance scaling and pinning;
  numpy's generator replaces jax.random, so draws are not bit-identical to JAX)
* ``export/import_legacy_haiku_params`` -- params.py:325-346
"""
from __future__ import annotations

from typing import NamedTuple

import numpy as np
import torch

from .topology import ChipTopology2D

STATE_ACTIVE = 0.7
STATE_SIGNAL = 0.2
STATE_ACTIVE_VALUE = 1.0
STATE_SIGNAL_VALUE = 0.0

SUPPORTED_CODD_MODES = ("continuous", "annealed", "ste_binary", "ste_ternary")


class VNNParams(NamedTuple):
    """Learnable parameters: ``cell_params`` (3,H,W) = [W, B, S_raw], ``greens_filters`` (M,1,Kh,Kw)."""
    cell_params: torch.Tensor
    greens_filters: torch.Tensor

    @property
    def weights(self) -> torch.Tensor:
        return self.cell_params[0]

    @property
    def biases(self) -> torch.Tensor:
        return self.cell_params[1]

    @property
    def states(self) -> torch.Tensor:
        return self.cell_params[2]

    @property
    def filters_ihwo(self) -> torch.Tensor:
        return self.greens_filters.permute(1, 2, 3, 0)

    def _replace_cell(self, cell):
        return VNNParams(cell, self.greens_filters)


def check_codd_mode(codd_mode: str) -> None:
    if codd_mode not in SUPPORTED_CODD_MODES:
        raise ValueError(
            f"Unsupported codd_mode '{codd_mode}'; choose from {SUPPORTED_CODD_MODES}.")


def compute_codd_state_probs(s_raw: torch.Tensor, io_state_mask, hard_pin_io: bool = False,
                             codd_mode: str = "continuous", state_temperature: float = 1.0,
                             active_threshold: float = 0.6) -> torch.Tensor:
    """Effective Codd gating probabilities on (H, W) (params.py:31-80), on the GPU."""
    check_codd_mode(codd_mode)
    from . import ops
    return ops.codd_states(s_raw, io_state_mask, hard_pin_io, codd_mode, state_temperature,
                           active_threshold)


def _truncated_normal(rng: np.random.Generator, shape, stddev: float) -> np.ndarray:
    # variance_scaling(truncated_normal): N(0, 1) truncated to [-2, 2], rescaled so the
    # truncated distribution has the requested stddev (constant 0.87962566103423978).
    out = rng.standard_normal(size=shape)
    bad = np.abs(out) > 2.0
    while bad.any():
        out[bad] = rng.standard_normal(size=int(bad.sum()))
        bad = np.abs(out) > 2.0
    return out * (stddev / 0.87962566103423978)


def init_vnn_params(rng, topology: ChipTopology2D, dtype=torch.float32, clear_outside_io=False,
                    legacy_compat: bool = True, device="cuda") -> VNNParams:
    """Initial ``VNNParams`` (params.py:145-217).  ``rng``: int seed or numpy Generator."""
    g = rng if isinstance(rng, np.random.Generator) else np.random.default_rng(int(rng))
    H, W = topology.grid_shape
    kh, kw = topology.kernel_size
    M = topology.directions
    init_scale = 1.0 / np.sqrt(topology.depth * topology.N)
    init_filter_scale = 1.0 / np.sqrt(kh * kw * M)
    states = _truncated_normal(g, (H, W), np.sqrt(init_scale / H))   # fan_in = shape[-2]
    states = 1.0 / (1.0 + np.exp(-states))
    weights = _truncated_normal(g, (H, W), np.sqrt(init_scale / H))
    if clear_outside_io:
        for port in topology.in_ports:
            c0 = port.offset[1]
            states[:, :c0 + 1] = 0.0
            weights[:, :c0 + 1] = 0.0
        out_c = topology.out_port.offset[1]
        states[:, out_c:] = 0.0
        weights[:, out_c:] = 0.0
    states = np.where(topology.io_state_mask, STATE_ACTIVE_VALUE, states)
    weights = np.where(topology.io_state_mask, 1.0, weights)
    biases = np.zeros((H, W))
    cell = np.stack([weights, biases, states]).astype(np.float32)
    # fan_in of the (1, kh, kw, M) filter tensor is 1*kh*kw
    f = _truncated_normal(g, (1, kh, kw, M), np.sqrt(init_filter_scale / (kh * kw)))
    filt = np.transpose(f, (3, 0, 1, 2)).astype(np.float32)
    return VNNParams(torch.tensor(cell, dtype=dtype, device=device),
                     torch.tensor(np.ascontiguousarray(filt), dtype=dtype, device=device))


def export_legacy_haiku_params(params: VNNParams, module_name: str = "universe_lp") -> dict:
    """{'universe_lp': {'w','b','s','f'}} (params.py:325-336)."""
    return {module_name: {"w": params.weights, "b": params.biases, "s": params.states,
                          "f": params.filters_ihwo}}


def import_legacy_haiku_params(hk_params: dict, module_name: str = "universe_lp") -> VNNParams:
    """Inverse of :func:`export_legacy_haiku_params` (params.py:339-346)."""
    sub = hk_params[module_name]
    as_t = lambda v: v if isinstance(v, torch.Tensor) else torch.as_tensor(np.asarray(v))
    cell = torch.stack([as_t(sub["w"]), as_t(sub["b"]), as_t(sub["s"])], dim=0)
    filt = as_t(sub["f"]).permute(3, 0, 1, 2).contiguous()
    return VNNParams(cell.contiguous(), filt)
