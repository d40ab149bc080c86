"""neurocell_b200 -- B200-native (sm_100a) VNN propagation hot path.

Public API mirrors the reference package ``neurocell`` for the propagation path:
topology, parameters, Codd modes, ``propagate_vnn_2d`` and the ``VonNeumannNetwork``
facade.  All compute runs in ``libneurocell_b200.so`` (C ABI: include/neurocell_b200.h).
"""
from .topology import PortSpec, CoordinatePortSpec, ChipTopology2D
from .params import (
    STATE_ACTIVE, STATE_SIGNAL, STATE_ACTIVE_VALUE, STATE_SIGNAL_VALUE, SUPPORTED_CODD_MODES,
    VNNParams, compute_codd_state_probs, init_vnn_params, export_legacy_haiku_params,
    import_legacy_haiku_params,
)
from .propagator import SUPPORTED_BACKENDS, select_optimal_backend, propagate_vnn_2d
from .model import VonNeumannNetwork
from .adaptive_mask import AdaptiveMaskSpec, compute_adaptive_spatial_mask, estimate_effective_filter_radii
from .trainer import (VNNTrainer, VNNTrainStep, compute_annealed_temperature, default_mse_loss,
                      default_exact_match_metric, packbits_u8_on_device)
from . import filters, ops
from .filters import apply_spatial_filter_2d
from ._lib import load as load_library, LIB_PATH

__all__ = [
    "PortSpec", "CoordinatePortSpec", "ChipTopology2D", "STATE_ACTIVE", "STATE_SIGNAL",
    "STATE_ACTIVE_VALUE", "STATE_SIGNAL_VALUE", "SUPPORTED_CODD_MODES", "VNNParams",
    "compute_codd_state_probs", "init_vnn_params", "export_legacy_haiku_params",
    "import_legacy_haiku_params", "SUPPORTED_BACKENDS", "select_optimal_backend",
    "propagate_vnn_2d", "VonNeumannNetwork", "VNNTrainer", "compute_annealed_temperature",
    "default_mse_loss", "ops", "load_library", "LIB_PATH", "AdaptiveMaskSpec",
    "compute_adaptive_spatial_mask", "estimate_effective_filter_radii", "VNNTrainStep",
    "default_exact_match_metric", "packbits_u8_on_device", "filters", "apply_spatial_filter_2d",
]
