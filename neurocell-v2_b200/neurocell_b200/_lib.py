"""ctypes binding of ``libneurocell_b200.so`` (declarations: ``include/neurocell_b200.h``).

The library is the only compute path of this package.  Loading fails loudly (ImportError
at first use) when the shared object is missing or was built for another ABI version;
there is no CPU or eager-PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libneurocell_b200.so")
ABI_VERSION = 7

NC_OK, NC_ERR_INVALID, NC_ERR_WORKSPACE, NC_ERR_UNSUPPORTED, NC_ERR_CUDA = 0, 1, 2, 3, 4
NC_PAD = {"VALID": 0, "SAME": 1, "CIRCULAR": 2}
NC_ACT = {"identity": 0, "tanh": 1, "sigmoid": 2, "relu": 3, "leaky_relu": 4, "gelu": 5}
NC_CODD = {"continuous": 0, "annealed": 1, "ste_binary": 2, "ste_ternary": 3}
NC_CONV = {"auto": 0, "direct": 1, "fft": 2}
NC_FLAG_TRAIN = 1

# Every symbol the header declares (checked by the CPU test-suite).
EXPORTED = (
    "nc_plan_bytes", "nc_plan_build", "nc_workspace_bytes", "nc_vnn_forward",
    "nc_vnn_backward", "nc_codd_states", "nc_mse_loss", "nc_softmax_ce_loss",
    "nc_sgd_update", "nc_last_error", "nc_abi_version", "nc_set_profile_events",
    "nc_fp32_peak_probe", "nc_vnn_forward_static", "nc_dp_shared_bytes", "nc_dp_state_bytes",
    "nc_dp_alloc", "nc_dp_free", "nc_ipc_get", "nc_ipc_open", "nc_ipc_close",
    "nc_dp_allreduce_sgd", "nc_dp_status", "nc_launch_count", "nc_conv_path",
    "nc_vnn_forward_universe", "nc_vnn_backward_universe", "nc_universe_embed_forward",
    "nc_universe_embed_backward", "nc_workspace_status", "nc_dp_reset", "nc_stage_from_host",
)
NC_DP_MAX_RANKS = 8
NC_IPC_HANDLE_BYTES = 64


class NcTopo(ctypes.Structure):
    _fields_ = [
        ("H", ctypes.c_int32), ("W", ctypes.c_int32),
        ("kh", ctypes.c_int32), ("kw", ctypes.c_int32),
        ("M", ctypes.c_int32), ("depth", ctypes.c_int32),
        ("padding", ctypes.c_int32),
        ("n_in", ctypes.c_int32), ("n_out", ctypes.c_int32),
        ("act", ctypes.c_int32), ("final_act", ctypes.c_int32),
        ("act_slope", ctypes.c_float), ("final_act_slope", ctypes.c_float),
        ("norm", ctypes.c_int32), ("hard_pin_io", ctypes.c_int32),
        ("gated_filters", ctypes.c_int32), ("conv_algo", ctypes.c_int32),
    ]


class NcCodd(ctypes.Structure):
    _fields_ = [("mode", ctypes.c_int32), ("temperature", ctypes.c_float),
                ("active_threshold", ctypes.c_float), ("temperature_dev", ctypes.c_void_p)]


class NcStageSeg(ctypes.Structure):
    _fields_ = [("dst", ctypes.c_void_p), ("src", ctypes.c_void_p), ("bytes", ctypes.c_size_t)]


NC_MAX_STAGE_SEGS = 4


_vp, _sz, _i32, _u32, _i64, _f32 = (ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32,
                                    ctypes.c_uint32, ctypes.c_int64, ctypes.c_float)
_TP = ctypes.POINTER(NcTopo)
_CP = ctypes.POINTER(NcCodd)

_SIGS = {
    "nc_plan_bytes": (_sz, [_TP]),
    "nc_plan_build": (_i32, [_TP, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "nc_workspace_bytes": (_sz, [_TP, _i32, _u32]),
    "nc_vnn_forward": (_i32, [_TP, _vp, _vp, _vp, _vp, _i32, _CP, _u32, _vp, _vp, _sz, _vp]),
    "nc_vnn_backward": (_i32, [_TP, _vp, _vp, _vp, _vp, _i32, _CP, _vp, _vp, _vp, _vp, _sz, _vp]),
    "nc_vnn_forward_universe": (_i32, [_TP, _vp, _vp, _vp, _vp, _i32, _CP, _u32, _vp, _vp, _vp, _sz,
                                        _vp]),
    "nc_vnn_backward_universe": (_i32, [_TP, _vp, _vp, _vp, _vp, _i32, _CP, _vp, _vp, _vp, _vp, _vp,
                                         _sz, _vp]),
    "nc_universe_embed_forward": (_i32, [_TP, _vp, _vp, _CP, _i32, _i32, _i32, _i32, _vp, _i32, _vp,
                                          _vp, _vp]),
    "nc_universe_embed_backward": (_i32, [_TP, _vp, _vp, _CP, _i32, _i32, _i32, _i32, _vp, _vp, _i32,
                                           _vp, _vp, _vp]),
    "nc_codd_states": (_i32, [_TP, _vp, _vp, _CP, _vp, _vp]),
    "nc_mse_loss": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _vp]),
    "nc_softmax_ce_loss": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _vp]),
    "nc_sgd_update": (_i32, [_vp, _vp, _i64, _f32, _vp]),
    "nc_vnn_forward_static": (_i32, [_TP, _vp, _vp, _vp, _vp, _i32, _CP, _vp, _vp]),
    "nc_set_profile_events": (None, [_vp, _vp, _vp, _vp]),
    "nc_fp32_peak_probe": (_i32, [_i32, ctypes.POINTER(ctypes.c_double), _vp, _vp]),
    "nc_dp_shared_bytes": (_sz, [_i64, _i32]),
    "nc_dp_state_bytes": (_sz, []),
    "nc_dp_alloc": (_i32, [_sz, ctypes.POINTER(_vp)]),
    "nc_dp_free": (_i32, [_vp]),
    "nc_ipc_get": (_i32, [_vp, _vp]),
    "nc_ipc_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "nc_ipc_close": (_i32, [_vp]),
    "nc_dp_allreduce_sgd": (_i32, [ctypes.POINTER(_vp), _i32, _i32, _vp, _vp, _vp, _i64, _f32,
                                   _i32, _vp]),
    "nc_dp_status": (_i32, [_vp, ctypes.POINTER(_i32), _vp]),
    "nc_last_error": (ctypes.c_char_p, []),
    "nc_abi_version": (_i32, []),
    "nc_launch_count": (ctypes.c_uint64, []),
    "nc_conv_path": (_i32, [_TP]),
    "nc_workspace_status": (_i32, [_vp, ctypes.POINTER(_i32), _vp]),
    "nc_dp_reset": (_i32, [_vp, _vp, _sz, _vp]),
    "nc_stage_from_host": (_i32, [ctypes.c_void_p, _i32, _vp]),
}

_lib = None
_lock = threading.Lock()


def load(path: str | None = None):
    """Loads (once) and returns the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = path or os.environ.get("NEUROCELL_B200_LIB", LIB_PATH)
        if not os.path.exists(p):
            raise ImportError(
                f"neurocell_b200: CUDA library not found at {p}; build it with "
                "`python neurocell-v2_b200/build.py` (there is no CPU fallback)")
        lib = ctypes.CDLL(p)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        v = lib.nc_abi_version()
        if v != ABI_VERSION:
            raise ImportError(f"neurocell_b200: library ABI {v} != expected {ABI_VERSION}")
        _lib = lib
        return lib


class NcError(RuntimeError):
    """A failing C-ABI call; ``status`` is the nc_status code."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


def check(status: int, what: str) -> None:
    if status == NC_OK:
        return
    msg = load().nc_last_error().decode(errors="replace")
    if status in (NC_ERR_INVALID,):
        raise ValueError(f"{what}: {msg}")
    if status == NC_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise NcError(status, f"{what}: {msg} (status {status})")
