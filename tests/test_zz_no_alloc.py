"""GPU test of nc_vnn_forward_static, the inference entry point that allocates nothing.

Some callers cannot call cudaMalloc: an XLA FFI custom call whose framework already owns
nearly all device memory, code running during stream capture, hosts that forbid
allocation after start-up.  nc_vnn_forward_static serves them from a static device array
inside the library.  This test calls it through the C ABI twice in a row (different
inputs, so stale scratch from the first call would show) on each kernel family and checks
both results against nc_vnn_forward with a caller workspace, within the parity tolerance
used elsewhere.  It
also checks that a call needing more scratch than the array holds is refused.
The file name sorts last so that a run stopping at the first failure has run every other
test first.
"""
import ctypes

import numpy as np
import pytest
import torch

from neurocell_b200 import _lib, ops
from neurocell_b200.topology import ChipTopology2D, CoordinatePortSpec, PortSpec

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _plan(topo, in_shapes, dev, conv="auto"):
    return ops.get_plan(topo, in_shapes, dev, "tanh", 0.0, "identity", 1.0, True, False, False, conv)


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _alu_case(rng, conv):
    topo = ChipTopology2D.alu_chip()
    cell = rng.normal(0, 0.1, (3, 62, 62)).astype(np.float32)
    u = rng.uniform(1e-6, 1 - 1e-6, (62, 62))
    cell[2] = np.log(u / (1 - u))
    filt = (rng.normal(0, 1, (16, 1, 23, 13)) / np.sqrt(299)).astype(np.float32)
    return topo, ((8, 1),) * 3, conv, cell, filt, 64


def _fft_regime_case(rng):
    # 40 x 40 SAME chip with 31 x 31 filters: a 128 x 128 FFT grid, the per-step FFT kernels
    ports = (PortSpec((4, 4), (6, 6)), CoordinatePortSpec([(20, 3), (21, 3), (22, 3)]))
    topo = ChipTopology2D.create(40, (31, 31), 8, 3, ports,
                                 CoordinatePortSpec([(r, 35) for r in range(15, 25)]),
                                 padding_mode="SAME")
    cell = rng.normal(0, 0.3, (3, 40, 40)).astype(np.float32)
    filt = (rng.normal(0, 1, (8, 1, 31, 31)) / 31.0).astype(np.float32)
    return topo, ((6, 6), (3,)), "fft", cell, filt, 6


@pytest.mark.parametrize("case", ["alu_fused_fft", "alu_direct", "fft_regime"])
def test_static_scratch_forward_matches_workspace_forward_twice(case):
    """Two calls in a row with different inputs on each kernel family (the fused per-sample
    FFT kernels, the direct kernels, the per-step FFT kernels, which use other scratch
    sections): each result equals nc_vnn_forward with a caller workspace."""
    lib = _lib.load()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(77)
    if case == "fft_regime":
        topo, in_shapes, conv, cell, filt, B = _fft_regime_case(rng)
        expect_path = 2
    else:
        topo, in_shapes, conv, cell, filt, B = _alu_case(rng, "direct" if case == "alu_direct" else "auto")
        expect_path = 1 if case == "alu_direct" else 3
    plan = _plan(topo, in_shapes, dev, conv)
    assert lib.nc_conv_path(ctypes.byref(plan.topo)) == expect_path
    cp = torch.tensor(cell, device=dev)
    fl = torch.tensor(filt, device=dev)
    codd = _lib.NcCodd(_lib.NC_CODD["ste_ternary"], 1.0, 0.6)
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    P = ops._ptr
    ws_bytes = lib.nc_workspace_bytes(ctypes.byref(plan.topo), B, 0)
    assert 0 < ws_bytes <= (8 << 20)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    for call in range(2):
        x = torch.tensor(rng.uniform(-0.2, 1.2, (B, plan.n_in)).astype(np.float32), device=dev)
        ref = torch.empty((B, plan.n_out), device=dev)
        got = torch.full((B, plan.n_out), float("nan"), device=dev)
        _lib.check(lib.nc_vnn_forward(ctypes.byref(plan.topo), P(plan.buf), P(cp), P(fl), P(x), B,
                                      ctypes.byref(codd), 0, P(ref), P(ws), ws_bytes, st),
                   "nc_vnn_forward")
        _lib.check(lib.nc_vnn_forward_static(ctypes.byref(plan.topo), P(plan.buf), P(cp), P(fl),
                                             P(x), B, ctypes.byref(codd), P(got), st),
                   "nc_vnn_forward_static")
        torch.cuda.synchronize()
        r, g = ref.cpu().numpy(), got.cpu().numpy()
        assert np.all(np.isfinite(g)), f"call {call}: non-finite output"
        assert _rel(g, r) <= TOL, f"call {call}: rel-L2 {_rel(g, r)}"


def test_static_scratch_refuses_oversized_calls():
    lib = _lib.load()
    dev = torch.device("cuda:0")
    ports = (PortSpec((0, 32), (32, 32)), PortSpec((32, 32), (32, 32)), PortSpec((64, 32), (32, 32)))
    topo = ChipTopology2D.create(96, (15, 15), 16, 2, ports,
                                 CoordinatePortSpec([(r, 80) for r in range(43, 53)]))
    plan = _plan(topo, ((32, 32),) * 3, dev)
    B = 64
    assert lib.nc_workspace_bytes(ctypes.byref(plan.topo), B, 0) > (8 << 20)
    codd = _lib.NcCodd(0, 1.0, 0.6)
    dummy = torch.zeros(16, device=dev)
    p = ops._ptr(dummy)
    status = lib.nc_vnn_forward_static(ctypes.byref(plan.topo), ops._ptr(plan.buf), p, p, p, B,
                                       ctypes.byref(codd), p, None)
    assert status == _lib.NC_ERR_WORKSPACE
    assert b"static scratch" in lib.nc_last_error()
