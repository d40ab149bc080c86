"""The oracle pinned to the reference's own definition chain (CPU).

The reference proves its v2 propagator against the legacy v1 network
(tests/unit_vnn_alu_parity.py:76-139): forward max-abs < 1e-5 on the outputs and on the
whole final grid, gradients of W, B, S within relative L2 1e-5 (filters 5e-5).  Here the
float64 oracle (oracle/vnn_oracle.py, hand-written adjoints) meets an independent float64
restatement of that legacy network (oracle/legacy_v1.py, autograd) on the ALU chip, with
the parameters passed through this package's legacy Haiku import.  Both sides are float64,
so the bars used here are far tighter than the reference's float32 ones.
"""
import os

import numpy as np
import pytest
import torch

from oracle import legacy_v1 as L1
from oracle import vnn_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# The ALU chip's geometry as literals (the reference's tests/unit_topology.py:29-50 pins):
GRID = (62, 62)
KERNEL = (23, 13)
M, DEPTH = 16, 4
IN_OFFSETS = ((23, 23), (32, 23), (18, 28))
IN_SIZES = ((8, 1), (8, 1), (1, 8))
OUT_OFFSET, OUT_SIZE = (27, 41), (8, 1)
FWD_BAR = 1e-10       # reference: 1e-5 max-abs (float32)
GRAD_BAR = 1e-9       # reference: 1e-5 rel-L2 (5e-5 for the filters, float32 cuDNN)


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / (np.linalg.norm(b) + 1e-12))


def _legacy_leaves(rng, b_scale=0.2):
    """UniverseLP.initialize's scales (contrib/universe.py:293-327) with non-zero biases, as
    the reference's parity test sets them so the border propagation is active."""
    N = GRID[0]
    init = 1.0 / np.sqrt(DEPTH * N)
    finit = 1.0 / np.sqrt(KERNEL[0] * KERNEL[1] * M)
    return {"w": rng.normal(0, init, GRID), "b": rng.normal(0, b_scale, GRID),
            "s": rng.normal(0, init, GRID), "f": rng.normal(0, finit, (1,) + KERNEL + (M,))}


def _to_v2(leaves):
    """The package's import_legacy_haiku_params (neurocell/params.py:339-346 semantics)."""
    import neurocell_b200 as nc
    hk = {"universe_lp": {k: torch.tensor(v, dtype=torch.float64) for k, v in leaves.items()}}
    p = nc.params.import_legacy_haiku_params(hk)
    return p.cell_params.numpy(), p.greens_filters.numpy()


def _legacy_run(leaves, x, final_activate=None):
    t = {k: torch.tensor(v, dtype=torch.float64) for k, v in leaves.items()}
    ports = [torch.tensor(x[:, i], dtype=torch.float64) for i in range(3)]
    cells, out = L1.universe_lp(t, ports, IN_OFFSETS, IN_SIZES, OUT_OFFSET, OUT_SIZE, DEPTH,
                                final_activate=final_activate)
    return cells.numpy(), out.numpy()


@pytest.mark.parametrize("final", [None, "tanh"])
def test_oracle_forward_and_universe_match_legacy_v1(final):
    rng = np.random.default_rng(42)
    leaves = _legacy_leaves(rng)
    x, _, _ = O.alu_batch(rng, 32, noise=0.0)
    cells_ref, out_ref = _legacy_run(leaves, x, final)
    cell, filt = _to_v2(leaves)
    geom = O.alu_geometry()
    cfg = O.Config(final_activate=final)
    out, _ = O.forward(cell, filt, x, geom, cfg)
    out_u, uni, _ = O.forward_universe(cell, filt, x, geom, cfg)
    assert out.shape == out_ref.shape == (32, 8, 1)
    assert np.max(np.abs(out - out_ref)) < FWD_BAR
    assert np.max(np.abs(out_u - out_ref)) < FWD_BAR
    assert np.max(np.abs(uni - cells_ref)) < FWD_BAR


def test_oracle_gradients_match_legacy_v1():
    rng = np.random.default_rng(55)
    leaves = _legacy_leaves(rng, b_scale=0.15)
    x, y, _ = O.alu_batch(rng, 32, noise=0.0)
    ports = [torch.tensor(x[:, i], dtype=torch.float64) for i in range(3)]
    t = {k: torch.tensor(v, dtype=torch.float64) for k, v in leaves.items()}
    loss_ref, g = L1.value_and_grad(t, ports, torch.tensor(y, dtype=torch.float64),
                                    in_offsets=IN_OFFSETS, in_sizes=IN_SIZES, out_offset=OUT_OFFSET,
                                    out_size=OUT_SIZE, depth=DEPTH)
    cell, filt = _to_v2(leaves)
    loss, _, _, gc, gf = O.train_step(cell, filt, x, y, O.alu_geometry(), O.Config(), lr=0.0)
    assert abs(loss - loss_ref) / loss_ref < FWD_BAR
    assert _rel(gc[0], g["w"].numpy()) < GRAD_BAR
    assert _rel(gc[1], g["b"].numpy()) < GRAD_BAR
    assert _rel(gc[2], g["s"].numpy()) < GRAD_BAR
    assert _rel(np.transpose(gf, (1, 2, 3, 0)), g["f"].numpy()) < GRAD_BAR


def test_trained_checkpoint_matches_legacy_v1():
    """The reference's trained checkpoint (ill-conditioned: filters in [-41, 42]) through both
    definitions, sigmoid states (the legacy network's only state rule)."""
    with np.load(os.path.join(GOLDEN, "alu_trained_cells.npz")) as d:
        keys = set(d.files)
        w, b, s = d["weights"], d["biases"], d["states"]
        f_ihwo = d["filters"]
    assert {"weights", "biases", "states", "filters"} <= keys
    leaves = {"w": w.astype(np.float64), "b": b.astype(np.float64), "s": s.astype(np.float64),
              "f": f_ihwo.astype(np.float64)}
    rng = np.random.default_rng(7)
    x, y, _ = O.alu_batch(rng, 16, noise=0.0)
    cells_ref, out_ref = _legacy_run(leaves, x)
    cell, filt = _to_v2(leaves)
    out, uni, _ = O.forward_universe(cell, filt, x, O.alu_geometry(), O.Config())
    scale = np.max(np.abs(out_ref))
    assert np.max(np.abs(out - out_ref)) < FWD_BAR * max(scale, 1.0)
    assert np.max(np.abs(uni - cells_ref)) < FWD_BAR * max(np.max(np.abs(cells_ref)), 1.0)


def test_three_step_sgd_trajectory_matches_legacy_v1():
    """Three SGD steps (the reference checks five AdamW steps, tests/unit_vnn_alu_parity.py:
    141-194): the oracle's parameters follow the legacy network's."""
    rng = np.random.default_rng(77)
    leaves = _legacy_leaves(rng)
    cell, filt = _to_v2(leaves)
    t = {k: torch.tensor(v, dtype=torch.float64) for k, v in leaves.items()}
    geom = O.alu_geometry()
    lr = 0.05
    for step in range(3):
        x, y, _ = O.alu_batch(rng, 16, noise=0.0)
        ports = [torch.tensor(x[:, i], dtype=torch.float64) for i in range(3)]
        loss_ref, g = L1.value_and_grad(t, ports, torch.tensor(y, dtype=torch.float64),
                                        in_offsets=IN_OFFSETS, in_sizes=IN_SIZES,
                                        out_offset=OUT_OFFSET, out_size=OUT_SIZE, depth=DEPTH)
        t = {k: t[k] - lr * g[k] for k in t}
        loss, cell, filt, _, _ = O.train_step(cell, filt, x, y, geom, O.Config(), lr=lr)
        assert abs(loss - loss_ref) / loss_ref < FWD_BAR, step
    assert _rel(cell[0], t["w"].numpy()) < GRAD_BAR
    assert _rel(cell[1], t["b"].numpy()) < GRAD_BAR
    assert _rel(cell[2], t["s"].numpy()) < GRAD_BAR
    assert _rel(np.transpose(filt, (1, 2, 3, 0)), t["f"].numpy()) < GRAD_BAR


def test_legacy_restatement_is_not_vacuous():
    """A planted mistake in the legacy restatement (the zero padding applied BEFORE the
    standardisation, which puts the dead ring into the plane statistics) is caught."""
    rng = np.random.default_rng(42)
    leaves = _legacy_leaves(rng)
    x, _, _ = O.alu_batch(rng, 8, noise=0.0)
    _, out_ref = _legacy_run(leaves, x)
    orig = L1.forward_full

    def pad_then_norm(cells, weights, biases, states, filters_ihwo, act, norm=True):
        kh, kw = filters_ihwo.shape[1:3]
        r = torch.nn.functional.conv2d(cells[:, None], filters_ihwo.permute(3, 0, 1, 2))
        r = torch.nn.functional.pad(r, ((kw - 1) // 2,) * 2 + ((kh - 1) // 2,) * 2)
        r = L1.standardize(r) if norm else r
        s = torch.sigmoid(states)
        r = r * weights * (1 - s) + (act(r + biases) if act else r + biases) * s
        return r.mean(dim=1)

    L1.forward_full = pad_then_norm
    try:
        _, out_bad = _legacy_run(leaves, x)
    finally:
        L1.forward_full = orig
    assert np.max(np.abs(out_bad - out_ref)) > 1e-3
