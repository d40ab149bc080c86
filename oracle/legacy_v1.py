"""Independent restatement of the reference's LEGACY (v1) VNN -- TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may import this module.  It is a second, independent definition of the
function the B200 path computes, written from the reference's legacy code rather than from
its v2 propagator, so that a misreading of ``neurocell/propagator.py`` shared by
``vnn_oracle.py`` and ``torch_port.py`` cannot pass unnoticed.  It imports nothing from
either of them.  The reference pins v2 against exactly this chain
(``tests/unit_vnn_alu_parity.py:76-139``: forward max-abs < 1e-5, gradients rel-L2 < 1e-5).

What it restates (paths relative to the shakes76/neurocell-v2 project root):

* ``contrib/universe.py:561-622``  ``UniverseLP.__call__`` (``sharpen=False``): the state
  of every input-port cell and output-port cell set to ``STATE_ACTIVE_VALUE`` = 1.0 before
  the sigmoid (port *sizes* give the pinned rectangles), the output-port weights set to
  1.0, filters optionally gated by a sigmoid, then the forward operator.
* ``contrib/universe.py:273-330``  ``UniverseLP.initialize``: the forward operator is
  ``_propagate_full_mlp_list`` vmapped over the batch; filters are IHWO (1, kh, kw, M).
* ``contrib/forward.py:161-178``   ``_propagate_full_mlp_list``: each input written into a
  zero grid with ``dynamic_update_slice`` using the input array's OWN shape (so an (8, 1)
  array on a (1, 8) port lands as a column); d - 1 hidden steps, a final step with the
  final activation inside the epilogue, that activation applied again to every cell; the
  output is the out-port rectangle of the final grid.
* ``contrib/forward.py:737-811``   ``_forward_full`` (mode COMPRESS): a VALID
  cross-correlation of the whole grid with the M filters, ``jax.nn.standardize`` over the
  spatial axes (variance as E[x^2] - E[x]^2, epsilon 1e-5), zero padding back to the grid
  AFTER the standardisation, ``r*w*(1-s) + act(r+b)*s`` with s = sigmoid(state) (``r + b``
  without an activation), then the mean over the M filters.
* ``contrib/convs.py:27-46``       ``_fast_conv``: ``lax.conv_general_dilated`` (a
  cross-correlation).

Gradients come from torch autograd in float64, not from hand-written adjoints.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

STATE_ACTIVE_VALUE = 1.0
STANDARDIZE_EPS = 1e-5
_GELU_C = math.sqrt(2.0 / math.pi)


def activation(name):
    """The activations the legacy drivers pass (jax.nn.*); None = no activation."""
    if name in (None, "identity"):
        return None
    return {
        "tanh": torch.tanh,
        "sigmoid": torch.sigmoid,
        "relu": torch.relu,
        "gelu": lambda x: 0.5 * x * (1.0 + torch.tanh(_GELU_C * (x + 0.044715 * x ** 3))),
    }[name]


def standardize(x: torch.Tensor) -> torch.Tensor:
    """jax.nn.standardize over the last two axes: (x - mean) / sqrt(E[x^2] - mean^2 + eps)."""
    mean = x.mean(dim=(-2, -1), keepdim=True)
    var = (x * x).mean(dim=(-2, -1), keepdim=True) - mean * mean
    return (x - mean) / torch.sqrt(var + STANDARDIZE_EPS)


def dynamic_update_slice(grid: torch.Tensor, update: torch.Tensor, start) -> torch.Tensor:
    """lax.dynamic_update_slice on (B, H, W) with a per-sample (h, w) update; the start
    index is clamped so the update fits, as XLA does."""
    H, W = grid.shape[-2:]
    h, w = update.shape[-2:]
    r0 = min(max(int(start[0]), 0), H - h)
    c0 = min(max(int(start[1]), 0), W - w)
    out = grid.clone()
    out[..., r0:r0 + h, c0:c0 + w] = update
    return out


def forward_full(cells, weights, biases, states, filters_ihwo, act, norm=True):
    """One step over the whole grid (contrib/forward.py:737-811), batched: cells (B, H, W)."""
    kh, kw = filters_ihwo.shape[1:3]
    w_oihw = filters_ihwo.permute(3, 0, 1, 2)                       # (M, 1, kh, kw)
    r = F.conv2d(cells[:, None], w_oihw)                            # VALID cross-correlation
    if norm:
        r = standardize(r)
    ph, pw = (kh - 1) // 2, (kw - 1) // 2
    r = F.pad(r, (pw, pw, ph, ph))                                  # zeros after the norm
    s = torch.sigmoid(states)
    if act is None:
        r = r * weights * (1.0 - s) + (r + biases) * s
    else:
        r = r * weights * (1.0 - s) + act(r + biases) * s
    return r.mean(dim=1)                                            # COMPRESS: mean over M


def propagate_full_mlp_list(inputs, in_offsets, out_offset, out_size, depth, grid_shape, weights,
                            biases, states, filters_ihwo, act, final_act, norm=True):
    """contrib/forward.py:161-178, batched.  Returns (cells (B, H, W), outputs)."""
    B = inputs[0].shape[0]
    cells = torch.zeros((B,) + tuple(grid_shape), dtype=weights.dtype)
    for x, off in zip(inputs, in_offsets):
        cells = dynamic_update_slice(cells, x, off)
    for _ in range(1, depth):
        cells = forward_full(cells, weights, biases, states, filters_ihwo, act, norm)
    cells = forward_full(cells, weights, biases, states, filters_ihwo, final_act, norm)
    if final_act is not None:
        cells = final_act(cells)
    r0, c0 = out_offset
    oh, ow = out_size
    return cells, cells[:, r0:r0 + oh, c0:c0 + ow]


def universe_lp(params: dict, inputs, in_offsets, in_sizes, out_offset, out_size, depth,
                activate="tanh", final_activate=None, norm=True, gated_filters=False):
    """UniverseLP.__call__ (contrib/universe.py:561-622) with sharpen off.

    ``params``: the legacy Haiku leaves {"w", "b", "s": (H, W), "f": (1, kh, kw, M)} as
    float64 torch tensors (autograd flows to them).  ``inputs``: per input port, (B, ih, iw).
    Returns (cells (B, H, W), outputs (B, oh, ow))."""
    grid_shape = tuple(params["w"].shape)
    states = params["s"]
    for size, off in zip(in_sizes, in_offsets):
        states = dynamic_update_slice(states, torch.full(tuple(size), STATE_ACTIVE_VALUE,
                                                         dtype=states.dtype), off)
    states = dynamic_update_slice(states, torch.full(tuple(out_size), STATE_ACTIVE_VALUE,
                                                     dtype=states.dtype), out_offset)
    weights = dynamic_update_slice(params["w"], torch.full(tuple(out_size), 1.0, dtype=states.dtype),
                                   out_offset)
    filters = torch.sigmoid(params["f"]) if gated_filters else params["f"]
    return propagate_full_mlp_list(inputs, in_offsets, out_offset, out_size, depth, grid_shape,
                                   weights, params["b"], states, filters, activation(activate),
                                   activation(final_activate), norm)


def value_and_grad(params: dict, inputs, targets, **kw):
    """MSE (optax.squared_error(...).mean()) of the squeezed outputs and its gradient with
    respect to the four legacy leaves (tests/unit_vnn_alu_parity.py:118-126)."""
    leaves = {k: v.detach().clone().requires_grad_(True) for k, v in params.items()}
    _, out = universe_lp(leaves, inputs, **kw)
    loss = ((out.reshape(out.shape[0], -1) - targets.reshape(out.shape[0], -1)) ** 2).mean()
    loss.backward()
    return float(loss.detach()), {k: v.grad for k, v in leaves.items()}
