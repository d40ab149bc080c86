"""Discrete spatial stencils and their application to a 2-D plane (mirrors
``neurocell/filters.py:12-83`` and ``apply_spatial_filter_2d``, ``neurocell/kernels_greens.py:220-237``).

The stencils are the reference's 3x3 (and 3x3x3) tables.  ``sharpen(norm=True)`` is what
``VonNeumannNetwork(sharpen=True)`` applies to the W plane of the cell parameters before the
output-port pin (``neurocell/params.py:246-249``).  This is a pre-step weight transform on one
(H, W) plane: it runs as a device-side 3x3 convolution in front of the library's kernels, and
autograd carries its gradient back to W.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _t(rows, dtype, device):
    return torch.tensor(rows, dtype=dtype, device=device)


def smooth(dtype=torch.float32, norm: bool = False, device=None):
    """3x3 window / smoothing stencil (filters.py:12-20)."""
    c = 8 if norm else 1
    return _t([[1, 1, 1], [1, c, 1], [1, 1, 1]], dtype, device)


def backward(dtype=torch.float32, norm: bool = False, device=None):
    """3x3 backward propagation stencil (filters.py:23-31)."""
    c = 3 if norm else 0
    return _t([[1, 0, 0], [1, c, 0], [1, 0, 0]], dtype, device)


def forward(dtype=torch.float32, norm: bool = False, device=None):
    """3x3 forward propagation stencil (filters.py:34-42)."""
    c = 3 if norm else 0
    return _t([[0, 0, 1], [0, c, 1], [0, 0, 1]], dtype, device)


def von_neumann(dtype=torch.float32, norm: bool = False, device=None):
    """3x3 bidirectional von Neumann stencil (filters.py:45-53)."""
    c = 6 if norm else 1
    return _t([[1, 0, 1], [1, c, 1], [1, 0, 1]], dtype, device)


def sharpen(dtype=torch.float32, norm: bool = True, device=None):
    """3x3 sharpen stencil, divided by 5 when ``norm`` (filters.py:56-68)."""
    k = _t([[0, -1, 0], [-1, 5, -1], [0, -1, 0]], dtype, device)
    return k / 5.0 if norm else k


def sharpen_3d(dtype=torch.float32, norm: bool = True, device=None):
    """3x3x3 sharpen stencil, divided by 5 when ``norm`` (filters.py:71-83)."""
    z = [[0, 0, 0], [0, -1, 0], [0, 0, 0]]
    k = _t([z, [[0, -1, 0], [-1, 5, -1], [0, -1, 0]], z], dtype, device)
    return k / 5.0 if norm else k


def apply_spatial_filter_2d(field_hw: torch.Tensor, kernel_hw: torch.Tensor, padding: str = "SAME"):
    """Cross-correlation of an (H, W) plane with a 2-D stencil, zeros outside the plane
    (``lax.conv_general_dilated`` NCHW/OIHW, stride 1).  ``padding``: "SAME" (output (H, W),
    odd stencils) or "VALID"."""
    if padding not in ("SAME", "VALID"):
        raise ValueError(f"padding must be 'SAME' or 'VALID', got {padding!r}")
    k = kernel_hw.to(device=field_hw.device, dtype=field_hw.dtype)
    if padding == "SAME":
        kh, kw = k.shape
        if kh % 2 == 0 or kw % 2 == 0:
            raise ValueError("SAME padding needs an odd stencil")
        pad = (kh // 2, kw // 2)
    else:
        pad = (0, 0)
    return F.conv2d(field_hw[None, None], k[None, None], padding=pad)[0, 0]
