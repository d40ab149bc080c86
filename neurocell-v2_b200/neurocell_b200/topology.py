"""Compile-time VNN geometry: ports, ROI bounds, static masks and chip presets.

Mirrors ``neurocell/topology.py`` of shakes76/neurocell-v2 (same class names, fields,
validation messages and presets) with numpy boolean masks in place of jax arrays:

* ``PortSpec``            -- topology.py:19-34
* ``CoordinatePortSpec``  -- topology.py:37-83
* ``ChipTopology2D``      -- topology.py:109-284 (``create``), presets 286-458
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Sequence

import numpy as np


@dataclass(frozen=True)
class PortSpec:
    """A rectangular input, control or output port on the cellular grid."""
    offset: tuple
    size: tuple
    name: str = ""

    def __post_init__(self):
        object.__setattr__(self, "offset", tuple(int(v) for v in self.offset))
        object.__setattr__(self, "size", tuple(int(v) for v in self.size))
        if len(self.offset) != len(self.size):
            raise ValueError(
                f"PortSpec offset {self.offset} and size {self.size} must have matching rank.")
        if any(s <= 0 for s in self.size):
            raise ValueError(f"PortSpec size dimensions must be positive, got {self.size}.")


@dataclass(frozen=True)
class CoordinatePortSpec:
    """A scattered coordinate port addressed by explicit ``(row, col)`` pairs."""
    coords: tuple
    name: str = ""

    def __init__(self, coords: Sequence[Sequence[int]], name: str = ""):
        ct = tuple((int(c[0]), int(c[1])) for c in np.asarray(coords).tolist())
        if len(ct) == 0:
            raise ValueError("CoordinatePortSpec coords must be non-empty.")
        object.__setattr__(self, "coords", ct)
        object.__setattr__(self, "name", str(name))

    @property
    def num_points(self) -> int:
        return len(self.coords)

    @property
    def size(self) -> tuple:
        return (len(self.coords), 1)

    @property
    def offset(self) -> tuple:
        return (min(r for r, _ in self.coords), min(c for _, c in self.coords))

    @property
    def rows(self) -> np.ndarray:
        return np.array([r for r, _ in self.coords], dtype=np.int32)

    @property
    def cols(self) -> np.ndarray:
        return np.array([c for _, c in self.coords], dtype=np.int32)

    def fits_in_roi(self, grid_shape, r_h: int, r_w: int) -> bool:
        H, W = grid_shape
        return all(r_h <= r < (H - r_h) and r_w <= c < (W - r_w) for r, c in self.coords)


AnyPortSpec = PortSpec | CoordinatePortSpec


def _next_power_of_two(x: int) -> int:
    return 1 << (x - 1).bit_length()


def _port_within_bounds(port, r_min, r_max, c_min, c_max) -> bool:
    if isinstance(port, CoordinatePortSpec):
        return all(r_min <= r < r_max and c_min <= c < c_max for r, c in port.coords)
    r0, c0 = port.offset
    rh, cw = port.size
    return r0 >= r_min and c0 >= c_min and (r0 + rh) <= r_max and (c0 + cw) <= c_max


@dataclass(frozen=True, eq=False)
class ChipTopology2D:
    """Immutable specification of a 2D VNN cellular topology (topology.py:109-150)."""
    grid_shape: tuple
    kernel_size: tuple
    directions: int
    depth: int
    in_ports: tuple
    out_port: AnyPortSpec
    pad_h: int
    pad_w: int
    roi_shape: tuple
    roi_out_offset: tuple
    io_state_mask: np.ndarray
    out_weight_mask: np.ndarray
    fft_shape: tuple
    padding_mode: str = "VALID"
    in_in_roi: bool = True
    out_in_roi: bool = True

    @property
    def H(self) -> int:
        return self.grid_shape[0]

    @property
    def W(self) -> int:
        return self.grid_shape[1]

    @property
    def N(self) -> int:
        return max(self.grid_shape)

    def key(self) -> tuple:
        """Hashable identity of the geometry (used to cache device plans)."""
        return (self.grid_shape, self.kernel_size, self.directions, self.depth, self.in_ports,
                self.out_port, self.padding_mode)

    @classmethod
    def create(cls, grid_shape, kernel_size, directions, depth, in_ports, out_port,
               fft_shape=None, padding_mode: str = "VALID", allow_border_output: bool = False):
        """Validated topology with ROI bounds and static masks (topology.py:152-284)."""
        if isinstance(grid_shape, int):
            grid_shape = (grid_shape, grid_shape)
        else:
            grid_shape = (int(grid_shape[0]), int(grid_shape[1]))
        kh, kw = int(kernel_size[0]), int(kernel_size[1])
        if kh % 2 == 0 or kw % 2 == 0:
            raise ValueError(f"Green's function kernel_size must be odd, got {kernel_size}.")
        padding_mode = padding_mode.upper()
        if padding_mode not in ("VALID", "SAME", "CIRCULAR"):
            raise ValueError(
                f"Unsupported padding_mode '{padding_mode}'; choose from ('VALID', 'SAME', 'CIRCULAR').")
        H, W = grid_shape
        if padding_mode == "VALID":
            pad_h, pad_w = (kh - 1) // 2, (kw - 1) // 2
        else:
            pad_h, pad_w = 0, 0
        roi_h, roi_w = H - 2 * pad_h, W - 2 * pad_w
        if roi_h <= 0 or roi_w <= 0:
            raise ValueError(
                f"Grid {grid_shape} is too small for kernel {kernel_size}; valid ROI is ({roi_h}, {roi_w}).")
        in_ports_tuple = tuple(in_ports)
        for port in in_ports_tuple + (out_port,):
            if not _port_within_bounds(port, 0, H, 0, W):
                raise ValueError(
                    f"Port '{port.name}' at offset={port.offset}, size={port.size} "
                    f"exceeds grid_shape={grid_shape}.")
        in_in_roi = all(_port_within_bounds(p, pad_h, H - pad_h, pad_w, W - pad_w)
                        for p in in_ports_tuple)
        out_in_roi = _port_within_bounds(out_port, pad_h, H - pad_h, pad_w, W - pad_w)
        is_full_grid_out = (isinstance(out_port, PortSpec) and out_port.offset == (0, 0)
                            and out_port.size == grid_shape)
        if padding_mode == "VALID" and not out_in_roi and not allow_border_output and not is_full_grid_out:
            raise ValueError(
                f"Output port {out_port} lies outside the active VALID convolution ROI "
                f"[{pad_h}:{H - pad_h}, {pad_w}:{W - pad_w}].")
        out_r, out_c = out_port.offset
        if isinstance(out_port, CoordinatePortSpec):
            roi_out_offset = (tuple(int(r - pad_h) for r, _ in out_port.coords),
                              tuple(int(c - pad_w) for _, c in out_port.coords))
        else:
            roi_out_offset = (max(0, out_r - pad_h), max(0, out_c - pad_w))
        io = np.zeros(grid_shape, dtype=bool)
        for port in in_ports_tuple:
            if isinstance(port, CoordinatePortSpec):
                io[port.rows, port.cols] = True
            else:
                r0, c0 = port.offset
                rh, cw = port.size
                io[r0:r0 + rh, c0:c0 + cw] = True
        ow = np.zeros(grid_shape, dtype=bool)
        if isinstance(out_port, CoordinatePortSpec):
            io[out_port.rows, out_port.cols] = True
            ow[out_port.rows, out_port.cols] = True
        else:
            oh_, ow_ = out_port.size
            io[out_r:out_r + oh_, out_c:out_c + ow_] = True
            ow[out_r:out_r + oh_, out_c:out_c + ow_] = True
        io.setflags(write=False)
        ow.setflags(write=False)
        if fft_shape is None:
            if padding_mode == "CIRCULAR":
                fft_shape = (H, W)
            else:
                fft_shape = (_next_power_of_two(roi_h + kh - 1), _next_power_of_two(roi_w + kw - 1))
        return cls(grid_shape=grid_shape, kernel_size=(kh, kw), directions=int(directions),
                   depth=int(depth), in_ports=in_ports_tuple, out_port=out_port, pad_h=pad_h,
                   pad_w=pad_w, roi_shape=(roi_h, roi_w), roi_out_offset=roi_out_offset,
                   io_state_mask=io, out_weight_mask=ow, fft_shape=tuple(fft_shape),
                   padding_mode=padding_mode, in_in_roi=in_in_roi, out_in_roi=out_in_roi)

    @classmethod
    def alu_chip(cls, n: int = 8, kernel_size=(23, 13), directions: int = 16, depth: int = 4,
                 gap: int = 5, ctrl_gap: int = 5):
        """The canonical 2D ALU chip of the VNN paper (topology.py:286-321)."""
        padding = 2 * max(kernel_size[0], kernel_size[1])
        N = 2 * n + padding
        center = N // 2
        input_top = center - (2 * n) // 2
        input_left = center - n
        output_mid = center - n // 2
        output_left = input_left + n + 2 * gap
        in_ports = (
            PortSpec(offset=(input_top, input_left), size=(n, 1), name="x1"),
            PortSpec(offset=(input_top + n + 1, input_left), size=(n, 1), name="x2"),
            PortSpec(offset=(input_top - ctrl_gap, input_left + gap), size=(1, n), name="ctrl"),
        )
        out_port = PortSpec(offset=(output_mid, output_left), size=(n, 1), name="out")
        return cls.create(grid_shape=(N, N), kernel_size=kernel_size, directions=directions,
                          depth=depth, in_ports=in_ports, out_port=out_port)

    @classmethod
    def mlp_chip(cls, n: int = 8, layers: int = 5, ctrl_gap: int = 1, kernel_size=(17, 3),
                 directions: int = 8):
        """Vertical 2D MLP chip (topology.py:323-357)."""
        padding = 2 * max(kernel_size[0], kernel_size[1])
        N = 2 * n + padding
        center = N // 2
        gap = 2 * layers + 1
        input_top = center - (3 * n + ctrl_gap) // 2
        input_left = center - gap // 2
        output_mid = center - n // 2
        output_left = input_left + gap
        depth = output_left - input_left
        in_ports = (PortSpec(offset=(input_top, input_left), size=(3 * n + ctrl_gap, 1), name="x_in"),)
        out_port = PortSpec(offset=(output_mid, output_left), size=(n, 1), name="out")
        return cls.create(grid_shape=(N, N), kernel_size=kernel_size, directions=directions,
                          depth=depth, in_ports=in_ports, out_port=out_port)

    @classmethod
    def clp_chip(cls, grid_shape=(8, 8), in_coords=None, out_coords=None, kernel_size=(3, 3),
                 directions: int = 1, depth: int = 4, padding_mode: str = "VALID", n=None):
        """Coordinate-addressed circular layered perceptron (topology.py:390-428)."""
        if n is not None:
            grid_shape = (int(n), int(n))
        elif isinstance(grid_shape, int):
            grid_shape = (grid_shape, grid_shape)
        H, W = grid_shape
        r_h = (kernel_size[0] - 1) // 2 if padding_mode.upper() == "VALID" else 0
        r_w = (kernel_size[1] - 1) // 2 if padding_mode.upper() == "VALID" else 0
        if in_coords is None:
            in_coords = ((r_h + 1, r_w + 1), (H - r_h - 2, r_w + 1))
        if out_coords is None:
            out_coords = ((r_h + 1, W - r_w - 2), (H - r_h - 2, W - r_w - 2))
        return cls.create(grid_shape=grid_shape, kernel_size=kernel_size, directions=directions,
                          depth=depth, in_ports=(CoordinatePortSpec(in_coords, name="clp_in"),),
                          out_port=CoordinatePortSpec(out_coords, name="clp_out"),
                          padding_mode=padding_mode, allow_border_output=True)

    @classmethod
    def tm_chip(cls, n: int = 8, kernel_size=(13, 13), directions: int = 16, gap: int = 1):
        """2D Turing-machine tape (topology.py:430-458)."""
        length = 2 * n
        padding = 2 * max(kernel_size[0], kernel_size[1])
        N = length + 2 * padding
        center = N // 2
        input_left = padding
        output_left = input_left + length + gap
        depth = output_left - input_left
        in_ports = (PortSpec(offset=(center, input_left), size=(1, length), name="tape_in"),)
        out_port = PortSpec(offset=(center, output_left), size=(1, n), name="tape_out")
        return cls.create(grid_shape=(N, N), kernel_size=kernel_size, directions=directions,
                          depth=depth, in_ports=in_ports, out_port=out_port)

    @classmethod
    def gol_chip(cls, grid_shape=(64, 64), kernel_size=(3, 3), directions: int = 64,
                 depth: int = 2, padding_mode: str = "VALID", n=None):
        """Full-grid cellular automaton (topology.py:359-388).  Its output port covers the
        whole grid, so propagate_vnn_2d reads it from the assembled universe (the reference's
        full-grid output path, propagator.py:684-734)."""
        if n is not None:
            grid_shape = (int(n), int(n))
        elif isinstance(grid_shape, int):
            grid_shape = (grid_shape, grid_shape)
        return cls.create(grid_shape=grid_shape, kernel_size=kernel_size, directions=directions,
                          depth=depth, in_ports=(PortSpec((0, 0), grid_shape, "universe_in"),),
                          out_port=PortSpec((0, 0), grid_shape, "universe_out"),
                          padding_mode=padding_mode, allow_border_output=True)
