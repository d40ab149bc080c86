"""Generates the committed golden fixtures under tests/golden/ (run in the dev container).

* ``alu_trained_cells.npz`` -- the reference's trained ALU checkpoint
  (``alu_arithmetic_cells.npz`` at the reference project root, written by
  neurocell/model.py:197-215) re-saved with only the parameter arrays.  It is the input of
  the functional known-answer test: evaluated under ``codd_mode="ste_ternary"`` it must
  reproduce the >= 98 % packed ALU accuracy the reference reports.
* ``alu_trained_eval.npz`` -- a seeded ALU evaluation batch (inputs, packed targets) and the
  float64 oracle's outputs for it, so GPU tests can compare against fixed vectors.

Usage: ``python tests/golden/make_golden.py /path/to/reference``.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import vnn_oracle as O  # noqa: E402


def main(ref_root: str) -> None:
    src = os.path.join(ref_root, "alu_arithmetic_cells.npz")
    with np.load(src, allow_pickle=False) as d:
        w, b, s, f = (d["weights"].astype(np.float32), d["biases"].astype(np.float32),
                      d["states"].astype(np.float32), d["filters"].astype(np.float32))
        meta = {k: d[k] for k in ("N", "depth", "kernel_size", "directions", "n", "gap", "ctrl_gap")}
    np.savez_compressed(os.path.join(HERE, "alu_trained_cells.npz"), weights=w, biases=b, states=s,
                        filters=f, **meta)
    cell = np.stack([w, b, s])
    filt = np.ascontiguousarray(np.transpose(f, (3, 0, 1, 2)))
    geom = O.alu_geometry()
    rng = np.random.default_rng(20261201)
    x, y, packed = O.alu_batch(rng, 256)
    cfg = O.Config(codd_mode="ste_ternary", state_temperature=0.2)
    out, _ = O.forward(cell, filt, x, geom, cfg)
    np.savez_compressed(os.path.join(HERE, "alu_trained_eval.npz"), inputs=x, targets=y,
                        packed=packed, out_f64=out)
    print("oracle packed accuracy on the fixture batch:", O.packed_accuracy(out, packed))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
