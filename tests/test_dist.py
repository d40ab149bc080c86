"""Data-parallel host logic on CPU: two `gloo` ranks each take half of a batch, compute
their shard's gradient with the float64 oracle, exchange it with the same helper the B200
train step uses (neurocell_b200.trainer.allreduce_mean_), and the resulting update must
equal the single-process update over the whole batch."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    from oracle import vnn_oracle as O
    rng = np.random.default_rng(5)
    geom = O.make_geometry((16, 16), (5, 3), 4, 3, (O.RectPort((5, 4), (4, 1)),),
                           O.RectPort((5, 10), (4, 1)))
    cell = rng.normal(0, 0.3, (3, 16, 16))
    filt = rng.normal(0, 0.3, (4, 1, 5, 3))
    x = rng.normal(size=(8, 4, 1))
    y = rng.normal(size=(8, 4))
    return O, geom, cell, filt, x, y


def _rank_main(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys
        root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
        sys.path[:0] = [root, os.path.join(root, "neurocell-v2_b200")]
        from neurocell_b200.trainer import allreduce_mean_
        O, geom, cell, filt, x, y = _problem()
        shard = slice(rank * 4, rank * 4 + 4)
        out, tape = O.forward(cell, filt, x[shard], geom)
        _, gout = O.mse_loss(out, y[shard])
        gc, gf = O.backward(gout, tape, geom)
        flat = torch.from_numpy(np.concatenate([gc.ravel(), gf.ravel()]).astype(np.float64))
        w = allreduce_mean_(flat, dist.group.WORLD)
        if rank == 0:
            np.save(out_path, flat.numpy() / w)
    finally:
        dist.destroy_process_group()


def test_two_rank_gradient_exchange_matches_full_batch(tmp_path):
    out_path = str(tmp_path / "g.npy")
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, out_path), nprocs=2, join=True,
                       start_method="spawn")
    O, geom, cell, filt, x, y = _problem()
    out, tape = O.forward(cell, filt, x, geom)
    _, gout = O.mse_loss(out, y)
    gc, gf = O.backward(gout, tape, geom)
    full = np.concatenate([gc.ravel(), gf.ravel()])
    got = np.load(out_path)
    assert np.linalg.norm(got - full) / np.linalg.norm(full) < 1e-12


def test_single_process_exchange_is_identity():
    from neurocell_b200.trainer import allreduce_mean_
    t = torch.arange(5.0)
    assert allreduce_mean_(t, None) == 1
    assert torch.equal(t, torch.arange(5.0))
