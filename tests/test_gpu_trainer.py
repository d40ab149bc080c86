"""The training engine on the GPU: the whole-epoch CUDA graph replays exactly the eager
steps, the epoch trainer mirrors the reference's scan (trainer.py:108-119), and packed
evaluation matches the oracle's accuracy."""
import numpy as np
import pytest
import torch

import neurocell_b200 as nc
from oracle import vnn_oracle as O

pytestmark = pytest.mark.gpu


def _alu(nb, B, seed):
    rng = np.random.default_rng(seed)
    cell = rng.normal(0, 0.1, (3, 62, 62)).astype(np.float32)
    filt = (rng.normal(0, 1, (16, 1, 23, 13)) / np.sqrt(299)).astype(np.float32)
    xs, ys = [], []
    for _ in range(nb):
        x, y, _ = O.alu_batch(rng, B, noise=0.0)
        xs.append(x.reshape(B, -1))
        ys.append(y)
    return cell, filt, np.stack(xs), np.stack(ys)


@pytest.mark.parametrize("conv", ["auto", "direct"])
def test_epoch_graph_equals_eager_steps(conv):
    cell, filt, xs, ys = _alu(3, 32, 5)
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()
    xd, yd = torch.tensor(xs, device=dev), torch.tensor(ys, device=dev)

    def runner():
        p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
        return nc.trainer.VNNTrainStep(topo, p, 32, lr=1e-2, in_shapes=((8, 1),) * 3, conv=conv)

    eager = runner()
    losses = []
    for i in range(3):
        losses.append(float(eager.step(xd[i], yd[i])))
    ep = runner()
    ep.capture_epoch(xd, yd)
    got = ep.train_epoch().cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(ep.flat.cpu().numpy(), eager.flat.cpu().numpy())
    assert np.array_equal(got, np.asarray(losses, np.float32))
    # a second epoch keeps training from the updated parameters
    got2 = ep.train_epoch().cpu().numpy()
    assert got2[0] < got[0] or not np.array_equal(got2, got)


def test_vnn_trainer_epoch_and_packed_evaluation():
    cell, filt, xs, ys = _alu(2, 16, 9)
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()
    p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
    tr = nc.VNNTrainer(lambda prm, bx: nc.propagate_vnn_2d(prm, bx, topo), lr=1e-2, batch_size=16)
    xd = [torch.tensor(x.reshape(16, 3, 8, 1), device=dev) for x in xs]
    yd = [torch.tensor(y, device=dev) for y in ys]
    p, loss = tr.train_epoch(p, xd, yd)
    # oracle: the same two SGD steps
    c, f = cell, filt
    total = 0.0
    for x, y in zip(xs, ys):
        lval, c, f, _, _ = O.train_step(c, f, x.reshape(16, 3, 8, 1), y, O.alu_geometry(), O.Config(), lr=1e-2)
        total += lval
    assert abs(float(loss) - total / 16) / (total / 16) <= 1e-5
    assert np.linalg.norm(p.cell_params.cpu().numpy() - c) / np.linalg.norm(c) <= 1e-6
    packed = [torch.tensor(np.packbits(np.asarray(y, np.uint8), axis=1), device=dev) for y in ys]
    acc, preds = tr.evaluate_packed(p, xd, packed)
    assert 0.0 <= acc <= 1.0 and len(preds) == 2
