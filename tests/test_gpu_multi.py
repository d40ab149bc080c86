"""Data parallelism on 2 GPUs with NCCL: two ranks each run the fused train step on half of
an ALU batch; the all-reduced gradient equals the single-GPU gradient of the whole batch
(relative L2 <= 1e-5) and both ranks end with identical parameters.  Skips on boxes with
fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(B):
    from oracle import vnn_oracle as O
    rng = np.random.default_rng(123)
    cell = rng.normal(0, 0.1, (3, 62, 62)).astype(np.float32)
    filt = (rng.normal(0, 1, (16, 1, 23, 13)) / np.sqrt(299)).astype(np.float32)
    x, y, _ = O.alu_batch(rng, B, noise=0.0)
    return cell, filt, x.reshape(B, -1), y


def _rank_main(rank, world, port, out_dir, exchange="nccl", graph=False, long_steps=0):
    import sys
    from datetime import timedelta
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "neurocell-v2_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        import neurocell_b200 as nc
        cell, filt, x, y = _problem(64)
        shard = slice(rank * 32, rank * 32 + 32)
        topo = nc.ChipTopology2D.alu_chip()
        p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
        st = nc.trainer.VNNTrainStep(topo, p, 32, lr=1e-2, in_shapes=((8, 1),) * 3,
                                     process_group=dist.group.WORLD, exchange=exchange)
        xs, ys = torch.tensor(x[shard], device=dev), torch.tensor(y[shard], device=dev)
        if graph:
            st.load_batch(xs, ys)
            st.capture()
        st.step(xs, ys)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"grads{rank}.npy"), st.grads.cpu().numpy())
        np.save(os.path.join(out_dir, f"params{rank}.npy"), st.flat.cpu().numpy())
        if graph:                       # three more steps through the graph
            for _ in range(3):
                st.step(xs, ys)
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"params4_{rank}.npy"), st.flat.cpu().numpy())
        if long_steps:                  # many graph replays over four batches per rank
            cellb, filtb, xb, yb = _problem(256)
            xr = torch.tensor(xb.reshape(4, 2, 32, -1)[:, rank], device=dev)
            yr = torch.tensor(yb.reshape(4, 2, 32, -1)[:, rank], device=dev)
            for i in range(long_steps):
                st.step(xr[i % 4], yr[i % 4])
            torch.cuda.synchronize()
            np.save(os.path.join(out_dir, f"params_long_{rank}.npy"), st.flat.cpu().numpy())
        np.save(os.path.join(out_dir, f"status{rank}.npy"), np.array([st.exchange_status()]))
        st.release()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _full_batch_reference(steps=1):
    import neurocell_b200 as nc
    cell, filt, x, y = _problem(64)
    dev = torch.device("cuda", 0)
    p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
    st = nc.trainer.VNNTrainStep(nc.ChipTopology2D.alu_chip(), p, 64, lr=1e-2,
                                 in_shapes=((8, 1),) * 3)
    xs, ys = torch.tensor(x, device=dev), torch.tensor(y, device=dev)
    st.step(xs, ys)
    torch.cuda.synchronize()
    full_g, full_p = st.grads.cpu().numpy(), st.flat.cpu().numpy()
    for _ in range(steps - 1):
        st.step(xs, ys)
    torch.cuda.synchronize()
    return full_g, full_p, st.flat.cpu().numpy()


def _run(tmp_path, exchange, graph=False, long_steps=0):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(2, _free_port(), str(tmp_path), exchange, graph, long_steps),
                       nprocs=2, join=True, start_method="spawn")


def _check_first_step(tmp_path, full_g, full_p):
    g0 = np.load(tmp_path / "grads0.npy") / 2.0
    g1 = np.load(tmp_path / "grads1.npy") / 2.0
    assert np.array_equal(g0, g1)                       # every rank holds the same sum
    assert np.linalg.norm(g0 - full_g) / np.linalg.norm(full_g) <= 1e-5
    p0, p1 = np.load(tmp_path / "params0.npy"), np.load(tmp_path / "params1.npy")
    assert np.array_equal(p0, p1)
    assert np.linalg.norm(p0 - full_p) / np.linalg.norm(p0) <= 1e-6
    assert np.load(tmp_path / "status0.npy")[0] == 0 and np.load(tmp_path / "status1.npy")[0] == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_data_parallel_step_matches_full_batch(tmp_path):
    _run(tmp_path, "nccl")
    full_g, full_p, _ = _full_batch_reference()
    _check_first_step(tmp_path, full_g, full_p)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_nvlink_exchange_matches_full_batch(tmp_path):
    """The fused peer-memory sum + SGD kernel, eager step then three graph replays: the
    ranks stay bitwise identical and track the single-GPU full-batch run."""
    _run(tmp_path, "nvlink", graph=True)
    full_g, full_p, full_p4 = _full_batch_reference(steps=4)
    _check_first_step(tmp_path, full_g, full_p)
    q0, q1 = np.load(tmp_path / "params4_0.npy"), np.load(tmp_path / "params4_1.npy")
    assert np.array_equal(q0, q1)
    assert np.linalg.norm(q0 - full_p4) / np.linalg.norm(full_p4) <= 1e-5


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_nvlink_exchange_long_graph_replay(tmp_path):
    """1,000 graph-captured steps with the NVLink exchange: both ranks end with bitwise
    identical parameters, every exchange completed, and the trajectory matches the same
    1,000 steps with NCCL's all-reduce to 1e-6."""
    a, b = tmp_path / "nvlink", tmp_path / "nccl"
    a.mkdir()
    b.mkdir()
    _run(a, "nvlink", graph=True, long_steps=1000)
    _run(b, "nccl", graph=True, long_steps=1000)
    p0, p1 = np.load(a / "params_long_0.npy"), np.load(a / "params_long_1.npy")
    assert np.array_equal(p0, p1)
    assert np.load(a / "status0.npy")[0] == 0 and np.load(a / "status1.npy")[0] == 0
    q0, q1 = np.load(b / "params_long_0.npy"), np.load(b / "params_long_1.npy")
    assert np.array_equal(q0, q1)
    assert np.linalg.norm(p0 - q0) / np.linalg.norm(q0) <= 1e-6
    start = _problem(64)
    init = np.concatenate([start[0].reshape(-1), start[1].reshape(-1)])
    assert np.linalg.norm(p0 - init) / np.linalg.norm(init) > 1e-3     # training moved them
