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
    # a second epoch keeps training from the updated parameters: it equals three more eager
    # steps on the same batches, bit for bit
    losses2 = [float(eager.step(xd[i], yd[i])) for i in range(3)]
    got2 = ep.train_epoch().cpu().numpy()
    torch.cuda.synchronize()
    assert np.array_equal(got2, np.asarray(losses2, np.float32))
    assert np.array_equal(ep.flat.cpu().numpy(), eager.flat.cpu().numpy())
    assert not np.array_equal(got2, got)


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
    # packed evaluation at the trained parameters against the oracle's logits packed with
    # the reference's bit-weight formula (trainer.py:49-54, 122-138)
    packed = [torch.tensor(O.packed_predictions(np.asarray(y, np.float64)), device=dev) for y in ys]
    acc, preds = tr.evaluate_packed(p, xd, packed)
    want, n_close, acc_ref = [], 0, 0.0
    for x, y in zip(xs, ys):
        logits, _ = O.forward(c, f, x.reshape(16, 3, 8, 1), O.alu_geometry(), O.Config())
        frac = np.abs(np.abs(logits - np.round(logits)) - 0.5)
        n_close += int((frac < 1e-4).any(axis=(1, 2)).sum())    # a rounding tie within fp32 noise
        want.append(O.packed_predictions(logits))
        acc_ref += O.packed_accuracy(logits, O.packed_predictions(np.asarray(y, np.float64))) / len(xs)
    mism = sum(int((pr.cpu().numpy() != w).sum()) for pr, w in zip(preds, want))
    assert len(preds) == 2 and mism <= n_close
    assert abs(acc - acc_ref) <= n_close / 32.0 + 1e-9


def test_packed_evaluation_bytes_follow_the_reference_formula():
    """evaluate_packed on logits that are not bits (2, -1, 300, ties at .5): the bytes equal
    the oracle's restatement of round -> saturating uint8 -> weights summed modulo 256."""
    crafted = np.array([[2.0, 0, 0, 0, 0, 0, 0, 1], [-1.0, 1, 0, 0, 0, 0, 0, 0],
                        [0.49, 0.51, 1.5, 2.5, 0, 0, 0, 0], [300.0, 0, 0, 0, 0, 0, 0, 3],
                        [1, 0, 1, 0, 1, 0, 1, 0]], dtype=np.float32)[:, :, None]
    dev = torch.device("cuda:0")
    tr = nc.VNNTrainer(lambda prm, bx: bx, lr=0.0)
    x = torch.tensor(crafted, device=dev)
    want = O.packed_predictions(crafted)
    target = torch.tensor(want, device=dev)
    acc, preds = tr.evaluate_packed(None, [x], [target])
    assert np.array_equal(preds[0].cpu().numpy().reshape(-1), want.reshape(-1))
    assert acc == 1.0


def test_train_step_sub_roi_graph_equals_eager_adaptive_steps():
    """VNNTrainStep on an adaptive sub-ROI (the window's cells in the packed buffer, one
    CUDA graph per epoch) trains exactly as VNNTrainer.train_step_adaptive does through the
    autograd operator (trainer.py:250-258)."""
    cell, filt, xs, ys = _alu(3, 32, 13)
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()
    p0 = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
    spec = nc.compute_adaptive_spatial_mask(nc.init_vnn_params(701, topo, device=dev), topo)
    assert not spec.is_full_roi
    xd, yd = torch.tensor(xs, device=dev), torch.tensor(ys, device=dev)

    model = nc.VonNeumannNetwork(topo)
    tr = nc.VNNTrainer(model.apply, lr=1e-2, batch_size=32)
    p = nc.VNNParams(p0.cell_params.clone(), p0.greens_filters.clone())
    ref_losses = []
    for i in range(3):
        p, loss = tr.train_step_adaptive(p, xd[i].reshape(32, 3, 8, 1), yd[i], spec)
        ref_losses.append(float(loss))

    st = nc.VNNTrainStep(topo, p0, 32, lr=1e-2, in_shapes=((8, 1),) * 3, spatial_mask=spec)
    assert st.window is not None and st.n_cell < 3 * 62 * 62
    st.capture_epoch(xd, yd)
    got = st.train_epoch().cpu().numpy()
    q = st.params
    torch.cuda.synchronize()
    assert q.cell_params.shape == (3, 62, 62)
    assert np.allclose(got, np.asarray(ref_losses, np.float32), rtol=1e-6, atol=0)
    rel = (torch.linalg.norm(q.cell_params - p.cell_params) / torch.linalg.norm(p.cell_params)).item()
    relf = (torch.linalg.norm(q.greens_filters - p.greens_filters) /
            torch.linalg.norm(p.greens_filters)).item()
    assert rel <= 1e-6 and relf <= 1e-6
    # cells outside the window keep their initial values
    r0, r1, c0, c1 = st.window
    outside = torch.ones((62, 62), dtype=torch.bool, device=dev)
    outside[r0:r1, c0:c1] = False
    assert torch.equal(q.cell_params[:, outside], p0.cell_params[:, outside])


def test_adaptive_epochs_one_bucket_and_convergence():
    """unit_milestone7_adaptive_mask.py:186-220: the mask is recomputed before every epoch,
    one sub-ROI bucket (one window plan) serves all three epochs, the loss falls, and the
    packed evaluation runs on the same mask."""
    from neurocell_b200 import ops
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()
    model = nc.VonNeumannNetwork(topo, backend="auto")
    params = nc.init_vnn_params(708, topo, device=dev)
    tr = nc.VNNTrainer(model.apply, lr=0.05, batch_size=32)
    g = torch.Generator(dev).manual_seed(709)
    x_ep = torch.randint(0, 2, (4, 32, 3, 8, 1), generator=g, device=dev).float()
    y_ep = torch.randint(0, 2, (4, 32, 8), generator=g, device=dev).float()
    losses, bboxes, plans = [], set(), []
    for _ in range(3):
        spec = model.compute_spatial_mask(params, margin=4, bucket_multiple=8)
        bboxes.add(spec.roi_bbox)
        params, ep_loss = tr.train_epoch_adaptive(params, x_ep, y_ep, spec)
        losses.append(float(ep_loss))
        plans.append({k for k in ops._PLANS if k[-2] is not None})
    # epochs 2 and 3 reuse the window plan built for the bucket in epoch 1
    assert len(bboxes) == 1 and plans[0] == plans[1] == plans[2]
    assert any(k[-2] == next(iter(bboxes)) for k in plans[0])
    assert losses[-1] < losses[0]
    y_packed = nc.packbits_u8_on_device(y_ep.to(torch.uint8))
    acc, preds = tr.evaluate_packed_adaptive(params, x_ep, y_packed, spec)
    assert len(preds) == 4 and preds[0].shape == (32, 1) and 0.0 <= acc <= 1.0
    m = tr.evaluate_metric_adaptive(params, x_ep, y_ep, spec)
    assert 0.0 <= m <= 1.0


def test_annealed_steps_and_multi_epoch_shuffle():
    """train_step_annealed / train_epochs (trainer.py:322-398): the temperature is a plain
    argument, the multi-epoch loop shuffles on the device."""
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()
    model = nc.VonNeumannNetwork(topo)
    params = nc.init_vnn_params(711, topo, device=dev)
    tr = nc.VNNTrainer(model.apply, lr=0.05, batch_size=16)
    g = torch.Generator(dev).manual_seed(712)
    x = torch.randint(0, 2, (16, 3, 8, 1), generator=g, device=dev).float()
    y = torch.randint(0, 2, (16, 8), generator=g, device=dev).float()
    taus = [nc.compute_annealed_temperature(e, 3) for e in range(3)]
    for tau in taus:
        params, loss = tr.train_step_annealed(params, x, y, state_temperature=tau, codd_mode="ste_ternary")
        assert torch.isfinite(loss)
    xt = torch.randint(0, 2, (40, 3, 8, 1), generator=g, device=dev).float()
    yt = torch.randint(0, 2, (40, 8), generator=g, device=dev).float()
    params, ep = tr.train_epochs(params, xt, yt, 5, 3)
    assert ep.shape == (3,) and bool(torch.isfinite(ep).all())


def test_graph_step_follows_the_annealed_temperature():
    """set_temperature reaches a captured step (tau is a device scalar the kernels read when
    they run): three graph replays at tau = 1.0, 0.4, 0.1 equal three eager steps at the same
    temperatures, and differ from replays at a fixed tau."""
    cell, filt, xs, ys = _alu(3, 32, 21)
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()
    xd, yd = torch.tensor(xs, device=dev), torch.tensor(ys, device=dev)

    def runner():
        p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
        return nc.trainer.VNNTrainStep(topo, p, 32, lr=5e-2, in_shapes=((8, 1),) * 3,
                                       codd_mode="annealed", state_temperature=1.0)

    taus = (1.0, 0.4, 0.1)
    eager, graph, fixed = runner(), runner(), runner()
    graph.load_batch(xd[0], yd[0])
    graph.capture()
    fixed.load_batch(xd[0], yd[0])
    fixed.capture()
    le, lg = [], []
    for i, tau in enumerate(taus):
        eager.set_temperature(tau)
        le.append(float(eager.step(xd[i], yd[i])))
        graph.set_temperature(tau)
        lg.append(float(graph.step(xd[i], yd[i])))
        fixed.step(xd[i], yd[i])
    torch.cuda.synchronize()
    assert le == lg
    assert torch.equal(graph.flat, eager.flat)
    assert not torch.equal(fixed.flat, eager.flat)


def _dp_call(lib, peers, world, rank, state, g, p, n, lr, max_wait, dev):
    import ctypes
    from neurocell_b200 import _lib
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(lib.nc_dp_allreduce_sgd(peers, world, rank, ctypes.c_void_p(state.data_ptr()),
                                       ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(p.data_ptr()),
                                       n, lr, max_wait, st), "nc_dp_allreduce_sgd")
    status = ctypes.c_int32(-1)
    _lib.check(lib.nc_dp_status(ctypes.c_void_p(state.data_ptr()), ctypes.byref(status), st),
               "nc_dp_status")
    return status.value


def _tagged(values: np.ndarray, step: int) -> torch.Tensor:
    """Elements of the receive buffer: (step << 32) | float bits, as int64."""
    bits = values.astype(np.float32).view(np.uint32).astype(np.uint64)
    return torch.tensor(((np.uint64(step) << np.uint64(32)) | bits).view(np.int64))


def test_exchange_timeout_is_terminal_until_reset():
    """Failure detection without a GPU fault.  Rank 0 of a two-rank exchange whose peer is
    a plain buffer on this GPU: rank 0's own receive buffer is pre-filled from the host with
    the peer's step-1 values for the first half of the lines only.  Lines that arrived are
    summed and updated; the others time out, stay untouched and set the status word.  The
    status is terminal: a second call changes nothing.  After nc_dp_reset and a complete
    pre-fill the exchange completes again."""
    import ctypes
    from neurocell_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    n, world, lr = 1000, 2, 0.1
    L = (n + 1) // 2                       # 16-byte lines of two elements
    good_lines = 256                       # lines 0..255 see their peer's values
    shared_bytes = lib.nc_dp_shared_bytes(n, world)
    assert shared_bytes >= 2 * world * L * 16
    own = torch.zeros(shared_bytes // 8, dtype=torch.int64, device=dev)
    peer = torch.zeros(shared_bytes // 8, dtype=torch.int64, device=dev)
    state = torch.zeros(lib.nc_dp_state_bytes() // 4, dtype=torch.int32, device=dev)
    peers = (ctypes.c_void_p * world)(own.data_ptr(), peer.data_ptr())
    rng = np.random.default_rng(3)
    v = rng.normal(size=2 * L).astype(np.float32)          # the peer's gradient, 2 per line
    slot = (1 * world + 1) * L * 2                         # (parity 1, source 1) in elements
    own[slot:slot + 2 * good_lines] = _tagged(v[:2 * good_lines], 1).to(dev)
    g = torch.tensor(rng.normal(size=n).astype(np.float32), device=dev)
    p = torch.tensor(rng.normal(size=n).astype(np.float32), device=dev)
    g0, p0 = g.clone(), p.clone()
    assert _dp_call(lib, peers, world, 0, state, g, p, n, lr, 2000, dev) == 1
    k = 2 * good_lines
    vt = torch.tensor(v[:n], device=dev)
    s = g0[:k] + vt[:k]
    assert torch.equal(g[:k], s)
    # the kernel's update is one fused multiply-add, torch rounds twice: compare to 1e-6
    assert torch.allclose(p[:k], p0[:k] - (lr / world) * s, rtol=1e-6, atol=1e-7)
    assert torch.equal(g[k:], g0[k:]) and torch.equal(p[k:], p0[k:])
    # rank 0 pushed its own values with tag 1 into the peer's slot (parity 1, source 0)
    pushed = peer[(1 * world + 0) * L * 2:(1 * world + 0) * L * 2 + n].cpu().numpy().view(np.uint64)
    assert np.all((pushed >> np.uint64(32)) == 1)
    # terminal: nothing moves, nothing is pushed
    g1, p1 = g.clone(), p.clone()
    peer.zero_()
    own[slot:slot + 2 * L] = _tagged(v, 2).to(dev)
    assert _dp_call(lib, peers, world, 0, state, g, p, n, lr, 2000, dev) == 1
    assert torch.equal(g, g1) and torch.equal(p, p1) and int(peer.abs().sum()) == 0
    # reset, complete pre-fill of step 1: the exchange completes
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(lib.nc_dp_reset(ctypes.c_void_p(state.data_ptr()), ctypes.c_void_p(own.data_ptr()),
                               shared_bytes, st), "nc_dp_reset")
    assert int(own.abs().sum()) == 0 and int(state.abs().sum()) == 0
    own[slot:slot + 2 * L] = _tagged(v, 1).to(dev)
    g2, p2 = g.clone(), p.clone()
    assert _dp_call(lib, peers, world, 0, state, g, p, n, lr, 2000, dev) == 0
    s = g2 + vt
    assert torch.equal(g, s) and torch.allclose(p, p2 - (lr / world) * s, rtol=1e-6, atol=1e-7)
    torch.cuda.synchronize()


def test_exchange_ignores_stale_step_tags():
    """A value whose tag is from an older step (the other parity's leftovers, or the same
    slot two steps back) is never summed: the block waits for the current tag."""
    import ctypes
    from neurocell_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    n, world, lr = 64, 2, 0.5
    L = (n + 1) // 2
    shared_bytes = lib.nc_dp_shared_bytes(n, world)
    own = torch.zeros(shared_bytes // 8, dtype=torch.int64, device=dev)
    peer = torch.zeros(shared_bytes // 8, dtype=torch.int64, device=dev)
    state = torch.zeros(lib.nc_dp_state_bytes() // 4, dtype=torch.int32, device=dev)
    peers = (ctypes.c_void_p * world)(own.data_ptr(), peer.data_ptr())
    v = np.arange(2 * L, dtype=np.float32)
    slot1 = (1 * world + 1) * L * 2
    slot0 = (0 * world + 1) * L * 2
    own[slot1:slot1 + 2 * L] = _tagged(v, 1).to(dev)            # step 1 (parity 1)
    g = torch.ones(n, device=dev)
    p = torch.zeros(n, device=dev)
    assert _dp_call(lib, peers, world, 0, state, g, p, n, lr, 4000, dev) == 0
    # step 2 (parity 0) finds only a stale step-0 tag there: it must time out, not sum
    own[slot0:slot0 + 2 * L] = _tagged(v + 100, 0).to(dev)
    g3, p3 = g.clone(), p.clone()
    assert _dp_call(lib, peers, world, 0, state, g, p, n, lr, 4000, dev) == 1
    assert torch.equal(g, g3) and torch.equal(p, p3)


def test_five_step_sgd_trajectory_matches_oracle():
    """Five graph-captured SGD steps of the fused step on the ALU chip follow the float64
    oracle's trajectory (the reference's multi-step trajectory parity,
    tests/unit_vnn_alu_parity.py:141-194 and tests/unit_kernels_pallas.py:130-198, with SGD
    instead of AdamW): parameters within rel-L2 1e-5 after five steps, every loss within
    1e-5 relative."""
    cell, filt, xs, ys = _alu(5, 32, 33)
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()
    p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
    st = nc.trainer.VNNTrainStep(topo, p, 32, lr=1e-2, in_shapes=((8, 1),) * 3)   # the bench's SGD
    xd, yd = torch.tensor(xs, device=dev), torch.tensor(ys, device=dev)
    st.load_batch(xd[0], yd[0])
    st.capture()
    geom = O.alu_geometry()
    c, f = cell.astype(np.float64), filt.astype(np.float64)
    for i in range(5):
        loss = float(st.step(xd[i], yd[i]))
        lval, c, f, _, _ = O.train_step(c, f, xs[i].reshape(32, 3, 8, 1), ys[i], geom, O.Config(), lr=1e-2)
        assert abs(loss - lval) / lval <= 1e-5, (i, loss, lval)
    q = st.params
    torch.cuda.synchronize()
    rc = np.linalg.norm(q.cell_params.cpu().numpy() - c) / np.linalg.norm(c)
    rf = np.linalg.norm(q.greens_filters.cpu().numpy() - f) / np.linalg.norm(f)
    assert rc <= 1e-5 and rf <= 1e-5, (rc, rf)


def test_stage_from_host_copies_pinned_batches_and_refuses_pageable_memory():
    """nc_stage_from_host: page-locked host tensors land in device buffers bit for bit (16-
    and 4-byte paths); a pageable source is refused on the host with NC_ERR_INVALID before
    any launch."""
    import ctypes
    from neurocell_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    a = torch.randn(3072).pin_memory()
    b = torch.arange(1001, dtype=torch.int32).pin_memory()        # 4004 bytes: 4-byte path
    da = torch.empty(3072, device=dev)
    db = torch.empty(1001, dtype=torch.int32, device=dev)
    segs = (_lib.NcStageSeg * 2)()
    segs[0].dst, segs[0].src, segs[0].bytes = da.data_ptr(), a.data_ptr(), 4 * a.numel()
    segs[1].dst, segs[1].src, segs[1].bytes = db.data_ptr(), b.data_ptr(), 4 * b.numel()
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    _lib.check(lib.nc_stage_from_host(segs, 2, st), "nc_stage_from_host")
    torch.cuda.synchronize()
    assert torch.equal(da.cpu(), a) and torch.equal(db.cpu(), b)
    pageable = torch.randn(64)
    assert not pageable.is_pinned()
    bad = (_lib.NcStageSeg * 1)()
    bad[0].dst, bad[0].src, bad[0].bytes = da.data_ptr(), pageable.data_ptr(), 256
    assert lib.nc_stage_from_host(bad, 1, st) == _lib.NC_ERR_INVALID
    assert b"pageable" in lib.nc_last_error()


def test_host_loss_train_step_matches_device_loss_step():
    """VNNTrainStep(host_loss=True) with page-locked batches (staging kernel, loss stored into
    page-locked host memory) trains exactly like the device-loss step, eager and graph."""
    cell, filt, xs, ys = _alu(3, 32, 12)
    dev = torch.device("cuda:0")
    topo = nc.ChipTopology2D.alu_chip()

    def runner(host_loss):
        p = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
        return nc.trainer.VNNTrainStep(topo, p, 32, lr=1e-2, in_shapes=((8, 1),) * 3,
                                       host_loss=host_loss)
    xh = torch.tensor(xs).pin_memory()
    yh = torch.tensor(ys).pin_memory()
    xd, yd = xh.to(dev), yh.to(dev)
    ref, hst, hg = runner(False), runner(True), runner(True)
    hg.load_batch(xh[0], yh[0])
    hg.capture()
    for i in range(3):
        l_ref = float(ref.step(xd[i], yd[i]))
        l_h = hst.step(xh[i], yh[i])
        l_g = hg.step(xh[i], yh[i])
        assert not l_h.is_cuda and l_h.is_pinned()
        torch.cuda.synchronize()
        assert float(l_h) == l_ref and float(l_g) == l_ref
    torch.cuda.synchronize()
    assert torch.equal(hst.flat, ref.flat) and torch.equal(hg.flat, ref.flat)
