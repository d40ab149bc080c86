"""Benchmark of the B200 VNN hot path on BASELINE config 0 (62x62 ALU train step).

``python bench.py --gpus N --steps K --warmup W [--impl b200|reference]``

* ``--impl b200`` (default): every rank trains the ALU chip (K=23x13, M=16, d=4,
  continuous Codd, MSE, SGD lr=1e-2) on its own 128-sample batches; gradients are
  summed over the ranks by one NVLink peer-memory kernel fused with the SGD update
  (``--exchange nccl``: NCCL all-reduce + SGD kernel) -- data parallel, weak scaling:
  global batch = 128*N.  Prints ONE
  JSON line on rank 0: device-resident throughput (``value``), the end-to-end figure through
  the public ``VNNTrainStep`` API with page-locked host batches in and the loss out to
  page-locked host memory inside the timed region (``e2e``), the fused-kernel
  roofline against a live-measured FP32 FFMA peak, the clocks seen during the timed region
  and a CPU baseline (the torch-CPU port of the same algorithm, rank 0, N=1 only).
* ``--impl reference``: the reference's JAX path cannot be installed here, so rank 0 times
  the CPU port of the reference algorithm (``oracle/torch_port.py``, float32, all host
  threads) on the same workload; other ranks exit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "neurocell-v2_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

BATCH = 128
SEED = 0            # config index 0 -> seeds 0 (params), 1 (filters), 2 (inputs)
LR = 1e-2
WORKLOAD = "BASELINE config 0: 62x62 ALU VNN train step (fwd+bwd+SGD)"
METRIC = "train samples/s (62x62 ALU VNN, B=128 per GPU)"   # both arms report this metric
# the workload fields both arms report
WORKLOAD_FIELDS = {"workload": WORKLOAD, "grid": [62, 62], "roi": [40, 50], "kernel": [23, 13], "M": 16,
                   "depth": 4, "codd_mode": "continuous", "loss": "mse", "optimizer": "sgd(1e-2)"}


L2_NOTE = "GPU arm: L2 flushed (256 MB write) before every timed step; CPU arm: not applicable"


def workload_config(world: int) -> dict:
    """The `config` object of the bench line: the same keys and values in both arms."""
    return {**WORKLOAD_FIELDS, "per_gpu_batch": BATCH, "global_batch": BATCH * world,
            "parallelism": f"dp{world}", "l2": L2_NOTE}


def fftf_executed_flops(M: int, roi_h: int, Fh: int, kh: int, d: int) -> tuple[float, float]:
    """FLOPs the fused 64 x 64 FFT kernels execute per sample (forward, backward), counted per
    transform and pointwise product: 5 N log2 N = 1920 per 64-point complex transform (the
    usual FFT count), 6 per complex product, 8 per complex multiply-accumulate.  Per step the
    forward transforms the field (Fh rows + 64 columns) and, per direction pair, forms
    X^.H_j and runs 64 inverse columns and roi_h inverse rows.  The backward, per pair, runs
    roi_h + 64 forward lines of the plane gradients, D += Q^.conj(H_j) (steps t > 0),
    X^.conj(Q^), 64 inverse columns and kh inverse lag rows, and per step t > 0 the
    inverse field adjoint (64 columns + Fh rows); it reloads the forward's field spectra."""
    c64, nn = 5.0 * 64 * 6, 64.0 * 64.0
    pairs = M // 2
    fwd_step = (Fh + 64) * c64 + pairs * (6 * nn + (64 + roi_h) * c64)
    bwd_pair = (roi_h + 64 + 64 + kh) * c64 + 6 * nn
    bwd = sum(pairs * (bwd_pair + (8 * nn if t > 0 else 0)) + ((64 + Fh) * c64 if t > 0 else 0)
              for t in range(d))
    return d * fwd_step, bwd


def alu_flops_per_sample(train: bool = True) -> float:
    """Effective direct-convolution FLOPs per sample: 2*M*P*K per pass; a train step makes
    d forward passes, d filter-gradient passes and d-1 field-adjoint passes."""
    M, P, K, d = 16, 40 * 50, 23 * 13, 4
    per_pass = 2.0 * M * P * K
    return per_pass * ((3 * d - 1) if train else d)


# ---------------------------------------------------------------------------------------
def make_problem(rank: int, n_batches: int, batch: int):
    from oracle import vnn_oracle as O   # seeded synthetic ALU data (datasets.py:77-130)
    rng_p = np.random.default_rng(SEED * 1000 + 0)
    rng_f = np.random.default_rng(SEED * 1000 + 1)
    rng_x = np.random.default_rng([SEED * 1000 + 2, rank])
    cell = rng_p.normal(0, 0.1, (3, 62, 62)).astype(np.float32)
    filt = (rng_f.normal(0, 1, (16, 1, 23, 13)) / np.sqrt(23 * 13)).astype(np.float32)
    xs, ys = [], []
    for _ in range(n_batches):
        x, y, _ = O.alu_batch(rng_x, batch, noise=0.0)
        xs.append(x)
        ys.append(y)
    return cell, filt, np.stack(xs), np.stack(ys)


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of one GPU, polled through NVML every
    2 ms in a background thread (the timed regions of config 0 last only a few ms, too short
    for nvidia-smi's 200 ms loop).  ``mark_start()`` / ``mark_stop()`` bracket the timed
    region; ``stop()`` summarises the samples taken inside it.  Falls back to nvidia-smi
    when NVML is unavailable."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, device):
        self.rows = []                 # (t, sm_mhz, max_mhz, reason bits)
        self.t0 = self.t1 = None
        self.source = "nvml (2 ms polling)"
        self._stop = threading.Event()
        self.nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            self.nvml, self.h = pynvml, h
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
        except Exception as e:   # noqa: BLE001 -- no NVML: nothing to sample
            self.source = f"unavailable ({type(e).__name__})"

    def _sample(self):
        nv, h = self.nvml, self.h
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                              getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
        try:
            sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
            bits = int(get_reasons(h)) if get_reasons else 0
            self.rows.append((time.perf_counter(), sm, bits))
        except Exception:   # noqa: BLE001
            pass

    def _poll(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(0.002)

    def mark_start(self):
        # the poller needs the interpreter lock while the timed loop launches: switch often
        self._switch = sys.getswitchinterval()
        sys.setswitchinterval(1e-4)
        self.t0 = time.perf_counter()

    def mark_stop(self):
        # one sample taken here as well, at the end of the work, for windows of a few ms
        if self.nvml is not None:
            self._sample()
        self.t1 = time.perf_counter()
        if getattr(self, "_switch", None):
            sys.setswitchinterval(self._switch)

    def stop(self) -> dict:
        if self.nvml is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0,
                    "source": self.source}
        self._stop.set()
        self.t.join(timeout=2)
        inside = [r for r in self.rows if self.t0 is not None and self.t1 is not None
                  and self.t0 <= r[0] <= self.t1]
        sm = [r[1] for r in inside]
        reasons = set()
        for name, const in self.REASONS:
            bit = getattr(self.nvml, const, 0)
            if any(r[2] & bit for r in inside):
                reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(sm),
                "window_ms": (self.t1 - self.t0) * 1e3 if self.t0 and self.t1 else None,
                "source": self.source}


def exchange_ms(runner, n: int, dev, pg):
    """Device time of the gradient exchange (the NVLink kernel, or the NCCL all-reduce and
    the SGD kernel): median over n eager steps taken after the timed region by every rank
    (same collective steps), max over ranks.  None on one GPU."""
    if pg is None or runner.world <= 1:
        return None
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for a, b in evs:            # torch creates the CUDA event on first record
        a.record()
        b.record()
    torch.cuda.synchronize()
    for i in range(n):
        runner.exchange_events = evs[i]
        runner._launch()
    runner.exchange_events = None
    torch.cuda.synchronize()
    return max_over_ranks(statistics.median(a.elapsed_time(b) for a, b in evs), dev)


def max_over_ranks(v: float, dev) -> float:
    """The largest v over the ranks of the default process group."""
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def spread(ms: list) -> dict:
    """Median and 10th / 90th percentiles of per-step times (ms)."""
    q = np.percentile(np.asarray(ms, dtype=np.float64), [10, 50, 90])
    return {"p10": float(q[0]), "median": float(q[1]), "p90": float(q[2]), "n": len(ms)}


def fp32_peak_tflops(device) -> float:
    """Live FP32 FFMA peak of this GPU (best of 3 probe launches, CUDA events)."""
    import ctypes
    from neurocell_b200 import _lib
    lib = _lib.load()
    sink = torch.zeros(1, device=device)
    flops = ctypes.c_double(0)
    st = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    best = 0.0
    for it in (2000, 20000, 20000, 20000):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        _lib.check(lib.nc_fp32_peak_probe(it, ctypes.byref(flops), ctypes.c_void_p(sink.data_ptr()), st),
                   "nc_fp32_peak_probe")
        e1.record()
        torch.cuda.synchronize()
        if it == 20000:
            best = max(best, flops.value / (e0.elapsed_time(e1) * 1e-3) / 1e12)
    return best


def cpu_baseline(steps_budget_s: float = 12.0) -> dict:
    """The torch-CPU port of the reference algorithm (float32, all host threads), timed on a
    bounded sample: full 128-sample train steps until the time budget is spent."""
    from oracle import torch_port as T
    from oracle import vnn_oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cell, filt, xs, ys = make_problem(0, 1, BATCH)
    g = O.alu_geometry()
    x, y = xs[0], ys[0]
    ports = [x[:, 0], x[:, 1], x[:, 2]]
    for _ in range(2):
        T.value_and_grad(g, O.Config(), cell, filt, ports, y, dtype=torch.float32)
    times = []
    t_end = time.perf_counter() + steps_budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        T.value_and_grad(g, O.Config(), cell, filt, ports, y, dtype=torch.float32)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": BATCH / med, "unit": "samples/s", "cores": threads, "kind": "port",
            "ms_per_step": med * 1e3,
            "sample": f"{len(times)} full B={BATCH} train steps (fwd+autograd bwd, float32) of "
                      f"oracle/torch_port.py on {threads} host threads, median"}


# ---------------------------------------------------------------------------------------
def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import torch_port as T
    from oracle import vnn_oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cell, filt, xs, ys = make_problem(0, 1, BATCH)
    g = O.alu_geometry()
    ports = [xs[0][:, 0], xs[0][:, 1], xs[0][:, 2]]
    for _ in range(args.warmup):
        T.value_and_grad(g, O.Config(), cell, filt, ports, ys[0], dtype=torch.float32)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        T.value_and_grad(g, O.Config(), cell, filt, ports, ys[0], dtype=torch.float32)
        times.append(time.perf_counter() - t0)
    sp = spread([1e3 * t for t in times])
    ms = sp["median"]
    val = BATCH / (ms * 1e-3)
    line = {
        "impl": "reference", "metric": METRIC, "value": val,
        "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "ms_spread": sp, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy ALU batches)",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": val, "unit": "samples/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} full B={BATCH} train steps of oracle/torch_port.py, "
                                   f"median, on {threads} host threads (one {BATCH}-sample batch of "
                                   f"the {BATCH * args.gpus}-sample global step; the reference's JAX "
                                   "CPU path is not installable here)"},
        "e2e": {"value": val, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args) -> None:
    import ctypes
    import torch.distributed as dist
    import neurocell_b200 as nc
    from neurocell_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        pg = dist.group.WORLD
    lib = _lib.load()

    nb = 8
    cell, filt, xs, ys = make_problem(rank, nb, BATCH)
    topo = nc.ChipTopology2D.alu_chip()
    params = nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev))
    spec, n_pix = None, 2000
    if args.adaptive:
        # the reference's adaptive-mask measurement (README stage 06/07): the pre-epoch mask
        # of a freshly initialised ALU chip, margin 4, buckets of 8 -> a 32x32 sub-ROI
        spec = nc.compute_adaptive_spatial_mask(nc.init_vnn_params(701, topo, device=dev), topo,
                                                margin=4, bucket_multiple=8)
        n_pix = spec.active_shape[0] * spec.active_shape[1]
    runner = nc.trainer.VNNTrainStep(topo, params, BATCH, lr=LR, in_shapes=((8, 1),) * 3,
                                     process_group=pg, exchange=args.exchange, conv=args.conv,
                                     spatial_mask=spec)
    x_dev = torch.tensor(xs.reshape(nb, BATCH, -1), device=dev)
    y_dev = torch.tensor(ys, device=dev)
    if not args.no_graph:
        runner.load_batch(x_dev[0], y_dev[0])
        runner.capture()            # the gradient exchange is captured too when world > 1
    l2_flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def barrier():
        if pg is not None:
            dist.barrier()

    # ---- warm-up
    for i in range(args.warmup):
        runner.step(x_dev[i % nb], y_dev[i % nb])
    torch.cuda.synchronize()

    # ---- timed region: device-resident batches, L2 flushed before every step
    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    kev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    for row in kev:            # torch creates the CUDA event on first record
        for e in row:
            e.record()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev)
    time.sleep(0.02)
    barrier()
    torch.cuda.synchronize()
    clocks.mark_start()
    for i in range(K):
        runner.load_batch(x_dev[i % nb], y_dev[i % nb])
        l2_flush.fill_(float(i))
        if runner.graph is None:
            lib.nc_set_profile_events(*(ctypes.c_void_p(e.cuda_event) for e in kev[i]))
        ev[i][0].record()
        runner.step()
        ev[i][1].record()
    lib.nc_set_profile_events(None, None, None, None)
    torch.cuda.synchronize()
    clocks.mark_stop()
    barrier()
    clk = clocks.stop()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    sp = spread(step_ms)
    ms = sp["median"]
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if pg is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = BATCH * world / (ms_max * 1e-3)

    # ---- fused-kernel durations (profile events; eager replays when the step is a graph)
    if runner.graph is not None:
        for i in range(min(K, 10)):
            runner.load_batch(x_dev[i % nb], y_dev[i % nb])
            l2_flush.fill_(float(i))
            lib.nc_set_profile_events(*(ctypes.c_void_p(e.cuda_event) for e in kev[i]))
            runner._launch()
        lib.nc_set_profile_events(None, None, None, None)
        torch.cuda.synchronize()
        kev = kev[:min(K, 10)]
    fwd_ms = statistics.median(e[0].elapsed_time(e[1]) for e in kev)
    xch_ms = exchange_ms(runner, 10, dev, pg)
    bwd_ms = statistics.median(e[2].elapsed_time(e[3]) for e in kev)

    # ---- end to end through the public API: pinned host batches in, the loss out to pinned
    # host memory, both inside the timed region.  A second train step with host_loss=True
    # (same initial parameters): one staging kernel reads each page-locked batch
    # (nc_stage_from_host), the loss kernel stores the loss into a page-locked host scalar.
    x_host = torch.tensor(xs.reshape(nb, BATCH, -1)).pin_memory()
    y_host = torch.tensor(ys).pin_memory()
    e2e_runner = nc.trainer.VNNTrainStep(
        topo, nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev)), BATCH,
        lr=LR, in_shapes=((8, 1),) * 3, process_group=pg, exchange=args.exchange, conv=args.conv,
        spatial_mask=spec, host_loss=True)
    if not args.no_graph:
        e2e_runner.load_batch(x_host[0], y_host[0])
        e2e_runner.capture()
    for i in range(args.warmup):
        e2e_runner.step(x_host[i % nb], y_host[i % nb])
    eev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    for i in range(K):
        l2_flush.fill_(float(i))
        eev[i][0].record()
        loss = e2e_runner.step(x_host[i % nb], y_host[i % nb])   # loss: page-locked host scalar
        eev[i][1].record()
    torch.cuda.synchronize()
    barrier()
    assert float(loss) == float(loss)                             # read on the host after the sync
    e2e_sp = spread([a.elapsed_time(b) for a, b in eev])
    e2e_ms = e2e_sp["median"]
    t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
    if pg is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item())
    bad = torch.tensor([max(runner.exchange_status(), e2e_runner.exchange_status())], dtype=torch.int32,
                       device=dev)
    if pg is not None:
        dist.all_reduce(bad, op=dist.ReduceOp.MAX)    # every rank takes the same exit
    if int(bad.item()) != 0:
        runner.graph = None
        e2e_runner.graph = None
        raise RuntimeError("NVLink gradient exchange: a peer timed out during the run")
    h2d = x_host[0].numel() * 4 + y_host[0].numel() * 4

    peak = fp32_peak_tflops(dev)
    flops_fwd = BATCH * 2.0 * 16 * n_pix * 299 * 4           # d forward passes
    flops_bwd = BATCH * 2.0 * 16 * n_pix * 299 * 7           # d dG + (d-1) dX passes
    path = lib.nc_conv_path(ctypes.byref(runner.plan.topo))
    names = {1: ("fast::fwd_kernel_mt<23, 13, 8>", "fast::bwd_kernel<23, 13>"),
             3: ("fftf_fwd_kernel", "fftf_bwd_kernel")}.get(path, ("forward kernels", "backward kernels"))
    dom = names[1] if bwd_ms >= fwd_ms else names[0]
    ach = (flops_bwd / (bwd_ms * 1e-3) if dom == names[1] else flops_fwd / (fwd_ms * 1e-3)) / 1e12

    if rank == 0:
        line = {
            "metric": (METRIC if spec is None else
                       "train samples/s (62x62 ALU VNN on its adaptive %dx%d sub-ROI, B=128 per GPU)"
                       % spec.active_shape), "value": value,
            "unit": "samples/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
            "ms_per_step": ms_max, "ms_spread": sp, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy ALU batches, random-init params as BASELINE config 0)",
            "config": workload_config(world),
            "run": {"cuda_graph": runner.graph is not None,
                    "grad_exchange": (args.exchange if world > 1 else "none"),
                    "conv": args.conv, "sub_roi": None if spec is None else list(spec.roi_bbox),
                    "timing": "median of per-step CUDA-event times on the launching stream, max over ranks"},
            "e2e": {"value": BATCH * world / (e2e_ms * 1e-3), "unit": "samples/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "ms_per_step": e2e_ms,
                    "ms_spread": e2e_sp},
            "gpu_launches": runner.launches_per_step() * K,
            "conv_path": {1: "direct per-sample kernels", 2: "FFT per-step kernels",
                          3: "fused per-sample FFT kernels"}.get(path, "?"),
            "kernels_ms": {names[0]: fwd_ms, names[1]: bwd_ms},
            **({"grad_exchange_ms": {"median_max_over_ranks": xch_ms, "share_of_step": xch_ms / ms_max,
                                     "how": "CUDA events around the exchange call, 10 eager steps "
                                            "after the timed region"}} if xch_ms is not None else {}),
            "roofline": {"bound": "fp32", "kernel": dom, "achieved": ach, "peak": peak,
                         "unit": "TFLOP/s", "frac": ach / peak if peak else None,
                         "work": "effective direct-convolution FLOPs (2*M*P*K per pass) per the "
                                 "reporting rule; the FFT kernels execute far fewer",
                         "peak_source": "live FFMA probe (nc_fp32_peak_probe); MEASURED_PEAKS.json has no FP32 figure",
                         "traffic": ncu_traffic(dom),
                         "traffic_source": "profiles/ncu_traffic.json (one ncu capture, dram read+write per launch)",
                         "fma_pipe_active_ncu": ncu_entry(dom, "fma_pipe_active"),
                         "issue_active_ncu": ncu_entry(dom, "issue_active")},
            "clocks": clk,
        }
        if path == 3:
            # what the FFT kernels really execute, beside the effective direct-convolution figure
            ef, eb = fftf_executed_flops(16, 40, 62, 23, 4)
            dom_ms = bwd_ms if dom == names[1] else fwd_ms
            ex = BATCH * (eb if dom == names[1] else ef) / (dom_ms * 1e-3) / 1e12
            line["roofline"].update(
                executed_tflops=ex, executed_frac=ex / peak if peak else None,
                executed_work="5 N log2 N per 64-point complex transform, 6 per complex product, "
                              "8 per complex multiply-accumulate (bench.py fftf_executed_flops)")
        tr = ncu_traffic(dom)
        if tr:
            # the same kernel against HBM: captured DRAM bytes per launch / its event time
            hp, hsrc = hbm_peak()
            dom_ms = bwd_ms if dom == names[1] else fwd_ms
            hgbs = tr / (dom_ms * 1e-3) / 1e9
            line["roofline"]["hbm"] = {"achieved": hgbs, "peak": hp, "unit": "GB/s", "frac": hgbs / hp,
                                       "peak_source": hsrc}
        if world == 1 and not args.no_cpu and spec is None:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    runner.release()                # graphs holding NCCL calls and the IPC maps go first
    e2e_runner.release()
    torch.cuda.synchronize()
    if pg is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------
# the other BASELINE configs (secondary measurements; the default run is config 0)
# ---------------------------------------------------------------------------------------
def hbm_peak() -> tuple[float, str]:
    """Measured HBM copy bandwidth of this pool (MEASURED_PEAKS.json), else the fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback (profiling recipe)"


def ncu_entry(kernel: str, key: str):
    """A figure of `kernel` from the committed ncu summary (profiles/ncu_traffic.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.json")) as f:
            return json.load(f).get(kernel, {}).get(key)
    except (OSError, ValueError):
        return None


def ncu_traffic(kernel: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, or None."""
    return ncu_entry(kernel, "bytes")


def config_problem(cfg: int, batch: int, seed_rank: int):
    """Topology and seeded synthetic data of BASELINE configs 1-4 (shapes, sizes and value
    distributions as the configs state; seeds cfg*1000 + {0 params, 1 filters, 2 inputs,
    3 targets})."""
    import neurocell_b200 as nc
    from oracle import vnn_oracle as O
    r = [np.random.default_rng([cfg * 1000 + k, seed_rank]) for k in range(4)]
    if cfg == 1:
        topo = nc.ChipTopology2D.alu_chip()
        cell = r[0].normal(0, 0.1, (3, 62, 62)).astype(np.float32)
        u = r[0].uniform(1e-6, 1 - 1e-6, (62, 62))
        cell[2] = np.log(u / (1 - u)).astype(np.float32)
        filt = (r[1].normal(0, 1, (16, 1, 23, 13)) / np.sqrt(299)).astype(np.float32)
        x, y, _ = O.alu_batch(r[2], batch, noise=0.0)
        return topo, ((8, 1),) * 3, cell, filt, x.reshape(batch, -1), y, dict(
            codd_mode="ste_ternary", loss="mse", train=False, K=23 * 13, M=16, P=2000, d=4)
    if cfg == 2:
        H, kh, M, d = 256, 31, 16, 8
        inp = nc.CoordinatePortSpec(tuple((rr, 64) for rr in range(96, 160)), "in")
        out = nc.CoordinatePortSpec(tuple((rr, 192) for rr in range(112, 144)), "out")
        topo = nc.ChipTopology2D.create((H, H), (kh, kh), M, d, (inp,), out, padding_mode="SAME")
        x = r[2].normal(size=(batch, 64)).astype(np.float32)
        y = r[3].integers(0, 2, size=(batch, 32)).astype(np.float32)
        shapes, P, loss = ((64,),), 256 * 256, "mse"
    elif cfg == 3:
        H, kh, M, d = 96, 15, 16, 6
        ports = tuple(nc.PortSpec((o, 32), (32, 32), f"in{i}") for i, o in enumerate((0, 32, 64)))
        out = nc.CoordinatePortSpec(tuple((rr, 80) for rr in range(43, 53)), "out")
        topo = nc.ChipTopology2D.create((H, H), (kh, kh), M, d, ports, out)
        x = r[2].normal(size=(batch, 3 * 32 * 32)).astype(np.float32)
        y = r[3].integers(0, 10, size=batch).astype(np.int32)
        shapes, P, loss = ((32, 32),) * 3, 82 * 82, "ce"
    else:
        H, kh, M, d = 1024, 63, 32, 8
        inp = nc.CoordinatePortSpec(tuple((rr, 128) for rr in range(448, 576)), "in")
        out = nc.CoordinatePortSpec(tuple((rr, 896) for rr in range(448, 576)), "out")
        topo = nc.ChipTopology2D.create((H, H), (kh, kh), M, d, (inp,), out)
        x = r[2].normal(size=(batch, 128)).astype(np.float32)
        y = r[3].normal(size=(batch, 128)).astype(np.float32)
        shapes, P, loss = ((128,),), 962 * 962, "mse"
    cell = r[0].normal(0, 0.1, (3, H, H)).astype(np.float32)
    filt = (r[1].normal(0, 1, (M, 1, kh, kh)) / kh).astype(np.float32)
    return topo, shapes, cell, filt, x, y, dict(
        codd_mode="annealed" if cfg == 4 else "continuous", loss=loss, train=True,
        K=kh * kh, M=M, P=P, d=d)


def run_config(args) -> None:
    """A BASELINE config other than 0 (secondary line, not the driver's bench line): CUDA-graph
    replays of the step with the L2 flushed before each, CUDA events, max over ranks.  Under
    torchrun the ranks train data-parallel with the gradient exchange in the graph: configs 2
    and 3 keep their batch per GPU (weak scaling), config 4 shards its batch of 16 over the
    GPUs (strong scaling, as BASELINE states); config 1 (inference) runs one replica per GPU."""
    import ctypes
    import torch.distributed as dist
    import neurocell_b200 as nc
    from neurocell_b200 import _lib, ops
    cfg = args.config
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
        pg = dist.group.WORLD
    B_total = args.batch or {1: 8192, 2: 64, 3: 256, 4: 16}[cfg]
    strong = cfg == 4
    if strong and B_total % world != 0:
        raise SystemExit(f"config 4 shards its batch of {B_total}; --gpus must divide it")
    B = B_total // world if strong else B_total
    topo, shapes, cell, filt, x, y, meta = config_problem(cfg, B, rank)
    if meta["train"]:
        cell, filt = config_problem(cfg, 1, 0)[2:4]       # every rank starts from the same params
    lib = _lib.load()
    conv = args.conv
    if meta["train"]:
        runner = nc.trainer.VNNTrainStep(
            topo, nc.VNNParams(torch.tensor(cell, device=dev), torch.tensor(filt, device=dev)), B,
            lr=LR, loss=meta["loss"], codd_mode=meta["codd_mode"], in_shapes=shapes, conv=conv,
            state_temperature=1.0, process_group=pg, exchange=args.exchange)
        runner.load_batch(torch.tensor(x, device=dev), torch.tensor(y, device=dev))
        step = runner.step
        if not args.no_graph:
            runner.capture()
        n_launch = None
    else:
        plan = ops.get_plan(topo, shapes, dev, "tanh", 0.0, "identity", 1.0, True, False, False, conv)
        cp, fl = torch.tensor(cell, device=dev), torch.tensor(filt, device=dev)
        xd = torch.tensor(x, device=dev)
        out = torch.empty((B, plan.n_out), device=dev)
        wsb = lib.nc_workspace_bytes(ctypes.byref(plan.topo), B, 0)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        codd = ops._codd(meta["codd_mode"], 1.0, 0.6)

        def launch():
            _lib.check(lib.nc_vnn_forward(ctypes.byref(plan.topo), ops._ptr(plan.buf), ops._ptr(cp),
                                          ops._ptr(fl), ops._ptr(xd), B, ctypes.byref(codd), 0,
                                          ops._ptr(out), ops._ptr(ws), wsb, ops._stream(dev)),
                       "nc_vnn_forward")
        n0 = lib.nc_launch_count()
        launch()
        n_launch = int(lib.nc_launch_count() - n0)
        graph = None
        if not args.no_graph:
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                launch()
            torch.cuda.current_stream(dev).wait_stream(s)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                launch()

        def step():
            if graph is not None:
                graph.replay()
            else:
                launch()
    l2_flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if pg is not None:
        dist.barrier()
        torch.cuda.synchronize()
    K = args.steps
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    clocks = ClockSampler(dev)
    time.sleep(0.02)
    clocks.mark_start()
    anneal = meta["train"] and meta["codd_mode"] == "annealed"
    for i in range(K):
        if anneal:       # tau 1.0 -> 0.1 over the steps (exponential)
            runner.set_temperature(nc.compute_annealed_temperature(i, K, 1.0, 0.1))
        l2_flush.fill_(float(i))
        ev[i][0].record()
        step()
        ev[i][1].record()
    torch.cuda.synchronize()
    clocks.mark_stop()
    clk = clocks.stop()
    ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    if pg is not None:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    xch_ms = exchange_ms(runner, 5, dev, pg) if meta["train"] else None
    M, P, Kk, d = meta["M"], meta["P"], meta["K"], meta["d"]
    passes = (3 * d - 1) if meta["train"] else d
    flops = 2.0 * M * P * Kk * passes * B
    zbytes = 4.0 * B * M * P * d * (5 if meta["train"] else 2)
    if cfg in (2, 4):
        peak, src = hbm_peak()
        roof = {"bound": "hbm", "achieved": zbytes / (ms * 1e-3) / 1e9, "peak": peak,
                "unit": "GB/s", "peak_source": src,
                "model": "5*|Z|*d bytes, |Z| = 4*B*M*P (reporting rule)"}
        roof["frac"] = roof["achieved"] / roof["peak"]
    else:
        peak = fp32_peak_tflops(dev)
        roof = {"bound": "fp32", "achieved": flops / (ms * 1e-3) / 1e12, "peak": peak,
                "unit": "TFLOP/s", "frac": flops / (ms * 1e-3) / 1e12 / peak,
                "model": "effective direct-convolution FLOPs 2*M*P*K per pass"}
    what = "train" if meta["train"] else "inference"
    line = {
        "metric": f"{what} samples/s (BASELINE config {cfg})", "value": B * world / (ms * 1e-3),
        "unit": "samples/s", "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "dtype": "f32", "data": "synthetic (seeded numpy, config shapes)",
        "config": {"workload": f"BASELINE config {cfg}" + (f" shapes at batch {B_total} (not the config's batch)"
                                                            if args.batch else ""),
                   "batch_per_gpu": B,
                   "global_batch": B * world, "conv": conv, "codd_mode": meta["codd_mode"],
                   "state_temperature": ("1.0 -> 0.1 over the timed steps (exponential)"
                                         if meta["codd_mode"] == "annealed" else 1.0),
                   "cuda_graph": not args.no_graph,
                   "parallelism": (f"dp{world}" if meta["train"] else f"{world} replicas"),
                   "grad_exchange": (args.exchange if world > 1 and meta["train"] else "none"),
                   "l2": "flushed (256 MB write) before every timed step"},
        "effective_tflops": flops / (ms * 1e-3) / 1e12, "roofline": roof, "clocks": clk,
        "gpu_launches_per_step": runner.launches_per_step() if meta["train"] else n_launch,
    }
    if xch_ms is not None:
        line["grad_exchange_ms"] = {"median_max_over_ranks": xch_ms, "share_of_step": xch_ms / ms,
                                    "how": "CUDA events around the exchange call, 5 eager steps after "
                                           "the timed region"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if meta["train"]:
        runner.release()           # graphs holding exchange calls and the IPC maps go first
    torch.cuda.synchronize()
    if pg is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--exchange", choices=("nccl", "nvlink"), default="nvlink",
                    help="data-parallel gradient exchange for --gpus > 1: the fused NVLink "
                         "peer-memory sum + SGD kernel (default) or NCCL all-reduce + SGD")
    ap.add_argument("--config", type=int, choices=(0, 1, 2, 3, 4), default=0,
                    help="BASELINE config; 1-4 print a secondary line (data parallel under torchrun)")
    ap.add_argument("--adaptive", action="store_true",
                    help="config 0 on the adaptive sub-ROI of a freshly initialised chip "
                         "(secondary measurement)")
    ap.add_argument("--conv", choices=("auto", "direct", "fft"), default="auto",
                    help="Green's convolution algorithm (nc_conv_algo)")
    ap.add_argument("--batch", type=int, default=0,
                    help="--config 1-4: batch in place of the config's own (reduced cases for "
                         "profiling; the line then names a batch the BASELINE config does not)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.config != 0:
        if args.impl == "b200":
            run_config(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
