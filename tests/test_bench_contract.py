"""bench.py's reference arm keeps the driver's JSON-line contract (host cores only, no GPU):
one line from rank 0 with the B200 arm's metric, a cpu_baseline and an e2e object with no
host-device traffic; other ranks and the secondary --config lines print nothing."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _run(args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [line for line in r.stdout.splitlines() if line.strip()]


def test_reference_arm_line():
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "3"])
    assert len(lines) == 1
    d = json.loads(lines[0])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "samples/s"
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"] == bench.workload_config(1)     # the B200 arm's config, key for key
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_other_ranks_print_nothing():
    assert _run(["--impl", "reference", "--steps", "1", "--warmup", "3", "--gpus", "2"],
                env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []


def test_reference_arm_has_no_secondary_config_lines():
    assert _run(["--impl", "reference", "--config", "2"]) == []


def _rank_max(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, bench.max_over_ranks(1.5 + rank, "cpu")))
    finally:
        dist.destroy_process_group()


def test_multi_gpu_helpers_on_gloo_ranks():
    """The max-over-ranks reduction behind the multi-GPU timings (step time and gradient
    exchange), run by two gloo ranks on the host; exchange_ms is None without a group."""
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_max, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert got == {0: 2.5, 1: 2.5}
    assert bench.exchange_ms(None, 3, "cpu", None) is None
