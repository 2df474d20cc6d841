"""CPU, world size 2 (gloo): the multi-rank parts of bench.py -- the max-over-ranks timing reduction, per-rank seat
shards, and the reference arm under torchrun (rank 0 runs and prints one line; the other rank exits without work)."""
import json
import os
import subprocess
import sys

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, REPO)
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        v = bench.reduce_max(10.0 + 5.0 * rank, dist, torch.device("cpu"))
        lay = bench.layout_for_rank(2, rank, 16)
        out.put((rank, v, lay.ctx.tolist()))
    finally:
        dist.destroy_process_group()


def test_reduce_max_and_rank_shards_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29000 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [15.0, 15.0], "every rank must see the slowest rank's time"
    assert res[0][2] != res[1][2], "ranks must own different seats"
    assert all(200 <= c <= 1200 for r in res for c in r[2])


def test_reference_arm_under_torchrun_prints_once():
    port = 29500 + os.getpid() % 1000
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(port), os.path.join(REPO, "bench.py"), "--impl", "reference", "--gpus", "2",
           "--steps", "2", "--warmup", "1", "--cpu-seats", "4"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["cpu_baseline"]["kind"] == "port" and d["e2e"]["h2d_bytes_per_step"] == 0


def test_peaks_file_parsing(tmp_path):
    """The roofline denominator: the driver-written peaks file's HBM figure (top-level `hbm_gbs`, or an HBM entry one
    level down); absent, unreadable or without an HBM number means the fallback figure."""
    sys.path.insert(0, REPO)
    import bench
    p = tmp_path / "peaks.json"
    p.write_text(json.dumps({"hbm_gbs": 6541.2, "bf16_tflops": 1590.0}))
    assert bench.read_hbm_peak(str(p)) == 6541.2
    p.write_text(json.dumps({"hbm": {"gbs": 6400.0}, "bf16": {"tflops": 1500}}))
    assert bench.read_hbm_peak(str(p)) == 6400.0
    p.write_text(json.dumps({"bf16_tflops": 1590.0}))
    assert bench.read_hbm_peak(str(p)) is None
    p.write_text("not json")
    assert bench.read_hbm_peak(str(p)) is None
    assert bench.read_hbm_peak(str(tmp_path / "missing.json")) is None
