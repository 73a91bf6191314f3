"""The multi-process (N > 1) host paths of bench.py on CPU: world-size-2 gloo groups.

* max_over_ranks: every rank gets the slowest rank's time (the bench's max-over-ranks rule).
* the reference arm under a 2-rank torchrun launch: rank 0 alone prints exactly one JSON line
  (impl "reference", n_gpus 2), the other rank exits 0 without output."""
import json
import os
import socket
import subprocess
import sys

import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _max_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path.insert(0, REPO)
    import bench
    got = bench.max_over_ranks(1.5 + 2.0 * rank, world, device="cpu")
    single = bench.max_over_ranks(7.0, 1)
    dist.destroy_process_group()
    q.put((rank, got, single))


def test_max_over_ranks_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_max_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == [(0, 3.5, 7.0), (1, 3.5, 7.0)]


def test_reference_arm_two_ranks_prints_one_line():
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--impl", "reference",
           "--workload", "whisper_dec", "--gpus", "2", "--steps", "1", "--warmup", "3"]
    out = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [json.loads(l) for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = lines[0]
    assert d["impl"] == "reference" and d["n_gpus"] == 2 and d["value"] > 0
    assert d["cpu_baseline"]["cores"] >= 1 and d["e2e"]["h2d_bytes_per_step"] == 0
