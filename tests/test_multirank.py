"""The multi-process (N > 1) host paths of bench.py on CPU: world-size-2 gloo groups.

* max_over_ranks: every rank gets the slowest rank's time (the bench's max-over-ranks rule).
* the reference arm under a 2-rank torchrun launch: rank 0 alone prints exactly one JSON line
  (impl "reference", n_gpus 2), the other rank exits 0 without output.
* the Gemma tensor-parallel split and merge arithmetic, restated in numpy over gloo ranks."""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
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


# --------------------------------------------------------------- Gemma tensor-parallel split
# A numpy restatement of how the Gemma decoder shards one layer over P ranks (gemma.cu, create:
# rank r holds the o-projection input rows [r*QD/P, (r+1)*QD/P) and the q heads covering them,
# the ffn columns [r*F/P, (r+1)*F/P) of gate and up with the matching down rows, and the
# vocabulary rows [r*ceil(V/P), ...) of the LM head) and merges it (partial sums added in rank
# order on every rank; per-stream (max logit, lowest index) gathered and reduced the same way),
# run as gloo ranks: every rank must hold identical bits, equal to the unsharded layer's within
# f32 reassociation.
def _gelu_tanh(x):
    return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))


def _tp_layer(rank, P, ctx, xn, xf, wo, wg, wu, wd, lm, HD):
    QD, F, V = wo.shape[0], wg.shape[1], lm.shape[1]
    k_loc = QD // P
    k0 = rank * k_loc
    h0, h1 = k0 // HD, (k0 + k_loc + HD - 1) // HD
    assert h0 * HD <= k0 and k0 + k_loc <= h1 * HD      # the rank's heads cover its o slice
    o_part = ctx[:, k0:k0 + k_loc] @ wo[k0:k0 + k_loc]
    f_loc = F // P
    f0 = rank * f_loc
    h = _gelu_tanh(xn @ wg[:, f0:f0 + f_loc]) * (xn @ wu[:, f0:f0 + f_loc])
    d_part = h @ wd[f0:f0 + f_loc]
    v_loc = -(-V // P)
    v0 = rank * v_loc
    v_loc = min(v_loc, V - v0)
    lg = xf @ lm[:, v0:v0 + v_loc]
    best_i = lg.argmax(axis=1)                          # first max = lowest index in the slice
    best_v = lg[np.arange(lg.shape[0]), best_i]
    return o_part.astype(np.float32), d_part.astype(np.float32), best_v.astype(np.float32), (best_i + v0)


def _tp_data(seed=5, B=3, QD=512, HD=256, D=96, F=160, V=1001):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32) * 0.2
    return dict(ctx=f(B, QD), xn=f(B, D), xf=f(B, D), wo=f(QD, D), wg=f(D, F), wu=f(D, F), wd=f(F, D),
                lm=f(D, V), HD=HD)


def _tp_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    d = _tp_data()
    o, dn, bv, bi = _tp_layer(rank, world, **d)
    outs = []
    for part in (o, dn):
        allp = [torch.zeros_like(torch.from_numpy(part)) for _ in range(world)]
        dist.all_gather(allp, torch.from_numpy(part))
        s = allp[0].numpy().copy()
        for r in range(1, world):                       # rank order, the same on every rank
            s = (s + allp[r].numpy()).astype(np.float32)
        outs.append(s)
    vs = [torch.zeros(len(bv)) for _ in range(world)]
    is_ = [torch.zeros(len(bi), dtype=torch.int64) for _ in range(world)]
    dist.all_gather(vs, torch.from_numpy(bv))
    dist.all_gather(is_, torch.from_numpy(bi.astype(np.int64)))
    best = []
    for b in range(len(bv)):                            # value order, then the lowest index
        cand = [(float(vs[r][b]), -int(is_[r][b])) for r in range(world)]
        best.append(-max(cand)[1])
    dist.destroy_process_group()
    q.put((rank, outs[0].tobytes(), outs[1].tobytes(), best))


@pytest.mark.parametrize("world", [2, 4])
def test_gemma_tp_split_and_merge_gloo(world):
    """world 4: each rank's o slice is half a head (the q heads cover it), the vocabulary splits
    unevenly (1001 rows)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    _, o0, d0, b0 = res[0]
    for _, o1, d1, b1 in res[1:]:
        assert o0 == o1 and d0 == d1 and b0 == b1       # identical bits on every rank
    d = _tp_data()
    o_full = d["ctx"] @ d["wo"]
    h = _gelu_tanh(d["xn"] @ d["wg"]) * (d["xn"] @ d["wu"])
    d_full = h @ d["wd"]
    np.testing.assert_allclose(np.frombuffer(o0, np.float32).reshape(o_full.shape), o_full, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(np.frombuffer(d0, np.float32).reshape(d_full.shape), d_full, rtol=1e-5, atol=1e-5)
    assert b0 == (d["xf"] @ d["lm"]).argmax(axis=1).tolist()
