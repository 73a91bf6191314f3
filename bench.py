#!/usr/bin/env python3
"""Benchmark of the opt-125m int8 greedy decode step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: opt-125m (12 layers, d 768, 12 heads x 64, ReLU FFN 3072, vocab 50272) with
random-init weights N(0, 0.02), biases 0, LN identity (seed 0), int8 per-output-channel
weights, bf16 activations, fp32 accumulation; batch 1, a 32-token prompt of ids uniform in
[2, 50272), greedy decode.  A "step" is one decoded token: one launch of the persistent
decode kernel at one position; positions cycle through 32..159 (the config's 128 decoded
tokens).  Between timed steps an untimed write of a 256 MiB buffer flushes the 126 MB L2,
so every token streams its weights from HBM (the token's working set, 128 MB, is as large
as L2: an in-loop number would partly read L2; it is reported separately as
`l2_warm_ms_per_token`).  Each step is timed with CUDA events on the launching stream.

Multi-GPU: opt-125m at batch 1 does not shard; N GPUs run N independent replicas (one
process per GPU, torchrun), `value` = tokens of all replicas / max-over-ranks time.

`--impl reference` times the reference's CPU path for the same step: the oracle's
restatement of rust/npu-whisper/src/bin/opt125m_decode.rs with OPT_INT8 (the reference's
Rust cannot be built here), on all host threads, rank 0 only.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

PROMPT_LEN, N_NEW = 32, 128
METRIC = "opt-125m int8 greedy decode throughput (batch 1, L2 flushed per token)"
UNIT = "tokens/s"
HBM_PEAK_FALLBACK = 6650.0


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_PEAK_FALLBACK, "fallback"


class Clocks:
    """Sample SM clocks and throttle reasons with nvidia-smi during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows if len(r) >= 9
                          for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


def cpu_port_tokens_per_s(cfg, w, prompt, steps, nthreads):
    """The reference's host path (OPT_INT8, f32 activations, f32 LM head) restated in C,
    timed per decode step after an untimed prefill.  Returns (tokens/s, ms/token)."""
    from oracle import oracle as O
    m = O.OracleOpt(cfg, w, O.MODE_REF_F32, nthreads)
    nxt = 0
    for p in range(len(prompt)):
        nxt = m.step(prompt[p], p)
    pos = len(prompt)
    t0 = time.perf_counter()
    for i in range(steps):
        nxt = m.step(nxt, pos)
        pos += 1
    dt = time.perf_counter() - t0
    m.close()
    return steps / dt, dt * 1e3 / steps


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from xdna_engine_b200.synth import OPT_125M, make_opt_weights, make_prompt
    w = make_opt_weights(OPT_125M, seed=0)
    prompt = make_prompt(OPT_125M, PROMPT_LEN, seed=0)
    cores = os.cpu_count() or 1
    steps = max(1, min(args.steps, 16))
    cpu_port_tokens_per_s(OPT_125M, w, prompt[:4], max(1, args.warmup), cores)
    tps, ms = cpu_port_tokens_per_s(OPT_125M, w, prompt, steps, cores)
    sample = (f"{steps} greedy decode steps after a {PROMPT_LEN}-token prefill (positions "
              f"{PROMPT_LEN}..{PROMPT_LEN + steps - 1}), per-step timing")
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "opt-125m int8 greedy decode, batch 1, prompt 32, 128 new tokens",
                       "model": "opt-125m (random init N(0,0.02))"},
            "cpu_baseline": {"value": tps, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": tps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import xdna_engine_b200 as X
    from xdna_engine_b200.synth import OPT_125M, make_opt_weights, make_prompt
    cfg = OPT_125M
    w = make_opt_weights(cfg, seed=0)
    prompt = make_prompt(cfg, PROMPT_LEN, seed=0)
    max_ctx = PROMPT_LEN + N_NEW
    dev = X.Device(local)
    dec = X.OptDecoder(dev, cfg, w, max_ctx=max_ctx)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    # prefill (untimed): tokens[0..32) -> tokens[32]
    dec.set_tokens(prompt)
    dec.launch(0, PROMPT_LEN, PROMPT_LEN, stream=sp)
    dec.sync(sp)

    def step(i):
        pos = PROMPT_LEN + (i % (N_NEW - 1))
        dec.launch(pos, 1, PROMPT_LEN, stream=sp)

    for i in range(args.warmup):
        flush.fill_(i & 0xFF)
        step(i)
    dec.sync(sp)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        for i in range(args.steps):
            flush.fill_((i + 7) & 0xFF)
            starts[i].record(stream)
            step(args.warmup + i)
            ends[i].record(stream)
        torch.cuda.synchronize()
    dec.sync(sp)
    if world > 1:
        torch.distributed.barrier()
    per = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = float(sum(per))
    if world > 1:
        t = torch.tensor([total_ms], device="cuda", dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_tok = total_ms / args.steps

    # L2-warm in-loop figure: one launch decoding the 127 remaining positions
    dec.set_tokens(prompt)
    dec.launch(0, PROMPT_LEN, PROMPT_LEN, stream=sp)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    dec.launch(PROMPT_LEN, N_NEW - 1, PROMPT_LEN, stream=sp)
    e1.record(stream)
    dec.sync(sp)
    warm_ms = e0.elapsed_time(e1) / (N_NEW - 1)

    # end to end through the public call: pinned host prompt in, host ids out, prefill included
    pin_prompt = torch.from_numpy(prompt.copy()).pin_memory()
    pin_out = torch.empty(N_NEW, dtype=torch.int64).pin_memory()
    e2e_ms = []
    for r in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record(torch.cuda.default_stream())
        X.lib().xdna_opt_generate(dec.handle, pin_prompt.data_ptr(), PROMPT_LEN, N_NEW,
                                  pin_out.data_ptr(), None)
        b.record(torch.cuda.default_stream())
        torch.cuda.synchronize()
        e2e_ms.append(a.elapsed_time(b))
    e2e_tok_s = N_NEW / (min(e2e_ms) / 1e3) * world

    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    peak, peak_kind = peaks()
    ctx_mean = PROMPT_LEN + (N_NEW - 1) / 2.0
    kv_bytes = 36864.0 * ctx_mean          # K+V bf16 of all layers per cached position
    algo_bytes = dec.stream_bytes_per_token + kv_bytes
    achieved = algo_bytes / (ms_tok * 1e-3) / 1e9
    traffic = None
    tf = os.path.join(REPO, "profiles", "opt_decode_traffic.json")
    if os.path.exists(tf):
        traffic = json.load(open(tf)).get("dram_bytes_per_launch")
    from xdna_engine_b200.synth import OPT_125M as C_
    cores = os.cpu_count() or 1
    cpu_tps, cpu_ms = cpu_port_tokens_per_s(C_, w, prompt, 6, cores)
    line = {
        "metric": METRIC, "value": world * 1000.0 / ms_tok, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_tok,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (random-init N(0,0.02) weights, seeded prompt)",
        "config": {"workload": "opt-125m int8 greedy decode, batch 1, prompt 32, 128 new tokens",
                   "model": "opt-125m (random init N(0,0.02))", "global_batch": world,
                   "seq_len": PROMPT_LEN + N_NEW, "parallelism": f"replicas x{world}",
                   "l2": "flushed between steps (256 MiB write)", "grid_ctas": dec.grid},
        "ms_per_token": ms_tok, "l2_warm_ms_per_token": warm_ms,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": algo_bytes},
        "cpu_baseline": {"value": cpu_tps, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"6 decode steps after a {PROMPT_LEN}-token prefill"},
        "e2e": {"value": e2e_tok_s, "unit": UNIT, "h2d_bytes_per_step": PROMPT_LEN * 8,
                "d2h_bytes_per_step": N_NEW * 8,
                "step": "one xdna_opt_generate call: 32-token prefill + 128 greedy tokens"},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
