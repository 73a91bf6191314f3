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
        self.gpu, self.rows, self.proc, self.first = gpu, [], None, 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            # the sampler is live once its first row is in; only later rows are in the region
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5.0:
                time.sleep(0.01)
            self.first = len(self.rows)
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
        rows = self.rows[self.first:]
        sm = [float(r[1]) for r in rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9
                          for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


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


def max_over_ranks(value, world, device="cuda"):
    """The largest `value` over the ranks of the process group (the slowest rank's time);
    `value` itself when world == 1."""
    if world <= 1:
        return value
    import torch
    t = torch.tensor([float(value)], device=device, dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle as O
    from xdna_engine_b200.synth import OPT_125M, make_opt_weights, make_prompt
    w = make_opt_weights(OPT_125M, seed=0)
    prompt = make_prompt(OPT_125M, PROMPT_LEN, seed=0)
    cores = os.cpu_count() or 1
    # the GPU arm's timed steps decode positions PROMPT_LEN + warmup + i (i < steps, cycling
    # through the 127 decode positions); the reference times exactly those steps
    m = O.OracleOpt(OPT_125M, w, O.MODE_REF_F32, cores)
    nxt = 0
    for p_ in range(PROMPT_LEN):
        nxt = m.step(prompt[p_], p_)
    pos = PROMPT_LEN
    for i in range(args.warmup):
        nxt = m.step(nxt, pos)
        pos += 1
    t0 = time.perf_counter()
    first = pos
    for i in range(args.steps):
        if pos >= PROMPT_LEN + N_NEW - 1:          # the GPU arm cycles back to PROMPT_LEN
            m.close()
            m = O.OracleOpt(OPT_125M, w, O.MODE_REF_F32, cores)
            for p_ in range(PROMPT_LEN):
                nxt = m.step(prompt[p_], p_)
            pos = PROMPT_LEN
        nxt = m.step(nxt, pos)
        pos += 1
    dt = time.perf_counter() - t0
    m.close()
    tps, ms = args.steps / dt, dt * 1e3 / args.steps
    sample = (f"{args.steps} greedy decode steps after a {PROMPT_LEN}-token prefill and {args.warmup} "
              f"untimed steps (positions {first}..{first + args.steps - 1}, the GPU arm's timed positions)")
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "opt-125m int8 greedy decode, batch 1, prompt 32, 128 new tokens",
                       "model": "opt-125m (random init N(0,0.02))", "global_batch": 1,
                       "seq_len": PROMPT_LEN + N_NEW, "parallelism": "host threads",
                       "l2": "n/a (host)"},
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
    # The timed region is K single-token launches with an L2 flush before each (per-launch
    # CUDA events, flush excluded).  One region of K = 20 tokens lasts a few milliseconds, far
    # below the clock sampler's 200 ms period, so the region is repeated back to back until
    # about one second has passed; ms/token is the mean over every timed launch of every
    # repetition, and the clock samples fall inside the repetitions.
    reps = max(1, args.reps) if args.reps else 0
    per = []
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        t_start = time.time()
        rep = 0
        while True:
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            for i in range(args.steps):
                flush.fill_((i + 7 + rep) & 0xFF)
                starts[i].record(stream)
                step(args.warmup + i)
                ends[i].record(stream)
            torch.cuda.synchronize()
            per += [s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)]
            rep += 1
            if (reps and rep >= reps) or (not reps and time.time() - t_start > 1.0):
                break
    dec.sync(sp)
    if world > 1:
        torch.distributed.barrier()
    total_ms = float(sum(per)) / rep
    total_ms = max_over_ranks(total_ms, world)
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
    # parity against the reference's own host path, with the oracle as the checker: the GPU's
    # 128-token stream and logits vs opt125m_decode.rs (OPT_INT8) teacher-forced on it, and the
    # free-running reference stream's first divergence
    from oracle import oracle as O_
    g_ids = np.empty(N_NEW, np.int64)
    g_lg = np.empty((N_NEW, C_.vocab), np.float32)
    dec.set_tokens(prompt)
    X.lib().xdna_opt_generate(dec.handle, prompt.ctypes.data, PROMPT_LEN, N_NEW, g_ids.ctypes.data,
                              g_lg.ctypes.data)
    rep_ = O_.opt_parity_report(C_, w, prompt, g_ids, g_lg, cores)
    parity = {"reference": "opt125m_decode.rs host path (OPT_INT8: int8 Lin, f32 activations, f32 LM head)",
              "tokens": N_NEW, "tf_max_rel_l2": max(rep_["tf_rel_l2"]),
              "tf_argmax_flips": [{"step": f["step"], "ref_top2_margin": f["ref_margin"],
                                   "max_abs_logit_diff": f["max_abs_diff"]} for f in rep_["tf_flips"]],
              "free_first_divergence": rep_["free_first_div"], "free_divergence_margin": rep_["free_div_margin"],
              "free_match_rate": rep_["free_match"]}
    line = {
        "metric": METRIC, "value": world * 1000.0 / ms_tok, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_tok,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (random-init N(0,0.02) weights, seeded prompt)",
        "config": {"workload": "opt-125m int8 greedy decode, batch 1, prompt 32, 128 new tokens",
                   "model": "opt-125m (random init N(0,0.02))", "global_batch": world,
                   "seq_len": PROMPT_LEN + N_NEW, "parallelism": f"replicas x{world}",
                   "l2": "flushed between steps (256 MiB write)", "grid_ctas": dec.grid,
                   "timed_repetitions": rep},
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
        "parity": parity,
        "gpu_launches": args.steps * rep,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------------------ BGE-base
BGE_METRIC = "BGE-base embeddings throughput (batch 256, lengths U[32,512], CLS + L2)"


def bge_batch_flops(lens):
    """Valid-token FLOPs of one batch: 12 layers x (14,155,776 L + 3,072 L^2) per
    sequence -- the four projections/FFN GEMMs plus QK^T and PV."""
    L = np.asarray(lens, np.float64)
    return 12.0 * (14155776.0 * L.sum() + 3072.0 * (L * L).sum())


def bge_gemm_flops(T):
    return 12.0 * 14155776.0 * T


def run_bge_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from oracle import oracle as O
    from xdna_engine_b200.synth import BGE_BASE, make_bert_weights, make_bge_batch
    w = make_bert_weights(BGE_BASE, seed=0)
    ids, lens = make_bge_batch(256, seed=0)
    cores = os.cpu_count() or 1
    # bounded sample: the first 2 sequences of the batch, scaled by valid-token FLOPs
    n = 2
    s_ids, s_lens = ids[:int(lens[:n].sum())], lens[:n]
    O.bert_embed(BGE_BASE, w, s_ids[:int(s_lens[0])], s_lens[:1], cores)
    t0 = time.perf_counter()
    O.bert_embed(BGE_BASE, w, s_ids, s_lens, cores)
    dt = time.perf_counter() - t0
    seqs_s = 256.0 / (dt * bge_batch_flops(lens) / bge_batch_flops(s_lens))
    line = {"impl": "reference", "metric": BGE_METRIC, "value": seqs_s, "unit": "seqs/s",
            "n_gpus": args.gpus, "steps": 1, "warmup": 1, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "BGE-base embeddings, batch 256, lengths U[32,512]"},
            "cpu_baseline": {"value": seqs_s, "unit": "seqs/s", "cores": cores, "kind": "port",
                             "sample": f"{n} sequences (lengths {s_lens.tolist()}), throughput scaled "
                                       "to the batch by valid-token FLOPs"},
            "e2e": {"value": seqs_s, "unit": "seqs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_bge(args):
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import xdna_engine_b200 as X
    from xdna_engine_b200.synth import BGE_BASE, make_bert_weights, make_bge_batch
    w = make_bert_weights(BGE_BASE, seed=0)
    ids, lens = make_bge_batch(256, seed=rank)      # 256 sequences per GPU (weak scaling)
    T, B = int(lens.sum()), int(lens.size)
    dev = X.Device(local)
    m = X.BertEmbedder(dev, BGE_BASE, w, max_tokens=T, max_seqs=B)
    cu = np.zeros(B + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    tokpos = np.concatenate([np.arange(L, dtype=np.int32) for L in lens])
    d_ids, d_tp, d_cu = (torch.from_numpy(a).cuda() for a in (ids, tokpos, cu))
    out = torch.empty(B, 768, device="cuda")
    st = torch.cuda.current_stream()
    sp = st.cuda_stream
    maxlen = int(lens.max())

    def step():
        m.encode_device(d_ids.data_ptr(), d_tp.data_ptr(), d_cu.data_ptr(), T, B, maxlen, out.data_ptr(), sp)

    for _ in range(args.warmup):
        step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    with Clocks(local) as clk:
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world)
    assert X.lib().xdna_gemm_check() == 0, X.last_error()
    # dominant kernel: the tcgen05 GEMM, timed alone on this batch's four GEMM shapes
    A = torch.randn(T, 3072, device="cuda").to(torch.bfloat16)
    Bw = torch.randn(3072, 3072, device="cuda").to(torch.bfloat16) * 0.02
    Cb = torch.empty(T, 3072, device="cuda", dtype=torch.bfloat16)
    shapes = [(2304, 768, 0), (768, 768, 0), (3072, 768, 1), (768, 3072, 0)]
    g0, g1 = torch.cuda.Event(True), torch.cuda.Event(True)
    for rep in range(2):
        g0.record(st)
        for (N, K, gelu) in shapes:
            X.lib().xdna_gemm_bf16(A.data_ptr(), Bw.data_ptr(), None, None, Cb.data_ptr(), T, N, K, gelu, sp)
        g1.record(st)
        torch.cuda.synchronize()
    gemm_ms_layer = g0.elapsed_time(g1)
    gemm_tflops = (14155776.0 * T) / (gemm_ms_layer * 1e-3) / 1e12
    # end to end through xdna_bert_embed: host ids in, host embeddings out
    e2e = []
    host_out = pinned_like(shape=(B, 768), dtype=np.float32)
    host_ids, host_lens = pinned_like(ids), pinned_like(lens)
    for _ in range(3):
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda.synchronize()
        a.record(torch.cuda.default_stream())
        rc = X.lib().xdna_bert_embed(m.handle, host_ids.ctypes.data, host_lens.ctypes.data, B, host_out.ctypes.data)
        b.record(torch.cuda.default_stream())
        torch.cuda.synchronize()
        assert rc == 0, X.last_error()
        e2e.append(a.elapsed_time(b))
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    peaks_d = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(REPO, "MEASURED_PEAKS.json")) else {}
    peak = float(peaks_d.get("bf16_tflops", 1590.0))
    # CPU baseline: the oracle port on 1 sequence of the batch, scaled by FLOPs
    from oracle import oracle as O
    cores = os.cpu_count() or 1
    t0 = time.perf_counter()
    O.bert_embed(BGE_BASE, w, ids[:int(lens[0])], lens[:1], cores)
    dt = time.perf_counter() - t0
    cpu_seqs = B / (dt * bge_batch_flops(lens) / bge_batch_flops(lens[:1]))
    line = {
        "metric": BGE_METRIC, "value": world * B / (ms * 1e-3), "unit": "seqs/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) bf16 weights, seeded ids and lengths)",
        "config": {"workload": "BGE-base embeddings, batch 256 per GPU, lengths U[32,512] packed (no padding)",
                   "model": "BGE-base / BERT-base (random init)", "global_batch": world * B,
                   "tokens_per_gpu": T, "parallelism": f"dp{world} (independent batches, no collective)",
                   "l2": "activations (414 MB FFN hidden) and weights larger than L2"},
        "valid_token_tflops": bge_batch_flops(lens) / (ms * 1e-3) / 1e12,
        "roofline": {"bound": "tensor", "achieved": gemm_tflops, "peak": peak, "unit": "TFLOP/s",
                     "frac": gemm_tflops / peak, "traffic": None, "peak_kind": "measured burst bf16",
                     "kernel": "gemm_bf16_kernel (one layer's four GEMM shapes at this batch's T)"},
        "cpu_baseline": {"value": cpu_seqs, "unit": "seqs/s", "cores": cores, "kind": "port",
                         "sample": f"1 sequence (length {int(lens[0])}), scaled to the batch by valid-token FLOPs"},
        "e2e": {"value": world * B / (min(e2e) * 1e-3), "unit": "seqs/s", "h2d_bytes_per_step": int(T * 8 + (B + 1) * 4),
                "d2h_bytes_per_step": B * 768 * 4, "step": "one xdna_bert_embed call (host ids in, host embeddings out)"},
        "gpu_launches": args.steps * (2 + 12 * 7),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------- Whisper-small encoder
WHISPER_METRIC = "Whisper-small encoder throughput (30 s clips: mel 80x3000 -> 1500x768, batch 32)"
WHISPER_BATCH = 32


def whisper_clip_flops(n_layers=12):
    """FLOPs of one 30 s clip: conv stem (2*3000*768*240 + 2*1500*768*2304) plus per layer the
    four GEMMs (2*1500*768*9216) and attention QK^T + PV (4*1500^2*768)."""
    stem = 2.0 * 3000 * 768 * 240 + 2.0 * 1500 * 768 * 2304
    layer = 2.0 * 1500 * 768 * 9216 + 4.0 * 1500 * 1500 * 768
    return stem + n_layers * layer


def whisper_cpu_sample(cores):
    """The oracle on one clip with one block, scaled to the 12-block encoder by FLOPs."""
    from oracle import oracle as O
    from xdna_engine_b200.synth import WHISPER_SMALL_ENC, WhisperEncConfig, make_whisper_enc_weights, make_mel
    cfg = WhisperEncConfig(n_layers=1)
    w = make_whisper_enc_weights(cfg, seed=0)
    mel = make_mel(cfg, batch=1, seed=0)
    t0 = time.perf_counter()
    O.whisper_encode(cfg, w, mel, cores)
    dt = time.perf_counter() - t0
    return 1.0 / (dt * whisper_clip_flops(12) / whisper_clip_flops(1)), dt


def run_whisper_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    clips_s, dt = whisper_cpu_sample(cores)
    line = {"impl": "reference", "metric": WHISPER_METRIC, "value": clips_s, "unit": "clips/s",
            "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "Whisper-small encoder, 30 s clips"},
            "cpu_baseline": {"value": clips_s, "unit": "clips/s", "cores": cores, "kind": "port",
                             "sample": "1 clip through the conv stem and 1 of 12 blocks, scaled by FLOPs"},
            "e2e": {"value": clips_s, "unit": "clips/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_whisper(args):
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import xdna_engine_b200 as X
    from xdna_engine_b200.synth import WHISPER_SMALL_ENC as cfg, make_whisper_enc_weights, make_mel
    B = WHISPER_BATCH
    w = make_whisper_enc_weights(cfg, seed=0)
    mel = make_mel(cfg, batch=B, seed=rank)           # 32 clips per GPU (weak scaling)
    enc = X.WhisperEncoder(X.Device(local), cfg, w, max_batch=B)
    d_mel = torch.from_numpy(mel).cuda()
    out = torch.empty(B, 1500, 768, device="cuda", dtype=torch.bfloat16)
    st = torch.cuda.current_stream()
    sp = st.cuda_stream

    def step():
        enc.encode_device(d_mel.data_ptr(), B, out.data_ptr(), sp)

    for _ in range(args.warmup):
        step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    with Clocks(local) as clk:
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world)
    assert X.lib().xdna_gemm_check() == 0, X.last_error()
    # dominant kernel: the tcgen05 GEMM, timed alone on one block's four GEMM shapes at M = B*1500
    M = B * 1500
    A = torch.randn(M, 3072, device="cuda").to(torch.bfloat16)
    Bw = torch.randn(3072, 3072, device="cuda").to(torch.bfloat16) * 0.02
    Cb = torch.empty(M, 3072, device="cuda", dtype=torch.bfloat16)
    shapes = [(2304, 768, 0), (768, 768, 0), (3072, 768, 1), (768, 3072, 0)]
    g0, g1 = torch.cuda.Event(True), torch.cuda.Event(True)
    for rep in range(2):
        g0.record(st)
        for (N, K, gelu) in shapes:
            X.lib().xdna_gemm_bf16(A.data_ptr(), Bw.data_ptr(), None, None, Cb.data_ptr(), M, N, K, gelu, sp)
        g1.record(st)
        torch.cuda.synchronize()
    gemm_tflops = (2.0 * M * 768 * 9216) / (g0.elapsed_time(g1) * 1e-3) / 1e12
    del A, Bw, Cb
    # end to end through xdna_whisper_encode: host mel in, host f32 encodings out
    host_out = pinned_like(shape=(B, 1500, 768), dtype=np.float32)
    host_mel = pinned_like(mel)
    e2e = []
    for _ in range(3):
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda.synchronize()
        a.record(torch.cuda.default_stream())
        rc = X.lib().xdna_whisper_encode(enc.handle, host_mel.ctypes.data, B, host_out.ctypes.data)
        b.record(torch.cuda.default_stream())
        torch.cuda.synchronize()
        assert rc == 0, X.last_error()
        e2e.append(a.elapsed_time(b))
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    peaks_d = json.load(open(os.path.join(REPO, "MEASURED_PEAKS.json"))) if os.path.exists(
        os.path.join(REPO, "MEASURED_PEAKS.json")) else {}
    peak = float(peaks_d.get("bf16_tflops", 1590.0))
    cores = os.cpu_count() or 1
    cpu_clips, _ = whisper_cpu_sample(cores)
    line = {
        "metric": WHISPER_METRIC, "value": world * B / (ms * 1e-3), "unit": "clips/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights, bfp16 linears, mel ~ N(0,1))",
        "config": {"workload": "Whisper-small encoder, 32 clips of 30 s per GPU",
                   "model": "whisper-small encoder (random init)", "global_batch": world * B,
                   "parallelism": f"dp{world} (independent batches, no collective)",
                   "l2": "activations (295 MB FFN hidden) larger than L2"},
        "tflops": B * whisper_clip_flops() / (ms * 1e-3) / 1e12,
        "roofline": {"bound": "tensor", "achieved": gemm_tflops, "peak": peak, "unit": "TFLOP/s",
                     "frac": gemm_tflops / peak, "traffic": None, "peak_kind": "measured burst bf16",
                     "kernel": "gemm_bf16_kernel (one block's four GEMM shapes at M = 48000)"},
        "cpu_baseline": {"value": cpu_clips, "unit": "clips/s", "cores": cores, "kind": "port",
                         "sample": "1 clip through the conv stem and 1 of 12 blocks, scaled by FLOPs"},
        "e2e": {"value": world * B / (min(e2e) * 1e-3), "unit": "clips/s",
                "h2d_bytes_per_step": int(mel.nbytes), "d2h_bytes_per_step": int(host_out.nbytes),
                "step": "one xdna_whisper_encode call (host mel in, host f32 encodings out)"},
        "gpu_launches": args.steps * (4 + 12 * 7 + 1),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------ Parakeet FastConformer encoder
PARAKEET_METRIC = "Parakeet FastConformer encoder throughput (10 s clips: mel 128x1000 -> 125x1024, batch 64)"
PARAKEET_BATCH = 64


def parakeet_clip_ops(n_layers=24, T=125):
    """Operations of one clip: the subsample stem (conv.0 147.5 M, conv.2 36.9 M, conv.3 1049 M,
    conv.5 9.2 M, conv.6 262 M, out linear 1049 M) plus per block the int8 linears (2 T x 1024
    x 23552: two FFNs 4 x 4096, qkv 3072, out 1024, pw1 2048, pw2 1024) and attention (AC,
    rel-pos BD over 2T-1 positions, PV: 2 x 8 x 128 x (T^2 + T(2T-1) + T^2)).  The rel-pos projection pos_enc . W_pos
    does not depend on the input and is computed once per model, so it is not counted."""
    stem = 147_456_000 + 36_864_000 + 1_048_576_000 + 9_216_000 + 262_144_000 + 1_048_576_000
    layer = 2.0 * T * 1024 * 23552 + 2.0 * 8 * 128 * (T * T + T * (2 * T - 1) + T * T)
    return stem + n_layers * layer


def parakeet_cpu_sample(cores):
    """The oracle on one clip with one block, scaled to the 24-block encoder by operations."""
    from oracle import oracle as O
    from xdna_engine_b200.synth import ParakeetConfig, make_parakeet_weights, make_parakeet_mel
    cfg = ParakeetConfig(n_layers=1)
    w = make_parakeet_weights(cfg, seed=0)
    mel = make_parakeet_mel(cfg, 1, seed=0)
    t0 = time.perf_counter()
    O.parakeet_encode(cfg, w, mel, int8=True, nthreads=cores)
    dt = time.perf_counter() - t0
    return 1.0 / (dt * parakeet_clip_ops(24) / parakeet_clip_ops(1)), dt


def run_parakeet_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    clips_s, dt = parakeet_cpu_sample(cores)
    line = {"impl": "reference", "metric": PARAKEET_METRIC, "value": clips_s, "unit": "clips/s",
            "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": {"workload": "Parakeet FastConformer encoder, 10 s clips"},
            "cpu_baseline": {"value": clips_s, "unit": "clips/s", "cores": cores, "kind": "port",
                             "sample": "1 clip through the subsample stem and 1 of 24 blocks, scaled by operations"},
            "e2e": {"value": clips_s, "unit": "clips/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def int8_peak_tops():
    """Dense int8 throughput of cuBLASLt (torch._int_mm) on 8192^3: the measured denominator
    for the int8 GEMM (the driver's peaks file has no int8 figure)."""
    import torch
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(10):
        torch._int_mm(a, b)
    e1.record()
    torch.cuda.synchronize()
    return 2.0 * n ** 3 * 10 / (e0.elapsed_time(e1) * 1e-3) / 1e12


def run_parakeet(args):
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import xdna_engine_b200 as X
    from xdna_engine_b200.synth import PARAKEET_V3 as cfg, make_parakeet_weights, make_parakeet_mel
    B = PARAKEET_BATCH
    w = make_parakeet_weights(cfg, seed=0)
    mel = make_parakeet_mel(cfg, B, seed=rank)            # 64 clips per GPU (weak scaling)
    enc = X.ParakeetEncoder(X.Device(local), cfg, w, max_batch=B)
    T = enc.frames_out
    d_mel = torch.from_numpy(mel).cuda()
    out = torch.empty(B, T, 1024, device="cuda")
    st = torch.cuda.current_stream()
    sp = st.cuda_stream

    def step():
        enc.encode_device(d_mel.data_ptr(), B, out.data_ptr(), sp)

    for _ in range(args.warmup):
        step()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    with Clocks(local) as clk:
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world)
    assert X.lib().xdna_gemm_check() == 0, X.last_error()
    # dominant kernel: the int8 tcgen05 GEMM, timed alone on one block's eight linears at M = B*T
    M = B * T
    A = torch.randint(-127, 128, (M, 4096), dtype=torch.int8, device="cuda")
    Wt = torch.randint(-127, 128, (4096, 4096), dtype=torch.int8, device="cuda")
    sa = torch.full((B,), 0.01, device="cuda")
    ws = torch.full((4096,), 0.001, device="cuda")
    Cf = torch.empty(M, 4096, device="cuda")
    shapes = [(4096, 1024, 1), (1024, 4096, 0), (3072, 1024, 0), (1024, 1024, 0), (2048, 1024, 3),
              (1024, 1024, 0), (4096, 1024, 1), (1024, 4096, 0)]
    g0, g1 = torch.cuda.Event(True), torch.cuda.Event(True)
    for rep in range(2):
        g0.record(st)
        for (N, K, act) in shapes:
            X.lib().xdna_gemm_i8(A.data_ptr(), Wt.data_ptr(), sa.data_ptr(), T, ws.data_ptr(), None, act, None,
                                 1.0, Cf.data_ptr(), None, M, N, K, sp)
        g1.record(st)
        torch.cuda.synchronize()
    gemm_tops = (2.0 * M * 1024 * 23552) / (g0.elapsed_time(g1) * 1e-3) / 1e12
    peak = int8_peak_tops()
    del A, Wt, Cf
    # end to end through xdna_parakeet_encode: host mel in, host encodings out
    host_out = pinned_like(shape=(B, T, 1024), dtype=np.float32)
    host_mel = pinned_like(mel)
    e2e = []
    for _ in range(3):
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda.synchronize()
        a.record(torch.cuda.default_stream())
        rc = X.lib().xdna_parakeet_encode(enc.handle, host_mel.ctypes.data, B, host_out.ctypes.data)
        b.record(torch.cuda.default_stream())
        torch.cuda.synchronize()
        assert rc == 0, X.last_error()
        e2e.append(a.elapsed_time(b))
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    cores = os.cpu_count() or 1
    cpu_clips, _ = parakeet_cpu_sample(cores)
    line = {
        "metric": PARAKEET_METRIC, "value": world * B / (ms * 1e-3), "unit": "clips/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (random-init N(0,0.02) linears, fan-in scaled convs, mel ~ N(0,1))",
        "config": {"workload": "Parakeet FastConformer encoder (24 blocks, int8 linears), 64 clips of 10 s per GPU",
                   "model": "parakeet-tdt-0.6b-v3 encoder shapes (random init)", "global_batch": world * B,
                   "parallelism": f"dp{world} (independent batches, no collective)",
                   "l2": "activations (131 MB FFN hidden) larger than L2"},
        "tops": B * parakeet_clip_ops() / (ms * 1e-3) / 1e12,
        "roofline": {"bound": "tensor", "achieved": gemm_tops, "peak": peak, "unit": "TOP/s",
                     "frac": gemm_tops / peak, "traffic": None,
                     "peak_kind": "measured: cuBLASLt int8 (torch._int_mm) 8192^3 on this GPU",
                     "kernel": "gemm_kernel<I8> (one block's eight int8 linears at M = 8000)"},
        "cpu_baseline": {"value": cpu_clips, "unit": "clips/s", "cores": cores, "kind": "port",
                         "sample": "1 clip through the subsample stem and 1 of 24 blocks, scaled by operations"},
        "e2e": {"value": world * B / (min(e2e) * 1e-3), "unit": "clips/s",
                "h2d_bytes_per_step": int(mel.nbytes), "d2h_bytes_per_step": int(host_out.nbytes),
                "step": "one xdna_parakeet_encode call (host mel in, host f32 encodings out)"},
        "gpu_launches": args.steps * (6 + 24 * 21),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------- Whisper-small decoder
WDEC_METRIC = "Whisper-small greedy decode throughput (bfp16 weights, batch 32 streams, 224 tokens)"
WDEC_BATCH, WDEC_NEW = 32, 224


def wdec_bytes_per_step(B, ctx_mean):
    """HBM bytes of one token for B streams: bfp16 linears 12 x (3 + 1 + 1 + 1 + 4 + 4) x 768^2 x
    1.125 B, proj_out 51872 x 768 x 1.125 B, the cross K/V of every stream (12 x 1500 x 768 x 2 x
    2 B) and its self K/V cache (12 x ctx x 768 x 2 x 2 B)."""
    lin = 12 * 14 * 768 * 768 * 1.125
    lm = 51872 * 768 * 1.125
    return lin + lm + B * (12 * 1500 * 768 * 4 + 12 * ctx_mean * 768 * 4)


def wdec_cpu_sample(cores):
    from oracle import oracle as O
    from xdna_engine_b200.synth import WHISPER_SMALL_DEC, WHISPER_PROMPT, make_whisper_dec_weights, make_encoder_states
    w = make_whisper_dec_weights(WHISPER_SMALL_DEC, seed=0)
    enc = make_encoder_states(WHISPER_SMALL_DEC, 1, seed=0)
    n = 6
    t0 = time.perf_counter()
    O.whisper_decode(WHISPER_SMALL_DEC, w, enc, WHISPER_PROMPT, n, nthreads=cores)
    dt = time.perf_counter() - t0
    return n / dt, dt, n


def run_wdec_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    tps, dt, n = wdec_cpu_sample(cores)
    line = {"impl": "reference", "metric": WDEC_METRIC, "value": tps, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": dt * 1e3 / n,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "Whisper-small greedy decoder"},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"1 stream: cross K/V precompute + 4 prompt + {n} greedy tokens"},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_wdec(args):
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import xdna_engine_b200 as X
    from xdna_engine_b200.synth import WHISPER_SMALL_DEC as cfg, WHISPER_PROMPT, make_whisper_dec_weights, \
        make_encoder_states
    B, n_new = WDEC_BATCH, WDEC_NEW
    w = make_whisper_dec_weights(cfg, seed=0)
    enc = make_encoder_states(cfg, B, seed=rank)          # 32 streams per GPU (weak scaling)
    dec = X.WhisperDecoder(X.Device(local), cfg, w, max_batch=B)
    L = X.lib()
    st = torch.cuda.current_stream()
    sp = st.cuda_stream
    d_enc = torch.from_numpy(enc).cuda()
    toks = torch.empty(B, n_new, dtype=torch.int64, device="cuda")
    prompt = np.array(WHISPER_PROMPT, np.int64)
    assert L.xdna_whisper_dec_set_encoder(dec.handle, d_enc.data_ptr(), B, sp) == 0, X.last_error()

    def run(b, n):
        assert L.xdna_whisper_dec_run(dec.handle, b, prompt.ctypes.data, len(prompt), n, toks.data_ptr(), None,
                                      sp) == 0, X.last_error()

    for _ in range(max(1, args.warmup // 3)):
        run(B, n_new)                                      # records the graph, then replays it
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    steps = len(prompt) - 1 + n_new
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    with Clocks(local) as clk:
        e0.record(st)
        for _ in range(args.steps):
            run(B, n_new)
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world)
    ms_token = ms / steps
    # batch 1 (one stream) per-token latency, same graph machinery
    assert L.xdna_whisper_dec_set_encoder(dec.handle, d_enc.data_ptr(), 1, sp) == 0
    run(1, 64)
    run(1, 64)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record(st)
    run(1, 64)
    b.record(st)
    torch.cuda.synchronize()
    ms_token_b1 = a.elapsed_time(b) / (len(prompt) - 1 + 64)
    # end to end: host encoder states in (cross K/V precompute included), host tokens out
    host_tok = pinned_like(shape=(B, n_new), dtype=np.int64)
    host_enc = pinned_like(enc)
    e2e = []
    for _ in range(2):
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda.synchronize()
        a.record(torch.cuda.default_stream())
        assert L.xdna_whisper_dec_generate(dec.handle, host_enc.ctypes.data, B, prompt.ctypes.data, len(prompt), n_new,
                                           host_tok.ctypes.data, None) == 0, X.last_error()
        b.record(torch.cuda.default_stream())
        torch.cuda.synchronize()
        e2e.append(a.elapsed_time(b))
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    peak, peak_kind = peaks()
    ctx_mean = len(prompt) + n_new / 2.0
    bytes_step = wdec_bytes_per_step(B, ctx_mean)
    achieved = bytes_step / (ms_token * 1e-3) / 1e9
    cores = os.cpu_count() or 1
    cpu_tps, _, n_cpu = wdec_cpu_sample(cores)
    line = {
        "metric": WDEC_METRIC, "value": world * B * n_new / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bfp16 weights, bf16 activations",
        "data": "synthetic (random-init N(0,0.02) weights, encoder states ~ N(0,1))",
        "config": {"workload": "Whisper-small decoder, 32 streams x (4-token prompt + 224 greedy tokens) per GPU",
                   "model": "whisper-small decoder (random init)", "global_batch": world * B,
                   "parallelism": f"dp{world} (independent streams, no collective)",
                   "l2": "per-token working set (1.9 GB of cross K/V + weights) larger than L2"},
        "ms_per_token_b32": ms_token, "ms_per_token_b1": ms_token_b1,
        # bfp16 blocks whose mantissas needed both +128 and -128 (stored with +128 as 127): the
        # one place the weight storage can differ from the reference's block rule
        "bfp16_clamped_blocks": int(dec.clamped_blocks),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_token": bytes_step,
                     "kernel": "whole decode step (bfp16 GEMVs + cross attention over 1500 positions)"},
        "cpu_baseline": {"value": cpu_tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"1 stream: cross K/V precompute + 4 prompt + {n_cpu} greedy tokens"},
        "e2e": {"value": world * B * n_new / (min(e2e) * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": int(enc.nbytes), "d2h_bytes_per_step": int(host_tok.nbytes),
                "step": "one xdna_whisper_dec_generate call (host encoder states in, cross K/V + 227 steps, tokens out)"},
        "gpu_launches": args.steps * (1 + steps * 148),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# --------------------------------------------------------------------- Gemma-3-1B decode
GEMMA_METRIC = "Gemma-3-1B int8 greedy decode throughput (context 4096, batch 64, 256 tokens, TP = GPUs)"
GEMMA_BATCH, GEMMA_CTX, GEMMA_NEW = 64, 4096, 256


def gemma_bytes_per_step(B, ctx, tp):
    """HBM bytes of one token on one rank: its int8 linears (q | k | v rows of its heads, o, gate,
    up, down slices; K/V rows replicated) and LM-head rows with their f32 row scales, plus the
    K/V cache every stream reads (4 global layers x ctx + 22 local layers x 512 positions,
    x 256 x 2 x 2 bytes)."""
    D, F, V = 1152, 6912, 262144
    lin = 26 * (D * (1024 // tp + 512) + (1024 // tp) * D + 2 * D * (F // tp) + (F // tp) * D)
    lm = D * (V // tp)
    kv = 4 * ctx * 1024 + 22 * 512 * 1024
    return lin + lm + B * kv


def gemma_cpu_sample(cores):
    from oracle import oracle as O
    from xdna_engine_b200.synth import GEMMA3_1B, make_gemma_weights
    w = make_gemma_weights(GEMMA3_1B, seed=0)
    n = 3
    t0 = time.perf_counter()
    O.gemma_decode(GEMMA3_1B, w, list(range(100, 108)), n, int8=True, nthreads=cores)
    dt = time.perf_counter() - t0
    return (n + 7) / dt, dt, n


def run_gemma_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    tps, dt, n = gemma_cpu_sample(cores)
    line = {"impl": "reference", "metric": GEMMA_METRIC, "value": tps, "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": 1, "warmup": 0, "ms_per_step": 1e3 / tps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8 weights, f32",
            "data": "synthetic", "config": {"workload": "Gemma-3-1B greedy decode"},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"1 stream, 8-token prompt + {n} tokens: every step (prefill ones too) counted as a token"},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_gemma_case(B, ctx):
    """One xdna_gemma generate of B streams x ctx-token prompts + 4 tokens."""
    import xdna_engine_b200 as X
    from xdna_engine_b200.synth import GEMMA3_1B as cfg, make_gemma_weights
    dec = X.GemmaDecoder(X.Device(0), cfg, make_gemma_weights(cfg, seed=0), max_batch=B, max_ctx=ctx + 8)
    prompts = np.random.default_rng(0).integers(2, cfg.vocab, (B, ctx)).astype(np.int64)
    print(dec.generate(prompts, 4)[0], flush=True)


def run_case(args):
    """Profiling cases: a small, fixed piece of one workload run a few times on cuda:0 and nothing
    timed, so that an ncu capture (-k <kernel> -s <skip> -c <count>) of it is reproducible from
    committed code.  NAME:ARGS --
      gemm_bf16:M,N,K,act   three xdna_gemm_bf16 launches (act 0 none, 1 GELU)
      gemm_i8:M,N,K,act     three xdna_gemm_i8 launches (act 0 none, 1 SiLU, 3 GLU)
      ffn_fused:M           three xdna_ffn_fused_bf16 launches at the BGE FFN shape (768, 3072, 768)
      bge:S                 two BERT-base forwards of S sequences of lengths U[32,512]
      whisper:B             two Whisper-small encoder forwards of B clips
      parakeet:B            two Parakeet encoder forwards of B clips (eager, then the graph)
      whisper_dec:B         two Whisper-small decoder runs of B streams x 4 tokens
      decode:N              one opt-125m generation of N tokens after a 32-token prompt
      prefill:N             three batched prefills of N opt-125m prompt positions (prints the last's time)
      gemma:B,ctx           one Gemma-3-1B generate (B streams, ctx-token prompts, + 4 tokens)
      (a bare "B,ctx" is the gemma case)"""
    import torch
    name, _, rest = args.case.partition(":") if ":" in args.case else ("gemma", "", args.case)
    vals = [int(v) for v in rest.split(",") if v]
    torch.cuda.set_device(0)
    import xdna_engine_b200 as X
    L = X.lib()
    st = torch.cuda.current_stream()
    sp = st.cuda_stream
    if name == "gemma":
        run_gemma_case(*vals)
    elif name in ("gemm_bf16", "gemm_i8"):
        M, N, K, act = vals
        if name == "gemm_bf16":
            A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
            B = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
            C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            bias = torch.zeros(N, device="cuda")
            for _ in range(3):
                assert L.xdna_gemm_bf16(A.data_ptr(), B.data_ptr(), bias.data_ptr(), None, C.data_ptr(), M, N, K,
                                        act, sp) == 0, X.last_error()
        else:
            A = torch.randint(-127, 128, (M, K), device="cuda", dtype=torch.int8)
            B = torch.randint(-127, 128, (N, K), device="cuda", dtype=torch.int8)
            sa = torch.full((1,), 1e-3, device="cuda")
            ws = torch.full((N,), 1e-3, device="cuda")
            C = torch.empty(M, N // 2 if act == 3 else N, device="cuda")
            for _ in range(3):
                assert L.xdna_gemm_i8(A.data_ptr(), B.data_ptr(), sa.data_ptr(), M, ws.data_ptr(), None, act, None,
                                      1.0, C.data_ptr(), None, M, N, K, sp) == 0, X.last_error()
        torch.cuda.synchronize()
        assert L.xdna_gemm_check() == 0, X.last_error()
    elif name == "ffn_fused":
        M, = vals
        K, P, N = 768, 3072, 768
        A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        W1 = (torch.randn(P, K, device="cuda") * 0.03).to(torch.bfloat16)
        W2 = (torch.randn(N, P, device="cuda") * 0.02).to(torch.bfloat16)
        b1, b2 = torch.zeros(P, device="cuda"), torch.zeros(N, device="cuda")
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        for _ in range(3):
            assert L.xdna_ffn_fused_bf16(A.data_ptr(), W1.data_ptr(), b1.data_ptr(), 1, W2.data_ptr(), b2.data_ptr(),
                                         None, C.data_ptr(), None, M, K, P, N, sp) == 0, X.last_error()
        torch.cuda.synchronize()
        assert L.xdna_ffn_fused_check() == 0, X.last_error()
    elif name == "bge":
        S, = vals
        from xdna_engine_b200.synth import BGE_BASE, make_bert_weights, make_bge_batch
        ids, lens = make_bge_batch(S, seed=0)
        m = X.BertEmbedder(X.Device(0), BGE_BASE, make_bert_weights(BGE_BASE, seed=0), max_tokens=int(lens.sum()),
                           max_seqs=S)
        for _ in range(2):
            m.embed(ids, lens)
    elif name == "whisper":
        B, = vals
        from xdna_engine_b200.synth import WHISPER_SMALL_ENC as cfg, make_whisper_enc_weights, make_mel
        enc = X.WhisperEncoder(X.Device(0), cfg, make_whisper_enc_weights(cfg, seed=0), max_batch=B)
        d_mel = torch.from_numpy(make_mel(cfg, batch=B, seed=0)).cuda()
        out = torch.empty(B, 1500, 768, device="cuda", dtype=torch.bfloat16)
        for _ in range(2):
            enc.encode_device(d_mel.data_ptr(), B, out.data_ptr(), sp)
    elif name == "parakeet":
        B, = vals
        from xdna_engine_b200.synth import PARAKEET_V3 as cfg, make_parakeet_weights, make_parakeet_mel
        enc = X.ParakeetEncoder(X.Device(0), cfg, make_parakeet_weights(cfg, seed=0), max_batch=B)
        d_mel = torch.from_numpy(make_parakeet_mel(cfg, B, seed=0)).cuda()
        out = torch.empty(B, enc.frames_out, 1024, device="cuda")
        for _ in range(2):
            enc.encode_device(d_mel.data_ptr(), B, out.data_ptr(), sp)
    elif name == "whisper_dec":
        B, = vals
        from xdna_engine_b200.synth import WHISPER_SMALL_DEC as cfg, WHISPER_PROMPT, make_whisper_dec_weights, \
            make_encoder_states
        dec = X.WhisperDecoder(X.Device(0), cfg, make_whisper_dec_weights(cfg, seed=0), max_batch=B)
        d_enc = torch.from_numpy(make_encoder_states(cfg, B, seed=0)).cuda()
        toks = torch.empty(B, 4, dtype=torch.int64, device="cuda")
        prompt = np.array(WHISPER_PROMPT, np.int64)
        assert L.xdna_whisper_dec_set_encoder(dec.handle, d_enc.data_ptr(), B, sp) == 0, X.last_error()
        for _ in range(2):
            assert L.xdna_whisper_dec_run(dec.handle, B, prompt.ctypes.data, len(prompt), 4, toks.data_ptr(), None,
                                          sp) == 0, X.last_error()
    elif name == "decode":
        N, = vals
        from xdna_engine_b200.synth import OPT_125M, make_opt_weights, make_prompt
        dec = X.OptDecoder(X.Device(0), OPT_125M, make_opt_weights(OPT_125M, seed=0), max_ctx=32 + N + 1)
        print(dec.generate(make_prompt(OPT_125M, 32, seed=0), N)[:8], flush=True)
    elif name == "prefill":
        N, = vals
        from xdna_engine_b200.synth import OPT_125M, make_opt_weights, make_prompt
        dec = X.OptDecoder(X.Device(0), OPT_125M, make_opt_weights(OPT_125M, seed=0), max_ctx=N + 1)
        prompt = make_prompt(OPT_125M, N, seed=0)
        dec.set_tokens(prompt, 0, sp)
        for _ in range(3):
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record(st)
            dec.prefill(0, N, sp)
            b.record(st)
            torch.cuda.synchronize()
        dec.sync(sp)
        print(f"prefill of {N} positions: {a.elapsed_time(b):.3f} ms", flush=True)
    else:
        raise SystemExit(f"unknown case {name!r}")
    torch.cuda.synchronize()
    print(f"case {args.case}: ok", flush=True)


def run_gemma(args):
    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    import xdna_engine_b200 as X
    from xdna_engine_b200.synth import GEMMA3_1B as cfg, make_gemma_weights
    B, ctx, n_new = GEMMA_BATCH, GEMMA_CTX, GEMMA_NEW
    w = make_gemma_weights(cfg, seed=0)
    dec = X.GemmaDecoder(X.Device(local), cfg, w, max_batch=B, max_ctx=ctx + n_new, tp_rank=rank, tp_size=world)
    if world > 1:
        hs = [None] * world
        torch.distributed.all_gather_object(hs, dec.ipc_handle())
        dec.connect(hs)
        torch.distributed.barrier()
    L = X.lib()
    rng = np.random.default_rng(0)
    prompts = rng.integers(2, cfg.vocab, (B, ctx)).astype(np.int64)
    st = torch.cuda.current_stream()
    sp = st.cuda_stream
    assert L.xdna_gemma_begin(dec.handle, B, prompts.ctypes.data, ctx, n_new) == 0, X.last_error()
    assert L.xdna_gemma_steps(dec.handle, ctx - 1, sp) == 0, X.last_error()      # prefill, untimed
    warm = max(3, args.warmup)
    assert L.xdna_gemma_steps(dec.handle, warm, sp) == 0, X.last_error()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    steps = n_new - warm
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    with Clocks(local) as clk:
        e0.record(st)
        assert L.xdna_gemma_steps(dec.handle, steps, sp) == 0, X.last_error()
        e1.record(st)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    toks = np.empty((B, n_new), np.int64)
    assert L.xdna_gemma_tokens(dec.handle, toks.ctypes.data, sp) == 0, X.last_error()
    ms = max_over_ranks(ms, world)
    # batch 1 per-token latency at a short context, and the end-to-end call (host prompt in)
    p1 = prompts[:1, :64]
    assert L.xdna_gemma_begin(dec.handle, 1, p1.ctypes.data, 64, 64) == 0
    assert L.xdna_gemma_steps(dec.handle, 63 + 8, sp) == 0
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record(st)
    assert L.xdna_gemma_steps(dec.handle, 48, sp) == 0
    b.record(st)
    torch.cuda.synchronize()
    ms_b1 = a.elapsed_time(b) / 48
    out1 = np.empty((1, 64), np.int64)
    assert L.xdna_gemma_tokens(dec.handle, out1.ctypes.data, sp) == 0
    pe = prompts[:, :128].copy()
    oute = np.empty((B, 64), np.int64)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(True), torch.cuda.Event(True)
    a.record(torch.cuda.default_stream())
    assert L.xdna_gemma_generate(dec.handle, B, pe.ctypes.data, 128, 64, oute.ctypes.data, sp) == 0, X.last_error()
    b.record(torch.cuda.default_stream())
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b)
    if rank != 0:
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    peak, peak_kind = peaks()
    bytes_step = gemma_bytes_per_step(B, ctx + n_new // 2, world)
    achieved = bytes_step / (ms * 1e-3) / 1e9
    cores = os.cpu_count() or 1
    cpu_tps, _, n_cpu = gemma_cpu_sample(cores)
    line = {
        "metric": GEMMA_METRIC, "value": B / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 weights, f16 activations",
        "data": "synthetic (random-init N(0,0.02) weights, uniform prompt ids)",
        "config": {"workload": "Gemma-3-1B, 64 streams, 4096-token prompts (prefill untimed), 256 greedy tokens",
                   "model": "gemma-3-1b text decoder shapes (random init)", "global_batch": B,
                   "parallelism": f"tp{world} (q heads, FFN columns, vocab rows; rank-order all-reduce over peer memory)",
                   "l2": "per-token working set (1 GB weights + 1.8 GB KV) larger than L2"},
        "ms_per_token_b64": ms, "ms_per_token_b1_ctx64": ms_b1,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_kind": peak_kind, "algorithmic_bytes_per_token_per_rank": bytes_step,
                     "kernel": "whole decode step on rank 0"},
        "cpu_baseline": {"value": cpu_tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"1 stream, 8-token prompt + {n_cpu} tokens: every step counted as a token"},
        "e2e": {"value": B * 64 / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": int(pe.nbytes),
                "d2h_bytes_per_step": int(oute.nbytes),
                "step": "one xdna_gemma_generate call: 64 streams, 128-token prompts (prefill included) + 64 tokens"},
        # per step: embed, 26 x (qkv, q/k prep, attention, merge, o, norm, gate|up, down, norm),
        # LM head + argmax, unpack, pick; with TP also 2 all-reduces per layer and the gather
        "gpu_launches": steps * (1 + 26 * 9 + 3 + (26 * 2 + 1 if world > 1 else 0)),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def pinned_like(a=None, shape=None, dtype=None):
    """A numpy view of page-locked host memory (the e2e legs copy from and to pinned buffers),
    filled with `a` when given."""
    import torch
    if a is not None:
        shape, dtype = a.shape, a.dtype
    t = torch.empty(tuple(shape), dtype=torch.from_numpy(np.empty(0, dtype)).dtype, pin_memory=True)
    out = t.numpy()
    if a is not None:
        out[...] = a
    pinned_like.keep.append(t)
    return out


pinned_like.keep = []


def _time_ms(fn, st, reps=10, warm=3):
    import torch
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record(st)
    for _ in range(reps):
        fn()
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def run_kernel_bench(args):
    """Op-level timings behind the design notes (one GPU, CUDA events, inputs larger than L2):
      ffn_fused  -- the BGE FFN at M = 69,632 rows (K 768, P 3072, N 768, GELU): the fused
                    kernel against the unfused pair and each of its GEMMs
      attention  -- tcgen05 encoder attention for 32 Whisper clips (1500 positions) and a
                    256-sequence BGE batch (lengths U[32, 512])"""
    import torch
    torch.cuda.set_device(0)
    import xdna_engine_b200 as X
    L = X.lib()
    st = torch.cuda.current_stream()
    sp = st.cuda_stream
    reps = max(args.steps, 3) if args.steps > 0 else 10
    out = {}
    if args.workload == "ffn_fused":
        M, K, P, N = 69632, 768, 3072, 768
        A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        W1 = (torch.randn(P, K, device="cuda") * 0.03).to(torch.bfloat16)
        W2 = (torch.randn(N, P, device="cuda") * 0.02).to(torch.bfloat16)
        b1, b2 = torch.zeros(P, device="cuda"), torch.zeros(N, device="cuda")
        R = torch.randn(M, N, device="cuda").to(torch.bfloat16)
        H = torch.empty(M, P, device="cuda", dtype=torch.bfloat16)
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        up = lambda: L.xdna_gemm_bf16(A.data_ptr(), W1.data_ptr(), b1.data_ptr(), None, H.data_ptr(), M, P, K, 1, sp)
        down = lambda: L.xdna_gemm_bf16(H.data_ptr(), W2.data_ptr(), b2.data_ptr(), R.data_ptr(), C.data_ptr(), M, N,
                                        P, 0, sp)
        fused = lambda: L.xdna_ffn_fused_bf16(A.data_ptr(), W1.data_ptr(), b1.data_ptr(), 1, W2.data_ptr(),
                                              b2.data_ptr(), R.data_ptr(), C.data_ptr(), None, M, K, P, N, sp)
        fl = 2.0 * M * K * P
        t = {"fused": _time_ms(fused, st, reps), "up": _time_ms(up, st, reps), "down": _time_ms(down, st, reps),
             "unfused": _time_ms(lambda: (up(), down()), st, reps)}
        assert L.xdna_ffn_fused_check() == 0 and L.xdna_gemm_check() == 0, X.last_error()
        out = {"metric": "BGE FFN (M 69,632, K 768, P 3072, N 768, GELU) time", "value": t["fused"], "unit": "ms",
               "higher_is_better": False, "unfused_ms": t["unfused"], "up_ms": t["up"], "down_ms": t["down"],
               "fused_tflops": 2 * fl / t["fused"] / 1e9, "unfused_tflops": 2 * fl / t["unfused"] / 1e9,
               "up_tflops": fl / t["up"] / 1e9, "down_tflops": fl / t["down"] / 1e9}
    else:
        res = {}
        for name, lens in (("whisper32", [1500] * 32),
                           ("bge256", [int(v) for v in np.random.default_rng(0).integers(32, 513, 256)])):
            T = int(sum(lens))
            qkv = torch.randn(T, 2304, device="cuda").to(torch.bfloat16)
            cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device="cuda")
            ctx = torch.empty(T, 768, device="cuda", dtype=torch.bfloat16)
            ms = _time_ms(lambda: L.xdna_attention_bf16(qkv.data_ptr(), T, cu.data_ptr(), len(lens), max(lens),
                                                        ctx.data_ptr(), sp), st, reps)
            res[name] = (ms, sum(4.0 * l * l * 64 * 12 for l in lens) / ms / 1e9)
        assert L.xdna_attention_check() == 0, X.last_error()
        out = {"metric": "encoder attention time per layer (32 Whisper clips x 1500)", "value": res["whisper32"][0],
               "unit": "ms", "higher_is_better": False, "whisper32_tflops": res["whisper32"][1],
               "bge256_ms": res["bge256"][0], "bge256_tflops": res["bge256"][1]}
    out.update({"n_gpus": 1, "steps": reps, "warmup": 3, "dtype": "bf16", "data": "synthetic (random)",
                "config": {"workload": args.workload}})
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0, help="timed steps (default: about half a second of work)")
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--reps", type=int, default=0, help="decode: repetitions of the K-step timed region "
                    "(default: as many as fit in about one second, so the clock sampler sees them)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "bge", "whisper", "parakeet", "whisper_dec", "gemma", "ffn_fused",
                                           "attention"], default="decode")
    ap.add_argument("--case", default="", help="a profiling case NAME:ARGS (see run_case); nothing is timed")
    args = ap.parse_args()
    if args.case:
        run_case(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.workload in ("ffn_fused", "attention"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "op-level timing of this backend's kernels; "
                              "the reference has no counterpart to time"}))
            return
        run_kernel_bench(args)
    elif args.workload == "gemma":
        run_gemma_reference(args) if args.impl == "reference" else run_gemma(args)
    elif args.workload == "whisper_dec":
        if args.steps <= 0:
            args.steps = 3
        (run_wdec_reference if args.impl == "reference" else run_wdec)(args)
    elif args.workload == "parakeet":
        if args.steps <= 0:
            args.steps = 10
        (run_parakeet_reference if args.impl == "reference" else run_parakeet)(args)
    elif args.workload == "whisper":
        if args.steps <= 0:
            args.steps = 30
        (run_whisper_reference if args.impl == "reference" else run_whisper)(args)
    elif args.workload == "bge":
        if args.steps <= 0:
            args.steps = 30
        (run_bge_reference if args.impl == "reference" else run_bge)(args)
    elif args.impl == "reference":
        if args.steps <= 0:
            args.steps = 256
        run_reference(args)
    else:
        if args.steps <= 0:
            args.steps = 2048
        run_ours(args)


if __name__ == "__main__":
    main()
