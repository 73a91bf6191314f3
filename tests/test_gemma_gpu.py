"""Gemma-3 decoder (xdna_gemma_*) against the oracle (npu-gemma pieces + the HF Gemma-3 model,
int8 Lin rule), single GPU and tensor parallel over 2 GPUs when the box has them.

The engine feeds f16 activations to its int8 GEMVs (the oracle: f32) and keeps the KV cache
in bf16, so the greedy stream is compared token by token only while the oracle's top-2 logit
margin exceeds the engine's expected error (the small test model's logits are ~0.08 rms;
tolerance 0.01)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG_KW = dict(n_layers=7, ffn=512, vocab=500, window=8)
PROMPT = list(range(2, 12))


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def model(X):
    cfg = X.GemmaConfig(**CFG_KW)
    return cfg, X.make_gemma_weights(cfg, seed=1, std=0.3, norm_std=0.5, embed_std=0.002)


def agree_until_close(got, want_t, want_l, tol=0.01):
    srt = np.sort(want_l, axis=1)
    for s in range(len(want_t)):
        if got[s] != want_t[s]:
            assert srt[s, -1] - srt[s, -2] < tol, (s, "token differs with a clear margin")
            return s
    return len(want_t)


def test_gemma_single_gpu_vs_oracle(X):
    from oracle import oracle as O
    cfg, w = model(X)
    dec = X.GemmaDecoder(X.Device(0), cfg, w, max_batch=4, max_ctx=64)
    wt, wl = O.gemma_decode(cfg, w, PROMPT, 12, int8=True, want_logits=True)
    got = dec.generate(np.array([PROMPT]), 12)[0]
    n = agree_until_close(got, wt, wl)
    assert n >= 4, (got, wt)
    # all 12 tokens, teacher-forced: each GPU choice within 0.15 logit-rms of the oracle's best
    gaps, _ = tf_gaps(cfg, w, PROMPT, got)
    assert gaps.max() <= 0.15, gaps
    # three streams with different prompts: each equals its own single-stream run
    prompts = np.array([PROMPT, list(range(20, 30)), list(range(40, 50))])
    batch = dec.generate(prompts, 12)
    for b in range(3):
        assert np.array_equal(batch[b], dec.generate(prompts[b:b + 1], 12)[0])
    dec.close()


@pytest.mark.parametrize("B", [20, 40])
def test_gemma_many_streams_vs_oracle(X, B):
    """More than 16 streams run the tcgen05 GEMV (32 or 64 accumulator columns): every stream
    against its own oracle run.  A stream may leave the oracle's sequence only where the
    oracle's top-2 margin is below the tolerance; with many streams a few meet such a near-tie
    early, so 90 % must agree for at least 4 tokens."""
    from oracle import oracle as O
    cfg, w = model(X)
    dec = X.GemmaDecoder(X.Device(0), cfg, w, max_batch=B, max_ctx=64)
    rng = np.random.default_rng(B)
    prompts = rng.integers(2, cfg.vocab, (B, 10))
    got = dec.generate(prompts, 12)
    lens = []
    for b in range(B):
        wt, wl = O.gemma_decode(cfg, w, list(prompts[b]), 12, int8=True, want_logits=True)
        lens.append(agree_until_close(got[b], wt, wl))     # any earlier split is a near-tie
    assert sum(n >= 4 for n in lens) >= 0.9 * B, lens
    dec.close()


def tf_gaps(cfg, w, prompt, toks):
    """The oracle teacher-forced on the GPU's tokens: per step, how far below the oracle's best
    logit the GPU's choice lies, in units of that step's logit rms (0 where they agree)."""
    from oracle import oracle as O
    wt, wl = O.gemma_decode(cfg, w, list(prompt), len(toks), int8=True, want_logits=True, force=toks)
    gaps = []
    for s in range(len(toks)):
        l = wl[s].astype(np.float64)
        gaps.append(float((l.max() - l[int(toks[s])]) / np.sqrt((l * l).mean())))
    return np.array(gaps), wt


def test_gemma_baseline_config_long_prompt(X):
    """The BASELINE shapes (26 layers, d 1152, vocab 262,144, window 512, 5 local : 1 global) with
    a 600-token prompt, so the local layers' 512-slot ring wraps and the global layers attend
    past the window, then 16 greedy tokens.  The GPU never stores the 262,144 logits (the argmax
    is fused into the LM-head GEMV), so the logits are compared through the oracle teacher-forced
    on the GPU's tokens: every GPU token's oracle logit is within 0.05 logit-rms of the oracle's
    best (f16 activations and a bf16 KV cache against f32), and most tokens are the oracle's own
    argmax."""
    cfg = X.GEMMA3_1B
    w = X.make_gemma_weights(cfg, seed=2)
    rng = np.random.default_rng(2)
    prompt = rng.integers(2, cfg.vocab, 600)
    dec = X.GemmaDecoder(X.Device(0), cfg, w, max_batch=1, max_ctx=640)
    got = dec.generate(prompt[None, :], 16)[0]
    dec.close()
    gaps, wt = tf_gaps(cfg, w, prompt, got)
    print("gemma 1B gaps (logit rms):", np.round(gaps, 4).tolist())
    assert gaps.max() <= 0.05, gaps
    assert (gaps == 0).sum() >= 12, gaps


def test_gemma_rejects_bad_input(X):
    cfg, w = model(X)
    with pytest.raises(X.XdnaError):
        X.GemmaDecoder(X.Device(0), X.GemmaConfig(**{**CFG_KW, "d_model": 1024}), w)
    dec = X.GemmaDecoder(X.Device(0), cfg, w, max_batch=1, max_ctx=16)
    with pytest.raises(X.XdnaError):
        dec.generate(np.array([PROMPT]), 12)          # beyond max_ctx
    with pytest.raises(X.XdnaError):
        dec.generate(np.array([[1, 999]]), 2)         # token outside the vocabulary
    dec.close()


def _tp_worker(rank, world, port, q):
    import os
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    import xdna_engine_b200 as X
    cfg, w = model(X)
    dec = X.GemmaDecoder(X.Device(rank), cfg, w, max_batch=2, max_ctx=64, tp_rank=rank, tp_size=world)
    hs = [None] * world
    dist.all_gather_object(hs, dec.ipc_handle())
    dec.connect(hs)
    dist.barrier()
    toks = dec.generate(np.array([PROMPT, list(range(20, 30))]), 12)
    dist.barrier()
    q.put((rank, toks))
    dec.close()
    dist.destroy_process_group()


def test_gemma_tensor_parallel_2gpu(X):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    assert np.array_equal(res[0], res[1]), "ranks disagree"
    # all 12 tokens of both streams: the tensor-parallel sums add the ranks' partials in rank
    # order (not the single GPU's order), so a token may differ from the single-GPU run only
    # at a near tie; checked against the oracle teacher-forced on the TP tokens
    cfg, w = model(X)
    for b, pr in enumerate([PROMPT, list(range(20, 30))]):
        gaps, _ = tf_gaps(cfg, w, pr, res[0][b])
        assert gaps.max() <= 0.15, (b, gaps)
