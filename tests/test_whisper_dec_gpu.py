"""Whisper-small greedy decoder (xdna_whisper_dec_*) against the oracle's restatement of the
reference's HostDecoder (whisper_decoder.rs), given the bfp16 weights the engine computes with.

The engine rounds GEMV inputs, the KV caches and the encoder states to bf16 (the reference's
fused NPU path does the same); the oracle is f32.  Attention scores grow with the square of
the weight scale, and a sharp softmax amplifies the bf16 rounding, so the test weights use
std 0.05 (scores of a few units).  Logits are compared with an absolute tolerance of
0.05 * rms(logits), and the greedy streams must agree until the oracle's top-2 margin at
some step falls below twice that tolerance."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def bfp_cols(w):
    """bfp16 along K (rows of a [K, N] weight) for every output column, as the engine stores
    it: 8-bit mantissas, so a block holding both +128 and -128 keeps +128 as 127 (a block
    holding only +128 is stored negated and stays exact)."""
    from oracle import oracle as O
    wt = np.ascontiguousarray(w.T)
    q = O.bfp16_blocks(wt).reshape(-1, 8)
    mx = np.abs(wt.reshape(-1, 8)).max(1)
    mx[mx == 0] = 1.0
    e = np.floor(np.log2(mx)).astype(np.int32)
    e = np.where(np.ldexp(1.0, e + 1) <= mx, e + 1, e)        # exact floor(log2) (as frexp)
    e = np.where(np.ldexp(1.0, e) > mx, e - 1, e)
    quantum = np.ldexp(np.float32(1.0), e - 6).astype(np.float32)[:, None]
    m = np.rint(q / quantum)
    both = (m == 128).any(1) & (m == -128).any(1)
    m[both] = np.where(m[both] == 128, 127, m[both])
    q = (m * quantum).astype(np.float32)
    return np.ascontiguousarray(q.reshape(wt.shape).T)


def engine_weights(w):
    q = dict(w)
    q["proj_out"] = bfp_cols(w["proj_out"])
    q["layers"] = []
    for ly in w["layers"]:
        d = dict(ly)
        for k in ("q", "k", "v", "out", "cross_q", "cross_k", "cross_v", "cross_out", "fc1", "fc2"):
            d[k + "_w"] = bfp_cols(ly[k + "_w"])
        q["layers"].append(d)
    return q


def check(got_t, got_l, want_t, want_l):
    rms = np.sqrt((want_l.astype(np.float64) ** 2).mean())
    tol = 0.05 * rms
    B, n = want_t.shape
    for b in range(B):
        for s in range(n):
            srt = np.sort(want_l[b, s])
            np.testing.assert_allclose(got_l[b, s], want_l[b, s], atol=tol, rtol=0)
            if got_t[b, s] != want_t[b, s]:
                assert srt[-1] - srt[-2] < 2 * tol, (b, s, "token differs with a clear margin")
                break                                   # later steps follow different histories


def test_whisper_decoder_small_vs_oracle(X):
    from oracle import oracle as O
    cfg = X.WhisperDecConfig(n_layers=2, vocab=1000, n_enc=200, max_tgt=64)
    w = X.make_whisper_dec_weights(cfg, seed=3, std=0.05, bias_std=0.02, ln_std=0.05)
    enc = X.make_encoder_states(cfg, 3, seed=3)
    dec = X.WhisperDecoder(X.Device(0), cfg, w, max_batch=4)
    prompt = [1, 5, 7]
    toks, lg = dec.generate(enc, prompt, 24, want_logits=True)
    wt, wl = O.whisper_decode(cfg, engine_weights(w), enc, prompt, 24, want_logits=True)
    assert len(set(wt.ravel().tolist())) > 8, "degenerate stream"
    check(toks, lg, wt, wl)
    # the second run replays the recorded graph: same bits
    t2, l2 = dec.generate(enc, prompt, 24, want_logits=True)
    assert np.array_equal(t2, toks) and np.array_equal(l2, lg)
    # one stream alone equals the same stream inside the batch
    t1, l1 = dec.generate(enc[1:2], prompt, 24, want_logits=True)
    assert np.array_equal(t1[0], toks[1])
    dec.close()


def test_whisper_decoder_full_shapes(X):
    """whisper-small shapes (12 layers, vocab 51865, 1500 encoder positions), 2 streams, a few
    tokens after the 4-token task prompt."""
    from oracle import oracle as O
    cfg = X.WHISPER_SMALL_DEC
    w = X.make_whisper_dec_weights(cfg, seed=5, std=0.03, bias_std=0.02)
    enc = X.make_encoder_states(cfg, 2, seed=5)
    dec = X.WhisperDecoder(X.Device(0), cfg, w, max_batch=2)
    toks, lg = dec.generate(enc, X.WHISPER_PROMPT, 4, want_logits=True)
    wt, wl = O.whisper_decode(cfg, engine_weights(w), enc, X.WHISPER_PROMPT, 4, want_logits=True)
    check(toks, lg, wt, wl)
    dec.close()


def test_whisper_decoder_bad_input(X):
    cfg = X.WhisperDecConfig(n_layers=1, vocab=512, n_enc=64, max_tgt=16)
    dec = X.WhisperDecoder(X.Device(0), cfg, X.make_whisper_dec_weights(cfg), max_batch=1)
    enc = X.make_encoder_states(cfg, 1)
    with pytest.raises(X.XdnaError):
        dec.generate(enc, [1, 2, 3], 20)          # beyond max_tgt
    with pytest.raises(X.XdnaError):
        dec.generate(enc, [1, 600], 4)            # token outside the vocabulary
    with pytest.raises(X.XdnaError):
        dec.generate(np.concatenate([enc, enc]), [1], 2)   # batch beyond max_batch
    dec.close()


def test_whisper_decoder_baseline_config(X):
    """The BASELINE shapes (12 layers, vocab 51865, 1500 encoder positions), 2 streams, 36 greedy
    tokens after the task prompt.  The oracle is teacher-forced on the GPU's tokens, so every
    step's logits are comparable: relative L2 <= 1e-2 at every step (bf16 activations against
    f32), and every step where the argmaxes differ is a near tie (the oracle's top-2 margin is
    below that step's largest |logit difference|; whisper.rs:749-757 first-max rule)."""
    from oracle import oracle as O
    cfg = X.WHISPER_SMALL_DEC
    w = X.make_whisper_dec_weights(cfg, seed=6, std=0.03, bias_std=0.02)
    enc = X.make_encoder_states(cfg, 2, seed=6)
    dec = X.WhisperDecoder(X.Device(0), cfg, w, max_batch=2)
    n = 36
    toks, lg = dec.generate(enc, X.WHISPER_PROMPT, n, want_logits=True)
    dec.close()
    wt, wl = O.whisper_decode(cfg, engine_weights(w), enc, X.WHISPER_PROMPT, n, want_logits=True,
                              force=toks)
    worst = 0.0
    for b in range(2):
        for s in range(n):
            g, r = lg[b, s].astype(np.float64), wl[b, s].astype(np.float64)
            rel = np.linalg.norm(g - r) / np.linalg.norm(r)
            worst = max(worst, rel)
            assert rel <= 1e-2, (b, s, rel)
            if wt[b, s] != toks[b, s]:
                srt = np.sort(r)
                assert srt[-1] - srt[-2] < np.abs(g - r).max(), (b, s, "flip with a clear margin")
    print("whisper dec worst rel-L2", worst)


def test_continuous_batching_matches_single_streams(X):
    """Continuous batching (xdna_whisper_dec_set_encoder_slot / step_slots): four streams with
    their own prompts and encoder states join three slots at different steps, run at their own
    positions (each self-attention spans only its own tokens), leave when done, and a later
    stream reuses a freed slot.  Every stream's greedy tokens equal its own single-stream run
    (xdna_whisper_dec_generate, batch 1) bit for bit, and so do its logits."""
    from xdna_engine_b200.synth import WhisperDecConfig, make_encoder_states, make_whisper_dec_weights
    cfg = WhisperDecConfig(n_layers=2)
    w = make_whisper_dec_weights(cfg, seed=6, bias_std=0.02, ln_std=0.05)
    encs = make_encoder_states(cfg, 4, seed=6)
    prompts = [[50258, 50259, 50359, 50363], [50258, 50260, 50359], [50258, 50261, 50359, 50363], [50258, 50262]]
    n_new = 10
    single = X.WhisperDecoder(X.Device(0), cfg, w, max_batch=1)
    want, want_lg = [], []
    for s in range(4):
        t, lg = single.generate(encs[s:s + 1], prompts[s], n_new, want_logits=True)
        want.append(t[0].tolist())
        want_lg.append(lg[0])
    single.close()

    dec = X.WhisperDecoder(X.Device(0), cfg, w, max_batch=3)
    joins = {0: (0, 0), 3: (1, 1), 5: (2, 2)}           # step -> (stream, slot)
    slot_of = {}
    state = {}                                          # stream -> [pos, generated, logits rows]
    free_after = {}
    step = 0
    while len(state) < 4 or any(len(v[1]) < n_new for v in state.values()):
        if step in joins:
            s, slot = joins[step]
            dec.set_encoder_slot(slot, encs[s])
            slot_of[slot] = s
            state[s] = [0, [], []]
        tokens = np.zeros(3, np.int64)
        positions = np.full(3, -1, np.int32)
        for slot, s in slot_of.items():
            pos, gen, _ = state[s]
            tokens[slot] = prompts[s][pos] if pos < len(prompts[s]) else gen[-1]
            positions[slot] = pos
        nxt, lg = dec.step_slots(tokens, positions, want_logits=True)
        for slot, s in list(slot_of.items()):
            st_ = state[s]
            if st_[0] >= len(prompts[s]) - 1:
                st_[1].append(int(nxt[slot]))
                st_[2].append(lg[slot].copy())
            st_[0] += 1
            if len(st_[1]) == n_new:                   # done: the slot is free again
                del slot_of[slot]
                if 3 not in state:                     # stream 3 joins the first freed slot
                    joins[step + 1] = (3, slot)
        assert all(nxt[b] == -1 for b in range(3) if positions[b] < 0)
        step += 1
        assert step < 200
    dec.close()
    for s in range(4):
        assert state[s][1] == want[s], (s, state[s][1], want[s])
        np.testing.assert_array_equal(np.stack(state[s][2]), want_lg[s])
