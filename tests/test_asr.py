"""The Whisper ASR scenario behind npu_transcribe (rust/npu-engine/src/asr/whisper.rs:682-745).

CPU: the detokenizer (xdna_bpe_decode) against the HuggingFace `tokenizers` library on a
Whisper-shaped byte-level BPE tokenizer.json (50,257 BPE tokens, the special tokens at the
reference's ids 50257..50363 -- <|endoftext|>, <|startoftranscript|>, 99 language tags,
<|transcribe|>, <|notimestamps|> -- and 1,501 timestamp tokens), on random id sequences that
mix specials, timestamps and byte fragments that form invalid UTF-8.  GPU: npu_model_load on an
ASR scenario in the reference's npy layout and npu_transcribe, against the same pipeline
assembled from the xdna_* objects in Python with the reference's control logic (language
detection over 50259..50357, prompt [SOT, lang, TRANSCRIBE, NOTIMESTAMPS], greedy to EOT, at most
200 tokens) and the HuggingFace decode, trimmed as Rust's str::trim."""
import ctypes as C
import dataclasses
import json
import os

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOT, EOT, TRANSCRIBE, NOTS = 50258, 50257, 50359, 50363
LANG_LO, LANG_HI = 50259, 50357


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def make_tokenizer(path):
    from tokenizers import Tokenizer, decoders, models
    from tokenizers.pre_tokenizers import ByteLevel
    alpha = sorted(ByteLevel.alphabet())
    rng = np.random.default_rng(0)
    vocab = {c: i for i, c in enumerate(alpha)}
    words = ["Ġthe", "Ġa", "ing", "Ġtranscript", "Ġhello", "Ġworld", ".", ",", "ĠB", "200"]
    for w in words:
        vocab.setdefault(w, len(vocab))
    while len(vocab) < 50257:
        n = int(rng.integers(2, 6))
        w = "".join(alpha[int(i)] for i in rng.integers(0, 256, n))
        vocab.setdefault(w, len(vocab))
    tok = Tokenizer(models.BPE(vocab=vocab, merges=[]))
    tok.decoder = decoders.ByteLevel()
    langs = [f"<|l{i}|>" for i in range(99)]
    specials = ["<|endoftext|>", "<|startoftranscript|>"] + langs + ["<|translate|>", "<|transcribe|>",
                                                                     "<|startoflm|>", "<|startofprev|>",
                                                                     "<|nocaptions|>", "<|notimestamps|>"]
    tok.add_special_tokens(specials)
    tok.add_tokens([f"<|{0.02 * i:.2f}|>" for i in range(1501)])
    assert tok.token_to_id("<|notimestamps|>") == NOTS and tok.get_vocab_size() == 51865
    tok.save(str(path))
    return tok


# Rust's str::trim (Unicode White_Space); Python's str.strip also strips U+001C..U+001F
_WS = set([0x20, 0x85, 0xa0, 0x1680, 0x2028, 0x2029, 0x202f, 0x205f, 0x3000] + list(range(9, 14)) +
          list(range(0x2000, 0x200b)))


def rust_trim(s):
    b, e = 0, len(s)
    while b < e and ord(s[b]) in _WS:
        b += 1
    while e > b and ord(s[e - 1]) in _WS:
        e -= 1
    return s[b:e]


def ours(X, path, ids, skip=True):
    ids = np.ascontiguousarray(ids, np.int64)
    n = X.lib().xdna_bpe_decode(str(path).encode(), ids.ctypes.data, ids.size, int(skip), None, 0)
    assert n >= 0, X.last_error()
    buf = C.create_string_buffer(n + 1)
    X.lib().xdna_bpe_decode(str(path).encode(), ids.ctypes.data, ids.size, int(skip), buf, n + 1)
    return buf.raw[:n].decode("utf-8")


def test_bpe_decode_matches_hf_tokenizers(X, tmp_path):
    tok = make_tokenizer(tmp_path / "tokenizer.json")
    rng = np.random.default_rng(1)
    cases = [[], [SOT, 50300, TRANSCRIBE, NOTS], [SOT, 256 + 0, 256 + 1, 256 + 2, EOT], [51000, 51864, 257]]
    for _ in range(300):
        n = int(rng.integers(1, 40))
        kind = rng.random()
        if kind < 0.3:      # single bytes: random fragments of multi-byte UTF-8
            ids = rng.integers(0, 256, n)
        elif kind < 0.6:
            ids = rng.integers(0, 51865, n)
        else:
            ids = np.concatenate([[SOT, int(rng.integers(LANG_LO, LANG_HI + 1)), TRANSCRIBE, NOTS],
                                  rng.integers(0, 50257, n)])
        cases.append([int(v) for v in ids])
    for ids in cases:
        for skip in (True, False):
            assert ours(X, tmp_path / "tokenizer.json", ids, skip) == tok.decode(ids, skip_special_tokens=skip), ids


def test_bpe_decode_errors(X, tmp_path):
    ids = np.zeros(1, np.int64)
    assert X.lib().xdna_bpe_decode(str(tmp_path / "missing.json").encode(), ids.ctypes.data, 1, 1, None, 0) == -1
    assert "No such file" in X.last_error()


def _write_asr_scenario(X, root, n_enc=2, n_dec=2):
    from xdna_engine_b200.synth import WhisperDecConfig, make_whisper_dec_weights, make_whisper_enc_weights
    ecfg = X.WhisperEncConfig(n_layers=n_enc)
    we = make_whisper_enc_weights(ecfg, seed=3, bias_std=0.02, ln_std=0.05)
    dcfg = WhisperDecConfig(n_layers=n_dec)
    wd = make_whisper_dec_weights(dcfg, seed=4, bias_std=0.02, ln_std=0.05)
    ws = root / "artifacts" / "whisper-small"

    def save(rel, a):
        p = ws / (rel + ".npy")
        p.parent.mkdir(parents=True, exist_ok=True)
        np.save(p, np.ascontiguousarray(a, np.float32))

    enc_names = {"ln1_w": "ln1.weight", "ln1_b": "ln1.bias", "q_w": "q.weight", "q_b": "q.bias",
                 "k_w": "k.weight", "k_b": "k.bias", "v_w": "v.weight", "v_b": "v.bias", "out_w": "out.weight",
                 "out_b": "out.bias", "ln2_w": "ln2.weight", "ln2_b": "ln2.bias", "fc1_w": "fc1.weight",
                 "fc1_b": "fc1.bias", "fc2_w": "fc2.weight", "fc2_b": "fc2.bias"}
    for i, ly in enumerate(we["layers"]):
        for k, n in enc_names.items():
            a = ly[k] if ly.get(k) is not None else np.zeros(768, np.float32)
            save(f"L{i}/{n}", a)
    for k, n in (("conv1_w", "conv1.weight"), ("conv1_b", "conv1.bias"), ("conv2_w", "conv2.weight"),
                 ("conv2_b", "conv2.bias"), ("embed_positions", "embed_positions")):
        save(f"conv/{n}", we[k])
    save("refs/ln_post.weight", we["ln_post_w"])
    save("refs/ln_post.bias", we["ln_post_b"])
    for k, n in (("embed_tokens", "embed_tokens"), ("embed_positions", "embed_positions"),
                 ("proj_out", "proj_out.weight"), ("ln_post_w", "ln_post.weight"), ("ln_post_b", "ln_post.bias")):
        save(f"whisper_decoder/{n}", wd[k])
    dec_names = {"ln_self_w": "ln_self.weight", "ln_self_b": "ln_self.bias", "ln_cross_w": "ln_cross.weight",
                 "ln_cross_b": "ln_cross.bias", "ln_final_w": "ln_final.weight", "ln_final_b": "ln_final.bias"}
    for p in ("q", "k", "v", "out", "cross_q", "cross_k", "cross_v", "cross_out", "fc1", "fc2"):
        dec_names[f"{p}_w"] = f"{p}.weight"
        dec_names[f"{p}_b"] = f"{p}.bias"
    for i, ly in enumerate(wd["layers"]):
        for k, n in dec_names.items():
            a = ly.get(k)
            if a is None:   # k biases absent in Whisper: zeros
                a = np.zeros(768, np.float32)
            save(f"whisper_decoder/L{i}/{n}", a)
    tok = make_tokenizer(ws / "tokenizer.json")
    scen = root / "whisper.toml"
    scen.write_text(f"""[scenario]
kind = "asr"
name = "whisper-small"

[model]
hidden = 768
ff = 3072
n_heads = 12
head_dim = 64
n_layers = {n_enc}
max_seq = 1500

[artifacts]
weights = "artifacts/whisper-small"
""")
    return scen, ecfg, we, dcfg, wd, tok


@pytest.mark.gpu
def test_npu_transcribe_end_to_end(X, tmp_path, monkeypatch):
    scen, ecfg, we, dcfg, wd, tok = _write_asr_scenario(X, tmp_path)
    monkeypatch.chdir(tmp_path)
    L = X.lib()
    L.npu_model_load.restype = C.c_void_p
    L.npu_model_load.argtypes = [C.c_char_p]
    L.npu_transcribe.restype = C.c_void_p
    L.npu_transcribe.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_uint32]
    L.npu_string_free.argtypes = [C.c_void_p]
    L.npu_model_free.argtypes = [C.c_void_p]
    L.npu_model_kind.argtypes = [C.c_void_p]
    L.npu_embed.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
    L.npu_last_error.restype = C.c_char_p
    m = L.npu_model_load(str(scen).encode())
    assert m, L.npu_last_error()
    dev = X.Device(0)
    enc = X.WhisperEncoder(dev, ecfg, we, max_batch=1)
    dec = X.WhisperDecoder(dev, dcfg, wd, max_batch=1)
    lm = L.xdna_log_mel_create(dev.handle)
    try:
        assert L.npu_model_kind(m) == 0
        assert L.npu_embed(m, None, None, 0) == -1
        assert L.npu_last_error() == b"model is not an embedder"
        rng = np.random.default_rng(5)
        t = np.arange(16000 * 4) / 16000.0
        clips = [(5000 * np.sin(2 * np.pi * 300 * t) + 800 * rng.standard_normal(t.size)).astype(np.int16),
                 np.zeros(0, np.int16), (3000 * rng.standard_normal(16000 * 31)).astype(np.int16)]
        for pcm in clips:
            pcm = np.ascontiguousarray(pcm)
            r = L.npu_transcribe(m, pcm.ctypes.data if pcm.size else None, pcm.size, 16000)
            assert r, L.npu_last_error()
            got = C.string_at(r).decode("utf-8")
            L.npu_string_free(r)
            # the same pipeline from the parts, with the reference's control logic
            mel = np.zeros((1, 80, 3000), np.float32)
            assert L.xdna_log_mel(lm, pcm.ctypes.data if pcm.size else None, pcm.size, mel.ctypes.data) == 0
            e = enc.encode(mel)
            _, lg = dec.generate(e, [SOT], 1, want_logits=True)
            block = lg[0, 0, LANG_LO:LANG_HI + 1]
            lang = LANG_LO + int(np.argmax(block))          # first maximum
            toks = dec.generate(e, [SOT, lang, TRANSCRIBE, NOTS], 200)[0]
            ids = [SOT, lang, TRANSCRIBE, NOTS]
            for v in toks:
                if v == EOT:
                    break
                ids.append(int(v))
            want = rust_trim(tok.decode(ids, skip_special_tokens=True))
            assert got == want, (got[:80], want[:80])
        assert L.npu_transcribe(m, None, 0, 8000) is None
        assert L.npu_last_error() == b"unsupported: sample_rate 8000 (need 16000)"
    finally:
        L.xdna_log_mel_free(lm)
        L.npu_model_free(m)


def test_asr_scenario_errors(X, tmp_path, monkeypatch):
    """Non-Whisper ASR scenarios are refused; a missing weight directory fails at load with the
    reference's "load failed: " prefix (no device needed for either)."""
    L = X.lib()
    L.npu_model_load.restype = C.c_void_p
    L.npu_last_error.restype = C.c_char_p
    monkeypatch.chdir(tmp_path)
    body = '[scenario]\nkind = "asr"\nname = "{n}"\n[model]\nhidden = 768\nff = 3072\nn_heads = 12\nhead_dim = 64\n' \
           'n_layers = 2\nmax_seq = 1500\n[artifacts]\nweights = "nowhere"\n'
    p = tmp_path / "pk.toml"
    p.write_text(body.format(n="parakeet-tdt-0.6b-v3"))
    assert L.npu_model_load(str(p).encode()) is None
    assert L.npu_last_error().startswith(b"unsupported: ASR model")
