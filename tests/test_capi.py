"""The reference's public C ABI (include/npu_engine.h, rust/npu-capi/include/npu_engine.h:28-103)
exported by the B200 library: a C program links against it and gets the reference's error
behaviour with no device (the port of rust/npu-capi/tests/c_smoke.rs:36-78); the embedding
front end tokenizes exactly like HuggingFace's BertTokenizer, which is what the reference's
tokenizer.json encodes (rust/npu-engine/src/bert/frontend.rs:29-35); and, on a GPU, npu_embed on a
scenario TOML + npy weight directory in the reference's layout (bert/weights.rs:25-70) matches the
oracle's host embedder."""
import ctypes as C
import dataclasses
import os
import subprocess

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(REPO, "xdna_engine_b200")


@pytest.fixture(scope="module")
def lib():
    from xdna_engine_b200 import _build
    _build.build()
    L = C.CDLL(os.path.join(LIBDIR, "libxdna_b200.so"))
    L.npu_last_error.restype = C.c_char_p
    L.npu_model_load.restype = C.c_void_p
    L.npu_model_load.argtypes = [C.c_char_p]
    L.npu_model_kind.argtypes = [C.c_void_p]
    L.npu_embed.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
    L.npu_model_free.argtypes = [C.c_void_p]
    L.npu_transcribe.restype = C.c_void_p
    L.npu_transcribe.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_uint32]
    L.xdna_wordpiece_encode.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_void_p, C.c_int]
    return L


C_SMOKE = r"""
#include "npu_engine.h"
#include <stdio.h>
#include <string.h>
int main(void) {
    int a = npu_available();
    const char *e = npu_last_error();
    printf("available=%d err=%s\n", a, e ? e : "(null)");
    if (npu_model_load(NULL) != NULL) return 2;
    printf("null_path=%s\n", npu_last_error());
    if (npu_model_load("/nonexistent/scenario.toml") != NULL) return 3;
    printf("missing=%s\n", npu_last_error());
    if (npu_model_kind(NULL) != -1) return 4;
    printf("kind_null=%s\n", npu_last_error());
    if (npu_embed(NULL, "x", NULL, 0) != -1) return 5;
    if (npu_transcribe(NULL, NULL, 0, 16000) != NULL) return 6;
    NpuRuntime *rt = npu_runtime_start("/nonexistent/engine.toml");   /* missing: empty config */
    if (rt == NULL) return 7;
    char *js = npu_runtime_models_json(rt);
    if (js == NULL) return 8;
    printf("models=%s\n", js);
    npu_string_free(js);
    if (npu_runtime_embed(rt, NULL, "x", NULL, 0) != -1) return 9;
    printf("rt_embed=%s\n", npu_last_error());
    npu_runtime_stop(rt);
    npu_string_free(NULL);
    npu_model_free(NULL);
    npu_runtime_stop(NULL);
    return 0;
}
"""


def test_c_program_links_and_reports_errors(lib, tmp_path):
    """c_smoke.rs:36-78: a C program compiled against the header and linked against the
    shared library calls the ABI with no device; then the reference's error rules."""
    src = tmp_path / "smoke.c"
    src.write_text(C_SMOKE)
    exe = tmp_path / "smoke"
    subprocess.run(["gcc", str(src), f"-I{REPO}/include", f"-L{LIBDIR}", f"-Wl,-rpath,{LIBDIR}",
                    "-lxdna_b200", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert "available=" in out.stdout
    assert "null_path=scenario_path is null" in out.stdout
    assert "missing=load failed: scenario /nonexistent/scenario.toml" in out.stdout
    assert "kind_null=model is null" in out.stdout
    assert 'models={"object":"list","data":[]}' in out.stdout
    assert "rt_embed=unsupported: no embed model loaded" in out.stdout


def test_scenario_errors(lib, tmp_path):
    bad = tmp_path / "bad.toml"
    bad.write_text('[scenario]\nkind = "embeddings"\nname = "x"\n[model]\nhidden = 768\n')
    assert lib.npu_model_load(str(bad).encode()) is None
    assert b"missing field `ff`" in lib.npu_last_error()
    asr = tmp_path / "asr.toml"
    asr.write_text('[scenario]\nkind = "asr"\nname = "whisper-small"\n[model]\nhidden = 768\nff = 3072\n'
                   'n_heads = 12\nhead_dim = 64\nn_layers = 12\nmax_seq = 1500\n')
    assert lib.npu_model_load(str(asr).encode()) is None      # no artifacts.weights directory
    assert lib.npu_last_error().startswith(b"load failed: ")
    odd = tmp_path / "odd.toml"
    odd.write_text(asr.read_text().replace('"asr"', '"speech"'))
    assert lib.npu_model_load(str(odd).encode()) is None
    assert b'unknown scenario kind "speech"' in lib.npu_last_error()


VOCAB = (["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"] + list("abcdefghijklmnopqrstuvwxyz0123456789")
         + list(".,!?;:'\"()-/") + ["##" + c for c in "abcdefghijklmnopqrstuvwxyz"]
         + ["hello", "world", "the", "token", "##izer", "##s", "un", "##aff", "##able", "cafe", "naive",
            "embed", "##ding", "##ings", "b200", "gpu", "中", "文"])


def _ours(lib, path, text, max_len=64):
    ids = np.zeros(256, np.int32)
    n = lib.xdna_wordpiece_encode(str(path).encode(), text.encode(), max_len, ids.ctypes.data, 256)
    assert n >= 0, lib.npu_last_error()
    return ids[:n].tolist()


TEXTS = ["Hello, world!", "The tokenizers' embeddings", "unaffable GPU B200", "Café naïve ÀÉÎÕÜ",
         "  tabs\tand\nnewlines  ", "中文 text", "xyzzy!!", "a" * 120, "", "embedding-embeddings/x"]


@pytest.mark.parametrize("fmt", ["txt", "json"])
def test_wordpiece_matches_hf_bert_tokenizer(lib, tmp_path, fmt):
    from transformers import BertTokenizer, BertTokenizerFast
    vocab = tmp_path / "vocab.txt"
    vocab.write_text("\n".join(VOCAB) + "\n")
    hf = BertTokenizer(str(vocab), do_lower_case=True)
    path = vocab
    if fmt == "json":
        # a tokenizer.json in the HuggingFace layout, its WordPiece vocabulary filled in
        # explicitly (the fast constructor of this transformers version drops vocab files)
        import json
        fast = BertTokenizerFast(vocab_file=str(vocab), do_lower_case=True)
        fast.save_pretrained(str(tmp_path / "hf"))
        path = tmp_path / "hf" / "tokenizer.json"
        tj = json.loads(path.read_text())
        tj["model"]["vocab"] = {t: i for i, t in enumerate(VOCAB)}
        path.write_text(json.dumps(tj, indent=2, ensure_ascii=False))
    for t in TEXTS:
        assert _ours(lib, path, t) == hf.encode(t), t
    # truncation to max_seq (frontend.rs:31-33)
    assert _ours(lib, path, "hello " * 20, max_len=8) == hf.encode("hello " * 20)[:8]


def _write_scenario(tmp_path, cfg, w, pooling="mean"):
    wd = tmp_path / "weights"
    (wd / "emb").mkdir(parents=True)
    for k in ("word_emb", "pos_emb", "type_emb", "emb_ln_w", "emb_ln_b"):
        np.save(wd / "emb" / f"{k}.npy", w[k])
    names = {"o_w": "attn_out_w", "o_b": "attn_out_b"}
    for i, ly in enumerate(w["layers"]):
        (wd / f"L{i}").mkdir()
        for k, v in ly.items():
            np.save(wd / f"L{i}" / f"{names.get(k, k)}.npy", v)
    (tmp_path / "vocab.txt").write_text("\n".join(VOCAB) + "\n")
    scen = tmp_path / "bge.toml"
    scen.write_text(f"""# a scenario in the reference's manifest format
[scenario]
kind = "embeddings"
name = "bge-base-en-v1.5"

[model]
hidden = 768
ff = 3072
n_heads = 12
head_dim = 64
n_layers = {cfg.n_layers}
max_seq = 512
precision = "bf16"

[artifacts]
weights = "weights"
tokenizer = "vocab.txt"

[embeddings]
pooling = "{pooling}"
normalize = true
""")
    return scen


@pytest.mark.gpu
@pytest.mark.parametrize("pooling", ["mean", "cls"])
def test_npu_embed_end_to_end(lib, tmp_path, monkeypatch, pooling):
    """npu_model_load + npu_embed on the GPU against the oracle's host embedder on the same ids:
    cosine >= 0.999; the dimension query and the short-buffer copy follow lib.rs:77-92."""
    from oracle import oracle as O
    from xdna_engine_b200.synth import BGE_BASE, make_bert_weights
    cfg = dataclasses.replace(BGE_BASE, n_layers=2, vocab=len(VOCAB), pooling=1 if pooling == "mean" else 0)
    w = make_bert_weights(cfg, seed=7, bias_std=0.02, ln_std=0.05)
    scen = _write_scenario(tmp_path, cfg, w, pooling)
    monkeypatch.chdir(tmp_path)
    m = lib.npu_model_load(str(scen).encode())
    assert m, lib.npu_last_error()
    try:
        assert lib.npu_model_kind(m) == 1
        assert lib.npu_embed(m, None, None, 0) == 768
        for text in ("Hello, world!", "unaffable GPU B200 embeddings"):
            out = np.zeros(768, np.float32)
            assert lib.npu_embed(m, text.encode(), out.ctypes.data, 768) == 768, lib.npu_last_error()
            ids = np.array(_ours(lib, tmp_path / "vocab.txt", text, 512), np.int32)
            ref = O.bert_embed(cfg, w, ids, np.array([ids.size], np.int32))[0]
            cos = float(out @ ref / np.linalg.norm(out) / np.linalg.norm(ref))
            assert cos >= 0.999, cos
            short = np.zeros(4, np.float32)
            assert lib.npu_embed(m, text.encode(), short.ctypes.data, 4) == 768
            np.testing.assert_array_equal(short, out[:4])
        assert lib.npu_embed(m, b"\xff\xfe", np.zeros(768, np.float32).ctypes.data, 768) == -1
        assert b"UTF-8" in lib.npu_last_error()
        assert lib.npu_transcribe(m, None, 0, 16000) is None
        assert lib.npu_last_error() == b"wrong model kind: wanted asr, got embed"
    finally:
        lib.npu_model_free(m)


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(a))


@pytest.mark.gpu
def test_npu_embed_from_baked_arena(lib, tmp_path, monkeypatch):
    """artifacts.source + arch + arena (BertWeights::load_for, bert/weights.rs:41-53): the same
    model baked into an npu-weights arena (linear weights and embeddings bf16, biases and norms
    f32, arch/bert.rs:121-125 names) embeds exactly as the npy directory holding the same
    (bf16-rounded) values."""
    from xdna_engine_b200 import arena
    from xdna_engine_b200.synth import BGE_BASE, make_bert_weights
    cfg = dataclasses.replace(BGE_BASE, n_layers=2, vocab=len(VOCAB), pooling=1)
    w = make_bert_weights(cfg, seed=9, bias_std=0.02, ln_std=0.05)
    names = {"o_w": "attn_out_w", "o_b": "attn_out_b"}
    t = {f"emb/{k}": (w[k], k in ("word_emb", "pos_emb", "type_emb"))
         for k in ("word_emb", "pos_emb", "type_emb", "emb_ln_w", "emb_ln_b")}
    for i, ly in enumerate(w["layers"]):
        for k, v in ly.items():
            n = names.get(k, k)
            t[f"L{i}/{n}"] = (v, n.endswith("_w") and "ln" not in n)
    arena.bake(str(tmp_path / "bge.safetensors"), t, arch="bert", source_ref="synthetic")
    wq = {k: (_bf16(v) if bf else v) for k, (v, bf) in
          ((k, (w[k], k in ("word_emb", "pos_emb", "type_emb"))) for k in ("word_emb", "pos_emb", "type_emb",
                                                                              "emb_ln_w", "emb_ln_b"))}
    wq["layers"] = [{k: (_bf16(v) if names.get(k, k).endswith("_w") and "ln" not in names.get(k, k) else v)
                     for k, v in ly.items()} for ly in w["layers"]]
    scen = _write_scenario(tmp_path, cfg, wq, "mean")
    arena_scen = tmp_path / "bge_arena.toml"
    arena_scen.write_text(scen.read_text().replace('[artifacts]\n',
                          '[artifacts]\nsource = "path:/models/bge"\narch = "bert"\narena = "bge.safetensors"\n'))
    monkeypatch.chdir(tmp_path)
    a = lib.npu_model_load(str(arena_scen).encode())
    assert a, lib.npu_last_error()
    b = lib.npu_model_load(str(scen).encode())
    assert b, lib.npu_last_error()
    try:
        for text in ("Hello, world!", "unaffable GPU B200 embeddings"):
            va, vb = np.zeros(768, np.float32), np.zeros(768, np.float32)
            assert lib.npu_embed(a, text.encode(), va.ctypes.data, 768) == 768, lib.npu_last_error()
            assert lib.npu_embed(b, text.encode(), vb.ctypes.data, 768) == 768
            np.testing.assert_array_equal(va, vb)
    finally:
        lib.npu_model_free(a)
        lib.npu_model_free(b)


def test_arena_scenario_errors(lib, tmp_path, monkeypatch):
    """No arena path -> unsupported (baking is not part of the backend); wrong arch -> the
    arena's own error; source without arch -> the reference's message."""
    from xdna_engine_b200 import arena
    monkeypatch.chdir(tmp_path)
    (tmp_path / "vocab.txt").write_text("\n".join(VOCAB) + "\n")
    arena.bake(str(tmp_path / "x.safetensors"), {"emb/word_emb": (np.zeros((4, 768), np.float32), True)}, arch="opt")
    base = ('[scenario]\nkind = "embeddings"\nname = "bge"\n[model]\nhidden = 768\nff = 3072\nn_heads = 12\n'
            'head_dim = 64\nn_layers = 2\nmax_seq = 512\n[artifacts]\ntokenizer = "vocab.txt"\n')
    cases = [('source = "hf:BAAI/bge-base-en-v1.5"\narch = "bert"\n', b"unsupported: baking a weight arena"),
             ('source = "hf:BAAI/bge-base-en-v1.5"\n', b"artifacts.arch is empty"),
             ('source = "path:/m"\narch = "bert"\narena = "x.safetensors"\n', b'arena arch "opt" != expected "bert"')]
    for extra, msg in cases:
        p = tmp_path / "s.toml"
        p.write_text(base + extra)
        assert lib.npu_model_load(str(p).encode()) is None
        assert msg in lib.npu_last_error(), lib.npu_last_error()
