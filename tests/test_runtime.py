"""The control plane behind npu_runtime_* (rust/npu-runtime: config.rs, registry.rs, reconcile.rs,
select.rs, actor.rs; C surface rust/npu-capi/src/lib.rs:125-214) with one worker per GPU.

CPU tests run the workers with the test loader (XDNA_RUNTIME_MOCK, the reference's MockLoader):
config parsing and its errors, load failures recorded but not fatal, the max_resident and
memory caps, model resolution (explicit, default, single, ambiguous, wrong kind), reconcile on
reload, one replica per worker and least-busy dispatch across workers, concurrent callers.  The
GPU test loads a real embedding scenario through the runtime and checks its embeddings are the
bits npu_embed gives."""
import ctypes as C
import json
import os
import threading

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
    L.npu_runtime_start.restype = C.c_void_p
    L.npu_runtime_start.argtypes = [C.c_char_p]
    L.npu_runtime_transcribe.restype = C.c_void_p
    L.npu_runtime_transcribe.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t, C.c_uint32]
    L.npu_runtime_embed.argtypes = [C.c_void_p, C.c_char_p, C.c_char_p, C.c_void_p, C.c_size_t]
    L.npu_runtime_reload.argtypes = [C.c_void_p]
    L.npu_runtime_models_json.restype = C.c_void_p
    L.npu_runtime_models_json.argtypes = [C.c_void_p]
    L.npu_runtime_stop.argtypes = [C.c_void_p]
    L.npu_string_free.argtypes = [C.c_void_p]
    L.npu_model_load.restype = C.c_void_p
    L.npu_model_load.argtypes = [C.c_char_p]
    L.npu_embed.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]
    L.npu_model_free.argtypes = [C.c_void_p]
    return L


def models(lib, rt):
    p = lib.npu_runtime_models_json(rt)
    assert p, lib.npu_last_error()
    s = C.string_at(p).decode()
    lib.npu_string_free(p)
    return {m["id"]: m for m in json.loads(s)["data"]}, s


def embed(lib, rt, model=None, text="hello"):
    out = np.zeros(8, np.float32)
    n = lib.npu_runtime_embed(rt, model.encode() if model else None, text.encode(), out.ctypes.data, 8)
    return n, out


def transcribe(lib, rt, model=None):
    pcm = np.zeros(160, np.int16)
    p = lib.npu_runtime_transcribe(rt, model.encode() if model else None, pcm.ctypes.data, pcm.size, 16000)
    if not p:
        return None
    s = C.string_at(p).decode()
    lib.npu_string_free(p)
    return s


def write_cfg(path, models_, server=None, defaults=None):
    t = []
    if server:
        t += ["[server]"] + [f"{k} = {v}" for k, v in server.items()]
    if defaults:
        t += ["[defaults]"] + [f'{k} = "{v}"' for k, v in defaults.items()]
    for name, scen in models_:
        t += ["[[model]]", f'name = "{name}"', f'scenario = "{scen}"']
    path.write_text("\n".join(t) + "\n")


SRV = {"port": 11434, "memory_ceiling_mb": 4096, "max_resident": 8}


def test_missing_config_is_empty_and_errors(lib, tmp_path, monkeypatch):
    """config.rs:27-34: a missing file is the empty config; select.rs:21-25 errors; lib.rs null
    checks."""
    monkeypatch.setenv("XDNA_RUNTIME_MOCK", "")
    rt = lib.npu_runtime_start(str(tmp_path / "none.toml").encode())
    assert rt, lib.npu_last_error()
    try:
        assert models(lib, rt)[1] == '{"object":"list","data":[]}'
        assert embed(lib, rt)[0] == -1
        assert lib.npu_last_error() == b"unsupported: no embed model loaded"
        assert transcribe(lib, rt) is None
        assert lib.npu_last_error() == b"unsupported: no asr model loaded"
        assert lib.npu_runtime_embed(rt, None, None, None, 0) == -1
        assert lib.npu_last_error() == b"text is null"
    finally:
        lib.npu_runtime_stop(rt)
    assert lib.npu_runtime_start(None) is None
    assert lib.npu_last_error() == b"config_path is null"
    assert lib.npu_runtime_embed(None, None, b"x", None, 0) == -1
    assert lib.npu_last_error() == b"runtime is null"
    assert lib.npu_runtime_reload(None) == -1
    assert lib.npu_runtime_models_json(None) is None
    lib.npu_runtime_stop(None)


def test_config_errors(lib, tmp_path, monkeypatch):
    """Config::from_str errors carry the path (config.rs:29-31): a [server] table needs all three
    fields; [[model]] entries need name and scenario."""
    monkeypatch.setenv("XDNA_RUNTIME_MOCK", "")
    p = tmp_path / "engine.toml"
    p.write_text("[server]\nport = 1\n")
    assert lib.npu_runtime_start(str(p).encode()) is None
    assert lib.npu_last_error() == f"{p}: missing field `memory_ceiling_mb`".encode()
    p.write_text('[[model]]\nname = "a"\n')
    assert lib.npu_runtime_start(str(p).encode()) is None
    assert lib.npu_last_error() == f"{p}: missing field `scenario`".encode()
    p.write_text("[server\n")
    assert lib.npu_runtime_start(str(p).encode()) is None
    assert str(p).encode() in lib.npu_last_error()


def test_failures_recorded_caps_and_replicas(lib, tmp_path, monkeypatch):
    """registry.rs:44-66: a failed load is a status, not an error; max_resident and the memory
    ceiling hold per GPU; every worker holds a replica."""
    monkeypatch.setenv("XDNA_RUNTIME_MOCK", "good=embed:10;bad=!boom;big=embed:5000000000;a=asr:1")
    p = tmp_path / "engine.toml"
    write_cfg(p, [("good", "g.toml"), ("bad", "b.toml"), ("big", "x.toml")], {**SRV, "gpus": 3})
    rt = lib.npu_runtime_start(str(p).encode())
    assert rt, lib.npu_last_error()
    try:
        m, _ = models(lib, rt)
        assert list(m) == ["good", "bad", "big"]
        assert m["good"]["state"] == "loaded" and m["good"]["replicas"] == 3 and m["good"]["devices"] == [0, 1, 2]
        assert m["good"]["kind"] == "embed" and m["good"]["bo_bytes"] == 30
        assert m["bad"]["state"] == "failed" and m["bad"]["detail"] == "load failed: boom" and m["bad"]["kind"] == "unknown"
        assert m["big"]["state"] == "failed" and m["big"]["detail"] == "over memory_ceiling"
        n, out = embed(lib, rt)
        assert n == 8, lib.npu_last_error()
        # max_resident = 1: the second model of each GPU is refused
        write_cfg(p, [("good", "g.toml"), ("a", "a.toml")], {**SRV, "max_resident": 1, "gpus": 3})
        assert lib.npu_runtime_reload(rt) == 0, lib.npu_last_error()
        m, _ = models(lib, rt)
        assert m["good"]["state"] == "loaded" and m["a"]["state"] == "failed"
        assert m["a"]["detail"] == "over max_resident (1)"
    finally:
        lib.npu_runtime_stop(rt)


def test_resolution_rules(lib, tmp_path, monkeypatch):
    """select.rs:5-26: explicit names (unknown / wrong kind), the configured default, the single
    loaded model of a capability, ambiguity without a default."""
    monkeypatch.setenv("XDNA_RUNTIME_MOCK", "bge=embed:1;e5=embed:1;asr1=asr:1")
    p = tmp_path / "engine.toml"
    write_cfg(p, [("bge", "a.toml"), ("e5", "b.toml"), ("asr1", "c.toml")], SRV)
    rt = lib.npu_runtime_start(str(p).encode())
    assert rt, lib.npu_last_error()
    try:
        assert embed(lib, rt, "bge")[0] == 8
        assert embed(lib, rt, "nope")[0] == -1
        assert lib.npu_last_error() == b'load failed: model "nope" not loaded'
        assert embed(lib, rt, "asr1")[0] == -1
        assert lib.npu_last_error() == b"wrong model kind: wanted embed, got asr"
        assert embed(lib, rt)[0] == -1
        assert lib.npu_last_error() == b"unsupported: model required for embed (multiple loaded)"
        assert transcribe(lib, rt) == "mock-text"              # the one ASR model
        assert transcribe(lib, rt, "bge") is None
        assert lib.npu_last_error() == b"wrong model kind: wanted asr, got embed"
        write_cfg(p, [("bge", "a.toml"), ("e5", "b.toml"), ("asr1", "c.toml")], SRV, {"embed": "e5"})
        assert lib.npu_runtime_reload(rt) == 0
        assert embed(lib, rt)[0] == 8                          # the default
    finally:
        lib.npu_runtime_stop(rt)


def test_reload_reconciles(lib, tmp_path, monkeypatch):
    """reconcile.rs:11-31: models the config drops are unloaded, failed ones are retried, kept
    ones stay; a config that no longer parses leaves the runtime as it was."""
    monkeypatch.setenv("XDNA_RUNTIME_MOCK", "a=embed:1;b=!fail")
    p = tmp_path / "engine.toml"
    write_cfg(p, [("a", "a.toml"), ("b", "b.toml")], SRV)
    rt = lib.npu_runtime_start(str(p).encode())
    try:
        m, _ = models(lib, rt)
        assert m["a"]["state"] == "loaded" and m["b"]["state"] == "failed"
        write_cfg(p, [("b", "b.toml")], SRV)
        assert lib.npu_runtime_reload(rt) == 0
        m, _ = models(lib, rt)
        assert list(m) == ["b"] and m["b"]["state"] == "failed"
        assert embed(lib, rt)[0] == -1
        p.write_text("[server]\nport = \n")
        assert lib.npu_runtime_reload(rt) == -1
        assert str(p).encode() in lib.npu_last_error()
        m, _ = models(lib, rt)
        assert list(m) == ["b"]
    finally:
        lib.npu_runtime_stop(rt)


def test_dispatch_spreads_over_workers(lib, tmp_path, monkeypatch):
    """With every worker idle, requests go round robin; from many threads at once every request
    is served once (the mock embedding's first value is the serving worker's GPU ordinal)."""
    monkeypatch.setenv("XDNA_RUNTIME_MOCK", "m=embed:1")
    p = tmp_path / "engine.toml"
    write_cfg(p, [("m", "m.toml")], {**SRV, "gpus": 4})
    rt = lib.npu_runtime_start(str(p).encode())
    try:
        seen = [int(embed(lib, rt)[1][0]) for _ in range(12)]
        assert sorted(seen) == sorted([0, 1, 2, 3] * 3), seen
        res, errs = [], []

        def worker():
            for _ in range(50):
                n, out = embed(lib, rt, "m")
                (res if n == 8 else errs).append(int(out[0]))
        ts = [threading.Thread(target=worker) for _ in range(8)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        assert not errs and len(res) == 400
        assert set(res) <= {0, 1, 2, 3}
    finally:
        lib.npu_runtime_stop(rt)


@pytest.mark.gpu
def test_runtime_embed_equals_npu_embed(lib, tmp_path, monkeypatch):
    """A real embedding scenario through the control plane: loaded on every GPU (up to 2), each
    replica's embedding is bit-identical to npu_embed's; the status reports device bytes."""
    import dataclasses
    import torch
    from tests.test_capi import VOCAB, _write_scenario
    from xdna_engine_b200.synth import BGE_BASE, make_bert_weights
    monkeypatch.delenv("XDNA_RUNTIME_MOCK", raising=False)
    cfg = dataclasses.replace(BGE_BASE, n_layers=2, vocab=len(VOCAB))
    w = make_bert_weights(cfg, seed=3, bias_std=0.02, ln_std=0.05)
    scen = _write_scenario(tmp_path, cfg, w)
    monkeypatch.chdir(tmp_path)
    ngpu = min(2, torch.cuda.device_count())
    p = tmp_path / "engine.toml"
    write_cfg(p, [("bge", str(scen))], {"port": 11434, "memory_ceiling_mb": 65536, "max_resident": 2,
                                        "gpus": ngpu})
    rt = lib.npu_runtime_start(str(p).encode())
    assert rt, lib.npu_last_error()
    m = lib.npu_model_load(str(scen).encode())
    assert m, lib.npu_last_error()
    try:
        st, _ = models(lib, rt)
        assert st["bge"]["state"] == "loaded", st
        assert st["bge"]["replicas"] == ngpu and st["bge"]["bo_bytes"] > 0
        for text in ("Hello, world!", "unaffable GPU B200 embeddings"):
            want = np.zeros(768, np.float32)
            assert lib.npu_embed(m, text.encode(), want.ctypes.data, 768) == 768
            for _ in range(2 * ngpu):                       # every replica serves at least once
                got = np.zeros(768, np.float32)
                assert lib.npu_runtime_embed(rt, b"bge", text.encode(), got.ctypes.data, 768) == 768, \
                    lib.npu_last_error()
                np.testing.assert_array_equal(got, want)
        write_cfg(p, [], {"port": 11434, "memory_ceiling_mb": 65536, "max_resident": 2, "gpus": ngpu})
        assert lib.npu_runtime_reload(rt) == 0
        assert models(lib, rt)[0] == {}
        assert lib.npu_runtime_embed(rt, None, b"x", None, 0) == -1
    finally:
        lib.npu_model_free(m)
        lib.npu_runtime_stop(rt)
