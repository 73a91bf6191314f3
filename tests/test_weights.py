"""Weight stores: the npu-weights arena (rust/npu-weights/src/arena.rs:13-100) and Opt::load over
it or over the npy directory it is baked from (opt125m_decode.rs:155-180, arch/opt.rs:7-16).

CPU: the ports of arena.rs's own tests (bake -> load round trip with exact f32 and bf16 values;
raw bf16 bits for a BF16 tensor and "none" for an F32 one), the arch and format_version checks
with the reference's messages, and refusal of damaged files.  GPU: a decoder loaded from an
arena, and one loaded from the npy directory, produce the same tokens as one built from the
same values in memory."""
import dataclasses
import json
import os
import struct

import numpy as np
import pytest

from xdna_engine_b200 import arena


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def _open(X, path, arch):
    h = X.lib().xdna_weights_open(str(path).encode(), None if arch is None else arch.encode())
    return h


def test_bake_then_load_roundtrip(X, tmp_path):
    """arena.rs bake_then_load_roundtrip + tensor_bf16_returns_raw_bits_for_bf16_and_none_for_f32."""
    L = X.lib()
    p = tmp_path / "a.safetensors"
    arena.bake(str(p), {"L0/q_w": (np.array([[1, 2], [3, 4]], np.float32), True),
                        "L0/q_b": (np.array([0.5, -0.5], np.float32), False)},
               arch="bert", source_ref="test", source_fingerprint="deadbeef")
    a = _open(X, p, "bert")
    assert a, X.last_error()
    try:
        assert L.xdna_weights_count(a) == 2
        assert [L.xdna_weights_name(a, i) for i in range(2)] == [b"L0/q_b", b"L0/q_w"]
        assert L.xdna_weights_name(a, 2) is None
        assert L.xdna_weights_meta(a, b"format_version") == b"1"
        assert L.xdna_weights_meta(a, b"source_fingerprint") == b"deadbeef"
        dt, sh = np.zeros(1, np.int32), np.zeros(4, np.int64)
        assert L.xdna_weights_info(a, b"L0/q_w", dt.ctypes.data, sh.ctypes.data, 4) == 2
        assert dt[0] == 1 and sh[:2].tolist() == [2, 2]
        b = np.zeros(2, np.float32)
        assert L.xdna_weights_read_f32(a, b"L0/q_b", b.ctypes.data, 2) == 0
        assert b.tolist() == [0.5, -0.5]
        w = np.zeros(4, np.float32)
        assert L.xdna_weights_read_f32(a, b"L0/q_w", w.ctypes.data, 4) == 0
        assert w.tolist() == [1.0, 2.0, 3.0, 4.0]
        bits = np.zeros(4, np.uint16)
        assert L.xdna_weights_read_bf16(a, b"L0/q_w", bits.ctypes.data, 4) == 0
        assert bits.tolist() == [0x3F80, 0x4000, 0x4040, 0x4080]
        assert L.xdna_weights_read_bf16(a, b"L0/q_b", bits.ctypes.data, 2) == 1      # F32: none
        assert L.xdna_weights_read_f32(a, b"L0/q_w", w.ctypes.data, 3) == -1
        assert L.xdna_weights_read_f32(a, b"nope", w.ctypes.data, 4) == -1
        assert b'"nope" not in the arena' in X.lib().xdna_last_error()
    finally:
        L.xdna_weights_close(a)


def test_bf16_rounding_is_round_to_nearest_even(X, tmp_path):
    rng = np.random.default_rng(0)
    v = rng.standard_normal(1000).astype(np.float32)
    v[:4] = [1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8, 65504.0]      # exact ties
    p = tmp_path / "r.safetensors"
    arena.bake(str(p), {"v": (v, True)}, arch="opt")
    a = _open(X, p, None)
    out = np.zeros(1000, np.float32)
    assert X.lib().xdna_weights_read_f32(a, b"v", out.ctypes.data, 1000) == 0
    X.lib().xdna_weights_close(a)
    import torch
    np.testing.assert_array_equal(out, torch.from_numpy(v).to(torch.bfloat16).float().numpy())


def test_arch_and_version_checks(X, tmp_path):
    p = tmp_path / "a.safetensors"
    arena.bake(str(p), {"x": (np.ones(3, np.float32), False)}, arch="bert")
    assert _open(X, p, "opt") is None
    assert 'arena arch "bert" != expected "opt"' in X.last_error()
    # rewrite the metadata's format_version
    raw = p.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    h = json.loads(raw[8:8 + n])
    h["__metadata__"]["format_version"] = "2"
    hb = json.dumps(h).encode()
    hb += b" " * (-len(hb) % 8)
    q = tmp_path / "v2.safetensors"
    q.write_bytes(struct.pack("<Q", len(hb)) + hb + raw[8 + n:])
    assert _open(X, q, "bert") is None
    assert "arena format_version 2 != 1 (rebake)" in X.last_error()


@pytest.mark.parametrize("damage", ["truncated", "header_len", "offsets", "dtype", "not_json"])
def test_damaged_files_are_refused(X, tmp_path, damage):
    p = tmp_path / "a.safetensors"
    arena.bake(str(p), {"x": (np.ones(8, np.float32), False)}, arch="opt")
    raw = bytearray(p.read_bytes())
    n = struct.unpack("<Q", raw[:8])[0]
    if damage == "truncated":
        raw = raw[:-4]
    elif damage == "header_len":
        raw[:8] = struct.pack("<Q", len(raw))
    else:
        h = json.loads(raw[8:8 + n])
        if damage == "offsets":
            h["x"]["data_offsets"] = [0, 16]
        elif damage == "dtype":
            h["x"]["dtype"] = "F16"
        hb = json.dumps(h).encode() if damage != "not_json" else b"[1, 2" + b" " * 3
        hb += b" " * (-len(hb) % 8)
        raw = struct.pack("<Q", len(hb)) + hb + raw[8 + n:]
    p.write_bytes(bytes(raw))
    assert _open(X, p, "opt") is None
    assert X.last_error().startswith("xdna_weights_open: ")


def test_opt_load_errors_without_device(X, tmp_path):
    assert X.lib().xdna_opt_load(None, str(tmp_path).encode(), 0, 0) is None
    assert "null" in X.last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("store", ["arena", "npy"])
def test_opt_load_matches_in_memory_weights(X, tmp_path, store):
    cfg = dataclasses.replace(X.OPT_125M, n_layers=2, vocab=4096, max_pos=512)
    w = X.make_opt_weights(cfg, seed=5, bias_std=0.02, ln_std=0.05)
    t = arena.opt_tensors(w)
    if store == "arena":
        path = tmp_path / "opt.safetensors"
        arena.bake(str(path), t, arch="opt", source_ref="synthetic")
    else:
        path = tmp_path / "npy"
        arena.write_npy_dir(str(path), t)
    # the same values in memory: bf16-stored tensors rounded as the store holds them
    bf = lambda a: (arena._bf16_bits(a).astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    w2 = {"emb_tok": bf(w["emb_tok"]), "emb_pos": bf(w["emb_pos"]), "lnf_w": w["lnf_w"], "lnf_b": w["lnf_b"],
          "layers": [{k: (bf(v) if k in ("wq", "wk", "wv", "wo", "w1", "w2") else v) for k, v in ly.items()}
                     for ly in w["layers"]]}
    dev = X.Device(0)
    prompt = X.make_prompt(cfg, 12, seed=2)
    a = X.OptDecoder.load(dev, str(path), max_ctx=64)
    assert a.cfg == cfg
    b = X.OptDecoder(dev, cfg, w2, max_ctx=64)
    np.testing.assert_array_equal(a.generate(prompt, 24), b.generate(prompt, 24))
    # an untied LM head is refused
    t["lm_head.weight"] = (t["lm_head.weight"][0] * 2, True)
    bad = tmp_path / "bad.safetensors"
    arena.bake(str(bad), t, arch="opt")
    with pytest.raises(X.XdnaError, match="untied"):
        X.OptDecoder.load(dev, str(bad))
