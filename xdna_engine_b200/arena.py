"""Weight arenas in the npu-weights format (rust/npu-weights/src/arena.rs:13-44): one
safetensors file, each tensor BF16 or F32 little-endian, with "__metadata__" holding
format_version, arch, source_ref and source_fingerprint; written atomically (a unique temporary
file, fsync, rename).  The engine reads them with xdna_weights_open / xdna_opt_load.

`opt_tensors` maps a weight dict in the engine's layout (xdna_engine_b200.synth) to the names
and storage types of rust/npu-weights/src/arch/opt.rs:7-16: linear weights [in, out] and the
embeddings bf16, biases and LayerNorm parameters f32, lm_head.weight = embed_tokens transposed
(OPT ties them)."""
from __future__ import annotations

import json
import os
import struct

import numpy as np

FORMAT_VERSION = 1


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    """f32 -> bf16 bit patterns, round to nearest even (half::bf16::from_f32)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bake(path: str, tensors: dict, arch: str, source_ref: str = "", source_fingerprint: str = "") -> None:
    """tensors: name -> (array, bf16: bool).  Names are written in sorted order, as a BTreeMap."""
    header, blobs, off = {}, [], 0
    for name in sorted(tensors):
        arr, as_bf16 = tensors[name]
        arr = np.asarray(arr, np.float32)
        raw = _bf16_bits(arr).tobytes() if as_bf16 else np.ascontiguousarray(arr, "<f4").tobytes()
        header[name] = {"dtype": "BF16" if as_bf16 else "F32", "shape": list(arr.shape),
                        "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    header["__metadata__"] = {"format_version": str(FORMAT_VERSION), "arch": arch, "source_ref": source_ref,
                              "source_fingerprint": source_fingerprint}
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)                       # safetensors pads the header to 8 bytes
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    tmp = f"{path}.tmp.{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def opt_tensors(w: dict) -> dict:
    """Engine-layout OPT weights -> {arena name: (array, bf16)} per arch/opt.rs."""
    t = {"embed_tokens": (w["emb_tok"], True), "embed_positions": (w["emb_pos"], True),
         "ln_final.weight": (w["lnf_w"], False), "ln_final.bias": (w["lnf_b"], False),
         "lm_head.weight": (np.ascontiguousarray(w["emb_tok"].T), True)}
    names = {"wq": "q.weight", "bq": "q.bias", "wk": "k.weight", "bk": "k.bias", "wv": "v.weight",
             "bv": "v.bias", "wo": "out.weight", "bo": "out.bias", "ln1_w": "ln_self.weight",
             "ln1_b": "ln_self.bias", "ln2_w": "ln_ffn.weight", "ln2_b": "ln_ffn.bias", "w1": "fc1.weight",
             "b1": "fc1.bias", "w2": "fc2.weight", "b2": "fc2.bias"}
    for i, ly in enumerate(w["layers"]):
        for k, n in names.items():
            t[f"L{i}/{n}"] = (ly[k], n.endswith(".weight") and not n.startswith("ln_"))
    return t


def write_npy_dir(path: str, tensors: dict) -> None:
    """The npy directory layout the arena is baked from: name + ".npy", f32 (bf16 values upcast)."""
    for name, (arr, as_bf16) in tensors.items():
        a = np.asarray(arr, np.float32)
        if as_bf16:
            a = (_bf16_bits(a).astype(np.uint32) << 16).view(np.float32)
        p = os.path.join(path, name + ".npy")
        os.makedirs(os.path.dirname(p), exist_ok=True)
        np.save(p, np.ascontiguousarray(a))
