"""Build the engine's shared library in-tree (nvcc, sm_100a only).

    python -m xdna_engine_b200._build
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libxdna_b200.so")
SOURCES = ["decode_kernel.cu", "gemv_op.cu", "engine.cu", "noalloc.cu", "capi.cu", "runtime.cu", "ops.cu", "weights.cu", "asr.cu", "logmel.cu", "ffn_fused.cu", "attention_tc.cu", "gemm_tc.cu", "encoders.cu", "parakeet.cu", "whisper_dec.cu", "gemma.cu"]
HEADERS = ["decode.h", "gemv_op.h", "ptx.cuh", "tc.cuh", "gelu.cuh", "json.h", "toml.h", "capi_internal.h"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "xdna_b200.h"))
    deps.append(os.path.join(os.path.dirname(HERE), "include", "npu_engine.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    if not force and not needs_build():
        return LIB
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off", "--fmad=false", "-shared",
           "-diag-suppress", "550",
           "-o", LIB + ".tmp"] + [os.path.join(CSRC, f) for f in SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
