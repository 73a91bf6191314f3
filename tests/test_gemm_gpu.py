"""Encoder GEMM on the tcgen05 tensor cores (xdna_gemm_bf16) against a plain PyTorch fp32
reference of the same op on the same bf16 operands.

Tolerance: the kernel accumulates in f32 (TMEM) and rounds the result to bf16, so each output
may differ from the fp32 reference by one bf16 rounding (2^-8 relative) plus f32
reduction-order noise: |got - ref| <= 1e-2 * |ref| + 1e-2 * rms(ref)."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def gelu_as(y):
    import torch
    x = y * 0.70710678118654752440
    sign = torch.where(x < 0, -1.0, 1.0)
    ax = x.abs()
    t = 1.0 / (1.0 + 0.3275911 * ax)
    e = 1.0 - (((((1.061405429 * t - 1.453152027) * t) + 1.421413741) * t - 0.284496736) * t
               + 0.254829592) * t * torch.exp(-ax * ax)
    return 0.5 * y * (1.0 + sign * e)


def run(X, M, N, K, bias=True, gelu=False, resid=False, seed=0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    b = torch.randn(N, device="cuda", generator=g) if bias else None
    R = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16) if resid else None
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    rc = X.lib().xdna_gemm_bf16(A.data_ptr(), B.data_ptr(), b.data_ptr() if bias else None,
                                R.data_ptr() if resid else None, C.data_ptr(), M, N, K, int(gelu),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0, X.last_error()
    torch.cuda.synchronize()
    assert X.lib().xdna_gemm_check() == 0, X.last_error()
    ref = A.float() @ B.float().T
    if bias:
        ref = ref + b
    if gelu:
        ref = gelu_as(ref)
    if resid:
        ref = ref + R.float()
    got = C.float()
    err = (got - ref).abs()
    tol = 1e-2 * ref.abs() + 1e-2 * ref.pow(2).mean().sqrt()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} elements out of tolerance, max err {err.max().item()}"
    return got, ref


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 256, 192), (1000, 2304, 768),
                                   (517, 768, 3072), (64, 3072, 768)])
def test_gemm_bias(X, M, N, K):
    run(X, M, N, K)


def test_gemm_gelu_and_residual(X):
    run(X, 640, 3072, 768, gelu=True, seed=3)
    run(X, 640, 768, 3072, resid=True, seed=4)
    run(X, 200, 768, 768, bias=False, resid=True, seed=5)


def test_gemm_repeat_deterministic(X):
    a, _ = run(X, 384, 768, 768, seed=7)
    b, _ = run(X, 384, 768, 768, seed=7)
    assert (a == b).all()
