"""The fused two-GEMM FFN (xdna_ffn_fused_bf16; ffn_gemm2, route_b_kernels/ffn_gemm2/
ffn_gemm2_iron.py:1-30) with the hidden kept on chip.

Against the unfused path on the same operands -- GEMM1 with the bias + activation epilogue
writing the bf16 hidden to HBM, then GEMM2 with bias + residual (two xdna_gemm_bf16 calls) --
the result is identical bit for bit: both accumulate each output over K in the same order in
TMEM and round the hidden once to bf16.  Against a plain PyTorch fp32 reference of
C = (A @ W1) @ W2 (the reference kernel's contract: bf16 in, f32 out, no activation) the bar is
the hidden's bf16 rounding: rel-L2 <= 4e-3."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def _ops(M, K, P, N, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    W1 = (torch.randn(P, K, device="cuda", generator=g) * K ** -0.5).to(torch.bfloat16)
    W2 = (torch.randn(N, P, device="cuda", generator=g) * P ** -0.5).to(torch.bfloat16)
    b1 = torch.randn(P, device="cuda", generator=g) * 0.1
    b2 = torch.randn(N, device="cuda", generator=g) * 0.1
    R = torch.randn(M, N, device="cuda", generator=g).to(torch.bfloat16)
    return A, W1, W2, b1, b2, R


def _fused(X, A, W1, W2, b1, b2, R, act, f32=False):
    import torch
    M, K = A.shape
    P, N = W1.shape[0], W2.shape[0]
    out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float32 if f32 else torch.bfloat16)
    rc = X.lib().xdna_ffn_fused_bf16(A.data_ptr(), W1.data_ptr(), None if b1 is None else b1.data_ptr(), act,
                                     W2.data_ptr(), None if b2 is None else b2.data_ptr(),
                                     None if R is None else R.data_ptr(), None if f32 else out.data_ptr(),
                                     out.data_ptr() if f32 else None, M, K, P, N,
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, X.last_error()
    torch.cuda.synchronize()
    assert X.lib().xdna_ffn_fused_check() == 0, X.last_error()
    return out


@pytest.mark.parametrize("M,K,P,N", [(300, 768, 3072, 768), (128, 64, 256, 64), (1, 768, 3072, 768),
                                     (517, 1024, 512, 512), (2048, 768, 3072, 768), (200, 256, 1024, 640)])
@pytest.mark.parametrize("act", [1, 2])
def test_fused_equals_unfused(X, M, K, P, N, act):
    import torch
    A, W1, W2, b1, b2, R = _ops(M, K, P, N, seed=M + N + act)
    got = _fused(X, A, W1, W2, b1, b2, R, act)
    L, st = X.lib(), torch.cuda.current_stream().cuda_stream
    if N % 256 == 0:
        H = torch.empty(M, P, device="cuda", dtype=torch.bfloat16)
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        assert L.xdna_gemm_bf16(A.data_ptr(), W1.data_ptr(), b1.data_ptr(), None, H.data_ptr(), M, P, K, act, st) == 0
        assert L.xdna_gemm_bf16(H.data_ptr(), W2.data_ptr(), b2.data_ptr(), R.data_ptr(), C.data_ptr(), M, N, P, 0,
                                st) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, C), (got.float() - C.float()).abs().max().item()
    # fp32 reference with the hidden rounded to bf16 where the kernels round it
    h = A.float() @ W1.float().T + b1
    h = torch.nn.functional.gelu(h) if act == 1 else torch.relu(h)
    ref = h.to(torch.bfloat16).float() @ W2.float().T + b2 + R.float()
    rel = ((got.float() - ref).norm() / ref.norm()).item()
    assert rel < 4e-3, rel


@pytest.mark.parametrize("M,K,P,N", [(256, 768, 3072, 768), (97, 512, 768, 384)])
def test_reference_contract_f32_out(X, M, K, P, N):
    """ffn_gemm2's contract: C = (A @ W1) @ W2, bf16 in, f32 out, no bias or activation."""
    import torch
    A, W1, W2, *_ = _ops(M, K, P, N, seed=11)
    got = _fused(X, A, W1, W2, None, None, None, 0, f32=True)
    ref = (A.float() @ W1.float().T).to(torch.bfloat16).float() @ W2.float().T
    rel = ((got - ref).norm() / ref.norm()).item()
    assert rel < 4e-3, rel
    exact = (A.float() @ W1.float().T) @ W2.float().T
    assert ((got - exact).norm() / exact.norm()).item() < 8e-3


def test_rejects_unsupported_shapes(X):
    L = X.lib()
    assert L.xdna_ffn_fused_bf16(1, 1, None, 0, 1, None, None, 1, None, 128, 768, 3072, 1024, None) == -1
    assert "N <= 768" in X.last_error()
    assert L.xdna_ffn_fused_bf16(1, 1, None, 0, 1, None, None, 1, 1, 128, 768, 3072, 768, None) == -1
