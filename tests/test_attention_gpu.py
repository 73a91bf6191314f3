"""Encoder self-attention on the tcgen05 tensor cores (xdna_attention_bf16; the reference's `mha`
with valid_len, rust/npu-asr-host/src/lib.rs:189-326) against a plain PyTorch fp32 reference of
the same op on the same bf16 q, k, v: packed sequences of lengths 1..1500, each attending only
to its own keys.  The kernel rounds the softmax weights P to bf16 before P.V (as the mma.sync
kernel it replaces did) and the output to bf16, so the bar is rel-L2 <= 1e-2 per sequence and
head, max error <= 2e-2 of the row scale."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def _run(X, lens, seed=0, scale=1.0):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = int(sum(lens))
    qkv = (torch.randn(T, 2304, device="cuda", generator=g) * scale).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32), device="cuda")
    ctx = torch.full((T, 768), float("nan"), device="cuda", dtype=torch.bfloat16)
    rc = X.lib().xdna_attention_bf16(qkv.data_ptr(), T, cu.data_ptr(), len(lens), int(max(lens)), ctx.data_ptr(),
                                     torch.cuda.current_stream().cuda_stream)
    assert rc == 0, X.last_error()
    torch.cuda.synchronize()
    assert X.lib().xdna_attention_check() == 0, X.last_error()
    return qkv.float(), cu.cpu().numpy(), ctx.float()


@pytest.mark.parametrize("lens", [[1], [17], [128], [129], [300, 5, 512], [1500], [64, 1, 255, 256, 257, 100],
                                  [1500, 1500]])
def test_attention_matches_fp32(X, lens):
    import torch
    qkv, cu, got = _run(X, lens, seed=len(lens) * 1000 + lens[0])
    assert not torch.isnan(got).any()
    for s in range(len(lens)):
        a, b = int(cu[s]), int(cu[s + 1])
        for h in range(12):
            q = qkv[a:b, 64 * h:64 * h + 64]
            k = qkv[a:b, 768 + 64 * h:768 + 64 * h + 64]
            v = qkv[a:b, 1536 + 64 * h:1536 + 64 * h + 64]
            ref = torch.softmax(q @ k.T / 8.0, dim=-1) @ v
            out = got[a:b, 64 * h:64 * h + 64]
            rel = ((out - ref).norm() / ref.norm()).item()
            assert rel < 1e-2, (s, h, rel)
            assert (out - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item()), (s, h)


def test_attention_peaked_scores(X):
    """Large logits (a nearly one-hot softmax) exercise the running-maximum correction."""
    import torch
    qkv, cu, got = _run(X, [700, 33], seed=3, scale=4.0)
    for s in range(2):
        a, b = int(cu[s]), int(cu[s + 1])
        for h in (0, 11):
            q, k, v = (qkv[a:b, o + 64 * h:o + 64 * h + 64] for o in (0, 768, 1536))
            ref = torch.softmax(q @ k.T / 8.0, dim=-1) @ v
            rel = ((got[a:b, 64 * h:64 * h + 64] - ref).norm() / ref.norm()).item()
            assert rel < 1e-2, (s, h, rel)
