"""Parakeet FastConformer encoder on B200: the int8 tcgen05 GEMM (bit-exact against the
reference's integer rule), the fused kernels, and the whole encoder against the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def _gemm_i8(X, A, B, sa, rpc, ws, bias=None, act=0, residual=None, alpha=1.0, amax=False):
    import torch
    M, K = A.shape
    N = B.shape[0]
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dsa, dws = torch.from_numpy(sa).cuda(), torch.from_numpy(ws).cuda()
    db = torch.from_numpy(bias).cuda() if bias is not None else None
    ncol = N // 2 if act == 3 else N
    C = torch.from_numpy(residual.copy()).cuda() if residual is not None else torch.empty(M, ncol, device="cuda")
    am = torch.zeros(len(sa), dtype=torch.int32, device="cuda") if amax else None
    rc = X.lib().xdna_gemm_i8(dA.data_ptr(), dB.data_ptr(), dsa.data_ptr(), rpc, dws.data_ptr(),
                              db.data_ptr() if db is not None else None, act,
                              C.data_ptr() if residual is not None else None, alpha, C.data_ptr(),
                              am.data_ptr() if am is not None else None, M, N, K,
                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0, X.last_error()
    torch.cuda.synchronize()
    assert X.lib().xdna_gemm_check() == 0, X.last_error()
    return C.cpu().numpy(), (am.cpu().numpy().view(np.float32) if am is not None else None)


@pytest.mark.parametrize("M,N,K,rpc", [(128, 256, 128, 128), (300, 512, 1024, 125), (1000, 1024, 4096, 125),
                                       (250, 4096, 1024, 125)])
def test_gemm_i8_dequant_bit_exact(X, M, N, K, rpc):
    """s32 accumulation is exact and the epilogue is (float(acc) * s_a) * ws + bias in f32,
    so the result equals numpy's integer matmul + the same f32 operations, bit for bit."""
    rng = np.random.default_rng(M + N + K)
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    clips = (M + rpc - 1) // rpc
    sa = rng.uniform(0.001, 0.05, clips).astype(np.float32)
    ws = rng.uniform(0.0001, 0.01, N).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32)
    C, am = _gemm_i8(X, A, B, sa, rpc, ws, bias, 0, res, 0.5, amax=True)
    acc = A.astype(np.int64) @ B.astype(np.int64).T
    assert np.abs(acc).max() < 2**31
    rows_sa = sa[np.arange(M) // rpc][:, None]
    y = (acc.astype(np.float32) * rows_sa).astype(np.float32) * ws
    y = y + bias
    want = res + np.float32(0.5) * y
    np.testing.assert_array_equal(C, want)
    for c in range(clips):
        assert am[c] == np.abs(want[c * rpc:(c + 1) * rpc]).max()


def test_gemm_i8_silu_and_glu(X):
    """SiLU / GLU epilogues: the sigmoid comes from the hardware tanh (sigmoid(g) =
    (1 + tanh(g/2)) / 2), whose absolute error is below 2^-10, so each output is within
    1e-3 * |value input| (+1e-6) of the exact form."""
    rng = np.random.default_rng(9)
    M, N, K = 250, 512, 256
    A = rng.integers(-127, 128, (M, K), dtype=np.int8)
    B = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sa = np.array([0.01, 0.02], np.float32)
    ws = np.full(N, 0.002, np.float32)
    y = (A.astype(np.int64) @ B.astype(np.int64).T).astype(np.float32) * sa[np.arange(M) // 125][:, None] * ws
    C, _ = _gemm_i8(X, A, B, sa, 125, ws, act=1)
    assert np.all(np.abs(C - y / (1 + np.exp(-y))) <= 1e-3 * np.abs(y) + 1e-6)
    C, _ = _gemm_i8(X, A, B, sa, 125, ws, act=3)
    want = y[:, 0::2] / (1 + np.exp(-y[:, 1::2]))
    assert np.all(np.abs(C - want) <= 1e-3 * np.abs(y[:, 0::2]) + 1e-6)


def _compare(got, want, cos_min=0.998, rel_max=0.1):
    g = got.reshape(-1, got.shape[-1]).astype(np.float64)
    r = want.reshape(-1, want.shape[-1]).astype(np.float64)
    cos = (g * r).sum(1) / np.linalg.norm(g, axis=1) / np.linalg.norm(r, axis=1)
    rel = np.abs(g - r).max(1) / np.sqrt((r * r).mean(1))
    assert cos.min() >= cos_min, (cos.min(), rel.max())
    assert rel.max() <= rel_max, (cos.min(), rel.max())
    return cos.min(), rel.max()


def test_parakeet_encoder_small_vs_oracle(X):
    """2 blocks on 200-frame clips (25 frames after subsampling), 3 clips, against the oracle's
    int8-engine encoder; each clip alone gives the same bits as inside the batch."""
    from oracle import oracle as O
    cfg = X.ParakeetConfig(n_layers=2, n_frames=200)
    w = X.make_parakeet_weights(cfg, seed=3, ln_std=0.05)
    mel = X.make_parakeet_mel(cfg, 3, seed=3)
    enc = X.ParakeetEncoder(X.Device(0), cfg, w, max_batch=4)
    assert enc.frames_out == 25
    got = enc.encode(mel)
    want = O.parakeet_encode(cfg, w, mel, int8=True)
    print("small", _compare(got, want))
    # the second and third calls replay a captured CUDA graph: same bits as the eager first call
    for _ in range(2):
        assert np.array_equal(enc.encode(mel), got)
    for b in range(3):
        assert np.array_equal(enc.encode(mel[b:b + 1])[0], got[b])
    enc.close()


def test_parakeet_encoder_full_clip_vs_oracle(X):
    """A 10 s clip (1000 frames -> 125), two blocks: attention over all 125 positions and the
    249-row rel-pos table; a batch of 2 clips."""
    from oracle import oracle as O
    cfg = X.ParakeetConfig(n_layers=2)
    w = X.make_parakeet_weights(cfg, seed=4)
    mel = X.make_parakeet_mel(cfg, 2, seed=4)
    enc = X.ParakeetEncoder(X.Device(0), cfg, w, max_batch=2)
    got = enc.encode(mel)
    print("full", _compare(got, O.parakeet_encode(cfg, w, mel, int8=True)))
    enc.close()


def test_parakeet_rejects_bad_shapes(X):
    bad = X.ParakeetConfig(n_layers=1, n_frames=2000)          # 250 frames after subsampling
    with pytest.raises(X.XdnaError):
        X.ParakeetEncoder(X.Device(0), bad, X.make_parakeet_weights(bad, n_layers=1))
    cfg = X.ParakeetConfig(n_layers=1, n_frames=64)
    enc = X.ParakeetEncoder(X.Device(0), cfg, X.make_parakeet_weights(cfg), max_batch=1)
    with pytest.raises(X.XdnaError):
        enc.encode(X.make_parakeet_mel(cfg, 2))
    enc.close()


def test_parakeet_encoder_baseline_config(X):
    """The BASELINE config: all 24 blocks on a 10 s clip (128 x 1000 mel -> 125 x 1024) against
    the oracle's int8-engine restatement of encoder.rs:572-654 at cos >= 0.999 (measured
    0.99967), and the same clip inside a batch of 64 gives the same bits as alone (per-clip
    activation scales).  The largest single error relative to its row's rms grows with depth (the
    GPU's bf16 activations between the int8 GEMMs re-quantise differently from the oracle's f32
    ones, 24 blocks deep: 0.106 measured), so that secondary bound is 0.15 here."""
    from oracle import oracle as O
    cfg = X.ParakeetConfig()
    w = X.make_parakeet_weights(cfg, seed=5)
    mel = X.make_parakeet_mel(cfg, 64, seed=5)
    enc = X.ParakeetEncoder(X.Device(0), cfg, w, max_batch=64)
    batch = enc.encode(mel)
    one = enc.encode(mel[:1])
    enc.close()
    assert np.array_equal(one[0], batch[0])
    print("baseline", _compare(one, O.parakeet_encode(cfg, w, mel[:1], int8=True), cos_min=0.999,
                                 rel_max=0.15))
