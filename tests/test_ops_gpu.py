"""The op-by-op device layer (the npu-xrt shim and CtxDecode replacement) against numpy
restatements of the reference's ops on the same seeded inputs:

* xdna_gemv_bf16 = CtxDecode::gemv (rust/npu-asr/src/ctx_decode.rs:325-369): bf16 operands,
  f32 accumulation.  Checked against an f64 dot of the same bf16 operands, within the f32
  accumulation bound written in `_gemv_tol`.
* the fused pre-norm = register_fused + fused_norm_gemv (ctx_decode.rs:566-643): the gamma
  fold, LayerNorm's folded bias and the f64 input statistics are restated step for step (the
  same summation order, so the normalised input is bit-identical); separately the folded
  result is checked against the unfolded norm -> GEMV in f64 (the separable identity the
  fold rests on) within bf16 rounding.
* xdna_mha_decode_paged = mha_tile (route_b_kernels/mha_decode/mha_decode.cc:90-168) over the
  tiles CtxDecode::attn packs (ctx_decode.rs:482-535): against an f64 softmax attention of the
  same bf16 q, K, V.  The reference evaluates exp in bf16 (exp_scalar, mha_decode.cc:81-86);
  the B200 kernel uses f32 expf, so the bar is the f32 one (rtol 1e-4).
* buffers and runs (xrt_shim.h:26-54): round trips, range errors, and the bounded wait."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def X():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


@pytest.fixture(scope="module")
def dev(X):
    d = X.Device(0)
    yield d
    d.close()


def bf16(a):
    """f32 -> bf16 (round to nearest even) -> f32, as f32_to_bf16_bits does."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def bf16_bits(a):
    return (bf16(a).view(np.uint32) >> 16).astype(np.uint16)


def _norm_input(x, norm, eps):
    """fused_norm_gemv's input reduction (ctx_decode.rs:621-636), summed left to right in f64."""
    x64 = x.astype(np.float64)
    K = x.size
    if norm == "rms":
        ms = np.cumsum(x64 * x64)[-1] / K
        return (x64 * (1.0 / np.sqrt(ms + np.float64(np.float32(eps))))).astype(np.float32)
    if norm == "ln":
        mean = np.cumsum(x64)[-1] / K
        var = np.cumsum((x64 - mean) * (x64 - mean))[-1] / K
        return ((x64 - mean) * (1.0 / np.sqrt(var + np.float64(np.float32(eps))))).astype(np.float32)
    return x


def _fold(w, bias, norm, gamma, beta):
    """register_fused (ctx_decode.rs:573-603): W'' = gamma[k] W[k][n] in f32, LN bias' = sum_k
    beta[k] W[k][n] accumulated in f32 over ascending k, + bias."""
    K, N = w.shape
    wpp = (w * gamma[:, None]).astype(np.float32) if norm else w
    if norm == "ln":
        bp = np.cumsum((beta[:, None] * w).astype(np.float32), axis=0, dtype=np.float32)[-1]
        bp = (bp + (bias if bias is not None else np.float32(0))).astype(np.float32)
    else:
        bp = bias if bias is not None else np.zeros(N, np.float32)
    return wpp, bp


def _gemv_tol(xb, wb):
    # f32 accumulation of K bf16 products (exact in f32): each partial sum rounds once, so the
    # error is below K * 2^-24 * sum_k |x_k w_kn|; bias add adds one more rounding.
    K = xb.size
    return (K + 2) * 2.0 ** -24 * (np.abs(xb.astype(np.float64)) @ np.abs(wb.astype(np.float64))) + 1e-30


@pytest.mark.parametrize("norm", [None, "rms", "ln"])
@pytest.mark.parametrize("shape", [(768, 768), (768, 2304), (3072, 768), (1000, 37), (1, 8)])
def test_gemv_bf16_matches_ctx_decode(X, dev, norm, shape):
    K, N = shape
    rng = np.random.default_rng(K * 7 + N + (0 if norm is None else len(norm)))
    w = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32) if N % 2 else (rng.standard_normal(N) * 0.1).astype(np.float32)
    gamma = (1.0 + 0.2 * rng.standard_normal(K)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(K)).astype(np.float32)
    x = (rng.standard_normal(K) * 3.0 + 0.5).astype(np.float32)
    eps = 1e-5
    g = X.GemvBf16(dev, w, bias=bias, norm=norm, gamma=gamma if norm else None,
                   beta=beta if norm == "ln" else None, eps=eps)
    try:
        y = g(x)
        y2 = g(x)
    finally:
        g.free()
    np.testing.assert_array_equal(y, y2)                   # deterministic
    wpp, bp = _fold(w, bias, norm, gamma, beta)
    xb, wb = bf16(_norm_input(x, norm, eps)), bf16(wpp)
    ref = xb.astype(np.float64) @ wb.astype(np.float64) + bp.astype(np.float64)
    err = np.abs(y.astype(np.float64) - ref)
    tol = _gemv_tol(xb, wb) + 2.0 ** -24 * np.abs(ref)
    assert np.all(err <= tol), (float(err.max()), float(tol[np.argmax(err - tol)]))
    if norm:
        # the separable identity: norm(x) -> (gamma, beta) -> W + bias, unfolded, in f64
        x64 = x.astype(np.float64)
        if norm == "rms":
            xn = x64 / np.sqrt(np.mean(x64 * x64) + eps) * gamma
        else:
            xn = (x64 - x64.mean()) / np.sqrt(x64.var() + eps) * gamma + beta
        direct = xn @ w.astype(np.float64) + bias
        scale = np.abs(xn) @ np.abs(w.astype(np.float64)) + 1e-12
        assert np.max(np.abs(y - direct) / scale) < 2 ** -7


def test_gemv_bf16_device_form_and_errors(X, dev):
    import torch
    K, N = 768, 512
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((K, N)) * 0.05).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    g = X.GemvBf16(dev, w)
    try:
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty(N, dtype=torch.float32, device="cuda")
        s = torch.cuda.current_stream()
        g.device(xd.data_ptr(), yd.data_ptr(), s.cuda_stream)
        s.synchronize()
        np.testing.assert_array_equal(yd.cpu().numpy(), g(x))
        with pytest.raises(ValueError):
            g(x[:10])
    finally:
        g.free()
    L = X.lib()
    assert L.xdna_gemv_bf16_register(dev.handle, w.ctypes.data, 0, N, None, 0, None, None, 1e-5) is None
    assert L.xdna_gemv_bf16_register(dev.handle, w.ctypes.data, K, N, None, 2, w.ctypes.data, None, 1e-5) is None
    assert "norm" in X.last_error()


def _pack_tiles(k, v, n_heads, n_tiles):
    """CtxDecode::attn's packing (ctx_decode.rs:497-535): per head and tile, K rows, V rows, the
    int32 key count in two bf16 lanes (> 0 full/partial, -count on the last non-empty tile,
    0 empty); rows past the real keys stay zero."""
    S = k.shape[0]
    T, HD = 64, 64
    tile = 2 * T * HD + 2
    kv = np.zeros((n_heads, n_tiles, tile), np.uint16)
    n_real = -(-S // T)
    for h in range(n_heads):
        for t in range(n_tiles):
            r = max(0, min(T, S - t * T))
            kv[h, t, :r * HD] = bf16_bits(k[t * T:t * T + r, h * HD:(h + 1) * HD]).reshape(-1)
            kv[h, t, T * HD:T * HD + r * HD] = bf16_bits(v[t * T:t * T + r, h * HD:(h + 1) * HD]).reshape(-1)
            cnt = 0 if t >= n_real else (-r if t == n_real - 1 else r)
            kv[h, t, 2 * T * HD:] = np.array([cnt], np.int32).view(np.uint16)
    return kv


@pytest.mark.parametrize("S", [1, 17, 63, 64, 65, 200, 448])
def test_mha_decode_paged_matches_f64_softmax(X, S):
    import torch
    H, HD, NT = 12, 64, 7
    rng = np.random.default_rng(S)
    q = (rng.standard_normal(H * HD) * 1.5).astype(np.float32)
    k = rng.standard_normal((S, H * HD)).astype(np.float32)
    v = rng.standard_normal((S, H * HD)).astype(np.float32)
    kv = _pack_tiles(k, v, H, NT)
    qd = torch.from_numpy(bf16_bits(q).view(np.int16)).cuda()
    kvd = torch.from_numpy(kv.view(np.int16)).cuda()
    ctx = torch.full((H * HD,), float("nan"), dtype=torch.float32, device="cuda")
    X.mha_decode_paged(qd.data_ptr(), kvd.data_ptr(), H, NT, ctx.data_ptr(), torch.cuda.current_stream().cuda_stream)
    got = ctx.cpu().numpy().reshape(H, HD)
    qb, kb, vb = (bf16(a).astype(np.float64) for a in (q, k, v))
    for h in range(H):
        sl = slice(h * HD, (h + 1) * HD)
        sc = kb[:, sl] @ qb[sl] / 8.0
        p = np.exp(sc - sc.max())
        ref = (p / p.sum()) @ vb[:, sl]
        np.testing.assert_allclose(got[h], ref, rtol=1e-4, atol=2e-5 * np.abs(vb[:, sl]).max())


def test_buffers_round_trip_and_range_errors(X, dev):
    L = X.lib()
    assert L.xdna_device_ordinal(dev.handle) == dev.ordinal
    n = 1 << 20
    b = L.xdna_buffer_alloc(dev.handle, n)
    assert b
    try:
        ptr = L.xdna_buffer_device_ptr(b)
        assert ptr and ptr % 256 == 0
        data = np.random.default_rng(0).integers(0, 256, n, dtype=np.uint8)
        assert L.xdna_buffer_write(b, data.ctypes.data, n, 0) == 0
        back = np.zeros(n, np.uint8)
        assert L.xdna_buffer_read(b, back.ctypes.data, n, 0) == 0
        np.testing.assert_array_equal(back, data)
        part = np.arange(100, dtype=np.uint8)
        assert L.xdna_buffer_write(b, part.ctypes.data, 100, n - 100) == 0
        tail = np.zeros(100, np.uint8)
        assert L.xdna_buffer_read(b, tail.ctypes.data, 100, n - 100) == 0
        np.testing.assert_array_equal(tail, part)
        assert L.xdna_buffer_write(b, part.ctypes.data, 100, n - 99) == -1
        assert "beyond" in X.last_error()
        assert L.xdna_buffer_read(b, tail.ctypes.data, 1, n) == -1
    finally:
        L.xdna_buffer_free(b)


def test_run_wait_is_bounded(X, dev):
    """shim_run_wait's contract with a limit: 1 while the marked work is still running (a
    bounded spin of ~0.2 s queued before the mark), then 0 once it has finished."""
    import torch
    L = X.lib()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        torch.cuda._sleep(400_000_000)
    r = L.xdna_run_start(dev.handle, s.cuda_stream)
    assert r
    try:
        assert L.xdna_run_wait(r, 0) == 1
        assert "timeout" in X.last_error()
        assert L.xdna_run_wait(r, 60_000) == 0
        assert L.xdna_run_wait(r, 0) == 0
    finally:
        L.xdna_run_free(r)


# ------------------------------------------------------------------ conformer bricks


def _conv_case(seed, ci, h, w, co, k, stride, pad, groups, B=2, zero_frac=0.1):
    rng = np.random.default_rng(seed)
    x = bf16(rng.standard_normal((B, ci, h, w)).astype(np.float32))
    wt = bf16((rng.standard_normal((co, ci // groups, k, k)) * 0.3).astype(np.float32))
    wt[rng.random(wt.shape) < zero_frac] = 0.0
    b = rng.standard_normal(co).astype(np.float32)
    return x, wt, b


@pytest.mark.parametrize("case", [
    dict(ci=1, h=125, w=80, co=256, k=3, stride=2, pad=1, groups=1, relu=1),     # conv.0 (odd frames)
    dict(ci=256, h=63, w=40, co=256, k=3, stride=2, pad=1, groups=256, relu=0),  # conv.2 depthwise
    dict(ci=256, h=32, w=20, co=256, k=1, stride=1, pad=0, groups=1, relu=1),    # conv.3 pointwise
    dict(ci=8, h=9, w=7, co=12, k=3, stride=1, pad=1, groups=4, relu=0),         # grouped, stride 1
])
def test_subsample_conv2d_bit_exact_with_oracle(X, case):
    """Bit-exact against the oracle's conv2d (ops.rs:38-89, pinned to golden_subsample.py's
    im2col == conv gate) on bf16 operands: bf16 x bf16 products are exact in f32, the adds
    follow the same order, one bf16 rounding of the result."""
    import torch
    from oracle import oracle as O
    c = dict(case)
    relu = c.pop("relu")
    x, wt, b = _conv_case(sum(c.values()), **c)
    B = x.shape[0]
    ho = (c["h"] + 2 * c["pad"] - c["k"]) // c["stride"] + 1
    wo = (c["w"] + 2 * c["pad"] - c["k"]) // c["stride"] + 1
    xd = torch.from_numpy(bf16_bits(x).view(np.int16)).cuda()
    wd = torch.from_numpy(bf16_bits(wt).view(np.int16)).cuda()
    bd = torch.from_numpy(b).cuda()
    out = torch.zeros((B, c["co"], ho, wo), dtype=torch.int16, device="cuda")
    rc = X.lib().xdna_subsample_conv2d(xd.data_ptr(), B, c["ci"], c["h"], c["w"], wd.data_ptr(), bd.data_ptr(),
                                       c["co"], c["k"], c["k"], c["stride"], c["pad"], c["groups"], relu,
                                       out.data_ptr(), None)
    assert rc == 0, X.last_error()
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    for bi in range(B):
        ref = O.conv2d(x[bi], wt, b, c["stride"], c["pad"], c["groups"])
        if relu:
            ref = np.maximum(ref, 0.0)
        np.testing.assert_array_equal(got[bi], bf16_bits(ref))


def test_subsample_conv2d_rejects_bad_groups(X):
    assert X.lib().xdna_subsample_conv2d(1, 1, 6, 4, 4, 1, None, 4, 3, 3, 1, 1, 4, 0, 1, None) == -1
    assert "groups" in X.last_error()


@pytest.mark.parametrize("k,T,C,B", [(9, 125, 1024, 2), (9, 1, 1024, 1), (5, 77, 512, 3), (3, 40, 100, 1),
                                     (31, 64, 256, 2)])
def test_dwconv1d_glu_silu_matches_conv_module(X, k, T, C, B):
    """GLU -> dwconv1d (the oracle's, ops.rs:92-110, pinned to golden_dwconv1d_k9.py) -> SiLU,
    as the conv module runs them, within f32 rounding (the exp of CUDA and of the host libm
    may differ by an ulp, so the bar is relative 1e-5 of the term magnitudes)."""
    import torch
    from oracle import oracle as O
    rng = np.random.default_rng(k * 1000 + T)
    x = rng.standard_normal((B, T, 2 * C)).astype(np.float32)
    taps = (rng.standard_normal((C, k)) * 0.3).astype(np.float32)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float32)
    xd, td, bd = (torch.from_numpy(a).cuda() for a in (x, taps, bias))
    yd = torch.full((B, T, C), float("nan"), dtype=torch.float32, device="cuda")
    rc = X.lib().xdna_dwconv1d_glu_silu(xd.data_ptr(), B, T, C, td.data_ptr(), k, bd.data_ptr(), yd.data_ptr(), None)
    assert rc == 0, X.last_error()
    got = yd.cpu().numpy()
    for bi in range(B):
        g = (x[bi, :, :C] * (1.0 / (1.0 + np.exp(-x[bi, :, C:].astype(np.float64))))).astype(np.float32)
        dw = O.dwconv1d(np.ascontiguousarray(g.T), taps, bias).astype(np.float64)
        ref = (dw * (1.0 / (1.0 + np.exp(-dw)))).T
        scale = np.abs(bias)[None, :] + sum(np.abs(np.roll(g, -(j - (k - 1) // 2), axis=0)) * np.abs(taps[:, j])
                                            for j in range(k)) + 1e-30
        np.testing.assert_array_less(np.abs(got[bi] - ref), 1e-5 * scale + 1e-6)
    assert X.lib().xdna_dwconv1d_glu_silu(xd.data_ptr(), B, T, C, td.data_ptr(), 4, bd.data_ptr(), yd.data_ptr(),
                                          None) == -1


@pytest.mark.parametrize("T,B", [(125, 2), (128, 1), (1, 1), (37, 3)])
def test_relpos_mha_matches_attention_core(X, T, B):
    """The rel-pos attention brick against attention_core restated in f64 (rel_shift through the
    oracle's, pinned bit-exact to the reference golden): bf16 tensor-core operands put the bar at
    rel-L2 1e-2 per clip and head."""
    import torch
    from oracle import oracle as O
    H, DK, D = 8, 128, 1024
    rng = np.random.default_rng(T * 10 + B)
    qkv = (rng.standard_normal((B, T, 3 * D)) * 0.5).astype(np.float32)
    pm = (rng.standard_normal((2 * T - 1, D)) * 0.5).astype(np.float32)
    pu = (rng.standard_normal(D) * 0.1).astype(np.float32)
    pv = (rng.standard_normal(D) * 0.1).astype(np.float32)
    qd, pmd, pud, pvd = (torch.from_numpy(a).cuda() for a in (qkv, pm, pu, pv))
    ctx = torch.full((B, T, D), float("nan"), dtype=torch.float32, device="cuda")
    rc = X.lib().xdna_relpos_mha(qd.data_ptr(), pmd.data_ptr(), pud.data_ptr(), pvd.data_ptr(), T, B,
                                 ctx.data_ptr(), None)
    assert rc == 0, X.last_error()
    got = ctx.cpu().numpy()
    for bi in range(B):
        q, k, v = (qkv[bi, :, i * D:(i + 1) * D].astype(np.float64) for i in range(3))
        bd = np.stack([(q[:, h * DK:(h + 1) * DK] + pv[h * DK:(h + 1) * DK]) @ pm[:, h * DK:(h + 1) * DK].T
                       for h in range(H)]).astype(np.float32)
        bds = O.rel_shift(bd).astype(np.float64)
        for h in range(H):
            sl = slice(h * DK, (h + 1) * DK)
            ac = (q[:, sl] + pu[sl]) @ k[:, sl].T
            s = (ac + bds[h]) / np.sqrt(DK)
            p = np.exp(s - s.max(axis=1, keepdims=True))
            ref = (p / p.sum(axis=1, keepdims=True)) @ v[:, sl]
            rel = np.linalg.norm(got[bi, :, sl] - ref) / np.linalg.norm(ref)
            assert rel < 1e-2, (bi, h, rel)
    assert X.lib().xdna_relpos_mha(qd.data_ptr(), pmd.data_ptr(), pud.data_ptr(), pvd.data_ptr(), 129, B,
                                   ctx.data_ptr(), None) == -1


def test_fused_arena_regions(X, dev):
    """FusedArena (lib.rs:641-744): three regions, byte-offset write_at / read_at, a zero-size
    region rounded up to 2 bytes, region index checked."""
    L = X.lib()
    a = L.xdna_arena_create(dev.handle, 4096, 0, 1 << 16)
    assert a, X.last_error()
    try:
        regs = [L.xdna_arena_region(a, i) for i in range(3)]
        ptrs = [L.xdna_buffer_device_ptr(r) for r in regs]
        assert all(ptrs) and len(set(ptrs)) == 3
        assert L.xdna_arena_region(a, 3) is None
        x = np.arange(256, dtype=np.uint8)
        assert L.xdna_arena_write(a, 2, 1000, x.ctypes.data, 256) == 0
        y = np.zeros(256, np.uint8)
        assert L.xdna_arena_read(a, 2, 1000, y.ctypes.data, 256) == 0
        np.testing.assert_array_equal(x, y)
        two = np.array([7, 9], np.uint8)
        assert L.xdna_arena_write(a, 1, 0, two.ctypes.data, 2) == 0
        assert L.xdna_arena_write(a, 1, 1, two.ctypes.data, 2) == -1
        assert L.xdna_arena_write(a, 0, 4095, x.ctypes.data, 2) == -1
    finally:
        L.xdna_arena_free(a)
