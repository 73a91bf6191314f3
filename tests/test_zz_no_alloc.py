"""xdna_gemv_i8_noalloc: the GEMV entry point for hosts that cannot allocate device memory
(their device memory belongs to another allocator or a reserved arena).  It stages through
one fixed 8 MiB device array instead of cudaMalloc, so its results must equal the allocating
xdna_gemv_i8 bit for bit -- the GEMV tests' bar -- on consecutive calls that reuse the
array, and oversized calls must be refused rather than overrun it.

This file is named to be collected last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process."""
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


def _call_noalloc(X, x, q_nk, scale, bias):
    N, K = q_nk.shape
    y = np.empty(N, np.float32)
    rc = X.lib().xdna_gemv_i8_noalloc(0, x.ctypes.data, K, q_nk.ctypes.data, scale.ctypes.data,
                                      None if bias is None else bias.ctypes.data, N, y.ctypes.data)
    if rc != 0:
        raise X.XdnaError(X.last_error())
    return y


def _case(seed, K, N, with_bias):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(K).astype(np.float32)
    q = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = (rng.random(N).astype(np.float32) * 1e-3 + 1e-4).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32) if with_bias else None
    return x, q, s, b


def test_noalloc_matches_allocating_gemv_twice(X):
    dev = X.Device(0)
    cases = [_case(1, 768, 2304, True), _case(2, 3072, 768, False)]
    for x, q, s, b in cases:                       # two calls in a row reuse the array
        got = _call_noalloc(X, x, q, s, b)
        want = dev.gemv_i8(x, q, s, b)
        np.testing.assert_array_equal(got, want)
    # the first case again after the second overwrote the array
    x, q, s, b = cases[0]
    np.testing.assert_array_equal(_call_noalloc(X, x, q, s, b), dev.gemv_i8(x, q, s, b))


def test_noalloc_rejects_oversized_call(X):
    x, q, s, b = _case(3, 3072, 2048, True)          # 2 x 6.3 MB of staging > 8 MiB
    with pytest.raises(X.XdnaError, match="8 MiB"):
        _call_noalloc(X, x, q, s, b)


def _call_noalloc_on(X, device, x, q_nk, scale, bias):
    N, K = q_nk.shape
    y = np.empty(N, np.float32)
    rc = X.lib().xdna_gemv_i8_noalloc(device, x.ctypes.data, K, q_nk.ctypes.data, scale.ctypes.data,
                                      None if bias is None else bias.ctypes.data, N, y.ctypes.data)
    if rc != 0:
        raise X.XdnaError(X.last_error())
    return y


def test_noalloc_restores_current_device(X):
    import torch
    before = torch.cuda.current_device()
    x, q, s, b = _case(4, 768, 768, True)
    _call_noalloc_on(X, 0, x, q, s, b)
    assert torch.cuda.current_device() == before


def test_noalloc_per_device_scratch():
    """device 0, then device 1, then device 0 again: each GPU has its own copy of the array
    and its own launch attributes, so every call equals that device's allocating GEMV."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import xdna_engine_b200 as X
    devs = [X.Device(0), X.Device(1)]
    x, q, s, b = _case(5, 768, 1536, True)
    for d in (0, 1, 0):
        got = _call_noalloc_on(X, d, x, q, s, b)
        np.testing.assert_array_equal(got, devs[d].gemv_i8(x, q, s, b))
