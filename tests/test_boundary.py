"""CPU-side checks of the C-ABI boundary: the library loads, exports every entry point the
public headers declare, reports errors the reference's way, and its host-side int8 quantiser
is bit-exact with the oracle (Lin::load, opt125m_decode.rs:41-60)."""
import os
import re

import numpy as np
import pytest

from oracle import oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    src = open(os.path.join(REPO, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(xdna_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def xl():
    import xdna_engine_b200 as X
    from xdna_engine_b200 import _build
    _build.build()
    return X


def test_library_exports_every_declared_symbol(xl):
    L = xl.lib()
    names = _declared("xdna_b200.h")
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), f"missing export {n}"


def test_error_convention_without_device(xl):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert xl.Device.count() == 0
    with pytest.raises(xl.XdnaError):
        xl.Device(0)
    assert xl.last_error() != ""


def test_null_pointer_errors(xl):
    L = xl.lib()
    assert L.xdna_quant_i8_cols(None, 4, 4, None, None) == -1
    assert "null" in xl.last_error()
    assert L.xdna_opt_create(None, None, None, 16, 0) is None
    assert "null" in xl.last_error()
    assert L.xdna_opt_launch(None, 0, 1, 1, None, None) == -1
    assert L.xdna_gemv_i8(None, None, 256, None, None, None, 8, None) == -1


@pytest.mark.parametrize("shape", [(768, 768), (768, 3072), (3072, 768), (256, 40)])
def test_quantiser_bit_exact_with_oracle(xl, shape):
    K, N = shape
    rng = np.random.default_rng(K + N)
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    w[:, 1] = 0.0
    w[5, 2] = 1.0           # one outlier column
    q, s = xl.quant_i8_cols(w)
    oq, os_ = O.quant_i8_cols(w)
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(q, oq.T)


def test_quant_i8_rows_matches_oracle(xl):
    """xdna_quant_i8_rows (qrow, the fused ELF's per-row rule) equals or_quant_i8_rows bit for
    bit; ties round half to even (a row with max 127 has scale exactly 1.0)."""
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((40, 96)) * 0.02).astype(np.float32)
    w[3] = 0.0
    w[7, :6] = [127.0, 2.5, -3.5, 0.5, -0.5, 126.5]
    q, s = xl.quant_i8_rows(w)
    oq, os_ = O.quant_i8_rows(w)
    np.testing.assert_array_equal(s, os_)
    np.testing.assert_array_equal(q, oq)
    assert s[3] == 1.0 and s[7] == 1.0
    assert list(q[7, :6]) == [127, 2, -4, 0, 0, 126]


def test_bfp16_quantize_matches_oracle():
    """xdna_bfp16_quantize (the engine's host-side weight quantiser for bfp16 linears) equals
    or_bfp16_blocks bit for bit, zero blocks and outliers included."""
    import xdna_engine_b200 as X
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(8 * 4096) * np.exp(rng.uniform(-12, 12, 8 * 4096))).astype(np.float32)
    x[:8] = 0.0
    x[8:16] = [1e-30, 0, 0, 0, 0, 0, 0, -1e-30]
    x[16:24] = [1.0, 2.0**-7, -2.0**-6, 3.0, 0, 0, 0, 0]
    got = X.bfp16_quantize(x)
    want = O.bfp16_blocks(x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    with pytest.raises(X.XdnaError):
        X.bfp16_quantize(x[:12])


def test_op_layer_null_errors(xl):
    """The op-by-op entries refuse NULL handles with an error message, no device needed."""
    L = xl.lib()
    assert L.xdna_device_ordinal(None) == -1
    assert L.xdna_buffer_alloc(None, 64) is None
    assert "null" in xl.last_error()
    assert L.xdna_buffer_write(None, None, 0, 0) == -1
    assert L.xdna_arena_create(None, 8, 8, 8) is None
    assert L.xdna_arena_write(None, 0, 0, None, 0) == -1
    L.xdna_arena_free(None)
    assert L.xdna_weights_open(None, None) is None
    assert L.xdna_weights_count(None) == -1
    assert L.xdna_opt_config(None, None) == -1
    assert L.xdna_run_start(None, None) is None
    assert L.xdna_run_wait(None, 0) == -1
    assert L.xdna_gemv_bf16_register(None, None, 8, 8, None, 0, None, None, 1e-5) is None
    assert L.xdna_gemv_bf16(None, None, None) == -1
    assert L.xdna_mha_decode_paged(None, None, 12, 7, None, None) == -1
    assert L.xdna_relpos_mha(None, None, None, None, 125, 1, None, None) == -1
    assert L.xdna_dwconv1d_glu_silu(None, 1, 125, 1024, None, 9, None, None, None) == -1
    assert L.xdna_subsample_conv2d(None, 1, 1, 8, 8, None, None, 4, 3, 3, 2, 1, 1, 1, None, None) == -1
    L.xdna_buffer_free(None)
    L.xdna_run_free(None)
    L.xdna_gemv_bf16_free(None)
