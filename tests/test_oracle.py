"""Pin the CPU oracle before trusting it: every function is checked against the
reference's own known-answer tests (tests/golden/ref_kats.json), the reference's numpy
bfp16 golden (bfp16_golden.npz) and HuggingFace OPT (opt_hf_golden.npz)."""
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_bf16_round_kats(kats):
    k = kats["bf16_round"]
    x = np.array([c[0] for c in k["cases"]], np.float32)
    want = np.array([c[1] for c in k["cases"]], np.float32)
    np.testing.assert_allclose(O.bf16_round(x), want, atol=k["tol"], rtol=0)
    assert np.isnan(O.bf16_round(np.array([np.nan], np.float32))[0])


def test_bf16_all_patterns_match_ml_dtypes():
    """rust/npu-xrt/src/lib.rs:1064-1123 sweeps every bf16 pattern and a 200k LCG sweep of
    f32 bits; here the independent reference is ml_dtypes' RNE cast (which the reference
    states it matches, rust/npu-asr-host/src/lib.rs:10-11)."""
    ml = pytest.importorskip("ml_dtypes")
    bits16 = np.arange(0, 1 << 16, dtype=np.uint32)
    f = (bits16 << 16).view(np.float32)
    got = O.f32_to_bf16_bits(f)
    finite = ~np.isnan(f)
    assert np.array_equal(got[finite], bits16[finite].astype(np.uint16))
    s = np.uint32(0x12345678)
    xs = np.empty(200_000, np.uint32)
    for i in range(xs.size):      # the reference's LCG: s = s*1664525 + 1013904223
        s = np.uint32((int(s) * 1664525 + 1013904223) & 0xFFFFFFFF)
        xs[i] = s
    x = xs.view(np.float32)
    ok = ~np.isnan(x)
    want = x[ok].astype(ml.bfloat16).view(np.uint16)
    assert np.array_equal(O.f32_to_bf16_bits(x)[ok], want)
    # NaNs stay NaN (quiet bit set), as f32_to_bf16_bits does
    nb = O.f32_to_bf16_bits(x[~ok])
    assert np.all((nb & 0x7F80) == 0x7F80) and np.all(nb & 0x0040)


def test_layer_norm_kats(kats):
    k = kats["layer_norm"]
    y = O.layer_norm(np.array(k["x"], np.float32), k["gamma"], k["beta"], k["eps"])
    np.testing.assert_allclose(y.ravel(), k["expected"], atol=k["tol"], rtol=0)
    k = kats["layer_norm_normalize"]
    y = O.layer_norm(np.array(k["x"], np.float32), None, None, k["eps"])
    np.testing.assert_allclose(y.ravel(), k["expected"], atol=k["tol"], rtol=0)


@pytest.mark.parametrize("round_probs", [False, True])
def test_mha_kats(kats, round_probs):
    k = kats["mha"]
    sh = (3, k["n_heads"] * k["head_dim"])
    q, kk, v = (np.array(k[n], np.float32).reshape(sh) for n in ("q", "k", "v"))
    out = O.mha(q, kk, v, k["n_heads"], k["head_dim"], round_probs, k["valid_len"])
    want = k["expected_round" if round_probs else "expected_no_round"]
    np.testing.assert_allclose(out.ravel(), want, atol=k["tol"], rtol=0)


def test_mha_valid_len_masks_keys():
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((6, 8)).astype(np.float32) for _ in range(3))
    a = O.mha(q, k, v, 2, 4, False, 4)
    # keys >= valid_len must not matter
    k2, v2 = k.copy(), v.copy()
    k2[4:] = 100.0
    v2[4:] = -7.0
    b = O.mha(q, k2, v2, 2, 4, False, 4)
    np.testing.assert_array_equal(a, b)


def test_activation_kats(kats):
    L = O.lib()
    k = kats["sigmoid_silu"]
    np.testing.assert_allclose([L.or_sigmoid(x) for x in k["x"]], k["sigmoid"], atol=k["tol"])
    np.testing.assert_allclose([L.or_silu(x) for x in k["x"]], k["silu"], atol=k["tol"])
    k = kats["gelu_erf"]
    np.testing.assert_allclose([L.or_gelu_erf(x) for x in k["x"]], k["expected"], atol=k["tol"])
    k = kats["glu"]
    x = np.array(k["x"], np.float32)
    c = x.shape[0] // 2
    glu = np.array([[x[i, t] * L.or_sigmoid(float(x[c + i, t])) for t in range(x.shape[1])]
                    for i in range(c)], np.float32)
    np.testing.assert_allclose(glu.ravel(), k["expected"], atol=k["tol"])
    k = kats["fast_exp"]
    xs = np.arange(k["lo"], k["hi"] + 1e-9, k["step"], dtype=np.float64).astype(np.float32)
    got = np.array([L.or_fast_exp_nonpos(float(x)) for x in xs[::7]], np.float64)
    ref = np.exp(xs[::7].astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < k["max_rel"]
    # gelu_tanh reference points (torch's gelu(approximate='tanh'))
    for xv, want in [(0.0, 0.0), (1.0, 0.841191990), (-1.0, -0.158808009), (2.0, 1.954597689)]:
        assert abs(L.or_gelu_tanh(xv) - want) < 1e-5


def test_kv_patch_kats(kats):
    k = kats["kv_patch"]
    L = O.lib()
    for base, want in zip(k["bases"], k["expected_kv"]):
        assert L.or_kv_byte_offset(base, k["n_preceding"], k["head_dim"]) == want
    assert L.or_softmax_len(k["n_preceding"]) == k["expected_softmax_len"]


def test_gemma_rmsnorm_unit(kats):
    k = kats["gemma_rmsnorm_unit"]
    y = np.empty(4, np.float32)
    O.lib().or_gemma_rmsnorm(np.array(k["x"], np.float32), np.array(k["w"], np.float32), 4,
                             k["eps"], y)
    assert np.all(np.abs(np.abs(y) - 1.0) < k["abs_one_tol"])


def test_bfp16_matches_reference_golden():
    g = np.load(os.path.join(GOLD, "bfp16_golden.npz"))
    np.testing.assert_array_equal(O.bf16_round(g["a"]), g["a_bf16"])
    # blocks run along K: axis 1 of A (rows contiguous), axis 0 of B (transpose first)
    np.testing.assert_array_equal(O.bfp16_blocks(O.bf16_round(g["a"])), g["a_blocks_ax1"])
    bt = np.ascontiguousarray(O.bf16_round(g["b"]).T)
    np.testing.assert_array_equal(O.bfp16_blocks(bt).T, g["b_blocks_ax0"])
    wt = np.ascontiguousarray(g["w02"].T)
    np.testing.assert_array_equal(O.bfp16_blocks(wt).T, g["w02_blocks_ax0"])
    np.testing.assert_array_equal(O.bfp16_blocks(g["edge"]), g["edge_blocks_ax1"])
    ab = O.bfp16_blocks(O.bf16_round(g["a"]))
    bb = O.bfp16_blocks(bt).T
    np.testing.assert_allclose(ab @ bb, g["gemm_bfp16"], rtol=1e-5, atol=1e-5)
    # storage form: mantissa * 2^(e-6) reproduces the block values; |m| may reach 128
    m, e = O.bfp16_pack(g["w02"].T.copy())
    vals = m.reshape(-1, 8).astype(np.float64) * np.exp2(e.astype(np.float64) - 6)[:, None]
    np.testing.assert_array_equal(vals.ravel().astype(np.float32), O.bfp16_blocks(wt).ravel())
    assert np.abs(m).max() <= 128


def test_int8_quant_rules():
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((96, 40)) * 0.02).astype(np.float32)
    w[:, 3] = 0.0                                   # all-zero column -> scale 1.0
    q, s = O.quant_i8_cols(w)
    amax = np.abs(w).max(axis=0)
    want_s = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    np.testing.assert_array_equal(s, want_s)
    r = w / s[None, :]
    want_q = np.clip(np.sign(r) * np.floor(np.abs(r) + np.float32(0.5)), -127, 127)
    np.testing.assert_array_equal(q, want_q.astype(np.int8))
    assert np.abs(q).max() == 127 and np.all(q[:, 3] == 0)
    # qrow (gen_decode.py:158-165) rounds half to even
    qr, sr = O.quant_i8_rows(w.T.copy())
    want = np.clip(np.round(w.T / sr[:, None]), -127, 127).astype(np.int8)
    np.testing.assert_array_equal(qr, want)


def test_lin_i8_fwd_matches_ref_loop():
    rng = np.random.default_rng(6)
    w = (rng.standard_normal((64, 24)) * 0.02).astype(np.float32)
    x = rng.standard_normal(64).astype(np.float32)
    b = rng.standard_normal(24).astype(np.float32)
    q, s = O.quant_i8_cols(w)
    y = np.zeros(24, np.float32)
    for k in range(64):                      # Lin::fwd order, f32
        y = (y + (x[k] * q[k].astype(np.float32)).astype(np.float32)).astype(np.float32)
    y = (y * s).astype(np.float32) + b
    np.testing.assert_array_equal(O.lin_i8_fwd(x, q, s, b), y)


def test_limbs_exact_dot():
    rng = np.random.default_rng(8)
    for K in (64, 768, 3072):
        x = O.bf16_round(rng.standard_normal(K).astype(np.float32) * 3)
        x[::17] *= 1e-6                          # tiny elements exercise the rounding
        s, a, b, c = O.limbs(x)
        X = a.astype(np.int64) * 65536 + b.astype(np.int64) * 256 + c
        assert np.all(np.abs(a.astype(int)) <= 64)
        np.testing.assert_array_equal(X, np.rint(x.astype(np.float64) * 2.0 ** s).astype(np.int64))
        w = rng.integers(-127, 128, size=(5, K)).astype(np.int8)
        sc = np.ones(5, np.float32)
        y = O.gemv_i8_exact(x, w, sc)
        exact = (w.astype(np.int64) @ X).astype(np.float64)
        np.testing.assert_array_equal(y, np.ldexp(exact.astype(np.float32), -s).astype(np.float32))
    s, a, b, c = O.limbs(np.zeros(16, np.float32))
    assert not a.any() and not b.any() and not c.any()


def test_argmax_tie_rules():
    x = np.array([1.0, 3.0, 2.0, 3.0, 0.5], np.float32)
    assert O.lib().or_argmax_last(x, 5) == 3
    assert O.lib().or_argmax_first(x, 5) == 1


def test_paged_kv_index():
    pt = np.array([5, 2, 7], np.int32)
    H, hd, P = 3, 4, 8
    L = O.lib()
    seen = set()
    for pos in range(24):
        for kv in range(2):
            for h in range(H):
                for d in range(hd):
                    i = L.or_paged_kv_index(pt, P, H, hd, kv, h, pos, d)
                    page = i // (2 * H * P * hd)
                    assert page == pt[pos // P]
                    seen.add(i)
    assert len(seen) == 24 * 2 * H * hd


def _opt_small():
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    cfg, w = G.opt_small_weights()
    return G, cfg, w


def test_opt_f32_matches_hf_golden():
    G, cfg, w = _opt_small()
    f = np.load(os.path.join(GOLD, "opt_hf_golden.npz"))
    assert abs(G.weights_checksum(w) - float(f["checksum"])) < 1e-6 * float(f["checksum"])
    m = O.OracleOpt(cfg, w, O.MODE_F32, 2)
    ids, lg = m.generate(f["prompt"], len(f["tokens"]), True)
    np.testing.assert_array_equal(ids, f["tokens"])
    rel = np.linalg.norm(lg - f["logits"], axis=1) / np.linalg.norm(f["logits"], axis=1)
    assert rel.max() < 1e-5


@pytest.mark.parametrize("mode", [O.MODE_REF_F32, O.MODE_DEVICE])
def test_opt_int8_modes_track_hf(mode):
    """int8 weights (and bf16 activations in device mode) stay within 3e-2 relative of the
    f32 HF logits when both are teacher-forced on HF's token stream."""
    G, cfg, w = _opt_small()
    f = np.load(os.path.join(GOLD, "opt_hf_golden.npz"))
    m = O.OracleOpt(cfg, w, mode, 2)
    ids, lg = m.generate(f["prompt"], len(f["tokens"]), True, force=f["tokens"])
    rel = np.linalg.norm(lg - f["logits"], axis=1) / np.linalg.norm(f["logits"], axis=1)
    assert rel.max() < 3e-2


def test_opt_thread_count_invariant():
    G, cfg, w = _opt_small()
    f = np.load(os.path.join(GOLD, "opt_hf_golden.npz"))
    outs = []
    for nt in (1, 3):
        m = O.OracleOpt(cfg, w, O.MODE_DEVICE, nt)
        outs.append(m.generate(f["prompt"], 6, True))
    np.testing.assert_array_equal(outs[0][0], outs[1][0])
    np.testing.assert_array_equal(outs[0][1], outs[1][1])


def test_bert_oracle_matches_hf_golden():
    """or_bert_embed (the reference's host BERT embedder restated) vs HF BertModel, the
    implementation the reference checks BGE against (scripts/bge_reference.py)."""
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    cfg, w = G.bert_small_weights()
    f = np.load(os.path.join(GOLD, "bert_hf_golden.npz"))
    e = O.bert_embed(cfg, w, f["ids"], f["lens"], 2)
    np.testing.assert_allclose(e, f["emb"], atol=1e-5, rtol=0)


def test_whisper_encoder_oracle_matches_hf_golden():
    """or_whisper_encode (encoder.rs conv_stem/block/forward_last restated) vs HF
    WhisperEncoder.last_hidden_state on a small seeded encoder, 2 clips."""
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    cfg, w, mel = G.whisper_small_weights()
    f = np.load(os.path.join(GOLD, "whisper_hf_golden.npz"))
    e = O.whisper_encode(cfg, w, mel, 2)
    np.testing.assert_allclose(e, f["enc"], atol=1e-4, rtol=0)  # A&S erf in GELU vs exact erf


# ------------------------------------------------------------------ Parakeet primitives
def _pk_gold():
    return np.load(os.path.join(GOLD, "parakeet_golden.npz"))


def test_parakeet_rel_shift_matches_reference_golden():
    """or_rel_shift (ops.rs:113-133) vs the reference's numpy rel_shift_host, bit-exact,
    including T = 1 and 2."""
    f = _pk_gold()
    for T in (1, 2, 9, 31):
        np.testing.assert_array_equal(O.rel_shift(f[f"bd_{T}"]), f[f"shift_{T}"])


def test_parakeet_dwconv_matches_reference_golden():
    """or_dwconv1d (ops.rs:92-110) vs golden_dwconv1d_k9.host_reference (fp32, C=1024, T=400)."""
    f = _pk_gold()
    x = np.random.default_rng(78).standard_normal((1024, 400)).astype(np.float32)
    dw = (np.random.default_rng(79).standard_normal((1024, 9)) / 3).astype(np.float32)
    db = (np.random.default_rng(80).standard_normal(1024) * 0.02).astype(np.float32)
    y = O.dwconv1d(x, dw, db)
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    np.testing.assert_allclose(y[G.PK_DW_CHANNELS], f["dw_out"], rtol=0, atol=2e-6)
    assert abs(np.sum(y.astype(np.float64)) - float(f["dw_sum"])) < 1e-3


def test_parakeet_conv2d_matches_reference_golden():
    """or_conv2d (ops.rs:38-89: strided, depthwise, pointwise) vs golden_subsample.conv2d_ref."""
    f = _pk_gold()
    for i in range(4):
        st, pd, g = (int(v) for v in f[f"c2d_meta{i}"])
        y = O.conv2d(f[f"c2d_x{i}"], f[f"c2d_w{i}"], f[f"c2d_b{i}"], st, pd, g)
        np.testing.assert_allclose(y, f[f"c2d_y{i}"], rtol=1e-5, atol=1e-5)


def test_parakeet_rel_pos_encoding_rows():
    """pos.rs:7-47: 2T-1 rows, positions T-1 .. 0 .. -(T-1); row T-1 is position 0
    (sin 0 = 0, cos 0 = 1) and rows T-1-p and T-1+p are mirror images (sin odd, cos even)."""
    for T in (1, 2, 5, 125):
        pe = O.rel_pos_encoding(T, 16)
        assert pe.shape == (2 * T - 1, 16)
        np.testing.assert_array_equal(pe[T - 1, 0::2], 0.0)
        np.testing.assert_array_equal(pe[T - 1, 1::2], 1.0)
        for p in range(1, T):
            np.testing.assert_array_equal(pe[T - 1 - p, 0::2], -pe[T - 1 + p, 0::2])
            np.testing.assert_array_equal(pe[T - 1 - p, 1::2], pe[T - 1 + p, 1::2])
    pe = O.rel_pos_encoding(3, 4)
    div1 = np.exp(-np.log(10000.0) * 2 / 4)
    np.testing.assert_allclose(pe[0], np.array([np.sin(2.0), np.cos(2.0), np.sin(2 * div1), np.cos(2 * div1)],
                                               np.float32), rtol=1e-7)


def test_parakeet_int8_linear_rule():
    """or_parakeet_quant_lin follows ctx2.rs: per-column weight scale, dynamic per-tensor
    activation scale, round-half-away quantisation, exact i32 dot, (acc * s_a) * ws + b."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((7, 64)).astype(np.float32)
    x[3, 5] = 4.0                                     # the tensor max -> +127 exactly
    w = (rng.standard_normal((64, 24)) * 0.02).astype(np.float32)
    w[:, 3] = 0.0                                     # zero column -> scale 1.0
    b = rng.standard_normal(24).astype(np.float32)
    y = O.quant_lin(x, w, b)
    sa = np.float32(np.abs(x).max()) / np.float32(127)
    xq = np.clip(np.trunc(x / sa + np.copysign(np.float32(0.5), x / sa)), -127, 127).astype(np.int64)
    amax = np.abs(w).max(0)
    ws = np.where(amax > 0, amax / np.float32(127), np.float32(1)).astype(np.float32)
    wq = np.clip(np.trunc(w / ws + np.copysign(np.float32(0.5), w / ws)), -127, 127).astype(np.int64)
    acc = xq @ wq
    want = ((acc.astype(np.float32) * sa).astype(np.float32) * ws).astype(np.float32) + b
    np.testing.assert_array_equal(y, want)
    assert xq[3, 5] == 127


def test_parakeet_oracle_int8_tracks_f32():
    """The int8-engine encoder stays close to the reference's f32 host encoder."""
    from xdna_engine_b200.synth import ParakeetConfig, make_parakeet_weights, make_parakeet_mel
    cfg = ParakeetConfig(n_layers=2, n_frames=120)
    w = make_parakeet_weights(cfg, seed=2)
    mel = make_parakeet_mel(cfg, 1, 2)
    a = O.parakeet_encode(cfg, w, mel, int8=True)
    b = O.parakeet_encode(cfg, w, mel, int8=False)
    cos = (a * b).sum(-1) / np.linalg.norm(a, axis=-1) / np.linalg.norm(b, axis=-1)
    assert a.shape == (1, 15, 1024) and cos.min() > 0.999


def test_whisper_decoder_oracle_matches_hf_golden():
    """or_whisper_decode (HostDecoder::step restated) vs HF WhisperDecoder + tied proj_out:
    the same greedy tokens, logits to 1e-4 (A&S erf in GELU vs the exact erf)."""
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    cfg, w, enc = G.whisper_dec_small()
    f = np.load(os.path.join(GOLD, "whisper_dec_hf_golden.npz"))
    toks, lg = O.whisper_decode(cfg, w, enc, G.WHISPER_DEC_PROMPT, 12, want_logits=True, nthreads=2)
    np.testing.assert_array_equal(toks, f["tokens"])
    np.testing.assert_allclose(lg, f["logits"], atol=1e-4, rtol=0)


def test_gemma_oracle_matches_hf_golden():
    """or_gemma_decode (npu-gemma's rmsnorm_ref / geglu_ref / is_global_layer + the HF Gemma-3
    model it ports) vs HF Gemma3ForCausalLM: same greedy tokens, logits to 1e-5, with a
    sliding window of 8 crossed by the 10-token prompt and one global layer in 7."""
    import sys
    sys.path.insert(0, GOLD)
    import make_golden as G
    cfg, w = G.gemma_small()
    f = np.load(os.path.join(GOLD, "gemma_hf_golden.npz"))
    toks, lg = O.gemma_decode(cfg, w, G.GEMMA_PROMPT, 12, int8=False, want_logits=True, nthreads=2)
    np.testing.assert_array_equal(toks, f["tokens"])
    np.testing.assert_allclose(lg, f["logits"], atol=1e-5, rtol=0)
    # the int8 Lin rule on the same model keeps the greedy stream for most steps
    t8 = O.gemma_decode(cfg, w, G.GEMMA_PROMPT, 12, int8=True, nthreads=2)
    assert (t8[:4] == f["tokens"][:4]).all()


def test_gemma_geglu_and_layer_pattern():
    """npu-gemma lib.rs geglu_shapes (gelu_tanh(0) * u = 0) and config.rs gqa_and_layer_pattern
    ((i + 1) % 6 == 0 is global: layers 5 and 17 of 18, not 0)."""
    import ctypes
    O.lib().or_gelu_tanh_gemma.restype = ctypes.c_float
    O.lib().or_gelu_tanh_gemma.argtypes = [ctypes.c_float]
    assert O.lib().or_gelu_tanh_gemma(0.0) == 0.0
    assert abs(O.lib().or_gelu_tanh_gemma(1.0) - 0.8411920) < 1e-6
    glob = [(i + 1) % 6 == 0 for i in range(18)]
    assert glob[5] and glob[17] and not glob[0]


def test_opt_device_numerics_track_reference_host_path():
    """The engine's device numerics (bf16 activations, 29-bit fixed-point exact int8 GEMVs,
    int8 LM head), restated by the oracle, against the reference's own host path
    (opt125m_decode.rs:252-315 with OPT_INT8) at the BASELINE config over all 128 tokens:
    teacher-forced logits within 1e-2 relative L2 at every step, and every argmax that differs
    is a near tie (reference top-2 margin below the step's largest |logit difference|)."""
    from xdna_engine_b200.synth import OPT_125M, make_opt_weights, make_prompt
    w = make_opt_weights(OPT_125M, seed=0)
    prompt = make_prompt(OPT_125M, 32, seed=0)
    ids, lg = O.OracleOpt(OPT_125M, w, O.MODE_DEVICE).generate(prompt, 128, want_logits=True)
    rep = O.opt_parity_report(OPT_125M, w, prompt, ids, lg)
    assert max(rep["tf_rel_l2"]) <= 1e-2
    for f in rep["tf_flips"]:
        assert f["ref_margin"] < f["max_abs_diff"], f
    if rep["free_first_div"] is not None:
        assert rep["free_div_margin"] < max(f["max_abs_diff"] for f in rep["tf_flips"] or [{"max_abs_diff": 1.0}])
