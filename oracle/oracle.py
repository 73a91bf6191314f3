"""ctypes binding of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of bench.py as the checker; the product package
never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I8P = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
I16P = np.ctypeslib.ndpointer(np.int16, flags="C_CONTIGUOUS")
U16P = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
I64P = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")

MODE_REF_F32, MODE_DEVICE, MODE_F32 = 0, 1, 2


def build():
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.or_f32_to_bf16_n.argtypes = [F32P, U16P, C.c_size_t]
        L.or_bf16_round_n.argtypes = [F32P, F32P, C.c_size_t]
        L.or_bf16_round.argtypes = [C.c_float]
        L.or_bf16_round.restype = C.c_float
        L.or_quant_i8_cols.argtypes = [F32P, C.c_int, C.c_int, I8P, F32P]
        L.or_quant_i8_rows.argtypes = [F32P, C.c_int, C.c_int, I8P, F32P]
        L.or_lin_i8_fwd.argtypes = [F32P, I8P, F32P, C.c_void_p, C.c_int, C.c_int, F32P]
        L.or_bfp16_blocks.argtypes = [F32P, F32P, C.c_size_t]
        L.or_bfp16_pack.argtypes = [F32P, C.c_size_t, I16P, I8P]
        L.or_layer_norm.argtypes = [F32P, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, F32P]
        L.or_ln_normalize_f64.argtypes = [F32P, C.c_int, C.c_float, F32P]
        L.or_rms_normalize_f64.argtypes = [F32P, C.c_int, C.c_float, F32P]
        L.or_gemma_rmsnorm.argtypes = [F32P, F32P, C.c_int, C.c_float, F32P]
        for fn in ("or_fast_exp_nonpos", "or_gelu_erf", "or_gelu_tanh", "or_sigmoid", "or_silu"):
            getattr(L, fn).argtypes = [C.c_float]
            getattr(L, fn).restype = C.c_float
        L.or_mha.argtypes = [F32P, F32P, F32P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, F32P]
        L.or_mha_tile_online.argtypes = [F32P, F32P, F32P, C.c_int, C.c_int, C.c_float, F32P]
        L.or_argmax_last.argtypes = [F32P, C.c_size_t]
        L.or_argmax_last.restype = C.c_int64
        L.or_argmax_first.argtypes = [F32P, C.c_size_t]
        L.or_argmax_first.restype = C.c_int64
        L.or_kv_byte_offset.argtypes = [C.c_uint32] * 3
        L.or_kv_byte_offset.restype = C.c_uint32
        L.or_softmax_len.argtypes = [C.c_uint32]
        L.or_softmax_len.restype = C.c_uint32
        L.or_paged_kv_index.argtypes = [np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS"),
                                        C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
        L.or_paged_kv_index.restype = C.c_size_t
        L.or_limbs.argtypes = [F32P, C.c_int, I8P, I8P, I8P]
        L.or_limbs.restype = C.c_int
        L.or_gemv_i8_exact.argtypes = [F32P, I8P, F32P, C.c_void_p, C.c_int, C.c_int, F32P]
        L.or_opt_create.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int]
        L.or_opt_create.restype = C.c_void_p
        L.or_opt_free.argtypes = [C.c_void_p]
        L.or_opt_generate.argtypes = [C.c_void_p, I64P, C.c_int, C.c_int, C.c_void_p, I64P, C.c_void_p]
        L.or_opt_generate.restype = C.c_int
        L.or_opt_set_trace.argtypes = [C.c_void_p, C.c_void_p]
        L.or_bert_embed.argtypes = [C.c_void_p, C.c_void_p, np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS"),
                                    np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS"), C.c_int, F32P, C.c_int]
        L.or_bert_embed.restype = C.c_int
        L.or_whisper_encode.argtypes = [C.c_void_p, C.c_void_p, F32P, C.c_int, F32P, C.c_int]
        L.or_whisper_encode.restype = C.c_int
        L.or_parakeet_encode.argtypes = [C.c_void_p, C.c_void_p, F32P, C.c_int, F32P, C.c_int]
        L.or_parakeet_quant_lin.argtypes = [F32P, C.c_int, C.c_int, F32P, C.c_void_p, C.c_int, F32P, C.c_int]
        L.or_conv2d.argtypes = [F32P, C.c_int, C.c_int, C.c_int, F32P, F32P, C.c_int, C.c_int, C.c_int,
                                C.c_int, C.c_int, C.c_int, F32P, C.c_int]
        L.or_dwconv1d.argtypes = [F32P, C.c_int, C.c_int, F32P, F32P, C.c_int, F32P]
        L.or_rel_shift.argtypes = [F32P, C.c_int, C.c_int, F32P]
        L.or_rel_pos_encoding.argtypes = [C.c_int, C.c_int, F32P]
        L.or_whisper_decode.argtypes = [C.c_void_p, C.c_void_p, F32P, C.c_int, C.c_void_p, C.c_int, C.c_int,
                                        C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]
        L.or_whisper_decode.restype = C.c_int
        L.or_gemma_decode.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p,
                                      C.c_void_p, C.c_int, C.c_void_p]
        L.or_gemma_decode.restype = C.c_int
        L.or_opt_step.argtypes = [C.c_void_p, C.c_int64, C.c_int, C.c_void_p]
        L.or_opt_step.restype = C.c_int64
        L.or_opt_qweight.argtypes = [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.POINTER(C.c_float))]
        L.or_opt_qweight.restype = C.POINTER(C.c_int8)
        _LIB = L
    return _LIB


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data


# ---------------------------------------------------------------- scalar / vector wrappers
def bf16_round(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_bf16_round_n(x.ravel(), y.ravel(), x.size)
    return y


def f32_to_bf16_bits(x):
    x = _f32(x)
    y = np.empty(x.shape, np.uint16)
    lib().or_f32_to_bf16_n(x.ravel(), y.ravel(), x.size)
    return y


def quant_i8_cols(w):
    w = _f32(w)
    K, N = w.shape
    q = np.empty((K, N), np.int8)
    s = np.empty(N, np.float32)
    lib().or_quant_i8_cols(w, K, N, q, s)
    return q, s


def quant_i8_rows(w):
    w = _f32(w)
    M, K = w.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float32)
    lib().or_quant_i8_rows(w, M, K, q, s)
    return q, s


def lin_i8_fwd(x, q, scale, bias=None):
    x, scale = _f32(x), _f32(scale)
    K, N = q.shape
    y = np.empty(N, np.float32)
    b = None if bias is None else _f32(bias)
    lib().or_lin_i8_fwd(x, np.ascontiguousarray(q), scale, _ptr(b), K, N, y)
    return y


def bfp16_blocks(x):
    x = _f32(x)
    y = np.empty_like(x)
    lib().or_bfp16_blocks(x.ravel(), y.ravel(), x.size)
    return y


def bfp16_pack(x):
    x = _f32(x)
    m = np.empty(x.size, np.int16)
    e = np.empty(x.size // 8, np.int8)
    lib().or_bfp16_pack(x.ravel(), x.size, m, e)
    return m, e


def layer_norm(x, g=None, b=None, eps=1e-5):
    x = _f32(x)
    T, D = x.shape
    y = np.empty_like(x)
    g = None if g is None else _f32(g)
    b = None if b is None else _f32(b)
    lib().or_layer_norm(x, _ptr(g), _ptr(b), T, D, eps, y)
    return y


def mha(q, k, v, n_heads, head_dim, round_probs, valid_len):
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty_like(q)
    lib().or_mha(q, k, v, q.shape[0], n_heads, head_dim, int(round_probs), valid_len, out)
    return out


def limbs(x):
    x = _f32(x)
    K = x.size
    a, b, c = (np.empty(K, np.int8) for _ in range(3))
    s = lib().or_limbs(x, K, a, b, c)
    return s, a, b, c


def gemv_i8_exact(x, wq_nk, scale, bias=None):
    x = _f32(x)
    N, K = wq_nk.shape
    y = np.empty(N, np.float32)
    b = None if bias is None else _f32(bias)
    lib().or_gemv_i8_exact(x, np.ascontiguousarray(wq_nk), _f32(scale), _ptr(b), K, N, y)
    return y


# ---------------------------------------------------------------- opt-125m decode
class _Cfg(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int),
                ("max_pos", C.c_int), ("eps", C.c_float)]


class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("ln1_w", "ln1_b", "wq", "wk", "wv", "wo", "bq", "bk",
                                          "bv", "bo", "ln2_w", "ln2_b", "w1", "b1", "w2", "b2")]


class _Weights(C.Structure):
    _fields_ = [("emb_tok", C.c_void_p), ("emb_pos", C.c_void_p), ("lnf_w", C.c_void_p),
                ("lnf_b", C.c_void_p), ("layers", C.c_void_p)]


class OracleOpt:
    """or_opt_* over numpy weights from xdna_engine_b200.synth.make_opt_weights."""

    def __init__(self, cfg, weights, mode=MODE_DEVICE, nthreads=None):
        self._keep = []

        def p(a):
            a = _f32(a)
            self._keep.append(a)
            return a.ctypes.data

        self.cfg = cfg
        c = _Cfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                 cfg.max_pos, cfg.eps)
        layers = (_Layer * cfg.n_layers)()
        for i, ly in enumerate(weights["layers"]):
            for k in _Layer._fields_:
                setattr(layers[i], k[0], p(ly[k[0]]))
        w = _Weights(p(weights["emb_tok"]), p(weights["emb_pos"]), p(weights["lnf_w"]),
                     p(weights["lnf_b"]), C.addressof(layers))
        self._c, self._w, self._layers = c, w, layers
        nt = nthreads or os.cpu_count() or 1
        self._h = lib().or_opt_create(C.addressof(c), C.addressof(w), mode, nt)
        self.mode = mode

    def generate(self, prompt, n_new, want_logits=False, force=None):
        prompt = np.ascontiguousarray(prompt, dtype=np.int64)
        out = np.empty(n_new, np.int64)
        lg = np.empty((n_new, self.cfg.vocab), np.float32) if want_logits else None
        fc = None if force is None else np.ascontiguousarray(force, dtype=np.int64)
        rc = lib().or_opt_generate(self._h, prompt, prompt.size, n_new, _ptr(fc), out, _ptr(lg))
        if rc != 0:
            raise RuntimeError("or_opt_generate failed")
        return (out, lg) if want_logits else out

    def step(self, token_id, pos):
        """One decode step at `pos` (earlier positions already cached); returns the argmax."""
        return int(lib().or_opt_step(self._h, int(token_id), int(pos), None))

    def set_trace(self, buf):
        self._trace = buf
        lib().or_opt_set_trace(self._h, None if buf is None else buf.ctypes.data)

    def qweight(self, layer, which):
        """int8 weight + scale as the oracle quantised them (which: 0..5 q k v o fc1 fc2,
        6 = LM head).  DEVICE mode layout: [N, K]."""
        sp = C.POINTER(C.c_float)()
        qp = lib().or_opt_qweight(self._h, layer, which, C.byref(sp))
        D, F, V = self.cfg.d_model, self.cfg.ffn, self.cfg.vocab
        shapes = [(D, D), (D, D), (D, D), (D, D), (D, F), (F, D), (D, V)]
        K, N = shapes[which]
        q = np.ctypeslib.as_array(qp, shape=(K * N,)).copy()
        s = np.ctypeslib.as_array(sp, shape=(N,)).copy()
        if self.mode == MODE_DEVICE:
            return q.reshape(N, K), s
        return q.reshape(K, N), s

    def close(self):
        if self._h:
            lib().or_opt_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _top2_margin(row):
    """top value minus the best other value (the greedy choice's margin)"""
    i = int(np.argmax(row[::-1]))
    i = row.size - 1 - i                      # last maximum (Iterator::max_by tie rule)
    rest = np.delete(row, i)
    return float(row[i] - rest.max())


def opt_parity_report(cfg, weights, prompt, ids, logits, nthreads=None):
    """Compare a decoded stream (ids [n], logits [n, V], e.g. the GPU's) with the reference's
    own host path (MODE_REF_F32: rust/npu-whisper/src/bin/opt125m_decode.rs:252-315 with
    OPT_INT8).  Returns
      tf_rel_l2      per step, relative L2 of logits against the reference teacher-forced on
                     `ids` (so both see the same history);
      tf_flips       steps where the teacher-forced argmaxes differ, each with the reference's
                     top-2 margin there and the step's max |logit difference|;
      free_first_div first step where the free-running reference stream differs (None if
                     never), with the reference's margin at that step;
      free_match     fraction of positions where the free-running streams agree."""
    n = len(ids)
    ref = OracleOpt(cfg, weights, MODE_REF_F32, nthreads)
    tf_ids, tf_lg = ref.generate(prompt, n, want_logits=True, force=ids)
    ref.close()
    ref = OracleOpt(cfg, weights, MODE_REF_F32, nthreads)
    fr_ids, fr_lg = ref.generate(prompt, n, want_logits=True)
    ref.close()
    rel = [float(np.linalg.norm(logits[t] - tf_lg[t]) / max(np.linalg.norm(tf_lg[t]), 1e-30))
           for t in range(n)]
    flips = []
    for t in range(n):
        if int(tf_ids[t]) != int(ids[t]):
            flips.append({"step": t, "ref_margin": _top2_margin(tf_lg[t]),
                          "max_abs_diff": float(np.abs(logits[t] - tf_lg[t]).max())})
    diff = np.nonzero(np.asarray(fr_ids) != np.asarray(ids))[0]
    first = int(diff[0]) if diff.size else None
    return {"tf_rel_l2": rel, "tf_flips": flips,
            "free_first_div": first,
            "free_div_margin": None if first is None else _top2_margin(fr_lg[first]),
            "free_match": float(np.mean(np.asarray(fr_ids) == np.asarray(ids))),
            "ref_ids": fr_ids}


# ---------------------------------------------------------------- BGE / BERT embedder
_BERT_LAYER = ("q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b", "attn_ln_w", "attn_ln_b",
               "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b", "out_ln_w", "out_ln_b")


class _BertCfg(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int), ("ffn", C.c_int),
                ("vocab", C.c_int), ("max_pos", C.c_int), ("eps", C.c_float), ("pooling", C.c_int)]


class _BertLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _BERT_LAYER]


class _BertWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("word_emb", "pos_emb", "type_emb", "emb_ln_w", "emb_ln_b", "layers")]


def bert_embed(cfg, w, ids, seq_lens, nthreads=None):
    """or_bert_embed: the reference's f32 host embedder on (ids, seq_lens); [n, D] f32."""
    keep = []

    def p(a):
        a = _f32(a)
        keep.append(a)
        return a.ctypes.data

    c = _BertCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.vocab, cfg.max_pos, cfg.eps,
                 cfg.pooling)
    layers = (_BertLayer * cfg.n_layers)()
    for i, ly in enumerate(w["layers"]):
        for n in _BERT_LAYER:
            setattr(layers[i], n, p(ly[n]))
    ww = _BertWeights(p(w["word_emb"]), p(w["pos_emb"]), p(w["type_emb"]), p(w["emb_ln_w"]),
                      p(w["emb_ln_b"]), C.addressof(layers))
    ids = np.ascontiguousarray(ids, np.int32)
    lens = np.ascontiguousarray(seq_lens, np.int32)
    out = np.empty((lens.size, cfg.d_model), np.float32)
    lib().or_bert_embed(C.addressof(c), C.addressof(ww), ids, lens, lens.size, out,
                        nthreads or os.cpu_count() or 1)
    return out


# ---------------------------------------------------------------- Whisper-small encoder
_WENC_LAYER = ("ln1_w", "ln1_b", "q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "out_w", "out_b",
               "ln2_w", "ln2_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")


class _WEncCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "n_heads", "ffn", "n_mels", "n_frames",
                                       "max_src")] + [("eps", C.c_float)]


class _WEncLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _WENC_LAYER]


class _WEncWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("conv1_w", "conv1_b", "conv2_w", "conv2_b", "embed_positions",
                                          "ln_post_w", "ln_post_b", "layers")]


def whisper_encode(cfg, w, mel, nthreads=None):
    """or_whisper_encode: the reference's f32 host encoder; mel [B, n_mels, n_frames]."""
    keep = []

    def p(a):
        a = _f32(a)
        keep.append(a)
        return a.ctypes.data

    c = _WEncCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.n_mels, cfg.n_frames, cfg.max_src, cfg.eps)
    layers = (_WEncLayer * cfg.n_layers)()
    for i, ly in enumerate(w["layers"]):
        for n in _WENC_LAYER:
            setattr(layers[i], n, p(ly[n]))
    ww = _WEncWeights(*[p(w[n]) for n in ("conv1_w", "conv1_b", "conv2_w", "conv2_b", "embed_positions",
                                          "ln_post_w", "ln_post_b")], C.addressof(layers))
    mel = _f32(mel)
    B = mel.shape[0]
    out = np.empty((B, cfg.n_frames // 2, cfg.d_model), np.float32)
    lib().or_whisper_encode(C.addressof(c), C.addressof(ww), mel.ravel(), B, out.ravel(),
                            nthreads or os.cpu_count() or 1)
    return out


# ---------------------------------------------------------------- Parakeet FastConformer encoder
_PK_LAYER = ("ff1_ln_w", "ff1_ln_b", "ff1_w1", "ff1_w2", "att_ln_w", "att_ln_b", "wq", "wk", "wv", "wpos",
             "wout", "pos_u", "pos_v", "conv_ln_w", "conv_ln_b", "pw1", "dw_w", "dw_b", "pw2",
             "ff2_ln_w", "ff2_ln_b", "ff2_w1", "ff2_w2", "out_ln_w", "out_ln_b")
_PK_TOP = ("c0_w", "c0_b", "c2_w", "c2_b", "c3_w", "c3_b", "c5_w", "c5_b", "c6_w", "c6_b", "out_w", "out_b")


class _PkCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "n_heads", "ffn", "n_mels", "n_frames", "sub_ch",
                                       "kconv", "int8")]


class _PkLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _PK_LAYER]


class _PkWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _PK_TOP + ("layers",)]


def parakeet_encode(cfg, w, mel, int8=True, nthreads=None):
    """or_parakeet_encode: the reference's host encoder (int8 engine linears when int8)."""
    keep = []

    def p(a):
        a = _f32(a)
        keep.append(a)
        return a.ctypes.data

    c = _PkCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.n_mels, cfg.n_frames, cfg.sub_ch,
               cfg.kconv, int(int8))
    layers = (_PkLayer * cfg.n_layers)()
    for i, ly in enumerate(w["layers"][:cfg.n_layers]):
        for n in _PK_LAYER:
            setattr(layers[i], n, p(ly[n]))
    ww = _PkWeights(*[p(w[n]) for n in _PK_TOP], C.addressof(layers))
    mel = _f32(mel)
    B = mel.shape[0]
    out = np.empty((B, cfg.frames_out, cfg.d_model), np.float32)
    lib().or_parakeet_encode(C.addressof(c), C.addressof(ww), mel.ravel(), B, out.ravel(),
                             nthreads or os.cpu_count() or 1)
    return out


def quant_lin(x, w, bias=None, nthreads=None):
    """The int8 GEMM engine rule (ctx2.rs): y = (acc * s_a) * ws[n] (+ bias)."""
    x, w = _f32(x), _f32(w)
    T, K = x.shape
    N = w.shape[1]
    y = np.empty((T, N), np.float32)
    b = _f32(bias) if bias is not None else None
    lib().or_parakeet_quant_lin(x.ravel(), T, K, w.ravel(), b.ctypes.data if b is not None else None, N,
                                y.ravel(), nthreads or os.cpu_count() or 1)
    return y


def conv2d(x, w, b, stride, pad, groups):
    x, w, b = _f32(x), _f32(w), _f32(b)
    ci, hin, win = x.shape
    co, _, kh, kw = w.shape
    ho, wo = (hin + 2 * pad - kh) // stride + 1, (win + 2 * pad - kw) // stride + 1
    y = np.empty((co, ho, wo), np.float32)
    lib().or_conv2d(x.ravel(), ci, hin, win, w.ravel(), b.ravel(), co, kh, kw, stride, pad, groups, y.ravel(), 1)
    return y


def dwconv1d(x, taps, bias):
    x, taps, bias = _f32(x), _f32(taps), _f32(bias)
    C_, T = x.shape
    y = np.empty_like(x)
    lib().or_dwconv1d(x.ravel(), C_, T, taps.ravel(), bias.ravel(), taps.shape[1], y.ravel())
    return y


def rel_shift(bd):
    bd = _f32(bd)
    H, T, _ = bd.shape
    y = np.empty((H, T, T), np.float32)
    lib().or_rel_shift(bd.ravel(), H, T, y.ravel())
    return y


def rel_pos_encoding(T, D):
    pe = np.empty((2 * T - 1, D), np.float32)
    lib().or_rel_pos_encoding(T, D, pe.ravel())
    return pe


# ---------------------------------------------------------------- Whisper-small decoder
_WDEC_LAYER = ("ln_self_w", "ln_self_b", "q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "out_w", "out_b",
               "ln_cross_w", "ln_cross_b", "cross_q_w", "cross_q_b", "cross_k_w", "cross_k_b",
               "cross_v_w", "cross_v_b", "cross_out_w", "cross_out_b",
               "ln_final_w", "ln_final_b", "fc1_w", "fc1_b", "fc2_w", "fc2_b")
_WDEC_TOP = ("embed_tokens", "embed_positions", "proj_out", "ln_post_w", "ln_post_b")


class _WDecCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "n_heads", "ffn", "vocab", "max_tgt", "n_enc")]


class _WDecLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _WDEC_LAYER]


class _WDecWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _WDEC_TOP + ("layers",)]


def whisper_decode(cfg, w, enc, prompt, n_new, want_logits=False, nthreads=None, force=None):
    """or_whisper_decode: greedy decode of B streams (enc [B, n_enc, D]) after a shared prompt;
    force ([B, n_new], optional) feeds those tokens instead of the argmaxes (teacher forcing)."""
    keep = []

    def p(a):
        a = _f32(a)
        keep.append(a)
        return a.ctypes.data

    c = _WDecCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.vocab, cfg.max_tgt, cfg.n_enc)
    layers = (_WDecLayer * cfg.n_layers)()
    for i, ly in enumerate(w["layers"][:cfg.n_layers]):
        for n in _WDEC_LAYER:
            setattr(layers[i], n, p(ly[n]))
    ww = _WDecWeights(*[p(w[n]) for n in _WDEC_TOP], C.addressof(layers))
    enc = _f32(enc)
    B = enc.shape[0]
    pr = np.ascontiguousarray(prompt, np.int64)
    fc = None if force is None else np.ascontiguousarray(force, np.int64).reshape(B, n_new)
    toks = np.empty((B, n_new), np.int64)
    lg = np.empty((B, n_new, cfg.vocab), np.float32) if want_logits else None
    rc = lib().or_whisper_decode(C.addressof(c), C.addressof(ww), enc.ravel(), B, pr.ctypes.data, len(pr), n_new,
                                 toks.ctypes.data, lg.ctypes.data if lg is not None else None,
                                 nthreads or os.cpu_count() or 1, _ptr(fc))
    if rc != 0:
        raise ValueError("or_whisper_decode: prompt + new tokens beyond max_tgt")
    return (toks, lg) if want_logits else toks


# ---------------------------------------------------------------- Gemma-3 text decoder
_GM_LAYER = ("in_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "post_attn_norm", "pre_ffn_norm", "wg", "wu",
             "wd", "post_ffn_norm")


class _GmCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "n_q_heads", "head_dim", "ffn", "vocab", "window",
                                       "pattern")] + \
               [(n, C.c_float) for n in ("theta_local", "theta_global", "query_pre_attn_scalar", "eps")] + \
               [("int8", C.c_int)]


class _GmLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _GM_LAYER]


class _GmWeights(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p), ("layers", C.c_void_p)]


def gemma_decode(cfg, w, prompt, n_new, int8=True, want_logits=False, nthreads=None, force=None):
    """or_gemma_decode: greedy decode of one stream after the prompt; force ([n_new], optional)
    feeds those tokens instead of the argmaxes (teacher forcing)."""
    keep = []

    def p(a):
        a = _f32(a)
        keep.append(a)
        return a.ctypes.data

    c = _GmCfg(cfg.n_layers, cfg.d_model, cfg.n_q_heads, cfg.head_dim, cfg.ffn, cfg.vocab, cfg.window, cfg.pattern,
               cfg.theta_local, cfg.theta_global, cfg.query_pre_attn_scalar, cfg.eps, int(int8))
    layers = (_GmLayer * cfg.n_layers)()
    for i, ly in enumerate(w["layers"][:cfg.n_layers]):
        for n in _GM_LAYER:
            setattr(layers[i], n, p(ly[n]))
    ww = _GmWeights(p(w["embed"]), p(w["final_norm"]), C.addressof(layers))
    pr = np.ascontiguousarray(prompt, np.int64)
    toks = np.empty(n_new, np.int64)
    lg = np.empty((n_new, cfg.vocab), np.float32) if want_logits else None
    fc = None if force is None else np.ascontiguousarray(force, np.int64)
    lib().or_gemma_decode(C.addressof(c), C.addressof(ww), pr.ctypes.data, len(pr), n_new, toks.ctypes.data,
                          lg.ctypes.data if lg is not None else None, nthreads or os.cpu_count() or 1, _ptr(fc))
    return (toks, lg) if want_logits else toks
