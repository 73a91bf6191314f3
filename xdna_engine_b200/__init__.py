"""xdna_engine_b200 -- B200 (sm_100a) backend for xdna-engine's fused transformer hot path.

The product is the C-ABI library libxdna_b200.so (include/xdna_b200.h), built in-tree by
xdna_engine_b200._build.  This module is a thin ctypes binding that mirrors the reference's
host interface for the decode path (rust/npu-whisper/src/bin/opt125m_decode.rs: Opt::load,
Opt::generate) so Python callers and the tests drive exactly the C ABI a Rust/C host would.

There is no CPU fallback: if the library or a B200 is missing, the calls raise.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .synth import (OPT_125M, OptConfig, make_opt_weights, make_prompt,  # noqa: F401
                    BGE_BASE, BertConfig, make_bert_weights, make_bge_batch,
                    WHISPER_SMALL_ENC, WhisperEncConfig, make_whisper_enc_weights, make_mel,
                    PARAKEET_V3, ParakeetConfig, make_parakeet_weights, make_parakeet_mel,
                    WHISPER_SMALL_DEC, WhisperDecConfig, make_whisper_dec_weights, make_encoder_states,
                    WHISPER_PROMPT, GEMMA3_1B, GemmaConfig, make_gemma_weights)

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libxdna_b200.so")
_LIB = None


class XdnaError(RuntimeError):
    pass


class _OptConfig(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int),
                ("max_pos", C.c_int), ("eps", C.c_float)]


_LAYER_FIELDS = ("ln1_w", "ln1_b", "wq", "wk", "wv", "wo", "bq", "bk", "bv", "bo",
                 "ln2_w", "ln2_b", "w1", "b1", "w2", "b2")


class _OptLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _LAYER_FIELDS]


class _OptWeights(C.Structure):
    _fields_ = [("emb_tok", C.c_void_p), ("emb_pos", C.c_void_p), ("lnf_w", C.c_void_p),
                ("lnf_b", C.c_void_p), ("layers", C.c_void_p)]


def lib():
    """Load libxdna_b200.so (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise XdnaError(f"{LIB_PATH} missing: run `python -m xdna_engine_b200._build`")
        L = C.CDLL(LIB_PATH)
        vp, i, sz = C.c_void_p, C.c_int, C.c_size_t
        L.xdna_last_error.restype = C.c_char_p
        L.xdna_device_count.restype = i
        L.xdna_device_open.argtypes = [i]
        L.xdna_device_open.restype = vp
        L.xdna_device_close.argtypes = [vp]
        L.xdna_quant_i8_cols.argtypes = [vp, i, i, vp, vp]
        L.xdna_quant_i8_cols.restype = i
        L.xdna_quant_i8_rows.argtypes = [vp, i, i, vp, vp]
        L.xdna_quant_i8_rows.restype = i
        L.xdna_gemv_i8.argtypes = [vp, vp, i, vp, vp, vp, i, vp]
        L.xdna_gemv_i8.restype = i
        L.xdna_gemv_i8_noalloc.argtypes = [i, vp, i, vp, vp, vp, i, vp]
        L.xdna_gemv_i8_noalloc.restype = i
        L.xdna_gemm_bf16.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, vp]
        L.xdna_gemm_bf16.restype = i
        L.xdna_gemm_check.restype = i
        L.xdna_ffn_fused_bf16.argtypes = [vp, vp, vp, i, vp, vp, vp, vp, vp, i, i, i, i, vp]
        L.xdna_ffn_fused_bf16.restype = i
        L.xdna_ffn_fused_check.restype = i
        L.xdna_ffn_fused_set_trace.argtypes = [vp]
        L.xdna_attention_bf16.argtypes = [vp, i, vp, i, i, vp, vp]
        L.xdna_attention_bf16.restype = i
        L.xdna_attention_check.restype = i
        L.xdna_attention_set_trace.argtypes = [vp]
        L.xdna_gemm_i8.argtypes = [vp, vp, vp, i, vp, vp, i, vp, C.c_float, vp, vp, i, i, i, vp]
        L.xdna_gemm_i8.restype = i
        L.xdna_bert_create.argtypes = [vp, vp, vp, i, i]
        L.xdna_bert_create.restype = vp
        L.xdna_bert_free.argtypes = [vp]
        L.xdna_bert_embed.argtypes = [vp, vp, vp, i, vp]
        L.xdna_bert_embed.restype = i
        L.xdna_bert_encode_device.argtypes = [vp, vp, vp, vp, i, i, i, vp, vp]
        L.xdna_bert_encode_device.restype = i
        L.xdna_bfp16_quantize.argtypes = [vp, sz, vp]
        L.xdna_bfp16_quantize.restype = i
        L.xdna_whisper_enc_create.argtypes = [vp, vp, vp, i]
        L.xdna_whisper_enc_create.restype = vp
        L.xdna_whisper_enc_free.argtypes = [vp]
        L.xdna_whisper_encode.argtypes = [vp, vp, i, vp]
        L.xdna_whisper_encode.restype = i
        L.xdna_whisper_encode_device.argtypes = [vp, vp, i, vp, vp]
        L.xdna_whisper_encode_device.restype = i
        L.xdna_parakeet_create.argtypes = [vp, vp, vp, i]
        L.xdna_parakeet_create.restype = vp
        L.xdna_parakeet_free.argtypes = [vp]
        L.xdna_parakeet_frames_out.argtypes = [vp]
        L.xdna_parakeet_frames_out.restype = i
        L.xdna_parakeet_encode.argtypes = [vp, vp, i, vp]
        L.xdna_parakeet_encode.restype = i
        L.xdna_parakeet_encode_device.argtypes = [vp, vp, i, vp, vp]
        L.xdna_parakeet_encode_device.restype = i
        L.xdna_whisper_dec_create.argtypes = [vp, vp, vp, i]
        L.xdna_whisper_dec_create.restype = vp
        L.xdna_whisper_dec_free.argtypes = [vp]
        L.xdna_whisper_dec_clamped_blocks.argtypes = [vp]
        L.xdna_whisper_dec_clamped_blocks.restype = C.c_longlong
        L.xdna_whisper_dec_set_encoder.argtypes = [vp, vp, i, vp]
        L.xdna_whisper_dec_set_encoder.restype = i
        L.xdna_whisper_dec_run.argtypes = [vp, i, vp, i, i, vp, vp, vp]
        L.xdna_whisper_dec_run.restype = i
        L.xdna_whisper_dec_generate.argtypes = [vp, vp, i, vp, i, i, vp, vp]
        L.xdna_whisper_dec_generate.restype = i
        L.xdna_whisper_dec_set_encoder_slot.argtypes = [vp, i, vp, vp]
        L.xdna_whisper_dec_set_encoder_slot.restype = i
        L.xdna_whisper_dec_step_slots.argtypes = [vp, i, vp, vp, vp, vp]
        L.xdna_whisper_dec_step_slots.restype = i
        L.xdna_gemma_create.argtypes = [vp, vp, vp, i, i, i, i]
        L.xdna_gemma_create.restype = vp
        L.xdna_gemma_free.argtypes = [vp]
        L.xdna_gemma_ipc_handle.argtypes = [vp, vp]
        L.xdna_gemma_ipc_handle.restype = i
        L.xdna_gemma_connect.argtypes = [vp, vp]
        L.xdna_gemma_connect.restype = i
        L.xdna_gemma_generate.argtypes = [vp, i, vp, i, i, vp, vp]
        L.xdna_gemma_generate.restype = i
        L.xdna_gemma_begin.argtypes = [vp, i, vp, i, i]
        L.xdna_gemma_begin.restype = i
        L.xdna_gemma_steps.argtypes = [vp, i, vp]
        L.xdna_gemma_steps.restype = i
        L.xdna_gemma_tokens.argtypes = [vp, vp, vp]
        L.xdna_gemma_tokens.restype = i
        L.xdna_opt_create.argtypes = [vp, vp, vp, i, i]
        L.xdna_opt_create.restype = vp
        L.xdna_opt_free.argtypes = [vp]
        L.xdna_opt_generate.argtypes = [vp, vp, sz, sz, vp, vp]
        L.xdna_opt_generate.restype = i
        L.xdna_opt_tokens_device.argtypes = [vp]
        L.xdna_opt_tokens_device.restype = vp
        L.xdna_opt_set_tokens.argtypes = [vp, vp, sz, sz, vp]
        L.xdna_opt_set_tokens.restype = i
        L.xdna_opt_get_tokens.argtypes = [vp, vp, sz, sz, vp]
        L.xdna_opt_get_tokens.restype = i
        L.xdna_opt_launch.argtypes = [vp, i, i, i, vp, vp]
        L.xdna_opt_launch.restype = i
        L.xdna_opt_sync.argtypes = [vp, vp]
        L.xdna_opt_prefill.argtypes = [vp, i, i, vp]
        L.xdna_opt_prefill.restype = i
        L.xdna_opt_sync.restype = i
        L.xdna_opt_stream_bytes_per_token.argtypes = [vp]
        L.xdna_opt_stream_bytes_per_token.restype = sz
        L.xdna_opt_grid.argtypes = [vp]
        L.xdna_opt_grid.restype = i
        L.xdna_opt_config.argtypes = [vp, vp]
        L.xdna_opt_config.restype = i
        L.xdna_opt_set_timing.argtypes = [vp, vp]
        L.xdna_opt_set_timing.restype = i
        L.xdna_opt_set_trace.argtypes = [vp, vp]
        L.xdna_opt_set_trace.restype = i
        L.xdna_device_ordinal.argtypes = [vp]
        L.xdna_device_ordinal.restype = i
        L.xdna_buffer_alloc.argtypes = [vp, sz]
        L.xdna_buffer_alloc.restype = vp
        L.xdna_buffer_free.argtypes = [vp]
        L.xdna_buffer_device_ptr.argtypes = [vp]
        L.xdna_buffer_device_ptr.restype = vp
        L.xdna_buffer_write.argtypes = [vp, vp, sz, sz]
        L.xdna_buffer_write.restype = i
        L.xdna_buffer_read.argtypes = [vp, vp, sz, sz]
        L.xdna_buffer_read.restype = i
        L.xdna_arena_create.argtypes = [vp, sz, sz, sz]
        L.xdna_arena_create.restype = vp
        L.xdna_arena_free.argtypes = [vp]
        L.xdna_arena_region.argtypes = [vp, i]
        L.xdna_arena_region.restype = vp
        L.xdna_arena_write.argtypes = [vp, i, sz, vp, sz]
        L.xdna_arena_write.restype = i
        L.xdna_arena_read.argtypes = [vp, i, sz, vp, sz]
        L.xdna_arena_read.restype = i
        L.xdna_run_start.argtypes = [vp, vp]
        L.xdna_run_start.restype = vp
        L.xdna_run_wait.argtypes = [vp, i]
        L.xdna_run_wait.restype = i
        L.xdna_run_free.argtypes = [vp]
        L.xdna_gemv_bf16_register.argtypes = [vp, vp, i, i, vp, i, vp, vp, C.c_float]
        L.xdna_gemv_bf16_register.restype = vp
        L.xdna_gemv_bf16_free.argtypes = [vp]
        L.xdna_gemv_bf16.argtypes = [vp, vp, vp]
        L.xdna_gemv_bf16.restype = i
        L.xdna_gemv_bf16_device.argtypes = [vp, vp, vp, vp]
        L.xdna_gemv_bf16_device.restype = i
        L.xdna_mha_decode_paged.argtypes = [vp, vp, i, i, vp, vp]
        L.xdna_mha_decode_paged.restype = i
        L.xdna_relpos_mha.argtypes = [vp, vp, vp, vp, i, i, vp, vp]
        L.xdna_relpos_mha.restype = i
        L.xdna_dwconv1d_glu_silu.argtypes = [vp, i, i, i, vp, i, vp, vp, vp]
        L.xdna_dwconv1d_glu_silu.restype = i
        L.xdna_subsample_conv2d.argtypes = [vp, i, i, i, i, vp, vp, i, i, i, i, i, i, i, vp, vp]
        L.xdna_subsample_conv2d.restype = i
        L.xdna_log_mel_create.argtypes = [vp]
        L.xdna_log_mel_create.restype = vp
        L.xdna_log_mel_free.argtypes = [vp]
        L.xdna_log_mel_device.argtypes = [vp, vp, i, vp, vp]
        L.xdna_log_mel_device.restype = i
        L.xdna_log_mel.argtypes = [vp, vp, sz, vp]
        L.xdna_log_mel.restype = i
        L.xdna_bpe_decode.argtypes = [C.c_char_p, vp, sz, i, vp, sz]
        L.xdna_bpe_decode.restype = i
        L.xdna_weights_open.argtypes = [C.c_char_p, C.c_char_p]
        L.xdna_weights_open.restype = vp
        L.xdna_weights_close.argtypes = [vp]
        L.xdna_weights_count.argtypes = [vp]
        L.xdna_weights_count.restype = i
        L.xdna_weights_name.argtypes = [vp, i]
        L.xdna_weights_name.restype = C.c_char_p
        L.xdna_weights_meta.argtypes = [vp, C.c_char_p]
        L.xdna_weights_meta.restype = C.c_char_p
        L.xdna_weights_info.argtypes = [vp, C.c_char_p, vp, vp, i]
        L.xdna_weights_info.restype = i
        L.xdna_weights_read_f32.argtypes = [vp, C.c_char_p, vp, sz]
        L.xdna_weights_read_f32.restype = i
        L.xdna_weights_read_bf16.argtypes = [vp, C.c_char_p, vp, sz]
        L.xdna_weights_read_bf16.restype = i
        L.xdna_opt_load.argtypes = [vp, C.c_char_p, i, i]
        L.xdna_opt_load.restype = vp
        _LIB = L
    return _LIB


def last_error() -> str:
    return lib().xdna_last_error().decode()


def _check(rc):
    if rc != 0:
        raise XdnaError(last_error())


def _addr(a: np.ndarray) -> int:
    return a.ctypes.data


def quant_i8_rows(w: np.ndarray):
    """qrow (the fused decode ELF's per-row int8 rule, round half to even) of an [M, K] weight:
    returns (q [M, K], scale [M]), ready for Device.gemv_i8."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, K = w.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float32)
    _check(lib().xdna_quant_i8_rows(_addr(w), M, K, _addr(q), _addr(s)))
    return q, s


def quant_i8_cols(w: np.ndarray):
    """Lin::load int8 quantisation as the engine performs it: returns (q [N, K], scale [N])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    K, N = w.shape
    q = np.empty((N, K), np.int8)
    s = np.empty(N, np.float32)
    _check(lib().xdna_quant_i8_cols(_addr(w), K, N, _addr(q), _addr(s)))
    return q, s


class Device:
    """An open sm_100 device (the npu-xrt Device replacement)."""

    def __init__(self, ordinal: int = 0):
        h = lib().xdna_device_open(ordinal)
        if not h:
            raise XdnaError(last_error())
        self.handle = h
        self.ordinal = ordinal

    @staticmethod
    def count() -> int:
        return lib().xdna_device_count()

    def gemv_i8(self, x, q_nk, scale, bias=None):
        x = np.ascontiguousarray(x, np.float32)
        q_nk = np.ascontiguousarray(q_nk, np.int8)
        N, K = q_nk.shape
        scale = np.ascontiguousarray(scale, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        y = np.empty(N, np.float32)
        _check(lib().xdna_gemv_i8(self.handle, _addr(x), K, _addr(q_nk), _addr(scale),
                                  None if b is None else _addr(b), N, _addr(y)))
        return y

    def close(self):
        if self.handle:
            lib().xdna_device_close(self.handle)
            self.handle = None


class GemvBf16:
    """A resident bf16 weight with an optional fused pre-norm: CtxDecode::register_weight / gemv
    (norm None) and register_fused / fused_norm_gemv (norm "rms" or "ln"),
    rust/npu-asr/src/ctx_decode.rs:269-369, 566-643.  w is [K, N] (in, out)."""

    _NORMS = {None: 0, "rms": 1, "ln": 2}

    def __init__(self, dev: Device, w, bias=None, norm=None, gamma=None, beta=None, eps=1e-5):
        w = np.ascontiguousarray(w, np.float32)
        self.K, self.N = w.shape
        keep = [np.ascontiguousarray(a, np.float32) if a is not None else None for a in (bias, gamma, beta)]
        ptr = [None if a is None else _addr(a) for a in keep]
        h = lib().xdna_gemv_bf16_register(dev.handle, _addr(w), self.K, self.N, ptr[0], self._NORMS[norm],
                                          ptr[1], ptr[2], eps)
        if not h:
            raise XdnaError(last_error())
        self.handle = h

    def __call__(self, x):
        x = np.ascontiguousarray(x, np.float32)
        if x.shape != (self.K,):
            raise ValueError(f"x has shape {x.shape}, want ({self.K},)")
        y = np.empty(self.N, np.float32)
        _check(lib().xdna_gemv_bf16(self.handle, _addr(x), _addr(y)))
        return y

    def device(self, x_dev: int, y_dev: int, stream: int = 0):
        """y_dev[N] = bf16(x_dev[K]) . W'' + bias' (x already normalised), async on `stream`."""
        _check(lib().xdna_gemv_bf16_device(self.handle, x_dev, y_dev, stream or None))

    def free(self):
        if self.handle:
            lib().xdna_gemv_bf16_free(self.handle)
            self.handle = None


def mha_decode_paged(q_dev: int, kv_dev: int, n_heads: int, n_tiles: int, ctx_dev: int, stream: int = 0):
    """The mha_decode kernel's contract over packed K/V tiles (mha_decode.cc:90-168)."""
    _check(lib().xdna_mha_decode_paged(q_dev, kv_dev, n_heads, n_tiles, ctx_dev, stream or None))


class OptDecoder:
    """opt-125m greedy decoder on one B200 (Opt::load + Opt::generate of the reference)."""

    def __init__(self, device: Device, cfg: OptConfig, weights: dict, max_ctx: int | None = None,
                 grid: int = 0):
        self.cfg = cfg
        self.device = device
        keep = []

        def p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return _addr(a)

        c = _OptConfig(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                       cfg.max_pos, cfg.eps)
        layers = (_OptLayer * cfg.n_layers)()
        for li, ly in enumerate(weights["layers"]):
            for n in _LAYER_FIELDS:
                setattr(layers[li], n, p(ly[n]))
        w = _OptWeights(p(weights["emb_tok"]), p(weights["emb_pos"]), p(weights["lnf_w"]),
                        p(weights["lnf_b"]), C.addressof(layers))
        self.max_ctx = max_ctx or cfg.max_pos
        h = lib().xdna_opt_create(device.handle, C.byref(c), C.byref(w), self.max_ctx, grid)
        if not h:
            raise XdnaError(last_error())
        self._adopt(h)

    def _adopt(self, h):
        self.handle = h
        self.grid = lib().xdna_opt_grid(h)
        self.stream_bytes_per_token = lib().xdna_opt_stream_bytes_per_token(h)

    @classmethod
    def load(cls, device: Device, path: str, max_ctx: int | None = None, grid: int = 0):
        """Opt::load from a baked arena (a .safetensors file of arch "opt") or the npy directory
        it was baked from; the configuration comes from the tensor shapes."""
        h = lib().xdna_opt_load(device.handle, os.fsencode(path), max_ctx or 0, grid)
        if not h:
            raise XdnaError(last_error())
        c = _OptConfig()
        _check(lib().xdna_opt_config(h, C.byref(c)))
        self = cls.__new__(cls)
        self.cfg = OptConfig(c.n_layers, c.d_model, c.n_heads, c.head_dim, c.ffn, c.vocab, c.max_pos,
                             float(str(np.float32(c.eps))))   # the shortest decimal of the f32
        self.device = device
        self.max_ctx = max_ctx or min(c.max_pos, 2048)
        self._adopt(h)
        return self

    def generate(self, prompt, n_new: int, want_logits: bool = False):
        """Greedy decode (host in, host out)."""
        prompt = np.ascontiguousarray(prompt, np.int64)
        out = np.empty(n_new, np.int64)
        lg = np.empty((n_new, self.cfg.vocab), np.float32) if want_logits else None
        _check(lib().xdna_opt_generate(self.handle, _addr(prompt), prompt.size, n_new, _addr(out),
                                       None if lg is None else _addr(lg)))
        return (out, lg) if want_logits else out

    # ---- device-resident control (streams as integer cudaStream_t handles)
    def tokens_device_ptr(self) -> int:
        return lib().xdna_opt_tokens_device(self.handle)

    def set_tokens(self, ids, off: int = 0, stream: int = 0):
        """Host ids -> device tokens[off:]; `ids` must stay alive until the stream passes."""
        _check(lib().xdna_opt_set_tokens(self.handle, _addr(ids), off, ids.size, stream or None))

    def get_tokens(self, out, off: int = 0, stream: int = 0):
        _check(lib().xdna_opt_get_tokens(self.handle, _addr(out), off, out.size, stream or None))

    def launch(self, start_pos: int, n_steps: int, n_prompt: int, logits_ptr: int = 0,
               stream: int = 0):
        _check(lib().xdna_opt_launch(self.handle, start_pos, n_steps, n_prompt,
                                     logits_ptr or None, stream or None))

    def prefill(self, start_pos: int, n: int, stream: int = 0):
        """K / V rows of prompt positions [start_pos, start_pos + n) as a batch (no LM head)."""
        _check(lib().xdna_opt_prefill(self.handle, start_pos, n, stream or None))

    def set_timing(self, timing_ptr: int):
        _check(lib().xdna_opt_set_timing(self.handle, timing_ptr or None))

    def set_trace(self, trace_ptr: int):
        _check(lib().xdna_opt_set_trace(self.handle, trace_ptr or None))

    def sync(self, stream: int = 0):
        _check(lib().xdna_opt_sync(self.handle, stream or None))

    def close(self):
        if getattr(self, "handle", None):
            lib().xdna_opt_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class _BertCfg(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("d_model", C.c_int), ("n_heads", C.c_int), ("ffn", C.c_int),
                ("vocab", C.c_int), ("max_pos", C.c_int), ("eps", C.c_float), ("pooling", C.c_int)]


_BERT_LAYER = ("q_w", "q_b", "k_w", "k_b", "v_w", "v_b", "o_w", "o_b", "attn_ln_w", "attn_ln_b",
               "ffn1_w", "ffn1_b", "ffn2_w", "ffn2_b", "out_ln_w", "out_ln_b")


class _BertLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _BERT_LAYER]


class _BertWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("word_emb", "pos_emb", "type_emb", "emb_ln_w", "emb_ln_b", "layers")]


class BertEmbedder:
    """BGE/BERT embedder on one B200 (EmbedPipeline::embed without the tokenizer)."""

    def __init__(self, device: Device, cfg, weights: dict, max_tokens: int, max_seqs: int):
        keep = []

        def p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return _addr(a)

        c = _BertCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.vocab, cfg.max_pos, cfg.eps,
                     cfg.pooling)
        layers = (_BertLayer * cfg.n_layers)()
        for li, ly in enumerate(weights["layers"]):
            for n in _BERT_LAYER:
                setattr(layers[li], n, p(ly[n]))
        w = _BertWeights(p(weights["word_emb"]), p(weights["pos_emb"]), p(weights["type_emb"]),
                         p(weights["emb_ln_w"]), p(weights["emb_ln_b"]), C.addressof(layers))
        h = lib().xdna_bert_create(device.handle, C.byref(c), C.byref(w), max_tokens, max_seqs)
        if not h:
            raise XdnaError(last_error())
        self.handle, self.cfg = h, cfg

    def embed(self, ids, seq_lens):
        ids = np.ascontiguousarray(ids, np.int32)
        lens = np.ascontiguousarray(seq_lens, np.int32)
        out = np.empty((lens.size, self.cfg.d_model), np.float32)
        _check(lib().xdna_bert_embed(self.handle, _addr(ids), _addr(lens), lens.size, _addr(out)))
        return out

    def encode_device(self, ids_ptr, tokpos_ptr, cu_ptr, n_tokens, n_seqs, max_len, out_ptr, stream=0):
        _check(lib().xdna_bert_encode_device(self.handle, ids_ptr, tokpos_ptr, cu_ptr, n_tokens, n_seqs,
                                             max_len, out_ptr, stream or None))

    def close(self):
        if getattr(self, "handle", None):
            lib().xdna_bert_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def bfp16_quantize(x):
    """The engine's bfp16 quantiser over contiguous blocks of 8 (same rule as the reference golden)."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    _check(lib().xdna_bfp16_quantize(_addr(x), x.size, _addr(y)))
    return y


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


class WhisperEncoder:
    """Whisper-small encoder on one B200 (WhisperEncoder::forward_last of the reference)."""

    def __init__(self, device: Device, cfg, weights: dict, max_batch: int = 1):
        keep = []

        def p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return _addr(a)

        c = _WEncCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.n_mels, cfg.n_frames, cfg.max_src,
                     cfg.eps)
        layers = (_WEncLayer * cfg.n_layers)()
        for li, ly in enumerate(weights["layers"]):
            for n in _WENC_LAYER:
                setattr(layers[li], n, p(ly[n]))
        w = _WEncWeights(*[p(weights[n]) for n in ("conv1_w", "conv1_b", "conv2_w", "conv2_b",
                                                    "embed_positions", "ln_post_w", "ln_post_b")],
                         C.addressof(layers))
        h = lib().xdna_whisper_enc_create(device.handle, C.byref(c), C.byref(w), max_batch)
        if not h:
            raise XdnaError(last_error())
        self.handle, self.cfg = h, cfg

    def encode(self, mel):
        mel = np.ascontiguousarray(mel, np.float32)
        B = mel.shape[0]
        out = np.empty((B, self.cfg.n_frames // 2, self.cfg.d_model), np.float32)
        _check(lib().xdna_whisper_encode(self.handle, _addr(mel), B, _addr(out)))
        return out

    def encode_device(self, mel_ptr, B, out_ptr, stream=0):
        _check(lib().xdna_whisper_encode_device(self.handle, mel_ptr, B, out_ptr, stream or None))

    def close(self):
        if getattr(self, "handle", None):
            lib().xdna_whisper_enc_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_PK_LAYER = ("ff1_ln_w", "ff1_ln_b", "ff1_w1", "ff1_w2", "att_ln_w", "att_ln_b", "wq", "wk", "wv", "wpos",
             "wout", "pos_u", "pos_v", "conv_ln_w", "conv_ln_b", "pw1", "dw_w", "dw_b", "pw2",
             "ff2_ln_w", "ff2_ln_b", "ff2_w1", "ff2_w2", "out_ln_w", "out_ln_b")
_PK_TOP = ("c0_w", "c0_b", "c2_w", "c2_b", "c3_w", "c3_b", "c5_w", "c5_b", "c6_w", "c6_b", "out_w", "out_b")


class _PkCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "n_heads", "ffn", "n_mels", "n_frames", "sub_ch",
                                       "kconv")]


class _PkLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _PK_LAYER]


class _PkWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _PK_TOP + ("layers",)]


class ParakeetEncoder:
    """Parakeet FastConformer encoder on one B200 (FastConformerEncoder::subsample +
    forward_last of the reference, int8 GEMM engine)."""

    def __init__(self, device: Device, cfg, weights: dict, max_batch: int = 1):
        keep = []

        def p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return _addr(a)

        c = _PkCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.n_mels, cfg.n_frames, cfg.sub_ch, cfg.kconv)
        layers = (_PkLayer * cfg.n_layers)()
        for li, ly in enumerate(weights["layers"][:cfg.n_layers]):
            for n in _PK_LAYER:
                setattr(layers[li], n, p(ly[n]))
        w = _PkWeights(*[p(weights[n]) for n in _PK_TOP], C.addressof(layers))
        h = lib().xdna_parakeet_create(device.handle, C.byref(c), C.byref(w), max_batch)
        if not h:
            raise XdnaError(last_error())
        self.handle, self.cfg = h, cfg
        self.frames_out = lib().xdna_parakeet_frames_out(h)

    def encode(self, mel):
        mel = np.ascontiguousarray(mel, np.float32)
        B = mel.shape[0]
        out = np.empty((B, self.frames_out, self.cfg.d_model), np.float32)
        _check(lib().xdna_parakeet_encode(self.handle, _addr(mel), B, _addr(out)))
        return out

    def encode_device(self, mel_ptr, B, out_ptr, stream=0):
        _check(lib().xdna_parakeet_encode_device(self.handle, mel_ptr, B, out_ptr, stream or None))

    def close(self):
        if getattr(self, "handle", None):
            lib().xdna_parakeet_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


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


class WhisperDecoder:
    """Whisper-small greedy decoder on one B200 (HostDecoder::precompute_cross + step loop of
    the reference, bfp16 weights), 1..32 streams in lockstep."""

    def __init__(self, device: Device, cfg, weights: dict, max_batch: int = 1):
        keep = []

        def p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return _addr(a)

        c = _WDecCfg(cfg.n_layers, cfg.d_model, cfg.n_heads, cfg.ffn, cfg.vocab, cfg.max_tgt, cfg.n_enc)
        layers = (_WDecLayer * cfg.n_layers)()
        for li, ly in enumerate(weights["layers"][:cfg.n_layers]):
            for n in _WDEC_LAYER:
                setattr(layers[li], n, p(ly[n]))
        w = _WDecWeights(*[p(weights[n]) for n in _WDEC_TOP], C.addressof(layers))
        h = lib().xdna_whisper_dec_create(device.handle, C.byref(c), C.byref(w), max_batch)
        if not h:
            raise XdnaError(last_error())
        self.handle, self.cfg = h, cfg

    @property
    def clamped_blocks(self) -> int:
        return lib().xdna_whisper_dec_clamped_blocks(self.handle)

    # ---- continuous batching
    def set_encoder_slot(self, slot: int, enc):
        """Load one stream's encoder states enc [n_enc, 768] (host) into `slot`."""
        import torch
        d = torch.from_numpy(np.ascontiguousarray(enc, np.float32)).cuda()
        _check(lib().xdna_whisper_dec_set_encoder_slot(self.handle, slot, d.data_ptr(), None))
        torch.cuda.synchronize()

    def step_slots(self, tokens, positions, want_logits=False):
        """One step for slots 0 .. len(tokens)-1 at their own positions (negative: empty slot)."""
        t = np.ascontiguousarray(tokens, np.int64)
        p = np.ascontiguousarray(positions, np.int32)
        nxt = np.empty(t.size, np.int64)
        lg = np.empty((t.size, self.cfg.vocab), np.float32) if want_logits else None
        _check(lib().xdna_whisper_dec_step_slots(self.handle, t.size, _addr(t), _addr(p), _addr(nxt),
                                                  None if lg is None else _addr(lg)))
        return (nxt, lg) if want_logits else nxt

    def generate(self, enc, prompt, n_new, want_logits=False):
        enc = np.ascontiguousarray(enc, np.float32)
        B = enc.shape[0]
        pr = np.ascontiguousarray(prompt, np.int64)
        toks = np.empty((B, n_new), np.int64)
        lg = np.empty((B, n_new, self.cfg.vocab), np.float32) if want_logits else None
        _check(lib().xdna_whisper_dec_generate(self.handle, _addr(enc), B, _addr(pr), len(pr), n_new, _addr(toks),
                                               _addr(lg) if lg is not None else None))
        return (toks, lg) if want_logits else toks

    def close(self):
        if getattr(self, "handle", None):
            lib().xdna_whisper_dec_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_GM_LAYER = ("in_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "post_attn_norm", "pre_ffn_norm", "wg", "wu",
             "wd", "post_ffn_norm")


class _GmCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layers", "d_model", "n_q_heads", "head_dim", "ffn", "vocab", "window",
                                       "pattern")] + \
               [(n, C.c_float) for n in ("theta_local", "theta_global", "query_pre_attn_scalar", "eps")]


class _GmLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _GM_LAYER]


class _GmWeights(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p), ("layers", C.c_void_p)]


class GemmaDecoder:
    """Gemma-3 greedy decoder on one B200, or one tensor-parallel rank (tp_size > 1: call
    ipc_handle() on every rank, exchange the handles, then connect(all_handles))."""

    def __init__(self, device: Device, cfg, weights: dict, max_batch=1, max_ctx=4352, tp_rank=0, tp_size=1):
        keep = []

        def p(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return _addr(a)

        c = _GmCfg(cfg.n_layers, cfg.d_model, cfg.n_q_heads, cfg.head_dim, cfg.ffn, cfg.vocab, cfg.window,
                   cfg.pattern, cfg.theta_local, cfg.theta_global, cfg.query_pre_attn_scalar, cfg.eps)
        layers = (_GmLayer * cfg.n_layers)()
        for li, ly in enumerate(weights["layers"][:cfg.n_layers]):
            for n in _GM_LAYER:
                setattr(layers[li], n, p(ly[n]))
        w = _GmWeights(p(weights["embed"]), p(weights["final_norm"]), C.addressof(layers))
        h = lib().xdna_gemma_create(device.handle, C.byref(c), C.byref(w), max_batch, max_ctx, tp_rank, tp_size)
        if not h:
            raise XdnaError(last_error())
        self.handle, self.cfg = h, cfg

    def ipc_handle(self) -> bytes:
        buf = (C.c_uint8 * 64)()
        _check(lib().xdna_gemma_ipc_handle(self.handle, buf))
        return bytes(buf)

    def connect(self, handles: list):
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _check(lib().xdna_gemma_connect(self.handle, buf))

    def generate(self, prompts, n_new, stream=0):
        pr = np.ascontiguousarray(np.atleast_2d(prompts), np.int64)
        B, n_prompt = pr.shape
        out = np.empty((B, n_new), np.int64)
        _check(lib().xdna_gemma_generate(self.handle, B, _addr(pr), n_prompt, n_new, _addr(out), stream or None))
        return out

    def close(self):
        if getattr(self, "handle", None):
            lib().xdna_gemma_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
